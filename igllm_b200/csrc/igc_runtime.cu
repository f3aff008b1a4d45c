// igc_runtime.cu - model load and upload, sessions, the verify-round pass and
// the C ABI of include/igllm_cuda.h.
//
// The pass follows app_core.c:11843 session_pass: embedding rows, the
// per-layer-embedding lift, 35 layers of (attention, feed-forward,
// per-layer-embedding feed), final norm, output head, logit cap.  Every step
// is a kernel of igc_kernels.cu; norms and residual adds ride inside the
// prologue of the projection that consumes them, so the residual stream is
// read and written by the projections themselves.  The position a pass starts
// at lives in device memory, which lets one captured CUDA graph per lane
// count serve every position.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <type_traits>
#include <unordered_map>
#include <vector>

#include "../../include/igllm_cuda.h"
#include "igc_json.h"
#include "igc_kernels.h"
#include "igc_lanes.h"
#include "igc_synth.h"

using namespace igc;

// ---------------------------------------------------------------------------
// errors and counters

static thread_local std::string g_last_error;
static thread_local long g_launches = 0;

static int fail_device(cudaError_t e, const char *where) {
  g_last_error = std::string(where) + ": " + cudaGetErrorString(e);
  return IGC_FAIL_DEVICE;
}

#define CK(call)                                       \
  do {                                                 \
    cudaError_t e_ = (call);                           \
    if (e_ != cudaSuccess) return fail_device(e_, #call); \
  } while (0)

#define CKL(call)                                      \
  do {                                                 \
    cudaError_t e_ = (call);                           \
    ++g_launches;                                      \
    if (e_ != cudaSuccess) return fail_device(e_, #call); \
  } while (0)

// An error a CUDA call left behind that its caller did not check would be
// reported by the next launch check, against the wrong call.  Entry points
// clear it first; IGC_DEBUG_ERRORS=1 names where a stale one was found.
static void clear_stale(const char *where) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    const char *dbg = getenv("IGC_DEBUG_ERRORS");
    if (dbg && dbg[0] == '1') fprintf(stderr, "igc: stale CUDA error before %s: %s\n", where, cudaGetErrorString(e));
  }
}

extern "C" const char *igc_last_error(void) { return g_last_error.c_str(); }
extern "C" long igc_launch_count(void) {
  long n = g_launches;
  g_launches = 0;
  return n;
}

// ---------------------------------------------------------------------------
// tensor sources: a safetensors folder (mmap) or a synthetic spec

enum { T_F32 = 1, T_F16 = 2, T_BF16 = 3, T_F64 = 4, T_I8 = 5, T_U8 = 6, T_I16 = 7, T_I32 = 8, T_I64 = 9 };

struct Tensor {
  int dtype = 0;
  int rank = 0;
  int64_t shape[4] = {0, 0, 0, 0};
  const uint8_t *data = nullptr;
  size_t bytes = 0;
};

static int dtype_of(const std::string &s) {
  if (s == "F32") return T_F32;
  if (s == "F16") return T_F16;
  if (s == "BF16") return T_BF16;
  if (s == "F64") return T_F64;
  if (s == "I8") return T_I8;
  if (s == "U8") return T_U8;
  if (s == "I16") return T_I16;
  if (s == "I32" || s == "U32") return T_I32;
  if (s == "I64" || s == "U64") return T_I64;
  return 0;
}

static size_t dtype_bytes(int t) {
  switch (t) {
    case T_F32: case T_I32: return 4;
    case T_F16: case T_BF16: case T_I16: return 2;
    case T_F64: case T_I64: return 8;
    default: return 1;
  }
}

static float f16_to_f32(uint16_t h) { return __half2float(*reinterpret_cast<const __half *>(&h)); }
static float bf16_to_f32(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static float real_at(const Tensor &t, size_t i) { /* app_core.c:1719 real_read */
  switch (t.dtype) {
    case T_F32: { float f; memcpy(&f, t.data + 4 * i, 4); return f; }
    case T_F16: { uint16_t h; memcpy(&h, t.data + 2 * i, 2); return f16_to_f32(h); }
    case T_BF16: { uint16_t h; memcpy(&h, t.data + 2 * i, 2); return bf16_to_f32(h); }
    case T_F64: { double d; memcpy(&d, t.data + 8 * i, 8); return (float)d; }
    case T_I8: return (float)(int8_t)t.data[i];
    case T_U8: return (float)t.data[i];
    default: return 0.0f;
  }
}

struct Source {
  virtual ~Source() {}
  virtual const Tensor *find(const std::string &name) = 0;
  virtual void release(const std::string &) {}
};

struct FileMap {
  void *base = nullptr;
  size_t size = 0;
  ~FileMap() {
    if (base) munmap(base, size);
  }
};

static bool slurp(const std::string &path, std::string &out) {
  FILE *f = fopen(path.c_str(), "rb");
  if (!f) return false;
  fseek(f, 0, SEEK_END);
  long n = ftell(f);
  fseek(f, 0, SEEK_SET);
  out.resize((size_t)(n > 0 ? n : 0));
  size_t got = n > 0 ? fread(&out[0], 1, (size_t)n, f) : 0;
  fclose(f);
  return got == (size_t)(n > 0 ? n : 0);
}

// app_core.c:1634 store_open: model.safetensors, or every shard the index
// names; tensors are views into the mapped files.
struct SafeSource : Source {
  std::vector<std::unique_ptr<FileMap>> maps;
  std::unordered_map<std::string, Tensor> tensors;

  int open_file(const std::string &path) {
    int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) return IGC_FAIL_FILE;
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < 8) { ::close(fd); return IGC_FAIL_FORMAT; }
    auto fm = std::make_unique<FileMap>();
    fm->size = (size_t)st.st_size;
    fm->base = mmap(nullptr, fm->size, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (fm->base == MAP_FAILED) { fm->base = nullptr; return IGC_FAIL_FILE; }
    const uint8_t *b = (const uint8_t *)fm->base;
    uint64_t hl;
    memcpy(&hl, b, 8);
    if (hl > fm->size - 8) return IGC_FAIL_FORMAT;
    Json head;
    JsonReader rd((const char *)b + 8, (size_t)hl);
    if (!rd.parse(head) || head.kind != Json::OBJ) return IGC_FAIL_FORMAT;
    const uint8_t *data = b + 8 + hl;
    size_t data_size = fm->size - 8 - hl;
    for (auto &kv : head.obj) {
      if (kv.first == "__metadata__") continue;
      const Json &j = kv.second;
      Tensor t;
      t.dtype = dtype_of(j.text("dtype", ""));
      const Json *sh = j.get("shape");
      const Json *off = j.get("data_offsets");
      if (!t.dtype || !sh || !off || off->kind != Json::ARR || off->arr.size() != 2) return IGC_FAIL_FORMAT;
      t.rank = (int)sh->arr.size();
      if (t.rank > 4) return IGC_FAIL_SUPPORT;
      for (int i = 0; i < t.rank; ++i) t.shape[i] = (int64_t)sh->arr[i].num;
      size_t a = (size_t)off->arr[0].num, e = (size_t)off->arr[1].num;
      if (e < a || e > data_size) return IGC_FAIL_FORMAT;
      t.data = data + a;
      t.bytes = e - a;
      tensors[kv.first] = t;
    }
    maps.push_back(std::move(fm));
    return IGC_OKAY;
  }

  int open(const std::string &folder) {
    std::string index;
    if (slurp(folder + "/model.safetensors.index.json", index)) {
      Json j;
      JsonReader rd(index.data(), index.size());
      if (!rd.parse(j)) return IGC_FAIL_FORMAT;
      const Json *wm = j.get("weight_map");
      if (!wm || wm->kind != Json::OBJ) return IGC_FAIL_FORMAT;
      std::map<std::string, int> files;
      for (auto &kv : wm->obj) files[kv.second.str] = 1;
      for (auto &f : files) {
        int c = open_file(folder + "/" + f.first);
        if (c != IGC_OKAY) return c;
      }
      return IGC_OKAY;
    }
    return open_file(folder + "/model.safetensors");
  }

  const Tensor *find(const std::string &name) override {
    auto it = tensors.find(name);
    return it == tensors.end() ? nullptr : &it->second;
  }
};

// A synthetic checkpoint: tensors generated on first use, dropped on release.
struct SynthSource : Source {
  igc_synth_spec spec;
  std::unordered_map<std::string, igc_synth_tensor> list;
  std::unordered_map<std::string, std::pair<std::vector<uint8_t>, Tensor>> made;
  int threads = 8;

  explicit SynthSource(const igc_synth_spec &s) : spec(s) {
    int n = igc_synth_list(&spec, nullptr, 0);
    std::vector<igc_synth_tensor> v((size_t)n);
    igc_synth_list(&spec, v.data(), n);
    for (auto &t : v) list[t.name] = t;
    long cpus = sysconf(_SC_NPROCESSORS_ONLN);
    threads = cpus > 0 ? (int)(cpus > 32 ? 32 : cpus) : 8;
  }
  const Tensor *find(const std::string &name) override {
    auto m = made.find(name);
    if (m != made.end()) return &m->second.second;
    auto it = list.find(name);
    if (it == list.end()) return nullptr;
    const igc_synth_tensor &st = it->second;
    auto &slot = made[name];
    slot.first.resize(st.bytes);
    igc_synth_tensor_fill(&spec, &st, slot.first.data(), threads);
    Tensor &t = slot.second;
    t.dtype = st.dtype;
    t.rank = st.rank;
    t.shape[0] = st.shape[0];
    t.shape[1] = st.shape[1];
    t.data = slot.first.data();
    t.bytes = st.bytes;
    return &t;
  }
  void release(const std::string &name) override { made.erase(name); }
};

// ---------------------------------------------------------------------------
// the model

struct RopeForm {
  double theta = 10000.0, share = 1.0;
  bool proportional = false;
};

struct DevPlane {
  // the lane GEMM's tensor maps of this plane's weights (igc_lane_tmaps)
  CUtensorMap tm_codes, tm_scales;
  bool tm_ok = false;
  uint4 *tiles = nullptr;
  uint2 *scales = nullptr;
  int n_rb = 0, n_cc = 0, rows = 0, cols = 0;
  int split = 1, grid = 1;
  bool pair = false;
  double bytes = 0.0;  // codes and scales a product streams (app_core.c:1860 plane_bytes)
  // a plane of a model the tiles do not hold (8-bit codes, dense planes,
  // activation grids): its parts as stored, one product each on the CUDA
  // cores (igc_launch_plain_product), writing the rows the tiles would
  std::vector<PlainArgs> plain;
  GemvPlane view() const { return GemvPlane{tiles, scales, n_rb, n_cc, rows, cols}; }
};

// Bind-time verdict that a model needs the plain planes (igc_model::plain).
constexpr int IGC_NEED_PLAIN = -100;

struct DevLayer {
  int kind = 0, share = 0, source = -1, hd = 0, kv_heads = 1, inner = 0;
  int q_rows = 0, kv_rows = 0, qkv_rows = 0;
  float gain = 1.0f;
  // the export's static ranges of an owner's key and value caches
  // (self_attn.k_cache_scale / v_cache_scale, 0 where it ships none), and the
  // rows the reference's ring of this layer holds (app_core.c:8723-8731
  // cache_span: 0 on a sharing layer; the window on a global layer or the
  // last owner of a kind that sharers read; else the sliding span)
  float k_scale = 0.0f, v_scale = 0.0f;
  int span = 0;
  DevPlane qkv, o, gateup, down, ple_gate, ple_proj;
  float *q_norm = nullptr, *k_norm = nullptr, *enter_norm = nullptr, *after_attn_norm = nullptr,
        *before_feed_norm = nullptr, *after_feed_norm = nullptr, *after_ple_norm = nullptr;
};

struct igc_model {
  int device = 0, sm_count = 148, smem_limit = 227 * 1024;
  int vocab = 0, hidden = 0, layers = 0, heads = 0, kv_heads = 1, inner = 0, ple_dim = 0, ple_vocab = 0;
  int slide_span = 512, window_limit = 0, share_count = 0, pad_id = 0;
  float eps = 1e-6f, softcap = 0.0f;
  int kind[128] = {0};
  RopeForm rope[2];
  int rope_hd[2] = {0, 0};
  float *rope_cs[2] = {nullptr, nullptr}, *rope_sn[2] = {nullptr, nullptr};
  uint16_t *embed = nullptr, *ple_embed = nullptr;
  // the embedding tables when the export stores them quantized
  // (`embedding_quantized` + `embedding_scale`): codes as stored, f16 scales
  // per 32-column group; `codes` null for a bf16 table
  EmbedCodes embed_q = {}, ple_q = {};
  DevPlane ple_lift, head;
  float *ple_norm = nullptr, *final_norm = nullptr;
  std::vector<DevLayer> layer;
  size_t decode_bytes = 0, device_bytes = 0;
  // bytes of every checkpoint tensor the text stack binds (app_core.c:12667
  // model_memory_bytes, the reference's model->weight_bytes)
  size_t weight_bytes = 0;
  // every projection as stored, on the CUDA cores, and every pass through the
  // lane stages (explicit norms, grids): set when a plane has 8-bit codes, is
  // dense, has scales f16 cannot hold, or carries activation grids
  bool plain = false;
  int plain_cols = 0;  // the widest input row a plain product reads
  // app_setup.cache_bits: 8 stores a cache side as e4m3 bytes wherever the
  // export ships that side's scale (app_core.c:14270-14284)
  int cache_bits = 0;
  int max_qkv = 0, max_inner = 0, max_q = 0, max_kvw = 0;
  std::vector<void *> owned;

  ~igc_model() {
    cudaSetDevice(device);
    for (void *p : owned) cudaFree(p);
    clear_stale("model free");
  }
  template <typename T>
  int alloc(T **p, size_t count) {
    void *v = nullptr;
    size_t bytes = count * sizeof(T);
    if (bytes == 0) bytes = 16;
    cudaError_t e = cudaMalloc(&v, bytes);
    if (e != cudaSuccess) return fail_device(e, "cudaMalloc(model)");
    owned.push_back(v);
    device_bytes += bytes;
    *p = (T *)v;
    return IGC_OKAY;
  }
};

static int layer_of_config(const Json &tc, int layers, int l) {
  const Json *lt = tc.get("layer_types");
  if (l == layers - 1) return 1; /* app_core.c:8395 */
  if (lt && lt->kind == Json::ARR && (size_t)l < lt->arr.size() && lt->arr[l].kind == Json::STR)
    return lt->arr[l].str == "sliding_attention" ? 0 : 1;
  return ((l + 1) % 6) ? 0 : 1;
}

// app_core.c:8325 config_read, the text stack's part.
static int read_config(igc_model *m, const std::string &text, const igc_setup *setup) {
  Json root;
  JsonReader rd(text.data(), text.size());
  if (!rd.parse(root)) return IGC_FAIL_FORMAT;
  const Json *tcp = root.get("text_config");
  const Json &tc = tcp ? *tcp : root;
  m->vocab = (int)tc.number("vocab_size", 262144);
  m->hidden = (int)tc.number("hidden_size", 2304);
  m->inner = (int)tc.number("intermediate_size", 9216);
  m->layers = (int)tc.number("num_hidden_layers", 30);
  m->heads = (int)tc.number("num_attention_heads", 8);
  m->kv_heads = (int)tc.number("num_key_value_heads", 4);
  m->slide_span = (int)tc.number("sliding_window", 512);
  m->ple_vocab = (int)tc.number("vocab_size_per_layer_input", 262144);
  m->ple_dim = (int)tc.number("hidden_size_per_layer_input", 256);
  m->share_count = (int)tc.number("num_kv_shared_layers", 0);
  m->eps = (float)tc.number("rms_norm_eps", 1e-6);
  m->softcap = (float)tc.number("final_logit_softcapping", 0.0);
  m->pad_id = (int)tc.number("pad_token_id", 0);
  int max_pos = (int)tc.number("max_position_embeddings", 131072);
  if (tc.flag("enable_moe_block", false) || tc.flag("attention_k_eq_v", false)) return IGC_FAIL_SUPPORT;
  if (tc.flag("use_double_wide_mlp", false) && m->share_count > 0) {
    // shared layers carry a doubled feed-forward; their planes say how wide
  }
  if (m->layers < 1 || m->layers > 128) return IGC_FAIL_SUPPORT;
  for (int l = 0; l < m->layers; ++l) m->kind[l] = layer_of_config(tc, m->layers, l);
  const Json *rp = tc.get("rope_parameters");
  const char *names[2] = {"sliding_attention", "full_attention"};
  for (int k = 0; k < 2; ++k) {
    RopeForm &r = m->rope[k];
    r.theta = k ? 1000000.0 : 10000.0;
    r.share = 1.0;
    r.proportional = (k == 1);
    if (k == 1) r.share = 0.25;
    const Json *kj = rp ? rp->get(names[k]) : nullptr;
    if (kj) {
      r.theta = kj->number("rope_theta", r.theta);
      r.share = kj->number("partial_rotary_factor", 1.0);
      r.proportional = kj->text("rope_type", "default") == "proportional";
    } else if (rp && rp->get("rope_theta")) {
      r.theta = rp->number("rope_theta", r.theta);
      r.share = rp->number("partial_rotary_factor", 1.0);
      r.proportional = rp->text("rope_type", "default") == "proportional";
    }
  }
  int window = max_pos < 32768 ? max_pos : 32768;
  if (setup && setup->window_limit > 0) window = setup->window_limit < max_pos ? setup->window_limit : max_pos;
  if (window < 8) window = 8;
  m->window_limit = window;
  return IGC_OKAY;
}

static std::string pick_prefix(Source &src) {
  const char *cands[] = {"model.language_model.", "language_model.model.", "model.", ""};
  for (const char *c : cands) {
    if (src.find(std::string(c) + "embed_tokens.weight") || src.find(std::string(c) + "embed_tokens.embedding_quantized"))
      return c;
  }
  return "#";
}

struct Binder {
  igc_model *m;
  Source &src;
  std::string prefix;
  cudaStream_t st;
  Binder(igc_model *mm, Source &s, const std::string &p, cudaStream_t stream) : m(mm), src(s), prefix(p), st(stream) {}

  // app_core.c:7941 vec_bind: any float type, materialised as f32 on the device.
  int vec(const std::string &stem, int hint, float **out, bool required = true) {
    const Tensor *t = src.find(stem + ".weight");
    std::string name = stem + ".weight";
    if (!t) { t = src.find(stem); name = stem; }
    if (!t) return required ? IGC_FAIL_MISSING : IGC_OKAY;
    size_t n = t->bytes / dtype_bytes(t->dtype);
    if (hint > 0 && n != (size_t)hint) return IGC_FAIL_FORMAT;
    std::vector<float> host(n);
    for (size_t i = 0; i < n; ++i) host[i] = real_at(*t, i);
    int c = m->alloc(out, n);
    if (c != IGC_OKAY) return c;
    CK(cudaMemcpy(*out, host.data(), n * sizeof(float), cudaMemcpyHostToDevice));
    m->decode_bytes += n * sizeof(float);
    m->weight_bytes += t->bytes;
    src.release(name);
    return IGC_OKAY;
  }

  // app_core.c:8104 scale_bind: a calibration scalar (one value of any float
  // type), 0 where the tensor is absent or holds more than one value.
  float scalar(const std::string &name) {
    const Tensor *t = src.find(name);
    if (!t) return 0.0f;
    size_t n = 1;
    for (int i = 0; i < t->rank; ++i) n *= (size_t)t->shape[i];
    if (n != 1 || dtype_bytes(t->dtype) == 0 || t->bytes < dtype_bytes(t->dtype)) return 0.0f;
    m->weight_bytes += t->bytes;
    const float v = real_at(*t, 0);
    src.release(name);
    return v;
  }

  // app_core.c:7886 plane_bind_gemma: offset codes of 1, 2 or 4 bits packed in
  // U8 bytes (the width fixed by `col_hint` and the row's byte count), group
  // scales of any float type with groups a multiple of 32 columns.  8-bit
  // codes (an I8 tensor, or U8 a byte a code) are refused: the tiles hold
  // 4-bit values.
  struct CodeView {
    const Tensor *code = nullptr, *scale = nullptr, *dense = nullptr;
    int rows = 0, cols = 0, groups = 0, bits = 4, group_size = 32;
    bool signed_codes = false;  // I8: app_core.c:7935 code_flip
    float enter = 0.0f, leave = 0.0f;  // the plane's activation grids (app_core.c:7941-7948)
    std::string name, code_name, scale_name;
  };
  int code_view(const std::string &stem, int col_hint, CodeView &v, const char *leaf = "weight",
                const char *scale_leaf = "weight_scale") {
    v.name = stem;
    v.code_name = stem + "." + leaf;
    v.scale_name = stem + "." + scale_leaf;
    v.code = src.find(v.code_name);
    if (!v.code) return IGC_FAIL_MISSING;
    v.scale = src.find(v.scale_name);
    // the grids are read, not counted (app_core.c:7941-7948)
    if (const Tensor *g = src.find(stem + ".input_activation_scale")) v.enter = real_at(*g, 0);
    if (const Tensor *g = src.find(stem + ".output_activation_scale")) v.leave = real_at(*g, 0);
    if (!(v.enter > 0.0f)) v.enter = 0.0f;
    if (!(v.leave > 0.0f)) v.leave = 0.0f;
    if (!v.scale && (v.code->dtype == T_F32 || v.code->dtype == T_F16 || v.code->dtype == T_BF16)) {
      // a dense plane (app_core.c:7980-7998)
      if (v.code->rank != 2 || (col_hint > 0 && v.code->shape[1] != col_hint)) return IGC_FAIL_FORMAT;
      if (!m->plain) return IGC_NEED_PLAIN;
      v.dense = v.code;
      v.code = nullptr;
      v.rows = (int)v.dense->shape[0];
      v.cols = (int)v.dense->shape[1];
      v.code_name = stem + "." + leaf;
      return IGC_OKAY;
    }
    if (!v.scale || (v.code->dtype != T_U8 && v.code->dtype != T_I8)) return IGC_FAIL_SUPPORT;
    if (v.code->rank != 2) return IGC_FAIL_FORMAT;
    int rows = (int)v.code->shape[0], bytes = (int)v.code->shape[1];
    int cols = col_hint;
    int bits = 0;
    if (v.code->dtype == T_I8) {
      bits = 8;
      v.signed_codes = true;
      if (cols > 0 && bytes != cols) return IGC_FAIL_FORMAT;
      cols = bytes;
    } else {
      const int widths[] = {8, 4, 2, 1};
      for (int w : widths)
        if (((int64_t)cols * w + 7) / 8 == bytes) { bits = w; break; }
      if (bits == 0) return IGC_FAIL_FORMAT;
    }
    int groups = v.scale->rank >= 2 ? (int)v.scale->shape[v.scale->rank - 1] : 1;
    if (groups < 1 || cols % groups) return IGC_FAIL_FORMAT;
    if (v.scale->dtype != T_F16 && v.scale->dtype != T_BF16 && v.scale->dtype != T_F32) return IGC_FAIL_SUPPORT;
    if ((int)v.scale->shape[0] != rows) return IGC_FAIL_FORMAT;
    v.rows = rows;
    v.cols = cols;
    v.groups = groups;
    v.bits = bits;
    v.group_size = cols / groups;
    if (!m->plain) {
      // what the 4-bit tiles cannot hold sends the model to the plain planes
      if (bits == 8 || v.group_size % 32 || v.enter > 0.0f || v.leave > 0.0f) return IGC_NEED_PLAIN;
      std::vector<uint16_t> sc;
      if (scales_f16(v, sc) != IGC_OKAY) return IGC_NEED_PLAIN;
    }
    return IGC_OKAY;
  }

  // A code view's scales as f16 per 32-column group; IGC_FAIL_SUPPORT when a
  // scale is not exact in f16.
  int scales_f16(const CodeView &p, std::vector<uint16_t> &out) {
    const int g32 = (p.cols + 31) / 32;
    out.assign((size_t)p.rows * g32, 0);
    return igc_scales_f16(p.scale->data, p.scale->dtype, p.rows, p.groups, p.group_size, p.cols, out.data()) == 0
               ? IGC_OKAY
               : IGC_FAIL_SUPPORT;
  }

  // A quantized embedding table (`stem.embedding_quantized` and
  // `stem.embedding_scale`) kept as stored for row lookups; `cols` the row's
  // values.  The view is left for a tied head to upload as a plane.
  int code_table(const std::string &stem, int cols, EmbedCodes &out, int *rows_out, CodeView &v) {
    int c = code_view(stem, cols, v, "embedding_quantized", "embedding_scale");
    if (c != IGC_OKAY) return c;
    // the row reads take 1, 2 or 4-bit codes with f16 scales per 32 columns
    if (v.bits == 8 || v.group_size % 32) return IGC_FAIL_SUPPORT;
    std::vector<uint16_t> sc;
    c = scales_f16(v, sc);
    if (c != IGC_OKAY) return c;
    uint8_t *codes = nullptr;
    uint16_t *scales = nullptr;
    c = m->alloc(&codes, v.code->bytes);
    if (c == IGC_OKAY) c = m->alloc(&scales, sc.size());
    if (c != IGC_OKAY) return c;
    CK(cudaMemcpy(codes, v.code->data, v.code->bytes, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(scales, sc.data(), sizeof(uint16_t) * sc.size(), cudaMemcpyHostToDevice));
    out.codes = codes;
    out.stride = (size_t)v.code->shape[1];
    out.bits = v.bits;
    out.scales = scales;
    out.g32 = (v.cols + 31) / 32;
    *rows_out = v.rows;
    // app_core.c:1880 plane_row_bytes: a row's codes and scales
    m->decode_bytes += out.stride + (size_t)v.groups * dtype_bytes(v.scale->dtype);
    m->weight_bytes += v.code->bytes + v.scale->bytes;
    return IGC_OKAY;
  }

  // Uploads one or more code planes of the same width into one tile array:
  // `parts` are stacked by row block (q|k|v) or, for a pair, interleaved
  // block by block (gate, up).
  // A plane's parts as stored for the plain products: codes, their scales as
  // f32, or the dense values; each part's rows at its place in the plane's
  // output (stacked, or a gate|up pair's interleaved 16-row blocks).
  int upload_plain(std::vector<CodeView> &parts, bool pair, DevPlane &out) {
    int rb_at = 0;
    for (size_t k = 0; k < parts.size(); ++k) {
      CodeView &p = parts[k];
      PlainArgs a;
      memset(&a, 0, sizeof(a));
      a.rows = p.rows;
      a.cols = p.cols;
      a.enter = p.enter;
      a.leave = p.leave;
      a.out_row0 = pair ? 0 : rb_at * 16;
      a.pair_half = pair ? (int)k : -1;
      size_t counted = 0;
      if (p.dense) {
        void *d = nullptr;
        int c = m->alloc(reinterpret_cast<uint8_t **>(&d), p.dense->bytes);
        if (c != IGC_OKAY) return c;
        CK(cudaMemcpy(d, p.dense->data, p.dense->bytes, cudaMemcpyHostToDevice));
        a.dense = d;
        a.dense_type = p.dense->dtype;  // the reference's store types: 1 F32, 2 F16, 3 BF16
        counted = p.dense->bytes;
        src.release(p.code_name);
      } else {
        std::vector<float> sc((size_t)p.rows * p.groups);
        for (size_t i = 0; i < sc.size(); ++i) sc[i] = real_at(*p.scale, i);
        uint8_t *codes = nullptr;
        float *scales = nullptr;
        int c = m->alloc(&codes, p.code->bytes);
        if (c == IGC_OKAY) c = m->alloc(&scales, sc.size());
        if (c != IGC_OKAY) return c;
        CK(cudaMemcpy(codes, p.code->data, p.code->bytes, cudaMemcpyHostToDevice));
        CK(cudaMemcpy(scales, sc.data(), sizeof(float) * sc.size(), cudaMemcpyHostToDevice));
        a.codes = codes;
        a.stride = (size_t)p.code->shape[1];
        a.bits = p.bits;
        a.bias = 1 << (p.bits - 1);
        a.flip = p.signed_codes ? (uint32_t)a.bias : 0u;
        a.scales = scales;
        a.groups = p.groups;
        a.group_size = p.group_size;
        counted = p.code->bytes + p.scale->bytes;
        src.release(p.code_name);
        src.release(p.scale_name);
      }
      m->decode_bytes += counted;  // app_core.c:1860 plane_bytes
      m->weight_bytes += counted;
      out.bytes += (double)counted;
      if (p.cols > m->plain_cols) m->plain_cols = p.cols;
      out.plain.push_back(a);
      rb_at += (p.rows + 15) / 16;
    }
    return IGC_OKAY;
  }

  int upload(std::vector<CodeView> parts, bool pair, DevPlane &out) {
    int cols = parts[0].cols;
    int n_cc = (cols + 63) / 64;
    int n_rb = 0;
    for (auto &p : parts) {
      if (p.cols != cols) return IGC_FAIL_FORMAT;
      if (!pair && parts.size() > 1 && p.rows % 16) return IGC_FAIL_SUPPORT;
      n_rb += (p.rows + 15) / 16;
    }
    if (pair && parts[0].rows != parts[1].rows) return IGC_FAIL_FORMAT;
    out.n_rb = n_rb;
    out.n_cc = n_cc;
    out.cols = cols;
    out.rows = pair ? parts[0].rows : n_rb * 16;
    if (!pair && parts.size() == 1) out.rows = parts[0].rows;
    out.pair = pair;
    if (m->plain) return upload_plain(parts, pair, out);
    int c = m->alloc(&out.tiles, (size_t)n_rb * n_cc * 32);
    if (c != IGC_OKAY) return c;
    c = m->alloc(&out.scales, (size_t)n_rb * n_cc * 8);
    if (c != IGC_OKAY) return c;
    int rb_at = 0;
    for (size_t k = 0; k < parts.size(); ++k) {
      CodeView &p = parts[k];
      uint8_t *dc = nullptr;
      uint16_t *ds = nullptr;
      size_t cb = p.code->bytes, sb = p.scale->bytes;
      std::vector<uint16_t> sc;
      int c = scales_f16(p, sc);
      if (c != IGC_OKAY) return c;
      CK(cudaMalloc(&dc, cb));
      CK(cudaMalloc(&ds, sizeof(uint16_t) * sc.size()));
      CK(cudaMemcpy(dc, p.code->data, cb, cudaMemcpyHostToDevice));
      CK(cudaMemcpy(ds, sc.data(), sizeof(uint16_t) * sc.size(), cudaMemcpyHostToDevice));
      int prb = (p.rows + 15) / 16;
      int mul = pair ? 2 : 1, add = pair ? (int)k : rb_at;
      cudaError_t e = igc_launch_repack(dc, (size_t)p.code->shape[1], p.bits, ds, (p.cols + 31) / 32, p.rows, p.cols,
                                        prb, n_cc, mul, add, out.tiles, out.scales, st);
      cudaError_t e2 = cudaStreamSynchronize(st);
      cudaFree(dc);
      cudaFree(ds);
      if (e != cudaSuccess) return fail_device(e, "repack");
      if (e2 != cudaSuccess) return fail_device(e2, "repack sync");
      rb_at += prb;
      // app_core.c:1860 plane_bytes: codes and scales a product streams
      m->decode_bytes += cb + sb;
      m->weight_bytes += cb + sb;
      out.bytes += (double)(cb + sb);
      src.release(p.code_name);
      src.release(p.scale_name);
    }
    plan(out);
    out.tm_ok = igc_lane_tmaps(out.tiles, out.scales, out.n_rb, out.n_cc, &out.tm_codes, &out.tm_scales) == 0;
    return IGC_OKAY;
  }

  // Warps per row block and blocks per launch.  Each block stages the whole
  // input once, so the grid stays near one or two blocks an SM (what the
  // staging leaves room for at eight lanes) and each block walks many row
  // blocks; a split shares one row block's chunks among warps where there
  // are too few row blocks to keep every warp busy.
  void plan(DevPlane &p) {
    int units = p.pair ? p.n_rb / 2 : p.n_rb;
    size_t stage = gemv_stage_bytes(p.n_cc, MODE_NT1) + 8 * 1024;
    int per_sm = (int)((size_t)m->smem_limit / stage);
    if (per_sm > 2) per_sm = 2;
    if (per_sm < 1) per_sm = 1;
    int cap = m->sm_count * per_sm;
    int S = 1;
    // the widest split that still gives every unit's group one warp slot,
    // so no group runs two units one after the other
    while (S < 8 && S * 2 <= p.n_cc && units * S * 2 <= cap * GEMV_WARPS) S *= 2;
    p.split = S;
    int per_iter = GEMV_WARPS / S;
    int need = (units + per_iter - 1) / per_iter;
    // a plane with many units a warp (the output head) streams through a
    // deep ring: one block an SM, with the shared memory to itself
    if (S == 1 && units > 2 * cap * GEMV_WARPS) cap = m->sm_count;
    p.grid = need < cap ? need : cap;
    if (p.grid < 1) p.grid = 1;
  }

  int plane(const std::string &stem, int col_hint, DevPlane &out) {
    CodeView v;
    int c = code_view(stem, col_hint, v);
    if (c != IGC_OKAY) return c;
    return upload({v}, false, out);
  }

  int table(const std::string &stem, int cols, uint16_t **out, int *rows_out) {
    const Tensor *t = src.find(stem + ".weight");
    if (!t) return IGC_FAIL_MISSING;
    if (t->dtype != T_BF16 || t->rank != 2) return IGC_FAIL_SUPPORT;
    if (cols > 0 && t->shape[1] != cols) return IGC_FAIL_FORMAT;
    int c = m->alloc(out, t->bytes / 2);
    if (c != IGC_OKAY) return c;
    CK(cudaMemcpy(*out, t->data, t->bytes, cudaMemcpyHostToDevice));
    *rows_out = (int)t->shape[0];
    m->decode_bytes += (size_t)t->shape[1] * 2; /* app_core.c:1880 plane_row_bytes */
    m->weight_bytes += t->bytes;
    src.release(stem + ".weight");
    return IGC_OKAY;
  }
};

// rope inverse frequencies (app_core.c:8121 rope_build) and the per-position
// cos/sin tables the attention reads (app_core.c:8147 rope_wave)
static int build_rope(igc_model *m, int kind, int hd, cudaStream_t st) {
  const RopeForm &r = m->rope[kind];
  int half = hd / 2, turn = half;
  if (r.proportional) turn = (int)(r.share * hd / 2.0);
  if (turn > half) turn = half;
  if (turn < 0) turn = 0;
  std::vector<float> steps((size_t)half, 0.0f);
  for (int i = 0; i < half; ++i)
    if (!r.proportional || i < turn) steps[i] = (float)(1.0 / pow(r.theta, (double)(2 * i) / (double)hd));
  float *d_steps = nullptr;
  CK(cudaMalloc(&d_steps, sizeof(float) * (size_t)half));
  CK(cudaMemcpy(d_steps, steps.data(), sizeof(float) * (size_t)half, cudaMemcpyHostToDevice));
  int c = m->alloc(&m->rope_cs[kind], (size_t)m->window_limit * half);
  if (c == IGC_OKAY) c = m->alloc(&m->rope_sn[kind], (size_t)m->window_limit * half);
  if (c != IGC_OKAY) { cudaFree(d_steps); return c; }
  cudaError_t e = igc_launch_rope_table(d_steps, half, m->window_limit, m->rope_cs[kind], m->rope_sn[kind], st);
  cudaError_t e2 = cudaStreamSynchronize(st);
  cudaFree(d_steps);
  if (e != cudaSuccess) return fail_device(e, "rope table");
  if (e2 != cudaSuccess) return fail_device(e2, "rope table sync");
  m->rope_hd[kind] = hd;
  return IGC_OKAY;
}

// app_core.c:8497 model_bind, for the text stack: shapes come from the
// tensors, the configuration is a hint.
static int bind_model(igc_model *m, Source &src) {
  std::string P = pick_prefix(src);
  if (P == "#") return IGC_FAIL_MISSING;
  cudaStream_t st;
  CK(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
  struct StreamGuard {
    cudaStream_t s;
    ~StreamGuard() { cudaStreamDestroy(s); }
  } guard{st};
  Binder b(m, src, P, st);
  int c, rows = 0;
  // the embedding: bf16 rows, or the export's quantized table (whose view a
  // tied head then uploads as its plane, app_core.c:8527-8538)
  Binder::CodeView embed_view;
  const bool embed_codes = src.find(P + "embed_tokens.embedding_quantized") != nullptr;
  if (embed_codes)
    c = b.code_table(P + "embed_tokens", m->hidden, m->embed_q, &rows, embed_view);
  else
    c = b.table(P + "embed_tokens", 0, &m->embed, &rows);
  if (c != IGC_OKAY) return c;
  m->vocab = rows;
  // the embedding table's width is the state size (app_core.c:8505)
  {
    int ple_rows = 0;
    if (m->ple_dim > 0) {
      if (src.find(P + "embed_tokens_per_layer.embedding_quantized")) {
        Binder::CodeView pv;
        c = b.code_table(P + "embed_tokens_per_layer", m->ple_dim * m->layers, m->ple_q, &ple_rows, pv);
        if (c == IGC_OKAY) {
          src.release(pv.code_name);
          src.release(pv.scale_name);
        }
      } else {
        c = b.table(P + "embed_tokens_per_layer", m->ple_dim * m->layers, &m->ple_embed, &ple_rows);
      }
      if (c != IGC_OKAY) return c;
      m->ple_vocab = ple_rows;
      c = b.plane(P + "per_layer_model_projection", m->hidden, m->ple_lift);
      if (c != IGC_OKAY) return c;
      c = b.vec(P + "per_layer_projection_norm", m->ple_dim, &m->ple_norm);
      if (c != IGC_OKAY) return c;
    }
  }
  c = b.vec(P + "norm", m->hidden, &m->final_norm);
  if (c != IGC_OKAY) return c;
  {
    const char *heads[] = {"lm_head", "model.lm_head", "language_model.lm_head"};
    c = IGC_FAIL_MISSING;
    for (const char *h : heads) {
      if (!src.find(std::string(h) + ".weight")) continue;
      c = b.plane(h, m->hidden, m->head);
      break;
    }
    if (c == IGC_FAIL_MISSING && embed_codes) {
      // no head of its own: the quantized embedding is the head (tied); its
      // bytes were counted once, with the table
      const size_t wb = m->weight_bytes, db = m->decode_bytes;
      c = b.upload({embed_view}, false, m->head);
      m->weight_bytes = wb;
      m->decode_bytes = db + (size_t)(m->head.bytes);
    } else if (embed_codes) {
      src.release(embed_view.code_name);
      src.release(embed_view.scale_name);
    }
    if (c != IGC_OKAY) return c; /* a tied head over a bf16 table is not supported */
  }
  m->layer.resize((size_t)m->layers);
  int first_share = m->layers - m->share_count;
  for (int l = 0; l < m->layers; ++l) {
    DevLayer &L = m->layer[l];
    char stem[512];
    L.kind = m->kind[l];
    L.share = m->share_count > 0 && l >= first_share;
    if (L.share) {
      for (int pi = first_share - 1; pi >= 0; --pi)
        if (m->kind[pi] == L.kind) { L.source = pi; break; }
      if (L.source < 0) return IGC_FAIL_FORMAT;
    }
#define STEM(fmt) (snprintf(stem, sizeof(stem), "%slayers.%d." fmt, P.c_str(), l), std::string(stem))
    Binder::CodeView q, k, v, o, gt, up, dn, pg, pp;
    c = b.code_view(STEM("self_attn.q_proj"), m->hidden, q);
    if (c != IGC_OKAY) return c;
    L.q_rows = q.rows;
    L.hd = q.rows / m->heads;
    if (L.hd * m->heads != q.rows || L.hd % 16 || L.hd > 512) return IGC_FAIL_SUPPORT;
    if (!L.share) {
      c = b.code_view(STEM("self_attn.k_proj"), m->hidden, k);
      if (c != IGC_OKAY) return c;
      c = b.code_view(STEM("self_attn.v_proj"), m->hidden, v);
      if (c != IGC_OKAY) return c; /* keys doubling as values is not supported */
      L.kv_rows = k.rows;
      L.kv_heads = k.rows / L.hd;
      if (v.rows != k.rows || L.kv_heads < 1) return IGC_FAIL_FORMAT;
      c = b.upload({q, k, v}, false, L.qkv);
      if (c != IGC_OKAY) return c;
      c = b.vec(STEM("self_attn.k_norm"), L.hd, &L.k_norm);
      if (c != IGC_OKAY) return c;
      L.k_scale = b.scalar(STEM("self_attn.k_cache_scale"));
      L.v_scale = b.scalar(STEM("self_attn.v_cache_scale"));
      if (!(L.k_scale > 0.0f)) L.k_scale = 0.0f;  // no grid to round onto (app_core.c:11199)
      if (!(L.v_scale > 0.0f)) L.v_scale = 0.0f;
    } else {
      const DevLayer &S = m->layer[L.source];
      L.kv_rows = S.kv_rows;
      L.kv_heads = S.kv_heads;
      if (S.hd != L.hd) return IGC_FAIL_FORMAT;
      c = b.upload({q}, false, L.qkv);
      if (c != IGC_OKAY) return c;
    }
    L.qkv_rows = L.share ? L.q_rows : L.q_rows + 2 * L.kv_rows;
    if (m->heads % L.kv_heads) return IGC_FAIL_FORMAT;
    c = b.code_view(STEM("self_attn.o_proj"), L.q_rows, o);
    if (c == IGC_OKAY) c = b.upload({o}, false, L.o);
    if (c != IGC_OKAY) return c;
    c = b.code_view(STEM("mlp.gate_proj"), m->hidden, gt);
    if (c == IGC_OKAY) c = b.code_view(STEM("mlp.up_proj"), m->hidden, up);
    if (c != IGC_OKAY) return c;
    L.inner = gt.rows;
    c = b.upload({gt, up}, true, L.gateup);
    if (c != IGC_OKAY) return c;
    c = b.code_view(STEM("mlp.down_proj"), L.inner, dn);
    if (c == IGC_OKAY) c = b.upload({dn}, false, L.down);
    if (c != IGC_OKAY) return c;
    c = b.vec(STEM("self_attn.q_norm"), L.hd, &L.q_norm);
    if (c == IGC_OKAY) c = b.vec(STEM("input_layernorm"), m->hidden, &L.enter_norm);
    if (c == IGC_OKAY) c = b.vec(STEM("post_attention_layernorm"), m->hidden, &L.after_attn_norm);
    if (c == IGC_OKAY) c = b.vec(STEM("pre_feedforward_layernorm"), m->hidden, &L.before_feed_norm);
    if (c == IGC_OKAY) c = b.vec(STEM("post_feedforward_layernorm"), m->hidden, &L.after_feed_norm);
    if (c != IGC_OKAY) return c;
    if (m->ple_dim > 0) {
      c = b.code_view(STEM("per_layer_input_gate"), m->hidden, pg);
      if (c == IGC_OKAY) c = b.upload({pg}, false, L.ple_gate);
      if (c == IGC_OKAY) c = b.code_view(STEM("per_layer_projection"), m->ple_dim, pp);
      if (c == IGC_OKAY) c = b.upload({pp}, false, L.ple_proj);
      if (c == IGC_OKAY) c = b.vec(STEM("post_per_layer_input_norm"), m->hidden, &L.after_ple_norm);
      if (c != IGC_OKAY) return c;
    }
    {
      const Tensor *g = src.find(STEM("layer_scalar"));
      L.gain = g ? real_at(*g, 0) : 1.0f; /* app_core.c:8700-8708, read and not counted in weight_bytes */
    }
#undef STEM
    if (!igc_attn_smem(L.hd) || igc_attn_smem(L.hd) > (size_t)m->smem_limit) return IGC_FAIL_SUPPORT;
    if (L.qkv_rows > m->max_qkv) m->max_qkv = L.qkv_rows;
    if (L.inner > m->max_inner) m->max_inner = L.inner;
    if (L.q_rows > m->max_q) m->max_q = L.q_rows;
    if (L.kv_rows > m->max_kvw) m->max_kvw = L.kv_rows;
  }
  // the reference's ring depth per layer (app_core.c:8553-8562 keep_flag,
  // :8723-8731 cache_span); this library keeps every owner full length, and
  // the spans describe its save files
  for (int l = 0; l < m->layers; ++l) {
    DevLayer &L = m->layer[l];
    if (L.share) { L.span = 0; continue; }
    int last = -1;
    for (int q = 0; q < first_share; ++q)
      if (m->kind[q] == L.kind) last = q;
    const bool keep_full = m->share_count > 0 && last == l;
    L.span = (L.kind == 1 || keep_full) ? m->window_limit
                                        : (m->slide_span < m->window_limit ? m->slide_span : m->window_limit);
    if (L.span < 1) L.span = 1;
  }
  for (int kind = 0; kind < 2; ++kind) {
    int hd = 0;
    for (auto &L : m->layer)
      if (L.kind == kind) hd = L.hd;
    if (hd) {
      c = build_rope(m, kind, hd, st);
      if (c != IGC_OKAY) return c;
    }
  }
  return IGC_OKAY;
}

static int model_prepare(igc_model *m, const igc_setup *setup) {
  clear_stale("model load");
  m->device = setup ? setup->device : 0;
  m->cache_bits = setup ? setup->cache_bits : 0;
  CK(cudaSetDevice(m->device));
  CK(cudaDeviceGetAttribute(&m->sm_count, cudaDevAttrMultiProcessorCount, m->device));
  CK(cudaDeviceGetAttribute(&m->smem_limit, cudaDevAttrMaxSharedMemoryPerBlockOptin, m->device));
  m->smem_limit -= 2048;  // the largest static part any kernel of igc_kernels.cu carries
  CK(igc_kernels_configure(m->smem_limit + 2048));
  CK(igc_lanes_configure());
  return IGC_OKAY;
}

extern "C" int igc_model_load(const char *folder, const igc_setup *setup, igc_model **model_out) {
  if (!folder || !model_out) return IGC_FAIL_ARGUMENT;
  *model_out = nullptr;
  std::string text;
  if (!slurp(std::string(folder) + "/config.json", text)) return IGC_FAIL_MISSING;
  SafeSource src;
  int c = src.open(folder);
  if (c != IGC_OKAY) return c;
  // the tiles first; a plane they cannot hold binds the whole model again
  // as plain planes
  for (int plain = 0; plain < 2; ++plain) {
    auto m = std::make_unique<igc_model>();
    m->plain = plain != 0;
    c = model_prepare(m.get(), setup);
    if (c != IGC_OKAY) return c;
    c = read_config(m.get(), text, setup);
    if (c != IGC_OKAY) return c;
    c = bind_model(m.get(), src);
    if (c == IGC_NEED_PLAIN && !plain) continue;
    if (c != IGC_OKAY) return c == IGC_NEED_PLAIN ? IGC_FAIL_SUPPORT : c;
    *model_out = m.release();
    return IGC_OKAY;
  }
  return IGC_FAIL_SUPPORT;
}

extern "C" int igc_model_synth(const igc_synth_spec *spec, const igc_setup *setup, igc_model **model_out) {
  if (!spec || !model_out) return IGC_FAIL_ARGUMENT;
  *model_out = nullptr;
  char *text = igc_synth_config_text(spec);
  if (!text) return IGC_FAIL_MEMORY;
  std::string t(text);
  free(text);
  SynthSource src(*spec);
  for (int plain = 0; plain < 2; ++plain) {
    auto m = std::make_unique<igc_model>();
    m->plain = plain != 0;
    int c = model_prepare(m.get(), setup);
    if (c != IGC_OKAY) return c;
    c = read_config(m.get(), t, setup);
    if (c != IGC_OKAY) return c;
    c = bind_model(m.get(), src);
    if (c == IGC_NEED_PLAIN && !plain) continue;
    if (c != IGC_OKAY) return c == IGC_NEED_PLAIN ? IGC_FAIL_SUPPORT : c;
    *model_out = m.release();
    return IGC_OKAY;
  }
  return IGC_FAIL_SUPPORT;
}

extern "C" void igc_model_free(igc_model *model) { delete model; }
extern "C" int igc_model_vocab_count(const igc_model *m) { return m ? m->vocab : 0; }
extern "C" int igc_model_layer_count(const igc_model *m) { return m ? m->layers : 0; }
extern "C" int igc_model_state_size(const igc_model *m) { return m ? m->hidden : 0; }
extern "C" int igc_model_window_limit(const igc_model *m) { return m ? m->window_limit : 0; }
extern "C" size_t igc_model_decode_bytes(const igc_model *m) { return m ? m->decode_bytes : 0; }
extern "C" size_t igc_model_device_bytes(const igc_model *m) { return m ? m->device_bytes : 0; }
// Weights of the int4 projections one lane multiplies (each product's rows x
// columns, both halves of a gate|up pair): half the FLOPs of a lane.
extern "C" size_t igc_model_weight_count(const igc_model *m) {
  if (!m) return 0;
  auto n = [](const DevPlane &p) -> size_t {
    return p.tiles || !p.plain.empty() ? (size_t)p.rows * p.cols * (p.pair ? 2 : 1) : 0;
  };
  size_t t = n(m->ple_lift) + n(m->head);
  for (auto &L : m->layer) t += n(L.qkv) + n(L.o) + n(L.gateup) + n(L.down) + n(L.ple_gate) + n(L.ple_proj);
  return t;
}

// ---------------------------------------------------------------------------
// sessions


// Device buffers of the batched-lane passes (igc_lanes.cu) for up to `cap`
// lanes: the residual stream, the per-layer inputs, q|k|v, attention, the
// K-slice partials, the staged operand blocks and their factors, and the
// output head's argmax partials.
struct LaneBuf {
  int cap = 0, split_lanes = 0;
  float *x0 = nullptr, *xa = nullptr, *xb = nullptr, *seed = nullptr, *ple_raw = nullptr, *ple = nullptr;
  float *qkv = nullptr, *attn = nullptr, *part = nullptr, *factor = nullptr;
  float *rows = nullptr;  // a plain model's staged input rows, [cap][model plain_cols]
  float *arg_val = nullptr;
  int *arg_idx = nullptr;
  void *a_tiles = nullptr;
};

// An attention cluster size from the environment (1, 2, 4, 8 or 16; for
// comparisons), else `fallback` (0: chosen per launch, attn_cluster_for).
static int cluster_env(const char *name, int fallback) {
  const char *v = getenv(name);
  const int c = v ? atoi(v) : 0;
  return c == 1 || c == 2 || c == 4 || c == 8 || c == 16 ? c : fallback;
}

// Whether lane passes ask for the light attention layout (two blocks an SM
// where a pass writes no new rows; IGC_NO_LIGHT=1 leaves it out, for
// comparison).
static int attn_light() {
  static const char *off = getenv("IGC_NO_LIGHT");
  return off && off[0] == '1' ? 0 : 1;
}

// Blocks a cluster for a lane pass's attention (a prime chunk or a crowd)
// of `units` clusters (16 query rows of one key/value head each): the fewest
// that still give about a wave of `slots` blocks (the SMs, twice over where
// the light layout lets two blocks share an SM).  Each block then walks more
// tiles and pays its fixed cost (its query rows, the cluster merge) fewer
// times.  Measured at E2B widths: a 4096-id prime took 187 ms at 16 blocks a
// cluster and 115 ms at 1 or 2; a 64-session crowd round took 11.1 ms at 8
// and 9.0 at 1, and with the light layout 7.9 at 1 and 7.7 at 2.
static int attn_cluster_for(long units, int slots) {
  int cx = 1;
  while (cx < 16 && units * cx * 4 < (long)slots * 3) cx *= 2;
  return cx;
}

struct igc_session {
  igc_model *m = nullptr;
  cudaStream_t st = nullptr;
  int fill = 0;
  int guess_count = 0, guess_from = 0, guess_echo = 0;
  std::vector<int32_t> echo;
  uint64_t draw_state = 0x2545F4914F6CDD1DULL;
  // every owner layer's caches, full length: float rows, or e4m3 bytes on a
  // side the model stores as bytes (layer_store); sharing layers hold none
  std::vector<float *> kc, vc;
  // the largest magnitude written to each owner's caches, [layer][key, value]
  // (app_core.c:11208 cache_lay's key_peak / value_peak), and the copy the
  // pass in flight started from (app_core.c:12153-12156)
  float *d_peak = nullptr, *d_peak_saved = nullptr;
  // where a layer with a byte side has its rows decoded to floats for the
  // attention kernel (window x widest row floats a side; one layer at a time)
  float *kf = nullptr, *vf = nullptr;
  // the first position whose rows every sliding layer holds: 0, except after
  // loading a file written from rings that had turned over
  int floor = 0;
  int *d_io = nullptr;  // [0] position, [1..16] ids
  int32_t *d_top = nullptr;  // [0..16) argmax ids, [16] the kernels' error word (d_err)
  int *d_err = nullptr;
  float *x0 = nullptr, *xa = nullptr, *xb = nullptr, *seed = nullptr, *ple_raw = nullptr, *ple = nullptr;
  float *qkv = nullptr, *attn = nullptr, *obuf = nullptr, *act = nullptr, *dbuf = nullptr, *pa = nullptr,
        *pp = nullptr, *logits = nullptr;
  float *arg_val = nullptr;
  float *ssq_o = nullptr, *ssq_d = nullptr, *ssq_pp = nullptr;
  float *amax_attn = nullptr, *amax_act = nullptr, *amax_pa = nullptr;  // magnitude partials
  int *arg_idx = nullptr;
  float *cand_v = nullptr, *top_v = nullptr;
  int *cand_i = nullptr, *top_i = nullptr;
  int32_t *d_echo = nullptr;
  int *d_echo_range = nullptr;
  int32_t *h_io = nullptr, *h_top = nullptr;  // pinned
  float *h_top_v = nullptr;
  int *h_top_i = nullptr;
  int logit_lanes = 0;  // rows the last pass left in `logits`
  int attn_cluster = 16;  // attention blocks a cluster, fixed for the session
  // blocks a cluster of a prime chunk's attention on sliding and on global
  // layers (0: attn_cluster_for)
  int chunk_cluster = 0, chunk_cluster_global = 0;
  int use_graphs = 1;
  int use_pdl = 1;
  int use_stamps = 1;  // IGC_NO_STAMPS=1 launches without launch stamps (for comparison)
  int use_chunks = 1;  // IGC_NO_CHUNKS=1 primes in 16-lane passes only
  std::map<int, long> kernels_per_chunk;
  int head_parts = 0;  // argmax partials the output head's launch left
  cudaGraphExec_t graph[IGC_LANE_LIMIT + 1][2] = {};
  double serve_seconds = 0.0;
  size_t serve_tokens = 0;
  long kernels_per_pass[IGC_LANE_LIMIT + 1][2] = {};
  std::vector<void *> owned;
  int arg_parts = 0;
  // per-launch timing for igc_session_profile: an event before every launch
  struct Mark {
    cudaEvent_t ev;
    int cls;
    double bytes;
  };
  bool prof_on = false;
  std::vector<Mark> marks;
  int32_t *d_rounds = nullptr;  // igc_session_bench's per-round [position, ids]
  size_t d_rounds_cap = 0;
  // launch stamps of the graphed pass (igc_session_stamps): [IGC_STAMP_LIMIT]
  // (begin, end) pairs the pass's kernels write, and per stamped launch the
  // total of its spans over every pass with a head since the last reset
  unsigned long long *d_stamp = nullptr, *d_stamp_sum = nullptr;
  struct StampMeta {
    int cls;
    double bytes;
  };
  // the batched-lane prime (igc_lanes.cu): buffers for chunks of up to
  // `cap` lanes, allocated on the first prime that uses them, and a captured
  // graph per chunk length
  struct Chunks {
    LaneBuf B;
    int32_t *d_ids = nullptr;  // [0] position, [1..cap] ids
    int *d_pos = nullptr;      // the 16-lane attention groups' positions
    // per layer, every group's caches (the layer's owner's, the same for all
    // groups): [layers][groups_cap], for the batched attention launch
    float **kc_tab = nullptr, **vc_tab = nullptr;
    int groups_cap = 0;
    int32_t *h_ids = nullptr;  // pinned
    std::map<int, cudaGraphExec_t> graph;
  } ch;
  int stamp_n = 0;                     // launches stamped in the pass being enqueued
  std::vector<StampMeta> stamp_build;  // their classes and weight bytes
  std::vector<StampMeta> stamp_meta[IGC_LANE_LIMIT + 1];  // of the pass with a head, per lane count

  ~igc_session() {
    cudaSetDevice(m->device);
    for (auto &kv : ch.graph) cudaGraphExecDestroy(kv.second);
    if (ch.h_ids) cudaFreeHost(ch.h_ids);
    for (auto &mk : marks) cudaEventDestroy(mk.ev);
    for (int k = 0; k <= IGC_LANE_LIMIT; ++k)
      for (int w = 0; w < 2; ++w)
        if (graph[k][w]) cudaGraphExecDestroy(graph[k][w]);
    for (void *p : owned) cudaFree(p);
    if (h_io) cudaFreeHost(h_io);
    if (st) cudaStreamDestroy(st);
    clear_stale("session close");
  }
  template <typename T>
  int alloc(T **p, size_t count) {
    void *v = nullptr;
    cudaError_t e = cudaMalloc(&v, (count ? count : 1) * sizeof(T));
    if (e != cudaSuccess) return fail_device(e, "cudaMalloc(session)");
    owned.push_back(v);
    *p = (T *)v;
    return IGC_OKAY;
  }
};

// How owner layer `owner`'s caches are stored: a side is e4m3 bytes where the
// setup asks for 8-bit caches and the export ships that side's scale
// (app_core.c:14270-14284), else float; `peak` (or per batched block
// peak_tab) takes the magnitudes of the rows written.
static CacheStore layer_store(const igc_model *m, int owner, float *peak, float *const *peak_tab = nullptr) {
  const DevLayer &O = m->layer[owner];
  const bool bytes = m->cache_bits == 8;
  CacheStore cq;
  cq.kq = bytes ? O.k_scale : 0.0f;
  cq.vq = bytes ? O.v_scale : 0.0f;
  cq.peak = peak;
  cq.peak_tab = peak_tab;
  return cq;
}

static size_t side_bytes(float q) { return q > 0.0f ? 1u : sizeof(float); }

static bool layer_bytes(const igc_model *m, int owner) {
  const CacheStore cq = layer_store(m, owner, nullptr);
  return cq.kq > 0.0f || cq.vq > 0.0f;
}

// Whether layer l's attention runs as separate launches (new rows written
// first, then attention reading every row from the cache): a byte side, or a
// head wider than 256 (the export's global layers), whose attention kernel
// has no room to hold the pass's new rows apart.
static bool layer_split(const igc_model *m, int l) {
  const DevLayer &L = m->layer[l];
  return layer_bytes(m, L.share ? L.source : l) || L.hd > 256;
}

// The float rows a layer's attention reads from: its owner's cache on a float
// side, the session's decoded rows on a byte side.
static float *attn_rows(const igc_session *s, int owner, int value_side) {
  const CacheStore cq = layer_store(s->m, owner, nullptr);
  if (value_side) return cq.vq > 0.0f ? s->vf : s->vc[owner];
  return cq.kq > 0.0f ? s->kf : s->kc[owner];
}

// The decode of owner `owner`'s byte rows that a pass of `lanes` lanes reads
// (a sliding layer's window behind its first lane, a global layer's prefix),
// and the most rows it can cover.
static WidenArgs widen_of(const igc_session *s, int owner, int sliding, int lanes) {
  const igc_model *m = s->m;
  const CacheStore cq = layer_store(m, owner, nullptr);
  WidenArgs w;
  memset(&w, 0, sizeof(w));
  w.kc = reinterpret_cast<const uint8_t *>(s->kc[owner]);
  w.vc = reinterpret_cast<const uint8_t *>(s->vc[owner]);
  w.kf = s->kf;
  w.vf = s->vf;
  w.kq = cq.kq;
  w.vq = cq.vq;
  w.kv_w = m->layer[owner].kv_rows;
  w.lanes = lanes;
  w.sliding = sliding;
  w.span = m->slide_span;
  return w;
}
static int widen_rows_most(const igc_model *m, int sliding, int lanes) {
  const int r = sliding ? m->slide_span + lanes - 1 : m->window_limit;
  return r < m->window_limit ? r : m->window_limit;
}

extern "C" int igc_session_open(igc_model *m, igc_session **out) {
  if (!m || !out) return IGC_FAIL_ARGUMENT;
  *out = nullptr;
  clear_stale("session open");
  CK(cudaSetDevice(m->device));
  auto s = std::make_unique<igc_session>();
  s->m = m;
  CK(cudaStreamCreateWithFlags(&s->st, cudaStreamNonBlocking));
  const int K = IGC_LANE_LIMIT, H = m->hidden, PS = m->layers * m->ple_dim;
  int c = IGC_OKAY;
  s->kc.assign((size_t)m->layers, nullptr);
  s->vc.assign((size_t)m->layers, nullptr);
  for (int l = 0; l < m->layers && c == IGC_OKAY; ++l) {
    const DevLayer &L = m->layer[l];
    if (L.share) continue;
    const CacheStore cq = layer_store(m, l, nullptr);
    const size_t kb = side_bytes(cq.kq) * (size_t)m->window_limit * L.kv_rows;
    const size_t vb = side_bytes(cq.vq) * (size_t)m->window_limit * L.kv_rows;
    uint8_t *kp = nullptr, *vp = nullptr;
    c = s->alloc(&kp, kb);
    if (c == IGC_OKAY) c = s->alloc(&vp, vb);
    if (c != IGC_OKAY) break;
    s->kc[l] = reinterpret_cast<float *>(kp);
    s->vc[l] = reinterpret_cast<float *>(vp);
    CK(cudaMemsetAsync(kp, 0, kb, s->st));  // a zero code decodes to zero: a cleared cache either way
    CK(cudaMemsetAsync(vp, 0, vb, s->st));
  }
  {
    int widest = 0;  // the widest row a byte side decodes into
    for (int l = 0; l < m->layers; ++l)
      if (!m->layer[l].share && layer_bytes(m, l)) widest = std::max(widest, m->layer[l].kv_rows);
    if (c == IGC_OKAY && widest > 0) c = s->alloc(&s->kf, (size_t)m->window_limit * widest);
    if (c == IGC_OKAY && widest > 0) c = s->alloc(&s->vf, (size_t)m->window_limit * widest);
  }
  if (c == IGC_OKAY) c = s->alloc(&s->d_peak, 2 * (size_t)m->layers);
  if (c == IGC_OKAY) c = s->alloc(&s->d_peak_saved, 2 * (size_t)m->layers);
  if (c == IGC_OKAY) CK(cudaMemsetAsync(s->d_peak, 0, sizeof(float) * 2 * (size_t)m->layers, s->st));
  if (c == IGC_OKAY) CK(cudaMemsetAsync(s->d_peak_saved, 0, sizeof(float) * 2 * (size_t)m->layers, s->st));
  s->arg_parts = m->sm_count * 4;
  if (c == IGC_OKAY) c = s->alloc(&s->d_io, 1 + K);
  if (c == IGC_OKAY) c = s->alloc(&s->d_top, K + 1);
  if (c == IGC_OKAY) {
    s->d_err = s->d_top + K;
    CK(cudaMemsetAsync(s->d_top, 0, sizeof(int32_t) * (K + 1), s->st));
  }
  if (c == IGC_OKAY) c = s->alloc(&s->x0, (size_t)K * H);
  if (c == IGC_OKAY) c = s->alloc(&s->xa, (size_t)K * H);
  if (c == IGC_OKAY) c = s->alloc(&s->xb, (size_t)K * H);
  if (c == IGC_OKAY) c = s->alloc(&s->seed, (size_t)K * (PS ? PS : 1));
  if (c == IGC_OKAY) c = s->alloc(&s->ple_raw, (size_t)K * (PS ? PS : 1));
  if (c == IGC_OKAY) c = s->alloc(&s->ple, (size_t)K * (PS ? PS : 1));
  if (c == IGC_OKAY) c = s->alloc(&s->qkv, (size_t)K * m->max_qkv);
  if (c == IGC_OKAY) c = s->alloc(&s->attn, (size_t)K * m->max_q);
  if (c == IGC_OKAY) c = s->alloc(&s->obuf, (size_t)K * H);
  if (c == IGC_OKAY) c = s->alloc(&s->act, (size_t)K * m->max_inner);
  if (c == IGC_OKAY) c = s->alloc(&s->dbuf, (size_t)K * H);
  if (c == IGC_OKAY) c = s->alloc(&s->pa, (size_t)K * (m->ple_dim ? m->ple_dim : 1));
  if (c == IGC_OKAY) c = s->alloc(&s->pp, (size_t)K * H);
  if (c == IGC_OKAY) c = s->alloc(&s->logits, (size_t)K * m->vocab);
  if (c == IGC_OKAY) c = s->alloc(&s->arg_val, (size_t)s->arg_parts * 16);
  if (c == IGC_OKAY) c = s->alloc(&s->arg_idx, (size_t)s->arg_parts * 16);
  if (c == IGC_OKAY) c = s->alloc(&s->ssq_o, (size_t)s->arg_parts * 16);
  if (c == IGC_OKAY) c = s->alloc(&s->ssq_d, (size_t)s->arg_parts * 16);
  if (c == IGC_OKAY) c = s->alloc(&s->ssq_pp, (size_t)s->arg_parts * 16);
  if (c == IGC_OKAY) c = s->alloc(&s->amax_attn, (size_t)s->arg_parts * 16);
  if (c == IGC_OKAY) c = s->alloc(&s->amax_act, (size_t)s->arg_parts * 16);
  if (c == IGC_OKAY) c = s->alloc(&s->amax_pa, (size_t)s->arg_parts * 16);
  int blocks = (m->vocab + 2047) / 2048;
  if (c == IGC_OKAY) c = s->alloc(&s->cand_v, (size_t)K * blocks * 256);
  if (c == IGC_OKAY) c = s->alloc(&s->cand_i, (size_t)K * blocks * 256);
  if (c == IGC_OKAY) c = s->alloc(&s->top_v, (size_t)K * 256);
  if (c == IGC_OKAY) c = s->alloc(&s->top_i, (size_t)K * 256);
  if (c == IGC_OKAY) c = s->alloc(&s->d_echo, (size_t)m->window_limit);
  if (c == IGC_OKAY) c = s->alloc(&s->d_echo_range, 2 * K);
  if (c == IGC_OKAY) c = s->alloc(&s->d_stamp, 2 * IGC_STAMP_LIMIT);
  if (c == IGC_OKAY) c = s->alloc(&s->d_stamp_sum, IGC_STAMP_LIMIT);
  if (c == IGC_OKAY) CK(cudaMemsetAsync(s->d_stamp_sum, 0, sizeof(unsigned long long) * IGC_STAMP_LIMIT, s->st));
  if (c != IGC_OKAY) return c;
  {
    void *h = nullptr;
    size_t bytes = sizeof(int32_t) * (size_t)(1 + K) + sizeof(int32_t) * (K + 1) + (sizeof(float) + sizeof(int)) * K * 256;
    CK(cudaMallocHost(&h, bytes));
    s->h_io = (int32_t *)h;
    s->h_top = s->h_io + 1 + K;
    s->h_top_v = (float *)(s->h_top + K + 1);
    s->h_top_i = (int *)(s->h_top_v + K * 256);
  }
  CK(cudaStreamSynchronize(s->st));
  s->echo.reserve((size_t)m->window_limit);
  const char *g = getenv("IGC_NO_GRAPHS");
  s->use_graphs = !(g && g[0] == '1');
  const char *np = getenv("IGC_NO_PDL");
  s->use_pdl = !(np && np[0] == '1');
  const char *ns = getenv("IGC_NO_STAMPS");
  s->use_stamps = !(ns && ns[0] == '1');
  const char *nc = getenv("IGC_NO_CHUNKS");
  s->use_chunks = !(nc && nc[0] == '1');
  // attention clusters of 16 blocks (half the tiles a block of 8 takes)
  // unless IGC_ATTN_CLUSTER=8 or the heads' magnitude partials would not fit
  const char *ac = getenv("IGC_ATTN_CLUSTER");
  s->attn_cluster = (ac && atoi(ac) == 8) || m->heads * 16 > GEMV_PART_LIMIT ? 8 : 16;
  s->chunk_cluster = cluster_env("IGC_CHUNK_CLUSTER", 0);
  s->chunk_cluster_global = cluster_env("IGC_CHUNK_CLUSTER_GLOBAL", s->chunk_cluster);
  *out = s.release();
  return IGC_OKAY;
}

extern "C" void igc_session_close(igc_session *s) { delete s; }

extern "C" void igc_session_reset(igc_session *s) { /* app_core.c:14375 */
  if (!s) return;
  s->guess_count = 0;
  s->fill = 0;
  s->floor = 0;
  s->echo.clear();
  s->serve_seconds = 0.0;
  s->serve_tokens = 0;
  cudaSetDevice(s->m->device);
  cudaMemsetAsync(s->d_peak, 0, sizeof(float) * 2 * (size_t)s->m->layers, s->st);
  cudaStreamSynchronize(s->st);
}

extern "C" int igc_session_fill(const igc_session *s) { return s ? s->fill : 0; }
extern "C" int igc_session_guess_span(const igc_session *s) { return s ? s->guess_count : 0; }
extern "C" int igc_session_guess_limit(const igc_session *s) { return s ? IGC_LANE_LIMIT : 0; }
extern "C" double igc_session_serve_seconds(const igc_session *s) { return s ? s->serve_seconds : 0.0; }
extern "C" size_t igc_session_serve_tokens(const igc_session *s) { return s ? s->serve_tokens : 0; }

extern "C" int igc_session_hold(igc_session *s, int keep) { /* app_core.c:13935 */
  if (!s || keep < 0) return IGC_FAIL_ARGUMENT;
  if (s->guess_count > 0) return IGC_FAIL_STATE;
  if (keep > s->fill) return IGC_FAIL_ARGUMENT;
  // full-length caches wind back anywhere, except below rows a loaded file
  // did not carry: the next id at `keep` reads the sliding window behind it
  if (s->floor > 0 && keep > 0 && keep - s->m->slide_span + 1 < s->floor) return IGC_FAIL_SUPPORT;
  if (keep == 0) s->floor = 0;
  s->fill = keep;
  if ((int)s->echo.size() > keep) s->echo.resize((size_t)keep);
  return IGC_OKAY;
}

// The sums of squares a projection's output leaves for its consumer's norm:
// one row of 16 lanes per block of the launch that wrote them.
struct Ssq {
  float *buf = nullptr;
  int parts = 0;
};

// Launch classes igc_session_profile reports.
enum { PROF_GEMV = 0, PROF_HEAD = 1, PROF_ATTN = 2, PROF_OTHER = 3, PROF_END = -1 };

static void prof_mark(igc_session *s, int cls, double bytes) {
  if (!s->prof_on) return;
  igc_session::Mark mk;
  mk.cls = cls;
  mk.bytes = bytes;
  cudaEventCreate(&mk.ev);
  cudaEventRecord(mk.ev, s->st);
  s->marks.push_back(mk);
}

// The next launch stamp of the pass being enqueued, with its class and the
// weight bytes its launch streams (null once the stamps run out).
static unsigned long long *next_stamp(igc_session *s, int cls, double bytes) {
  if (!s->use_stamps || s->stamp_n >= IGC_STAMP_LIMIT) return nullptr;
  s->stamp_build.push_back({cls, bytes});
  return s->d_stamp + 2 * (size_t)s->stamp_n++;
}

static int gemv(igc_session *s, const DevPlane &pl, int K, int pro, int epi, const float *x, int x_stride,
                const float *p, const float *w_res, float gain, const float *w_in, float *x_out, float *out,
                int out_stride, float out_scale = 1.0f, const float *aux = nullptr, int aux_stride = 0,
                const Ssq *p_ssq = nullptr, Ssq *out_ssq = nullptr, const Ssq *x_amax = nullptr,
                Ssq *out_amax = nullptr) {
  const int cls = &pl == &s->m->head ? PROF_HEAD : PROF_GEMV;
  prof_mark(s, cls, pl.bytes);
  GemvArgs a;
  memset(&a, 0, sizeof(a));
  a.stamp = next_stamp(s, cls, pl.bytes);
  if (p_ssq) {
    a.p_ssq = p_ssq->buf;
    a.p_parts = p_ssq->parts;
    if (a.p_parts > GEMV_PART_LIMIT) return IGC_FAIL_SUPPORT;  // more partials than the prologue reads
  }
  if (out_ssq) {
    a.out_ssq = out_ssq->buf;
    out_ssq->parts = pl.grid;
  }
  if (x_amax) {  // the producer left x's magnitudes: one-pass staging
    a.x_amax = x_amax->buf;
    a.x_amax_parts = x_amax->parts;
    if (a.x_amax_parts > GEMV_PART_LIMIT) return IGC_FAIL_SUPPORT;
  }
  if (out_amax) a.out_amax = out_amax->buf;
  a.pl = pl.view();
  a.lanes = K;
  a.split = pl.split;
  a.x = x;
  a.x_stride = x_stride;
  a.p = p;
  a.p_stride = x_stride;
  a.w_res = w_res;
  a.gain = gain;
  a.w_in = w_in;
  a.eps = s->m->eps;
  a.x_out = x_out;
  a.out = out;
  a.out_stride = out_stride;
  a.out_scale = out_scale;
  a.aux = aux;
  a.aux_stride = aux_stride;
  a.cap = s->m->softcap;
  a.part_val = s->arg_val;
  a.part_idx = s->arg_idx;
  a.err = s->d_err;
  const int pair = pl.pair ? 1 : 0;
  int used = pl.grid;  // blocks the launch took: the partials it leaves
  // IGC_NO_LANE_BATCH=1 keeps them on the wide modes (for comparison)
  static const char *nb_env = getenv("IGC_NO_LANE_BATCH");
  const bool wide = pl.n_cc > 32;                                         // 8-lane staging leaves no weight ring
  const bool one_wave = (pl.grid + 1) / 2 * ((K + 3) / 4) <= s->m->sm_count;  // 16-warp blocks, one an SM
  int lb = 0;                                                             // lanes a batch
  bool wave_cap = false;                                                  // batches of four held to one wave
  if (K > 4 && epi != EPI_LOGITS && !(nb_env && nb_env[0] == '1')) {
    if (wide || one_wave) {
      lb = 4;
    } else if (!out_ssq) {
      lb = 4;
      wave_cap = true;
    } else if (K > 8) {
      lb = 8;
    }
  }
  if (lb) {
    // A projection runs its lanes in batches, side by side in one launch
    // (blockIdx.y): of four (the packed mode) where that keeps every block in
    // one wave of the SMs, and always for a plane too wide to stage eight
    // lanes with a weight ring (the 6144-column down projection would leave
    // none).  A projection that leaves no sums-of-squares partials (q|k|v,
    // gate|up) also takes batches of four where they would need a second
    // wave: its grid is held to the SMs' count over the batches, and some
    // warp groups take a second row block (each output is still summed in
    // the same order, so results do not change).  Above eight lanes
    // otherwise of eight, which takes as many blocks as one sixteen-lane
    // launch but stages a quarter of the words a warp.  The batches' weight
    // reads meet in L2.
    a.lanes = lb;
    a.lanes_total = K;
    a.batches = (K + lb - 1) / lb;
    if (igc_gemv_smem_min(&a, pair) > (size_t)s->m->smem_limit) {
      // too wide even for batches of four (the 12288-column down projection):
      // the narrower launches below
      a.lanes = K;
      a.lanes_total = 0;
      a.batches = 0;
      lb = 0;
    }
  }
  if (lb) {
    int g = pl.grid;
    if (wave_cap) {
      const int per = s->m->sm_count / a.batches;
      if (g > per) g = per > 0 ? per : 1;
    }
    CKL(igc_launch_gemv(&a, pair, pro, epi, g, (size_t)s->m->smem_limit, s->st, &used));
    if (out_ssq) out_ssq->parts = used;
    if (out_amax) out_amax->parts = used;
    return IGC_OKAY;
  }
  if (igc_gemv_smem_min(&a, pair) <= (size_t)s->m->smem_limit) {
    CKL(igc_launch_gemv(&a, pair, pro, epi, pl.grid, (size_t)s->m->smem_limit, s->st, &used));
    if (out_ssq) out_ssq->parts = used;
    if (out_amax) out_amax->parts = used;
    if (epi == EPI_LOGITS) s->head_parts = used;
    return IGC_OKAY;
  }
  // Too wide to stage every lane at once (the 6144-column down projection
  // at sixteen lanes, the doubled 12288-column one at four): launches of the
  // most lanes that fit, 8, 4, 2 or 1, each lane independent.
  if (epi == EPI_LOGITS) return IGC_FAIL_SUPPORT;
  int sub = 8;
  while (sub > 1) {
    GemvArgs t = a;
    t.lanes = K < sub ? K : sub;
    if (t.lanes < K && igc_gemv_smem_min(&t, pair) <= (size_t)s->m->smem_limit) break;
    sub /= 2;
  }
  for (int j0 = 0; j0 < K; j0 += sub) {
    GemvArgs b = a;
    b.lanes = K - j0 < sub ? K - j0 : sub;
    b.x = x + (size_t)j0 * x_stride;
    b.p = p ? p + (size_t)j0 * x_stride : nullptr;
    b.x_out = x_out ? x_out + (size_t)j0 * x_stride : nullptr;
    b.out = out + (size_t)j0 * out_stride;
    b.aux = aux ? aux + (size_t)j0 * aux_stride : nullptr;
    b.p_ssq = a.p_ssq ? a.p_ssq + (size_t)j0 * GEMV_PART_LIMIT : nullptr;  // lane-major partials
    b.out_ssq = a.out_ssq ? a.out_ssq + (size_t)j0 * GEMV_PART_LIMIT : nullptr;
    b.x_amax = a.x_amax ? a.x_amax + (size_t)j0 * GEMV_PART_LIMIT : nullptr;
    b.out_amax = a.out_amax ? a.out_amax + (size_t)j0 * GEMV_PART_LIMIT : nullptr;
    if (igc_gemv_smem_min(&b, pair) > (size_t)s->m->smem_limit) return IGC_FAIL_SUPPORT;
    CKL(igc_launch_gemv(&b, pair, pro, epi, pl.grid, (size_t)s->m->smem_limit, s->st, &used));
    if (out_ssq) out_ssq->parts = used;
    if (out_amax) out_amax->parts = used;
  }
  return IGC_OKAY;
}

// After a synchronised pass: a kernel that gave up waiting for its own bulk
// copies left the error word set (its results are not to be trusted).
static int check_err(igc_session *s) {
  if (s->h_top[IGC_LANE_LIMIT] == 0) return IGC_OKAY;
  s->h_top[IGC_LANE_LIMIT] = 0;
  cudaMemsetAsync(s->d_err, 0, sizeof(int), s->st);
  cudaStreamSynchronize(s->st);
  g_last_error = "a kernel gave up waiting for its weight copies";
  return IGC_FAIL_DEVICE;
}

// One pass of K lanes at the position in d_io[0], ids in d_io[1..K]
// (app_core.c:11843 session_pass).  want: 0 no head, 1 head and argmax.
struct PdlScope {  // kernels of a pass may start while the one ahead finishes
  explicit PdlScope(bool on) { igc_kernels_pdl(on ? 1 : 0); }
  ~PdlScope() { igc_kernels_pdl(0); }
};

static int enqueue_pass(igc_session *s, int K, int want) {
  igc_model *m = s->m;
  PdlScope pdl(s->use_pdl != 0);
  const int H = m->hidden, PS = m->layers * m->ple_dim;
  const int *d_p0 = s->d_io;
  const int32_t *d_ids = s->d_io + 1;
  s->stamp_n = 0;
  s->stamp_build.clear();
  prof_mark(s, PROF_OTHER, 0.0);
  CKL(igc_launch_embed(d_ids, K, m->embed, H, (float)sqrt((double)H), m->ple_embed, m->ple_vocab ? m->ple_vocab : 1,
                       PS, (float)sqrt((double)m->ple_dim), s->x0, s->seed, s->use_stamps ? s->d_stamp : nullptr,
                       IGC_STAMP_LIMIT, s->d_peak, s->d_peak_saved, 2 * m->layers, &m->embed_q, &m->ple_q, s->st));
  if (m->ple_dim > 0) {
    int c = gemv(s, m->ple_lift, K, PRO_F32, EPI_STORE, s->x0, H, nullptr, nullptr, 1.0f, nullptr, nullptr,
                 s->ple_raw, PS, (float)(1.0 / sqrt((double)H)));
    if (c != IGC_OKAY) return c;
    prof_mark(s, PROF_OTHER, 0.0);
    CKL(igc_launch_ple_finish(s->ple_raw, s->seed, K, m->layers, m->ple_dim, m->ple_norm, m->eps,
                              (float)(1.0 / sqrt(2.0)), s->ple, s->st));
  }
  // the residual stream ping-pongs between xa and xb; `pend` is the last
  // block's output still to be normed and added (with its gain) by the next
  // consumer's prologue, `pend_ssq` the sums of squares its producer left
  float *cur = s->x0;
  float *bufs[2] = {s->xa, s->xb};
  int flip = 0;
  const float *pend = nullptr, *pend_w = nullptr;
  float pend_gain = 1.0f;
  Ssq so{s->ssq_o, 0}, sd{s->ssq_d, 0}, spp{s->ssq_pp, 0};
  Ssq ma{s->amax_attn, 0}, mact{s->amax_act, 0}, mpa{s->amax_pa, 0};
  // producers leave magnitudes for one-pass staging downstream; the scale is
  // the one a two-pass prologue would find, so results do not depend on it
  const bool mags = true;
  Ssq *mact_out = mags ? &mact : nullptr, *mpa_out = mags ? &mpa : nullptr;
  const Ssq *ma_in = mags ? &ma : nullptr, *mact_in = mags ? &mact : nullptr, *mpa_in = mags ? &mpa : nullptr;
  const Ssq *pend_ssq = nullptr;
  auto next_x = [&]() -> float * { float *o = bufs[flip]; flip ^= 1; return o; };
  for (int l = 0; l < m->layers; ++l) {
    const DevLayer &L = m->layer[l];
    int c;
    float *xo = nullptr;
    if (pend) {
      xo = next_x();
      c = gemv(s, L.qkv, K, PRO_RESID_NORM, EPI_STORE, cur, H, pend, pend_w, pend_gain, L.enter_norm, xo, s->qkv,
               L.qkv_rows, 1.0f, nullptr, 0, pend_ssq, nullptr);
      cur = xo;
    } else {
      c = gemv(s, L.qkv, K, PRO_NORM, EPI_STORE, cur, H, nullptr, nullptr, 1.0f, L.enter_norm, nullptr, s->qkv,
               L.qkv_rows);
    }
    if (c != IGC_OKAY) return c;
    const int owner = L.share ? L.source : l;
    const DevLayer &O = m->layer[owner];
    prof_mark(s, PROF_ATTN, 0.0);
    const int sliding = L.kind == 0 ? 1 : 0;
    if (!layer_split(m, l)) {
      // queries, an owner's new rows and the attention in one kernel
      const CacheStore cq = layer_store(m, owner, L.share ? nullptr : s->d_peak + 2 * l);
      CKL(igc_launch_attn(s->qkv, L.qkv_rows, m->heads, O.kv_heads, L.hd, L.q_norm, L.k_norm, m->rope_cs[L.kind],
                          m->rope_sn[L.kind], m->eps, L.share ? 0 : 1, s->kc[owner], s->vc[owner], sliding,
                          m->slide_span, d_p0, K, s->attn_cluster, s->attn, L.q_rows, mags ? ma.buf : nullptr,
                          next_stamp(s, PROF_ATTN, 0.0), &cq, s->st));
    } else {
      // an owner's new rows written first (onto the grid on a byte side),
      // a byte side's rows the pass reads decoded to floats, then the
      // attention over those (as a sharing layer reads).  No overlap:
      // attention copies rows before its wait.
      const CacheStore cq = layer_store(m, owner, s->d_peak + 2 * l);
      igc_kernels_pdl(0);
      if (!L.share)
        CKL(igc_launch_lane_kv(s->qkv, L.qkv_rows, m->heads, O.kv_heads, L.hd, L.k_norm, m->rope_cs[L.kind],
                               m->rope_sn[L.kind], m->eps, d_p0, K, s->kc[owner], s->vc[owner], &cq, s->st));
      if (layer_bytes(m, owner)) {
        WidenArgs w = widen_of(s, owner, sliding, K);
        w.p0 = d_p0;
        CKL(igc_launch_lane_widen(&w, 1, widen_rows_most(m, sliding, K), m->sm_count, s->st));
      }
      CKL(igc_launch_attn(s->qkv, L.qkv_rows, m->heads, O.kv_heads, L.hd, L.q_norm, L.k_norm, m->rope_cs[L.kind],
                          m->rope_sn[L.kind], m->eps, 0, attn_rows(s, owner, 0), attn_rows(s, owner, 1), sliding,
                          m->slide_span, d_p0, K, s->attn_cluster, s->attn, L.q_rows, mags ? ma.buf : nullptr,
                          next_stamp(s, PROF_ATTN, 0.0), nullptr, s->st));
      igc_kernels_pdl(s->use_pdl != 0);
    }
    ma.parts = m->heads * (L.hd > 256 ? 16 : s->attn_cluster);  // a 512 head runs in clusters of 16
    c = gemv(s, L.o, K, PRO_F32, EPI_STORE, s->attn, L.q_rows, nullptr, nullptr, 1.0f, nullptr, nullptr, s->obuf, H,
             1.0f, nullptr, 0, nullptr, &so, ma_in);
    if (c != IGC_OKAY) return c;
    xo = next_x();
    c = gemv(s, L.gateup, K, PRO_RESID_NORM, EPI_GELU_PAIR, cur, H, s->obuf, L.after_attn_norm, 1.0f,
             L.before_feed_norm, xo, s->act, L.inner, 1.0f, nullptr, 0, &so, nullptr, nullptr, mact_out);
    if (c != IGC_OKAY) return c;
    cur = xo;
    c = gemv(s, L.down, K, PRO_F32, EPI_STORE, s->act, L.inner, nullptr, nullptr, 1.0f, nullptr, nullptr, s->dbuf, H,
             1.0f, nullptr, 0, nullptr, &sd, mact_in);
    if (c != IGC_OKAY) return c;
    if (m->ple_dim > 0) {
      xo = next_x();
      c = gemv(s, L.ple_gate, K, PRO_RESID, EPI_GELU_MUL, cur, H, s->dbuf, L.after_feed_norm, 1.0f, nullptr, xo,
               s->pa, m->ple_dim, 1.0f, s->ple + (size_t)l * m->ple_dim, PS, &sd, nullptr, nullptr, mpa_out);
      if (c != IGC_OKAY) return c;
      cur = xo;
      c = gemv(s, L.ple_proj, K, PRO_F32, EPI_STORE, s->pa, m->ple_dim, nullptr, nullptr, 1.0f, nullptr, nullptr,
               s->pp, H, 1.0f, nullptr, 0, nullptr, &spp, mpa_in);
      if (c != IGC_OKAY) return c;
      pend = s->pp;
      pend_w = L.after_ple_norm;
      pend_ssq = &spp;
    } else {
      pend = s->dbuf;
      pend_w = L.after_feed_norm;
      pend_ssq = &sd;
    }
    pend_gain = L.gain;
  }
  if (want) {
    float *xo = next_x();
    int c = gemv(s, m->head, K, PRO_RESID_NORM, EPI_LOGITS, cur, H, pend, pend_w, pend_gain, m->final_norm, xo,
                 s->logits, m->vocab, 1.0f, nullptr, 0, pend_ssq, nullptr);
    if (c != IGC_OKAY) return c;
    prof_mark(s, PROF_OTHER, 0.0);
    CKL(igc_launch_argmax(s->arg_val, s->arg_idx, s->head_parts, K, s->d_top, s->d_stamp,
                          s->use_stamps ? s->d_stamp_sum : nullptr, s->stamp_n, s->st));
    s->stamp_meta[K] = s->stamp_build;
  }
  prof_mark(s, PROF_END, 0.0);
  return IGC_OKAY;
}

// Runs one pass: ids and position in, argmax ids out (when want), with a
// captured graph per (K, want) after the first pass of that shape.
static int run_chunk(igc_session *s, const int32_t *ids, int M, bool head, bool want);

static int run_pass(igc_session *s, const int32_t *ids, int K, int want) {
  igc_model *m = s->m;
  if (K < 1 || K > IGC_LANE_LIMIT) return IGC_FAIL_ARGUMENT;
  if (s->fill + K > m->window_limit) return IGC_FAIL_STATE;
  for (int j = 0; j < K; ++j)
    if (ids[j] < 0 || ids[j] >= m->vocab) return IGC_FAIL_ARGUMENT;
  // a plain model's passes run through the lane stages (explicit norms and
  // grids) and its planes' CUDA-core products, the head included
  if (m->plain) return run_chunk(s, ids, K, true, want != 0);
  clear_stale("pass");
  CK(cudaSetDevice(m->device));
  s->h_io[0] = s->fill;
  memcpy(s->h_io + 1, ids, sizeof(int32_t) * (size_t)K);
  CK(cudaMemcpyAsync(s->d_io, s->h_io, sizeof(int32_t) * (size_t)(1 + K), cudaMemcpyHostToDevice, s->st));
  int w = want ? 1 : 0;
  if (s->use_graphs) {
    if (!s->graph[K][w]) {
      cudaGraph_t g;
      long before = g_launches;
      CK(cudaStreamBeginCapture(s->st, cudaStreamCaptureModeThreadLocal));
      int c = enqueue_pass(s, K, want);
      cudaError_t e = cudaStreamEndCapture(s->st, &g);
      if (c != IGC_OKAY) return c;
      if (e != cudaSuccess) return fail_device(e, "capture");
      s->kernels_per_pass[K][w] = g_launches - before;
      g_launches = before;
      e = cudaGraphInstantiate(&s->graph[K][w], g, 0);
      cudaGraphDestroy(g);
      if (e != cudaSuccess) return fail_device(e, "graph instantiate");
    }
    CK(cudaGraphLaunch(s->graph[K][w], s->st));
    g_launches += s->kernels_per_pass[K][w];
  } else {
    int c = enqueue_pass(s, K, want);
    if (c != IGC_OKAY) return c;
  }
  CK(cudaMemcpyAsync(s->h_top, s->d_top, sizeof(int32_t) * (IGC_LANE_LIMIT + 1), cudaMemcpyDeviceToHost, s->st));
  CK(cudaStreamSynchronize(s->st));
  if (int ce = check_err(s)) return ce;
  s->fill += K;
  for (int j = 0; j < K; ++j)
    if ((int)s->echo.size() < m->window_limit) s->echo.push_back(ids[j]);
  s->logit_lanes = want ? K : 0;
  return IGC_OKAY;
}

// ---------------------------------------------------------------------------
// the batched-lane passes: every projection a tcgen05 GEMM (igc_lanes.cu)
// with a row-wise stage before it.  Two callers: the prime, in chunks of up
// to 512 lanes of one session (the keys and values of all its lanes written
// to the cache first, then the attention of all its 16-lane groups in one
// launch), and the crowd (igc_crowd_round), one block of k lanes from each of
// many sessions (attention for all of them in one launch).

// Lanes a prime chunk.  512 measured 11% faster than 256 at 4096 and 8192
// ids (fewer weight sweeps; IGC_CHUNK_LANES=256 or 128 in the environment
// for comparison).
constexpr int IGC_CHUNK_LANES = 512;

static int chunk_lanes() {
  static const int n = [] {
    const char *e = getenv("IGC_CHUNK_LANES");
    const int v = e ? atoi(e) : 0;
    return v == 256 || v == 128 ? v : IGC_CHUNK_LANES;
  }();
  return n;
}
constexpr int IGC_CHUNK_MIN = 64;     // fewer lanes than this run as 16-lane passes

// Sizes `B` for passes of up to `cap` lanes.  `split_lanes` > 0 fixes every
// product's K slices to those of a pass of that many lanes (results then do
// not depend on how many lanes a pass carries); 0 lets each pass choose.
static int lane_buf_alloc(igc_model *m, LaneBuf &B, int cap, int split_lanes, std::vector<void *> &owned) {
  const int H = m->hidden, PS = m->layers * m->ple_dim;
  size_t part = 0;
  int max_cc = 1;
  auto see = [&](const DevPlane &pl) {
    if (!pl.tiles && pl.plain.empty()) return;
    if (m->plain)
      part = std::max(part, (size_t)cap * pl.n_rb * 16);  // one slice: the products write whole sums
    else if (split_lanes > 0)
      part = std::max(part, (size_t)igc_lane_gemm_split(split_lanes, pl.n_rb, pl.n_cc, m->sm_count) * cap * pl.n_rb * 16);
    else
      for (int lanes = 1; lanes <= cap; ++lanes)
        part = std::max(part, (size_t)igc_lane_gemm_split(lanes, pl.n_rb, pl.n_cc, m->sm_count) * lanes * pl.n_rb * 16);
    max_cc = std::max(max_cc, pl.n_cc);
  };
  see(m->ple_lift);
  for (auto &L : m->layer) {
    see(L.qkv);
    see(L.o);
    see(L.gateup);
    see(L.down);
    see(L.ple_gate);
    see(L.ple_proj);
  }
  max_cc = std::max(max_cc, m->head.n_cc);
  auto grab = [&](auto **p, size_t count) -> int {
    void *v = nullptr;
    cudaError_t e = cudaMalloc(&v, (count ? count : 1) * sizeof(**p));
    if (e != cudaSuccess) return fail_device(e, "cudaMalloc(lanes)");
    owned.push_back(v);
    *p = (std::remove_reference_t<decltype(*p)>)v;
    return IGC_OKAY;
  };
  int c = IGC_OKAY;
  if (c == IGC_OKAY) c = grab(&B.x0, (size_t)cap * H);
  if (c == IGC_OKAY) c = grab(&B.xa, (size_t)cap * H);
  if (c == IGC_OKAY) c = grab(&B.xb, (size_t)cap * H);
  if (c == IGC_OKAY) c = grab(&B.seed, (size_t)cap * (PS ? PS : 1));
  if (c == IGC_OKAY) c = grab(&B.ple_raw, (size_t)cap * (PS ? PS : 1));
  if (c == IGC_OKAY) c = grab(&B.ple, (size_t)cap * (PS ? PS : 1));
  if (c == IGC_OKAY) c = grab(&B.qkv, (size_t)cap * m->max_qkv);
  if (c == IGC_OKAY) c = grab(&B.attn, (size_t)cap * m->max_q);
  if (c == IGC_OKAY) c = grab(&B.part, part);
  if (c == IGC_OKAY) c = grab(&B.factor, (size_t)cap);
  if (c == IGC_OKAY && m->plain) c = grab(&B.rows, (size_t)cap * std::max(m->plain_cols, H));
  if (c == IGC_OKAY) c = grab((uint8_t **)&B.a_tiles, (size_t)((cap + LG_M - 1) / LG_M) * max_cc * LG_A_STEP_BYTES);
  // the head's argmax partials: one a 128-row tile, or a plain product's block
  const size_t head_tiles = m->plain ? (size_t)igc_plain_blocks(m->head.rows)
                                     : (size_t)(m->head.n_rb + LG_N / 16 - 1) / (LG_N / 16);
  if (c == IGC_OKAY) c = grab(&B.arg_val, head_tiles * cap);
  if (c == IGC_OKAY) c = grab(&B.arg_idx, head_tiles * cap);
  if (c != IGC_OKAY) return c;
  B.cap = cap;
  B.split_lanes = split_lanes;
  return IGC_OKAY;
}

// One pass of the batched-lane path over the stack's layers.
struct LaneRun {
  igc_model *m;
  cudaStream_t st;
  LaneBuf *B;
  int *d_err;
  int M;  // lanes
  // a session's cache peaks, copied by the embedding kernel before a block
  // that may be undone (a plain model's steps and blocks)
  float *peak = nullptr, *peak_saved = nullptr;
};

static LaneStageArgs stage_of(int mode, const float *x, int x_stride) {
  LaneStageArgs a;
  memset(&a, 0, sizeof(a));
  a.mode = mode;
  a.x = x;
  a.x_stride = x_stride;
  a.gain = 1.0f;
  a.out_scale = 1.0f;
  return a;
}

// A stage into the pass's operand blocks for the product `pl` (its columns
// and steps), then the product: K-slice partials into B.part, or with `head`
// set the output head's argmax partials (and logits into `logits` when given).
static int lane_product(LaneRun &r, const DevPlane &pl, LaneStageArgs sa, int *split_out, bool head = false,
                        float *logits = nullptr, int *head_parts = nullptr) {
  LaneBuf &B = *r.B;
  if (!pl.plain.empty()) {
    // a plain plane: the staged rows as f32, then one CUDA-core product a
    // part, each writing whole sums into its rows of the plane's output
    const int stride = std::max(r.m->plain_cols, r.m->hidden);
    sa.lanes = r.M;
    sa.cols = pl.cols;
    sa.n_cc = 0;
    sa.a_tiles = nullptr;
    sa.factor = B.factor;
    sa.eps = r.m->eps;
    sa.row_out = B.rows;
    sa.row_stride = stride;
    CKL(igc_launch_lane_stage(&sa, r.st));
    for (const PlainArgs &part : pl.plain) {
      PlainArgs a = part;
      a.x = B.rows;
      a.x_stride = stride;
      a.lanes = r.M;
      a.out_scale = sa.out_scale;
      if (head) {
        a.out = logits;
        a.out_stride = pl.rows;
        a.cap = r.m->softcap;
        a.arg_val = B.arg_val;
        a.arg_idx = B.arg_idx;
      } else {
        a.out = B.part;
        a.out_stride = pl.n_rb * 16;
      }
      int blocks = 0;
      CKL(igc_launch_plain_product(&a, r.m->sm_count, &blocks, r.st));
      if (head_parts) *head_parts = blocks;
    }
    *split_out = 1;
    return IGC_OKAY;
  }
  sa.lanes = r.M;
  sa.cols = pl.cols;
  sa.n_cc = pl.n_cc;
  sa.a_tiles = B.a_tiles;
  sa.factor = B.factor;
  sa.eps = r.m->eps;
  CKL(igc_launch_lane_stage(&sa, r.st));
  LaneGemmArgs ga;
  memset(&ga, 0, sizeof(ga));
  ga.tiles = pl.tiles;
  ga.scales = pl.scales;
  ga.n_rb = pl.n_rb;
  ga.n_cc = pl.n_cc;
  ga.a_tiles = reinterpret_cast<const uint4 *>(B.a_tiles);
  ga.factor = B.factor;
  ga.lanes = r.M;
  ga.err = r.d_err;
  if (head) {
    ga.split = 1;
    ga.out = logits;
    ga.out_stride = pl.rows;
    ga.arg_val = B.arg_val;
    ga.arg_idx = B.arg_idx;
    ga.rows = pl.rows;
    ga.cap = r.m->softcap;
  } else {
    ga.out = B.part;
    ga.out_stride = pl.n_rb * 16;
    ga.split = igc_lane_gemm_split(B.split_lanes > 0 ? B.split_lanes : r.M, pl.n_rb, pl.n_cc, r.m->sm_count);
  }
  if (!pl.tm_ok) return IGC_FAIL_SUPPORT;  // the driver offered no tensor-map encoder
  CKL(igc_launch_lane_gemm(&ga, &pl.tm_codes, &pl.tm_scales, r.st));
  *split_out = ga.split;
  return IGC_OKAY;
}

// embed, the per-layer-embedding lift, the layers (attention by `attend`),
// and with `top` the final norm, the head and each lane's argmax.
template <typename Attend>
static int lane_stack(LaneRun &r, const int32_t *d_ids, Attend attend, int32_t *top = nullptr,
                      float *logits = nullptr) {
  igc_model *m = r.m;
  LaneBuf &B = *r.B;
  const int H = m->hidden, PS = m->layers * m->ple_dim, M = r.M;
  int c, split = 1;
  CKL(igc_launch_embed(d_ids, M, m->embed, H, (float)sqrt((double)H), m->ple_embed, m->ple_vocab ? m->ple_vocab : 1,
                       PS, (float)sqrt((double)m->ple_dim), B.x0, B.seed, nullptr, 0, r.peak, r.peak_saved,
                       r.peak_saved ? 2 * m->layers : 0, &m->embed_q, &m->ple_q, r.st));
  if (m->ple_dim > 0) {
    LaneStageArgs sa = stage_of(LS_PLAIN, B.x0, H);
    sa.out_scale = (float)(1.0 / sqrt((double)H));
    c = lane_product(r, m->ple_lift, sa, &split);
    if (c != IGC_OKAY) return c;
    CKL(igc_launch_lane_sum(B.part, split, M, PS, m->ple_lift.n_rb * 16, B.ple_raw, PS, r.st));
    CKL(igc_launch_ple_finish(B.ple_raw, B.seed, M, m->layers, m->ple_dim, m->ple_norm, m->eps,
                              (float)(1.0 / sqrt(2.0)), B.ple, r.st));
  }
  // the residual stream ping-pongs between xa and xb; `pend` (in B.part,
  // `pend_split` slices of `pend_stride`) is the last block's output still
  // to be normed and added (with its gain) by the next stage
  float *cur = B.x0;
  float *bufs[2] = {B.xa, B.xb};
  int flip = 0;
  auto next_x = [&]() -> float * { float *o = bufs[flip]; flip ^= 1; return o; };
  bool pend = false;
  int pend_split = 1, pend_stride = 0;
  const float *pend_w = nullptr;
  float pend_gain = 1.0f;
  auto resid = [&](LaneStageArgs &sa) {  // the next stage adds the pending block
    float *xo = next_x();
    sa.p = B.part;
    sa.p_splits = pend_split;
    sa.p_stride = pend_stride;
    sa.w_res = pend_w;
    sa.gain = pend_gain;
    sa.x_out = xo;
    cur = xo;
  };
  for (int l = 0; l < m->layers; ++l) {
    const DevLayer &L = m->layer[l];
    {  // q|k|v
      LaneStageArgs sa = stage_of(pend ? LS_RESID_NORM : LS_NORM, cur, H);
      sa.w_in = L.enter_norm;
      if (pend) resid(sa);
      c = lane_product(r, L.qkv, sa, &split);
      if (c != IGC_OKAY) return c;
      CKL(igc_launch_lane_sum(B.part, split, M, L.qkv_rows, L.qkv.n_rb * 16, B.qkv, L.qkv_rows, r.st));
    }
    c = attend(l, L);
    if (c != IGC_OKAY) return c;
    c = lane_product(r, L.o, stage_of(LS_PLAIN, B.attn, L.q_rows), &split);
    if (c != IGC_OKAY) return c;
    {  // gate|up: x += norm(o) * w, then norm(x) * w
      pend_split = split;
      pend_stride = L.o.n_rb * 16;
      pend_w = L.after_attn_norm;
      pend_gain = 1.0f;
      LaneStageArgs sa = stage_of(LS_RESID_NORM, cur, H);
      resid(sa);
      sa.w_in = L.before_feed_norm;
      c = lane_product(r, L.gateup, sa, &split);
      if (c != IGC_OKAY) return c;
    }
    {  // down: gelu(gate) * up
      LaneStageArgs sa = stage_of(LS_GELU_PAIR, nullptr, 0);
      sa.p = B.part;
      sa.p_splits = split;
      sa.p_stride = L.gateup.n_rb * 16;
      c = lane_product(r, L.down, sa, &split);
      if (c != IGC_OKAY) return c;
    }
    pend_split = split;
    pend_stride = L.down.n_rb * 16;
    pend_w = L.after_feed_norm;
    pend_gain = 1.0f;
    if (m->ple_dim > 0) {
      // per-layer-embedding gate: x += norm(down) * w
      LaneStageArgs sa = stage_of(LS_RESID, cur, H);
      resid(sa);
      c = lane_product(r, L.ple_gate, sa, &split);
      if (c != IGC_OKAY) return c;
      // its projection: gelu(gate) * the layer's per-layer input
      LaneStageArgs sb = stage_of(LS_GELU_MUL, nullptr, 0);
      sb.p = B.part;
      sb.p_splits = split;
      sb.p_stride = L.ple_gate.n_rb * 16;
      sb.aux = B.ple + (size_t)l * m->ple_dim;
      sb.aux_stride = PS;
      c = lane_product(r, L.ple_proj, sb, &split);
      if (c != IGC_OKAY) return c;
      pend_split = split;
      pend_stride = L.ple_proj.n_rb * 16;
      pend_w = L.after_ple_norm;
    }
    pend = true;
    pend_gain = L.gain;
  }
  if (top) {
    // app_core.c:11897-11976: final norm, head, soft cap, argmax
    LaneStageArgs sa = stage_of(pend ? LS_RESID_NORM : LS_NORM, cur, H);
    sa.w_in = m->final_norm;
    if (pend) resid(sa);
    int parts = (m->head.n_rb + LG_N / 16 - 1) / (LG_N / 16);
    c = lane_product(r, m->head, sa, &split, true, logits, &parts);
    if (c != IGC_OKAY) return c;
    CKL(igc_launch_lane_argmax(B.arg_val, B.arg_idx, parts, M, top, r.st));
  }
  return IGC_OKAY;
}

static int chunks_ready(igc_session *s) {
  auto &C = s->ch;
  if (C.B.cap) return IGC_OKAY;
  const int M = chunk_lanes();
  igc_model *m = s->m;
  int c = lane_buf_alloc(m, C.B, M, 0, s->owned);
  C.groups_cap = M / 16 + 1;
  if (c == IGC_OKAY) c = s->alloc(&C.d_ids, 1 + M);
  if (c == IGC_OKAY) c = s->alloc(&C.d_pos, C.groups_cap);
  if (c == IGC_OKAY) c = s->alloc(&C.kc_tab, (size_t)m->layers * C.groups_cap);
  if (c == IGC_OKAY) c = s->alloc(&C.vc_tab, (size_t)m->layers * C.groups_cap);
  if (c != IGC_OKAY) return c;
  std::vector<float *> hk((size_t)m->layers * C.groups_cap), hv(hk.size());
  for (int l = 0; l < m->layers; ++l) {
    const int owner = m->layer[l].share ? m->layer[l].source : l;
    for (int z = 0; z < C.groups_cap; ++z) {
      hk[(size_t)l * C.groups_cap + z] = attn_rows(s, owner, 0);
      hv[(size_t)l * C.groups_cap + z] = attn_rows(s, owner, 1);
    }
  }
  CK(cudaMemcpy(C.kc_tab, hk.data(), sizeof(float *) * hk.size(), cudaMemcpyHostToDevice));
  CK(cudaMemcpy(C.vc_tab, hv.data(), sizeof(float *) * hv.size(), cudaMemcpyHostToDevice));
  CK(cudaMallocHost(&C.h_ids, sizeof(int32_t) * (1 + M)));
  return IGC_OKAY;
}

// One chunk of M lanes at the position in ch.d_ids[0], ids in ch.d_ids[1..M]
// (app_core.c:11843 session_pass without the head: a prime keeps no logits).
static int enqueue_chunk(igc_session *s, int M, bool head, bool want) {
  igc_model *m = s->m;
  auto &C = s->ch;
  // kernels overlap the one ahead (each waits before reading its results),
  // except the attention groups: a group copies cached rows before its wait,
  // and those rows are the previous group's own writes
  PdlScope pdl(s->use_pdl != 0);
  const int groups = (M + 15) / 16;
  CKL(igc_launch_lane_positions(C.d_ids, groups, C.d_pos, s->st));
  LaneRun r{m, s->st, &C.B, s->d_err, M};
  // Attention: an owner layer first writes every lane's new key and value
  // rows to its cache; then every 16-lane group reads all its rows from the
  // cache (as a sharing layer does), all full groups in one launch
  // (blockIdx.z the group) and a ragged last group in another.  These launch
  // without overlap: a group copies cached rows before its own wait, and
  // those rows are the prep launch's writes.
  auto attend = [&](int l, const DevLayer &L) -> int {
    const int owner = L.share ? L.source : l;
    const DevLayer &O = m->layer[owner];
    const int full = M / 16, tail = M - 16 * full, sliding = L.kind == 0 ? 1 : 0;
    const int G = m->heads / O.kv_heads;
    const int cx_set = sliding ? s->chunk_cluster : s->chunk_cluster_global;
    const int slots = m->sm_count * (attn_light() ? 2 : 1);
    const int cx = cx_set ? cx_set : attn_cluster_for((long)(full > 0 ? full : 1) * O.kv_heads * ((16 * G + 15) / 16), slots);
    // the ragged last group runs alone, so it takes clusters sized for its own few blocks
    const int cx_tail = cx_set ? cx_set : attn_cluster_for((long)O.kv_heads * ((tail * G + 15) / 16), slots);
    igc_kernels_pdl(0);
    const CacheStore kv = layer_store(m, owner, s->d_peak + 2 * owner);
    if (!L.share)
      CKL(igc_launch_lane_kv(C.B.qkv, L.qkv_rows, m->heads, O.kv_heads, L.hd, L.k_norm, m->rope_cs[L.kind],
                             m->rope_sn[L.kind], m->eps, C.d_ids, M, s->kc[owner], s->vc[owner], &kv, s->st));
    if (layer_bytes(m, owner)) {
      // a byte cache's rows the chunk reads, decoded to floats (all groups at once)
      WidenArgs w = widen_of(s, owner, sliding, M);
      w.p0 = C.d_ids;
      CKL(igc_launch_lane_widen(&w, 1, widen_rows_most(m, sliding, M), m->sm_count, s->st));
    }
    if (full > 0)
      CKL(igc_launch_attn_many(C.B.qkv, L.qkv_rows, m->heads, O.kv_heads, L.hd, L.q_norm, L.k_norm,
                               m->rope_cs[L.kind], m->rope_sn[L.kind], m->eps, 0, nullptr, nullptr, sliding,
                               m->slide_span, C.d_pos, 16, cx, C.B.attn, L.q_rows, nullptr, nullptr,
                               C.kc_tab + (size_t)l * C.groups_cap, C.vc_tab + (size_t)l * C.groups_cap, C.d_pos,
                               full, nullptr, s->st, attn_light()));
    if (tail > 0)
      CKL(igc_launch_attn(C.B.qkv + (size_t)16 * full * L.qkv_rows, L.qkv_rows, m->heads, O.kv_heads, L.hd, L.q_norm,
                          L.k_norm, m->rope_cs[L.kind], m->rope_sn[L.kind], m->eps, 0, attn_rows(s, owner, 0),
                          attn_rows(s, owner, 1), sliding, m->slide_span, C.d_pos + full, tail, cx_tail,
                          C.B.attn + (size_t)16 * full * L.q_rows, L.q_rows, nullptr, nullptr, nullptr, s->st,
                          attn_light()));
    igc_kernels_pdl(s->use_pdl != 0);
    return IGC_OKAY;
  };
  if (head) {
    r.peak = s->d_peak;
    r.peak_saved = s->d_peak_saved;
    return lane_stack(r, C.d_ids + 1, attend, s->d_top, want ? s->logits : nullptr);
  }
  return lane_stack(r, C.d_ids + 1, attend);
}

// One chunk of M lanes (64 <= M <= chunk_lanes(); any M for a plain model),
// kept, with a captured graph per chunk shape.  With `head` (a plain model's
// step or block, M <= 16) it ends in each lane's argmax, and with `want` the
// lanes' logits too.
static int run_chunk(igc_session *s, const int32_t *ids, int M, bool head = false, bool want = false) {
  igc_model *m = s->m;
  auto &C = s->ch;
  int c = chunks_ready(s);
  if (c != IGC_OKAY) return c;
  clear_stale("prime chunk");
  CK(cudaSetDevice(m->device));
  C.h_ids[0] = s->fill;
  memcpy(C.h_ids + 1, ids, sizeof(int32_t) * (size_t)M);
  CK(cudaMemcpyAsync(C.d_ids, C.h_ids, sizeof(int32_t) * (size_t)(1 + M), cudaMemcpyHostToDevice, s->st));
  const int key = 4 * M + (head ? 2 : 0) + (want ? 1 : 0);
  if (s->use_graphs) {
    auto it = C.graph.find(key);
    if (it == C.graph.end()) {
      cudaGraph_t g;
      long before = g_launches;
      CK(cudaStreamBeginCapture(s->st, cudaStreamCaptureModeThreadLocal));
      c = enqueue_chunk(s, M, head, want);
      cudaError_t e = cudaStreamEndCapture(s->st, &g);
      if (c != IGC_OKAY) return c;
      if (e != cudaSuccess) return fail_device(e, "capture");
      cudaGraphExec_t ex;
      e = cudaGraphInstantiate(&ex, g, 0);
      cudaGraphDestroy(g);
      if (e != cudaSuccess) return fail_device(e, "graph instantiate");
      it = C.graph.emplace(key, ex).first;
      s->kernels_per_chunk[key] = g_launches - before;
      g_launches = before;
    }
    CK(cudaGraphLaunch(it->second, s->st));
    g_launches += s->kernels_per_chunk[key];
  } else {
    c = enqueue_chunk(s, M, head, want);
    if (c != IGC_OKAY) return c;
  }
  CK(cudaMemcpyAsync(s->h_top, s->d_top, sizeof(int32_t) * (IGC_LANE_LIMIT + 1), cudaMemcpyDeviceToHost, s->st));
  CK(cudaStreamSynchronize(s->st));
  if (int ce = check_err(s)) return ce;
  s->fill += M;
  for (int j = 0; j < M; ++j)
    if ((int)s->echo.size() < m->window_limit) s->echo.push_back(ids[j]);
  s->logit_lanes = head && want ? M : 0;
  return IGC_OKAY;
}

extern "C" int igc_session_prime(igc_session *s, const int32_t *ids, int n) { /* app_core.c:14443 */
  if (!s || !ids || n < 1) return IGC_FAIL_ARGUMENT;
  if (s->guess_count > 0) return IGC_FAIL_STATE;
  if (s->fill + n > s->m->window_limit) return IGC_FAIL_STATE;
  for (int i = 0; i < n; ++i)
    if (ids[i] < 0 || ids[i] >= s->m->vocab) return IGC_FAIL_ARGUMENT;
  // every id but the last (which the caller steps): chunks of many lanes
  // through the tcgen05 path while at least IGC_CHUNK_MIN remain, then
  // passes of at most 16 lanes (the reference's chunking, app_core.c:14443)
  for (int i = 0; i + 1 < n;) {
    int left = n - 1 - i, c;
    if (s->m->plain || (s->use_chunks && left >= IGC_CHUNK_MIN)) {
      const int lanes = left < chunk_lanes() ? left : chunk_lanes();
      c = run_chunk(s, ids + i, lanes);
      i += lanes;
    } else {
      const int lanes = left > IGC_LANE_LIMIT ? IGC_LANE_LIMIT : left;
      c = run_pass(s, ids + i, lanes, 0);
      i += lanes;
    }
    if (c != IGC_OKAY) return c;
  }
  return IGC_OKAY;
}

static double now_seconds() {
  return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

extern "C" int igc_session_step(igc_session *s, int32_t id, float *logits_out, int32_t *top_out) {
  if (!s) return IGC_FAIL_ARGUMENT;
  if (s->guess_count > 0) return IGC_FAIL_STATE;
  double t0 = now_seconds();
  int c = run_pass(s, &id, 1, 1);
  if (c != IGC_OKAY) return c;
  s->serve_seconds += now_seconds() - t0;
  s->serve_tokens += 1;
  if (top_out) *top_out = s->h_top[0];
  if (logits_out) CK(cudaMemcpy(logits_out, s->logits, sizeof(float) * (size_t)s->m->vocab, cudaMemcpyDeviceToHost));
  return IGC_OKAY;
}

extern "C" int igc_session_guess(igc_session *s, const int32_t *ids, int k, float *logits_out) {
  if (!s || !ids) return IGC_FAIL_ARGUMENT;
  if (s->guess_count > 0) return IGC_FAIL_STATE;
  if (k < 1 || k > IGC_LANE_LIMIT) return IGC_FAIL_ARGUMENT;
  if (s->fill + k > s->m->window_limit) return IGC_FAIL_STATE;
  s->guess_from = s->fill;
  s->guess_echo = (int)s->echo.size();
  double t0 = now_seconds();
  int c = run_pass(s, ids, k, 1);
  if (c != IGC_OKAY) return c;
  s->serve_seconds += now_seconds() - t0;
  s->guess_count = k;
  if (logits_out)
    CK(cudaMemcpy(logits_out, s->logits, sizeof(float) * (size_t)s->m->vocab * k, cudaMemcpyDeviceToHost));
  return IGC_OKAY;
}

extern "C" int igc_session_guess_top(igc_session *s, int32_t *top_out) {
  if (!s || !top_out) return IGC_FAIL_ARGUMENT;
  if (s->guess_count <= 0) return IGC_FAIL_STATE;
  memcpy(top_out, s->h_top, sizeof(int32_t) * (size_t)s->guess_count);
  return IGC_OKAY;
}

extern "C" int igc_session_guess_keep(igc_session *s, int keep) { /* app_core.c:12205 */
  if (!s || s->guess_count <= 0) return IGC_FAIL_STATE;
  if (keep < 0 || keep > s->guess_count) return IGC_FAIL_ARGUMENT;
  s->serve_tokens += (size_t)keep;
  s->fill = s->guess_from + keep;
  s->echo.resize((size_t)std::min(s->guess_echo + keep, s->m->window_limit));
  s->guess_count = 0;
  if (keep == 0) {
    // a block undone whole leaves the peaks where they stood (app_core.c:12208-12213)
    CK(cudaMemcpyAsync(s->d_peak, s->d_peak_saved, sizeof(float) * 2 * (size_t)s->m->layers,
                       cudaMemcpyDeviceToDevice, s->st));
    CK(cudaStreamSynchronize(s->st));
  }
  return IGC_OKAY;
}

// ---------------------------------------------------------------------------
// cache files (app_core.c:13864-14182 session_save / session_load): the
// reference's layout, so a file either engine writes is one the other reads.
//
//   16 bytes   "igllm cache 4\n\0\0"
//   7 x u64    keep mark, caller's stamp, fill, ids held, layers, cache_bits,
//              kind (IGC_KEEP_PROMPT / IGC_KEEP_TALK)
//   u64        runs, then 3 x u64 a run (first id, one past the last, mark)
//   i32 x ids  the ids held
//   per owner layer with rows: its key rows, then its value rows, as the
//              reference's ring holds them (slot = position mod span), each
//              value a float or an e4m3 byte as the side stores it
//   f32 x layers  key peaks, then f32 x layers value peaks
//
// This library's caches are full length, so a save gathers the ring's order
// (a turned-over ring is the last `span` positions, rotated) and a load puts
// rows back at their positions; a load from a turned-over ring leaves the
// rows before it absent, which `floor` records for igc_session_hold.

static const char k_keep_text[16] = {'i', 'g', 'l', 'l', 'm', ' ', 'c', 'a', 'c', 'h', 'e', ' ', '4', '\n', 0, 0};

// the file's 64-bit fold (app_core.c:12888 keep_mix; the boost hash_combine step)
static uint64_t keep_mix(uint64_t mark, uint64_t value) {
  mark ^= value + 0x9E3779B97F4A7C15ull + (mark << 6) + (mark >> 2);
  return mark;
}

// What decides a cache's layout, folded (app_core.c:13869 keep_mark): the
// shapes, the storage, the checkpoint's size, and per layer its ring, heads
// and bytes a value.
static uint64_t keep_mark(const igc_session *s) {
  const igc_model *m = s->m;
  uint64_t mark = 0x243F6A8885A308D3ull;
  mark = keep_mix(mark, (uint64_t)m->layers);
  mark = keep_mix(mark, (uint64_t)m->heads);
  mark = keep_mix(mark, (uint64_t)m->hidden);
  mark = keep_mix(mark, (uint64_t)m->window_limit);
  mark = keep_mix(mark, (uint64_t)m->slide_span);
  mark = keep_mix(mark, (uint64_t)(int64_t)m->cache_bits);
  mark = keep_mix(mark, (uint64_t)m->vocab);
  mark = keep_mix(mark, (uint64_t)m->weight_bytes);
  for (int l = 0; l < m->layers; ++l) {
    const DevLayer &L = m->layer[l];
    const CacheStore cq = layer_store(m, L.share ? L.source : l, nullptr);
    mark = keep_mix(mark, (uint64_t)L.span);
    mark = keep_mix(mark, (uint64_t)L.kv_heads);
    mark = keep_mix(mark, (uint64_t)L.hd);
    mark = keep_mix(mark, (uint64_t)L.share);
    mark = keep_mix(mark, (uint64_t)(L.share ? sizeof(float) : side_bytes(cq.kq)));
    mark = keep_mix(mark, (uint64_t)(L.share ? sizeof(float) : side_bytes(cq.vq)));
  }
  return mark;
}

// app_core.c:13957 keep_note_sane: runs in order, each non-empty, none past
// the context.
static bool note_sane(const igc_keep_note *n, int window) {
  if (n->run_count < 0 || n->run_count > IGC_KEEP_RUNS) return false;
  for (int i = 0; i < n->run_count; ++i) {
    if (n->from_list[i] < 0 || n->till_list[i] <= n->from_list[i]) return false;
    if (n->till_list[i] > window) return false;
    if (i > 0 && n->from_list[i] < n->till_list[i - 1]) return false;
  }
  return true;
}

// app_core.c:13991 keep_note_share: the shared prefix ends at the first run,
// inside it, that either side lacks, that the two place or fold differently,
// or that reaches past it.
extern "C" int igc_keep_note_share(const igc_keep_note *held, const igc_keep_note *now, int same_count) {
  if (!held || !now || same_count < 0) return 0;
  const int most = std::max(held->run_count, now->run_count);
  for (int i = 0; i < most; ++i) {
    const bool in_h = i < held->run_count, in_n = i < now->run_count;
    const int hf = in_h ? held->from_list[i] : same_count, nf = in_n ? now->from_list[i] : same_count;
    const int from = std::min(hf, nf);
    if (from >= same_count) break;
    if (!in_h || !in_n || hf != nf || held->till_list[i] != now->till_list[i] ||
        held->mark_list[i] != now->mark_list[i] || held->till_list[i] > same_count)
      return from;
  }
  return same_count;
}

// The ring order of an owner's `rows` kept rows at fill `fill`: the file's
// slots [0, rows) come from positions [first[0], first[0] + count[0]) then
// [first[1], first[1] + count[1]).
struct RingRuns {
  int first[2], count[2];
};
static RingRuns ring_runs(int fill, int span) {
  RingRuns r{{0, 0}, {0, 0}};
  if (fill <= span) {
    r.count[0] = fill;
    return r;
  }
  const int turn = fill % span;  // slots [0, turn) hold the newest positions
  r.first[0] = fill - turn;
  r.count[0] = turn;
  r.first[1] = fill - span;
  r.count[1] = span - turn;
  return r;
}

extern "C" size_t igc_model_memory_bytes(const igc_model *m) { return m ? m->weight_bytes : 0; }

extern "C" float igc_model_cache_scale(const igc_model *m, int layer, int value_side) { /* app_core.c:14515 */
  if (!m || layer < 0 || layer >= m->layers) return 0.0f;
  return value_side ? m->layer[layer].v_scale : m->layer[layer].k_scale;
}

extern "C" float igc_session_cache_peak(const igc_session *s, int layer, int value_side) { /* app_core.c:14540 */
  if (!s || layer < 0 || layer >= s->m->layers) return 0.0f;
  float v = 0.0f;
  cudaSetDevice(s->m->device);
  if (cudaMemcpyAsync(&v, s->d_peak + 2 * layer + (value_side ? 1 : 0), sizeof(float), cudaMemcpyDeviceToHost,
                      s->st) != cudaSuccess ||
      cudaStreamSynchronize(s->st) != cudaSuccess)
    return 0.0f;
  return v;
}

// Bytes the caches occupy at `cache_bits` storage: this library keeps every
// owner full length (window_limit rows), so this is more than the
// reference's rings for the same model (app_core.c:14522 counts rings).
extern "C" size_t igc_session_cache_room_at(const igc_session *s, int cache_bits) {
  if (!s) return 0;
  const igc_model *m = s->m;
  size_t total = 0;
  for (int l = 0; l < m->layers; ++l) {
    const DevLayer &L = m->layer[l];
    if (L.share) continue;
    const size_t slots = (size_t)m->window_limit * L.kv_rows;
    total += slots * (cache_bits == 8 && L.k_scale > 0.0f ? 1u : sizeof(float));
    total += slots * (cache_bits == 8 && L.v_scale > 0.0f ? 1u : sizeof(float));
  }
  return total;
}
extern "C" size_t igc_session_cache_room(const igc_session *s) {
  return s ? igc_session_cache_room_at(s, s->m->cache_bits) : 0;
}

extern "C" int igc_session_ids(const igc_session *s, int32_t *ids, int limit) { /* app_core.c:14183 */
  if (!s) return -1;
  const int n = (int)s->echo.size();
  if (!ids || limit < n) return n;
  if (n > 0) memcpy(ids, s->echo.data(), sizeof(int32_t) * (size_t)n);
  return n;
}

namespace {
struct FileCloser {
  FILE *f;
  ~FileCloser() {
    if (f) fclose(f);
  }
};
}  // namespace

extern "C" int igc_session_save(const igc_session *s, const char *path, uint64_t stamp, const igc_keep_note *note,
                                int kind) { /* app_core.c:14010 */
  if (!s || !path) return IGC_FAIL_ARGUMENT;
  if (s->guess_count > 0) return IGC_FAIL_STATE;
  if (kind != IGC_KEEP_PROMPT && kind != IGC_KEEP_TALK) return IGC_FAIL_ARGUMENT;
  const igc_model *m = s->m;
  if (note && !note_sane(note, m->window_limit)) return IGC_FAIL_ARGUMENT;
  clear_stale("session save");
  CK(cudaSetDevice(m->device));
  // everything off the device first, so a failed copy writes no file
  std::vector<std::vector<uint8_t>> rows((size_t)m->layers);
  for (int l = 0; l < m->layers; ++l) {
    const DevLayer &L = m->layer[l];
    if (L.share) continue;
    const int n = std::min(s->fill, L.span);
    if (n < 1) continue;
    const CacheStore cq = layer_store(m, l, nullptr);
    const RingRuns rr = ring_runs(s->fill, L.span);
    const size_t kw = side_bytes(cq.kq) * L.kv_rows, vw = side_bytes(cq.vq) * L.kv_rows;
    auto &buf = rows[l];
    buf.resize((size_t)n * (kw + vw));
    uint8_t *kdst = buf.data(), *vdst = buf.data() + (size_t)n * kw;
    for (int part = 0; part < 2; ++part) {
      if (rr.count[part] == 0) continue;
      const uint8_t *ks = reinterpret_cast<const uint8_t *>(s->kc[l]) + (size_t)rr.first[part] * kw;
      const uint8_t *vs = reinterpret_cast<const uint8_t *>(s->vc[l]) + (size_t)rr.first[part] * vw;
      CK(cudaMemcpyAsync(kdst, ks, (size_t)rr.count[part] * kw, cudaMemcpyDeviceToHost, s->st));
      CK(cudaMemcpyAsync(vdst, vs, (size_t)rr.count[part] * vw, cudaMemcpyDeviceToHost, s->st));
      kdst += (size_t)rr.count[part] * kw;
      vdst += (size_t)rr.count[part] * vw;
    }
  }
  std::vector<float> peak(2 * (size_t)m->layers);
  CK(cudaMemcpyAsync(peak.data(), s->d_peak, sizeof(float) * peak.size(), cudaMemcpyDeviceToHost, s->st));
  CK(cudaStreamSynchronize(s->st));

  FileCloser fc{fopen(path, "wb")};
  if (!fc.f) return IGC_FAIL_MISSING;
  uint64_t head[7] = {keep_mark(s), stamp, (uint64_t)s->fill, (uint64_t)s->echo.size(), (uint64_t)m->layers,
                      (uint64_t)(int64_t)m->cache_bits, (uint64_t)kind};
  const uint64_t runs = note ? (uint64_t)note->run_count : 0;
  bool ok = fwrite(k_keep_text, 1, 16, fc.f) == 16 && fwrite(head, 8, 7, fc.f) == 7 && fwrite(&runs, 8, 1, fc.f) == 1;
  for (int i = 0; ok && i < (int)runs; ++i) {
    const uint64_t run[3] = {(uint64_t)(uint32_t)note->from_list[i], (uint64_t)(uint32_t)note->till_list[i],
                             note->mark_list[i]};
    ok = fwrite(run, 8, 3, fc.f) == 3;
  }
  if (ok && !s->echo.empty()) ok = fwrite(s->echo.data(), 4, s->echo.size(), fc.f) == s->echo.size();
  for (int l = 0; ok && l < m->layers; ++l)
    if (!rows[l].empty()) ok = fwrite(rows[l].data(), 1, rows[l].size(), fc.f) == rows[l].size();
  std::vector<float> side((size_t)m->layers);
  for (int v = 0; ok && v < 2; ++v) {
    for (int l = 0; l < m->layers; ++l) side[l] = peak[2 * (size_t)l + v];
    ok = fwrite(side.data(), 4, side.size(), fc.f) == side.size();
  }
  FILE *f = fc.f;
  fc.f = nullptr;
  if (fclose(f) != 0) ok = false;
  return ok ? IGC_OKAY : IGC_FAIL_FORMAT;
}

extern "C" int igc_session_load(igc_session *s, const char *path, uint64_t *stamp_out, igc_keep_note *note_out,
                                int *kind_out) { /* app_core.c:14076 */
  if (!s || !path) return IGC_FAIL_ARGUMENT;
  if (s->guess_count > 0) return IGC_FAIL_STATE;
  if (stamp_out) *stamp_out = 0;
  if (kind_out) *kind_out = IGC_KEEP_PROMPT;
  if (note_out) memset(note_out, 0, sizeof(*note_out));
  igc_model *m = s->m;
  FileCloser fc{fopen(path, "rb")};
  if (!fc.f) return IGC_FAIL_MISSING;
  char text[16];
  uint64_t head[7], runs = 0;
  if (fread(text, 1, 16, fc.f) != 16 || memcmp(text, k_keep_text, 16) != 0 || fread(head, 8, 7, fc.f) != 7 ||
      fread(&runs, 8, 1, fc.f) != 1)
    return IGC_FAIL_FORMAT;
  if (runs > (uint64_t)IGC_KEEP_RUNS) return IGC_FAIL_FORMAT;
  igc_keep_note note;
  memset(&note, 0, sizeof(note));
  note.run_count = (int)runs;
  for (int i = 0; i < note.run_count; ++i) {
    uint64_t run[3];
    if (fread(run, 8, 3, fc.f) != 3) return IGC_FAIL_FORMAT;
    note.from_list[i] = (int32_t)(uint32_t)run[0];
    note.till_list[i] = (int32_t)(uint32_t)run[1];
    note.mark_list[i] = run[2];
  }
  if (!note_sane(&note, m->window_limit)) return IGC_FAIL_FORMAT;
  if (head[6] != IGC_KEEP_PROMPT && head[6] != IGC_KEEP_TALK) return IGC_FAIL_FORMAT;
  // a cache belongs to the shapes it was written from (app_core.c:14127-14134)
  if (head[0] != keep_mark(s) || head[4] != (uint64_t)m->layers || head[5] != (uint64_t)(int64_t)m->cache_bits)
    return IGC_FAIL_STATE;
  const int64_t fill = (int64_t)head[2], held = (int64_t)head[3];
  if (fill < 0 || fill > m->window_limit || held < 0 || held > m->window_limit) return IGC_FAIL_FORMAT;

  // whatever is read replaces what the session held; a read that stops half
  // way leaves it cleared
  igc_session_reset(s);
  clear_stale("session load");
  CK(cudaSetDevice(m->device));
  std::vector<int32_t> ids((size_t)held);
  bool ok = held == 0 || fread(ids.data(), 4, (size_t)held, fc.f) == (size_t)held;
  std::vector<uint8_t> buf;
  int floor = 0;
  for (int l = 0; ok && l < m->layers; ++l) {
    const DevLayer &L = m->layer[l];
    if (L.share) continue;
    const int n = (int)std::min<int64_t>(fill, L.span);
    if (n < 1) continue;
    const CacheStore cq = layer_store(m, l, nullptr);
    const size_t kw = side_bytes(cq.kq) * L.kv_rows, vw = side_bytes(cq.vq) * L.kv_rows;
    buf.resize((size_t)n * (kw + vw));
    if (fread(buf.data(), 1, buf.size(), fc.f) != buf.size()) {
      ok = false;
      break;
    }
    const RingRuns rr = ring_runs((int)fill, L.span);
    const uint8_t *ksrc = buf.data(), *vsrc = buf.data() + (size_t)n * kw;
    for (int part = 0; part < 2; ++part) {
      if (rr.count[part] == 0) continue;
      uint8_t *kd = reinterpret_cast<uint8_t *>(s->kc[l]) + (size_t)rr.first[part] * kw;
      uint8_t *vd = reinterpret_cast<uint8_t *>(s->vc[l]) + (size_t)rr.first[part] * vw;
      CK(cudaMemcpyAsync(kd, ksrc, (size_t)rr.count[part] * kw, cudaMemcpyHostToDevice, s->st));
      CK(cudaMemcpyAsync(vd, vsrc, (size_t)rr.count[part] * vw, cudaMemcpyHostToDevice, s->st));
      ksrc += (size_t)rr.count[part] * kw;
      vsrc += (size_t)rr.count[part] * vw;
    }
    // the pageable copies return once the source is consumed, so the buffer may be reused
    if (fill > L.span) floor = std::max(floor, (int)fill - L.span);
  }
  std::vector<float> kpk((size_t)m->layers), vpk((size_t)m->layers);
  if (ok)
    ok = fread(kpk.data(), 4, kpk.size(), fc.f) == kpk.size() && fread(vpk.data(), 4, vpk.size(), fc.f) == vpk.size();
  if (!ok) {
    igc_session_reset(s);
    return IGC_FAIL_FORMAT;
  }
  std::vector<float> peak(2 * (size_t)m->layers);
  for (int l = 0; l < m->layers; ++l) {
    peak[2 * (size_t)l] = kpk[l];
    peak[2 * (size_t)l + 1] = vpk[l];
  }
  CK(cudaMemcpyAsync(s->d_peak, peak.data(), sizeof(float) * peak.size(), cudaMemcpyHostToDevice, s->st));
  CK(cudaStreamSynchronize(s->st));
  s->fill = (int)fill;
  s->floor = floor;
  s->echo.assign(ids.begin(), ids.end());
  s->logit_lanes = 0;
  if (stamp_out) *stamp_out = head[1];
  if (note_out) *note_out = note;
  if (kind_out) *kind_out = (int)head[6];
  return IGC_OKAY;
}

// ---------------------------------------------------------------------------
// the crowd: one verify round for many sessions in one pass (no counterpart
// in the reference, which runs one session at a time, app_core.c:7789-7793)
//
// Every session of a crowd round shares the model; each brings a block of k
// ids at its own position and its own caches.  The block's lanes of all
// sessions go through one weight sweep per projection (the tcgen05 lane
// GEMM), attention runs once per layer for all sessions (blockIdx.z the
// session, its caches and position from device tables), and the head ends
// in each lane's argmax.  Each session then keeps its leading matches, as
// igc_session_round does for one.  The K slices of every product are fixed
// by the crowd's capacity, so a session's results do not depend on how many
// sessions share its round.

// Attention blocks a cluster in a crowd round: with many sessions in one
// launch, clusters of 8 take half the blocks (and waves) clusters of 16 do.

struct igc_crowd {
  igc_model *m = nullptr;
  cudaStream_t st = nullptr;
  int cap = 0, k = 0, lanes = 0;
  int cluster = 0;  // attention blocks a cluster (0: attn_cluster_for)
  LaneBuf B;
  // device: [ids: lanes][pos: cap] then per layer and session [caches: key, value][peaks][the float rows
  // attention reads: key, value], mirrored in pinned host memory
  uint8_t *d_tab = nullptr, *h_tab = nullptr;
  size_t tab_bytes = 0;
  int32_t *d_top = nullptr;  // [lanes] argmax, then the kernels' error word
  int32_t *h_top = nullptr;
  float *logits = nullptr;   // [lanes][vocab], allocated on the first round that asks for rows
  std::map<std::pair<int, int>, cudaGraphExec_t> graph;  // (sessions, rows wanted)
  std::map<std::pair<int, int>, long> launches;
  std::vector<void *> owned;

  int32_t *ids() { return reinterpret_cast<int32_t *>(d_tab); }
  int *pos() { return reinterpret_cast<int *>(d_tab + sizeof(int32_t) * lanes); }
  // the pointer tables start on a 16-byte boundary whatever the lane and
  // session counts (a pointer load from a 4-byte boundary is misaligned)
  size_t ptr_at() const { return (sizeof(int32_t) * lanes + sizeof(int) * cap + 15) / 16 * 16; }
  float **kc() { return reinterpret_cast<float **>(d_tab + ptr_at()); }
  float **vc() { return kc() + (size_t)m->layers * cap; }
  float **pk() { return vc() + (size_t)m->layers * cap; }
  float **kf() { return pk() + (size_t)m->layers * cap; }
  float **vf() { return kf() + (size_t)m->layers * cap; }

  ~igc_crowd() {
    cudaSetDevice(m->device);
    for (auto &kv : graph) cudaGraphExecDestroy(kv.second);
    for (void *p : owned) cudaFree(p);
    if (h_tab) cudaFreeHost(h_tab);
    if (h_top) cudaFreeHost(h_top);
    if (st) cudaStreamDestroy(st);
    clear_stale("crowd close");
  }
};

extern "C" int igc_crowd_open(igc_model *m, int session_limit, int lanes_per_session, igc_crowd **out) {
  if (!m || !out || session_limit < 1 || lanes_per_session < 1 || lanes_per_session > IGC_LANE_LIMIT)
    return IGC_FAIL_ARGUMENT;
  if (session_limit * lanes_per_session > IGC_CROWD_LANE_LIMIT) return IGC_FAIL_ARGUMENT;
  *out = nullptr;
  clear_stale("crowd open");
  CK(cudaSetDevice(m->device));
  auto cr = std::make_unique<igc_crowd>();
  cr->m = m;
  cr->cap = session_limit;
  cr->k = lanes_per_session;
  cr->cluster = cluster_env("IGC_CROWD_CLUSTER", 0);
  cr->lanes = session_limit * lanes_per_session;
  CK(cudaStreamCreateWithFlags(&cr->st, cudaStreamNonBlocking));
  int c = lane_buf_alloc(m, cr->B, cr->lanes, cr->lanes, cr->owned);
  if (c != IGC_OKAY) return c;
  cr->tab_bytes = cr->ptr_at() + 5 * sizeof(float *) * m->layers * cr->cap;
  void *v = nullptr;
  CK(cudaMalloc(&v, cr->tab_bytes));
  cr->owned.push_back(v);
  cr->d_tab = (uint8_t *)v;
  CK(cudaMalloc(&v, sizeof(int32_t) * (cr->lanes + 1)));
  cr->owned.push_back(v);
  cr->d_top = (int32_t *)v;
  CK(cudaMemset(cr->d_top, 0, sizeof(int32_t) * (cr->lanes + 1)));
  CK(cudaMallocHost(&v, cr->tab_bytes));
  cr->h_tab = (uint8_t *)v;
  CK(cudaMallocHost(&v, sizeof(int32_t) * (cr->lanes + 1)));
  cr->h_top = (int32_t *)v;
  *out = cr.release();
  return IGC_OKAY;
}

extern "C" void igc_crowd_close(igc_crowd *cr) { delete cr; }

static int enqueue_crowd(igc_crowd *cr, int S, bool rows) {
  igc_model *m = cr->m;
  // kernels overlap the one ahead (each waits before reading its results;
  // attention copies only rows written by earlier rounds before its wait)
  PdlScope pdl(true);
  const int k = cr->k;
  LaneRun r{m, cr->st, &cr->B, cr->d_top + cr->lanes, S * k};
  auto attend = [&](int l, const DevLayer &L) -> int {
    const int owner = L.share ? L.source : l;
    const DevLayer &O = m->layer[owner];
    const int sliding = L.kind == 0 ? 1 : 0;
    const size_t at = (size_t)l * cr->cap;
    const int cx = cr->cluster ? cr->cluster
                               : attn_cluster_for((long)S * O.kv_heads * ((k * (m->heads / O.kv_heads) + 15) / 16),
                                                  m->sm_count * (attn_light() ? 2 : 1));
    if (!layer_split(m, l)) {
      const CacheStore cq = layer_store(m, owner, nullptr, L.share ? nullptr : cr->pk() + at);
      CKL(igc_launch_attn_many(cr->B.qkv, L.qkv_rows, m->heads, O.kv_heads, L.hd, L.q_norm, L.k_norm,
                               m->rope_cs[L.kind], m->rope_sn[L.kind], m->eps, L.share ? 0 : 1, nullptr, nullptr,
                               sliding, m->slide_span, cr->pos(), k, cx, cr->B.attn, L.q_rows, nullptr,
                               nullptr, cr->kc() + at, cr->vc() + at, cr->pos(), S, &cq, cr->st, attn_light()));
      return IGC_OKAY;
    }
    // every session's new rows written first (onto the grid on a byte
    // side), a byte side's rows each reads decoded to floats, then attention
    // over those without overlap (it copies rows before its wait)
    const CacheStore cq = layer_store(m, owner, nullptr);
    igc_kernels_pdl(0);
    if (!L.share)
      CKL(igc_launch_lane_kv_many(cr->B.qkv, L.qkv_rows, m->heads, O.kv_heads, L.hd, L.k_norm, m->rope_cs[L.kind],
                                  m->rope_sn[L.kind], m->eps, nullptr, S * k, nullptr, nullptr, &cq, cr->pos(),
                                  cr->kc() + at, cr->vc() + at, cr->pk() + at, k, cr->st));
    if (!layer_bytes(m, owner)) {
      CKL(igc_launch_attn_many(cr->B.qkv, L.qkv_rows, m->heads, O.kv_heads, L.hd, L.q_norm, L.k_norm,
                               m->rope_cs[L.kind], m->rope_sn[L.kind], m->eps, 0, nullptr, nullptr, sliding,
                               m->slide_span, cr->pos(), k, cx, cr->B.attn, L.q_rows, nullptr, nullptr,
                               cr->kc() + at, cr->vc() + at, cr->pos(), S, nullptr, cr->st, attn_light()));
      igc_kernels_pdl(1);
      return IGC_OKAY;
    }
    WidenArgs w;
    memset(&w, 0, sizeof(w));
    w.kc_tab = cr->kc() + at;
    w.vc_tab = cr->vc() + at;
    w.kf_tab = cr->kf() + at;
    w.vf_tab = cr->vf() + at;
    w.pos_tab = cr->pos();
    w.kq = cq.kq;
    w.vq = cq.vq;
    w.kv_w = O.kv_rows;
    w.lanes = k;
    w.sliding = sliding;
    w.span = m->slide_span;
    CKL(igc_launch_lane_widen(&w, S, widen_rows_most(m, sliding, k), m->sm_count, cr->st));
    CKL(igc_launch_attn_many(cr->B.qkv, L.qkv_rows, m->heads, O.kv_heads, L.hd, L.q_norm, L.k_norm, m->rope_cs[L.kind],
                             m->rope_sn[L.kind], m->eps, 0, nullptr, nullptr, sliding, m->slide_span, cr->pos(), k,
                             cx, cr->B.attn, L.q_rows, nullptr, nullptr, cr->kf() + at, cr->vf() + at,
                             cr->pos(), S, nullptr, cr->st, attn_light()));
    igc_kernels_pdl(1);
    return IGC_OKAY;
  };
  return lane_stack(r, cr->ids(), attend, cr->d_top, rows ? cr->logits : nullptr);
}

extern "C" int igc_crowd_round(igc_crowd *cr, igc_session **sessions, int count, const int32_t *ids,
                               int32_t *take_out, int32_t *made_out, float *logits_out) {
  if (!cr || !sessions || !ids || count < 1 || count > cr->cap) return IGC_FAIL_ARGUMENT;
  igc_model *m = cr->m;
  const int k = cr->k;
  for (int j = 0; j < count; ++j) {
    igc_session *s = sessions[j];
    if (!s || s->m != m) return IGC_FAIL_ARGUMENT;
    if (s->guess_count > 0) return IGC_FAIL_STATE;
    if (s->fill + k > m->window_limit) return IGC_FAIL_STATE;
    for (int q = 0; q < j; ++q)
      if (sessions[q] == s) return IGC_FAIL_ARGUMENT;  // a session once a round
  }
  for (int i = 0; i < count * k; ++i)
    if (ids[i] < 0 || ids[i] >= m->vocab) return IGC_FAIL_ARGUMENT;
  clear_stale("crowd round");
  CK(cudaSetDevice(m->device));
  if (logits_out && !cr->logits) {
    void *v = nullptr;
    CK(cudaMalloc(&v, sizeof(float) * (size_t)cr->lanes * m->vocab));
    cr->owned.push_back(v);
    cr->logits = (float *)v;
  }
  // the tables: ids, positions and every layer's (owner's) caches per session
  int32_t *h_ids = reinterpret_cast<int32_t *>(cr->h_tab);
  int *h_pos = reinterpret_cast<int *>(cr->h_tab + sizeof(int32_t) * cr->lanes);
  float **h_kc = reinterpret_cast<float **>(cr->h_tab + cr->ptr_at());
  float **h_vc = h_kc + (size_t)m->layers * cr->cap;
  float **h_pk = h_vc + (size_t)m->layers * cr->cap;
  float **h_kf = h_pk + (size_t)m->layers * cr->cap;
  float **h_vf = h_kf + (size_t)m->layers * cr->cap;
  memcpy(h_ids, ids, sizeof(int32_t) * (size_t)count * k);
  for (int j = 0; j < count; ++j) {
    h_pos[j] = sessions[j]->fill;
    for (int l = 0; l < m->layers; ++l) {
      const DevLayer &L = m->layer[l];
      const int owner = L.share ? L.source : l;
      h_kc[(size_t)l * cr->cap + j] = sessions[j]->kc[owner];
      h_vc[(size_t)l * cr->cap + j] = sessions[j]->vc[owner];
      h_pk[(size_t)l * cr->cap + j] = sessions[j]->d_peak + 2 * l;
      h_kf[(size_t)l * cr->cap + j] = attn_rows(sessions[j], owner, 0);
      h_vf[(size_t)l * cr->cap + j] = attn_rows(sessions[j], owner, 1);
    }
  }
  CK(cudaMemcpyAsync(cr->d_tab, cr->h_tab, cr->tab_bytes, cudaMemcpyHostToDevice, cr->st));
  const bool rows = logits_out != nullptr;
  const auto key = std::make_pair(count, rows ? 1 : 0);
  auto it = cr->graph.find(key);
  if (it == cr->graph.end()) {
    cudaGraph_t g;
    long before = g_launches;
    CK(cudaStreamBeginCapture(cr->st, cudaStreamCaptureModeThreadLocal));
    int c = enqueue_crowd(cr, count, rows);
    cudaError_t e = cudaStreamEndCapture(cr->st, &g);
    if (c != IGC_OKAY) return c;
    if (e != cudaSuccess) return fail_device(e, "capture");
    cudaGraphExec_t ex;
    e = cudaGraphInstantiate(&ex, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return fail_device(e, "graph instantiate");
    it = cr->graph.emplace(key, ex).first;
    cr->launches[key] = g_launches - before;
    g_launches = before;
  }
  CK(cudaGraphLaunch(it->second, cr->st));
  g_launches += cr->launches[key];
  CK(cudaMemcpyAsync(cr->h_top, cr->d_top, sizeof(int32_t) * (cr->lanes + 1), cudaMemcpyDeviceToHost, cr->st));
  if (rows)
    CK(cudaMemcpyAsync(logits_out, cr->logits, sizeof(float) * (size_t)count * k * m->vocab, cudaMemcpyDeviceToHost,
                       cr->st));
  CK(cudaStreamSynchronize(cr->st));
  if (cr->h_top[cr->lanes]) {
    cr->h_top[cr->lanes] = 0;
    cudaMemsetAsync(cr->d_top + cr->lanes, 0, sizeof(int32_t), cr->st);
    cudaStreamSynchronize(cr->st);
    g_last_error = "a kernel gave up waiting for its copies";
    return IGC_FAIL_DEVICE;
  }
  // greedy verify and keep, per session (igc_session_round's rule)
  int total = 0;
  for (int j = 0; j < count; ++j) {
    igc_session *s = sessions[j];
    const int32_t *blk = ids + (size_t)j * k, *top = cr->h_top + (size_t)j * k;
    int take = 0;
    while (take + 1 < k && top[take] == blk[take + 1]) ++take;
    if (take_out) take_out[j] = take;
    if (made_out) made_out[j] = top[take];
    s->fill += take + 1;
    s->serve_tokens += (size_t)(take + 1);
    for (int i = 0; i <= take && (int)s->echo.size() < m->window_limit; ++i) s->echo.push_back(blk[i]);
    s->logit_lanes = 0;
    total += take + 1;
  }
  return total;
}

// ---------------------------------------------------------------------------
// the sampler (app_core.c:14572 pick_shape, :14653 pick_draw, :14706
// guess_draw_state, :14762 session_guess_taste).  The top candidates are
// selected on the GPU; the shaping of at most top_count values, the draws and
// the rejection rule are the reference's arithmetic on the host.

struct Slot {
  float w;
  int32_t id;
};

static uint64_t draw_next(uint64_t *st) {
  uint64_t v = *st;
  v ^= v << 13;
  v ^= v >> 7;
  v ^= v << 17;
  *st = v;
  return v;
}
static float draw_unit(uint64_t *st) { return (float)((draw_next(st) >> 40) / 16777216.0); }

static uint64_t guess_draw_state(uint64_t seed, uint64_t place, uint64_t part) {
  uint64_t st = seed ^ (place * 0xD1342543DE82EF95ull) ^ part;
  st ^= st >> 30;
  st *= 0xBF58476D1CE4E5B9ull;
  st ^= st >> 27;
  st *= 0x94D049BB133111EBull;
  st ^= st >> 31;
  return st ? st : 0x2545F4914F6CDD1Dull;
}

// Top candidates of `lanes` rows of the logits, echo penalty applied per lane
// over ids [from_j, upto_j) of the session's history.  Fills out[j] with the
// kept candidates in descending order.
static int device_top(igc_session *s, int lanes, int keep, const igc_taste *t, const int *echo_from,
                      const int *echo_upto, std::vector<std::vector<Slot>> &out) {
  igc_model *m = s->m;
  const int32_t *d_echo = nullptr;
  const int *d_from = nullptr, *d_upto = nullptr;
  if (t->echo_penalty != 1.0f && t->echo_window > 0 && !s->echo.empty()) {
    CK(cudaMemcpyAsync(s->d_echo, s->echo.data(), sizeof(int32_t) * s->echo.size(), cudaMemcpyHostToDevice, s->st));
    std::vector<int> rng((size_t)2 * lanes);
    for (int j = 0; j < lanes; ++j) {
      rng[j] = echo_from[j];
      rng[lanes + j] = echo_upto[j];
    }
    CK(cudaMemcpyAsync(s->d_echo_range, rng.data(), sizeof(int) * rng.size(), cudaMemcpyHostToDevice, s->st));
    CK(cudaStreamSynchronize(s->st));
    d_echo = s->d_echo;
    d_from = s->d_echo_range;
    d_upto = s->d_echo_range + lanes;
  }
  CKL(igc_launch_topk(s->logits, m->vocab, lanes, keep, d_echo, d_from, d_upto, t->echo_penalty, s->cand_v,
                      s->cand_i, s->top_v, s->top_i, s->st));
  ++g_launches;
  CK(cudaMemcpyAsync(s->h_top_v, s->top_v, sizeof(float) * (size_t)lanes * keep, cudaMemcpyDeviceToHost, s->st));
  CK(cudaMemcpyAsync(s->h_top_i, s->top_i, sizeof(int) * (size_t)lanes * keep, cudaMemcpyDeviceToHost, s->st));
  CK(cudaStreamSynchronize(s->st));
  out.assign((size_t)lanes, {});
  for (int j = 0; j < lanes; ++j) {
    out[j].resize((size_t)keep);
    for (int i = 0; i < keep; ++i) out[j][i] = Slot{s->h_top_v[j * keep + i], s->h_top_i[j * keep + i]};
  }
  return IGC_OKAY;
}

// pick_shape after the selection: softmax at the heat, top-p cut, renorm.
static int shape_slots(std::vector<Slot> &sl, const igc_taste *t) {
  int keep = (int)sl.size();
  float total = 0.0f;
  float peak = sl[0].w;
  for (int i = 0; i < keep; ++i) {
    sl[i].w = expf((sl[i].w - peak) / t->heat_value);
    total += sl[i].w;
  }
  if (total <= 0.0f) {
    sl[0].w = 1.0f;
    return 1;
  }
  for (int i = 0; i < keep; ++i) sl[i].w /= total;
  if (t->top_portion > 0.0f && t->top_portion < 1.0f) {
    float run = 0.0f;
    for (int i = 0; i < keep; ++i) {
      run += sl[i].w;
      if (run >= t->top_portion) {
        keep = i + 1;
        break;
      }
    }
    total = 0.0f;
    for (int i = 0; i < keep; ++i) total += sl[i].w;
    for (int i = 0; i < keep; ++i) sl[i].w /= total;
  }
  return keep;
}

static int32_t pick_draw(const std::vector<Slot> &sl, int keep, float u) {
  for (int i = 0; i < keep; ++i) {
    u -= sl[i].w;
    if (u <= 0.0f) return sl[i].id;
  }
  return sl[keep - 1].id;
}

static int taste_keep(const igc_model *m, const igc_taste *t) {
  return t->top_count > 0 && t->top_count < m->vocab ? t->top_count : m->vocab;
}

// Candidate rows for the sampler: the device selection where top-k bounds the
// set (at most 256), the whole row otherwise.
static int shaped_rows(igc_session *s, int lanes, const igc_taste *t, const int *from, const int *upto,
                       std::vector<std::vector<Slot>> &rows) {
  int keep = taste_keep(s->m, t);
  if (keep <= 256) return device_top(s, lanes, keep, t, from, upto, rows);
  std::vector<float> all((size_t)lanes * s->m->vocab);
  CK(cudaMemcpy(all.data(), s->logits, sizeof(float) * all.size(), cudaMemcpyDeviceToHost));
  rows.assign((size_t)lanes, {});
  for (int j = 0; j < lanes; ++j) {
    std::vector<Slot> &sl = rows[j];
    sl.resize((size_t)s->m->vocab);
    for (int i = 0; i < s->m->vocab; ++i) sl[i] = Slot{all[(size_t)j * s->m->vocab + i], i};
    if (t->echo_penalty != 1.0f && t->echo_window > 0)
      for (int e = from[j]; e < upto[j]; ++e) {
        int32_t id = s->echo[e];
        if (id < 0 || id >= s->m->vocab) continue;
        sl[id].w = sl[id].w > 0.0f ? sl[id].w / t->echo_penalty : sl[id].w * t->echo_penalty;
      }
    std::stable_sort(sl.begin(), sl.end(), [](const Slot &a, const Slot &b) { return a.w > b.w; });
    sl.resize((size_t)keep);
  }
  return IGC_OKAY;
}

extern "C" int32_t igc_session_pick(igc_session *s, const igc_taste *t) { /* app_core.c:14810 */
  if (!s || !t || s->logit_lanes < 1) return -1;
  if (t->seed_value) s->draw_state = t->seed_value ^ (uint64_t)s->fill;
  int last = s->logit_lanes - 1;
  if (t->heat_value <= 0.0f) return s->h_top[last];
  int n = (int)s->echo.size();
  int from = n - t->echo_window > 0 ? n - t->echo_window : 0;
  std::vector<std::vector<Slot>> rows;
  // the step's row is the last lane of the last pass; shaping it alone
  if (last != 0) return -1;
  if (shaped_rows(s, 1, t, &from, &n, rows) != IGC_OKAY) return -1;
  int keep = shape_slots(rows[0], t);
  return pick_draw(rows[0], keep, draw_unit(&s->draw_state));
}

#define DRAW_TAKE 0x9E3779B97F4A7C15ull
#define DRAW_MAKE 0xC2B2AE3D27D4EB4Full

extern "C" int igc_session_guess_taste(igc_session *s, const int32_t *ids, int k, const igc_taste *t,
                                       int32_t *made_out) {
  if (!s || !ids || !made_out || !t) return -1;
  if (k < 1 || s->guess_count != k) return -1;
  if (t->heat_value <= 0.0f) return -1;
  std::vector<int> from((size_t)k), upto((size_t)k);
  for (int j = 0; j < k; ++j) {
    int echo_count = s->guess_echo + j + 1;
    if (echo_count > s->m->window_limit) echo_count = s->m->window_limit;
    upto[j] = echo_count;
    from[j] = echo_count - t->echo_window > 0 ? echo_count - t->echo_window : 0;
  }
  std::vector<std::vector<Slot>> rows;
  if (shaped_rows(s, k, t, from.data(), upto.data(), rows) != IGC_OKAY) return -1;
  int take = 0;
  for (int j = 0; j < k; ++j) {
    std::vector<Slot> &sl = rows[j];
    uint64_t place = (uint64_t)(s->guess_from + j + 1);
    int keep = shape_slots(sl, t);
    if (j + 1 < k) {
      int32_t want = ids[j + 1];
      float share = 0.0f;
      for (int i = 0; i < keep; ++i)
        if (sl[i].id == want) { share = sl[i].w; break; }
      uint64_t st = t->seed_value ? guess_draw_state(t->seed_value, place, DRAW_TAKE) : s->draw_state;
      float u = draw_unit(&st);
      if (!t->seed_value) s->draw_state = st;
      if (u < share) {
        take += 1;
        continue;
      }
      int fill = 0;
      float total = 0.0f;
      for (int i = 0; i < keep; ++i) {
        if (sl[i].id == want) continue;
        sl[fill++] = sl[i];
        total += sl[i].w;
      }
      if (fill < 1 || !(total > 0.0f)) {
        *made_out = want;
        return take;
      }
      for (int i = 0; i < fill; ++i) sl[i].w /= total;
      keep = fill;
    }
    uint64_t st = t->seed_value ? guess_draw_state(t->seed_value, place, DRAW_MAKE) : s->draw_state;
    float u = draw_unit(&st);
    if (!t->seed_value) s->draw_state = st;
    *made_out = pick_draw(sl, keep, u);
    return take;
  }
  return take;
}

// app_main.c:520 main_answer_guess's round body: guess, verify, keep.
extern "C" int igc_session_round(igc_session *s, const int32_t *ids, int k, const igc_taste *t, int32_t *take_out,
                                 int32_t *made_out) {
  if (!s || !ids || k < 1) return IGC_FAIL_ARGUMENT;
  int c = igc_session_guess(s, ids, k, nullptr);
  if (c != IGC_OKAY) return c;
  int take = 0;
  int32_t made = 0;
  if (t && t->heat_value > 0.0f) {
    take = igc_session_guess_taste(s, ids, k, t, &made);
    if (take < 0) {
      igc_session_guess_keep(s, 0);
      return IGC_FAIL_STATE;
    }
  } else {
    while (take + 1 < k && s->h_top[take] == ids[take + 1]) ++take;
    made = s->h_top[take];
  }
  c = igc_session_guess_keep(s, take + 1);
  if (c != IGC_OKAY) return c;
  if (take_out) *take_out = take;
  if (made_out) *made_out = made;
  return take + 1;
}

// ---------------------------------------------------------------------------
// measurement entries (no counterpart in the reference)

// `rounds` verify passes of `k` lanes with every block already in HBM: round
// r runs blocks[r*k .. r*k+k) at the session's fill plus r*k, as a proposer
// that is always right would, and the rounds follow one another on the
// stream with no host round trip.  The span between the first and the last
// pass is timed with CUDA events on the session's stream.  The session ends
// with every round kept; `last_top` gets the last round's argmax ids.
extern "C" int igc_session_bench(igc_session *s, const int32_t *blocks, int rounds, int k, float *device_ms,
                                 int32_t *last_top) {
  if (!s || !blocks || rounds < 1 || k < 1 || k > IGC_LANE_LIMIT) return IGC_FAIL_ARGUMENT;
  if (s->guess_count > 0) return IGC_FAIL_STATE;
  igc_model *m = s->m;
  if (m->plain) return IGC_FAIL_SUPPORT;  // measures the decode GEMV passes
  if (s->fill + rounds * k > m->window_limit) return IGC_FAIL_STATE;
  for (int i = 0; i < rounds * k; ++i)
    if (blocks[i] < 0 || blocks[i] >= m->vocab) return IGC_FAIL_ARGUMENT;
  clear_stale("bench");
  CK(cudaSetDevice(m->device));
  const size_t rec = (size_t)(1 + k);
  if (s->d_rounds_cap < rec * rounds) {
    if (s->d_rounds) cudaFree(s->d_rounds);
    s->d_rounds = nullptr;
    CK(cudaMalloc(&s->d_rounds, sizeof(int32_t) * rec * rounds));
    s->owned.push_back(s->d_rounds);
    s->d_rounds_cap = rec * rounds;
  }
  std::vector<int32_t> host(rec * rounds);
  for (int r = 0; r < rounds; ++r) {
    host[r * rec] = s->fill + r * k;
    memcpy(&host[r * rec + 1], blocks + (size_t)r * k, sizeof(int32_t) * k);
  }
  CK(cudaMemcpy(s->d_rounds, host.data(), sizeof(int32_t) * host.size(), cudaMemcpyHostToDevice));
  // the pass of this shape, captured once
  if (s->use_graphs && !s->graph[k][1]) {
    CK(cudaMemcpyAsync(s->d_io, s->d_rounds, sizeof(int32_t) * rec, cudaMemcpyDeviceToDevice, s->st));
    cudaGraph_t g;
    long before = g_launches;
    CK(cudaStreamBeginCapture(s->st, cudaStreamCaptureModeThreadLocal));
    int c = enqueue_pass(s, k, 1);
    cudaError_t e = cudaStreamEndCapture(s->st, &g);
    if (c != IGC_OKAY) return c;
    if (e != cudaSuccess) return fail_device(e, "capture");
    s->kernels_per_pass[k][1] = g_launches - before;
    g_launches = before;
    e = cudaGraphInstantiate(&s->graph[k][1], g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return fail_device(e, "graph instantiate");
  }
  cudaEvent_t a, b;
  CK(cudaEventCreate(&a));
  CK(cudaEventCreate(&b));
  CK(cudaEventRecord(a, s->st));
  for (int r = 0; r < rounds; ++r) {
    CK(cudaMemcpyAsync(s->d_io, s->d_rounds + (size_t)r * rec, sizeof(int32_t) * rec, cudaMemcpyDeviceToDevice,
                       s->st));
    if (s->use_graphs) {
      CK(cudaGraphLaunch(s->graph[k][1], s->st));
      g_launches += s->kernels_per_pass[k][1];
    } else {
      int c = enqueue_pass(s, k, 1);
      if (c != IGC_OKAY) return c;
    }
  }
  CK(cudaEventRecord(b, s->st));
  CK(cudaMemcpyAsync(s->h_top, s->d_top, sizeof(int32_t) * (IGC_LANE_LIMIT + 1), cudaMemcpyDeviceToHost, s->st));
  CK(cudaStreamSynchronize(s->st));
  if (int ce = check_err(s)) return ce;
  float ms = 0.0f;
  CK(cudaEventElapsedTime(&ms, a, b));
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  if (device_ms) *device_ms = ms;
  if (last_top) memcpy(last_top, s->h_top, sizeof(int32_t) * k);
  s->fill += rounds * k;
  for (int i = 0; i < rounds * k && (int)s->echo.size() < m->window_limit; ++i) s->echo.push_back(blocks[i]);
  s->logit_lanes = k;
  return IGC_OKAY;
}

// One pass of `k` lanes (ids from `ids`, position the session's fill, kept)
// with a CUDA event before every launch: for each launch its class (0 a
// projection, 1 the output head, 2 attention, 3 the rest), the weight bytes
// it streams and its device time in ms.  Returns the launches recorded.
extern "C" int igc_session_profile(igc_session *s, const int32_t *ids, int k, int *cls_out, double *bytes_out,
                                   float *ms_out, int capacity) {
  if (!s || !ids || k < 1 || k > IGC_LANE_LIMIT) return IGC_FAIL_ARGUMENT;
  if (s->guess_count > 0) return IGC_FAIL_STATE;
  igc_model *m = s->m;
  if (m->plain) return IGC_FAIL_SUPPORT;
  if (s->fill + k > m->window_limit) return IGC_FAIL_STATE;
  clear_stale("profile");
  CK(cudaSetDevice(m->device));
  s->h_io[0] = s->fill;
  memcpy(s->h_io + 1, ids, sizeof(int32_t) * (size_t)k);
  CK(cudaMemcpyAsync(s->d_io, s->h_io, sizeof(int32_t) * (size_t)(1 + k), cudaMemcpyHostToDevice, s->st));
  for (auto &mk : s->marks) cudaEventDestroy(mk.ev);
  s->marks.clear();
  s->prof_on = true;
  int c = enqueue_pass(s, k, 1);
  s->prof_on = false;
  if (c != IGC_OKAY) return c;
  CK(cudaMemcpyAsync(s->h_top, s->d_top, sizeof(int32_t) * (IGC_LANE_LIMIT + 1), cudaMemcpyDeviceToHost, s->st));
  CK(cudaStreamSynchronize(s->st));
  if (int ce = check_err(s)) return ce;
  int n = 0;
  for (size_t i = 0; i + 1 < s->marks.size() && n < capacity; ++i, ++n) {
    float ms = 0.0f;
    CK(cudaEventElapsedTime(&ms, s->marks[i].ev, s->marks[i + 1].ev));
    if (cls_out) cls_out[n] = s->marks[i].cls;
    if (bytes_out) bytes_out[n] = s->marks[i].bytes;
    if (ms_out) ms_out[n] = ms;
  }
  s->fill += k;
  for (int j = 0; j < k && (int)s->echo.size() < m->window_limit; ++j) s->echo.push_back(ids[j]);
  s->logit_lanes = k;
  return n;
}

// The launch stamps of the graphed passes with a head: for each stamped
// launch of the `k`-lane pass, its class (as igc_session_profile), the
// weight bytes it streams and the total of its spans, in ns, over every such
// pass since the last reset (each span runs from the first block past its
// wait on the kernel ahead to the last block's end).  With `reset` the totals
// start over after the read.  Returns the launches written.
extern "C" int igc_session_stamps(igc_session *s, int k, int *cls_out, double *bytes_out, double *ns_out,
                                  int capacity, int reset) {
  if (!s || k < 1 || k > IGC_LANE_LIMIT || capacity < 0) return IGC_FAIL_ARGUMENT;
  if (s->m->plain) return IGC_FAIL_SUPPORT;
  clear_stale("stamps");
  CK(cudaSetDevice(s->m->device));
  std::vector<unsigned long long> sum(IGC_STAMP_LIMIT);
  CK(cudaStreamSynchronize(s->st));
  CK(cudaMemcpy(sum.data(), s->d_stamp_sum, sizeof(unsigned long long) * IGC_STAMP_LIMIT, cudaMemcpyDeviceToHost));
  const auto &meta = s->stamp_meta[k];
  int n = 0;
  for (size_t i = 0; i < meta.size() && n < capacity; ++i, ++n) {
    if (cls_out) cls_out[n] = meta[i].cls;
    if (bytes_out) bytes_out[n] = meta[i].bytes;
    if (ns_out) ns_out[n] = (double)sum[i];
  }
  if (reset) {
    CK(cudaMemsetAsync(s->d_stamp_sum, 0, sizeof(unsigned long long) * IGC_STAMP_LIMIT, s->st));
    CK(cudaStreamSynchronize(s->st));
  }
  return n;
}

// ---------------------------------------------------------------------------
// norm_rms with no allocation (no counterpart in the reference)
//
// The desk's norm_rms grows device buffers with cudaMalloc whenever a longer
// vector arrives.  Two kinds of caller cannot allow that.  One is a host token
// loop that promised to allocate nothing once it runs; the reference sizes
// its backend's staging when the table opens for exactly this reason.  The
// other is a caller that holds no desk and would otherwise open one, with
// its buffers, to normalise a single vector.  This entry keeps its three
// vectors (input, gain, output) in one array that is part of the library's
// device image, and calls nothing that allocates.
//
// No word of the array has to start at zero: a call writes every word it
// reads (the input, then the gain when one is given, then the kernel's
// output) before reading it.  All calls on one device share the array, so
// two calls that overlap in time on the same device, from two host threads
// for instance, race: each may read the other's vectors.  Callers serialise
// them.
static __device__ __align__(256) float g_fixed_norm[3 * IGC_FIXED_NORM_LIMIT];  // 768 KiB a device
static float *g_fixed_norm_at[IGC_FIXED_DEVICE_LIMIT];  // its address on each device, found on first use
static std::mutex g_fixed_norm_lock;

static int norm_rms_fixed_on(int device, const float *value_list, const float *gain_list, int value_count,
                             float eps_value, float *value_out) {
  CK(cudaSetDevice(device));
  float *base = nullptr;
  cudaError_t e = cudaSuccess;
  {
    // the address, looked up once per device with that device current
    std::lock_guard<std::mutex> hold(g_fixed_norm_lock);
    base = g_fixed_norm_at[device];
    if (!base) {
      e = cudaGetSymbolAddress((void **)&base, g_fixed_norm);
      if (e == cudaSuccess) g_fixed_norm_at[device] = base;
    }
  }
  if (e != cudaSuccess) return fail_device(e, "cudaGetSymbolAddress(g_fixed_norm)");
  float *d_x = base, *d_w = base + IGC_FIXED_NORM_LIMIT, *d_out = base + 2 * IGC_FIXED_NORM_LIMIT;
  const size_t bytes = sizeof(float) * (size_t)value_count;
  cudaStream_t st = cudaStreamPerThread;
  CK(cudaMemcpyAsync(d_x, value_list, bytes, cudaMemcpyHostToDevice, st));
  if (gain_list) CK(cudaMemcpyAsync(d_w, gain_list, bytes, cudaMemcpyHostToDevice, st));
  CKL(igc_launch_desk_norm(d_x, gain_list ? d_w : nullptr, value_count, eps_value, d_out, st));
  CK(cudaMemcpyAsync(value_out, d_out, bytes, cudaMemcpyDeviceToHost, st));
  CK(cudaStreamSynchronize(st));
  return IGC_OKAY;
}

extern "C" int igc_norm_rms_fixed(int device, const float *value_list, const float *gain_list, int value_count,
                                  float eps_value, float *value_out) {
  if (!value_list || !value_out || value_count < 1 || device < 0 || device >= IGC_FIXED_DEVICE_LIMIT)
    return IGC_FAIL_ARGUMENT;
  if (value_count > IGC_FIXED_NORM_LIMIT) return IGC_FAIL_ARGUMENT;  // longer than the fixed array holds
  clear_stale("norm_rms_fixed");
  int before = -1;
  if (cudaGetDevice(&before) != cudaSuccess) before = -1;
  int c = norm_rms_fixed_on(device, value_list, gain_list, value_count, eps_value, value_out);
  if (before >= 0 && before != device) cudaSetDevice(before);  // the caller's device stays current
  return c;
}
