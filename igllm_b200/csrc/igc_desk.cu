// igc_desk.cu - the device backend table: the six entries of the reference's
// back_desk (app_core.c:5222-5245) with host pointers in and out.
//
// A code plane is uploaded the first time a product names it, keyed by its
// code pointer, and reused afterwards: the "device handle beside each plane"
// the reference's design notes ask for.  Each entry copies its activations
// in, runs the same kernel the session pass runs, and copies the result out,
// synchronously, so a reference build can swap its table for this one and
// compare entry by entry.
#include <cuda_runtime.h>

#include <cstring>
#include <unordered_map>
#include <vector>

#include "../../include/igllm_cuda.h"
#include "igc_kernels.h"
#include "igc_lanes.h"

using namespace igc;

namespace {

struct DeskPlane {
  CUtensorMap tm_codes, tm_scales;  // the lane GEMM's tensor maps (igc_lane_tmaps)
  bool tm_ok = false;
  uint4 *tiles = nullptr;
  uint2 *scales = nullptr;
  int n_rb = 0, n_cc = 0, rows = 0, cols = 0, split = 1, grid = 1;
  // a plane the tiles do not hold (8-bit codes, a dense plane, scales f16
  // cannot hold): kept as stored for the CUDA-core product (`plain.codes` or
  // `plain.dense` set), its device copies freed with the desk
  bool is_plain = false;
  PlainArgs plain = {};
  void *plain_data = nullptr, *plain_scales = nullptr;
};

struct DeskState {
  int device = 0;
  int sm_count = 148;
  int smem_limit = 200 * 1024;
  int status = IGC_OKAY;
  cudaStream_t st = nullptr;
  std::unordered_map<const void *, DeskPlane> planes;
  float *buf_a = nullptr, *buf_b = nullptr, *buf_c = nullptr;
  size_t buf_floats = 0;
  float *arg_val = nullptr;
  int *arg_idx = nullptr;
  int *err = nullptr;  // set by a projection that gave up waiting for its weights
  // the batched-lane path (igc_lanes.cu): activations, staged operand
  // blocks, per-lane factors, K-slice partials and the summed product
  float *lane_act = nullptr, *lane_factor = nullptr, *lane_part = nullptr, *lane_out = nullptr;
  void *lane_tiles = nullptr;
  size_t lane_act_n = 0, lane_factor_n = 0, lane_part_n = 0, lane_out_n = 0, lane_tiles_n = 0;
};

DeskState *state_of(igc_desk *d) {
  cudaGetLastError();  // an unchecked failure elsewhere must not be charged to this entry
  return static_cast<DeskState *>(d->state);
}

bool note(DeskState *s, int code) {
  if (code != IGC_OKAY && s->status == IGC_OKAY) s->status = code;
  return code == IGC_OKAY;
}

bool ok(DeskState *s, cudaError_t e) { return note(s, e == cudaSuccess ? IGC_OKAY : IGC_FAIL_DEVICE); }

bool grow(DeskState *s, size_t floats) {
  if (floats <= s->buf_floats) return true;
  cudaFree(s->buf_a);
  cudaFree(s->buf_b);
  cudaFree(s->buf_c);
  s->buf_a = s->buf_b = s->buf_c = nullptr;
  if (!ok(s, cudaMalloc(&s->buf_a, floats * 4)) || !ok(s, cudaMalloc(&s->buf_b, floats * 4)) ||
      !ok(s, cudaMalloc(&s->buf_c, floats * 4)))
    return false;
  s->buf_floats = floats;
  return true;
}

// A plane the tiles do not hold, kept as stored for the CUDA-core product:
// offset codes of 1-8 bits (signed bytes through their flip) with scales of
// any float type widened to f32, or a dense F32/F16/BF16 plane
// (app_core.c:1775-1797).  Zero points are refused.  The reference applies a
// plane's activation grids itself around the table's product
// (app_core.c:7814 plane_lift_many), so the product here takes none.
const DeskPlane *plain_plane_of(DeskState *s, const igc_plane *p, const void *key) {
  DeskPlane dp;
  dp.is_plain = true;
  dp.rows = p->row_count;
  dp.cols = p->col_count;
  PlainArgs &a = dp.plain;
  memset(&a, 0, sizeof(a));
  a.rows = p->row_count;
  a.cols = p->col_count;
  a.pair_half = -1;
  a.out_scale = 1.0f;
  auto type_bytes = [](int t) -> size_t { return t == 1 ? 4u : (t == 2 || t == 3) ? 2u : 0u; };
  if (p->form == 1) {
    const size_t tb = type_bytes(p->real_type);
    if (!tb || !p->real_data) return void(note(s, IGC_FAIL_SUPPORT)), nullptr;
    const size_t bytes = (size_t)p->row_count * p->col_count * tb;
    if (!ok(s, cudaMalloc(&dp.plain_data, bytes)) ||
        !ok(s, cudaMemcpy(dp.plain_data, p->real_data, bytes, cudaMemcpyHostToDevice)))
      return nullptr;
    a.dense = dp.plain_data;
    a.dense_type = p->real_type;
  } else {
    const int bits = p->bit_count;
    const size_t gb = type_bytes(p->gain_type);
    if (p->form != 2 || bits < 1 || bits > 8 || p->code_bias != (1 << (bits - 1)) ||
        (p->code_flip != 0 && p->code_flip != p->code_bias) || p->bias_data || !gb || p->group_count < 1 ||
        p->group_size < 1 || (size_t)p->group_count * p->group_size < (size_t)p->col_count)
      return void(note(s, IGC_FAIL_SUPPORT)), nullptr;
    std::vector<float> sc((size_t)p->row_count * p->group_count);
    for (size_t i = 0; i < sc.size(); ++i) {
      const uint8_t *g = static_cast<const uint8_t *>(p->gain_data) + i * gb;
      if (p->gain_type == 1) {
        memcpy(&sc[i], g, 4);
      } else {
        uint16_t h;
        memcpy(&h, g, 2);
        if (p->gain_type == 2) {
          __half hh;
          memcpy(&hh, &h, 2);
          sc[i] = __half2float(hh);
        } else {
          const uint32_t u = (uint32_t)h << 16;
          memcpy(&sc[i], &u, 4);
        }
      }
    }
    const size_t cb = (size_t)p->row_count * p->row_stride;
    if (!ok(s, cudaMalloc(&dp.plain_data, cb)) || !ok(s, cudaMalloc(&dp.plain_scales, sizeof(float) * sc.size())) ||
        !ok(s, cudaMemcpy(dp.plain_data, p->code_data, cb, cudaMemcpyHostToDevice)) ||
        !ok(s, cudaMemcpy(dp.plain_scales, sc.data(), sizeof(float) * sc.size(), cudaMemcpyHostToDevice)))
      return nullptr;
    a.codes = static_cast<const uint8_t *>(dp.plain_data);
    a.stride = p->row_stride;
    a.bits = bits;
    a.flip = (uint32_t)p->code_flip;
    a.bias = p->code_bias;
    a.scales = static_cast<const float *>(dp.plain_scales);
    a.groups = p->group_count;
    a.group_size = p->group_size;
  }
  return &(s->planes[key] = dp);
}

// app_core.c:1775 plane: offset codes of 1, 2 or 4 bits, no flip, no zero
// points, groups a multiple of 32 columns, scales of any float type that f16
// holds exactly go to the tiles; anything else to plain_plane_of.
const DeskPlane *plane_of(DeskState *s, const igc_plane *p) {
  const void *key = p->code_data ? (const void *)p->code_data : p->real_data;
  auto it = s->planes.find(key);
  if (it != s->planes.end()) return &it->second;
  const int bits = p->bit_count;
  if (p->form != 2 || (bits != 1 && bits != 2 && bits != 4) || p->code_flip != 0 || p->bias_data ||
      p->group_size < 32 || p->group_size % 32 || p->group_count * p->group_size < p->col_count ||
      p->code_bias != (1 << (bits - 1)))
    return plain_plane_of(s, p, key);
  const int g32 = (p->col_count + 31) / 32;
  std::vector<uint16_t> sc((size_t)p->row_count * g32);
  if (igc_scales_f16(p->gain_data, p->gain_type, p->row_count, p->group_count, p->group_size, p->col_count,
                     sc.data()) != 0)
    return plain_plane_of(s, p, key);
  DeskPlane dp;
  dp.rows = p->row_count;
  dp.cols = p->col_count;
  dp.n_rb = (p->row_count + 15) / 16;
  dp.n_cc = (p->col_count + 63) / 64;
  size_t cb = (size_t)p->row_count * p->row_stride, sb = sizeof(uint16_t) * sc.size();
  uint8_t *dc = nullptr;
  uint16_t *ds = nullptr;
  if (!ok(s, cudaMalloc(&dp.tiles, (size_t)dp.n_rb * dp.n_cc * 512)) ||
      !ok(s, cudaMalloc(&dp.scales, (size_t)dp.n_rb * dp.n_cc * 64)) || !ok(s, cudaMalloc(&dc, cb)) ||
      !ok(s, cudaMalloc(&ds, sb)))
    return nullptr;
  bool good = ok(s, cudaMemcpy(dc, p->code_data, cb, cudaMemcpyHostToDevice)) &&
              ok(s, cudaMemcpy(ds, sc.data(), sb, cudaMemcpyHostToDevice)) &&
              ok(s, igc_launch_repack(dc, p->row_stride, bits, ds, g32, p->row_count, p->col_count, dp.n_rb,
                                      dp.n_cc, 1, 0, dp.tiles, dp.scales, s->st)) &&
              ok(s, cudaStreamSynchronize(s->st));
  cudaFree(dc);
  cudaFree(ds);
  if (!good) return nullptr;
  int target = s->sm_count * GEMV_WARPS * 2;
  while (dp.split < 8 && dp.split * 2 <= dp.n_cc && dp.n_rb * dp.split < target) dp.split *= 2;
  int per_iter = GEMV_WARPS / dp.split;
  dp.grid = (dp.n_rb + per_iter - 1) / per_iter;
  if (dp.grid > s->sm_count * 4) dp.grid = s->sm_count * 4;
  dp.tm_ok = igc_lane_tmaps(dp.tiles, dp.scales, dp.n_rb, dp.n_cc, &dp.tm_codes, &dp.tm_scales) == 0;
  return &(s->planes[key] = dp);
}

// A device buffer of at least `bytes`, grown (never shrunk) on demand.
template <typename T>
bool room(DeskState *s, T **p, size_t *have, size_t bytes) {
  if (bytes <= *have) return true;
  cudaFree(*p);
  *p = nullptr;
  *have = 0;
  if (!ok(s, cudaMalloc((void **)p, bytes))) return false;
  *have = bytes;
  return true;
}

// Lanes at which a product runs as the tcgen05 GEMM of igc_lanes.cu (the
// reference never passes more than 16; a caller batching many lanes - a
// prefill chunk, or many streams' blocks - does).
constexpr int DESK_LANE_GEMM = 64;

// A plain plane's product, 16 lanes a launch: the activations in, one
// CUDA-core product, the rows out.
void desk_mat_mat_plain(DeskState *s, const DeskPlane *p, const float *act, int act_stride, int lanes, float *out,
                        int out_stride) {
  for (int done = 0; done < lanes;) {
    const int k = lanes - done < IGC_LANE_LIMIT ? lanes - done : IGC_LANE_LIMIT;
    if (!grow(s, (size_t)IGC_LANE_LIMIT * (size_t)(p->cols > p->rows ? p->cols : p->rows))) return;
    for (int j = 0; j < k; ++j)
      if (!ok(s, cudaMemcpyAsync(s->buf_a + (size_t)j * p->cols, act + (size_t)(done + j) * act_stride,
                                 sizeof(float) * p->cols, cudaMemcpyHostToDevice, s->st)))
        return;
    PlainArgs a = p->plain;
    a.x = s->buf_a;
    a.x_stride = p->cols;
    a.lanes = k;
    a.out = s->buf_b;
    a.out_stride = p->rows;
    if (!ok(s, igc_launch_plain_product(&a, s->sm_count, nullptr, s->st))) return;
    for (int j = 0; j < k; ++j)
      if (!ok(s, cudaMemcpyAsync(out + (size_t)(done + j) * out_stride, s->buf_b + (size_t)j * p->rows,
                                 sizeof(float) * p->rows, cudaMemcpyDeviceToHost, s->st)))
        return;
    if (!ok(s, cudaStreamSynchronize(s->st))) return;
    done += k;
  }
}

void desk_mat_mat_lanes(DeskState *s, const DeskPlane *p, const float *act, int act_stride, int lanes, float *out,
                        int out_stride) {
  const int m_tiles = (lanes + LG_M - 1) / LG_M, rows_pad = p->n_rb * 16;
  const int split = igc_lane_gemm_split(lanes, p->n_rb, p->n_cc, s->sm_count);
  if (!room(s, &s->lane_act, &s->lane_act_n, sizeof(float) * (size_t)lanes * p->cols) ||
      !room(s, &s->lane_factor, &s->lane_factor_n, sizeof(float) * (size_t)lanes) ||
      !room(s, &s->lane_tiles, &s->lane_tiles_n, (size_t)m_tiles * p->n_cc * LG_A_STEP_BYTES) ||
      !room(s, &s->lane_part, &s->lane_part_n, sizeof(float) * (size_t)split * lanes * rows_pad) ||
      !room(s, &s->lane_out, &s->lane_out_n, sizeof(float) * (size_t)lanes * p->rows))
    return;
  if (!ok(s, cudaMemcpy2DAsync(s->lane_act, sizeof(float) * p->cols, act, sizeof(float) * act_stride,
                               sizeof(float) * p->cols, lanes, cudaMemcpyHostToDevice, s->st)))
    return;
  LaneStageArgs sa;
  memset(&sa, 0, sizeof(sa));
  sa.mode = LS_PLAIN;
  sa.lanes = lanes;
  sa.cols = p->cols;
  sa.x = s->lane_act;
  sa.x_stride = p->cols;
  sa.gain = 1.0f;
  sa.out_scale = 1.0f;
  sa.a_tiles = s->lane_tiles;
  sa.n_cc = p->n_cc;
  sa.factor = s->lane_factor;
  if (!ok(s, igc_launch_lane_stage(&sa, s->st))) return;
  LaneGemmArgs ga;
  memset(&ga, 0, sizeof(ga));
  ga.tiles = p->tiles;
  ga.scales = p->scales;
  ga.n_rb = p->n_rb;
  ga.n_cc = p->n_cc;
  ga.a_tiles = reinterpret_cast<const uint4 *>(s->lane_tiles);
  ga.factor = s->lane_factor;
  ga.out = s->lane_part;
  ga.lanes = lanes;
  ga.out_stride = rows_pad;
  ga.split = split;
  ga.err = s->err;
  if (!p->tm_ok) return void(note(s, IGC_FAIL_SUPPORT));
  if (!ok(s, igc_launch_lane_gemm(&ga, &p->tm_codes, &p->tm_scales, s->st))) return;
  if (!ok(s, igc_launch_lane_sum(s->lane_part, split, lanes, p->rows, rows_pad, s->lane_out, p->rows, s->st)))
    return;
  if (!ok(s, cudaMemcpy2DAsync(out, sizeof(float) * out_stride, s->lane_out, sizeof(float) * p->rows,
                               sizeof(float) * p->rows, lanes, cudaMemcpyDeviceToHost, s->st)))
    return;
  if (!ok(s, cudaStreamSynchronize(s->st))) return;
  int gave_up = 0;
  if (!ok(s, cudaMemcpy(&gave_up, s->err, sizeof(int), cudaMemcpyDeviceToHost))) return;
  if (gave_up) {
    cudaMemset(s->err, 0, sizeof(int));
    note(s, IGC_FAIL_DEVICE);
  }
}

void desk_mat_mat(igc_desk *d, const igc_plane *sheet, const float *act, int act_stride, int lanes, float *out,
                  int out_stride) {
  DeskState *s = state_of(d);
  if (cudaSetDevice(s->device) != cudaSuccess) return void(note(s, IGC_FAIL_DEVICE));
  const DeskPlane *p = plane_of(s, sheet);
  if (!p) return;
  if (p->is_plain) return desk_mat_mat_plain(s, p, act, act_stride, lanes, out, out_stride);
  if (lanes >= DESK_LANE_GEMM) return desk_mat_mat_lanes(s, p, act, act_stride, lanes, out, out_stride);
  for (int done = 0; done < lanes;) {  // app_core.c:5250: chunks of 16 lanes
    int k = lanes - done < IGC_LANE_LIMIT ? lanes - done : IGC_LANE_LIMIT;
    if (!grow(s, (size_t)IGC_LANE_LIMIT * (size_t)(p->cols > p->rows ? p->cols : p->rows))) return;
    for (int j = 0; j < k; ++j)
      if (!ok(s, cudaMemcpyAsync(s->buf_a + (size_t)j * p->cols, act + (size_t)(done + j) * act_stride,
                                 sizeof(float) * p->cols, cudaMemcpyHostToDevice, s->st)))
        return;
    GemvArgs a;
    memset(&a, 0, sizeof(a));
    a.pl = GemvPlane{p->tiles, p->scales, p->n_rb, p->n_cc, p->rows, p->cols};
    a.lanes = k;
    a.split = p->split;
    a.x = s->buf_a;
    a.x_stride = p->cols;
    a.out = s->buf_b;
    a.out_stride = p->rows;
    a.out_scale = 1.0f;
    a.part_val = s->arg_val;
    a.part_idx = s->arg_idx;
    a.err = s->err;
    if (igc_gemv_smem_min(&a, 0) > (size_t)s->smem_limit) {
      // wide planes stage at most eight lanes at a time
      int k8 = k < 8 ? k : 8;
      for (int j0 = 0; j0 < k; j0 += k8) {
        GemvArgs b = a;
        b.lanes = k - j0 < k8 ? k - j0 : k8;
        b.x = s->buf_a + (size_t)j0 * p->cols;
        b.out = s->buf_b + (size_t)j0 * p->rows;
        if (igc_gemv_smem_min(&b, 0) > (size_t)s->smem_limit) return void(note(s, IGC_FAIL_SUPPORT));
        if (!ok(s, igc_launch_gemv(&b, 0, PRO_F32, EPI_STORE, p->grid, (size_t)s->smem_limit, s->st, nullptr))) return;
      }
    } else if (!ok(s, igc_launch_gemv(&a, 0, PRO_F32, EPI_STORE, p->grid, (size_t)s->smem_limit, s->st, nullptr))) {
      return;
    }
    for (int j = 0; j < k; ++j)
      if (!ok(s, cudaMemcpyAsync(out + (size_t)(done + j) * out_stride, s->buf_b + (size_t)j * p->rows,
                                 sizeof(float) * p->rows, cudaMemcpyDeviceToHost, s->st)))
        return;
    if (!ok(s, cudaStreamSynchronize(s->st))) return;
    int gave_up = 0;  // a projection that gave up waiting for its weight copies
    if (!ok(s, cudaMemcpy(&gave_up, s->err, sizeof(int), cudaMemcpyDeviceToHost))) return;
    if (gave_up) {
      cudaMemset(s->err, 0, sizeof(int));
      return void(note(s, IGC_FAIL_DEVICE));
    }
    done += k;
  }
}

void desk_mat_vec(igc_desk *d, const igc_plane *sheet, const float *act, float *out) {
  desk_mat_mat(d, sheet, act, 0, 1, out, 0);
}

void desk_norm_rms(igc_desk *d, const float *x, const float *w, int n, float eps, float *out) {
  DeskState *s = state_of(d);
  if (cudaSetDevice(s->device) != cudaSuccess || !grow(s, (size_t)n)) return;
  if (!ok(s, cudaMemcpyAsync(s->buf_a, x, sizeof(float) * n, cudaMemcpyHostToDevice, s->st))) return;
  if (w && !ok(s, cudaMemcpyAsync(s->buf_c, w, sizeof(float) * n, cudaMemcpyHostToDevice, s->st))) return;
  if (!ok(s, igc_launch_desk_norm(s->buf_a, w ? s->buf_c : nullptr, n, eps, s->buf_b, s->st))) return;
  if (!ok(s, cudaMemcpyAsync(out, s->buf_b, sizeof(float) * n, cudaMemcpyDeviceToHost, s->st))) return;
  ok(s, cudaStreamSynchronize(s->st));
}

void desk_soft_max(igc_desk *d, float *x, int n) {
  DeskState *s = state_of(d);
  if (cudaSetDevice(s->device) != cudaSuccess || !grow(s, (size_t)n)) return;
  if (!ok(s, cudaMemcpyAsync(s->buf_a, x, sizeof(float) * n, cudaMemcpyHostToDevice, s->st))) return;
  if (!ok(s, igc_launch_desk_softmax(s->buf_a, n, s->st))) return;
  if (!ok(s, cudaMemcpyAsync(x, s->buf_a, sizeof(float) * n, cudaMemcpyDeviceToHost, s->st))) return;
  ok(s, cudaStreamSynchronize(s->st));
}

void desk_gelu_gate(igc_desk *d, float *gate, const float *rise, int n) {
  DeskState *s = state_of(d);
  if (cudaSetDevice(s->device) != cudaSuccess || !grow(s, (size_t)n)) return;
  if (!ok(s, cudaMemcpyAsync(s->buf_a, gate, sizeof(float) * n, cudaMemcpyHostToDevice, s->st))) return;
  if (!ok(s, cudaMemcpyAsync(s->buf_b, rise, sizeof(float) * n, cudaMemcpyHostToDevice, s->st))) return;
  if (!ok(s, igc_launch_desk_gelu(s->buf_a, s->buf_b, n, s->st))) return;
  if (!ok(s, cudaMemcpyAsync(gate, s->buf_a, sizeof(float) * n, cudaMemcpyDeviceToHost, s->st))) return;
  ok(s, cudaStreamSynchronize(s->st));
}

void desk_rope_turn(igc_desk *d, float *x, int head, const float *cs, const float *sn) {
  DeskState *s = state_of(d);
  int half = head / 2;
  if (cudaSetDevice(s->device) != cudaSuccess || !grow(s, (size_t)head)) return;
  if (!ok(s, cudaMemcpyAsync(s->buf_a, x, sizeof(float) * head, cudaMemcpyHostToDevice, s->st))) return;
  if (!ok(s, cudaMemcpyAsync(s->buf_b, cs, sizeof(float) * half, cudaMemcpyHostToDevice, s->st))) return;
  if (!ok(s, cudaMemcpyAsync(s->buf_c, sn, sizeof(float) * half, cudaMemcpyHostToDevice, s->st))) return;
  if (!ok(s, igc_launch_desk_rope(s->buf_a, head, s->buf_b, s->buf_c, s->st))) return;
  if (!ok(s, cudaMemcpyAsync(x, s->buf_a, sizeof(float) * head, cudaMemcpyDeviceToHost, s->st))) return;
  ok(s, cudaStreamSynchronize(s->st));
}

}  // namespace

extern "C" int igc_back_open(igc_desk *desk, int device) {
  if (!desk) return IGC_FAIL_ARGUMENT;
  memset(desk, 0, sizeof(*desk));
  if (cudaSetDevice(device) != cudaSuccess) return IGC_FAIL_DEVICE;
  DeskState *s = new DeskState();
  s->device = device;
  if (cudaDeviceGetAttribute(&s->sm_count, cudaDevAttrMultiProcessorCount, device) != cudaSuccess ||
      cudaDeviceGetAttribute(&s->smem_limit, cudaDevAttrMaxSharedMemoryPerBlockOptin, device) != cudaSuccess ||
      cudaStreamCreateWithFlags(&s->st, cudaStreamNonBlocking) != cudaSuccess ||
      igc_kernels_configure(227 * 1024) != cudaSuccess || igc_lanes_configure() != cudaSuccess ||
      cudaMalloc(&s->arg_val, (size_t)s->sm_count * 4 * 16 * 4) != cudaSuccess ||
      cudaMalloc(&s->arg_idx, (size_t)s->sm_count * 4 * 16 * 4) != cudaSuccess ||
      cudaMalloc(&s->err, sizeof(int)) != cudaSuccess || cudaMemset(s->err, 0, sizeof(int)) != cudaSuccess) {
    delete s;
    return IGC_FAIL_DEVICE;
  }
  s->smem_limit -= 2048;
  desk->name_text = "cuda/sm_100a";
  desk->state = s;
  desk->mat_vec = desk_mat_vec;
  desk->mat_mat = desk_mat_mat;
  desk->norm_rms = desk_norm_rms;
  desk->soft_max = desk_soft_max;
  desk->gelu_gate = desk_gelu_gate;
  desk->rope_turn = desk_rope_turn;
  return IGC_OKAY;
}

extern "C" void igc_back_close(igc_desk *desk) {
  if (!desk || !desk->state) return;
  DeskState *s = state_of(desk);
  cudaSetDevice(s->device);
  for (auto &kv : s->planes) {
    cudaFree(kv.second.tiles);
    cudaFree(kv.second.scales);
    cudaFree(kv.second.plain_data);
    cudaFree(kv.second.plain_scales);
  }
  cudaFree(s->buf_a);
  cudaFree(s->buf_b);
  cudaFree(s->buf_c);
  cudaFree(s->arg_val);
  cudaFree(s->arg_idx);
  cudaFree(s->err);
  cudaFree(s->lane_act);
  cudaFree(s->lane_factor);
  cudaFree(s->lane_part);
  cudaFree(s->lane_out);
  cudaFree(s->lane_tiles);
  if (s->st) cudaStreamDestroy(s->st);
  delete s;
  desk->state = nullptr;
}

extern "C" int igc_desk_status(igc_desk *desk) {
  if (!desk || !desk->state) return IGC_FAIL_ARGUMENT;
  DeskState *s = state_of(desk);
  int c = s->status;
  s->status = IGC_OKAY;
  return c;
}
