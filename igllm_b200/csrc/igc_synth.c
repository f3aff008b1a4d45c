/* igc_synth.c - seeded synthetic checkpoints (see igc_synth.h). */
#define _POSIX_C_SOURCE 200809L
#include "igc_synth.h"

#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

/* ---- values ------------------------------------------------------------- */

static uint64_t mix64(uint64_t z) { /* splitmix64 finalizer */
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

uint64_t igc_synth_stream(const char *name) {
  uint64_t h = 0xCBF29CE484222325ull;
  for (; *name; ++name) h = (h ^ (uint8_t)*name) * 0x100000001B3ull;
  return h;
}

static uint64_t stream_base(uint64_t seed, uint64_t stream) {
  return mix64(seed * 0xD1342543DE82EF95ull ^ stream * 0x9E3779B97F4A7C15ull ^ 0x5851F42D4C957F2Dull);
}

static uint64_t value_hash(uint64_t base, uint64_t index) {
  return mix64(base + (index + 1) * 0x9E3779B97F4A7C15ull);
}

/* Standard normal quantile by Newton's method on erfc from libm; the table is
 * computed once on the host and is the only source of every normal value. */
static double normal_quantile(double p) {
  double x = p < 0.5 ? -sqrt(-2.0 * log(p)) : sqrt(-2.0 * log(1.0 - p));
  for (int it = 0; it < 60; ++it) {
    double cdf = 0.5 * erfc(-x / sqrt(2.0));
    double pdf = exp(-0.5 * x * x) / sqrt(2.0 * 3.14159265358979323846);
    double step = (cdf - p) / pdf;
    x -= step;
    if (fabs(step) < 1e-15 * (1.0 + fabs(x))) break;
  }
  return x;
}

static double quantile_table[65536];
static pthread_once_t table_once = PTHREAD_ONCE_INIT;

static void table_build(void) {
  for (int i = 0; i < 65536; ++i) quantile_table[i] = normal_quantile(((double)i + 0.5) / 65536.0);
}

static uint16_t f32_to_bf16(float f) { /* round to nearest even */
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7F800000u) == 0x7F800000u) return (uint16_t)(u >> 16);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

static uint16_t f32_to_f16(float f) { /* correctly rounded by the compiler */
  _Float16 h = (_Float16)f;
  uint16_t u;
  memcpy(&u, &h, 2);
  return u;
}

typedef struct fill_job {
  uint64_t base;
  int kind;
  float offset;
  size_t from, upto; /* stream indices to generate */
  size_t origin;     /* the stream index that lands at out[0] */
  void *out;
} fill_job;

static void fill_range(const fill_job *j) {
  const float sigma = 0.02f;
  size_t i;
  if (j->kind == IGC_SYNTH_CONST) {
    float *o = (float *)j->out;
    for (i = j->from; i < j->upto; ++i) o[i - j->origin] = j->offset;
  } else if (j->kind == IGC_SYNTH_CODE) {
    uint8_t *o = (uint8_t *)j->out;
    for (i = j->from; i < j->upto; ++i) o[i - j->origin] = (uint8_t)(value_hash(j->base, i) & 0xFFu);
  } else {
    uint16_t *o = (uint16_t *)j->out;
    for (i = j->from; i < j->upto; ++i) {
      double q = quantile_table[value_hash(j->base, i) >> 48];
      if (j->kind == IGC_SYNTH_SCALE)
        o[i - j->origin] = f32_to_f16((float)fabs((double)sigma * q));
      else if (j->kind == IGC_SYNTH_SCALE_BF16) /* not below f16's smallest normal, 2^-14 */
        o[i - j->origin] = f32_to_bf16((float)fmax(fabs((double)sigma * q), 1.0 / 16384.0));
      else if (j->kind == IGC_SYNTH_NORMAL)
        o[i - j->origin] = f32_to_bf16((float)((double)sigma * q));
      else
        o[i - j->origin] = f32_to_bf16((float)((double)j->offset + (double)sigma * q));
    }
  }
}

static void *fill_thread(void *arg) {
  fill_range((const fill_job *)arg);
  return NULL;
}

int igc_synth_fill(uint64_t seed, uint64_t stream, int kind, float offset, size_t count, void *out,
                   int threads) {
  fill_job jobs[64];
  pthread_t tid[64];
  int n = threads < 1 ? 1 : (threads > 64 ? 64 : threads);
  if (!out || kind < 0 || kind > IGC_SYNTH_SCALE_BF16) return IGC_FAIL_ARGUMENT;
  pthread_once(&table_once, table_build);
  if (count < ((size_t)1 << 20)) n = 1;
  for (int t = 0; t < n; ++t) {
    jobs[t].base = stream_base(seed, stream);
    jobs[t].kind = kind;
    jobs[t].offset = offset;
    jobs[t].from = count * (size_t)t / (size_t)n;
    jobs[t].upto = count * (size_t)(t + 1) / (size_t)n;
    jobs[t].origin = 0;
    jobs[t].out = out;
  }
  if (n == 1) {
    fill_range(&jobs[0]);
    return IGC_OKAY;
  }
  for (int t = 0; t < n; ++t) pthread_create(&tid[t], NULL, fill_thread, &jobs[t]);
  for (int t = 0; t < n; ++t) pthread_join(tid[t], NULL);
  return IGC_OKAY;
}

/* ---- the tensor list ------------------------------------------------------ */

static int layer_global(const igc_synth_spec *s, int l) {
  if (l == s->layers - 1) return 1; /* app_core.c:8395 the last layer is global */
  return s->global_every > 0 && ((l + 1) % s->global_every) == 0;
}

static size_t dtype_size(int dtype) { return dtype == 6 || dtype == 5 ? 1u : dtype == 1 ? 4u : 2u; }

static void add(igc_synth_tensor *room, int room_count, int *n, const char *name, int dtype,
                int64_t r, int64_t c, int rank, int kind, float offset) {
  if (room && *n < room_count) {
    igc_synth_tensor *t = &room[*n];
    size_t el = dtype_size(dtype);
    memset(t, 0, sizeof(*t));
    snprintf(t->name, sizeof(t->name), "%s", name);
    t->dtype = dtype;
    t->rank = rank;
    t->shape[0] = r;
    t->shape[1] = c;
    t->kind = kind;
    t->offset = offset;
    t->bytes = (size_t)r * (size_t)(rank == 2 ? c : 1) * el;
  }
  *n += 1;
}

/* A code plane as the export stores it (app_core.c:7886 plane_bind_gemma):
 * `bits`-bit codes packed from the low bit in U8 rows, and a scale for every
 * `group` columns (F16, or BF16 when `bf16`), under `leaf` / `scale_leaf`. */
static void add_codes(igc_synth_tensor *room, int room_count, int *n, const char *stem, int64_t rows,
                      int64_t cols, int bits, int group, int bf16, const char *leaf, const char *scale_leaf) {
  char name[128];
  snprintf(name, sizeof(name), "%s.%s", stem, leaf);
  add(room, room_count, n, name, 6, rows, (cols * bits + 7) / 8, 2, IGC_SYNTH_CODE, 0.0f);
  snprintf(name, sizeof(name), "%s.%s", stem, scale_leaf);
  add(room, room_count, n, name, bf16 ? 3 : 2, rows, cols / group, 2, bf16 ? IGC_SYNTH_SCALE_BF16 : IGC_SYNTH_SCALE,
      0.0f);
}

static int spec_group(const igc_synth_spec *s) { return s->group > 0 ? s->group : 32; }

/* The export's activation grids of a projection (app_core.c:7941-7948): F32
 * scalars, varied by a hash of the stem so planes differ. */
static void add_grids(igc_synth_tensor *room, int room_count, int *n, const igc_synth_spec *s, const char *stem) {
  char name[160];
  const float vary = 1.0f + (float)(igc_synth_stream(stem) % 4) / 4.0f;
  if (s->grid_in > 0.0f) {
    snprintf(name, sizeof(name), "%s.input_activation_scale", stem);
    add(room, room_count, n, name, 1, 1, 0, 1, IGC_SYNTH_CONST, s->grid_in * vary);
  }
  if (s->grid_out > 0.0f) {
    snprintf(name, sizeof(name), "%s.output_activation_scale", stem);
    add(room, room_count, n, name, 1, 1, 0, 1, IGC_SYNTH_CONST, s->grid_out * vary);
  }
}

static void add_plane_bits(igc_synth_tensor *room, int room_count, int *n, const igc_synth_spec *s,
                           const char *stem, int64_t rows, int64_t cols, int bits) {
  if (bits == 8) { /* signed bytes, a scale a row (app_core.c:7910-7912) */
    char name[128];
    snprintf(name, sizeof(name), "%s.weight", stem);
    add(room, room_count, n, name, 5, rows, cols, 2, IGC_SYNTH_CODE, 0.0f);
    snprintf(name, sizeof(name), "%s.weight_scale", stem);
    add(room, room_count, n, name, 2, rows, 1, 2, IGC_SYNTH_SCALE, 0.0f);
  } else {
    add_codes(room, room_count, n, stem, rows, cols, bits, spec_group(s), s->bf16_scales, "weight", "weight_scale");
  }
  add_grids(room, room_count, n, s, stem);
}

static void add_plane(igc_synth_tensor *room, int room_count, int *n, const igc_synth_spec *s, const char *stem,
                      int64_t rows, int64_t cols) {
  add_plane_bits(room, room_count, n, s, stem, rows, cols, 4);
}

int igc_synth_list(const igc_synth_spec *s, igc_synth_tensor *room, int room_count) {
  const char *P = "model.language_model.";
  char name[128];
  int n = 0;
  int first_share = s->layers - s->share_count;
  int PS = s->layers * s->ple_dim;
  float no = s->norm_offset;
  if (s->embed_bits > 0) { /* the export's quantized tables (app_core.c:7968) */
    snprintf(name, sizeof(name), "%sembed_tokens", P);
    add_codes(room, room_count, &n, name, s->vocab, s->hidden, s->embed_bits, spec_group(s), s->bf16_scales,
              "embedding_quantized", "embedding_scale");
  } else {
    snprintf(name, sizeof(name), "%sembed_tokens.weight", P);
    add(room, room_count, &n, name, 3, s->vocab, s->hidden, 2, IGC_SYNTH_NORMAL, 0.0f);
  }
  if (s->ple_embed_bits > 0) {
    snprintf(name, sizeof(name), "%sembed_tokens_per_layer", P);
    add_codes(room, room_count, &n, name, s->vocab, PS, s->ple_embed_bits, spec_group(s), s->bf16_scales,
              "embedding_quantized", "embedding_scale");
  } else {
    snprintf(name, sizeof(name), "%sembed_tokens_per_layer.weight", P);
    add(room, room_count, &n, name, 3, s->vocab, PS, 2, IGC_SYNTH_NORMAL, 0.0f);
  }
  snprintf(name, sizeof(name), "%sper_layer_model_projection", P);
  if (s->dense_ple_lift) { /* left unquantized by the export: bf16 N(0, 0.02) */
    char wname[160];
    snprintf(wname, sizeof(wname), "%s.weight", name);
    add(room, room_count, &n, wname, 3, PS, s->hidden, 2, IGC_SYNTH_NORMAL, 0.0f);
  } else {
    add_plane(room, room_count, &n, s, name, PS, s->hidden);
  }
  snprintf(name, sizeof(name), "%sper_layer_projection_norm.weight", P);
  add(room, room_count, &n, name, 3, s->ple_dim, 0, 1, IGC_SYNTH_OFFSET, no);
  snprintf(name, sizeof(name), "%snorm.weight", P);
  add(room, room_count, &n, name, 3, s->hidden, 0, 1, IGC_SYNTH_OFFSET, no);
  if (!s->tied_head) /* the head carries no activation grids in the export */
    add_codes(room, room_count, &n, "lm_head", s->vocab, s->hidden, 4, spec_group(s), s->bf16_scales, "weight",
              "weight_scale");
  for (int l = 0; l < s->layers; ++l) {
    char stem[128];
    int share = s->share_count > 0 && l >= first_share;
    /* a global layer's head width (global_head_dim), and the doubled
     * feed-forward of the layers that share another's cache */
    int hd = layer_global(s, l) && s->global_head_dim > 0 ? s->global_head_dim : s->head_dim;
    int qw = s->heads * hd, kvw = s->kv_heads * hd;
    int inner = share && s->double_wide ? 2 * s->inner : s->inner;
#define STEM(fmt) snprintf(stem, sizeof(stem), "%slayers.%d." fmt, P, l)
    STEM("self_attn.q_proj");
    add_plane(room, room_count, &n, s, stem, qw, s->hidden);
    if (!share) {
      STEM("self_attn.k_proj");
      add_plane(room, room_count, &n, s, stem, kvw, s->hidden);
      STEM("self_attn.v_proj");
      add_plane(room, room_count, &n, s, stem, kvw, s->hidden);
      STEM("self_attn.k_norm.weight");
      add(room, room_count, &n, stem, 3, hd, 0, 1, IGC_SYNTH_OFFSET, no);
      /* the export's static cache ranges (app_core.c:8596-8601), varied by layer */
      if (s->cache_scale_k > 0.0f) {
        STEM("self_attn.k_cache_scale");
        add(room, room_count, &n, stem, 1, 1, 0, 1, IGC_SYNTH_CONST, s->cache_scale_k * (1.0f + (float)(l % 4) / 8.0f));
      }
      if (s->cache_scale_v > 0.0f) {
        STEM("self_attn.v_cache_scale");
        add(room, room_count, &n, stem, 1, 1, 0, 1, IGC_SYNTH_CONST, s->cache_scale_v * (1.0f + (float)(l % 4) / 8.0f));
      }
    }
    STEM("self_attn.o_proj");
    add_plane(room, room_count, &n, s, stem, s->hidden, qw);
    STEM("self_attn.q_norm.weight");
    add(room, room_count, &n, stem, 3, hd, 0, 1, IGC_SYNTH_OFFSET, no);
    {
      /* the export codes the sharing layers' feed-forward narrower */
      const int mb = share && s->late_mlp_bits > 0 ? s->late_mlp_bits : 4;
      STEM("mlp.gate_proj");
      add_plane_bits(room, room_count, &n, s, stem, inner, s->hidden, mb);
      STEM("mlp.up_proj");
      add_plane_bits(room, room_count, &n, s, stem, inner, s->hidden, mb);
      STEM("mlp.down_proj");
      add_plane_bits(room, room_count, &n, s, stem, s->hidden, inner, mb);
    }
    STEM("input_layernorm.weight");
    add(room, room_count, &n, stem, 3, s->hidden, 0, 1, IGC_SYNTH_OFFSET, no);
    STEM("post_attention_layernorm.weight");
    add(room, room_count, &n, stem, 3, s->hidden, 0, 1, IGC_SYNTH_OFFSET, no);
    STEM("pre_feedforward_layernorm.weight");
    add(room, room_count, &n, stem, 3, s->hidden, 0, 1, IGC_SYNTH_OFFSET, no);
    STEM("post_feedforward_layernorm.weight");
    add(room, room_count, &n, stem, 3, s->hidden, 0, 1, IGC_SYNTH_OFFSET, no);
    if (s->ple_dim > 0) {
      STEM("per_layer_input_gate");
      add_plane_bits(room, room_count, &n, s, stem, s->ple_dim, s->hidden, s->ple_bits8 ? 8 : 4);
      STEM("per_layer_projection");
      add_plane_bits(room, room_count, &n, s, stem, s->hidden, s->ple_dim, s->ple_bits8 ? 8 : 4);
      STEM("post_per_layer_input_norm.weight");
      add(room, room_count, &n, stem, 3, s->hidden, 0, 1, IGC_SYNTH_OFFSET, no);
    }
    if (s->with_layer_scalar) {
      STEM("layer_scalar");
      add(room, room_count, &n, stem, 3, 1, 0, 1, IGC_SYNTH_OFFSET, 1.0f);
    }
#undef STEM
  }
  return n;
}

int igc_synth_tensor_fill(const igc_synth_spec *spec, const igc_synth_tensor *t, void *out,
                          int threads) {
  size_t count = t->bytes / dtype_size(t->dtype);
  return igc_synth_fill(spec->seed, igc_synth_stream(t->name), t->kind, t->offset, count, out,
                        threads);
}

/* ---- files ---------------------------------------------------------------- */

typedef struct text_buf { char *data; size_t len, cap; } text_buf;

static void tb_add(text_buf *b, const char *fmt, ...) __attribute__((format(printf, 2, 3)));
#include <stdarg.h>
static void tb_add(text_buf *b, const char *fmt, ...) {
  va_list ap;
  for (;;) {
    int need;
    va_start(ap, fmt);
    need = vsnprintf(b->data ? b->data + b->len : NULL, b->data ? b->cap - b->len : 0, fmt, ap);
    va_end(ap);
    if (b->data && (size_t)need < b->cap - b->len) { b->len += (size_t)need; return; }
    b->cap = (b->cap + (size_t)need + 1) * 2;
    b->data = (char *)realloc(b->data, b->cap);
    if (b->len == 0) b->data[0] = 0;
  }
}

char *igc_synth_config_text(const igc_synth_spec *s) {
  text_buf b = {0, 0, 0};
  tb_add(&b, "{\n  \"model_type\": \"gemma4\",\n  \"tie_word_embeddings\": false,\n");
  tb_add(&b, "  \"quantization_config\": {\"quant_method\": \"gemma\", \"num_bits\": 4},\n");
  tb_add(&b, "  \"text_config\": {\n");
  tb_add(&b, "    \"model_type\": \"gemma4_text\",\n");
  tb_add(&b, "    \"vocab_size\": %d,\n    \"vocab_size_per_layer_input\": %d,\n", s->vocab, s->vocab);
  tb_add(&b, "    \"hidden_size\": %d,\n    \"intermediate_size\": %d,\n", s->hidden, s->inner);
  tb_add(&b, "    \"num_hidden_layers\": %d,\n    \"num_attention_heads\": %d,\n", s->layers, s->heads);
  tb_add(&b, "    \"num_key_value_heads\": %d,\n    \"head_dim\": %d,\n    \"global_head_dim\": %d,\n",
         s->kv_heads, s->head_dim, s->global_head_dim > 0 ? s->global_head_dim : s->head_dim);
  tb_add(&b, "    \"hidden_size_per_layer_input\": %d,\n    \"num_kv_shared_layers\": %d,\n",
         s->ple_dim, s->share_count);
  tb_add(&b, "    \"sliding_window\": %d,\n    \"max_position_embeddings\": %d,\n", s->slide_span,
         s->window_limit);
  tb_add(&b, "    \"use_double_wide_mlp\": %s,\n    \"attention_k_eq_v\": false,\n",
         s->double_wide ? "true" : "false");
  tb_add(&b, "    \"enable_moe_block\": false,\n    \"rms_norm_eps\": 1e-06,\n");
  tb_add(&b, "    \"final_logit_softcapping\": 30.0,\n    \"hidden_activation\": \"gelu_pytorch_tanh\",\n");
  tb_add(&b, "    \"bos_token_id\": 2,\n    \"eos_token_id\": 1,\n    \"pad_token_id\": 0,\n");
  tb_add(&b, "    \"rope_parameters\": {\n");
  tb_add(&b, "      \"full_attention\": {\"partial_rotary_factor\": 0.25, \"rope_theta\": 1000000.0, "
             "\"rope_type\": \"proportional\"},\n");
  tb_add(&b, "      \"sliding_attention\": {\"rope_theta\": 10000.0, \"rope_type\": \"default\"}\n    },\n");
  tb_add(&b, "    \"layer_types\": [");
  for (int l = 0; l < s->layers; ++l)
    tb_add(&b, "%s\"%s\"", l ? ", " : "", layer_global(s, l) ? "full_attention" : "sliding_attention");
  tb_add(&b, "]\n  }\n}\n");
  return b.data;
}

static int write_text(const char *folder, const char *leaf, const char *text) {
  char path[4096];
  FILE *f;
  snprintf(path, sizeof(path), "%s/%s", folder, leaf);
  f = fopen(path, "wb");
  if (!f) return IGC_FAIL_FILE;
  fwrite(text, 1, strlen(text), f);
  fclose(f);
  return IGC_OKAY;
}

static const char *dtype_name(int dtype) {
  switch (dtype) {
    case 1: return "F32";
    case 2: return "F16";
    case 3: return "BF16";
    case 5: return "I8";
    case 6: return "U8";
    default: return "?";
  }
}

int igc_synth_write(const igc_synth_spec *spec, const char *folder, int threads) {
  int n = igc_synth_list(spec, NULL, 0);
  igc_synth_tensor *list = (igc_synth_tensor *)calloc((size_t)n, sizeof(igc_synth_tensor));
  text_buf hb = {0, 0, 0};
  size_t offset = 0;
  char path[4096];
  char *config;
  FILE *f;
  int code;
  uint64_t header_len;
  const size_t chunk = (size_t)64 << 20;
  void *buf;
  if (!list) return IGC_FAIL_MEMORY;
  igc_synth_list(spec, list, n);
  config = igc_synth_config_text(spec);
  code = write_text(folder, "config.json", config);
  free(config);
  if (code == IGC_OKAY)
    code = write_text(folder, "tokenizer.json",
                      "{\"model\": {\"type\": \"BPE\", \"vocab\": {\"<pad>\": 0, \"<eos>\": 1, "
                      "\"<bos>\": 2}, \"merges\": []}, \"added_tokens\": []}\n");
  if (code != IGC_OKAY) { free(list); return code; }
  tb_add(&hb, "{\"__metadata__\":{\"format\":\"pt\"}");
  for (int i = 0; i < n; ++i) {
    const igc_synth_tensor *t = &list[i];
    tb_add(&hb, ",\"%s\":{\"dtype\":\"%s\",\"shape\":[", t->name, dtype_name(t->dtype));
    if (t->rank == 2) tb_add(&hb, "%lld,%lld", (long long)t->shape[0], (long long)t->shape[1]);
    else tb_add(&hb, "%lld", (long long)t->shape[0]);
    tb_add(&hb, "],\"data_offsets\":[%zu,%zu]}", offset, offset + t->bytes);
    offset += t->bytes;
  }
  tb_add(&hb, "}");
  while (hb.len % 8) tb_add(&hb, " ");
  snprintf(path, sizeof(path), "%s/model.safetensors", folder);
  f = fopen(path, "wb");
  if (!f) { free(list); free(hb.data); return IGC_FAIL_FILE; }
  header_len = (uint64_t)hb.len;
  fwrite(&header_len, 8, 1, f);
  fwrite(hb.data, 1, hb.len, f);
  free(hb.data);
  buf = malloc(chunk);
  if (!buf) { fclose(f); free(list); return IGC_FAIL_MEMORY; }
  for (int i = 0; i < n && code == IGC_OKAY; ++i) {
    const igc_synth_tensor *t = &list[i];
    size_t el = dtype_size(t->dtype), count = t->bytes / el, per = chunk / el;
    uint64_t base_stream = igc_synth_stream(t->name);
    for (size_t from = 0; from < count; from += per) {
      size_t take = count - from < per ? count - from : per;
      size_t nt = (size_t)(threads < 1 ? 1 : (threads > 64 ? 64 : threads));
      fill_job jobs[64];
      pthread_t tid[64];
      pthread_once(&table_once, table_build);
      if (take < ((size_t)1 << 20)) nt = 1;
      for (size_t k = 0; k < nt; ++k) {
        jobs[k].base = stream_base(spec->seed, base_stream);
        jobs[k].kind = t->kind;
        jobs[k].offset = t->offset;
        jobs[k].from = from + take * k / nt;
        jobs[k].upto = from + take * (k + 1) / nt;
        jobs[k].origin = from;
        jobs[k].out = buf;
      }
      if (nt == 1) {
        fill_range(&jobs[0]);
      } else {
        for (size_t k = 0; k < nt; ++k) pthread_create(&tid[k], NULL, fill_thread, &jobs[k]);
        for (size_t k = 0; k < nt; ++k) pthread_join(tid[k], NULL);
      }
      if (fwrite(buf, el, take, f) != take) code = IGC_FAIL_FILE;
    }
  }
  free(buf);
  if (fclose(f) != 0) code = IGC_FAIL_FILE;
  free(list);
  return code;
}
