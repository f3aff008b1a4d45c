/* igo.h - CPU oracle for the speculative verify round (TEST INFRASTRUCTURE).
 *
 * This is a plain-C restatement of the reference engine's text-stack verify
 * round (iamhaymc/igllm, app_core.c), written to check the CUDA build against.
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may
 * load it.  Nothing in the product links or calls it.
 *
 * Parity pin: the restatement is held to the reference itself, compiled from
 * its own sources into oracle/_ref by oracle/Makefile, and to the known-answer
 * values of the reference's own unit tests (app_test.c test_gemma, test_kernel,
 * test_scout, test_guess).  See tests/test_oracle_*.py.
 *
 * Every function cites the reference function it restates.
 */
#ifndef IGO_H
#define IGO_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define IGO_LANE_LIMIT 16 /* app_core.c:1980 KERN_LANE_LIMIT */

/* One int4 group-quantized projection in the Gemma U8 layout
 * (app_core.c:7886-7949 plane_bind_gemma): `code` holds two codes a byte, low
 * nibble first, `row_stride` bytes a row; the stored code carries an offset of
 * eight; `scale` is one float a (row, group). */
typedef struct igo_plane {
  const uint8_t *code;
  const float   *scale;
  int rows, cols, row_stride, groups, group_size;
} igo_plane;

typedef struct igo_layer {
  int kind;   /* 0 sliding, 1 global (app_core.c:7502 MODEL_KIND_*) */
  int share;  /* reads another layer's cache (app_core.c:8581) */
  int source; /* the owner layer when share is set */
  float gain; /* layer_scalar, 1 when absent (app_core.c:8700-8708) */
  igo_plane q, k, v, o, gate, up, down, ple_gate, ple_proj;
  int has_v;  /* v_proj bound; keys double as values when not (app_core.c:11497) */
  const float *q_norm, *k_norm;
  const float *enter_norm, *after_attn_norm, *before_feed_norm, *after_feed_norm, *after_ple_norm;
} igo_layer;

typedef struct igo_model {
  int vocab, hidden, layers, heads, kv_heads, head_dim, inner, ple_dim, ple_vocab;
  int slide_span;  /* sliding_window */
  int window_limit;/* context length */
  float eps, softcap;
  /* rope per kind: theta, partial share, proportional flag (app_core.c:8121-8145) */
  double rope_theta[2];
  double rope_share[2];
  int rope_proportional[2];
  const uint16_t *embed;     /* bf16 [vocab][hidden] */
  const uint16_t *ple_embed; /* bf16 [ple_vocab][layers*ple_dim] */
  igo_plane ple_lift;        /* [layers*ple_dim][hidden] */
  const float *ple_norm, *final_norm;
  igo_plane head;            /* [vocab][hidden] */
  igo_layer *layer;
} igo_model;

/* Taste, app_core.c:60-67 app_taste */
typedef struct igo_taste {
  float heat;
  int top_count;
  float top_portion;
  float echo_penalty;
  int echo_window;
  uint64_t seed;
} igo_taste;

typedef struct igo_session igo_session;

igo_session *igo_session_open(const igo_model *model, int threads);
void igo_session_close(igo_session *s);
int igo_session_fill(const igo_session *s);
/* app_core.c:14443 session_prime: every id but the last, 16 lanes a pass */
int igo_session_prime(igo_session *s, const int32_t *ids, int n);
/* app_core.c:14473 session_step: one lane, logits of that lane (vocab floats) */
int igo_session_step(igo_session *s, int32_t id, float *logits_out);
/* app_core.c:12139 session_guess: K lanes, K rows of logits */
int igo_session_guess(igo_session *s, const int32_t *ids, int k, float *logits_out);
/* app_core.c:12205 session_guess_keep */
int igo_session_guess_keep(igo_session *s, int keep);
/* app_core.c:13935 session_hold, without the ring refusal (full-length caches) */
int igo_session_hold(igo_session *s, int keep);
/* app_core.c:14762 session_guess_taste */
int igo_session_guess_taste(igo_session *s, const float *rows, const int32_t *ids, int k,
                            const igo_taste *taste, int32_t *made_out);
/* app_core.c:14844 session_pick (greedy when heat <= 0) */
int32_t igo_session_pick(igo_session *s, const float *logits, const igo_taste *taste);
/* Kept echo history (ids fed), for checking the host/device agree. */
int igo_session_echo(const igo_session *s, int32_t *out, int limit);

/* The byte cache's e4m3 grid (app_core.c:10975-11035 cache_pack8 /
 * cache_code8 / cache_real8): a value (already divided by its layer's scale)
 * to its code, rounding to nearest with ties to even and saturating at
 * +-448 (a NaN to +448), and a code back to its value. */
uint8_t igo_cache_code8(float x);
float igo_cache_real8(uint8_t code);

/* Kernel-level restatements, exported for known-answer tests. */
float igo_row_code(const igo_plane *p, int row, const float *act);           /* kern_row_code :3688 */
void igo_mat_mat(const igo_plane *p, const float *act, int act_stride, int lanes, float *out,
                 int out_stride, int threads);                               /* back_mat_mat :5247 */
void igo_norm_rms(const float *x, const float *w, int n, float eps, float *out); /* :4667 */
float igo_gelu_tanh(float x);                                                /* :5109 */
void igo_logit_cap(float *x, int n, float cap);                              /* :5016 */
void igo_soft_max(float *x, int n);                                          /* :4856 */
void igo_rope_turn(float *x, int head, const float *cs, const float *sn);    /* :5196 */
void igo_rope_steps(double theta, double share, int proportional, int head, float *step_out,
                    int *turn_out);                                          /* :8121 */
void igo_plane_row(const igo_plane *p, int row, float *out);                 /* plane_row :1826 */

/* n-gram scout, app_core.c:12277-12361 */
typedef struct igo_scout igo_scout;
igo_scout *igo_scout_open(void);
void igo_scout_close(igo_scout *s);
void igo_scout_clear(igo_scout *s);
int igo_scout_note(igo_scout *s, const int32_t *ids, int n);
int igo_scout_span(const igo_scout *s);
int igo_scout_draw(const igo_scout *s, int32_t *out, int want);

/* Shaped distribution of app_core.c:14572 pick_shape, exported for tests:
 * fills ids/weights (caller room of vocab entries), returns kept count. */
int igo_pick_shape(const float *logits, int vocab, const igo_taste *taste, const int32_t *echo,
                   int echo_count, int32_t *id_out, float *weight_out);
uint64_t igo_guess_draw_state(uint64_t seed, uint64_t place, uint64_t part); /* :14706 */
float igo_draw_unit(uint64_t *state);                                         /* :12384 */

#ifdef __cplusplus
}
#endif
#endif
