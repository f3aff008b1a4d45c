/* igo.c - CPU oracle for the speculative verify round (TEST INFRASTRUCTURE).
 *
 * A plain-C restatement of the reference engine's text-stack pass, block
 * verify, undo, tempered verify and n-gram scout (iamhaymc/igllm app_core.c),
 * used only to check the CUDA build.  Arithmetic follows the reference's
 * float path step for step; summation order inside a dot product is plain
 * sequential rather than the reference's SIMD lanes, which moves results by a
 * few float ulps and nothing more.  Caches are full length rather than rings,
 * which holds the same rows at every position the reference reads.
 *
 * Each function names the reference function it restates (file:line).
 */
#include "igo.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ---- scalar conversions ------------------------------------------------ */

/* app_core.c:10980 cache_pack8 + :11008 cache_code8, from the format: field
 * 0 counts steps of 2^-9 (a value that rounds to no step is code 0 whatever
 * its sign); a value in [2^e, 2^(e+1)), e >= -6, has steps of
 * 2^(e-3), and its rounded step count q (8..16) is the code ((e+7) << 3) +
 * q - 8, carrying into the next exponent at q = 16. */
uint8_t igo_cache_code8(float x) {
  uint8_t sign = x < 0.0f ? 0x80u : 0u;
  float a = fabsf(x);
  int e;
  if (!(a < 448.0f)) return (uint8_t)(sign | 0x7Eu);
  if (a < 1.0f / 64.0f) { /* a value that rounds to zero keeps no sign */
    uint8_t q = (uint8_t)nearbyintf(a * 512.0f);
    return q ? (uint8_t)(sign | q) : 0u;
  }
  frexpf(a, &e); /* a in [2^(e-1), 2^e) */
  e -= 1;
  return (uint8_t)(sign | (uint8_t)(((e + 7) << 3) + (int)nearbyintf(ldexpf(a, 3 - e)) - 8));
}

/* app_core.c:11025 cache_real8 */
float igo_cache_real8(uint8_t code) {
  int f = (code >> 3) & 15, m = code & 7;
  float a = f == 0 ? (float)m / 512.0f : ldexpf((float)(8 + m), f - 10);
  return (code & 0x80u) ? -a : a;
}

static float bf16_to_f32(uint16_t h) { /* app_core.c:1689 real_from_bf16 */
  union { uint32_t u; float f; } c;
  c.u = (uint32_t)h << 16;
  return c.f;
}

/* ---- kernels ------------------------------------------------------------ */

/* app_core.c:1826 plane_row: w = (code - 8) * scale, one scale a group. */
void igo_plane_row(const igo_plane *p, int row, float *out) {
  const uint8_t *code_row = p->code + (size_t)row * (size_t)p->row_stride;
  for (int c = 0; c < p->cols; ++c) {
    int g = c / p->group_size;
    int nib = (code_row[c >> 1] >> ((c & 1) * 4)) & 15;
    out[c] = (float)(nib - 8) * p->scale[(size_t)row * p->groups + g];
  }
}

/* app_core.c:4288 kern_group_sum: per-group activation sums. */
static void group_sums(const igo_plane *p, const float *act, float *sum) {
  for (int g = 0; g < p->groups; ++g) {
    int from = g * p->group_size, upto = from + p->group_size;
    float t = 0.0f;
    if (upto > p->cols) upto = p->cols;
    for (int c = from; c < upto; ++c) t += act[c];
    sum[g] = t;
  }
}

/* app_core.c:3688 kern_row_code: row = sum_g s_g * (sum a*code - 8 * sum a). */
static float row_code_sum(const igo_plane *p, int row, const float *act, const float *sum) {
  const uint8_t *code_row = p->code + (size_t)row * (size_t)p->row_stride;
  float total = 0.0f;
  for (int g = 0; g < p->groups; ++g) {
    int from = g * p->group_size, upto = from + p->group_size;
    float part = 0.0f;
    if (upto > p->cols) upto = p->cols;
    for (int c = from; c < upto; ++c)
      part += (float)((code_row[c >> 1] >> ((c & 1) * 4)) & 15) * act[c];
    total += p->scale[(size_t)row * p->groups + g] * (part - 8.0f * sum[g]);
  }
  return total;
}

float igo_row_code(const igo_plane *p, int row, const float *act) {
  float *sum = (float *)malloc(sizeof(float) * (size_t)p->groups);
  float r;
  group_sums(p, act, sum);
  r = row_code_sum(p, row, act, sum);
  free(sum);
  return r;
}

/* app_core.c:5247 back_mat_mat over app_core.c:4075 kern_row_code_many. */
void igo_mat_mat(const igo_plane *p, const float *act, int act_stride, int lanes, float *out,
                 int out_stride, int threads) {
  float *sum = (float *)malloc(sizeof(float) * (size_t)p->groups * (size_t)lanes);
  for (int l = 0; l < lanes; ++l) group_sums(p, act + (size_t)l * act_stride, sum + (size_t)l * p->groups);
#ifdef _OPENMP
  int nt = threads > 0 ? threads : 1;
#pragma omp parallel for num_threads(nt) schedule(static)
#else
  (void)threads;
#endif
  for (int r = 0; r < p->rows; ++r)
    for (int l = 0; l < lanes; ++l)
      out[(size_t)l * out_stride + r] =
          row_code_sum(p, r, act + (size_t)l * act_stride, sum + (size_t)l * p->groups);
  free(sum);
}

/* app_core.c:4667 kern_norm_rms: double sum of squares, weight used as is. */
void igo_norm_rms(const float *x, const float *w, int n, float eps, float *out) {
  double sq = 0.0;
  for (int i = 0; i < n; ++i) sq += (double)x[i] * (double)x[i];
  float shrink = (float)pow(sq / (double)n + (double)eps, -0.5);
  for (int i = 0; i < n; ++i) out[i] = w ? x[i] * shrink * w[i] : x[i] * shrink;
}

/* app_core.c:5109 kern_gelu_tanh: x * t / (t + 1), t = e^{2y}, clamped. */
float igo_gelu_tanh(float x) {
  const float root = 0.7978845608028654f, bend = 0.044715f, reach = 30.0f;
  float cube = x * x * x;
  float turn = 2.0f * root * (x + bend * cube);
  float rise;
  if (!(turn > -reach)) return x * 0.0f;
  if (turn > reach) turn = reach;
  rise = expf(turn);
  return x * (rise / (rise + 1.0f));
}

/* app_core.c:5016 kern_logit_cap: cap * (1 - 2 / (e^{2x/cap} + 1)), clamp 10. */
void igo_logit_cap(float *x, int n, float cap) {
  float back = 1.0f / cap;
  for (int i = 0; i < n; ++i) {
    float t = x[i] * back;
    if (t > 10.0f) t = 10.0f;
    if (t < -10.0f) t = -10.0f;
    x[i] = cap * (1.0f - 2.0f / (expf(t + t) + 1.0f));
  }
}

/* app_core.c:4856 kern_soft_max */
void igo_soft_max(float *x, int n) {
  float peak = -FLT_MAX, total = 0.0f;
  for (int i = 0; i < n; ++i) if (x[i] > peak) peak = x[i];
  for (int i = 0; i < n; ++i) { x[i] = expf(x[i] - peak); total += x[i]; }
  for (int i = 0; i < n; ++i) x[i] /= total;
}

/* app_core.c:5196 kern_rope_turn: rotate-half over pairs (i, i + head/2). */
void igo_rope_turn(float *x, int head, const float *cs, const float *sn) {
  int half = head / 2;
  for (int i = 0; i < half; ++i) {
    float lo = x[i], hi = x[i + half];
    x[i] = lo * cs[i] - hi * sn[i];
    x[i + half] = hi * cs[i] + lo * sn[i];
  }
}

/* app_core.c:8121 rope_build: inverse frequencies; a "proportional" rope turns
 * only share*head/2 pairs, each at the full head's exponent, the rest stay. */
void igo_rope_steps(double theta, double share, int proportional, int head, float *step_out,
                    int *turn_out) {
  int half = head / 2, turn = half;
  if (proportional) turn = (int)(share * head / 2.0);
  if (turn > half) turn = half;
  if (turn < 0) turn = 0;
  for (int i = 0; i < half; ++i)
    step_out[i] = i < turn ? (float)(1.0 / pow(theta, (double)(2 * i) / (double)head)) : 0.0f;
  if (turn_out) *turn_out = turn;
}

/* ---- session ------------------------------------------------------------ */

struct igo_session {
  const igo_model *m;
  int threads;
  int fill;
  float **kc, **vc;           /* full-length caches per owner layer [window][kv*hd] */
  float *step[2];             /* rope inverse frequencies per kind */
  int32_t *echo;
  int echo_count, echo_limit;
  int guess_count, guess_from, guess_echo;
  uint64_t draw_state;
  /* lane rooms */
  float *x, *h, *q, *k, *v, *blend, *lift, *gate, *up, *ple, *seed, *score, *cs, *sn;
};

static float *room(size_t n) { return (float *)calloc(n ? n : 1, sizeof(float)); }

igo_session *igo_session_open(const igo_model *m, int threads) {
  igo_session *s = (igo_session *)calloc(1, sizeof(igo_session));
  int L = IGO_LANE_LIMIT, hd = m->head_dim, qw = m->heads * hd, kvw = m->kv_heads * hd;
  int wide = m->hidden > qw ? m->hidden : qw;
  s->m = m;
  s->threads = threads;
  s->kc = (float **)calloc((size_t)m->layers, sizeof(float *));
  s->vc = (float **)calloc((size_t)m->layers, sizeof(float *));
  for (int l = 0; l < m->layers; ++l)
    if (!m->layer[l].share) {
      s->kc[l] = room((size_t)m->window_limit * kvw);
      s->vc[l] = room((size_t)m->window_limit * kvw);
    }
  for (int kind = 0; kind < 2; ++kind) {
    s->step[kind] = room((size_t)hd / 2);
    igo_rope_steps(m->rope_theta[kind], m->rope_share[kind], m->rope_proportional[kind], hd,
                   s->step[kind], NULL);
  }
  s->echo_limit = m->window_limit;
  s->echo = (int32_t *)calloc((size_t)s->echo_limit, sizeof(int32_t));
  s->draw_state = 0x2545F4914F6CDD1DULL;
  s->x = room((size_t)L * m->hidden);
  s->h = room((size_t)L * m->hidden);
  s->q = room((size_t)L * qw);
  s->k = room((size_t)L * kvw);
  s->v = room((size_t)L * kvw);
  s->blend = room((size_t)L * qw);
  s->lift = room((size_t)L * wide);
  s->gate = room((size_t)L * (m->inner > m->ple_dim ? m->inner : m->ple_dim));
  s->up = room((size_t)L * m->inner);
  s->ple = room((size_t)L * m->layers * m->ple_dim);
  s->seed = room((size_t)m->layers * m->ple_dim);
  s->score = room((size_t)m->window_limit + 1);
  s->cs = room((size_t)hd / 2);
  s->sn = room((size_t)hd / 2);
  return s;
}

void igo_session_close(igo_session *s) {
  if (!s) return;
  for (int l = 0; l < s->m->layers; ++l) { free(s->kc[l]); free(s->vc[l]); }
  free(s->kc); free(s->vc); free(s->step[0]); free(s->step[1]); free(s->echo);
  free(s->x); free(s->h); free(s->q); free(s->k); free(s->v); free(s->blend); free(s->lift);
  free(s->gate); free(s->up); free(s->ple); free(s->seed); free(s->score); free(s->cs); free(s->sn);
  free(s);
}

int igo_session_fill(const igo_session *s) { return s->fill; }

int igo_session_echo(const igo_session *s, int32_t *out, int limit) {
  int n = s->echo_count < limit ? s->echo_count : limit;
  memcpy(out, s->echo, sizeof(int32_t) * (size_t)n);
  return s->echo_count;
}

static void lift(igo_session *s, const igo_plane *p, const float *act, int act_stride, int lanes,
                 float *out, int out_stride) {
  igo_mat_mat(p, act, act_stride, lanes, out, out_stride, s->threads);
}

/* app_core.c:8147 rope_wave: double angle, float cos/sin. */
static void rope_wave(igo_session *s, int kind, int place) {
  for (int i = 0; i < s->m->head_dim / 2; ++i) {
    double a = (double)place * (double)s->step[kind][i];
    s->cs[i] = (float)cos(a);
    s->sn[i] = (float)sin(a);
  }
}

/* app_core.c:11455 session_attend: q/k/v lifts, then lane by lane the head
 * norms, rotary turn, cache write and grouped attention, then the exit lift. */
static void attend(igo_session *s, int li, int place_from, int lanes, const float *enter,
                   float *exit_out) {
  const igo_model *m = s->m;
  const igo_layer *w = &m->layer[li];
  int hd = m->head_dim, qw = m->heads * hd, kvw = m->kv_heads * hd;
  int owner = w->share ? w->source : li;
  int group = m->heads / m->kv_heads;
  lift(s, &w->q, enter, m->hidden, lanes, s->q, qw);
  if (!w->share) {
    lift(s, &w->k, enter, m->hidden, lanes, s->k, kvw);
    if (w->has_v) lift(s, &w->v, enter, m->hidden, lanes, s->v, kvw);
  }
  for (int j = 0; j < lanes; ++j) {
    int place = place_from + j;
    float *ql = s->q + (size_t)j * qw;
    float *bl = s->blend + (size_t)j * qw;
    int start = 0;
    rope_wave(s, w->kind, place);
    for (int hh = 0; hh < m->heads; ++hh) {
      float *qh = ql + (size_t)hh * hd;
      igo_norm_rms(qh, w->q_norm, hd, m->eps, qh);
      igo_rope_turn(qh, hd, s->cs, s->sn);
    }
    if (!w->share) {
      float *kl = s->k + (size_t)j * kvw, *vl = s->v + (size_t)j * kvw;
      if (!w->has_v) memcpy(vl, kl, sizeof(float) * (size_t)kvw);
      for (int kh = 0; kh < m->kv_heads; ++kh) {
        float *kk = kl + (size_t)kh * hd, *vv = vl + (size_t)kh * hd;
        igo_norm_rms(kk, w->k_norm, hd, m->eps, kk);
        igo_rope_turn(kk, hd, s->cs, s->sn);
        igo_norm_rms(vv, NULL, hd, m->eps, vv);
      }
      memcpy(s->kc[li] + (size_t)place * kvw, kl, sizeof(float) * (size_t)kvw);
      memcpy(s->vc[li] + (size_t)place * kvw, vl, sizeof(float) * (size_t)kvw);
    }
    if (w->kind == 0) {
      start = place - m->slide_span + 1;
      if (start < 0) start = 0;
    }
    for (int hh = 0; hh < m->heads; ++hh) {
      const float *qh = ql + (size_t)hh * hd;
      int kvh = hh / group, span = place - start + 1;
      float *bh = bl + (size_t)hh * hd;
      for (int i = 0; i < span; ++i) {
        const float *kr = s->kc[owner] + (size_t)(start + i) * kvw + (size_t)kvh * hd;
        float t = 0.0f;
        for (int d = 0; d < hd; ++d) t += kr[d] * qh[d];
        s->score[i] = t; /* score scale is 1.0 (app_core.c:11314) */
      }
      igo_soft_max(s->score, span);
      for (int d = 0; d < hd; ++d) bh[d] = 0.0f;
      for (int i = 0; i < span; ++i) {
        const float *vr = s->vc[owner] + (size_t)(start + i) * kvw + (size_t)kvh * hd;
        float wgt = s->score[i];
        for (int d = 0; d < hd; ++d) bh[d] += wgt * vr[d];
      }
    }
  }
  lift(s, &w->o, s->blend, qw, lanes, exit_out, m->hidden);
}

static void vec_add(float *a, const float *b, int n) { for (int i = 0; i < n; ++i) a[i] += b[i]; }

/* app_core.c:11637 session_layer */
static void layer(igo_session *s, int li, int place_from, int lanes) {
  const igo_model *m = s->m;
  const igo_layer *w = &m->layer[li];
  int H = m->hidden;
  for (int j = 0; j < lanes; ++j)
    igo_norm_rms(s->x + (size_t)j * H, w->enter_norm, H, m->eps, s->h + (size_t)j * H);
  attend(s, li, place_from, lanes, s->h, s->lift);
  for (int j = 0; j < lanes; ++j) {
    float *ld = s->lift + (size_t)j * H;
    igo_norm_rms(ld, w->after_attn_norm, H, m->eps, ld);
    vec_add(s->x + (size_t)j * H, ld, H);
    igo_norm_rms(s->x + (size_t)j * H, w->before_feed_norm, H, m->eps, s->h + (size_t)j * H);
  }
  lift(s, &w->gate, s->h, H, lanes, s->gate, m->inner);
  lift(s, &w->up, s->h, H, lanes, s->up, m->inner);
  for (int j = 0; j < lanes; ++j)
    for (int i = 0; i < m->inner; ++i)
      s->gate[(size_t)j * m->inner + i] =
          igo_gelu_tanh(s->gate[(size_t)j * m->inner + i]) * s->up[(size_t)j * m->inner + i];
  lift(s, &w->down, s->gate, m->inner, lanes, s->lift, H);
  for (int j = 0; j < lanes; ++j) {
    float *ld = s->lift + (size_t)j * H;
    igo_norm_rms(ld, w->after_feed_norm, H, m->eps, ld);
    vec_add(s->x + (size_t)j * H, ld, H);
  }
  if (m->ple_dim > 0) {
    int P = m->ple_dim, PS = m->layers * m->ple_dim;
    lift(s, &w->ple_gate, s->x, H, lanes, s->gate, P);
    for (int j = 0; j < lanes; ++j)
      for (int i = 0; i < P; ++i)
        s->gate[(size_t)j * P + i] = igo_gelu_tanh(s->gate[(size_t)j * P + i]) *
                                     s->ple[(size_t)j * PS + (size_t)li * P + i];
    lift(s, &w->ple_proj, s->gate, P, lanes, s->lift, H);
    for (int j = 0; j < lanes; ++j) {
      float *ld = s->lift + (size_t)j * H;
      igo_norm_rms(ld, w->after_ple_norm, H, m->eps, ld);
      vec_add(s->x + (size_t)j * H, ld, H);
    }
  }
  if (w->gain != 1.0f)
    for (int j = 0; j < lanes; ++j)
      for (int i = 0; i < H; ++i) s->x[(size_t)j * H + i] *= w->gain;
}

/* app_core.c:11843 session_pass.  want: 0 none, 1 last lane, 2 every lane. */
static int pass(igo_session *s, const int32_t *ids, int lanes, int want, float *logits_out) {
  const igo_model *m = s->m;
  int H = m->hidden, place_from = s->fill;
  if (lanes < 1 || lanes > IGO_LANE_LIMIT) return -1;
  if (place_from + lanes > m->window_limit) return -1;
  for (int j = 0; j < lanes; ++j) if (ids[j] < 0 || ids[j] >= m->vocab) return -1;
  for (int j = 0; j < lanes; ++j) {
    const uint16_t *row = m->embed + (size_t)ids[j] * H;
    float g = (float)sqrt((double)H);
    for (int i = 0; i < H; ++i) s->x[(size_t)j * H + i] = bf16_to_f32(row[i]) * g;
  }
  if (m->ple_dim > 0) {
    int P = m->ple_dim, PS = m->layers * P;
    float blend = (float)(1.0 / sqrt(2.0));
    lift(s, &m->ple_lift, s->x, H, lanes, s->ple, PS);
    for (int j = 0; j < lanes; ++j) {
      float *lr = s->ple + (size_t)j * PS;
      const uint16_t *srow = m->ple_embed + (size_t)(ids[j] % m->ple_vocab) * PS;
      float sg = (float)sqrt((double)P), lg = (float)(1.0 / sqrt((double)H));
      for (int i = 0; i < PS; ++i) s->seed[i] = bf16_to_f32(srow[i]) * sg;
      for (int i = 0; i < PS; ++i) lr[i] *= lg;
      for (int c = 0; c < m->layers; ++c) {
        float *cd = lr + (size_t)c * P;
        igo_norm_rms(cd, m->ple_norm, P, m->eps, cd);
        for (int i = 0; i < P; ++i) cd[i] = (cd[i] + s->seed[(size_t)c * P + i]) * blend;
      }
    }
  }
  for (int l = 0; l < m->layers; ++l) layer(s, l, place_from, lanes);
  s->fill += lanes;
  for (int j = 0; j < lanes; ++j)
    if (s->echo_count < s->echo_limit) s->echo[s->echo_count++] = ids[j];
  if (want == 0) return 0;
  {
    int from = want == 2 ? 0 : lanes - 1, span = lanes - from;
    for (int t = 0; t < span; ++t)
      igo_norm_rms(s->x + (size_t)(from + t) * H, m->final_norm, H, m->eps, s->h + (size_t)t * H);
    lift(s, &m->head, s->h, H, span, logits_out, m->vocab);
    if (m->softcap > 0.0f)
      for (int t = 0; t < span; ++t) igo_logit_cap(logits_out + (size_t)t * m->vocab, m->vocab, m->softcap);
  }
  return 0;
}

/* app_core.c:14443 session_prime_media */
int igo_session_prime(igo_session *s, const int32_t *ids, int n) {
  if (!s || !ids || n < 1 || s->guess_count > 0) return -1;
  if (s->fill + n > s->m->window_limit) return -7;
  for (int i = 0; i < n; ++i) if (ids[i] < 0 || ids[i] >= s->m->vocab) return -1;
  for (int i = 0; i + 1 < n;) {
    int lanes = n - 1 - i;
    if (lanes > IGO_LANE_LIMIT) lanes = IGO_LANE_LIMIT;
    pass(s, ids + i, lanes, 0, NULL);
    i += lanes;
  }
  return 0;
}

/* app_core.c:14473 session_step_state */
int igo_session_step(igo_session *s, int32_t id, float *logits_out) {
  if (!s || s->guess_count > 0) return -7;
  return pass(s, &id, 1, 1, logits_out);
}

/* app_core.c:12139 session_guess.  No rows need saving with full-length
 * caches: the rows a rejected lane wrote sit past the kept fill and are
 * rewritten before any later lane reads them. */
int igo_session_guess(igo_session *s, const int32_t *ids, int k, float *logits_out) {
  if (!s || !ids || s->guess_count > 0) return -7;
  if (k < 1 || k > IGO_LANE_LIMIT) return -1;
  if (s->fill + k > s->m->window_limit) return -1;
  s->guess_from = s->fill;
  s->guess_echo = s->echo_count;
  s->guess_count = k;
  if (pass(s, ids, k, 2, logits_out) != 0) { s->guess_count = 0; return -1; }
  return 0;
}

/* app_core.c:12205 session_guess_keep */
int igo_session_guess_keep(igo_session *s, int keep) {
  if (!s || s->guess_count <= 0) return -7;
  if (keep < 0 || keep > s->guess_count) return -1;
  s->fill = s->guess_from + keep;
  s->echo_count = s->guess_echo + keep;
  if (s->echo_count > s->echo_limit) s->echo_count = s->echo_limit;
  s->guess_count = 0;
  return 0;
}

/* app_core.c:13935 session_hold */
int igo_session_hold(igo_session *s, int keep) {
  if (!s || keep < 0) return -1;
  if (s->guess_count > 0) return -7;
  if (keep > s->fill) return -1;
  s->fill = keep;
  s->echo_count = keep < s->echo_limit ? keep : s->echo_limit;
  return 0;
}

/* ---- sampler ------------------------------------------------------------ */

typedef struct slot_t { float w; int32_t id; } slot_t;

static int slot_order(const void *a, const void *b) { /* app_core.c:12394 pick_order */
  const slot_t *l = (const slot_t *)a, *r = (const slot_t *)b;
  if (l->w < r->w) return 1;
  if (l->w > r->w) return -1;
  return 0;
}

static uint64_t draw_next(uint64_t *st) { /* app_core.c:12376 xorshift64 */
  uint64_t v = *st;
  v ^= v << 13;
  v ^= v >> 7;
  v ^= v << 17;
  *st = v;
  return v;
}

float igo_draw_unit(uint64_t *st) { /* app_core.c:12384: top 24 bits */
  return (float)((draw_next(st) >> 40) / 16777216.0);
}

/* app_core.c:14706 guess_draw_state: splitmix64 finalizer over seed, place, part. */
uint64_t igo_guess_draw_state(uint64_t seed, uint64_t place, uint64_t part) {
  uint64_t st = seed ^ (place * 0xD1342543DE82EF95ull) ^ part;
  st ^= st >> 30;
  st *= 0xBF58476D1CE4E5B9ull;
  st ^= st >> 27;
  st *= 0x94D049BB133111EBull;
  st ^= st >> 31;
  return st ? st : 0x2545F4914F6CDD1Dull;
}

/* app_core.c:14572 pick_shape: echo penalty, top-k partial selection, softmax
 * at the heat, top-p cut at run >= p, renormalised. */
static int pick_shape_slots(const float *logits, int vocab, const igo_taste *t, const int32_t *echo,
                            int echo_count, slot_t *sl) {
  int keep;
  float total = 0.0f;
  for (int i = 0; i < vocab; ++i) { sl[i].w = logits[i]; sl[i].id = i; }
  if (t->echo_penalty != 1.0f && t->echo_window > 0) {
    int from = echo_count - t->echo_window;
    if (from < 0) from = 0;
    for (int e = from; e < echo_count; ++e) {
      int32_t id = echo[e];
      if (id < 0 || id >= vocab) continue;
      if (sl[id].w > 0.0f) sl[id].w /= t->echo_penalty;
      else sl[id].w *= t->echo_penalty;
    }
  }
  keep = t->top_count > 0 && t->top_count < vocab ? t->top_count : vocab;
  if (keep < vocab) {
    float bar = -FLT_MAX;
    int fill = 0;
    for (int i = 0; i < vocab; ++i) {
      if (fill < keep) {
        sl[fill++] = sl[i];
        if (fill == keep) {
          qsort(sl, (size_t)keep, sizeof(slot_t), slot_order);
          bar = sl[keep - 1].w;
        }
      } else if (sl[i].w > bar) {
        sl[keep - 1] = sl[i];
        qsort(sl, (size_t)keep, sizeof(slot_t), slot_order);
        bar = sl[keep - 1].w;
      }
    }
  }
  qsort(sl, (size_t)keep, sizeof(slot_t), slot_order);
  {
    float peak = sl[0].w;
    for (int i = 0; i < keep; ++i) {
      sl[i].w = expf((sl[i].w - peak) / t->heat);
      total += sl[i].w;
    }
  }
  if (total <= 0.0f) { sl[0].w = 1.0f; return 1; }
  for (int i = 0; i < keep; ++i) sl[i].w /= total;
  if (t->top_portion > 0.0f && t->top_portion < 1.0f) {
    float run = 0.0f;
    for (int i = 0; i < keep; ++i) {
      run += sl[i].w;
      if (run >= t->top_portion) { keep = i + 1; break; }
    }
    total = 0.0f;
    for (int i = 0; i < keep; ++i) total += sl[i].w;
    for (int i = 0; i < keep; ++i) sl[i].w /= total;
  }
  return keep;
}

int igo_pick_shape(const float *logits, int vocab, const igo_taste *t, const int32_t *echo,
                   int echo_count, int32_t *id_out, float *weight_out) {
  slot_t *sl = (slot_t *)malloc(sizeof(slot_t) * (size_t)vocab);
  int keep = pick_shape_slots(logits, vocab, t, echo, echo_count, sl);
  for (int i = 0; i < keep; ++i) { id_out[i] = sl[i].id; weight_out[i] = sl[i].w; }
  free(sl);
  return keep;
}

static int32_t pick_draw(const slot_t *sl, int keep, float u) { /* app_core.c:14653 */
  for (int i = 0; i < keep; ++i) {
    u -= sl[i].w;
    if (u <= 0.0f) return sl[i].id;
  }
  return sl[keep - 1].id;
}

/* app_core.c:14810 session_pick_at */
int32_t igo_session_pick(igo_session *s, const float *logits, const igo_taste *t) {
  int vocab = s->m->vocab;
  if (t->seed) s->draw_state = t->seed ^ (uint64_t)s->fill;
  if (t->heat <= 0.0f) {
    int best = 0;
    for (int i = 1; i < vocab; ++i) if (logits[i] > logits[best]) best = i;
    return best;
  }
  {
    slot_t *sl = (slot_t *)malloc(sizeof(slot_t) * (size_t)vocab);
    int keep = pick_shape_slots(logits, vocab, t, s->echo, s->echo_count, sl);
    int32_t id = pick_draw(sl, keep, igo_draw_unit(&s->draw_state));
    free(sl);
    return id;
  }
}

#define DRAW_TAKE 0x9E3779B97F4A7C15ull
#define DRAW_MAKE 0xC2B2AE3D27D4EB4Full

/* app_core.c:14762 session_guess_taste: accept guess t with p(t), otherwise
 * draw from p with t removed and renormalised. */
int igo_session_guess_taste(igo_session *s, const float *rows, const int32_t *ids, int k,
                            const igo_taste *t, int32_t *made_out) {
  int vocab = s->m->vocab, take = 0;
  slot_t *sl;
  if (!s || !rows || !ids || !made_out) return -1;
  if (k < 1 || s->guess_count != k) return -1;
  if (t->heat <= 0.0f) return -1;
  sl = (slot_t *)malloc(sizeof(slot_t) * (size_t)vocab);
  for (int j = 0; j < k; ++j) {
    const float *lg = rows + (size_t)j * vocab;
    int echo_count = s->guess_echo + j + 1;
    uint64_t place = (uint64_t)(s->guess_from + j + 1);
    int keep;
    if (echo_count > s->echo_limit) echo_count = s->echo_limit;
    keep = pick_shape_slots(lg, vocab, t, s->echo, echo_count, sl);
    if (j + 1 < k) {
      int32_t want = ids[j + 1];
      float share = 0.0f;
      uint64_t st;
      float u;
      for (int i = 0; i < keep; ++i) if (sl[i].id == want) { share = sl[i].w; break; }
      st = t->seed ? igo_guess_draw_state(t->seed, place, DRAW_TAKE) : s->draw_state;
      u = igo_draw_unit(&st);
      if (!t->seed) s->draw_state = st;
      if (u < share) { take += 1; continue; }
      {
        int fill = 0;
        float total = 0.0f;
        for (int i = 0; i < keep; ++i) {
          if (sl[i].id == want) continue;
          sl[fill++] = sl[i];
          total += sl[i].w;
        }
        if (fill < 1 || !(total > 0.0f)) { *made_out = want; free(sl); return take; }
        for (int i = 0; i < fill; ++i) sl[i].w /= total;
        keep = fill;
      }
    }
    {
      uint64_t st = t->seed ? igo_guess_draw_state(t->seed, place, DRAW_MAKE) : s->draw_state;
      float u = igo_draw_unit(&st);
      if (!t->seed) s->draw_state = st;
      *made_out = pick_draw(sl, keep, u);
    }
    free(sl);
    return take;
  }
  free(sl);
  return take;
}

/* ---- scout (app_core.c:12277-12361) -------------------------------------- */

struct igo_scout { int32_t *ids; int n, room; };

igo_scout *igo_scout_open(void) { return (igo_scout *)calloc(1, sizeof(igo_scout)); }
void igo_scout_close(igo_scout *s) { if (s) { free(s->ids); free(s); } }
void igo_scout_clear(igo_scout *s) { if (s) s->n = 0; }
int igo_scout_span(const igo_scout *s) { return s ? s->n : 0; }

int igo_scout_note(igo_scout *s, const int32_t *ids, int n) {
  if (!s || n < 0 || (!ids && n > 0)) return -1;
  if (s->n + n > s->room) {
    int want = s->room ? s->room : 1024;
    while (want < s->n + n) want *= 2;
    s->ids = (int32_t *)realloc(s->ids, sizeof(int32_t) * (size_t)want);
    s->room = want;
  }
  memcpy(s->ids + s->n, ids, sizeof(int32_t) * (size_t)n);
  s->n += n;
  return 0;
}

/* Longest reach first (3 then 2), latest match first, refused when nothing
 * follows the match. */
int igo_scout_draw(const igo_scout *s, int32_t *out, int want) {
  if (!s || !out || want < 1) return 0;
  for (int reach = 3; reach >= 2; --reach) {
    const int32_t *tail;
    if (s->n < reach + 1) continue;
    tail = s->ids + s->n - reach;
    for (int place = s->n - reach - 1; place >= 0; --place) {
      int slot, take;
      for (slot = 0; slot < reach; ++slot) if (s->ids[place + slot] != tail[slot]) break;
      if (slot < reach) continue;
      take = s->n - (place + reach);
      if (take < 1) continue;
      if (take > want) take = want;
      memcpy(out, s->ids + place + reach, sizeof(int32_t) * (size_t)take);
      return take;
    }
  }
  return 0;
}
