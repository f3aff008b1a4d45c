/* ref_harness.c - drives the reference engine itself (TEST INFRASTRUCTURE).
 *
 * Compiled by oracle/Makefile together with the reference's own single
 * translation unit (app_core.c, included here exactly as the reference's
 * app_test.c:22 does) into oracle/_ref/libref_*.so.  It adds no arithmetic:
 * each wrapper calls one public entry point of the reference and copies out
 * what that entry point hands back, so Python tests and bench.py's reference
 * arm can call the reference through ctypes.
 */
#include "app_core.c"

typedef struct ref_taste {
  float heat;
  int top_count;
  float top_portion;
  float echo_penalty;
  int echo_window;
  uint64_t seed;
} ref_taste;

static app_taste ref_taste_of(const ref_taste *t) {
  app_taste a;
  a.heat_value = t->heat;
  a.top_count = t->top_count;
  a.top_portion = t->top_portion;
  a.echo_penalty = t->echo_penalty;
  a.echo_window = t->echo_window;
  a.seed_value = t->seed;
  return a;
}

int ref_model_load(const char *folder, int threads, int window_limit, app_model **out) {
  app_setup setup = app_setup_plain();
  setup.thread_count = threads;
  setup.window_limit = window_limit;
  return (int)model_load(folder, &setup, out);
}

void ref_model_free(app_model *m) { model_free(m); }
int ref_model_vocab(const app_model *m) { return model_vocab_count(m); }
size_t ref_model_decode_bytes(const app_model *m) { return model_decode_bytes(m); }
int ref_model_window(const app_model *m) { return model_window_limit(m); }

int ref_session_open(app_model *m, app_session **out) { return (int)session_open(m, out); }
void ref_session_close(app_session *s) { session_close(s); }
void ref_session_reset(app_session *s) { session_reset(s); }
int ref_session_fill(const app_session *s) { return session_fill(s); }
int ref_session_hold(app_session *s, int keep) { return (int)session_hold(s, keep); }

int ref_session_prime(app_session *s, const int32_t *ids, int n) {
  return (int)session_prime(s, ids, n);
}

/* session_step: copies the one row of logits, or returns -1 on refusal. */
int ref_session_step(app_session *s, int32_t id, float *logits_out) {
  const float *row = session_step(s, id);
  if (!row) return -1;
  if (logits_out)
    memcpy(logits_out, row, sizeof(float) * (size_t)s->model->head_sheet.row_count);
  return 0;
}

/* session_guess: copies K rows of logits, or returns -1 on refusal. */
int ref_session_guess(app_session *s, const int32_t *ids, int k, float *logits_out) {
  const float *rows = session_guess(s, ids, k);
  if (!rows) return -1;
  if (logits_out)
    memcpy(logits_out, rows, sizeof(float) * (size_t)s->model->head_sheet.row_count * (size_t)k);
  return 0;
}

/* The rows session_guess left in the session, for a caller that asked for
 * none copied but wants to verify from them. */
const float *ref_session_rows(const app_session *s) { return s->logit_room; }

int ref_session_keep(app_session *s, int keep) { return (int)session_guess_keep(s, keep); }

int ref_session_taste(app_session *s, const float *rows, const int32_t *ids, int k,
                      const ref_taste *t, int32_t *made) {
  app_taste a = ref_taste_of(t);
  return session_guess_taste(s, rows, ids, k, &a, made);
}

int32_t ref_session_pick(app_session *s, const float *logits, const ref_taste *t) {
  app_taste a = ref_taste_of(t);
  return session_pick(s, logits, &a);
}

double ref_session_serve_seconds(const app_session *s) { return session_tally(s).serve_seconds; }
size_t ref_session_serve_tokens(const app_session *s) { return session_tally(s).serve_tokens; }

/* model_load with the setup's cache_bits (8: byte caches where the export
 * ships scales, app_core.c:14270-14284). */
int ref_model_load_bits(const char *folder, int threads, int window_limit, int cache_bits, app_model **out) {
  app_setup setup = app_setup_plain();
  setup.thread_count = threads;
  setup.window_limit = window_limit;
  setup.cache_bits = cache_bits;
  return (int)model_load(folder, &setup, out);
}

size_t ref_model_memory_bytes(const app_model *m) { return model_memory_bytes(m); }
float ref_model_cache_scale(const app_model *m, int layer, int value_side) {
  return model_cache_scale(m, layer, value_side);
}
float ref_session_cache_peak(const app_session *s, int layer, int value_side) {
  return session_cache_peak(s, layer, value_side);
}
size_t ref_session_cache_room(const app_session *s) { return session_cache_room(s); }

int ref_session_save(const app_session *s, const char *path, uint64_t stamp, const app_keep_note *note, int kind) {
  return (int)session_save(s, path, stamp, note, kind);
}
int ref_session_load(app_session *s, const char *path, uint64_t *stamp, app_keep_note *note, int *kind) {
  return (int)session_load(s, path, stamp, note, kind);
}
int ref_session_ids(const app_session *s, int32_t *ids, int limit) { return session_ids(s, ids, limit); }
int ref_keep_note_share(const app_keep_note *held, const app_keep_note *now, int same_count) {
  return keep_note_share(held, now, same_count);
}

/* The cache grid's own conversions (app_core.c:10980-11035), over arrays. */
void ref_cache_code8(const float *x, int n, uint8_t *out) {
  int i;
  for (i = 0; i < n; ++i) out[i] = cache_code8(x[i]);
}
void ref_cache_real8(const uint8_t *c, int n, float *out) {
  int i;
  for (i = 0; i < n; ++i) out[i] = cache_real8(c[i]);
}
