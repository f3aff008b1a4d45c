/* igllm_cuda.h - libigllm_cuda: the B200 backend for the speculative verify
 * round of the Gemma-4-E2B text stack (iamhaymc/igllm, "INFERGEM").
 *
 * A plain C ABI: no C++ types, no device pointers cross it.  Every entry that
 * has a counterpart in the reference engine names it (file:line in the
 * reference's app_core.c / app_main.c) and keeps its argument meaning and its
 * error behaviour: results are the reference's app_code values, zero for
 * success and negative for failure, and a refused call leaves the session as
 * it was.
 *
 * Two layers are exported.
 *
 *  1. The backend table (`igc_desk`), the device twin of the reference's
 *     `back_desk` (app_core.c:5222-5245): the six entries the engine reaches
 *     through `model->desk.X`, with host pointers in and out, synchronous.  A
 *     reference build binds it where it calls `back_open` (app_core.c:5415).
 *  2. The session layer, the device twin of the reference's public API
 *     (app_core.c:158-425): model load, session open/prime/step, the guess
 *     block, its keep and its tempered verify.  The whole pass runs on the
 *     GPU with the weights resident in HBM; only ids go in and only ids (or,
 *     on request, logit rows) come out.
 *
 * Threading: one caller at a time per session (the reference's rule,
 * app_core.c:7789-7793).  Separate sessions, and separate models on separate
 * devices, may be driven from separate threads.
 */
#ifndef IGLLM_CUDA_H
#define IGLLM_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* app_core.c:40-49 app_code, plus one code the CPU engine never needed. */
#define IGC_OKAY 0
#define IGC_FAIL_ARGUMENT (-1)
#define IGC_FAIL_MEMORY (-2)
#define IGC_FAIL_FILE (-3)
#define IGC_FAIL_FORMAT (-4)
#define IGC_FAIL_MISSING (-5)
#define IGC_FAIL_SUPPORT (-6)
#define IGC_FAIL_STATE (-7)
#define IGC_FAIL_DEVICE (-8) /* a CUDA call failed; igc_last_error() says which */

#define IGC_LANE_LIMIT 16 /* app_core.c:1980 KERN_LANE_LIMIT */

/* app_core.c:52-57 app_setup.  `thread_count` becomes the device ordinal:
 * intra-op parallelism is the GPU's, and a process picks its GPU here.
 * `window_limit` is the context length (0 keeps the checkpoint's
 * max_position_embeddings, capped at 32768 so a default session stays a few
 * hundred MB of HBM). */
typedef struct igc_setup {
  int device;
  int window_limit;
  int verbose_level;
  int cache_bits; /* 8 stores a cache side as e4m3 bytes where the export ships
                    its scale (app_core.c:14270-14284); anything else keeps floats */
} igc_setup;

/* app_core.c:60-67 app_taste, field for field. */
typedef struct igc_taste {
  float heat_value;
  int top_count;
  float top_portion;
  float echo_penalty;
  int echo_window;
  uint64_t seed_value;
} igc_taste;

/* A weight matrix as the reference's `plane` describes it (app_core.c:1775-1797),
 * restated with plain types so the reference can hand one across without
 * this library seeing its struct.  `form` is 1 for a dense matrix (real_data
 * of real_type) and 2 for a packed code plane.  Type codes are the
 * reference's store_type values (app_core.c:1412): 1 F32, 2 F16, 3 BF16. */
typedef struct igc_plane {
  int form;
  int row_count;
  int col_count;
  const void *real_data;
  int real_type;
  const uint8_t *code_data;
  size_t row_stride;
  const void *gain_data;
  int gain_type;
  const int8_t *bias_data;
  int bit_count;
  int code_bias;
  int code_flip;
  int group_size;
  int group_count;
  float enter_gain;
  float leave_gain;
} igc_plane;

/* ---- 1. the backend table (app_core.c:5222-5245 back_desk) ------------- */

typedef struct igc_desk igc_desk;
struct igc_desk {
  const char *name_text; /* "cuda/sm_100a" */
  void *state;           /* the device, its stream, uploaded planes */
  void (*mat_vec)(igc_desk *desk, const igc_plane *sheet, const float *act_data, float *out_data);
  void (*mat_mat)(igc_desk *desk, const igc_plane *sheet, const float *act_data, int act_stride,
                  int lane_count, float *out_data, int out_stride);
  void (*norm_rms)(igc_desk *desk, const float *value_list, const float *gain_list,
                   int value_count, float eps_value, float *value_out);
  void (*soft_max)(igc_desk *desk, float *value_list, int value_count);
  void (*gelu_gate)(igc_desk *desk, float *gate_list, const float *rise_list, int value_count);
  void (*rope_turn)(igc_desk *desk, float *value_list, int head_size, const float *cos_list,
                    const float *sin_list);
};

/* Replaces app_core.c:5415 back_open.  Each code plane is uploaded to HBM the
 * first time a product names it (keyed by its code pointer) and stays there
 * until igc_back_close.  Codes of 1, 2 or 4 bits with groups of 32k columns
 * and f16-exact gains go to the int4 tiles; other code planes (8-bit, signed
 * through their flip, any group) and dense planes stay as stored for a
 * CUDA-core product.  A plane with zero points makes the entry return
 * without writing and set igc_desk_status to IGC_FAIL_SUPPORT. */
int igc_back_open(igc_desk *desk, int device);
/* Replaces app_core.c:5445 back_close. */
void igc_back_close(igc_desk *desk);
/* The first failure any entry of this desk met since the last call, then 0. */
int igc_desk_status(igc_desk *desk);

/* ---- 2. the session layer ----------------------------------------------- */

typedef struct igc_model igc_model;
typedef struct igc_session igc_session;

/* app_core.c:12439 model_load: config.json + model.safetensors (or a sharded
 * index) from `folder`, every bound plane uploaded once to HBM. */
int igc_model_load(const char *folder, const igc_setup *setup, igc_model **model_out);
/* app_core.c:12602 model_free */
void igc_model_free(igc_model *model);
int igc_model_vocab_count(const igc_model *model);  /* app_core.c:12664 */
int igc_model_layer_count(const igc_model *model);  /* app_core.c:12663 */
int igc_model_state_size(const igc_model *model);   /* app_core.c:12666 */
int igc_model_window_limit(const igc_model *model); /* app_core.c:12665 */
/* app_core.c:12747 model_decode_bytes: the bytes one decode step reads by the
 * reference's rule, counted on this library's own bound planes. */
size_t igc_model_decode_bytes(const igc_model *model);
/* Device bytes the model holds (weights as uploaded, packed). */
size_t igc_model_device_bytes(const igc_model *model);
/* Weights of the int4 projections one lane multiplies, head included (no
 * counterpart in the reference): a lane's FLOPs are twice this. */
size_t igc_model_weight_count(const igc_model *model);

/* app_core.c:14219 session_open / :14368 session_close / :14375 session_reset */
int igc_session_open(igc_model *model, igc_session **session_out);
void igc_session_close(igc_session *session);
void igc_session_reset(igc_session *session);
/* app_core.c:13935 session_hold.  Caches are full length, so no ring turns
 * over and the reference's IGC_FAIL_SUPPORT refusal does not arise from one;
 * it does arise after igc_session_load of a file written from a ring that had
 * turned over, for a keep_count whose sliding window reaches rows the file
 * did not carry. */
int igc_session_hold(igc_session *session, int keep_count);
/* app_core.c:14443 session_prime: every id but the last, 16 lanes a pass. */
int igc_session_prime(igc_session *session, const int32_t *id_list, int id_count);
/* app_core.c:14473 session_step.  The reference returns a pointer to the
 * logit row; here the row is copied to `logits_out` when it is not NULL and
 * its argmax (app_main.c:482 main_guess_top) to `top_out` when that is not
 * NULL.  IGC_FAIL_STATE while a block is in flight. */
int igc_session_step(igc_session *session, int32_t id_value, float *logits_out, int32_t *top_out);
/* app_core.c:12139 session_guess: `id_count` (1..16) lanes in one pass, one
 * row of logits a lane kept on the device; copied to `logits_out`
 * (id_count x vocab floats) when it is not NULL.  Refused (IGC_FAIL_STATE)
 * while a block is already in flight. */
int igc_session_guess(igc_session *session, const int32_t *id_list, int id_count,
                      float *logits_out);
/* The argmax of each row of the block in flight (app_main.c:482, first index
 * on a tie), id_count ids into `top_out`. */
int igc_session_guess_top(igc_session *session, int32_t *top_out);
/* app_core.c:12205 session_guess_keep */
int igc_session_guess_keep(igc_session *session, int keep_count);
/* app_core.c:14762 session_guess_taste on the rows of the block in flight
 * (the reference takes them as `row_list`; here they never leave the GPU).
 * Returns the guesses kept and writes the following token to `made_out`;
 * -1 when refused (greedy taste, no block, count mismatch). */
int igc_session_guess_taste(igc_session *session, const int32_t *id_list, int id_count,
                            const igc_taste *taste, int32_t *made_out);
/* app_core.c:14844 session_pick on the row the last step produced. */
int32_t igc_session_pick(igc_session *session, const igc_taste *taste);
int igc_session_fill(const igc_session *session);        /* app_core.c:14513 */
int igc_session_guess_span(const igc_session *session);  /* app_core.c:12364 */
int igc_session_guess_limit(const igc_session *session); /* app_core.c:12368 */

/* One whole verify round, the body of app_main.c:520 main_answer_guess's
 * loop after the scout has drawn: guess the block, verify it (argmax
 * comparison at heat 0, the rejection rule above it), keep the accepted
 * lanes and the token after them.  Writes the kept guess count to
 * `take_out` and the token after them to `made_out`, and returns
 * take + 1, the tokens committed; negative on refusal. */
int igc_session_round(igc_session *session, const int32_t *id_list, int id_count,
                      const igc_taste *taste, int32_t *take_out, int32_t *made_out);

/* Wall-clock seconds and committed tokens of the passes this session ran as
 * steps and blocks (app_core.c:70-77 app_tally serve_seconds/serve_tokens). */
double igc_session_serve_seconds(const igc_session *session);
size_t igc_session_serve_tokens(const igc_session *session);

/* ---- cache files and the cache's storage (app_core.c:320-425) -----------
 *
 * igc_session_save / igc_session_load write and read the reference's cache
 * file (app_core.c:14010 session_save, :14076 session_load, layout "igllm
 * cache 4"): the ids the session holds and the rows of its caches that carry
 * anything, float or e4m3 bytes as the session stores them, in the order the
 * reference's rings hold them.  A file written by either engine loads into
 * the other for the same checkpoint, window and cache_bits; one written for
 * other shapes is refused with IGC_FAIL_STATE, a damaged one with
 * IGC_FAIL_FORMAT (the session is then left cleared).  `stamp_value`, the
 * note and `kind_mark` are the caller's, written beside the cache and handed
 * back unread.  Refused with IGC_FAIL_STATE while a block is in flight.
 *
 * igc_session_ids: the ids the session holds (app_core.c:14183); returns
 * their count, and copies them only when `id_limit` has room.
 *
 * igc_keep_note_share: app_core.c:13991 keep_note_share, how much of
 * `same_count` shared ids the two notes' runs leave reusable.
 *
 * igc_model_cache_scale / igc_session_cache_peak: a layer's calibrated range
 * (0 when the export ships none) and the largest magnitude the session has
 * written to that cache side (app_core.c:14515, :14540).
 * igc_session_cache_room(_at): bytes this session's caches occupy (at
 * `cache_bits` storage); every owner layer is held full length here, so the
 * figure exceeds the reference's rings (app_core.c:14522).
 * igc_model_memory_bytes: app_core.c:12667 model_memory_bytes, the bytes of
 * the checkpoint's tensors the text stack binds. */
#define IGC_KEEP_PROMPT 0 /* app_core.c:367 */
#define IGC_KEEP_TALK 1   /* app_core.c:368 */
#define IGC_KEEP_RUNS 16  /* app_core.c:385 */
typedef struct igc_keep_note { /* app_core.c:387-392 app_keep_note */
  int run_count;
  int32_t from_list[IGC_KEEP_RUNS];
  int32_t till_list[IGC_KEEP_RUNS];
  uint64_t mark_list[IGC_KEEP_RUNS];
} igc_keep_note;
int igc_session_save(const igc_session *session, const char *path_text, uint64_t stamp_value,
                     const igc_keep_note *note_in, int kind_mark);
int igc_session_load(igc_session *session, const char *path_text, uint64_t *stamp_out, igc_keep_note *note_out,
                     int *kind_out);
int igc_session_ids(const igc_session *session, int32_t *id_list, int id_limit);
int igc_keep_note_share(const igc_keep_note *held, const igc_keep_note *now, int same_count);
float igc_model_cache_scale(const igc_model *model, int layer_index, int value_side);
float igc_session_cache_peak(const igc_session *session, int layer_index, int value_side);
size_t igc_session_cache_room(const igc_session *session);
size_t igc_session_cache_room_at(const igc_session *session, int cache_bits);
size_t igc_model_memory_bytes(const igc_model *model);

/* ---- the crowd: many sessions' blocks in one pass (no counterpart in the
 * reference, which serialises sessions, app_core.c:7789-7793 and
 * TODO.md:126-132) --------------------------------------------------------
 *
 * igc_crowd_open: room for rounds of up to `session_limit` sessions of one
 * model, each verifying a block of `lanes_per_session` ids (1..16); at most
 * IGC_CROWD_LANE_LIMIT lanes in all.
 *
 * igc_crowd_round: one greedy verify round for `count` sessions at once:
 * session j's block is ids[j*k .. j*k+k) at its own position.  The lanes of
 * all blocks share one weight sweep per projection (the tcgen05 lane GEMM),
 * attention runs for every session in one launch per layer, and each
 * session keeps its leading matches exactly as igc_session_round does:
 * take_out[j] the guesses kept, made_out[j] the id after them, fill advanced
 * by take + 1.  `logits_out`, when not NULL, gets every lane's soft-capped
 * logits (count*k x vocab floats).  Returns the ids committed in all, or a
 * negative app_code (a session with a block in flight, a full window, a
 * session named twice or another model's session are refused before
 * anything runs).  A session's results do not depend on how many sessions
 * share its round. */
#define IGC_CROWD_LANE_LIMIT 512
typedef struct igc_crowd igc_crowd;
int igc_crowd_open(igc_model *model, int session_limit, int lanes_per_session, igc_crowd **crowd_out);
void igc_crowd_close(igc_crowd *crowd);
int igc_crowd_round(igc_crowd *crowd, igc_session **sessions, int count, const int32_t *id_list, int32_t *take_out,
                    int32_t *made_out, float *logits_out);

/* ---- measurement (no counterpart in the reference) ----------------------
 *
 * igc_session_bench: `rounds` verify passes of `k` lanes whose blocks are all
 * uploaded to HBM first; round r runs blocks[r*k .. r*k+k) at the session's
 * fill plus r*k - the always-right proposer of the reference's guess bracket
 * (app_main.c:1235 main_guess_run, MAIN_GUESS_ORACLE) - with no host round
 * trip between rounds.  `device_ms` gets the CUDA-event time of the rounds,
 * `last_top` the last round's argmax ids (k of them); the rounds are kept.
 *
 * igc_session_profile: one kept pass of `k` lanes with a CUDA event before
 * every launch; per launch its class (0 a layer projection, 1 the output
 * head, 2 attention, 3 the rest), the weight bytes it streams and its device
 * time.  Returns the number of launches written (at most `capacity`).
 *
 * igc_session_stamps: the launch stamps every pass with a head leaves, read
 * from the graphed passes themselves (no events between launches).  Each
 * projection and attention launch records when its first block got past its
 * wait on the kernel ahead and when its last block finished; the pass's last
 * kernel adds that span to the launch's total.  For each stamped launch of
 * the `k`-lane pass: its class (as above), its weight bytes and its total in
 * ns over every pass with a head since the last reset.  Read them after
 * passes of one lane count only.  With `reset` the totals start over after
 * the read.  Returns the number of launches written. */
#define IGC_STAMP_LIMIT 512
int igc_session_bench(igc_session *session, const int32_t *blocks, int rounds, int k, float *device_ms,
                      int32_t *last_top);
int igc_session_profile(igc_session *session, const int32_t *ids, int k, int *cls_out, double *bytes_out,
                        float *ms_out, int capacity);
int igc_session_stamps(igc_session *session, int k, int *cls_out, double *bytes_out, double *ns_out, int capacity,
                       int reset);

/* ---- normalisation with no allocation (no counterpart in the reference) --
 *
 * igc_norm_rms_fixed: the desk's norm_rms (app_core.c:4667 kern_norm_rms,
 * host pointers in and out, synchronous) for callers that must not allocate:
 * a token loop that promised to allocate nothing once running, or a caller
 * holding no desk.  The input, gain and output live in one fixed array of the
 * library's device image (3 x IGC_FIXED_NORM_LIMIT floats, 768 KiB a device);
 * the call makes no allocating CUDA or library call.  The array's address is
 * looked up on the first call on each device, with that device current; make
 * that first call before any stream capture starts.  That first call may also
 * be the one that creates the device's context or loads the library's device
 * image (CUDA loads modules lazily), which the driver allocates for; the
 * no-allocation guarantee holds from the second call on a device.  The looked
 * up address is kept for the life of the process: a caller that resets the
 * device (cudaDeviceReset) or tears its primary context down must not call
 * this entry on that device again.  `device` is made current
 * for the call and the caller's device restored after it.  `gain_list` may be
 * NULL (no gain).  Vectors longer than IGC_FIXED_NORM_LIMIT, or a device at or
 * beyond IGC_FIXED_DEVICE_LIMIT, are refused with IGC_FAIL_ARGUMENT and nothing
 * is copied.  Nothing in the array needs to start at zero.  Calls on one
 * device share the array: calls that overlap in time on the same device race,
 * so callers serialise them. */
#define IGC_FIXED_NORM_LIMIT 65536
#define IGC_FIXED_DEVICE_LIMIT 64
int igc_norm_rms_fixed(int device, const float *value_list, const float *gain_list, int value_count,
                       float eps_value, float *value_out);

/* ---- n-gram scout (app_core.c:12277-12361), host C --------------------- */

typedef struct igc_scout igc_scout;
int igc_scout_open(igc_scout **scout_out);
void igc_scout_close(igc_scout *scout);
void igc_scout_clear(igc_scout *scout);
int igc_scout_note(igc_scout *scout, const int32_t *id_list, int id_count);
int igc_scout_span(const igc_scout *scout);
int igc_scout_draw(const igc_scout *scout, int32_t *id_out, int want_count);

/* ---- synthetic checkpoints (no counterpart in the reference) ------------
 *
 * Seeded weights of a stated shape, generated by a counter-based hash so the
 * same value lands at the same index whether it is written to a safetensors
 * file for the CPU engine or generated straight into HBM. */
typedef struct igc_synth_spec {
  int vocab, hidden, layers, heads, kv_heads, head_dim, inner, ple_dim;
  int slide_span, share_count, global_every; /* global layer when (l+1) % every == 0, last forced */
  int window_limit;
  float norm_offset;   /* 0: norms N(0,0.02); 1: norms 1+N(0,0.02) */
  int with_layer_scalar; /* write layer_scalar = 1+N(0,0.02); 0 leaves it out (gain 1) */
  uint64_t seed;
  /* > 0: write each owner layer's self_attn.k_cache_scale / v_cache_scale as
   * an F32 scalar, this value times (1 + (layer mod 4) / 8); 0 writes none */
  float cache_scale_k, cache_scale_v;
  /* 1: the layers that share another's cache get a feed-forward twice
   * `inner` wide (use_double_wide_mlp); 0: every layer `inner` */
  int double_wide;
  /* > 0: global layers' head width (global_head_dim); 0: head_dim */
  int global_head_dim;
  /* the export's stored forms (0 keeps the benchmark's): the sharing layers'
   * feed-forward codes `late_mlp_bits` wide (2 or 4); a scale every `group`
   * columns (a multiple of 32; 0: 32), BF16 when `bf16_scales`; the embedding
   * tables quantized to `embed_bits` / `ple_embed_bits` (2 or 4; 0: bf16
   * rows); no lm_head when `tied_head` (the quantized embedding is the head) */
  int late_mlp_bits, group, bf16_scales, embed_bits, ple_embed_bits, tied_head;
  /* the forms the 4-bit tiles do not hold (a model with any of them runs its
   * projections as stored on the CUDA cores): the per-layer input gate and
   * projection as signed 8-bit codes with a scale a row (`ple_bits8`), the
   * per-layer model projection left dense bf16 (`dense_ple_lift`), and every
   * projection's activation grids, input and output steps `grid_in` /
   * `grid_out` times 1, 1.25, 1.5 or 1.75 by plane (0: none) */
  int ple_bits8, dense_ple_lift;
  float grid_in, grid_out;
} igc_synth_spec;

/* Fill `out` with `count` values of stream `stream` of the spec's seed.
 * kind 0: packed int4 bytes (two uniform codes a byte, low nibble first);
 * kind 1: f16 |N(0,0.02)| bits; kind 2: bf16 N(0,0.02) bits;
 * kind 3: bf16 offset + N(0,0.02) bits (offset = norm_offset);
 * kind 4: f32, every value `offset`; kind 5: bf16 |N(0,0.02)| bits, raised
 * to 2^-14 where smaller (scales f16 holds exactly). */
int igc_synth_fill(uint64_t seed, uint64_t stream, int kind, float offset, size_t count, void *out,
                   int threads);
/* Write config.json, tokenizer.json and model.safetensors for the spec under
 * `folder` (which must exist), readable by the reference's model_load. */
int igc_synth_write(const igc_synth_spec *spec, const char *folder, int threads);
/* Build a model of that spec directly in HBM, no file in between. */
int igc_model_synth(const igc_synth_spec *spec, const igc_setup *setup, igc_model **model_out);

/* The message of the last CUDA failure on this thread ("" when none). */
const char *igc_last_error(void);
/* Kernels this library launched on this thread since the last call, then 0. */
long igc_launch_count(void);

#ifdef __cplusplus
}
#endif
#endif /* IGLLM_CUDA_H */
