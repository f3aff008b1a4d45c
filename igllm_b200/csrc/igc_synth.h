/* igc_synth.h - seeded synthetic checkpoints for the verify-round benchmark.
 *
 * The reference measures on its shipped QAT export, which is not available
 * here; the benchmark configuration instead fixes shapes and value
 * distributions (int4 codes uniform in [-8,7], group 32, f16 scales
 * |N(0,0.02)|, bf16 norms and embeddings N(0,0.02)).  Values are a pure
 * function of (seed, tensor name, element index): a splitmix64 counter hash
 * picks either two uniform nibbles or one of 65536 equiprobable normal
 * quantiles, so a file written for the CPU engine and weights generated
 * straight into HBM hold the same bits.
 */
#ifndef IGC_SYNTH_H
#define IGC_SYNTH_H

#include <stddef.h>
#include <stdint.h>

#include "../../include/igllm_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

#define IGC_SYNTH_CODE 0   /* packed int4 bytes */
#define IGC_SYNTH_SCALE 1  /* f16 |N(0,0.02)| */
#define IGC_SYNTH_NORMAL 2 /* bf16 N(0,0.02) */
#define IGC_SYNTH_OFFSET 3 /* bf16 offset + N(0,0.02) */
#define IGC_SYNTH_CONST 4  /* f32, every value the offset */
#define IGC_SYNTH_SCALE_BF16 5 /* bf16 |N(0,0.02)|, raised to 2^-14 where smaller */

/* One tensor of a synthetic checkpoint, in the layout the reference binds
 * (app_core.c:7886 plane_bind_gemma for U8 codes with F16 scales). */
typedef struct igc_synth_tensor {
  char name[128];
  int dtype;         /* 1 F32, 2 F16, 3 BF16, 6 U8 (app_core.c:1412 store_type) */
  int rank;
  int64_t shape[2];
  int kind;          /* IGC_SYNTH_* */
  float offset;
  size_t bytes;
} igc_synth_tensor;

/* Every tensor of the spec, in file order; returns the count (room may be
 * NULL to count only). */
int igc_synth_list(const igc_synth_spec *spec, igc_synth_tensor *room, int room_count);
/* The config.json text for the spec (caller frees with free()). */
char *igc_synth_config_text(const igc_synth_spec *spec);
/* Stream id of a tensor name (FNV-1a). */
uint64_t igc_synth_stream(const char *name);
/* Fill one tensor's bytes. */
int igc_synth_tensor_fill(const igc_synth_spec *spec, const igc_synth_tensor *t, void *out,
                          int threads);
/* Write config.json, tokenizer.json and model.safetensors under `folder`. */
int igc_synth_write(const igc_synth_spec *spec, const char *folder, int threads);

#ifdef __cplusplus
}
#endif
#endif
