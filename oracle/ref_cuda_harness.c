/* ref_cuda_harness.c - the reference engine with its backend table on the GPU
 * (TEST INFRASTRUCTURE).
 *
 * oracle/Makefile compiles this file into oracle/_ref/libref_cuda.so: the
 * reference's own app_core.c (through ref_harness.c, which includes it
 * unchanged) plus the maintainer's shim oracle/app_cuda.c, linked against
 * libigllm_cuda.so.  Every ref_* wrapper of ref_harness.c is exported as
 * before; a model loaded by ref_model_load_cuda runs the reference's own
 * session_pass, layer wiring and sampler, with each of its back_desk products
 * (mat_vec, mat_mat, norm_rms, soft_max, gelu_gate, rope_turn) served by the
 * CUDA table.  Tests compare it with the unmodified reference build.
 */
#include "ref_harness.c"

#include "app_cuda.c"

/* model_load, then the desk pointed at `device`. */
int ref_model_load_cuda(const char *folder, int threads, int window_limit, int device, app_model **out) {
  int code = ref_model_load(folder, threads, window_limit, out);
  if (code != 0) return code;
  code = (int)cuda_take_desk(&(*out)->desk, device);
  if (code != 0) {
    model_free(*out);
    *out = NULL;
  }
  return code;
}

const char *ref_desk_name(const app_model *m) { return m->desk.name_text; }

int ref_cuda_status(void) { return cuda_desk_status(); }

void ref_cuda_close(void) { cuda_drop_desk(); }
