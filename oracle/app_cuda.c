/* app_cuda.c - the reference engine's backend table pointed at libigllm_cuda
 * (the shim a maintainer of the reference adds; TEST INFRASTRUCTURE here).
 *
 * The reference reaches every heavy product through model->desk, a back_desk
 * of six function pointers (app_core.c:5222-5245) that back_open fills
 * (app_core.c:5415, called from model_load at app_core.c:12585).  This file
 * adds a CUDA table beside it: each entry copies the reference's `plane`
 * into the C ABI's igc_plane (the same fields with plain types) and calls the
 * matching entry of igc_desk (include/igllm_cuda.h).  It is compiled after
 * app_core.c in one translation unit, so `plane`, `back_desk` and
 * `app_code` are the reference's own types.
 *
 * Use: after model_load succeeds, call cuda_take_desk(&model->desk, device);
 * call cuda_drop_desk() beside model_free.
 */
#include "igllm_cuda.h"

static igc_desk cuda_table;
static int cuda_open = 0;

static void cuda_sheet(const plane *from, igc_plane *to) {
  to->form = (int)from->form;
  to->row_count = from->row_count;
  to->col_count = from->col_count;
  to->real_data = from->real_data;
  to->real_type = (int)from->real_type;
  to->code_data = from->code_data;
  to->row_stride = from->row_stride;
  to->gain_data = from->gain_data;
  to->gain_type = (int)from->gain_type;
  to->bias_data = from->bias_data;
  to->bit_count = from->bit_count;
  to->code_bias = from->code_bias;
  to->code_flip = from->code_flip;
  to->group_size = from->group_size;
  to->group_count = from->group_count;
  to->enter_gain = from->enter_gain;
  to->leave_gain = from->leave_gain;
}

static void cuda_mat_vec(back_desk *desk, const plane *sheet, const float *act_data, float *out_data) {
  igc_plane p;
  (void)desk;
  cuda_sheet(sheet, &p);
  cuda_table.mat_vec(&cuda_table, &p, act_data, out_data);
}

static void cuda_mat_mat(back_desk *desk, const plane *sheet, const float *act_data, int act_stride,
                         int lane_count, float *out_data, int out_stride) {
  igc_plane p;
  (void)desk;
  cuda_sheet(sheet, &p);
  cuda_table.mat_mat(&cuda_table, &p, act_data, act_stride, lane_count, out_data, out_stride);
}

static void cuda_norm_rms(back_desk *desk, const float *value_list, const float *gain_list, int value_count,
                          float eps_value, float *value_out) {
  (void)desk;
  cuda_table.norm_rms(&cuda_table, value_list, gain_list, value_count, eps_value, value_out);
}

static void cuda_soft_max(back_desk *desk, float *value_list, int value_count) {
  (void)desk;
  cuda_table.soft_max(&cuda_table, value_list, value_count);
}

static void cuda_gelu_gate(back_desk *desk, float *gate_list, const float *rise_list, int value_count) {
  (void)desk;
  cuda_table.gelu_gate(&cuda_table, gate_list, rise_list, value_count);
}

static void cuda_rope_turn(back_desk *desk, float *value_list, int head_size, const float *cos_list,
                           const float *sin_list) {
  (void)desk;
  cuda_table.rope_turn(&cuda_table, value_list, head_size, cos_list, sin_list);
}

/* Points an opened back_desk at the GPU.  The reference's own CPU state in
 * the desk (its pool, its staging rooms) stays as back_open left it, unused. */
static app_code cuda_take_desk(back_desk *desk, int device) {
  if (!cuda_open) {
    if (igc_back_open(&cuda_table, device) != IGC_OKAY) return APP_FAIL_SUPPORT;
    cuda_open = 1;
  }
  desk->name_text = cuda_table.name_text;
  desk->mat_vec = cuda_mat_vec;
  desk->mat_mat = cuda_mat_mat;
  desk->norm_rms = cuda_norm_rms;
  desk->soft_max = cuda_soft_max;
  desk->gelu_gate = cuda_gelu_gate;
  desk->rope_turn = cuda_rope_turn;
  return APP_OKAY;
}

/* The first failure any CUDA entry met since the last call (0 when none). */
static int cuda_desk_status(void) { return cuda_open ? igc_desk_status(&cuda_table) : 0; }

static void cuda_drop_desk(void) {
  if (cuda_open) igc_back_close(&cuda_table);
  cuda_open = 0;
}
