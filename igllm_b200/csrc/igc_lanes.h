// igc_lanes.h - the batched-lane path (igc_lanes.cu): row-wise stages and the
// tcgen05 int4 GEMM for chunks of many lanes.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace igc {

constexpr int LG_M = 128;  // lanes a tile (tensor-memory lanes)
constexpr int LG_N = 128;  // weight rows a tile (tensor-memory columns)
constexpr int LG_A_STEP_BYTES = 2 * 128 * 64 * 2;  // staged activations a (lane tile, 64-column step): hi and lo blocks

// What a stage computes for its lane before staging it (app_core.c:11637-11743).
enum : int {
  LS_PLAIN = 0,       // y = x
  LS_NORM = 1,        // y = norm(x) * w_in
  LS_RESID = 2,       // x_out = (x + norm(p) * w_res) * gain; y = x_out
  LS_RESID_NORM = 3,  // the same, then y = norm(x_out) * w_in
  LS_GELU_PAIR = 4,   // y = gelu(gate) * up, p the pair plane's rows (16-row blocks of gate, then up)
  LS_GELU_MUL = 5     // y = gelu(p) * aux
};

struct LaneStageArgs {
  int mode, lanes, cols;  // cols: the staged row's length (the next product's input columns)
  const float *x;         // [lanes][x_stride]: the input (PLAIN, NORM) or residual stream (RESID*)
  int x_stride;
  const float *p;         // [p_splits][lanes][p_stride]: the producer's K-slice partials
  int p_stride, p_splits;
  const float *w_res;
  float gain;
  const float *w_in;
  float eps;
  float *x_out;           // RESID*: the new residual stream, same layout as x
  const float *aux;       // GELU_MUL: [lanes][aux_stride]
  int aux_stride;
  float out_scale;        // folded into the lane's factor
  void *a_tiles;          // out: [lane tile][n_cc][hi, lo][16 KB] f16 operand blocks (null: none)
  int n_cc;               // 64-column steps of the next product
  float *factor;          // out: [lanes] the factor undoing the staging scale (times out_scale)
  float *row_out;         // out (nullable): [lanes][row_stride] the staged rows as f32, unscaled
  int row_stride;
};

// One product of a plane the tiles do not hold, on the CUDA cores
// (igc_launch_plain_product): offset codes of 1-8 bits packed from the low bit
// (app_core.c:1757 pack_read), a value being (code ^ flip) - bias times the
// f32 scale of its group, or a dense float plane; the input taken through its
// activation grid and the output put through its own (app_core.c:1930
// quant_step, :7814 plane_lift_many).
struct PlainArgs {
  const uint8_t *codes;   // [rows][stride] (null: dense)
  size_t stride;
  int bits;
  uint32_t flip;
  int bias;
  const float *scales;    // [rows][groups]
  int groups, group_size;
  const void *dense;      // [rows][cols] of dense_type: 1 F32, 2 F16, 3 BF16
  int dense_type;
  int rows, cols;
  float enter, leave;     // grid steps of the input and the output (0: none)
  const float *x;         // [lanes][x_stride] the staged input rows
  int x_stride, lanes;
  float *out;             // [lanes][out_stride] at row out_row0 + r, or for pair_half >= 0 the
  int out_stride, out_row0, pair_half;  // 16-row blocks of a gate|up pair (gate 0, up 1)
  float out_scale;        // applied after the output grid
  float cap;              // > 0: the head's soft cap, then argmax partials
  float *arg_val;         // [block][lanes] the largest value of each block's rows, and its row
  int *arg_idx;
  int vec;                // set by the launcher: eight columns a load
};

struct LaneGemmArgs {
  const uint4 *tiles;     // the plane, as the upload repack lays it out
  const uint2 *scales;
  int n_rb, n_cc;
  const uint4 *a_tiles;   // staged activations (LaneStageArgs::a_tiles)
  const float *factor;    // [lanes]
  float *out;             // [split][lanes][out_stride] partial sums, plane row order
  int lanes, out_stride, split;
  int *err;               // set nonzero when a wait gave up
  // the output head's epilogue (split 1): each value times the lane's factor
  // and soft-capped (`cap` > 0), the largest of the tile's first `rows` rows
  // per lane (first index on a tie) to arg_val / arg_idx [tile][lanes], and
  // the capped values to `out` only when it is not null
  float *arg_val;
  int *arg_idx;
  int rows;
  float cap;
};

// A byte cache's rows decoded into float rows (igc_launch_lane_widen): one
// session by pointers, or block row z's session by the tables.
struct WidenArgs {
  const uint8_t *kc, *vc;  // the byte caches (a side whose scale is 0 is not read)
  float *kf, *vf;          // the float rows, the same layout
  const int *p0;           // the pass's first position
  float *const *kc_tab, *const *vc_tab, *const *kf_tab, *const *vf_tab;
  const int *pos_tab;
  float kq, vq;            // the sides' scales, 0 for a float side
  int kv_w, lanes, sliding, span;
};

}  // namespace igc

extern "C" {
// Lets the stage and GEMM kernels take their shared memory (once per device).
cudaError_t igc_lanes_configure(void);
size_t igc_lane_stage_smem(int mode, int cols);
cudaError_t igc_launch_lane_stage(const igc::LaneStageArgs *a, cudaStream_t st);
// K slices that keep about one wave of the SMs busy for this product.
int igc_lane_gemm_split(int lanes, int n_rb, int n_cc, int sm_count);
// The two tensor maps a plane's lane GEMMs load its weights through (3-D,
// 32-bit elements): the code tiles [row block][step][128 words] and the scale
// records [row block][step][16 words], each read 8 row blocks of one step at
// a time.  Host only (the driver's encoder); 0 on success.
int igc_lane_tmaps(const void *tiles, const void *scales, int n_rb, int n_cc, CUtensorMap *codes_map,
                   CUtensorMap *scales_map);
cudaError_t igc_launch_lane_gemm(const igc::LaneGemmArgs *a, const CUtensorMap *codes_map,
                                 const CUtensorMap *scales_map, cudaStream_t st);
// A pass's `lanes` new key and value rows (normed; keys turned) into an
// owner layer's caches at positions *p0 + lane; `store` (nullable) says which
// sides are e4m3 bytes and where the rows' peaks go.
cudaError_t igc_launch_lane_kv(const float *qkv, int qkv_stride, int heads, int kv_heads, int hd, const float *k_norm,
                               const float *cs, const float *sn, float eps, const int *p0, int lanes, float *kc,
                               float *vc, const igc::CacheStore *store, cudaStream_t st);
// The same for many sessions' blocks of `per` lanes: lane j is session
// j / per's lane j % per, at pos_tab[j / per] + j % per, into that session's
// caches kc_tab / vc_tab and peaks peak_tab (nullable).
cudaError_t igc_launch_lane_kv_many(const float *qkv, int qkv_stride, int heads, int kv_heads, int hd,
                                    const float *k_norm, const float *cs, const float *sn, float eps, const int *p0,
                                    int lanes, float *kc, float *vc, const igc::CacheStore *store, const int *pos_tab,
                                    float *const *kc_tab, float *const *vc_tab, float *const *peak_tab, int per,
                                    cudaStream_t st);
// Byte cache rows decoded into float rows for the attention kernel: for each
// of `batch` sessions (tables) or one (pointers), rows [lo, p0 + lanes) of
// each byte side (lo = p0 - span + 1 on a sliding layer, clipped at 0; 0 on
// a global one).  `rows_most` bounds the rows any launch of this shape sees
// (it sizes the grid); kv_w, a row's values, is a multiple of 16.
cudaError_t igc_launch_lane_widen(const igc::WidenArgs *w, int batch, int rows_most, int sm_count, cudaStream_t st);
// A plain plane's product for `lanes` lanes, one block of 8 warps a
// igc_plain_blocks(rows)'th of the rows (with the head's cap, as many argmax
// partials a lane).  Returns the blocks launched in *blocks_out when it is
// not null.
cudaError_t igc_launch_plain_product(const igc::PlainArgs *a, int sm_count, int *blocks_out, cudaStream_t st);
int igc_plain_blocks(int rows);
// out[i] = *p0 + 16 i for i < groups (a prefill chunk's attention groups).
cudaError_t igc_launch_lane_positions(const int *p0, int groups, int *out, cudaStream_t st);
// Per lane the largest of `parts` argmax partials [part][lanes] (first index
// on a tie), into top[lanes].
cudaError_t igc_launch_lane_argmax(const float *val, const int *idx, int parts, int lanes, int32_t *top,
                                   cudaStream_t st);
cudaError_t igc_launch_lane_sum(const float *p, int splits, int lanes, int cols, int p_stride, float *out,
                                int out_stride, cudaStream_t st);
}
