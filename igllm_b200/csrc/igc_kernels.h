// igc_kernels.h - host-side launchers of igc_kernels.cu.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "igc_gemv.cuh"

extern "C" {

cudaError_t igc_kernels_configure(int bytes);

cudaError_t igc_launch_repack(const uint8_t *code, size_t row_stride, int bits, const uint16_t *scale, int groups,
                              int rows, int cols, int n_rb, int n_cc, int out_mul, int out_add, uint4 *tiles,
                              uint2 *scales, cudaStream_t st);
// Host: a plane's scales as f16 per 32-column group (see igc_kernels.cu); 0, or
// -1 when a group is not a multiple of 32 columns or a scale is not exact in f16.
int igc_scales_f16(const void *src, int dtype, int rows, int groups, int group_size, int cols, uint16_t *out);

// Launches from the calling thread may overlap the kernel ahead of them
// (programmatic dependent launch) while `on` is set.
void igc_kernels_pdl(int on);
int igc_kernels_pdl_get(void);
// Launches at most `grid` blocks (fewer when the lane mode's wider blocks
// need fewer; the count used goes to *grid_used), picking the weight ring
// within `smem_limit` bytes of shared memory (filling a->piece, a->depth and
// the layout offsets); cudaErrorInvalidValue when the lanes' staging leaves
// no room for it.
cudaError_t igc_launch_gemv(igc::GemvArgs *a, int pair, int pro, int epi, int grid, size_t smem_limit,
                            cudaStream_t st, int *grid_used);
// Shared memory the smallest ring needs.
size_t igc_gemv_smem_min(const igc::GemvArgs *a, int pair);

cudaError_t igc_launch_embed(const int32_t *ids, int lanes, const uint16_t *embed, int hidden, float embed_gain,
                             const uint16_t *ple_embed, int ple_vocab, int ple_width, float ple_gain,
                             float *x_out, float *seed_out, unsigned long long *stamp, int stamp_n,
                             const float *peak, float *peak_saved, int peak_n, const igc::EmbedCodes *embed_q,
                             const igc::EmbedCodes *ple_q, cudaStream_t st);
cudaError_t igc_launch_ple_finish(const float *raw, const float *seed, int lanes, int layers, int ple_dim,
                                  const float *w, float eps, float blend, float *out, cudaStream_t st);
size_t igc_attn_smem(int hd);
// The light layout's (igc_launch_attn_many with `light`): heads of at most 256.
size_t igc_attn_smem_light(int hd);
// Attention for one layer in one kernel (query norm and rope, an owner
// layer's cache writes, scores, softmax and values over 16-position tiles,
// and the merge of the cluster's partials); `cluster` (8 or 16) blocks a
// cluster, a session constant.  `out_amax`, when given, gets each lane's
// largest |out| per (head, cluster block), [heads * cluster][16].  `store`
// (nullable: float sides, no peaks) says which sides of the cache are e4m3
// bytes and where the rows' largest magnitudes go.
cudaError_t igc_launch_attn(const float *qkv, int qkv_stride, int heads, int kv_heads, int hd, const float *q_norm,
                            const float *k_norm, const float *cs, const float *sn, float eps, int owner, float *kc,
                            float *vc, int sliding, int span, const int *d_p0, int lanes, int cluster, float *out,
                            int out_stride, float *out_amax, unsigned long long *stamp, const igc::CacheStore *store,
                            cudaStream_t st, int light = 0);
// The same for `batch` sessions' blocks of `lanes` lanes each in one launch
// (blockIdx.z the session): session z's caches are kc_tab[z] / vc_tab[z],
// its first position pos_tab[z], its rows of q|k|v and of the output follow
// the sessions before it.  `light` asks for the layout with two tiles in
// flight and no room for new rows (two blocks an SM), taken where no new
// rows are written (owner 0), the head is at most 256 wide and clusters are
// of at most 4 blocks; otherwise ignored.
cudaError_t igc_launch_attn_many(const float *qkv, int qkv_stride, int heads, int kv_heads, int hd,
                                 const float *q_norm, const float *k_norm, const float *cs, const float *sn, float eps,
                                 int owner, float *kc, float *vc, int sliding, int span, const int *d_p0, int lanes,
                                 int cluster, float *out, int out_stride, float *out_amax, unsigned long long *stamp,
                                 float *const *kc_tab, float *const *vc_tab, const int *pos_tab, int batch,
                                 const igc::CacheStore *store, cudaStream_t st, int light = 0);
// `stamp_sum`, when given, gets each of the pass's `stamp_n` stamped launches'
// spans added (igc_device.cuh stamp_begin / stamp_end).
cudaError_t igc_launch_argmax(const float *part_val, const int *part_idx, int parts, int lanes, int32_t *top,
                              const unsigned long long *stamp, unsigned long long *stamp_sum, int stamp_n,
                              cudaStream_t st);
cudaError_t igc_launch_rope_table(const float *steps, int half, int window, float *cs, float *sn,
                                  cudaStream_t st);
cudaError_t igc_launch_topk(const float *logits, int vocab, int lanes, int keep, const int32_t *echo_ids,
                            const int *echo_from, const int *echo_upto, float penalty, float *cand_v, int *cand_i,
                            float *top_v, int *top_i, cudaStream_t st);
cudaError_t igc_launch_desk_norm(const float *x, const float *w, int n, float eps, float *out, cudaStream_t st);
cudaError_t igc_launch_desk_softmax(float *x, int n, cudaStream_t st);
cudaError_t igc_launch_desk_gelu(float *gate, const float *rise, int n, cudaStream_t st);
cudaError_t igc_launch_desk_rope(float *x, int head, const float *cs, const float *sn, cudaStream_t st);
}
