// igc_gemv.cuh - the K-lane int4 skinny GEMM and its fused prologues and
// epilogues.
//
// Every projection of the verify round (q/k/v, o, gate/up, down, the
// per-layer-embedding gate and projection, the per-layer model projection
// and the 262144-row output head) is out[lane][row] = sum_g s[row][g] *
// sum_{c in g} (code[row][c] - 8) * act[lane][c] for K <= 16 lanes
// (app_core.c:3688 kern_row_code, :4075 kern_row_code_many, :5247
// back_mat_mat).  The weights are streamed once from HBM; the lanes ride
// along as the N dimension of m16n8k16 tensor-core products, so adding lanes
// adds almost nothing until the sweep stops being memory bound.
//
// Precision: a weight code minus eight is an exact f16 integer, so the only
// rounding before the f32 accumulator is the activation's.  Each activation
// is staged as two f16 values, hi = f16(a) and lo = f16(a - hi), and both go
// through the tensor core against the same dequantised weights: the product
// carries about 22 significant bits of the activation, against the
// reference's 24, at the cost of a second MMA per 16 columns.
//
// Layout in HBM (written once by the upload repack, igc_repack_kernel):
//   tiles  : [row_block][chunk][32 threads] uint4 - one 16-row x 64-column
//            tile is 512 contiguous bytes; thread t's 16 bytes are exactly the
//            A fragments of the four 16-column products it takes part in.
//   scales : [row_block][chunk][8] uint2 - for the thread group g = lane/4,
//            the f16 scales of rows g and g+8 for the chunk's two groups.
// Row blocks are 16 rows; chunks are 64 columns (two groups of 32).
#pragma once

#include "igc_device.cuh"

namespace igc {

enum : int { PRO_F32 = 0, PRO_NORM = 1, PRO_RESID = 2, PRO_RESID_NORM = 3 };
enum : int { EPI_STORE = 0, EPI_GELU_PAIR = 1, EPI_GELU_MUL = 2, EPI_LOGITS = 3 };

struct GemvPlane {
  const uint4 *tiles;
  const uint2 *scales;
  int n_rb;   // row blocks in the plane (pairs count two)
  int n_cc;   // 64-column chunks
  int rows;   // valid output rows (per half for a pair plane)
  int cols;   // valid input columns
};

struct GemvArgs {
  GemvPlane pl;
  int lanes;
  int split;  // warps that share one row block's chunks (1, 2, 4 or 8)
  // prologue
  const float *x;
  int x_stride;
  const float *p;
  int p_stride;
  const float *w_res;
  float gain;
  const float *w_in;
  float eps;
  float *x_out;
  // epilogue
  float *out;
  int out_stride;
  float out_scale;
  const float *aux;
  int aux_stride;
  float cap;
  float *part_val;  // EPI_LOGITS argmax partials [gridDim.x][16]
  int *part_idx;
};

constexpr int GEMV_THREADS = 256;
constexpr int GEMV_WARPS = GEMV_THREADS / 32;

// Staged activations: for chunk cc, lane tile nt and thread slot s, 16
// consecutive u32 words - the hi B fragments of the chunk's four 16-column
// products (b0, b1 each) and then the lo ones.  Word of (lane n, column c):
__device__ __forceinline__ int stage_word(int n, int c, int NT) {
  int cc = c >> 6, kb = (c >> 4) & 3, k = c & 15;
  int nt = n >> 3, g = n & 7, t = (k & 7) >> 1;
  return (((cc * NT + nt) * 32 + g * 4 + t) * 16) + kb * 2 + (k >> 3);
}

__host__ __device__ inline size_t gemv_stage_bytes(int n_cc, int NT) { return (size_t)n_cc * NT * 32 * 64; }

// app_core.c:4667 kern_norm_rms's shrink: (mean of squares + eps)^-1/2 in
// double, applied in float as x * shrink * w.
__device__ __forceinline__ float rms_shrink(float ssq, int n, float eps) {
  return (float)(1.0 / sqrt((double)ssq / (double)n + (double)eps));
}

// Writes two consecutive columns (c even) of lane n as hi/lo f16 pairs.
__device__ __forceinline__ void stage_pair(uint32_t *stage, int n, int c, float a0, float a1, int NT) {
  __half h0 = __float2half_rn(a0), h1 = __float2half_rn(a1);
  __half l0 = __float2half_rn(a0 - __half2float(h0)), l1 = __float2half_rn(a1 - __half2float(h1));
  int w = stage_word(n, c, NT);
  __half2 hi = __halves2half2(h0, h1), lo = __halves2half2(l0, l1);
  stage[w] = *reinterpret_cast<uint32_t *>(&hi);
  stage[w + 8] = *reinterpret_cast<uint32_t *>(&lo);
}

// Per-lane block reduction of up to 16 partial sums; every thread gets all.
__device__ __forceinline__ void block_sum16(float (&v)[16], int K, float *red /* [8][16] */) {
  const int warp = threadIdx.x >> 5, l32 = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < 16; ++j)
    if (j < K) v[j] = warp_sum(v[j]);
  if (l32 == 0)
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (j < K) red[warp * 16 + j] = v[j];
  __syncthreads();
#pragma unroll
  for (int j = 0; j < 16; ++j)
    if (j < K) {
      float s = 0.0f;
#pragma unroll
      for (int w = 0; w < GEMV_WARPS; ++w) s += red[w * 16 + j];
      v[j] = s;
    }
  __syncthreads();
}

// The prologue: every thread takes float4 columns for every lane, so the
// loads of one phase are all in flight together.  Norms need a reduction over
// the lane's whole vector: one phase per reduction.
template <int PRO>
__device__ void gemv_prologue(const GemvArgs &a, uint32_t *stage, float *red, int NT) {
  const int cols = a.pl.cols, K = a.lanes, n4 = cols >> 2;
  const int stage_words = (int)(gemv_stage_bytes(a.pl.n_cc, NT) / 4);
  for (int i = threadIdx.x; i < stage_words / 4; i += blockDim.x)
    reinterpret_cast<uint4 *>(stage)[i] = make_uint4(0u, 0u, 0u, 0u);
  __syncthreads();
  const float4 *__restrict__ x4 = reinterpret_cast<const float4 *>(a.x);
  const int xs4 = a.x_stride >> 2;
  if (PRO == PRO_F32) {
    for (int e = threadIdx.x; e < K * n4; e += blockDim.x) {
      int j = e / n4, c4 = e - j * n4;
      float4 v = x4[(size_t)j * xs4 + c4];
      stage_pair(stage, j, c4 * 4, v.x, v.y, NT);
      stage_pair(stage, j, c4 * 4 + 2, v.z, v.w, NT);
    }
    __syncthreads();
    return;
  }
  const float4 *__restrict__ win4 = reinterpret_cast<const float4 *>(a.w_in);
  float s[16];
  if (PRO == PRO_NORM) {
#pragma unroll
    for (int j = 0; j < 16; ++j) s[j] = 0.0f;
    for (int c4 = threadIdx.x; c4 < n4; c4 += blockDim.x)
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (j < K) {
          float4 v = x4[(size_t)j * xs4 + c4];
          s[j] += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
    block_sum16(s, K, red);
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (j < K) s[j] = rms_shrink(s[j], cols, a.eps);
    for (int c4 = threadIdx.x; c4 < n4; c4 += blockDim.x) {
      float4 w = win4[c4];
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (j < K) {
          float4 v = x4[(size_t)j * xs4 + c4];
          stage_pair(stage, j, c4 * 4, v.x * s[j] * w.x, v.y * s[j] * w.y, NT);
          stage_pair(stage, j, c4 * 4 + 2, v.z * s[j] * w.z, v.w * s[j] * w.w, NT);
        }
    }
    __syncthreads();
    return;
  }
  // residual forms: y = (x + norm(p) * w_res) * gain
  const float4 *__restrict__ p4 = reinterpret_cast<const float4 *>(a.p);
  const float4 *__restrict__ wr4 = reinterpret_cast<const float4 *>(a.w_res);
  const int ps4 = a.p_stride >> 2;
  float sp[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) sp[j] = 0.0f;
  for (int c4 = threadIdx.x; c4 < n4; c4 += blockDim.x)
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (j < K) {
        float4 v = p4[(size_t)j * ps4 + c4];
        sp[j] += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
      }
  block_sum16(sp, K, red);
#pragma unroll
  for (int j = 0; j < 16; ++j)
    if (j < K) sp[j] = rms_shrink(sp[j], cols, a.eps);
  const bool writer = blockIdx.x == 0 && a.x_out;
  float4 *xo4 = reinterpret_cast<float4 *>(a.x_out);
  const float gain = a.gain;
  auto resid = [&](int j, int c4, float4 wr) {
    float4 xv = x4[(size_t)j * xs4 + c4], pv = p4[(size_t)j * ps4 + c4];
    float4 y;
    y.x = xv.x + pv.x * sp[j] * wr.x;
    y.y = xv.y + pv.y * sp[j] * wr.y;
    y.z = xv.z + pv.z * sp[j] * wr.z;
    y.w = xv.w + pv.w * sp[j] * wr.w;
    if (gain != 1.0f) {
      y.x *= gain;
      y.y *= gain;
      y.z *= gain;
      y.w *= gain;
    }
    return y;
  };
#pragma unroll
  for (int j = 0; j < 16; ++j) s[j] = 0.0f;
  for (int c4 = threadIdx.x; c4 < n4; c4 += blockDim.x) {
    float4 wr = wr4[c4];
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (j < K) {
        float4 y = resid(j, c4, wr);
        if (writer) xo4[(size_t)j * xs4 + c4] = y;
        if (PRO == PRO_RESID) {
          stage_pair(stage, j, c4 * 4, y.x, y.y, NT);
          stage_pair(stage, j, c4 * 4 + 2, y.z, y.w, NT);
        } else {
          s[j] += y.x * y.x + y.y * y.y + y.z * y.z + y.w * y.w;
        }
      }
  }
  if (PRO == PRO_RESID_NORM) {
    block_sum16(s, K, red);
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (j < K) s[j] = rms_shrink(s[j], cols, a.eps);
    for (int c4 = threadIdx.x; c4 < n4; c4 += blockDim.x) {
      float4 wr = wr4[c4], w = win4[c4];
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (j < K) {
          float4 y = resid(j, c4, wr);
          stage_pair(stage, j, c4 * 4, y.x * s[j] * w.x, y.y * s[j] * w.y, NT);
          stage_pair(stage, j, c4 * 4 + 2, y.z * s[j] * w.z, y.w * s[j] * w.w, NT);
        }
    }
  }
  __syncthreads();
}

// Accumulates one 64-column chunk of one row block into tot[NT][4].
template <int NT>
__device__ __forceinline__ void chunk_product(const uint4 &w, const uint2 &s, const uint4 (&b)[NT][4],
                                              float (&tot)[NT][4]) {
  const float zero[4] = {0.f, 0.f, 0.f, 0.f};
  __half2 s01 = *reinterpret_cast<const __half2 *>(&s.x);
  __half2 s23 = *reinterpret_cast<const __half2 *>(&s.y);
  float sg0 = __low2float(s01), sg8_0 = __high2float(s01);
  float sg1 = __low2float(s23), sg8_1 = __high2float(s23);
  uint32_t a0[4], a1[4], a2[4], a3[4];
  dequant_i4(w.x, a0);
  dequant_i4(w.y, a1);
  dequant_i4(w.z, a2);
  dequant_i4(w.w, a3);
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    // b[nt][0..1]: hi fragments of products 0..3, b[nt][2..3]: lo fragments
    float g0[4], g1[4];
    mma16816(g0, a0, b[nt][0].x, b[nt][0].y, zero);
    mma16816(g0, a1, b[nt][0].z, b[nt][0].w, g0);
    mma16816(g0, a0, b[nt][2].x, b[nt][2].y, g0);
    mma16816(g0, a1, b[nt][2].z, b[nt][2].w, g0);
    mma16816(g1, a2, b[nt][1].x, b[nt][1].y, zero);
    mma16816(g1, a3, b[nt][1].z, b[nt][1].w, g1);
    mma16816(g1, a2, b[nt][3].x, b[nt][3].y, g1);
    mma16816(g1, a3, b[nt][3].z, b[nt][3].w, g1);
    tot[nt][0] += sg0 * g0[0] + sg1 * g1[0];
    tot[nt][1] += sg0 * g0[1] + sg1 * g1[1];
    tot[nt][2] += sg8_0 * g0[2] + sg8_1 * g1[2];
    tot[nt][3] += sg8_0 * g0[3] + sg8_1 * g1[3];
  }
}

template <int NT>
__device__ __forceinline__ void load_b(const uint32_t *stage, int cc, int lane32, uint4 (&b)[NT][4]) {
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const uint4 *p = reinterpret_cast<const uint4 *>(stage + ((cc * NT + nt) * 32 + lane32) * 16);
    b[nt][0] = p[0];
    b[nt][1] = p[1];
    b[nt][2] = p[2];
    b[nt][3] = p[3];
  }
}

}  // namespace igc
