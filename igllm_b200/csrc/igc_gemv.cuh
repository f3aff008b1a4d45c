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
// rounding before the f32 accumulator is the activation's.  Each lane's
// activations are first scaled by a power of two that puts the lane's largest
// magnitude at 2^14 (exact, undone in the epilogue), then staged as two f16
// values, hi = f16(a) and lo = f16(a - hi); both go through the tensor core
// against the same dequantised weights, so the product carries about 22
// significant bits of the activation at the cost of a second MMA per 16
// columns, and no lane can overflow f16.
//
// Norms ride on linearity: W (norm(y) * w) = shrink(y) * W (y * w), so the
// prologue stages y * w in one elementwise pass and the epilogue multiplies by
// the shrink, whose sum of squares the same pass collects.  A residual
// y = x + norm(p) * w_res needs p's shrink first; p's producer wrote the sum
// of its squares as one partial per block (fixed order, so deterministic).
//
// Layout in HBM (written once by the upload repack, igc_repack_kernel):
//   tiles  : [row_block][chunk][32 threads] uint4 - one 16-row x 64-column
//            tile is 512 contiguous bytes; thread t's 16 bytes are exactly the
//            A fragments of the four 16-column products it takes part in.
//   scales : [row_block][chunk][8] uint2 - for the thread group g = lane/4,
//            the f16 scales of rows g and g+8 for the chunk's two groups.
// Row blocks are 16 rows; chunks are 64 columns (two groups of 32).
#pragma once

#include <cuda_bf16.h>

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
  const float *p_ssq;  // producer's partial sums of squares of p, [p_parts][16]
  int p_parts;
  float *out_ssq;      // this launch's partial sums of squares of out, [gridDim.x][16]
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

// First pass: two consecutive columns (c even) of lane n as raw f32 in the
// two words their hi and lo f16 pairs will occupy.
__device__ __forceinline__ void stage_pair(uint32_t *stage, int n, int c, float a0, float a1, int NT) {
  int w = stage_word(n, c, NT);
  stage[w] = __float_as_uint(a0);
  stage[w + 8] = __float_as_uint(a1);
}

// Second pass, over the same words the same thread wrote: scaled, split into
// hi/lo f16 pairs.
__device__ __forceinline__ void stage_seal(uint32_t *stage, int n, int c, float scale, int NT) {
  int w = stage_word(n, c, NT);
  float a0 = __uint_as_float(stage[w]) * scale, a1 = __uint_as_float(stage[w + 8]) * scale;
  __half h0 = __float2half_rn(a0), h1 = __float2half_rn(a1);
  __half l0 = __float2half_rn(a0 - __half2float(h0)), l1 = __float2half_rn(a1 - __half2float(h1));
  __half2 hi = __halves2half2(h0, h1), lo = __halves2half2(l0, l1);
  stage[w] = *reinterpret_cast<uint32_t *>(&hi);
  stage[w + 8] = *reinterpret_cast<uint32_t *>(&lo);
}

// The power of two that puts a lane's largest magnitude at or under 2^14.
__device__ __forceinline__ float lane_scale(float amax) {
  if (!(amax > 0.0f) || !isfinite(amax)) return 1.0f;
  int e;
  frexpf(amax, &e);  // amax in [2^(e-1), 2^e)
  return ldexpf(1.0f, 14 - e);
}

__device__ __forceinline__ float fmax4(float4 v) { return fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))); }

// Shared-memory scratch the prologue leaves for the epilogue and uses for its
// own reductions (floats, after the staged activations):
//   [0, 16)      per-lane factor the epilogue applies (norm shrink / 2^e)
//   [16, 32)     per-lane power-of-two staging scale
//   [32, 48)     per-lane shrink of the residual's norm
//   [64, 192)    per-(lane, part) sums of squares
//   [192, 320)   per-(lane, part) magnitudes
//   [320, 576)   per-thread stripes of the residual's sums of squares
constexpr int SCR_FACTOR = 0, SCR_SCALE = 16, SCR_SHRINK_P = 32, SCR_SSQ = 64, SCR_AMAX = 192, SCR_STRIPE = 320;
constexpr int SCR_FLOATS = 576;

// The prologue, one elementwise pass and one shared-memory pass.  Warps take
// lanes: with K < 8 lanes, 8/K warps (a power of two) split one lane's
// columns; with more, a warp takes lanes w and w + 8.  Each thread walks its
// float4 columns with four loads in flight, and the per-lane reductions are
// a fixed-order sum over the parts.
template <int PRO>
__device__ void gemv_prologue(const GemvArgs &a, uint32_t *stage, float *scr, int NT) {
  const int cols = a.pl.cols, K = a.lanes, n4 = cols >> 2;
  const int warp = threadIdx.x >> 5, l32 = threadIdx.x & 31;
  const int stage_words = (int)(gemv_stage_bytes(a.pl.n_cc, NT) / 4);
  for (int i = threadIdx.x; i < stage_words / 4; i += blockDim.x)
    reinterpret_cast<uint4 *>(stage)[i] = make_uint4(0u, 0u, 0u, 0u);
  if (PRO == PRO_RESID || PRO == PRO_RESID_NORM) {
    // the residual's shrink from its producer's partials: thread (lane j,
    // stripe q0) sums parts q0, q0 + 16, ...; stripes are then added in order
    const int j = threadIdx.x & 15, q0 = threadIdx.x >> 4;
    float t = 0.0f;
    if (j < K)
      for (int q = q0; q < a.p_parts; q += 16) t += a.p_ssq[q * 16 + j];
    scr[SCR_STRIPE + threadIdx.x] = t;
    __syncthreads();
    if (threadIdx.x < 16 && (int)threadIdx.x < K) {
      float u = 0.0f;
      for (int q = 0; q < 16; ++q) u += scr[SCR_STRIPE + q * 16 + threadIdx.x];
      scr[SCR_SHRINK_P + threadIdx.x] = rms_shrink(u, cols, a.eps);
    }
  }
  __syncthreads();
  int wpl = 1;  // warps a lane
  while (wpl * 2 * K <= GEMV_WARPS) wpl *= 2;
  const int n_slots = (K + GEMV_WARPS - 1) / GEMV_WARPS;  // lanes a warp (1 or 2)
  const float4 *__restrict__ x4 = reinterpret_cast<const float4 *>(a.x);
  const float4 *__restrict__ p4 = reinterpret_cast<const float4 *>(a.p);
  const float4 *__restrict__ wr4 = reinterpret_cast<const float4 *>(a.w_res);
  const float4 *__restrict__ win4 = reinterpret_cast<const float4 *>(a.w_in);
  float4 *__restrict__ xo4 = (blockIdx.x == 0 && a.x_out) ? reinterpret_cast<float4 *>(a.x_out) : nullptr;
  const int xs4 = a.x_stride >> 2, ps4 = a.p_stride >> 2;
  const float gain = a.gain;
  for (int slot = 0; slot < n_slots; ++slot) {
    const int j = wpl > 1 ? warp / wpl : warp + slot * GEMV_WARPS;
    const int part = wpl > 1 ? warp % wpl : 0;
    float ssq = 0.0f, amax = 0.0f;
    if (j < K) {
      const int lo = (n4 * part) / wpl, hi = (n4 * (part + 1)) / wpl;
      const float sp = (PRO == PRO_RESID || PRO == PRO_RESID_NORM) ? scr[SCR_SHRINK_P + j] : 0.0f;
#pragma unroll 4
      for (int c4 = lo + l32; c4 < hi; c4 += 32) {
        float4 y = x4[(size_t)j * xs4 + c4];
        if (PRO == PRO_RESID || PRO == PRO_RESID_NORM) {
          // app_core.c:11690-11740: x += norm(p) * w, then the layer gain
          float4 pv = p4[(size_t)j * ps4 + c4], wr = wr4[c4];
          y.x = y.x + pv.x * sp * wr.x;
          y.y = y.y + pv.y * sp * wr.y;
          y.z = y.z + pv.z * sp * wr.z;
          y.w = y.w + pv.w * sp * wr.w;
          if (gain != 1.0f) {
            y.x *= gain;
            y.y *= gain;
            y.z *= gain;
            y.w *= gain;
          }
          if (xo4) xo4[(size_t)j * xs4 + c4] = y;
        }
        if (PRO != PRO_F32) ssq += y.x * y.x + y.y * y.y + y.z * y.z + y.w * y.w;
        if (PRO == PRO_NORM || PRO == PRO_RESID_NORM) {
          float4 w = win4[c4];
          y.x *= w.x;
          y.y *= w.y;
          y.z *= w.z;
          y.w *= w.w;
        }
        amax = fmaxf(amax, fmax4(y));
        stage_pair(stage, j, c4 * 4, y.x, y.y, NT);
        stage_pair(stage, j, c4 * 4 + 2, y.z, y.w, NT);
      }
    }
    ssq = warp_sum(ssq);
    amax = warp_max(amax);
    if (l32 == 0 && j < K) {
      scr[SCR_SSQ + j * 8 + part] = ssq;
      scr[SCR_AMAX + j * 8 + part] = amax;
    }
  }
  __syncthreads();
  if (threadIdx.x < 16 && (int)threadIdx.x < K) {
    const int j = threadIdx.x;
    float ssq = 0.0f, amax = 0.0f;
    for (int q = 0; q < wpl; ++q) {
      ssq += scr[SCR_SSQ + j * 8 + q];
      amax = fmaxf(amax, scr[SCR_AMAX + j * 8 + q]);
    }
    const float sc = lane_scale(amax);
    const float shrink = (PRO == PRO_NORM || PRO == PRO_RESID_NORM) ? rms_shrink(ssq, cols, a.eps) : 1.0f;
    scr[SCR_SCALE + j] = sc;
    scr[SCR_FACTOR + j] = shrink * (1.0f / sc);
  }
  __syncthreads();
  for (int slot = 0; slot < n_slots; ++slot) {
    const int j = wpl > 1 ? warp / wpl : warp + slot * GEMV_WARPS;
    const int part = wpl > 1 ? warp % wpl : 0;
    if (j >= K) continue;
    const int lo = (n4 * part) / wpl, hi = (n4 * (part + 1)) / wpl;
    const float sc = scr[SCR_SCALE + j];
    for (int c4 = lo + l32; c4 < hi; c4 += 32) {
      stage_seal(stage, j, c4 * 4, sc, NT);
      stage_seal(stage, j, c4 * 4 + 2, sc, NT);
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
