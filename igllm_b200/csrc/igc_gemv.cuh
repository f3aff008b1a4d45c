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
// significant bits of the activation, and no lane can overflow f16.  The hi
// and lo products are accumulated apart and added once per output, in the
// same order whatever the lane count, so a lane's result does not depend on
// how many lanes shared its pass.
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
// Row blocks are 16 rows; chunks are 64 columns (two groups of 32).  One row
// block's chunks are contiguous, so a warp fetches a run of them with one
// bulk copy into shared memory.
#pragma once

#include <cuda_bf16.h>

#include "igc_device.cuh"

namespace igc {

// PRO_F32S: unnormed input whose producer left its magnitudes (one-pass staging).
enum : int { PRO_F32 = 0, PRO_NORM = 1, PRO_RESID = 2, PRO_RESID_NORM = 3, PRO_F32S = 4 };
enum : int { EPI_STORE = 0, EPI_GELU_PAIR = 1, EPI_GELU_MUL = 2, EPI_LOGITS = 3 };

// Lane modes.  PACK (up to 4 lanes): one 8-column B tile carries lanes 0-3 hi
// in columns 0-3 and their lo halves in columns 4-7, so one product does both.
// NT1 / NT2 (up to 8 / 16 lanes): hi and lo are separate B tiles, 8 lanes each.
enum : int { MODE_PACK = 0, MODE_NT1 = 1, MODE_NT2 = 2 };

__host__ __device__ inline int gemv_mode(int lanes) { return lanes <= 4 ? MODE_PACK : lanes <= 8 ? MODE_NT1 : MODE_NT2; }

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
  int split;  // warps that share one row block's chunks (1, 2, 4 or 8), fixed per plane
  // weight ring (set by the launcher): chunks a piece, pieces in flight a warp,
  // and where the reduction space, barriers and ring sit in shared memory
  int piece, depth;
  int off_red, off_bars, off_ring;
  // unit slots (block, group) the units are spread over, and groups a
  // virtual 8-warp block holds: partial sums are written one per virtual
  // block, so their grouping is the same whatever a launch's block width
  int slots, vgroups;
  int *err;  // set nonzero when a wait gave up
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
  // partials are lane-major: [16 lanes][GEMV_PART_LIMIT parts]
  const float *p_ssq;  // producer's partial sums of squares of p
  int p_parts;
  float *out_ssq;      // this launch's partial sums of squares of out, one a virtual block
  // magnitudes: the producer's per-part largest |x|, which
  // lets an unnormed prologue stage in one pass, and this launch's per virtual
  // block largest |out| for its own consumer
  const float *x_amax;
  int x_amax_parts;
  float *out_amax;
  // epilogue
  float *out;
  int out_stride;
  float out_scale;
  const float *aux;
  int aux_stride;
  float cap;
  float *part_val;  // EPI_LOGITS argmax partials [gridDim.x][16]
  int *part_idx;
  // lane batches: with batches > 1 the launch's blockIdx.y takes lanes
  // [y * lanes, (y + 1) * lanes) of lanes_total, every pointer above moved
  // to its first lane (the lanes are independent, so the batches run side by
  // side with the staging of `lanes` lanes each)
  int batches, lanes_total;
  // launch stamp (igc_device.cuh stamp_begin / stamp_end), or null
  unsigned long long *stamp;
};

// Warps a block: the planning unit of a plane (its split and block count
// are chosen for 8-warp blocks).  Launches of up to 8 lanes run 16-warp
// blocks where their shared memory fits, each holding two 8-warp blocks'
// worth of groups, so a block's staging work is spread over twice the
// threads; results are the same either way.
constexpr int GEMV_WARPS = 8;
constexpr int GEMV_MAX_WARPS = 16;
constexpr int GEMV_PIECE_BYTES = 576;  // one chunk of one row block: 512 B of codes + 64 B of scales
constexpr int GEMV_MAX_DEPTH = 8;
constexpr int GEMV_PART_LIMIT = 320;  // producer partials the prologue reads (16 stripes x 20)

// Staged activations, per chunk: PACK 32 thread slots x 8 words (the four
// 16-column products' b0, b1), NT 32 slots x 16 words per 8-lane tile (hi
// b0, b1 of the four products, then lo).  Word of (lane n, column c, half):
// In the 8-lane-tile modes the 16-byte quarters of a slot are swizzled
// (quarter j of slot L at j ^ ((L >> 1) & 3)), so that the four fragment
// reads of a quarter-warp meet every bank once instead of four times.  The
// packed mode's 32-byte slots are left as they are.
__device__ __forceinline__ int stage_quad(int slot, int MODE) { return MODE == MODE_PACK ? 0 : (slot >> 1) & 3; }

__device__ __forceinline__ int stage_word(int n, int c, int lo, int MODE) {
  const int cc = c >> 6, kb = (c >> 4) & 3, k = c & 15, t = (k & 7) >> 1;
  if (MODE == MODE_PACK) {
    const int L = (n + (lo ? 4 : 0)) * 4 + t, w = kb * 2 + (k >> 3);
    return (cc * 32 + L) * 8 + ((((w >> 2) ^ stage_quad(L, MODE)) << 2) | (w & 3));
  }
  const int NT = MODE == MODE_NT2 ? 2 : 1;
  const int nt = n >> 3, L = (n & 7) * 4 + t, w = kb * 2 + (k >> 3) + (lo ? 8 : 0);
  return (((cc * NT + nt) * 32 + L) * 16) + ((((w >> 2) ^ stage_quad(L, MODE)) << 2) | (w & 3));
}

__host__ __device__ inline int stage_chunk_words(int MODE) { return MODE == MODE_PACK ? 256 : MODE == MODE_NT1 ? 512 : 1024; }

__host__ __device__ inline size_t gemv_stage_bytes(int n_cc, int MODE) { return (size_t)n_cc * stage_chunk_words(MODE) * 4; }

// Accumulator floats a thread keeps per half (gate or up) of a unit.
__host__ __device__ inline int gemv_acc_floats(int MODE) { return MODE == MODE_PACK ? 4 : MODE == MODE_NT1 ? 8 : 16; }

// app_core.c:4667 kern_norm_rms's shrink: (mean of squares + eps)^-1/2,
// applied in float as x * shrink * w.  The reference forms it in double; in
// float it differs by about an ulp and stays off the double units' latency,
// which sits on every residual prologue's critical path.
__device__ __forceinline__ float rms_shrink(float ssq, int n, float eps) {
  return 1.0f / sqrtf(ssq / (float)n + eps);
}

// The pair of words that hold columns c, c + 1 (c even) of one lane: the
// first pass leaves their raw f32 values there (c in the hi word, c + 1 in
// the lo word); this turns them, scaled, into the hi and lo f16 pairs.
__device__ __forceinline__ void seal_words(uint32_t *stage, int wh, int wl, float scale) {
  float a0 = __uint_as_float(stage[wh]) * scale, a1 = __uint_as_float(stage[wl]) * scale;
  __half h0 = __float2half_rn(a0), h1 = __float2half_rn(a1);
  __half l0 = __float2half_rn(a0 - __half2float(h0)), l1 = __float2half_rn(a1 - __half2float(h1));
  __half2 hi = __halves2half2(h0, h1), lo = __halves2half2(l0, l1);
  stage[wh] = *reinterpret_cast<uint32_t *>(&hi);
  stage[wl] = *reinterpret_cast<uint32_t *>(&lo);
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
//   [64, 832)     per-(lane, 128-column part) sums of squares, 48 parts a lane
//   [832, 1088)   per-(lane, warp) magnitudes, 16 warps a lane
//   [1600, 2112)  per-thread stripes of the residual's sums of squares
constexpr int SCR_FACTOR = 0, SCR_SCALE = 16, SCR_SHRINK_P = 32, SCR_SSQ = 64, SCR_AMAX = 832, SCR_STRIPE = 1600;
constexpr int SCR_FLOATS = 2112;
// A plane wider than 6144 columns (the doubled feed-forward's 12288-column
// down projection) keeps the sums of its parts 48-95 after the rest:
//   [2112, 2880)  per-(lane, part) sums of squares of parts 48-95
// and only its launches take those 3 KB.
constexpr int SCR_SSQ_FAR = SCR_FLOATS, SCR_FLOATS_WIDE = SCR_FLOATS + 16 * 48;
__host__ __device__ __forceinline__ int scr_ssq(int j, int part) {
  return part < 48 ? SCR_SSQ + j * 48 + part : SCR_SSQ_FAR + j * 48 + (part - 48);
}

// float4 columns a thread loads before computing on them: as many as keep
// the register file in bounds for the arrays the prologue reads.
template <int PRO>
struct ProBatch {
  static constexpr int value = PRO == PRO_F32 ? 8 : PRO == PRO_NORM ? 6 : 4;
};

// The prologue.  A lane's columns are cut into fixed parts of 128 (32
// float4, one a thread), and every per-lane sum is a fixed tree over those
// parts, so a lane's staged values and sums do not depend on how many lanes
// or warps a launch has.  Warps take lanes: with fewer lanes than warps,
// `wpl` warps (a power of two) share one lane's parts round robin; with
// more, a warp takes lanes w and w + WARPS.  A part's stage words sit two
// chunks further on per part, so each thread computes its four word offsets
// once and then only adds.  The producer partials and the first batch of
// activations are loaded before anything waits on either.
constexpr int GEMV_MAX_PARTS = 96;  // 12288 columns

// The unnormed prologue when the producer left the magnitudes of x: the
// lanes' staging scales are known before any activation arrives, so each
// value is loaded, scaled and split into its final hi/lo words in one pass
// (the same scale the general prologue would take: the power of two of the
// same largest magnitude).
template <int MODE, int WARPS>
__device__ void gemv_prologue_scaled(const GemvArgs &a, uint32_t *stage, float *scr) {
  constexpr int B = 8;
  const int cols = a.pl.cols, K = a.lanes, n4 = cols >> 2;
  const int warp = threadIdx.x >> 5, l32 = threadIdx.x & 31;
  if (cols & 63) {
    const int words = (int)(gemv_stage_bytes(a.pl.n_cc, MODE) / 16);
    for (int i = threadIdx.x; i < words; i += blockDim.x) reinterpret_cast<uint4 *>(stage)[i] = make_uint4(0u, 0u, 0u, 0u);
    __syncthreads();
  }
  int wpl = 1;
  while (wpl * 2 * K <= WARPS) wpl *= 2;
  const int n_slots = (K + WARPS - 1) / WARPS;
  const int w_local = wpl > 1 ? warp % wpl : 0;
  const int span4 = (n4 + wpl - 1) / wpl, lo = w_local * span4, hi = min(n4, lo + span4);
  const int c4_0 = lo + l32;
  const int count = c4_0 < hi ? (hi - c4_0 + 31) >> 5 : 0;
  const int step = 2 * stage_chunk_words(MODE);  // 128 columns further on: two chunks
  const float4 *__restrict__ x4 = reinterpret_cast<const float4 *>(a.x);
  const int xs4 = a.x_stride >> 2;
  int jj[2];
  bool live[2];
  int wh0[2], wl0[2], wh2[2], wl2[2];
#pragma unroll
  for (int slot = 0; slot < 2; ++slot) {
    jj[slot] = wpl > 1 ? warp / wpl : warp + slot * WARPS;
    live[slot] = slot < n_slots && jj[slot] < K;
    const int c = c4_0 * 4;
    wh0[slot] = stage_word(jj[slot], c, 0, MODE);
    wl0[slot] = stage_word(jj[slot], c, 1, MODE);
    wh2[slot] = stage_word(jj[slot], c + 2, 0, MODE);
    wl2[slot] = stage_word(jj[slot], c + 2, 1, MODE);
  }
  float4 X[B];
  auto load = [&](int slot, int i0) {
#pragma unroll
    for (int b = 0; b < B; ++b)
      if (i0 + b < count) X[b] = x4[(size_t)jj[slot] * xs4 + c4_0 + 32 * (i0 + b)];
  };
  auto put = [&](int wh, int wl, float a0, float a1) {
    __half h0 = __float2half_rn(a0), h1 = __float2half_rn(a1);
    __half l0 = __float2half_rn(a0 - __half2float(h0)), l1 = __float2half_rn(a1 - __half2float(h1));
    __half2 hv = __halves2half2(h0, h1), lv = __halves2half2(l0, l1);
    stage[wh] = *reinterpret_cast<uint32_t *>(&hv);
    stage[wl] = *reinterpret_cast<uint32_t *>(&lv);
  };
  auto seal = [&](int slot, int i0) {
    const float sc = scr[SCR_SCALE + jj[slot]];
#pragma unroll
    for (int b = 0; b < B; ++b) {
      if (i0 + b < count) {
        const int o = step * (i0 + b);
        const float4 y = X[b];
        put(wh0[slot] + o, wl0[slot] + o, y.x * sc, y.y * sc);
        put(wh2[slot] + o, wl2[slot] + o, y.z * sc, y.w * sc);
      }
    }
  };
  if (live[0]) load(0, 0);
  // warp w reduces lane w's (and w + WARPS's) magnitude partials, 32 at a time
  for (int j = warp; j < K; j += WARPS) {
    float m = 0.0f;
#pragma unroll
    for (int i = 0; i < GEMV_PART_LIMIT / 32; ++i) {
      const int q = l32 + 32 * i;
      if (q < a.x_amax_parts) m = fmaxf(m, a.x_amax[j * GEMV_PART_LIMIT + q]);
    }
    m = warp_max(m);
    if (l32 == 0) {
      const float sc = lane_scale(m);
      scr[SCR_SCALE + j] = sc;
      scr[SCR_FACTOR + j] = 1.0f / sc;
    }
  }
  __syncthreads();
#pragma unroll
  for (int slot = 0; slot < 2; ++slot) {
    if (!live[slot]) continue;
    if (slot > 0) load(slot, 0);
    seal(slot, 0);
    for (int i0 = B; i0 < count; i0 += B) {
      load(slot, i0);
      seal(slot, i0);
    }
  }
  __syncthreads();
}

template <int PRO, int MODE, int WARPS>
__device__ void gemv_prologue(const GemvArgs &a, uint32_t *stage, float *scr) {
  constexpr bool RES = PRO == PRO_RESID || PRO == PRO_RESID_NORM;
  constexpr bool NRM = PRO == PRO_NORM || PRO == PRO_RESID_NORM;
  constexpr int B = ProBatch<PRO>::value;
  const int cols = a.pl.cols, K = a.lanes, n4 = cols >> 2;
  const int nparts = (n4 + 31) >> 5;
  const int warp = threadIdx.x >> 5, l32 = threadIdx.x & 31;
  if (cols & 63) {
    // columns past `cols` in the last chunk meet zero weights, and must be
    // zero (not stale NaN patterns) for the products to stay exact
    const int words = (int)(gemv_stage_bytes(a.pl.n_cc, MODE) / 16);
    for (int i = threadIdx.x; i < words; i += blockDim.x) reinterpret_cast<uint4 *>(stage)[i] = make_uint4(0u, 0u, 0u, 0u);
    __syncthreads();
  }
  float part[RES ? 2 : 1][GEMV_PART_LIMIT / 32];
  int wpl = 1;  // warps a lane
  while (wpl * 2 * K <= WARPS) wpl *= 2;
  const int n_slots = (K + WARPS - 1) / WARPS;  // lanes a warp (1 or 2)
  const int w_local = wpl > 1 ? warp % wpl : 0;
  const int count = w_local < nparts ? (nparts - w_local + wpl - 1) / wpl : 0;  // parts of this warp per slot
  const int c4_0 = w_local * 32 + l32, c4_step = 32 * wpl;
  const int step = 2 * wpl * stage_chunk_words(MODE);  // stage words between consecutive parts of this warp
  const float4 *__restrict__ x4 = reinterpret_cast<const float4 *>(a.x);
  const float4 *__restrict__ p4 = reinterpret_cast<const float4 *>(a.p);
  const float4 *__restrict__ wr4 = reinterpret_cast<const float4 *>(a.w_res);
  const float4 *__restrict__ win4 = reinterpret_cast<const float4 *>(a.w_in);
  const bool write_x = blockIdx.x == 0 && a.x_out;
  const int xs4 = a.x_stride >> 2, ps4 = a.p_stride >> 2;
  const float gain = a.gain;

  int jj[2];
  bool live[2];
  int wh0[2], wl0[2], wh2[2], wl2[2];  // word offsets of part w_local: columns c, c + 1 (hi, lo) and c + 2, c + 3
#pragma unroll
  for (int slot = 0; slot < 2; ++slot) {
    jj[slot] = wpl > 1 ? warp / wpl : warp + slot * WARPS;
    live[slot] = slot < n_slots && jj[slot] < K;
    const int c = c4_0 * 4;
    wh0[slot] = stage_word(jj[slot], c, 0, MODE);
    wl0[slot] = stage_word(jj[slot], c, 1, MODE);
    wh2[slot] = stage_word(jj[slot], c + 2, 0, MODE);
    wl2[slot] = stage_word(jj[slot], c + 2, 1, MODE);
  }

  float4 X[B], Pv[B], WR[B], WI[B];
  float amax_acc[2] = {0.0f, 0.0f};  // magnitudes need no fixed order: one max per thread
  // x and the norm weights (`l2` reads x past L1: before the wait it was
  // written by a kernel two or more launches back), then the producer's p
  auto load_x = [&](int slot, int i0, bool l2) {
    const int j = jj[slot];
#pragma unroll
    for (int b = 0; b < B; ++b) {
      const int c4 = c4_0 + c4_step * (i0 + b);
      if (i0 + b < count && c4 < n4) {
        X[b] = l2 ? __ldcg(x4 + (size_t)j * xs4 + c4) : x4[(size_t)j * xs4 + c4];
        if (RES) WR[b] = wr4[c4];
        if (NRM) WI[b] = win4[c4];
      }
    }
  };
  auto load_p = [&](int slot, int i0) {
    const int j = jj[slot];
#pragma unroll
    for (int b = 0; b < B; ++b) {
      const int c4 = c4_0 + c4_step * (i0 + b);
      if (RES && i0 + b < count && c4 < n4) Pv[b] = p4[(size_t)j * ps4 + c4];
    }
  };
  auto load = [&](int slot, int i0) {
    load_x(slot, i0, false);
    load_p(slot, i0);
  };
  auto compute = [&](int slot, int i0) {
    const int j = jj[slot];
    const float sp = RES ? scr[SCR_SHRINK_P + j] : 0.0f;
#pragma unroll
    for (int b = 0; b < B; ++b) {
      const int i = i0 + b;
      if (i < count) {  // warp-uniform: the part's sums are warp reductions
        const int c4 = c4_0 + c4_step * i;
        float ssq = 0.0f;
        if (c4 < n4) {
          float4 y = X[b];
          if (RES) {
            // app_core.c:11690-11740: x += norm(p) * w, then the layer gain
            y.x = y.x + Pv[b].x * sp * WR[b].x;
            y.y = y.y + Pv[b].y * sp * WR[b].y;
            y.z = y.z + Pv[b].z * sp * WR[b].z;
            y.w = y.w + Pv[b].w * sp * WR[b].w;
            if (gain != 1.0f) {
              y.x *= gain;
              y.y *= gain;
              y.z *= gain;
              y.w *= gain;
            }
            if (write_x) reinterpret_cast<float4 *>(a.x_out)[(size_t)j * xs4 + c4] = y;
          }
          if (NRM) {
            ssq = y.x * y.x + y.y * y.y + y.z * y.z + y.w * y.w;
            y.x *= WI[b].x;
            y.y *= WI[b].y;
            y.z *= WI[b].z;
            y.w *= WI[b].w;
          }
          amax_acc[slot] = fmaxf(amax_acc[slot], fmax4(y));
          const int o = step * i;
          stage[wh0[slot] + o] = __float_as_uint(y.x);
          stage[wl0[slot] + o] = __float_as_uint(y.y);
          stage[wh2[slot] + o] = __float_as_uint(y.z);
          stage[wl2[slot] + o] = __float_as_uint(y.w);
        }
        if (NRM) {  // a norm's sum of squares: one fixed tree per part
          ssq = warp_sum(ssq);
          if (l32 == 0) scr[scr_ssq(j, w_local + wpl * i)] = ssq;
        }
      }
    }
  };

  if (RES) {
    // a residual prologue runs ahead of the kernel's wait: the residual
    // stream and the norm weights do not come from the kernel just before
    if (live[0]) load_x(0, 0, true);
    pdl_wait();
    stamp_begin(a.stamp);
    // the residual's partials: warp w holds lane w's (and w + WARPS's),
    // thread l the parts l, l + 32, ... (a fixed tree whatever the lane count)
#pragma unroll
    for (int sl = 0; sl < 2; ++sl) {
      const int j = warp + sl * WARPS;
#pragma unroll
      for (int i = 0; i < GEMV_PART_LIMIT / 32; ++i) {
        const int q = l32 + 32 * i;
        part[sl][i] = (j < K && q < a.p_parts) ? a.p_ssq[j * GEMV_PART_LIMIT + q] : 0.0f;
      }
    }
    if (live[0]) load_p(0, 0);
  } else if (live[0]) {
    load(0, 0);
  }
  if (RES) {
#pragma unroll
    for (int sl = 0; sl < 2; ++sl) {
      const int j = warp + sl * WARPS;
      if (j >= K) continue;
      float tsum = 0.0f;
#pragma unroll
      for (int i = 0; i < GEMV_PART_LIMIT / 32; ++i) tsum += part[sl][i];
      tsum = warp_sum(tsum);
      if (l32 == 0) scr[SCR_SHRINK_P + j] = rms_shrink(tsum, cols, a.eps);
    }
    __syncthreads();
  }
#pragma unroll
  for (int slot = 0; slot < 2; ++slot) {
    if (!live[slot]) continue;
    if (slot > 0) load(slot, 0);
    compute(slot, 0);
    for (int i0 = B; i0 < count; i0 += B) {
      load(slot, i0);
      compute(slot, i0);
    }
  }
#pragma unroll
  for (int slot = 0; slot < 2; ++slot) {
    if (!live[slot]) continue;
    const float m_ = warp_max(amax_acc[slot]);
    if (l32 == 0) scr[SCR_AMAX + jj[slot] * 16 + w_local] = m_;
  }
  __syncthreads();
  // each warp takes its lane's scale from the lane's warp magnitudes and
  // seals its own words; the warp holding the lane's first part also sums
  // the parts' squares in a fixed tree and leaves the epilogue factor
#pragma unroll
  for (int slot = 0; slot < 2; ++slot) {
    if (!live[slot]) continue;
    const int j = jj[slot];
    const float sc = lane_scale(warp_max(l32 < wpl ? scr[SCR_AMAX + j * 16 + l32] : 0.0f));
    if (w_local == 0) {
      float s_ = 0.0f;
      if (NRM) {
        // a fixed tree: parts l32, l32 + 32 and l32 + 64 a lane (the third is
        // 0 below 65 parts, which leaves narrower planes' sums as they were)
        s_ = warp_sum(((l32 < nparts ? scr[scr_ssq(j, l32)] : 0.0f) +
                       (l32 + 32 < nparts ? scr[scr_ssq(j, l32 + 32)] : 0.0f)) +
                      (l32 + 64 < nparts ? scr[scr_ssq(j, l32 + 64)] : 0.0f));
      }
      if (l32 == 0) {
        const float shrink = NRM ? rms_shrink(s_, cols, a.eps) : 1.0f;
        scr[SCR_SCALE + j] = sc;
        scr[SCR_FACTOR + j] = shrink * (1.0f / sc);
      }
    }
#pragma unroll 4
    for (int i = 0; i < count; ++i) {
      if (c4_0 + c4_step * i < n4) {
        const int o = step * i;
        seal_words(stage, wh0[slot] + o, wl0[slot] + o, sc);
        seal_words(stage, wh2[slot] + o, wl2[slot] + o, sc);
      }
    }
  }
  __syncthreads();
}

// The four A fragments of one chunk (two 32-column groups, two 16-column
// products each) and the group scales of rows g and g + 8.
struct ChunkA {
  uint32_t a0[4], a1[4], a2[4], a3[4];
  float sg0, sg1, sg8_0, sg8_1;
};

__device__ __forceinline__ void chunk_a(const uint4 &w, const uint2 &s, ChunkA &A) {
  __half2 s01 = *reinterpret_cast<const __half2 *>(&s.x);
  __half2 s23 = *reinterpret_cast<const __half2 *>(&s.y);
  A.sg0 = __low2float(s01);
  A.sg8_0 = __high2float(s01);
  A.sg1 = __low2float(s23);
  A.sg8_1 = __high2float(s23);
  dequant_i4(w.x, A.a0);
  dequant_i4(w.y, A.a1);
  dequant_i4(w.z, A.a2);
  dequant_i4(w.w, A.a3);
}

// One chunk against one 8-column B tile (the four products' b0, b1 in two
// uint4): acc[i] += sg(group 0) * g0[i] + sg(group 1) * g1[i], rows g (i < 2)
// and g + 8, in one fixed order of fused multiply-adds.
__device__ __forceinline__ void chunk_tile(const ChunkA &A, const uint4 &b01, const uint4 &b23, float *acc) {
  const float zero[4] = {0.f, 0.f, 0.f, 0.f};
  float g0[4], g1[4];
  mma16816(g0, A.a0, b01.x, b01.y, zero);
  mma16816(g0, A.a1, b01.z, b01.w, g0);
  mma16816(g1, A.a2, b23.x, b23.y, zero);
  mma16816(g1, A.a3, b23.z, b23.w, g1);
  acc[0] = fmaf(A.sg1, g1[0], fmaf(A.sg0, g0[0], acc[0]));
  acc[1] = fmaf(A.sg1, g1[1], fmaf(A.sg0, g0[1], acc[1]));
  acc[2] = fmaf(A.sg8_1, g1[2], fmaf(A.sg8_0, g0[2], acc[2]));
  acc[3] = fmaf(A.sg8_1, g1[3], fmaf(A.sg8_0, g0[3], acc[3]));
}

// One chunk of one row block into the thread's accumulators: PACK one tile
// (hi and lo in its columns), NT per 8-lane tile a hi and a lo accumulator.
template <int MODE>
__device__ __forceinline__ void chunk_product(const uint4 &w, const uint2 &s, const uint32_t *stage_chunk, int lane32,
                                              float *acc) {
  ChunkA A;
  chunk_a(w, s, A);
  const int q = stage_quad(lane32, MODE);  // the swizzle of this thread's slot
  if (MODE == MODE_PACK) {
    const uint4 *p = reinterpret_cast<const uint4 *>(stage_chunk + lane32 * 8);
    chunk_tile(A, p[q], p[1 ^ q], acc);
  } else {
    constexpr int NT = MODE == MODE_NT2 ? 2 : 1;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const uint4 *p = reinterpret_cast<const uint4 *>(stage_chunk + (nt * 32 + lane32) * 16);
      chunk_tile(A, p[q], p[1 ^ q], acc + nt * 8);          // hi
      chunk_tile(A, p[2 ^ q], p[3 ^ q], acc + nt * 8 + 4);  // lo
    }
  }
}

}  // namespace igc
