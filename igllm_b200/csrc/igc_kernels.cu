// igc_kernels.cu - the sm_100a kernels of the verify round.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <float.h>
#include <stdint.h>

#include "igc_gemv.cuh"
#include "igc_kernels.h"

namespace igc {

// ---------------------------------------------------------------------------
// upload repack: raw U8 codes (two a byte, low nibble first, row_stride bytes a
// row) and f16 scales [rows][groups] into the tile layout of igc_gemv.cuh.
// One thread writes one thread-slot (16 bytes) of one tile and, for t == 0,
// that slot group's 8-byte scale record.
__global__ void repack_kernel(const uint8_t *code, size_t row_stride, const uint16_t *scale,
                              int groups, int rows, int cols, int n_rb, int n_cc, int out_mul, int out_add,
                              uint4 *tiles, uint2 *scales) {
  long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  long total = (long)n_rb * n_cc * 32;
  if (idx >= total) return;
  int slot = (int)(idx & 31);
  long tile = idx >> 5;
  int cc = (int)(tile % n_cc);
  int rb = (int)(tile / n_cc);
  int g = slot >> 2, t = slot & 3;
  int r0 = rb * 16 + g, r8 = r0 + 8;
  long out_tile = (long)(rb * out_mul + out_add) * n_cc + cc;
  auto nib = [&](int r, int c) -> uint32_t {
    if (r >= rows || c >= cols) return 8u;  // zero weight
    uint8_t byte = code[(size_t)r * row_stride + (size_t)(c >> 1)];
    return (c & 1) ? (uint32_t)(byte >> 4) : (uint32_t)(byte & 15u);
  };
  uint32_t word[4];
#pragma unroll
  for (int kb = 0; kb < 4; ++kb) {
    int base = cc * 64 + kb * 16;
    uint32_t n0 = nib(r0, base + 2 * t), n4 = nib(r0, base + 2 * t + 1);
    uint32_t n1 = nib(r8, base + 2 * t), n5 = nib(r8, base + 2 * t + 1);
    uint32_t n2 = nib(r0, base + 2 * t + 8), n6 = nib(r0, base + 2 * t + 9);
    uint32_t n3 = nib(r8, base + 2 * t + 8), n7 = nib(r8, base + 2 * t + 9);
    word[kb] = n0 | (n1 << 4) | (n2 << 8) | (n3 << 12) | (n4 << 16) | (n5 << 20) | (n6 << 24) |
               (n7 << 28);
  }
  tiles[out_tile * 32 + slot] = make_uint4(word[0], word[1], word[2], word[3]);
  if (t == 0) {
    auto sc = [&](int r, int gr) -> uint32_t {
      if (r >= rows || gr >= groups) return 0u;
      return scale[(size_t)r * groups + gr];
    };
    uint32_t lo = sc(r0, 2 * cc) | (sc(r8, 2 * cc) << 16);
    uint32_t hi = sc(r0, 2 * cc + 1) | (sc(r8, 2 * cc + 1) << 16);
    scales[out_tile * 8 + g] = make_uint2(lo, hi);
  }
}

// ---------------------------------------------------------------------------
// the skinny GEMM
//
// Work: a unit is one row block (a gate/up pair for PAIR planes).  The S
// warps of a group share a unit, each taking a fixed slice of its chunks
// (S is a property of the plane, so the summation order never depends on the
// lane count); groups are spread over (block, group) slots round robin.
// Each warp streams its own pieces (runs of chunks of one unit) through a
// private ring of `depth` shared-memory slots filled by bulk copies that lane
// 0 issues; the first pieces are in flight before the kernel waits for the
// kernel ahead of it and before the activation prologue runs.
template <int MODE, int WARPS, int PAIR, int PRO, int EPI>
__global__ void __launch_bounds__(WARPS * 32) gemv_kernel(GemvArgs a) {
  constexpr int NT = MODE == MODE_NT2 ? 2 : 1;
  constexpr int H = PAIR + 1;
  constexpr int ACC = MODE == MODE_PACK ? 4 : 8 * NT;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  uint32_t *stage = reinterpret_cast<uint32_t *>(smem_raw);
  float *scr = reinterpret_cast<float *>(smem_raw + gemv_stage_bytes(a.pl.n_cc, MODE));
  float *red = reinterpret_cast<float *>(smem_raw + a.off_red);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem_raw + a.off_bars);
  unsigned char *ring = smem_raw + a.off_ring;

  const int warp = threadIdx.x >> 5, lane32 = threadIdx.x & 31;
  const int g = lane32 >> 2, t = lane32 & 3;
  const int S = a.split, G = WARPS / S, grp = warp / S, slice = warp % S;
  const int n_cc = a.pl.n_cc;
  const int c_lo = (n_cc * slice) / S, c_hi = (n_cc * (slice + 1)) / S;
  const int n_units = PAIR ? a.pl.n_rb / 2 : a.pl.n_rb;
  const int Q = a.slots, q = blockIdx.x * G + grp;
  const int my_units = (q < n_units && q < Q) ? (n_units - q + Q - 1) / Q : 0;
  const int P = a.piece, D = a.depth;
  const int np = (c_hi - c_lo + P - 1) / P;  // pieces a unit
  const int n_pieces = my_units * np;
  const int slot_bytes = H * P * GEMV_PIECE_BYTES;
  uint64_t *mb = bars + warp * D;
  unsigned char *mr = ring + (size_t)warp * D * slot_bytes;

  const uint64_t policy = l2_evict_first();
  // piece n of this warp: unit q + (n / np) Q, chunks from c_lo + (n % np) P
  auto issue = [&](int n) {
    const int unit = q + (n / np) * Q, c0 = c_lo + (n % np) * P;
    const int nc = min(P, c_hi - c0);
    uint64_t *bar = &mb[n % D];
    unsigned char *dst = mr + (size_t)(n % D) * slot_bytes;
    mbar_expect(bar, (uint32_t)(H * nc * GEMV_PIECE_BYTES));
#pragma unroll
    for (int h = 0; h < H; ++h) {
      const size_t tile = (size_t)(PAIR ? 2 * unit + h : unit) * n_cc + c0;
      bulk_load(dst + h * P * 512, a.pl.tiles + tile * 32, (uint32_t)(nc * 512), bar, policy);
      bulk_load(dst + H * P * 512 + h * P * 64, a.pl.scales + tile * 8, (uint32_t)(nc * 64), bar, policy);
    }
  };
  if (lane32 == 0) {
    for (int d = 0; d < D; ++d) mbar_init(&mb[d], 1);
    mbar_init_fence();
    for (int n = 0; n < D && n < n_pieces; ++n) issue(n);
  }
  __syncwarp();

  pdl_wait();
  // the multiplier of the GELU product, loaded now so its latency hides
  // behind the prologue (this thread's outputs: rows unit*16 + g (+8), lanes 2t+k)
  float mul_pre[NT][4];
  if (EPI == EPI_GELU_MUL && slice == 0 && my_units == 1) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int row = q * 16 + g + (i >= 2 ? 8 : 0);
        const int ln = MODE == MODE_PACK ? 2 * t + (i & 1) : nt * 8 + 2 * t + (i & 1);
        const bool ok = row < a.pl.rows && ln < a.lanes && !(MODE == MODE_PACK && t >= 2);
        mul_pre[nt][i] = ok ? a.aux[(size_t)ln * a.aux_stride + row] : 0.0f;
      }
  }
  if constexpr (PRO == PRO_F32S)
    gemv_prologue_scaled<MODE, WARPS>(a, stage, scr);
  else
    gemv_prologue<PRO, MODE, WARPS>(a, stage, scr);
  // the next kernel may start (and fetch its weights) once this one is past
  // its own wait: released any earlier, kernels still waiting would release
  // the ones after them and pile up on the SMs
  pdl_release();

  // the epilogue factor of the lanes each accumulator column holds
  float sh[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int ln = MODE == MODE_PACK ? (2 * t + k) & 3 : nt * 8 + 2 * t + k;
      sh[nt][k] = scr[SCR_FACTOR + ln];
    }

  // EPI_LOGITS running argmax, EPI_STORE running sum of squares, per (nt, lane parity)
  float best_v[NT][2];
  int best_i[NT][2];
  float ssq[NT][2], mag[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    best_v[nt][0] = best_v[nt][1] = -FLT_MAX;
    best_i[nt][0] = best_i[nt][1] = 0x7fffffff;
    ssq[nt][0] = ssq[nt][1] = 0.0f;
    mag[nt][0] = mag[nt][1] = 0.0f;
  }

  bool failed = false;
  int n = 0;
  for (int u = 0; u < my_units; ++u) {
    const int unit = q + u * Q;
    float acc[H][ACC];
#pragma unroll
    for (int h = 0; h < H; ++h)
#pragma unroll
      for (int i = 0; i < ACC; ++i) acc[h][i] = 0.0f;

    for (int k = 0; k < np; ++k, ++n) {
      const int c0 = c_lo + k * P, nc = min(P, c_hi - c0);
      const int d = n % D;
      if (!mbar_wait(&mb[d], (uint32_t)((n / D) & 1), failed ? 1 : (1 << 22))) {
        if (!failed && lane32 == 0) atomicOr(a.err, 1);
        failed = true;
      }
      const unsigned char *src = mr + (size_t)d * slot_bytes;
      const uint4 *wt = reinterpret_cast<const uint4 *>(src);
      const uint2 *ws = reinterpret_cast<const uint2 *>(src + H * P * 512);
#pragma unroll 2
      for (int c = 0; c < nc; ++c) {
        const uint32_t *sc = stage + (size_t)(c0 + c) * stage_chunk_words(MODE);
#pragma unroll
        for (int h = 0; h < H; ++h)
          chunk_product<MODE>(wt[h * P * 32 + c * 32 + lane32], ws[h * P * 8 + c * 8 + g], sc, lane32, acc[h]);
      }
      __syncwarp();
      if (lane32 == 0 && n + D < n_pieces && !failed) {
        fence_async_smem();
        issue(n + D);
      }
    }

    // the S warps of the group add their slices in a fixed order
    if (S > 1) {
      float *mine = red + (size_t)threadIdx.x * (H * ACC);
#pragma unroll
      for (int h = 0; h < H; ++h)
#pragma unroll
        for (int i = 0; i < ACC; ++i) mine[h * ACC + i] = acc[h][i];
      named_sync(1 + grp, S * 32);
      if (slice == 0) {
        for (int o = 1; o < S; ++o) {
          const float *other = red + (size_t)(threadIdx.x + o * 32) * (H * ACC);
#pragma unroll
          for (int h = 0; h < H; ++h)
#pragma unroll
            for (int i = 0; i < ACC; ++i) acc[h][i] += other[h * ACC + i];
        }
      }
      named_sync(1 + grp, S * 32);
    }

    if (slice == 0) {
      // hi + lo for each output: PACK adds the lo columns (threads t + 2)
      float v[H][NT][4];
#pragma unroll
      for (int h = 0; h < H; ++h)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            if (MODE == MODE_PACK) {
              const float lo = __shfl_xor_sync(0xffffffffu, acc[h][i], 2);
              v[h][nt][i] = acc[h][i] + lo;
            } else {
              v[h][nt][i] = acc[h][nt * 8 + i] + acc[h][nt * 8 + 4 + i];
            }
          }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int row = unit * 16 + g + (i >= 2 ? 8 : 0);
          const int k = i & 1;
          const int ln = MODE == MODE_PACK ? 2 * t + k : nt * 8 + 2 * t + k;
          if (MODE == MODE_PACK && t >= 2) continue;
          if (row >= a.pl.rows || ln >= a.lanes) continue;
          const float x = v[0][nt][i] * sh[nt][k];
          if (EPI == EPI_STORE) {
            const float o = x * a.out_scale;
            a.out[(size_t)ln * a.out_stride + row] = o;
            ssq[nt][k] += o * o;
            mag[nt][k] = fmaxf(mag[nt][k], fabsf(o));
          } else if (EPI == EPI_GELU_PAIR) {
            const float o = gelu_tanh(x) * (v[PAIR][nt][i] * sh[nt][k]);
            a.out[(size_t)ln * a.out_stride + row] = o;
            mag[nt][k] = fmaxf(mag[nt][k], fabsf(o));
          } else if (EPI == EPI_GELU_MUL) {
            const float mul = my_units == 1 ? mul_pre[nt][i] : a.aux[(size_t)ln * a.aux_stride + row];
            const float o = gelu_tanh(x) * mul;
            a.out[(size_t)ln * a.out_stride + row] = o;
            mag[nt][k] = fmaxf(mag[nt][k], fabsf(o));
          } else {  // EPI_LOGITS
            const float cv = a.cap > 0.0f ? logit_cap(x, a.cap) : x;
            a.out[(size_t)ln * a.out_stride + row] = cv;
            if (cv > best_v[nt][k] || (cv == best_v[nt][k] && row < best_i[nt][k])) {
              best_v[nt][k] = cv;
              best_i[nt][k] = row;
            }
          }
        }
    }
  }

  if (EPI == EPI_STORE && a.out_ssq) {
    // per-lane sums of squares of this block's outputs: across the 8 thread
    // groups that hold the same lanes, then across warps in order
    __syncthreads();
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        float v = ssq[nt][k];
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        const int ln = nt * 8 + 2 * t + k;
        if (g == 0) red[warp * 16 + ln] = (MODE == MODE_PACK && t >= 2) ? 0.0f : v;
      }
    __syncthreads();
    // one partial per virtual 8-warp block: warps 8h .. 8h + 7
    const int n_vb = (Q + a.vgroups - 1) / a.vgroups;
    if (threadIdx.x < (WARPS / 8) * 16) {
      const int h = threadIdx.x >> 4, ln = threadIdx.x & 15;
      const int vb = blockIdx.x * (WARPS / 8) + h;
      if (ln < NT * 8 && vb < n_vb) {
        float v = 0.0f;
        for (int w = 8 * h; w < 8 * h + 8; ++w) v += red[w * 16 + ln];
        a.out_ssq[ln * GEMV_PART_LIMIT + vb] = v;
      }
    }
  }

  if (EPI != EPI_LOGITS && a.out_amax) {
    // per-lane largest |out| of each virtual 8-warp block, for the consumer's
    // one-pass staging (a maximum: any order gives the same value)
    __syncthreads();
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        float v = mag[nt][k];
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
        const int ln = nt * 8 + 2 * t + k;
        if (g == 0) red[warp * 16 + ln] = (MODE == MODE_PACK && t >= 2) ? 0.0f : v;
      }
    __syncthreads();
    const int n_vb = (Q + a.vgroups - 1) / a.vgroups;
    if (threadIdx.x < (WARPS / 8) * 16) {
      const int h = threadIdx.x >> 4, ln = threadIdx.x & 15;
      const int vb = blockIdx.x * (WARPS / 8) + h;
      if (ln < NT * 8 && vb < n_vb) {
        float v = 0.0f;
        for (int w = 8 * h; w < 8 * h + 8; ++w) v = fmaxf(v, red[w * 16 + ln]);
        a.out_amax[ln * GEMV_PART_LIMIT + vb] = v;
      }
    }
  }

  if (EPI == EPI_LOGITS) {
    // reduce across the 8 thread groups that hold the same lanes, then across
    // the warps of the block; block partials go to part_val / part_idx
    __shared__ float bv[GEMV_MAX_WARPS][16];
    __shared__ int bi[GEMV_MAX_WARPS][16];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        float v = best_v[nt][k];
        int i = best_i[nt][k];
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
          float ov = __shfl_xor_sync(0xffffffffu, v, o);
          int oi = __shfl_xor_sync(0xffffffffu, i, o);
          if (ov > v || (ov == v && oi < i)) {
            v = ov;
            i = oi;
          }
        }
        if (g == 0) {
          bv[warp][nt * 8 + 2 * t + k] = v;
          bi[warp][nt * 8 + 2 * t + k] = i;
        }
      }
    __syncthreads();
    const int n_vb = (Q + a.vgroups - 1) / a.vgroups;
    if (threadIdx.x < (WARPS / 8) * 16) {
      const int h = threadIdx.x >> 4, ln = threadIdx.x & 15;
      const int vb = blockIdx.x * (WARPS / 8) + h;
      if (ln < NT * 8 && vb < n_vb) {
        float v = bv[8 * h][ln];
        int i = bi[8 * h][ln];
        for (int w = 8 * h + 1; w < 8 * h + 8; ++w) {
          float ov = bv[w][ln];
          int oi = bi[w][ln];
          if (ov > v || (ov == v && oi < i)) {
            v = ov;
            i = oi;
          }
        }
        a.part_val[vb * 16 + ln] = v;
        a.part_idx[vb * 16 + ln] = i;
      }
    }
  }
}
// ---------------------------------------------------------------------------
// embedding rows (app_core.c:11863-11874, :11886-11891)
// bf16 -> f32 of eight values, times `gain`.
__device__ __forceinline__ void bf16x8_scaled(const uint4 &w, float gain, float4 &a, float4 &b) {
  a = make_float4(__uint_as_float(w.x << 16) * gain, __uint_as_float(w.x & 0xffff0000u) * gain,
                  __uint_as_float(w.y << 16) * gain, __uint_as_float(w.y & 0xffff0000u) * gain);
  b = make_float4(__uint_as_float(w.z << 16) * gain, __uint_as_float(w.z & 0xffff0000u) * gain,
                  __uint_as_float(w.w << 16) * gain, __uint_as_float(w.w & 0xffff0000u) * gain);
}

// Blocks (lane, slice): each takes every gridDim.y-th run of eight values of
// the lane's embedding row and per-layer-embedding row, 16-byte loads
// (widths are multiples of eight; rows start 16-byte aligned).
__global__ void embed_kernel(const int32_t *ids, int lanes, const uint16_t *embed, int hidden,
                             float embed_gain, const uint16_t *ple_embed, int ple_vocab,
                             int ple_width, float ple_gain, float *x_out, float *seed_out) {
  pdl_release();
  const int j = blockIdx.x;
  if (j >= lanes) return;
  const int id = ids[j];
  const int step = gridDim.y * blockDim.x, first = blockIdx.y * blockDim.x + threadIdx.x;
  const uint4 *row = reinterpret_cast<const uint4 *>(embed + (size_t)id * hidden);
  float4 *xo = reinterpret_cast<float4 *>(x_out + (size_t)j * hidden);
  for (int i = first; i < hidden / 8; i += step) {
    float4 a, b;
    bf16x8_scaled(row[i], embed_gain, a, b);
    xo[2 * i] = a;
    xo[2 * i + 1] = b;
  }
  if (ple_embed) {
    const uint4 *srow = reinterpret_cast<const uint4 *>(ple_embed + (size_t)(id % ple_vocab) * ple_width);
    float4 *so = reinterpret_cast<float4 *>(seed_out + (size_t)j * ple_width);
    for (int i = first; i < ple_width / 8; i += step) {
      float4 a, b;
      bf16x8_scaled(srow[i], ple_gain, a, b);
      so[2 * i] = a;
      so[2 * i + 1] = b;
    }
  }
}

// app_core.c:11892-11903: each per-layer chunk normed with the shared weight,
// then (chunk + seed) / sqrt(2).  One block a (lane, chunk).
__global__ void ple_finish_kernel(const float *raw, const float *seed, int lanes, int layers,
                                  int ple_dim, const float *w, float eps, float blend, float *out) {
  pdl_release();
  pdl_wait();
  int j = blockIdx.x / layers, c = blockIdx.x % layers;
  if (j >= lanes) return;
  int width = layers * ple_dim;
  const float *v = raw + (size_t)j * width + (size_t)c * ple_dim;
  const float *sd = seed + (size_t)j * width + (size_t)c * ple_dim;
  __shared__ float part[32];
  float s = 0.0f;
  for (int i = threadIdx.x; i < ple_dim; i += blockDim.x) s += v[i] * v[i];
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0.0f;
    t = warp_sum(t);
    if (threadIdx.x == 0) part[0] = t;
  }
  __syncthreads();
  float sh = (float)(1.0 / sqrt((double)part[0] / (double)ple_dim + (double)eps));
  float *o = out + (size_t)j * width + (size_t)c * ple_dim;
  for (int i = threadIdx.x; i < ple_dim; i += blockDim.x) o[i] = (v[i] * sh * w[i] + sd[i]) * blend;
}

// ---------------------------------------------------------------------------
// attention (app_core.c:11455 session_attend, :11415 session_attend_group,
// :11296 attend_score_band, :11333 attend_blend_band): for each (lane, head)
// pair, the query normed and turned (app_core.c:11492-11494), scores with
// scale 1.0 (app_core.c:11314) over the lane's own span ([pos - window + 1,
// pos] on sliding layers, [0, pos] on global ones, app_core.c:11515-11518),
// softmax, weighted values.  On an owner layer the block's new key and value
// rows are normed, turned and written into the cache here too
// (app_core.c:11505-11512).
//
// The span is cut into chunks whose boundaries sit at fixed multiples of the
// session's chunk length, so a position's partial sums never depend on how
// many lanes a pass carried.  A block takes eight pairs, one a warp, and
// walks chunks blockIdx.x, + gridDim.x, ...  Per 16-position tile, threads
// l and l + 16 of a warp score position l over the two halves of the head
// (the query read from shared memory by broadcast, the key row padded so the
// warp's reads do not collide) and add their halves; the warp updates its
// online softmax, and then thread l blends dimensions [l*DPL, (l+1)*DPL) of
// the values.  Partials per chunk go to attn_combine_kernel.
constexpr int ATT_T = 16;        // positions a tile
constexpr int ATT_PAIRS = 8;     // (lane, head) pairs a block, one a warp
constexpr int ATT_BLOCK_ROWS = 16;  // block positions a chunk can hold

__host__ __device__ inline size_t attn_smem_floats(int hd, int kv_w) {
  const size_t ks = (size_t)kv_w + 4;
  return (size_t)ATT_PAIRS * hd + 2 * (size_t)ATT_T * ks + 2 * (size_t)ATT_BLOCK_ROWS * ks;
}

template <int DPL>
__device__ __forceinline__ void load_dpl(const float *src, float (&v)[DPL]) {
  if constexpr (DPL % 4 == 0) {
#pragma unroll
    for (int e = 0; e < DPL; e += 4) {
      const float4 x = *reinterpret_cast<const float4 *>(src + e);
      v[e] = x.x;
      v[e + 1] = x.y;
      v[e + 2] = x.z;
      v[e + 3] = x.w;
    }
  } else {
#pragma unroll
    for (int e = 0; e < DPL; ++e) v[e] = src[e];
  }
}

template <int DPL>
__device__ __forceinline__ void store_dpl(float *dst, const float (&v)[DPL]) {
  if constexpr (DPL % 4 == 0) {
#pragma unroll
    for (int e = 0; e < DPL; e += 4) *reinterpret_cast<float4 *>(dst + e) = make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
  } else {
#pragma unroll
    for (int e = 0; e < DPL; ++e) dst[e] = v[e];
  }
}

// The blend's dimensions of thread l: with four or more a thread, the
// float4s l, l + 32, ... of the head (consecutive threads on consecutive
// banks); with fewer, the DPL consecutive dimensions from l * DPL.
template <int DPL>
__device__ __forceinline__ void load_blend(const float *row, int l, float (&v)[DPL]) {
  if constexpr (DPL % 4 == 0) {
#pragma unroll
    for (int k = 0; k < DPL / 4; ++k) {
      const float4 x = reinterpret_cast<const float4 *>(row)[l + 32 * k];
      v[4 * k] = x.x;
      v[4 * k + 1] = x.y;
      v[4 * k + 2] = x.z;
      v[4 * k + 3] = x.w;
    }
  } else {
    load_dpl<DPL>(row + l * DPL, v);
  }
}

template <int DPL>
__device__ __forceinline__ void store_blend(float *row, int l, const float (&v)[DPL]) {
  if constexpr (DPL % 4 == 0) {
#pragma unroll
    for (int k = 0; k < DPL / 4; ++k)
      reinterpret_cast<float4 *>(row)[l + 32 * k] = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
  } else {
    store_dpl<DPL>(row + l * DPL, v);
  }
}

// One head of 32 * DPL dimensions, DPL a thread: normed (app_core.c:4667,
// double mean of squares) with an optional gain, then turned by the rope
// tables of its position (pairs (d, d + hd/2), threads l and l + 16).
template <int DPL>
__device__ __forceinline__ void head_norm_turn(float (&v)[DPL], const float *gain, const float *cs, const float *sn,
                                               float eps, bool turn, int l) {
  constexpr int HD = 32 * DPL;
  float c_[DPL], s_[DPL];
  if (turn) {
    const int d0 = (l & 15) * DPL;
#pragma unroll
    for (int e = 0; e < DPL; ++e) {
      c_[e] = cs[d0 + e];
      s_[e] = sn[d0 + e];
    }
  }
  float s = 0.0f;
#pragma unroll
  for (int e = 0; e < DPL; ++e) s += v[e] * v[e];
  s = warp_sum(s);
  const float sh = (float)(1.0 / sqrt((double)s / (double)HD + (double)eps));
#pragma unroll
  for (int e = 0; e < DPL; ++e) v[e] = gain ? v[e] * sh * gain[l * DPL + e] : v[e] * sh;
  if (turn) {
    float other[DPL];
#pragma unroll
    for (int e = 0; e < DPL; ++e) other[e] = __shfl_xor_sync(0xffffffffu, v[e], 16);
#pragma unroll
    for (int e = 0; e < DPL; ++e) v[e] = l < 16 ? v[e] * c_[e] - other[e] * s_[e] : v[e] * c_[e] + other[e] * s_[e];
  }
}

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

template <int DPL>
__global__ void __launch_bounds__(256) attn_kernel(const float *qkv, int qkv_stride, int heads, int kv_heads,
                                                   const float *q_norm, const float *k_norm, const float *cs_tab,
                                                   const float *sn_tab, float eps, int owner, float *kc, float *vc,
                                                   int sliding, int span, const int *d_p0, int lanes, int chunk_len,
                                                   float *part_ml, float *part_acc) {
  constexpr int HD = DPL * 32;
  const int kv_w = kv_heads * HD, KS = kv_w + 4, half = HD / 2;
  extern __shared__ __align__(16) float sm[];
  float *qs = sm;                                // [8][HD]
  float *ks = qs + ATT_PAIRS * HD;               // [ATT_T][KS]
  float *vs = ks + (size_t)ATT_T * KS;           // [ATT_T][KS]
  float *bk = vs + (size_t)ATT_T * KS;           // [16][KS] the block's new keys (owner layers)
  float *bv = bk + (size_t)ATT_BLOCK_ROWS * KS;  // [16][KS] and values
  const int warp = threadIdx.x >> 5, l = threadIdx.x & 31;
  pdl_release();
  pdl_wait();
  const int p0 = *d_p0;
  const int lo_all = sliding ? max(0, p0 - span + 1) : 0;
  const int hi_all = p0 + lanes;
  const int c_first = lo_all / chunk_len;
  const int n_chunks = (hi_all - 1) / chunk_len - c_first + 1;
  if ((int)blockIdx.x >= n_chunks) return;

  // this warp's query, normed and turned at its lane's position
  const int pair = blockIdx.y * ATT_PAIRS + warp;
  const bool has = pair < lanes * heads;
  const int j = has ? pair / heads : 0, h = has ? pair - (pair / heads) * heads : 0;
  const int kvoff = (h / (heads / kv_heads)) * HD;
  if (has) {
    float qv[DPL];
    load_dpl<DPL>(qkv + (size_t)j * qkv_stride + (size_t)h * HD + l * DPL, qv);
    const int pos = p0 + j;
    head_norm_turn<DPL>(qv, q_norm, cs_tab + (size_t)pos * half, sn_tab + (size_t)pos * half, eps, true, l);
    store_dpl<DPL>(qs + warp * HD + l * DPL, qv);
  }
  // the pair this warp scores: its lane's span
  const int lane_lo = sliding ? max(0, p0 + j - span + 1) : 0;
  const int lane_hi = p0 + j;
  const int r_pos = l & (ATT_T - 1), hhalf = l >> 4;  // position and head half this thread scores
  const int w4 = kv_w / 4;

  for (int cr = blockIdx.x; cr < n_chunks; cr += gridDim.x) {
    const int c = c_first + cr;
    const int c_lo = max(c * chunk_len, lo_all), c_hi = min((c + 1) * chunk_len, hi_all);
    __syncthreads();  // the previous chunk's block rows and tiles are consumed
    // an owner layer's new keys and values that fall in this chunk: normed,
    // turned (keys), kept in shared memory, and written to the cache once
    int jb_lo = 0, jb_hi = 0;
    if (owner) {
      jb_lo = max(0, c * chunk_len - p0);
      jb_hi = min(lanes, (c + 1) * chunk_len - p0);
      const int per = 2 * kv_heads, items = max(0, jb_hi - jb_lo) * per;
      for (int it = warp; it < items; it += ATT_PAIRS) {
        const int jj = jb_lo + it / per, rest = it % per, kh = rest >> 1, is_v = rest & 1;
        float v[DPL];
        load_dpl<DPL>(qkv + (size_t)jj * qkv_stride + (size_t)heads * HD + (is_v ? kv_w : 0) + kh * HD + l * DPL, v);
        const int pos = p0 + jj;
        head_norm_turn<DPL>(v, is_v ? nullptr : k_norm, cs_tab + (size_t)pos * half, sn_tab + (size_t)pos * half, eps,
                            !is_v, l);
        store_dpl<DPL>((is_v ? bv : bk) + (size_t)(jj - jb_lo) * KS + kh * HD + l * DPL, v);
        if (blockIdx.y == 0) store_dpl<DPL>((is_v ? vc : kc) + (size_t)pos * kv_w + kh * HD + l * DPL, v);
      }
    }

    float m_run = -FLT_MAX, l_run = 0.0f, acc[DPL];
#pragma unroll
    for (int e = 0; e < DPL; ++e) acc[e] = 0.0f;
    for (int tb = c * chunk_len; tb < c_hi; tb += ATT_T) {
      if (tb + ATT_T <= c_lo) continue;
      __syncthreads();  // the previous tile is consumed (and the query and block rows are written)
      for (int i = threadIdx.x; i < ATT_T * w4; i += blockDim.x) {
        const int r = i / w4, d4 = i - r * w4, pos = tb + r;
        float *kd = ks + (size_t)r * KS + d4 * 4, *vd = vs + (size_t)r * KS + d4 * 4;
        if (pos < c_lo || pos >= c_hi) {
          *reinterpret_cast<float4 *>(kd) = make_float4(0.f, 0.f, 0.f, 0.f);
          *reinterpret_cast<float4 *>(vd) = make_float4(0.f, 0.f, 0.f, 0.f);
        } else if (owner && pos - p0 >= jb_lo && pos - p0 < jb_hi) {
          const int rb = pos - p0 - jb_lo;
          *reinterpret_cast<float4 *>(kd) = *reinterpret_cast<const float4 *>(bk + (size_t)rb * KS + d4 * 4);
          *reinterpret_cast<float4 *>(vd) = *reinterpret_cast<const float4 *>(bv + (size_t)rb * KS + d4 * 4);
        } else {
          cp_async16(kd, kc + (size_t)pos * kv_w + d4 * 4);
          cp_async16(vd, vc + (size_t)pos * kv_w + d4 * 4);
        }
      }
      asm volatile("cp.async.wait_all;\n" ::: "memory");
      __syncthreads();
      if (has) {
        // scores: threads r and r + 16 take the even and odd float4s of
        // position tb + r (the two halves' query reads then fall in
        // different banks)
        const int pos = tb + r_pos;
        const float4 *qr = reinterpret_cast<const float4 *>(qs + warp * HD) + hhalf;
        const float4 *kr = reinterpret_cast<const float4 *>(ks + (size_t)r_pos * KS + kvoff) + hhalf;
        float a0 = 0.f, a1 = 0.f;
#pragma unroll 4
        for (int m = 0; m < HD / 8; m += 2) {
          const float4 q0 = qr[2 * m], k0 = kr[2 * m];
          a0 = fmaf(q0.x, k0.x, a0); a0 = fmaf(q0.y, k0.y, a0); a0 = fmaf(q0.z, k0.z, a0); a0 = fmaf(q0.w, k0.w, a0);
          if (m + 1 < HD / 8) {
            const float4 q1 = qr[2 * m + 2], k1 = kr[2 * m + 2];
            a1 = fmaf(q1.x, k1.x, a1); a1 = fmaf(q1.y, k1.y, a1); a1 = fmaf(q1.z, k1.z, a1); a1 = fmaf(q1.w, k1.w, a1);
          }
        }
        const float part = a0 + a1;
        const float other = __shfl_xor_sync(0xffffffffu, part, 16);
        const float s = hhalf == 0 ? part + other : other + part;  // the same sum in both threads
        const bool valid = pos >= c_lo && pos < c_hi && pos >= lane_lo && pos <= lane_hi;
        const float sc = valid ? s : -FLT_MAX;
        // online softmax over the tile's 16 positions (each held twice)
        const float m_new = fmaxf(m_run, warp_max(sc));
        const float f = (m_new == -FLT_MAX) ? 1.0f : (m_run == -FLT_MAX ? 0.0f : expf(m_run - m_new));
        const float pe = valid ? expf(sc - m_new) : 0.0f;
        float psum = pe;
#pragma unroll
        for (int o = 1; o < ATT_T; o <<= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o);
        l_run = l_run * f + psum;
        m_run = m_new;
#pragma unroll
        for (int e = 0; e < DPL; ++e) acc[e] *= f;
        // blend: thread l takes the dimensions of blend_dim(l, e) of every
        // position (float4s l, l + 32, ... where the head has them)
#pragma unroll 4
        for (int r = 0; r < ATT_T; ++r) {
          const float pr = __shfl_sync(0xffffffffu, pe, r);
          float vv[DPL];
          load_blend<DPL>(vs + (size_t)r * KS + kvoff, l, vv);
#pragma unroll
          for (int e = 0; e < DPL; ++e) acc[e] = fmaf(pr, vv[e], acc[e]);
        }
      }
    }
    if (has) {
      const size_t slot = ((size_t)cr * 16 + j) * heads + h;
      if (l == 0) {
        part_ml[slot * 2 + 0] = m_run;
        part_ml[slot * 2 + 1] = l_run;
      }
      store_blend<DPL>(part_acc + slot * HD, l, acc);
    }
  }
}

// attention, second step: the chunks' partials merged into each head's
// output, (sum_c acc_c e^{m_c - M}) / (sum_c l_c e^{m_c - M}).  Blocks
// (lane, head, 64-dimension slice).  Every sum is keyed on the absolute
// chunk index, so a chunk outside a lane's span (zero weight, zero partials)
// changes nothing and the result does not depend on how many lanes shared
// the pass: warp 0's thread t adds the weighted l_c of chunks c = t mod 32 in
// ascending order and the warp adds the 32 sums in a fixed tree; thread
// (g, d) adds acc_c of chunks c = g mod 4 in ascending order and the four
// groups are added in order.
constexpr int COMB_GROUPS = 4, COMB_DIMS = 64;

__global__ void __launch_bounds__(COMB_GROUPS * COMB_DIMS) attn_combine_kernel(const float *part_ml, const float *part_acc,
                                                                               int lanes, int heads, int hd, int sliding,
                                                                               int span, int chunk_len, const int *d_p0,
                                                                               float *out, int out_stride,
                                                                               float *out_amax) {
  __shared__ float wgt[1024];
  __shared__ float grp[COMB_GROUPS][COMB_DIMS];
  __shared__ float tot;
  pdl_release();
  pdl_wait();
  const int slices = (hd + COMB_DIMS - 1) / COMB_DIMS;
  const int pair = blockIdx.x / slices, dslice = blockIdx.x - pair * slices;
  const int j = pair / heads, h = pair % heads;
  if (j >= lanes) return;
  const int p0 = *d_p0;
  const int lo_all = sliding ? max(0, p0 - span + 1) : 0;
  const int hi_all = p0 + lanes;
  const int c_first = lo_all / chunk_len;
  const int n_chunks = (hi_all - 1) / chunk_len - c_first + 1;
  const size_t cstride = (size_t)16 * heads;  // slots between chunks
  const size_t s0 = (size_t)j * heads + h;
  if (threadIdx.x < 32) {
    constexpr int MAXC = 1024 / 32;
    // thread t holds the chunks whose absolute index is t mod 32
    const int t0 = (threadIdx.x - c_first % 32 + 32) % 32;  // first relative chunk of this thread
    float m[MAXC], lv[MAXC];
#pragma unroll
    for (int i = 0; i < MAXC; ++i) {
      const int c = t0 + 32 * i;
      m[i] = c < n_chunks ? part_ml[(c * cstride + s0) * 2] : -FLT_MAX;
      lv[i] = c < n_chunks ? part_ml[(c * cstride + s0) * 2 + 1] : 0.0f;
    }
    float M = -FLT_MAX;
#pragma unroll
    for (int i = 0; i < MAXC; ++i) M = fmaxf(M, m[i]);
    M = warp_max(M);
    float L = 0.0f;
#pragma unroll
    for (int i = 0; i < MAXC; ++i) {
      const int c = t0 + 32 * i;
      const float w = (m[i] == -FLT_MAX) ? 0.0f : expf(m[i] - M);
      if (c < n_chunks) wgt[c] = w;
      L += lv[i] * w;
    }
    L = warp_sum(L);
    if (threadIdx.x == 0) tot = L;
  }
  __syncthreads();
  const int g = threadIdx.x / COMB_DIMS, dl = threadIdx.x - g * COMB_DIMS, d = dslice * COMB_DIMS + dl;
  float o = 0.0f;
  if (d < hd) {
    const int cg0 = (g - c_first % COMB_GROUPS + COMB_GROUPS) % COMB_GROUPS;  // first relative chunk of group g
#pragma unroll 4
    for (int c = cg0; c < n_chunks; c += COMB_GROUPS) o += part_acc[(c * cstride + s0) * hd + d] * wgt[c];
  }
  grp[g][dl] = o;
  __syncthreads();
  float v = 0.0f;
  if (threadIdx.x < COMB_DIMS && d < hd) {
    v = grp[0][dl];
#pragma unroll
    for (int q = 1; q < COMB_GROUPS; ++q) v += grp[q][dl];
    v *= 1.0f / tot;
    out[(size_t)j * out_stride + (size_t)h * hd + d] = v;
  }
  if (out_amax && threadIdx.x < COMB_DIMS) {
    // this block's largest |out|: one partial a (head, slice) for lane j
    __shared__ float amx[COMB_DIMS / 32];
    const float m = warp_max(fabsf(v));
    if ((threadIdx.x & 31) == 0) amx[threadIdx.x >> 5] = m;
    named_sync(1, COMB_DIMS);
    if (threadIdx.x == 0) out_amax[(size_t)j * GEMV_PART_LIMIT + h * slices + dslice] = fmaxf(amx[0], amx[1]);
  }
}

// argmax partials of the output head merged per lane (app_main.c:482: the
// first index of the largest value).  Thread (lane, stripe) scans parts
// stripe, stripe + 32, ...; the stripes then meet in shared memory.
__global__ void argmax_final_kernel(const float *part_val, const int *part_idx, int parts, int lanes,
                                    int32_t *top_out) {
  __shared__ float sv[32][16];
  __shared__ int si[32][16];
  pdl_release();
  pdl_wait();
  const int j = threadIdx.x & 15, stripe = threadIdx.x >> 4;
  float v = -FLT_MAX;
  int i = 0x7fffffff;
  for (int p = stripe; p < parts; p += 32) {
    float ov = part_val[p * 16 + j];
    int oi = part_idx[p * 16 + j];
    if (ov > v || (ov == v && oi < i)) {
      v = ov;
      i = oi;
    }
  }
  sv[stripe][j] = v;
  si[stripe][j] = i;
  __syncthreads();
  if (threadIdx.x < 16 && (int)threadIdx.x < lanes) {
    for (int s = 1; s < 32; ++s) {
      float ov = sv[s][j];
      int oi = si[s][j];
      if (ov > v || (ov == v && oi < i)) {
        v = ov;
        i = oi;
      }
    }
    top_out[j] = i;
  }
}

// rope tables: cos/sin of pos * step in double (app_core.c:8147 rope_wave)
__global__ void rope_table_kernel(const float *steps, int half, int window, float *cs, float *sn) {
  long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long)window * half) return;
  int pos = (int)(idx / half), i = (int)(idx % half);
  double a = (double)pos * (double)steps[i];
  double s, c;
  sincos(a, &s, &c);
  cs[idx] = (float)c;
  sn[idx] = (float)s;
}

// top candidates of each logit row for the sampler (app_core.c:14572
// pick_shape's top-k): every block sorts 2048 logits of one lane (echo
// penalty applied on the way in) and keeps its best `keep`; a second pass
// sorts the survivors.  Order: larger value first, lower id on a tie.
__device__ __forceinline__ bool cand_before(float av, int ai, float bv, int bi) {
  return av > bv || (av == bv && ai < bi);
}

template <int N>
__device__ void bitonic_sort(float *v, int *id) {
  for (int k = 2; k <= N; k <<= 1)
    for (int jj = k >> 1; jj > 0; jj >>= 1) {
      for (int i = threadIdx.x; i < N; i += blockDim.x) {
        int ixj = i ^ jj;
        if (ixj > i) {
          bool up = (i & k) == 0;
          bool sw = up ? cand_before(v[ixj], id[ixj], v[i], id[i])
                       : cand_before(v[i], id[i], v[ixj], id[ixj]);
          if (sw) {
            float tv = v[i];
            v[i] = v[ixj];
            v[ixj] = tv;
            int ti = id[i];
            id[i] = id[ixj];
            id[ixj] = ti;
          }
        }
      }
      __syncthreads();
    }
}

__global__ void topk_stage1_kernel(const float *logits, int vocab, int lanes, int keep,
                                   const int32_t *echo_ids, const int *echo_from, const int *echo_upto,
                                   float penalty, float *cand_v, int *cand_i) {
  __shared__ float v[2048];
  __shared__ int id[2048];
  int j = blockIdx.y, blk = blockIdx.x;
  if (j >= lanes) return;
  const float *row = logits + (size_t)j * vocab;
  int base = blk * 2048;
  int ef = echo_from ? echo_from[j] : 0, eu = echo_upto ? echo_upto[j] : 0;
  for (int i = threadIdx.x; i < 2048; i += blockDim.x) {
    int r = base + i;
    float x = r < vocab ? row[r] : -FLT_MAX;
    if (r < vocab && penalty != 1.0f) {
      bool hit = false;
      for (int e = ef; e < eu; ++e) hit |= (echo_ids[e] == r);
      if (hit) x = x > 0.0f ? x / penalty : x * penalty;
    }
    v[i] = x;
    id[i] = r < vocab ? r : 0x7fffffff;
  }
  __syncthreads();
  bitonic_sort<2048>(v, id);
  for (int i = threadIdx.x; i < keep; i += blockDim.x) {
    cand_v[((size_t)j * gridDim.x + blk) * keep + i] = v[i];
    cand_i[((size_t)j * gridDim.x + blk) * keep + i] = id[i];
  }
}

__global__ void topk_stage2_kernel(const float *cand_v, const int *cand_i, int n_cand, int keep,
                                   int lanes, float *top_v, int *top_i) {
  extern __shared__ __align__(16) unsigned char sm2[];
  int j = blockIdx.x;
  if (j >= lanes) return;
  int N = 1;
  while (N < n_cand) N <<= 1;
  float *v = reinterpret_cast<float *>(sm2);
  int *id = reinterpret_cast<int *>(v + N);
  for (int i = threadIdx.x; i < N; i += blockDim.x) {
    v[i] = i < n_cand ? cand_v[(size_t)j * n_cand + i] : -FLT_MAX;
    id[i] = i < n_cand ? cand_i[(size_t)j * n_cand + i] : 0x7fffffff;
  }
  __syncthreads();
  for (int k = 2; k <= N; k <<= 1)
    for (int jj = k >> 1; jj > 0; jj >>= 1) {
      for (int i = threadIdx.x; i < N; i += blockDim.x) {
        int ixj = i ^ jj;
        if (ixj > i) {
          bool up = (i & k) == 0;
          bool sw = up ? cand_before(v[ixj], id[ixj], v[i], id[i])
                       : cand_before(v[i], id[i], v[ixj], id[ixj]);
          if (sw) {
            float tv = v[i];
            v[i] = v[ixj];
            v[ixj] = tv;
            int ti = id[i];
            id[i] = id[ixj];
            id[ixj] = ti;
          }
        }
      }
      __syncthreads();
    }
  for (int i = threadIdx.x; i < keep; i += blockDim.x) {
    top_v[(size_t)j * keep + i] = v[i];
    top_i[(size_t)j * keep + i] = id[i];
  }
}

// elementwise entries of the backend table (app_core.c:4667, :4856, :5119,
// :5196), one block a call
__global__ void desk_norm_kernel(const float *x, const float *w, int n, float eps, float *out) {
  __shared__ float part[32];
  float s = 0.0f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s += x[i] * x[i];
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0.0f;
    t = warp_sum(t);
    if (threadIdx.x == 0) part[0] = t;
  }
  __syncthreads();
  float sh = (float)(1.0 / sqrt((double)part[0] / (double)n + (double)eps));
  for (int i = threadIdx.x; i < n; i += blockDim.x) out[i] = w ? x[i] * sh * w[i] : x[i] * sh;
}

__global__ void desk_softmax_kernel(float *x, int n) {
  __shared__ float part[32];
  __shared__ float bcast;
  float m = -FLT_MAX;
  for (int i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, x[i]);
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = part[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) t = fmaxf(t, part[w]);
    bcast = t;
  }
  __syncthreads();
  m = bcast;
  float s = 0.0f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    float e = expf(x[i] - m);
    x[i] = e;
    s += e;
  }
  s = warp_sum(s);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.0f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += part[w];
    bcast = t;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) x[i] /= bcast;
}

__global__ void desk_gelu_kernel(float *gate, const float *rise, int n) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    gate[i] = gelu_tanh(gate[i]) * rise[i];
}

__global__ void desk_rope_kernel(float *x, int head, const float *cs, const float *sn) {
  int half = head / 2;
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    float lo = x[i], hi = x[i + half];
    x[i] = lo * cs[i] - hi * sn[i];
    x[i + half] = hi * cs[i] + lo * sn[i];
  }
}

// ---------------------------------------------------------------------------
// launchers

// Whether launches from this thread may overlap the kernel ahead of them
// (programmatic dependent launch); the session turns it on while it records
// a pass, whose kernels all wait for their predecessor before touching its
// results.
static thread_local int g_pdl = 0;

template <typename... KArgs, typename... Args>
static cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                            Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = g_pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

static size_t align128(size_t x) { return (x + 127) & ~(size_t)127; }

// Shared memory of one launch: staged activations | scratch | reduction
// space | ring barriers | ring slots.
struct GemvLayout {
  size_t red, bars, ring, total;
};

static GemvLayout gemv_layout(const GemvArgs &a, int pair, int W, int P, int D) {
  const int MODE = gemv_mode(a.lanes), H = pair + 1;
  GemvLayout L;
  L.red = align128(gemv_stage_bytes(a.pl.n_cc, MODE) + SCR_FLOATS * 4);
  size_t red_floats = a.split > 1 ? (size_t)W * 32 * H * gemv_acc_floats(MODE) : 0;
  if (red_floats < (size_t)W * 16) red_floats = (size_t)W * 16;
  L.bars = align128(L.red + red_floats * 4);
  L.ring = align128(L.bars + (size_t)W * D * 8);
  L.total = L.ring + (size_t)W * D * H * P * GEMV_PIECE_BYTES;
  return L;
}

// Pieces and depth for a launch of `grid` blocks within `smem_limit`: every
// piece a warp will take in flight at once when they fit (one piece a unit),
// else four pieces in flight of as many chunks as fit.  Fills the layout
// fields of `a`; false when not even one chunk a warp fits.
static bool gemv_fit(GemvArgs &a, int pair, int W, int grid, size_t smem_limit, size_t *smem) {
  const int H = pair + 1, S = a.split, G = W / S;
  const int slen = (a.pl.n_cc + S - 1) / S;
  const int n_units = pair ? a.pl.n_rb / 2 : a.pl.n_rb;
  const int per_slot = (n_units + grid * G - 1) / (grid * G);
  const GemvLayout base = gemv_layout(a, pair, W, 0, GEMV_MAX_DEPTH);
  if (base.ring >= smem_limit) return false;
  const long per_warp = (long)(smem_limit - base.ring) / (W * H * GEMV_PIECE_BYTES);
  if (per_warp < 1) return false;
  int P, D;
  if ((long)per_slot * slen <= per_warp && per_slot <= GEMV_MAX_DEPTH) {
    P = slen;
    D = per_slot > 0 ? per_slot : 1;
  } else {
    D = per_warp < 4 ? (int)per_warp : 4;
    P = (int)(per_warp / D);
    if (P > slen) P = slen;
    const int pieces = (slen + P - 1) / P;
    P = (slen + pieces - 1) / pieces;
  }
  a.piece = P;
  a.depth = D;
  const GemvLayout L = gemv_layout(a, pair, W, P, D);
  a.off_red = (int)L.red;
  a.off_bars = (int)L.bars;
  a.off_ring = (int)L.ring;
  *smem = L.total;
  return L.total <= smem_limit;
}

template <int MODE, int WARPS, int PAIR>
static cudaError_t launch_gemv_pe(const GemvArgs &a, int pro, int epi, int grid, size_t smem, cudaStream_t st) {
#define IGC_CASE(P, E) \
  if (pro == P && epi == E) return launch_k(gemv_kernel<MODE, WARPS, PAIR, P, E>, dim3(grid), dim3(WARPS * 32), smem, st, a);
  if constexpr (PAIR) {
    IGC_CASE(PRO_RESID_NORM, EPI_GELU_PAIR)
    IGC_CASE(PRO_NORM, EPI_GELU_PAIR)
    IGC_CASE(PRO_F32, EPI_GELU_PAIR)
  } else {
    IGC_CASE(PRO_F32, EPI_STORE)
    IGC_CASE(PRO_F32S, EPI_STORE)
    IGC_CASE(PRO_NORM, EPI_STORE)
    IGC_CASE(PRO_RESID_NORM, EPI_STORE)
    IGC_CASE(PRO_RESID, EPI_GELU_MUL)
    IGC_CASE(PRO_RESID_NORM, EPI_LOGITS)
    IGC_CASE(PRO_NORM, EPI_LOGITS)
    IGC_CASE(PRO_F32, EPI_LOGITS)
  }
#undef IGC_CASE
  return cudaErrorInvalidValue;
}

// The opt-in limit covers static and dynamic shared memory together, so each
// kernel may ask for the limit less its own static part.
template <typename F>
static cudaError_t allow_smem_fn(F *fn, int bytes) {
  cudaFuncAttributes at;
  cudaError_t e = cudaFuncGetAttributes(&at, fn);
  if (e != cudaSuccess) return e;
  int dyn = bytes - (int)at.sharedSizeBytes;
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn > 0 ? dyn : 0);
  // one shared-memory split for every kernel of the pass, so an SM never
  // waits to re-split L1 between consecutive kernels
  if (e == cudaSuccess) e = cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  return e;
}

template <int MODE, int WARPS>
static cudaError_t allow_smem_mode(int bytes) {
  cudaError_t e = cudaSuccess;
#define IGC_ALLOW(PAIR, P, E) \
  if (e == cudaSuccess) e = allow_smem_fn(gemv_kernel<MODE, WARPS, PAIR, P, E>, bytes);
  IGC_ALLOW(1, PRO_RESID_NORM, EPI_GELU_PAIR)
  IGC_ALLOW(1, PRO_NORM, EPI_GELU_PAIR)
  IGC_ALLOW(1, PRO_F32, EPI_GELU_PAIR)
  IGC_ALLOW(0, PRO_F32, EPI_STORE)
  IGC_ALLOW(0, PRO_F32S, EPI_STORE)
  IGC_ALLOW(0, PRO_NORM, EPI_STORE)
  IGC_ALLOW(0, PRO_RESID_NORM, EPI_STORE)
  IGC_ALLOW(0, PRO_RESID, EPI_GELU_MUL)
  IGC_ALLOW(0, PRO_RESID_NORM, EPI_LOGITS)
  IGC_ALLOW(0, PRO_NORM, EPI_LOGITS)
  IGC_ALLOW(0, PRO_F32, EPI_LOGITS)
#undef IGC_ALLOW
  return e;
}

}  // namespace igc

using namespace igc;

extern "C" {

// Lets every kernel of this file use up to `bytes` of dynamic shared memory
// on the current device; called once per device before the first launch.
cudaError_t igc_kernels_configure(int bytes) {
  int dev = 0, optin = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (e != cudaSuccess) return e;
  if (bytes > optin) bytes = optin;
  e = allow_smem_mode<MODE_PACK, 16>(bytes);
  if (e == cudaSuccess) e = allow_smem_mode<MODE_PACK, 8>(bytes);
  if (e == cudaSuccess) e = allow_smem_mode<MODE_NT1, 16>(bytes);
  if (e == cudaSuccess) e = allow_smem_mode<MODE_NT1, 8>(bytes);
  if (e == cudaSuccess) e = allow_smem_mode<MODE_NT2, 8>(bytes);
  if (e == cudaSuccess) e = allow_smem_fn(attn_kernel<1>, bytes);
  if (e == cudaSuccess) e = allow_smem_fn(attn_kernel<2>, bytes);
  if (e == cudaSuccess) e = allow_smem_fn(attn_kernel<4>, bytes);
  if (e == cudaSuccess) e = allow_smem_fn(attn_kernel<8>, bytes);
  if (e == cudaSuccess) e = allow_smem_fn(topk_stage2_kernel, bytes);
  return e;
}

cudaError_t igc_launch_repack(const uint8_t *code, size_t row_stride, const uint16_t *scale, int groups,
                              int rows, int cols, int n_rb, int n_cc, int out_mul, int out_add, uint4 *tiles,
                              uint2 *scales, cudaStream_t st) {
  long total = (long)n_rb * n_cc * 32;
  int blocks = (int)((total + 255) / 256);
  repack_kernel<<<blocks, 256, 0, st>>>(code, row_stride, scale, groups, rows, cols, n_rb, n_cc, out_mul,
                                        out_add, tiles, scales);
  return cudaGetLastError();
}

void igc_kernels_pdl(int on) { g_pdl = on; }

cudaError_t igc_launch_gemv(GemvArgs *a, int pair, int pro, int epi, int grid, size_t smem_limit, cudaStream_t st,
                            int *grid_used) {
  if (a->pl.cols > GEMV_MAX_PARTS * 128) return cudaErrorInvalidValue;  // wider than the prologue's parts
  const int mode = gemv_mode(a->lanes);
  const int units = pair ? a->pl.n_rb / 2 : a->pl.n_rb;
  const int G8 = GEMV_WARPS / a->split;
  // 16-warp blocks where the mode allows them and their shared memory fits
  int W = GEMV_WARPS;
  if (mode != MODE_NT2 && gemv_layout(*a, pair, 16, 0, GEMV_MAX_DEPTH).ring + (size_t)16 * (pair + 1) * GEMV_PIECE_BYTES <=
                              smem_limit)
    W = 16;
  const int G = W / a->split;
  if (a->out_ssq) {
    // the planned 8-warp slots exactly, whatever the block width, so the
    // sums-of-squares partials group the same rows in every lane mode
    a->slots = grid * G8;
    grid = (a->slots + G - 1) / G;
  } else {
    if (grid > (units + G - 1) / G) grid = (units + G - 1) / G;
    if (grid < 1) grid = 1;
    a->slots = grid * G;
  }
  a->vgroups = G8;
  if (grid_used) *grid_used = (a->slots + G8 - 1) / G8;  // partials written: one a virtual 8-warp block
  size_t smem = 0;
  if (!gemv_fit(*a, pair, W, grid, smem_limit, &smem)) return cudaErrorInvalidValue;
  if (pro == PRO_F32 && a->x_amax) pro = PRO_F32S;
  if (mode == MODE_PACK)
    return W == 16 ? (pair ? launch_gemv_pe<MODE_PACK, 16, 1>(*a, pro, epi, grid, smem, st)
                           : launch_gemv_pe<MODE_PACK, 16, 0>(*a, pro, epi, grid, smem, st))
                   : (pair ? launch_gemv_pe<MODE_PACK, 8, 1>(*a, pro, epi, grid, smem, st)
                           : launch_gemv_pe<MODE_PACK, 8, 0>(*a, pro, epi, grid, smem, st));
  if (mode == MODE_NT1)
    return W == 16 ? (pair ? launch_gemv_pe<MODE_NT1, 16, 1>(*a, pro, epi, grid, smem, st)
                           : launch_gemv_pe<MODE_NT1, 16, 0>(*a, pro, epi, grid, smem, st))
                   : (pair ? launch_gemv_pe<MODE_NT1, 8, 1>(*a, pro, epi, grid, smem, st)
                           : launch_gemv_pe<MODE_NT1, 8, 0>(*a, pro, epi, grid, smem, st));
  return pair ? launch_gemv_pe<MODE_NT2, 8, 1>(*a, pro, epi, grid, smem, st)
              : launch_gemv_pe<MODE_NT2, 8, 0>(*a, pro, epi, grid, smem, st);
}

// The smallest ring of the narrowest block: one chunk a warp, with room for
// the deepest barriers.
size_t igc_gemv_smem_min(const GemvArgs *a, int pair) {
  return gemv_layout(*a, pair, GEMV_WARPS, 0, GEMV_MAX_DEPTH).ring + (size_t)GEMV_WARPS * (pair + 1) * GEMV_PIECE_BYTES;
}

cudaError_t igc_launch_embed(const int32_t *ids, int lanes, const uint16_t *embed, int hidden, float embed_gain,
                             const uint16_t *ple_embed, int ple_vocab, int ple_width, float ple_gain,
                             float *x_out, float *seed_out, cudaStream_t st) {
  if ((hidden & 7) || (ple_embed && (ple_width & 7))) return cudaErrorInvalidValue;
  embed_kernel<<<dim3(lanes, 8), 256, 0, st>>>(ids, lanes, embed, hidden, embed_gain, ple_embed, ple_vocab, ple_width,
                                      ple_gain, x_out, seed_out);
  return cudaGetLastError();
}

cudaError_t igc_launch_ple_finish(const float *raw, const float *seed, int lanes, int layers, int ple_dim,
                                  const float *w, float eps, float blend, float *out, cudaStream_t st) {
  return launch_k(ple_finish_kernel, dim3(lanes * layers), dim3(256), 0, st, raw, seed, lanes, layers, ple_dim, w, eps,
                  blend, out);
}

size_t igc_attn_smem(int hd, int kv_w) { return sizeof(float) * attn_smem_floats(hd, kv_w); }

cudaError_t igc_launch_attn(const float *qkv, int qkv_stride, int heads, int kv_heads, int hd, const float *q_norm,
                            const float *k_norm, const float *cs, const float *sn, float eps, int owner, float *kc,
                            float *vc, int sliding, int span, const int *d_p0, int lanes, int chunk_len, int grid_x,
                            float *part_ml, float *part_acc, float *out, int out_stride, float *out_amax,
                            cudaStream_t st) {
  const size_t smem = igc_attn_smem(hd, kv_heads * hd);
  const dim3 grid(grid_x, (lanes * heads + ATT_PAIRS - 1) / ATT_PAIRS);
  cudaError_t e;
#define IGC_ATT(D)                                                                                              \
  e = launch_k(attn_kernel<D>, grid, dim3(256), smem, st, qkv, qkv_stride, heads, kv_heads, q_norm, k_norm, cs, sn, \
               eps, owner, kc, vc, sliding, span, d_p0, lanes, chunk_len, part_ml, part_acc);
  switch (hd) {
    case 32: IGC_ATT(1) break;
    case 64: IGC_ATT(2) break;
    case 128: IGC_ATT(4) break;
    case 256: IGC_ATT(8) break;
    default: return cudaErrorInvalidValue;
  }
#undef IGC_ATT
  if (e != cudaSuccess) return e;
  const int slices = (hd + COMB_DIMS - 1) / COMB_DIMS;
  return launch_k(attn_combine_kernel, dim3(lanes * heads * slices), dim3(COMB_GROUPS * COMB_DIMS), 0, st, part_ml,
                  part_acc, lanes, heads, hd, sliding, span, chunk_len, d_p0, out, out_stride, out_amax);
}

cudaError_t igc_launch_argmax(const float *part_val, const int *part_idx, int parts, int lanes, int32_t *top,
                              cudaStream_t st) {
  return launch_k(argmax_final_kernel, dim3(1), dim3(512), 0, st, part_val, part_idx, parts, lanes, top);
}

cudaError_t igc_launch_rope_table(const float *steps, int half, int window, float *cs, float *sn,
                                  cudaStream_t st) {
  long total = (long)window * half;
  rope_table_kernel<<<(int)((total + 255) / 256), 256, 0, st>>>(steps, half, window, cs, sn);
  return cudaGetLastError();
}

cudaError_t igc_launch_topk(const float *logits, int vocab, int lanes, int keep, const int32_t *echo_ids,
                            const int *echo_from, const int *echo_upto, float penalty, float *cand_v, int *cand_i,
                            float *top_v, int *top_i, cudaStream_t st) {
  int blocks = (vocab + 2047) / 2048;
  dim3 g1(blocks, lanes);
  topk_stage1_kernel<<<g1, 512, 0, st>>>(logits, vocab, lanes, keep, echo_ids, echo_from, echo_upto, penalty,
                                         cand_v, cand_i);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  int n_cand = blocks * keep;
  int N = 1;
  while (N < n_cand) N <<= 1;
  size_t smem = (size_t)N * 8;
  topk_stage2_kernel<<<lanes, 1024, smem, st>>>(cand_v, cand_i, n_cand, keep, lanes, top_v, top_i);
  return cudaGetLastError();
}

cudaError_t igc_launch_desk_norm(const float *x, const float *w, int n, float eps, float *out, cudaStream_t st) {
  desk_norm_kernel<<<1, 256, 0, st>>>(x, w, n, eps, out);
  return cudaGetLastError();
}
cudaError_t igc_launch_desk_softmax(float *x, int n, cudaStream_t st) {
  desk_softmax_kernel<<<1, 1024, 0, st>>>(x, n);
  return cudaGetLastError();
}
cudaError_t igc_launch_desk_gelu(float *gate, const float *rise, int n, cudaStream_t st) {
  int blocks = (n + 255) / 256;
  if (blocks > 1024) blocks = 1024;
  desk_gelu_kernel<<<blocks, 256, 0, st>>>(gate, rise, n);
  return cudaGetLastError();
}
cudaError_t igc_launch_desk_rope(float *x, int head, const float *cs, const float *sn, cudaStream_t st) {
  desk_rope_kernel<<<1, 256, 0, st>>>(x, head, cs, sn);
  return cudaGetLastError();
}

}  // extern "C"
