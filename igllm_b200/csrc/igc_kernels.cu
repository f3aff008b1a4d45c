// igc_kernels.cu - the sm_100a kernels of the verify round.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <float.h>
#include <stdint.h>
#include <string.h>

#include "igc_gemv.cuh"
#include "igc_kernels.h"

namespace igc {

// ---------------------------------------------------------------------------
// upload repack: raw U8 codes of `bits` (1, 2 or 4) bits, packed from the low
// bit up (app_core.c:1757 pack_read: code c at bits [c*bits, (c+1)*bits) of
// its row, row_stride bytes a row), each the value plus 2^(bits-1), and f16
// scales [rows][groups of 32 columns] into the tile layout of igc_gemv.cuh,
// where every code is a 4-bit value + 8 (a 1- or 2-bit value fits exactly).
// One thread writes one thread-slot (16 bytes) of one tile and, for t == 0,
// that slot group's 8-byte scale record.
__global__ void repack_kernel(const uint8_t *code, size_t row_stride, int bits, const uint16_t *scale,
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
    const size_t bit = (size_t)c * bits;  // a code of 1, 2 or 4 bits never straddles a byte
    const uint32_t v = (uint32_t)(code[(size_t)r * row_stride + (bit >> 3)] >> (bit & 7)) & ((1u << bits) - 1u);
    return v + 8u - (1u << (bits - 1));
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
__global__ void __launch_bounds__(WARPS * 32, 1) gemv_kernel(GemvArgs args) {
  GemvArgs a = args;
  if (args.batches > 1) {
    const int j0 = blockIdx.y * args.lanes;
    a.lanes = min(args.lanes, args.lanes_total - j0);
    a.x += (size_t)j0 * args.x_stride;
    if (args.p) a.p += (size_t)j0 * args.p_stride;
    if (args.x_out) a.x_out += (size_t)j0 * args.x_stride;
    a.out += (size_t)j0 * args.out_stride;
    if (args.aux) a.aux += (size_t)j0 * args.aux_stride;
    if (args.p_ssq) a.p_ssq += (size_t)j0 * GEMV_PART_LIMIT;  // partials are lane-major
    if (args.out_ssq) a.out_ssq += (size_t)j0 * GEMV_PART_LIMIT;
    if (args.x_amax) a.x_amax += (size_t)j0 * GEMV_PART_LIMIT;
    if (args.out_amax) a.out_amax += (size_t)j0 * GEMV_PART_LIMIT;
  }
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

  // a residual prologue waits inside, once its first loads are out
  constexpr bool RES_PRO = PRO == PRO_RESID || PRO == PRO_RESID_NORM;
  if constexpr (!RES_PRO) {
    pdl_wait();
    stamp_begin(a.stamp);
  }
  // the multiplier of the GELU product (rows written at the start of the
  // pass), loaded now so its latency hides behind the prologue (this
  // thread's outputs: rows unit*16 + g (+8), lanes 2t+k)
  float mul_pre[NT][4];
  if (EPI == EPI_GELU_MUL && slice == 0 && my_units == 1) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int row = q * 16 + g + (i >= 2 ? 8 : 0);
        const int ln = MODE == MODE_PACK ? 2 * t + (i & 1) : nt * 8 + 2 * t + (i & 1);
        const bool ok = row < a.pl.rows && ln < a.lanes && !(MODE == MODE_PACK && t >= 2);
        mul_pre[nt][i] = ok ? __ldcg(a.aux + (size_t)ln * a.aux_stride + row) : 0.0f;
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
      // the warp agrees on the outcome: a lane whose poll gave up marks the
      // whole warp failed, so no lane computes on bytes that never arrived
      // unnoticed and every lane sees the same `failed` from here on
      const bool ok = mbar_wait(&mb[d], (uint32_t)((n / D) & 1), failed ? 1 : (1 << 22));
      const bool now_failed = __any_sync(0xffffffffu, !ok);
      if (now_failed && !failed && lane32 == 0) atomicOr(a.err, 1);
      failed = failed || now_failed;
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
      if (ln < a.lanes && vb < n_vb) {
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
      if (ln < a.lanes && vb < n_vb) {
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
      if (ln < a.lanes && vb < n_vb) {
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
  stamp_end(a.stamp);
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
                             int ple_width, float ple_gain, float *x_out, float *seed_out,
                             unsigned long long *stamp, int stamp_n, const float *peak, float *peak_saved,
                             int peak_n, EmbedCodes eq, EmbedCodes pq) {
  pdl_release();
  // the pass's launch stamps start over (every later kernel of the pass
  // stamps only after its wait, so after this kernel has finished)
  if (stamp && blockIdx.x == 0 && blockIdx.y == 0)
    for (int i = threadIdx.x; i < stamp_n; i += blockDim.x) {
      stamp[2 * i] = ~0ull;
      stamp[2 * i + 1] = 0ull;
    }
  // the cache peaks as they stand before this pass writes any row, for a
  // block that is then kept with no lane (app_core.c:12153-12156)
  if (peak_saved && blockIdx.x == 1 % gridDim.x && blockIdx.y == 0)
    for (int i = threadIdx.x; i < peak_n; i += blockDim.x) peak_saved[i] = peak[i];
  const int j = blockIdx.x;
  if (j >= lanes) return;
  const int id = ids[j];
  const int step = gridDim.y * blockDim.x, first = blockIdx.y * blockDim.x + threadIdx.x;
  if (eq.codes) {
    // a quantized table: each value decoded, then scaled as a bf16 row is
    float *xo = x_out + (size_t)j * hidden;
    for (int c = first; c < hidden; c += step) xo[c] = embed_code(eq, (size_t)id, c) * embed_gain;
  } else {
    const uint4 *row = reinterpret_cast<const uint4 *>(embed + (size_t)id * hidden);
    float4 *xo = reinterpret_cast<float4 *>(x_out + (size_t)j * hidden);
    for (int i = first; i < hidden / 8; i += step) {
      float4 a, b;
      bf16x8_scaled(row[i], embed_gain, a, b);
      xo[2 * i] = a;
      xo[2 * i + 1] = b;
    }
  }
  if (pq.codes) {
    float *so = seed_out + (size_t)j * ple_width;
    const size_t pr = (size_t)(id % ple_vocab);
    for (int c = first; c < ple_width; c += step) so[c] = embed_code(pq, pr, c) * ple_gain;
  } else if (ple_embed) {
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
// softmax, weighted values.  On an owner layer the pass's new key and value
// rows are normed, turned and written into the cache here too
// (app_core.c:11505-11512).
//
// One kernel: a cluster of CX blocks for each 16 query rows, the rows being
// (lane, head) pairs of one key/value head, so that all of a block's rows
// read the same keys and values.  Positions come in tiles of 16 at fixed
// multiples of 16; block r of the cluster takes the tiles whose index is r
// modulo CX, in ascending order, with an online softmax per row.  Scores
// (16 rows x 16 positions) and weighted values are tensor-core products of
// f16 hi/lo splits of both operands (hi*hi + hi*lo + lo*hi, f32 accumulate),
// about 22 bits.  A tile's cached rows arrive by 16-byte asynchronous
// copies spread over the block, the first tiles' issued before the kernel
// waits on the projection ahead of it; the pass's new rows are computed
// after the wait.  The cluster then merges its blocks'
// partials through distributed shared memory: each block pushes its row
// maxima, totals and values to the blocks that merge them, and block r
// writes dimensions [r, r + 1) * hd / CX of every row.  Every sum is keyed on absolute
// positions and runs in a fixed order, so a lane's output does not depend on
// how many lanes share the pass.
constexpr int AT_ROWS = 16;        // query rows a block
constexpr int AT_POS = 16;         // positions a tile
constexpr int AT_DEPTH = 3;        // tiles in flight a block
constexpr int AT_SRED = 24;        // row stride of the score partials and weights
constexpr int AT_MAX_CLUSTER = 16;

template <int HD, bool LITE = false>
struct AttnLayout {                  // offsets in floats
  // A head of 512 (the export's global layers) keeps two tiles in flight and
  // reads the pass's new rows through the tiles like any cached row (they are
  // in the cache before it runs, written by lane_kv_kernel); narrower heads
  // keep three and hold the pass's new rows apart, computed here.  The light
  // layout (lane passes, whose new rows are all in the cache before the
  // launch) reads them through the tiles too, keeps two tiles in flight and
  // puts the cluster's pushed values in the ring once every block of the
  // cluster is past its tiles: about 100 KB at a head of 256, so two blocks
  // share an SM.
  static constexpr int DEPTH = (HD > 256 || LITE) ? 2 : AT_DEPTH;
  static constexpr bool NEW_ROWS = HD <= 256 && !LITE;
  static constexpr int KS = HD + 8;  // key rows: a half-warp's float2 reads meet 32 banks
  static constexpr int VS = HD + 4;  // value rows: a warp's scalar reads meet 32 banks
  static constexpr int QS = HD + 4;
  static constexpr int TILE = AT_POS * (KS + VS);  // a slot: 16 key rows, then 16 value rows
  static constexpr int O_NEWK = DEPTH * TILE;
  static constexpr int O_NEWV = O_NEWK + (NEW_ROWS ? AT_POS * KS : 0);
  static constexpr int O_Q = O_NEWV + (NEW_ROWS ? AT_POS * VS : 0);
  static constexpr int O_ZERO = O_Q + AT_ROWS * QS;
  static constexpr int O_SRED = O_ZERO + KS;                    // [8 warps][16][AT_SRED]
  static constexpr int O_P = O_SRED + 8 * AT_ROWS * AT_SRED;    // hi, lo weights: 2 x [16][AT_SRED] halves
  static constexpr int O_F = O_P + AT_ROWS * AT_SRED;
  static constexpr int O_RO = LITE ? 0 : O_F + AT_ROWS;   // pushed values: [sender][16][hd / CX]
  static constexpr int O_RML = LITE ? O_F + AT_ROWS : O_RO + AT_ROWS * HD;  // pushed maxima, totals: [sender][16][2]
  static constexpr int O_W = O_RML + 2 * AT_ROWS * AT_MAX_CLUSTER;  // merge weights [16][16]
  static constexpr int O_LINV = O_W + AT_ROWS * AT_MAX_CLUSTER;
  static constexpr int O_AMX = O_LINV + AT_ROWS;
  static constexpr int FLOATS = O_AMX + AT_ROWS;
  static_assert(!LITE || AT_ROWS * HD <= DEPTH * TILE, "pushed values fit the ring");
};

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

// One head of 32 * DPL dimensions, DPL a thread: normed (app_core.c:4667,
// the shrink in float, see rms_shrink) with an optional gain, then turned by the rope
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
  const float sh = 1.0f / sqrtf(s / (float)HD + eps);
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

__device__ __forceinline__ void cp_async16(float *dst, const float *src, uint64_t policy) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;\n" ::"r"(smem_u32(dst)), "l"(src),
               "l"(policy)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// head_norm_turn in two halves, so that several rows' loads can be in
// flight before any row's arithmetic: the row, its rope tables and gain
template <int DPL>
struct HeadRow {
  float v[DPL], c[DPL], s[DPL], gn[DPL];
};

template <int DPL>
__device__ __forceinline__ void head_row_load(HeadRow<DPL> &R, const float *src, const float *gain, const float *cs,
                                              const float *sn, bool turn, int l) {
  if (src) {
    load_dpl<DPL>(src + l * DPL, R.v);
  } else {
#pragma unroll
    for (int e = 0; e < DPL; ++e) R.v[e] = 0.0f;
  }
  if (turn) {
    const int d0 = (l & 15) * DPL;
    load_dpl<DPL>(cs + d0, R.c);
    load_dpl<DPL>(sn + d0, R.s);
  }
  if (gain) load_dpl<DPL>(gain + l * DPL, R.gn);
}

__device__ __forceinline__ void prefetch_l1(const void *p) { asm volatile("prefetch.global.L1 [%0];\n" ::"l"(p)); }

// the same arithmetic as head_norm_turn
template <int DPL>
__device__ __forceinline__ void head_row_finish(HeadRow<DPL> &R, bool gain, float eps, bool turn, int l) {
  constexpr int HD = 32 * DPL;
  float s = 0.0f;
#pragma unroll
  for (int e = 0; e < DPL; ++e) s += R.v[e] * R.v[e];
  s = warp_sum(s);
  const float sh = 1.0f / sqrtf(s / (float)HD + eps);
#pragma unroll
  for (int e = 0; e < DPL; ++e) R.v[e] = gain ? R.v[e] * sh * R.gn[e] : R.v[e] * sh;
  if (turn) {
    float other[DPL];
#pragma unroll
    for (int e = 0; e < DPL; ++e) other[e] = __shfl_xor_sync(0xffffffffu, R.v[e], 16);
#pragma unroll
    for (int e = 0; e < DPL; ++e)
      R.v[e] = l < 16 ? R.v[e] * R.c[e] - other[e] * R.s[e] : R.v[e] * R.c[e] + other[e] * R.s[e];
  }
}

__device__ __forceinline__ void split_h2(float x, float y, uint32_t &hi, uint32_t &lo) {
  const __half2 h = __floats2half2_rn(x, y);
  const float2 b = __half22float2(h);
  const __half2 r = __floats2half2_rn(x - b.x, y - b.y);
  hi = *reinterpret_cast<const uint32_t *>(&h);
  lo = *reinterpret_cast<const uint32_t *>(&r);
}

template <int HD, int CX, bool LITE = false>
__global__ void __launch_bounds__(256) attn_kernel(const float *qkv, int qkv_stride, int heads, int kv_heads,
                                                   const float *q_norm, const float *k_norm, const float *cs_tab,
                                                   const float *sn_tab, float eps, int owner, float *kc, float *vc,
                                                   int sliding, int span, const int *d_p0, int lanes, float *out,
                                                   int out_stride, float *out_amax, unsigned long long *stamp,
                                                   float *const *kc_tab, float *const *vc_tab, const int *pos_tab,
                                                   CacheStore cq) {
  using LY = AttnLayout<HD, LITE>;
  float *peak = cq.peak;
  if (kc_tab) {
    // one of many sessions' blocks (blockIdx.z): its caches, peaks and
    // position from the tables, its `lanes` rows of the batch's q|k|v and
    // output
    const int zb = blockIdx.z;
    kc = kc_tab[zb];
    vc = vc_tab[zb];
    if (cq.peak_tab) peak = cq.peak_tab[zb];
    d_p0 = pos_tab + zb;
    qkv += (size_t)zb * lanes * qkv_stride;
    out += (size_t)zb * lanes * out_stride;
  }
  constexpr int DPL = HD / 32, NKS = HD / 16, KPW = (NKS + 7) / 8, NNT = HD / 8, NPW = (NNT + 7) / 8;
  constexpr int KS = LY::KS, VS = LY::VS, QS = LY::QS, DS = HD / CX;
  static_assert(CX <= AT_MAX_CLUSTER && HD % CX == 0, "cluster size");
  extern __shared__ __align__(128) float sm[];
  float *ring = sm, *newk = sm + LY::O_NEWK, *newv = sm + LY::O_NEWV, *qs = sm + LY::O_Q, *zrow = sm + LY::O_ZERO;
  float *sred = sm + LY::O_SRED, *fsc = sm + LY::O_F, *ro = sm + LY::O_RO, *rml = sm + LY::O_RML;
  float *amx = sm + LY::O_AMX, *wts = sm + LY::O_W, *linv = sm + LY::O_LINV;
  __half *ph = reinterpret_cast<__half *>(sm + LY::O_P), *pl = ph + AT_ROWS * AT_SRED;
  const int tid = threadIdx.x, warp = tid >> 5, l = tid & 31, g = l >> 2, t = l & 3;
  const int r = blockIdx.x;  // rank in the cluster, which spans the grid's x
  const int G = heads / kv_heads, row_blocks = (lanes * G + AT_ROWS - 1) / AT_ROWS;
  const int kh = blockIdx.y / row_blocks, rb = blockIdx.y - kh * row_blocks;
  const int kv_w = kv_heads * HD, half = HD / 2;
  pdl_release();

  // this block's tiles: t0, t0 + CX, ... up to the pass's last position.  The
  // position is written before the pass starts, so it is read before the wait.
  const int p0 = __ldcg(d_p0);
  const int lo_all = sliding ? max(0, p0 - span + 1) : 0, hi_all = p0 + lanes;
  const int t_first = lo_all / AT_POS, t_last = (hi_all - 1) / AT_POS;
  const int t0 = t_first + (r - t_first % CX + CX) % CX;
  const int n_tiles = t0 <= t_last ? (t_last - t0) / CX + 1 : 0;
  const uint64_t policy = l2_evict_last();
  // the cached rows of tile i (positions before the pass) into slot i %
  // depth: 16-byte asynchronous copies spread over the block (thread t the
  // column 4 (t mod hd/4) of rows t / (hd/4), + 256 / (hd/4), ...), one
  // commit group a tile
  constexpr int CP_C4 = HD / 4, CP_RPP = 256 / CP_C4;
  const int cp_col = 4 * (tid % CP_C4), cp_r0 = tid / CP_C4;
  auto issue = [&](int i) {
    const int tb = (t0 + i * CX) * AT_POS;
    const int a = max(tb, lo_all), b = min(tb + AT_POS, LY::NEW_ROWS ? p0 : hi_all);
    float *slot = ring + (i % LY::DEPTH) * LY::TILE;
#pragma unroll
    for (int row = cp_r0; row < AT_POS; row += CP_RPP) {
      const int pos = tb + row;
      if (pos >= a && pos < b) {
        const size_t src = (size_t)pos * kv_w + (size_t)kh * HD + cp_col;
        cp_async16(slot + row * KS + cp_col, kc + src, policy);
        cp_async16(slot + AT_POS * KS + row * VS + cp_col, vc + src, policy);
      }
    }
  };
  for (int i = tid; i < KS; i += blockDim.x) zrow[i] = 0.0f;
  for (int i = 0; i < LY::DEPTH; ++i) {
    if (i < n_tiles) issue(i);
    cp_async_commit();
  }
  // the norm gains and the pass's rope rows into L1: they do not depend on
  // the projection, so their latency passes while this kernel waits on it
  {
    constexpr int GL = HD / 32;                 // 128-byte lines a gain vector (hd floats)
    constexpr int RL = HD >= 64 ? HD / 64 : 1;  // lines a rope row (hd / 2 floats)
    const int n_pre = 2 * GL + lanes * 2 * RL;
    for (int i = tid; i < n_pre; i += blockDim.x) {
      if (i < 2 * GL) {
        const float *gv = i < GL ? q_norm : k_norm;
        if (gv) prefetch_l1(gv + (i % GL) * 32);
      } else {
        const int k = i - 2 * GL, jj = k / (2 * RL), part = k - jj * 2 * RL;  // cs lines, then sn lines
        const float *tab = part < RL ? cs_tab : sn_tab;
        prefetch_l1(tab + (size_t)(p0 + jj) * half + (part % RL) * 32);
      }
    }
  }

  pdl_wait();
  stamp_begin(stamp);
  // the rows a warp prepares: query rows warp and warp + 8 (normed and
  // turned at their lane's position), then the pass's new key and value rows
  // it = warp, warp + 8, ... that fall in this block's tiles (on an owner
  // layer normed, turned (keys) and written to the cache by the first row
  // block; on a sharing layer read back from the owner's cache).  Three at
  // a time: all three rows' loads issue before any row's arithmetic.
  {
    const int n_items = LY::NEW_ROWS ? 2 + (2 * lanes - warp + 7) / 8 : 2;
    for (int k0 = 0; k0 < n_items; k0 += 3) {
      HeadRow<DPL> R[3];
      bool live[3], norm[3], turn[3];
      const float *gain[3];
      float *dst[3], *cache[3];
      int side[3];  // 0 key, 1 value
#pragma unroll
      for (int b = 0; b < 3; ++b) {
        const int k = k0 + b;
        live[b] = false;
        norm[b] = turn[b] = false;
        gain[b] = nullptr;
        dst[b] = cache[b] = nullptr;
        side[b] = 0;
        const float *src = nullptr;
        int pos = 0;
        if (k < 2) {
          const int row = warp + 8 * k, f = rb * AT_ROWS + row, j = f / G, h = kh * G + (f - j * G);
          dst[b] = qs + row * QS;
          live[b] = true;  // rows past the lanes are staged as zeros
          if (j < lanes) {
            src = qkv + (size_t)j * qkv_stride + (size_t)h * HD;
            pos = p0 + j;
            norm[b] = turn[b] = true;
            gain[b] = q_norm;
          }
        } else if (k < n_items) {
          const int it = warp + 8 * (k - 2), jj = it >> 1, is_v = it & 1, tile = (p0 + jj) / AT_POS;
          if (it < 2 * lanes && tile >= t0 && (tile - t0) % CX == 0) {
            pos = p0 + jj;
            live[b] = true;
            dst[b] = is_v ? newv + jj * VS : newk + jj * KS;
            side[b] = is_v;
            float *crow = (is_v ? vc : kc) + (size_t)pos * kv_w + (size_t)kh * HD;
            if (owner) {
              src = qkv + (size_t)jj * qkv_stride + (size_t)heads * HD + (is_v ? kv_w : 0) + (size_t)kh * HD;
              norm[b] = true;
              turn[b] = !is_v;
              gain[b] = is_v ? nullptr : k_norm;
              if (rb == 0) cache[b] = crow;
            } else {
              src = crow;
            }
          }
        }
        head_row_load<DPL>(R[b], src, gain[b], cs_tab + (size_t)pos * half, sn_tab + (size_t)pos * half, turn[b], l);
      }
#pragma unroll
      for (int b = 0; b < 3; ++b) {
        if (!live[b]) continue;
        if (norm[b]) head_row_finish<DPL>(R[b], gain[b] != nullptr, eps, turn[b], l);
        if (cache[b] && peak) {
          // the row's largest magnitude (app_core.c:11208 cache_lay; a NaN is passed over)
          float mx = 0.0f;
#pragma unroll
          for (int e = 0; e < DPL; ++e) mx = fmaxf(mx, fabsf(R[b].v[e]));
          mx = warp_max(mx);
          if (l == 0) atomicMax(reinterpret_cast<int *>(peak) + side[b], __float_as_int(mx));
        }
        store_dpl<DPL>(dst[b] + l * DPL, R[b].v);
        if (cache[b]) store_dpl<DPL>(cache[b] + l * DPL, R[b].v);
      }
    }
  }

  cp_async_wait<LY::DEPTH - 1>();  // this thread's copies of tile 0
  __syncthreads();
  // the query A fragments of this warp's k-steps (warp w: 16 columns from
  // 16 (w + 8 i)); warps past the head's last k-step hold unused copies
  uint32_t qh[KPW][4], ql[KPW][4];
#pragma unroll
  for (int i = 0; i < KPW; ++i) {
    const float *q0 = qs + g * QS + 16 * min(warp + 8 * i, NKS - 1) + 2 * t, *q8 = q0 + 8 * QS;
    split_h2(q0[0], q0[1], qh[i][0], ql[i][0]);
    split_h2(q8[0], q8[1], qh[i][1], ql[i][1]);
    split_h2(q0[8], q0[9], qh[i][2], ql[i][2]);
    split_h2(q8[8], q8[9], qh[i][3], ql[i][3]);
  }
  // the softmax thread of (row sr, position sp of a tile) and its row's span
  const int sr = tid >> 4, sp = tid & 15;
  const int sj = (rb * AT_ROWS + sr) / G;
  const bool row_ok = sj < lanes;
  const int lo_r = sliding ? max(0, p0 + sj - span + 1) : 0, hi_r = p0 + sj;
  float m_run = -FLT_MAX, l_run = 0.0f;
  float oacc[NPW][4];
#pragma unroll
  for (int i = 0; i < NPW; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) oacc[i][e] = 0.0f;

  // tile i: scores, then (barrier) tile i - 1 + depth into the slot tile
  // i - 1 left and the softmax, then (barrier, after which tile i + 1 is in
  // place: one commit group a step keeps the count regular) the values
  for (int i = 0; i < n_tiles; ++i) {
    if constexpr (LITE) {
      // tile i, issued a step ago, in place (its copy ran under the values
      // of tile i - 1)
      if (i > 0) {
        cp_async_wait<0>();
        __syncthreads();
      }
    }
    const int tb = (t0 + i * CX) * AT_POS;
    const float *slot = ring + (i % LY::DEPTH) * LY::TILE;
    // a position's key and value rows: new, cached, or zeros outside the pass's span
    auto krow = [&](int pos) -> const float * {
      return (pos < lo_all || pos >= hi_all)   ? zrow
             : (LY::NEW_ROWS && pos >= p0) ? newk + (pos - p0) * KS
                                           : slot + (pos - tb) * KS;
    };
    auto vrow = [&](int pos) -> const float * {
      return (pos < lo_all || pos >= hi_all) ? zrow
             : (LY::NEW_ROWS && pos >= p0)    ? newv + (pos - p0) * VS
                                              : slot + AT_POS * KS + (pos - tb) * VS;
    };
    // scores: this warp's k-steps of the 16 x 16 tile, into the partials;
    // the three split products in separate accumulators (short chains),
    // added as hi*hi + (hi*lo + lo*hi)
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      float shh[4] = {0.0f, 0.0f, 0.0f, 0.0f}, shl[4] = {0.0f, 0.0f, 0.0f, 0.0f}, slh[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      const float *kr = krow(tb + 8 * nt + g) + 2 * t;
#pragma unroll
      for (int i2 = 0; i2 < KPW; ++i2) {
        const int ks = warp + 8 * i2;
        if (ks < NKS) {
          const float2 k01 = *reinterpret_cast<const float2 *>(kr + 16 * ks);
          const float2 k89 = *reinterpret_cast<const float2 *>(kr + 16 * ks + 8);
          uint32_t bh0, bl0, bh1, bl1;
          split_h2(k01.x, k01.y, bh0, bl0);
          split_h2(k89.x, k89.y, bh1, bl1);
          mma16816(shh, qh[i2], bh0, bh1, shh);
          mma16816(shl, qh[i2], bl0, bl1, shl);
          mma16816(slh, ql[i2], bh0, bh1, slh);
        }
      }
      float sc[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) sc[e] = shh[e] + (shl[e] + slh[e]);
      float *sw = sred + (warp * AT_ROWS + g) * AT_SRED + 8 * nt + 2 * t;
      *reinterpret_cast<float2 *>(sw) = make_float2(sc[0], sc[1]);
      *reinterpret_cast<float2 *>(sw + 8 * AT_SRED) = make_float2(sc[2], sc[3]);
    }
    __syncthreads();  // the partials are written, and every warp is past tile i - 1
    if (i >= 1) {
      if (i - 1 + LY::DEPTH < n_tiles) issue(i - 1 + LY::DEPTH);
      cp_async_commit();
    }
    // online softmax of row sr, one thread a position; the warps' partials
    // added in warp order
    float s = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) s += sred[(w * AT_ROWS + sr) * AT_SRED + sp];
    const int pos = tb + sp;
    const bool valid = row_ok && pos >= lo_r && pos <= hi_r;
    const float sv = valid ? s : -FLT_MAX;
    float mt = sv;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, o));
    const float m_new = fmaxf(m_run, mt);
    const float fct = (m_new == -FLT_MAX) ? 1.0f : (m_run == -FLT_MAX ? 0.0f : expf(m_run - m_new));
    const float e = valid ? expf(sv - m_new) : 0.0f;
    float es = e;
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) es += __shfl_xor_sync(0xffffffffu, es, o);
    l_run = l_run * fct + es;
    m_run = m_new;
    const __half eh = __float2half_rn(e);
    ph[sr * AT_SRED + sp] = eh;
    pl[sr * AT_SRED + sp] = __float2half_rn(e - __half2float(eh));
    if (sp == 0) fsc[sr] = fct;
    if constexpr (!LITE) cp_async_wait<LY::DEPTH - 2>();  // this thread's copies of tile i + 1 (all but the newest group)
    __syncthreads();     // the weights and factors are written; tile i + 1 is in place (light: in flight)
    // weighted values: this warp's 8-dimension tiles n = warp + 8 i
    {
      const uint32_t *h32 = reinterpret_cast<const uint32_t *>(ph), *l32 = reinterpret_cast<const uint32_t *>(pl);
      constexpr int W = AT_SRED / 2;  // words a row
      const uint32_t pah[4] = {h32[g * W + t], h32[(g + 8) * W + t], h32[g * W + t + 4], h32[(g + 8) * W + t + 4]};
      const uint32_t pal[4] = {l32[g * W + t], l32[(g + 8) * W + t], l32[g * W + t + 4], l32[(g + 8) * W + t + 4]};
      const float f0 = fsc[g], f8 = fsc[g + 8];
      const float *v0 = vrow(tb + 2 * t), *v1 = vrow(tb + 2 * t + 1), *v8 = vrow(tb + 2 * t + 8),
                  *v9 = vrow(tb + 2 * t + 9);
#pragma unroll
      for (int i2 = 0; i2 < NPW; ++i2) {
        const int nt = warp + 8 * i2;
        if (nt < NNT) {
          const int n = 8 * nt + g;
          uint32_t bh0, bl0, bh1, bl1;
          split_h2(v0[n], v1[n], bh0, bl0);
          split_h2(v8[n], v9[n], bh1, bl1);
          const float z[4] = {0.0f, 0.0f, 0.0f, 0.0f};
          float thh[4], thl[4], tlh[4];
          mma16816(thh, pah, bh0, bh1, z);
          mma16816(thl, pah, bl0, bl1, z);
          mma16816(tlh, pal, bh0, bh1, z);
          oacc[i2][0] = fmaf(oacc[i2][0], f0, thh[0] + (thl[0] + tlh[0]));
          oacc[i2][1] = fmaf(oacc[i2][1], f0, thh[1] + (thl[1] + tlh[1]));
          oacc[i2][2] = fmaf(oacc[i2][2], f8, thh[2] + (thl[2] + tlh[2]));
          oacc[i2][3] = fmaf(oacc[i2][3], f8, thh[3] + (thl[3] + tlh[3]));
        }
      }
    }
  }
  // push this block's partials to the blocks that merge them: the weighted
  // values of dimensions [q DS, (q + 1) DS) to block q, and every row's
  // maximum and total to every block (remote stores into buffers nothing
  // else uses, made visible by the cluster barrier)
  if constexpr (LITE) {
    // the pushed values land in the ring: every block of the cluster first
    // finishes with its tiles
    cp_async_wait<0>();
    cluster_sync();
  }
#pragma unroll
  for (int i2 = 0; i2 < NPW; ++i2) {
    const int nt = warp + 8 * i2;
    if (nt < NNT) {
      const int d = 8 * nt + 2 * t, q = d / DS;
      float *at = ro + (r * AT_ROWS + g) * DS + (d - q * DS);
      st_cluster2(at, q, oacc[i2][0], oacc[i2][1]);
      st_cluster2(at + 8 * DS, q, oacc[i2][2], oacc[i2][3]);
    }
  }
  if (sp < CX) st_cluster2(rml + 2 * (r * AT_ROWS + sr), sp, m_run, l_run);
  if (tid < AT_ROWS) amx[tid] = 0.0f;
  cluster_sync();
  // each row's block weights e^{m_q - M} and total: thread (row, q), the
  // maximum and the total over the row's 16 threads in fixed trees
  {
    const int wr = tid >> 4, wq = tid & 15;
    const float2 mq = wq < CX ? *reinterpret_cast<const float2 *>(rml + 2 * (wq * AT_ROWS + wr))
                              : make_float2(-FLT_MAX, 0.0f);
    float M = mq.x;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    const float w = mq.x == -FLT_MAX ? 0.0f : expf(mq.x - M);
    float L = mq.y * w;
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
    wts[wr * AT_MAX_CLUSTER + wq] = w;
    if (wq == 0) linv[wr] = 1.0f / L;
  }
  __syncthreads();
  // block r merges dimensions [r * DS, (r + 1) * DS) of every row, a thread a
  // pair of them (in passes of the block where a block merges more than 32
  // dimensions), blocks in rank order
  constexpr int DP = DS / 2;
  for (int it = tid; it < AT_ROWS * DP; it += 256) {
    const int row = it / DP, dd = 2 * (it - row * DP), d = r * DS + dd;
    float o0 = 0.0f, o1 = 0.0f;
#pragma unroll
    for (int q = 0; q < CX; ++q) {
      const float w = wts[row * AT_MAX_CLUSTER + q];
      const float2 x = *reinterpret_cast<const float2 *>(ro + (q * AT_ROWS + row) * DS + dd);
      o0 = fmaf(x.x, w, o0);
      o1 = fmaf(x.y, w, o1);
    }
    const float inv = linv[row], v0 = o0 * inv, v1 = o1 * inv;
    const int f = rb * AT_ROWS + row, j = f / G, h = kh * G + (f - j * G);
    if (j < lanes) {
      *reinterpret_cast<float2 *>(out + (size_t)j * out_stride + (size_t)h * HD + d) = make_float2(v0, v1);
      if (out_amax) atomicMax(reinterpret_cast<int *>(amx + row), __float_as_int(fmaxf(fabsf(v0), fabsf(v1))));
    }
  }
  __syncthreads();
  if (out_amax && tid < AT_ROWS) {
    // one magnitude partial a (head, block) for lane j
    const int f = rb * AT_ROWS + tid, j = f / G, h = kh * G + (f - j * G);
    if (j < lanes) out_amax[(size_t)j * GEMV_PART_LIMIT + h * CX + r] = amx[tid];
  }
  stamp_end(stamp);
}

// argmax partials of the output head merged per lane (app_main.c:482: the
// first index of the largest value).  Thread (lane, stripe) scans parts
// stripe, stripe + 32, ...; the stripes then meet in shared memory.
__global__ void argmax_final_kernel(const float *part_val, const int *part_idx, int parts, int lanes,
                                    int32_t *top_out, const unsigned long long *stamp,
                                    unsigned long long *stamp_sum, int stamp_n) {
  __shared__ float sv[32][16];
  __shared__ int si[32][16];
  pdl_release();
  pdl_wait();
  // the last kernel of a pass adds each stamped launch's span to its total
  if (stamp_sum)
    for (int k = threadIdx.x; k < stamp_n; k += blockDim.x) {
      const unsigned long long b = stamp[2 * k], e = stamp[2 * k + 1];
      if (b != ~0ull && e > b) stamp_sum[k] += e - b;
    }
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

// launch_k with a cluster of `cx` blocks along x (none when cx is 1).
template <typename... KArgs, typename... Args>
static cudaError_t launch_kc(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, int cx,
                             Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  int na = 0;
  if (cx > 1) {
    at[na].id = cudaLaunchAttributeClusterDimension;
    at[na].val.clusterDim.x = cx;
    at[na].val.clusterDim.y = 1;
    at[na].val.clusterDim.z = 1;
    ++na;
  }
  if (g_pdl) {
    at[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = at;
  cfg.numAttrs = na;
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
  L.red = align128(gemv_stage_bytes(a.pl.n_cc, MODE) + (a.pl.cols > 48 * 128 ? SCR_FLOATS_WIDE : SCR_FLOATS) * 4);
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

// The per-layer-embedding gate (residual prologue, GELU x input epilogue)
// launches its blocks as clusters of eight, which keeps each eight in one GPC:
// measured 5-20 us a verify round faster at 1, 4 and 8 lanes.  Clusters for the
// other projections measured the same (pairs) or slower (fours).
template <int MODE, int WARPS, int PAIR>
static cudaError_t launch_gemv_pe(const GemvArgs &a, int pro, int epi, int grid, size_t smem, cudaStream_t st) {
#define IGC_CASE(P, E) \
  if (pro == P && epi == E)                                                                                   \
    return launch_kc(gemv_kernel<MODE, WARPS, PAIR, P, E>, dim3(grid, a.batches > 1 ? a.batches : 1), dim3(WARPS * 32), \
                    smem, st, (P == PRO_RESID && E == EPI_GELU_MUL && grid % 8 == 0 ? 8 : 1), a);
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

extern "C++" {
template <int HD>
static cudaError_t allow_attn(int bytes) {
  cudaError_t e = cudaSuccess;
  if constexpr (HD <= 256) {  // a 512 head runs in clusters of 16 only
    e = allow_smem_fn(attn_kernel<HD, 1, true>, bytes);
    if (e == cudaSuccess) e = allow_smem_fn(attn_kernel<HD, 2, true>, bytes);
    if (e == cudaSuccess) e = allow_smem_fn(attn_kernel<HD, 4, true>, bytes);
    if (e == cudaSuccess) e = allow_smem_fn(attn_kernel<HD, 1>, bytes);
    if (e == cudaSuccess) e = allow_smem_fn(attn_kernel<HD, 2>, bytes);
    if (e == cudaSuccess) e = allow_smem_fn(attn_kernel<HD, 4>, bytes);
    if (e == cudaSuccess) e = allow_smem_fn(attn_kernel<HD, 8>, bytes);
  }
  if (e == cudaSuccess) e = allow_smem_fn(attn_kernel<HD, 16>, bytes);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(attn_kernel<HD, 16>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  return e;
}
}  // extern "C++"

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
  if (e == cudaSuccess) e = allow_attn<32>(bytes);
  if (e == cudaSuccess) e = allow_attn<64>(bytes);
  if (e == cudaSuccess) e = allow_attn<128>(bytes);
  if (e == cudaSuccess) e = allow_attn<256>(bytes);
  if (e == cudaSuccess) e = allow_attn<512>(bytes);
  if (e == cudaSuccess) e = allow_smem_fn(topk_stage2_kernel, bytes);
  return e;
}

cudaError_t igc_launch_repack(const uint8_t *code, size_t row_stride, int bits, const uint16_t *scale, int groups,
                              int rows, int cols, int n_rb, int n_cc, int out_mul, int out_add, uint4 *tiles,
                              uint2 *scales, cudaStream_t st) {
  if (bits != 1 && bits != 2 && bits != 4) return cudaErrorInvalidValue;
  long total = (long)n_rb * n_cc * 32;
  int blocks = (int)((total + 255) / 256);
  repack_kernel<<<blocks, 256, 0, st>>>(code, row_stride, bits, scale, groups, rows, cols, n_rb, n_cc, out_mul,
                                        out_add, tiles, scales);
  return cudaGetLastError();
}

// A plane's group scales as f16 [rows][ceil(cols / 32)]: each group of
// `group_size` columns (a multiple of 32) spreads its scale over its 32-column
// groups, converted from F32 (1), F16 (2) or BF16 (3) storage.  Refused (-1)
// unless every scale survives the conversion exactly, since the products use
// it as stored.
int igc_scales_f16(const void *src, int dtype, int rows, int groups, int group_size, int cols, uint16_t *out) {
  if (rows < 1 || groups < 1 || group_size < 32 || group_size % 32 || cols < 1) return -1;
  const int g32 = (cols + 31) / 32, per = group_size / 32;
  for (int r = 0; r < rows; ++r)
    for (int g = 0; g < groups; ++g) {
      float v;
      const size_t i = (size_t)r * groups + g;
      if (dtype == 1) {
        memcpy(&v, (const uint8_t *)src + 4 * i, 4);
      } else if (dtype == 2 || dtype == 3) {
        uint16_t h;
        memcpy(&h, (const uint8_t *)src + 2 * i, 2);
        if (dtype == 2) {
          __half hh;
          memcpy(&hh, &h, 2);
          v = __half2float(hh);
        } else {
          const uint32_t u = (uint32_t)h << 16;
          memcpy(&v, &u, 4);
        }
      } else {
        return -1;
      }
      const __half h16 = __float2half_rn(v);
      if (__half2float(h16) != v && !(v != v)) return -1;
      uint16_t bits16;
      memcpy(&bits16, &h16, 2);
      for (int k = 0; k < per; ++k) {
        const int c32 = g * per + k;
        if (c32 < g32) out[(size_t)r * g32 + c32] = bits16;
      }
    }
  return 0;
}

void igc_kernels_pdl(int on) { g_pdl = on; }
int igc_kernels_pdl_get(void) { return g_pdl; }

cudaError_t igc_launch_gemv(GemvArgs *a, int pair, int pro, int epi, int grid, size_t smem_limit, cudaStream_t st,
                            int *grid_used) {
  if (a->pl.cols > GEMV_MAX_PARTS * 128) return cudaErrorInvalidValue;  // wider than the prologue's parts
  const int mode = gemv_mode(a->lanes);
  const int units = pair ? a->pl.n_rb / 2 : a->pl.n_rb;
  const int G8 = GEMV_WARPS / a->split;
  // 16-warp blocks where the mode allows them and their shared memory fits,
  // except for one or two lanes when the 8-warp blocks fit one wave of the
  // SMs (the products then spread over twice the SMs, and with so few lanes
  // the per-warp staging stays short)
  int W = GEMV_WARPS;
  int sms = 0, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const bool spread = a->lanes <= 2 && sms > 0 && grid * (a->batches > 1 ? a->batches : 1) <= sms;
  if (mode != MODE_NT2 && !spread &&
      gemv_layout(*a, pair, 16, 0, GEMV_MAX_DEPTH).ring + (size_t)16 * (pair + 1) * GEMV_PIECE_BYTES <= smem_limit)
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
                             float *x_out, float *seed_out, unsigned long long *stamp, int stamp_n,
                             const float *peak, float *peak_saved, int peak_n, const EmbedCodes *embed_q,
                             const EmbedCodes *ple_q, cudaStream_t st) {
  if ((hidden & 7) || (ple_embed && (ple_width & 7)) || (peak_saved && (!peak || peak_n < 0)))
    return cudaErrorInvalidValue;
  EmbedCodes eq = {}, pq = {};
  if (embed_q) eq = *embed_q;
  if (ple_q) pq = *ple_q;
  if ((!eq.codes && !embed) || (eq.codes && eq.bits != 1 && eq.bits != 2 && eq.bits != 4) ||
      (pq.codes && pq.bits != 1 && pq.bits != 2 && pq.bits != 4))
    return cudaErrorInvalidValue;
  embed_kernel<<<dim3(lanes, 8), 256, 0, st>>>(ids, lanes, embed, hidden, embed_gain, ple_embed, ple_vocab, ple_width,
                                      ple_gain, x_out, seed_out, stamp, stamp_n, peak, peak_saved, peak_n, eq, pq);
  return cudaGetLastError();
}

cudaError_t igc_launch_ple_finish(const float *raw, const float *seed, int lanes, int layers, int ple_dim,
                                  const float *w, float eps, float blend, float *out, cudaStream_t st) {
  return launch_k(ple_finish_kernel, dim3(lanes * layers), dim3(256), 0, st, raw, seed, lanes, layers, ple_dim, w, eps,
                  blend, out);
}

size_t igc_attn_smem_light(int hd) {
  switch (hd) {
    case 32: return sizeof(float) * AttnLayout<32, true>::FLOATS;
    case 64: return sizeof(float) * AttnLayout<64, true>::FLOATS;
    case 128: return sizeof(float) * AttnLayout<128, true>::FLOATS;
    case 256: return sizeof(float) * AttnLayout<256, true>::FLOATS;
    default: return 0;
  }
}

size_t igc_attn_smem(int hd) {
  switch (hd) {
    case 32: return sizeof(float) * AttnLayout<32>::FLOATS;
    case 64: return sizeof(float) * AttnLayout<64>::FLOATS;
    case 128: return sizeof(float) * AttnLayout<128>::FLOATS;
    case 256: return sizeof(float) * AttnLayout<256>::FLOATS;
    case 512: return sizeof(float) * AttnLayout<512>::FLOATS;
    default: return 0;
  }
}

extern "C++" {
template <int HD, int CX, bool LITE = false>
static cudaError_t launch_attn(dim3 grid, size_t smem, cudaStream_t st, const float *qkv, int qkv_stride, int heads,
                               int kv_heads, const float *q_norm, const float *k_norm, const float *cs,
                               const float *sn, float eps, int owner, float *kc, float *vc, int sliding, int span,
                               const int *d_p0, int lanes, float *out, int out_stride, float *out_amax,
                               unsigned long long *stamp, float *const *kc_tab, float *const *vc_tab,
                               const int *pos_tab, CacheStore cq) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = CX;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = g_pdl ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, attn_kernel<HD, CX, LITE>, qkv, qkv_stride, heads, kv_heads, q_norm, k_norm, cs, sn, eps,
                            owner, kc, vc, sliding, span, d_p0, lanes, out, out_stride, out_amax, stamp, kc_tab,
                            vc_tab, pos_tab, cq);
}
}  // extern "C++"

cudaError_t igc_launch_attn(const float *qkv, int qkv_stride, int heads, int kv_heads, int hd, const float *q_norm,
                            const float *k_norm, const float *cs, const float *sn, float eps, int owner, float *kc,
                            float *vc, int sliding, int span, const int *d_p0, int lanes, int cluster, float *out,
                            int out_stride, float *out_amax, unsigned long long *stamp, const igc::CacheStore *store,
                            cudaStream_t st, int light) {
  return igc_launch_attn_many(qkv, qkv_stride, heads, kv_heads, hd, q_norm, k_norm, cs, sn, eps, owner, kc, vc, sliding,
                              span, d_p0, lanes, cluster, out, out_stride, out_amax, stamp, nullptr, nullptr, nullptr, 1,
                              store, st, light);
}

cudaError_t igc_launch_attn_many(const float *qkv, int qkv_stride, int heads, int kv_heads, int hd,
                                 const float *q_norm, const float *k_norm, const float *cs, const float *sn, float eps,
                                 int owner, float *kc, float *vc, int sliding, int span, const int *d_p0, int lanes,
                                 int cluster, float *out, int out_stride, float *out_amax, unsigned long long *stamp,
                                 float *const *kc_tab, float *const *vc_tab, const int *pos_tab, int batch,
                                 const igc::CacheStore *store, cudaStream_t st, int light) {
  if (lanes < 1 || lanes > AT_POS || kv_heads < 1 || heads % kv_heads ||
      (cluster != 1 && cluster != 2 && cluster != 4 && cluster != 8 && cluster != 16) || batch < 1 ||
      (batch > 1 && !kc_tab))
    return cudaErrorInvalidValue;
  igc::CacheStore cq = {};
  if (store) cq = *store;
  // float caches only: a byte side is decoded into float rows first (igc_launch_lane_widen)
  if (cq.kq != 0.0f || cq.vq != 0.0f || (cq.peak_tab && !kc_tab)) return cudaErrorInvalidValue;
  // the light layout (two blocks an SM) where asked for and possible: no
  // new rows to write (every row of the pass already in the cache), a head
  // of at most 256, clusters of at most 4
  const bool lite = light && !owner && hd <= 256 && cluster <= 4;
  const size_t smem = lite ? igc_attn_smem_light(hd) : igc_attn_smem(hd);
  const int G = heads / kv_heads;
  const dim3 grid(cluster, kv_heads * ((lanes * G + AT_ROWS - 1) / AT_ROWS), batch);
  const dim3 grid16(16, grid.y, batch);
#define IGC_ATT_CX(HD, CX, L)                                                                                  \
  launch_attn<HD, CX, L>(grid, smem, st, qkv, qkv_stride, heads, kv_heads, q_norm, k_norm, cs, sn, eps, owner, kc, vc, \
                         sliding, span, d_p0, lanes, out, out_stride, out_amax, stamp, kc_tab, vc_tab, pos_tab, cq)
#define IGC_ATT(HD)                                                                      \
  if (lite)                                                                              \
    return cluster == 1 ? IGC_ATT_CX(HD, 1, true)                                        \
           : cluster == 2 ? IGC_ATT_CX(HD, 2, true)                                      \
                          : IGC_ATT_CX(HD, 4, true);                                     \
  return cluster == 1   ? IGC_ATT_CX(HD, 1, false)                                       \
         : cluster == 2 ? IGC_ATT_CX(HD, 2, false)                                       \
         : cluster == 4 ? IGC_ATT_CX(HD, 4, false)                                       \
         : cluster == 8 ? IGC_ATT_CX(HD, 8, false)                                       \
                        : IGC_ATT_CX(HD, 16, false);
  switch (hd) {
    case 32: IGC_ATT(32)
    case 64: IGC_ATT(64)
    case 128: IGC_ATT(128)
    case 256: IGC_ATT(256)
    case 512:
      // a 512-wide head: clusters of 16 always (the merge takes 32 dimensions
      // a block), and the pass's new rows must already be in the cache
      if (owner) return cudaErrorInvalidValue;
      return launch_attn<512, 16>(grid16, smem, st, qkv, qkv_stride, heads, kv_heads, q_norm, k_norm, cs, sn, eps,
                                  owner, kc, vc, sliding, span, d_p0, lanes, out, out_stride, out_amax, stamp, kc_tab,
                                  vc_tab, pos_tab, cq);
    default: return cudaErrorInvalidValue;
  }
#undef IGC_ATT
#undef IGC_ATT_CX
}

cudaError_t igc_launch_argmax(const float *part_val, const int *part_idx, int parts, int lanes, int32_t *top,
                              const unsigned long long *stamp, unsigned long long *stamp_sum, int stamp_n,
                              cudaStream_t st) {
  return launch_k(argmax_final_kernel, dim3(1), dim3(512), 0, st, part_val, part_idx, parts, lanes, top, stamp,
                  stamp_sum, stamp_n);
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
