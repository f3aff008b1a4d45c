// igc_lanes.cu - the batched-lane path: many lanes through one weight sweep
// on the tcgen05 tensor cores.
//
// The K-lane skinny GEMM of igc_gemv.cuh streams each weight once for at most
// sixteen lanes.  A prefill chunk (app_core.c:14443-14467 session_prime runs
// its prompt 16 lanes a pass; here a chunk is up to 512) carries enough lanes
// that the product is a real dense contraction: out[m][n] = sum_k A[m][k] *
// W[n][k] with M lanes, N weight rows and K input columns.  That runs here as
// a tcgen05 GEMM:
//
//   lane_stage_kernel   one block a lane: the row-wise work between two
//                       products (residual add, RMS norms, the GELU pair and
//                       GELU x input of app_core.c:11637-11743) in f32, then
//                       the lane scaled by a power of two and stored as f16
//                       in the operand layout the tensor core reads (below),
//                       with the factor that undoes the scale.
//   lane_gemm_kernel    one block a (128-lane, 128-row) tile and K slice:
//                       a producer warp bulk-copies the staged activations
//                       and the packed int4 weights (with their f16 group
//                       scales) of each 64-column step from this GPU's HBM
//                       into a four-deep shared-memory ring; eight warps turn
//                       the codes into f16 hi/lo weights, (code - 8) * scale,
//                       in the operand layout (eight warps, one 16-byte tile
//                       slot each); one thread issues the step's
//                       twelve tcgen05.mma (M 128, N 128, K 16, f32
//                       accumulate in TMEM) and commits them to the ring
//                       slot's barrier; at
//                       the end the four warps read the accumulators back
//                       with tcgen05.ld and store them, times each lane's
//                       factor, as the slice's partial sums.
//   lane_sum_kernel     adds the K slices' partials in a fixed order.
//
// Operand layout (both operands K-major, 128-byte swizzle, the canonical
// form a tcgen05 shared-memory descriptor names): a 64-column step of 128
// rows is 16 KB, rows in groups of eight 128-byte rows (1 KB apart), and the
// 16-byte piece j of row r sits at piece j ^ (r mod 8).  The staged
// activations are stored in global memory already in this layout, a hi and
// a lo block per (128-lane tile, 64-column step), so bulk copies move them
// as they are.
//
// Precision: both operands are split into f16 hi and lo parts.  A weight
// (code - 8) * scale is a 4-bit integer times an f16 scale, so hi + lo holds
// it exactly; an activation (after the lane's power-of-two scaling) keeps
// about 22 bits in hi + lo.  Each 16-column step is three products into the
// same f32 accumulators, A_hi W_hi + A_lo W_hi + A_hi W_lo (the lo x lo term
// is below f32's own rounding), so the result matches the fp32 product to
// the accumulator's precision, as the decode path's hi/lo staging does.
// Results of a lane depend only on that lane's row and the K slices.
//
// Every wait on a barrier gives up after a bounded number of polls and sets
// the error word; the block then runs to its end and frees its tensor memory.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <float.h>
#include <stdint.h>

#include "igc_device.cuh"
#include "igc_gemv.cuh"
#include "igc_kernels.h"
#include "igc_lanes.h"

namespace igc {

// ---------------------------------------------------------------------------
// tcgen05 helpers (PTX ISA 8.6+, sm_100a)

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (stride byte offset), leading byte offset unused (1),
// descriptor version 1, base offset 0 (every operand block is 1 KB aligned).
__device__ __forceinline__ uint64_t lg_desc(uint32_t smem_addr) {
  return (uint64_t)((smem_addr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor, kind::f16: f32 accumulator, f16 A and B, both
// K-major, N = LG_N, M = LG_M.
constexpr uint32_t LG_IDESC = (1u << 4) | ((uint32_t)(LG_N >> 3) << 17) | ((uint32_t)(LG_M >> 4) << 24);

__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(LG_IDESC), "r"(accumulate)
      : "memory");
}

// Arrives on `bar` once every earlier tcgen05.mma of this thread has completed.
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}

// 32 lanes x 32 columns of f32 accumulators: thread i gets row (lane base +
// i), columns col .. col + 31.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// One 3-D tensor load into shared memory, completed on an mbarrier (no
// multicast; the map covers this GPU's own memory only).  x, the innermost
// coordinate, is always 0 here.
__device__ __forceinline__ void tma_load3(void *dst, const CUtensorMap *map, int x, int y, int z, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];\n" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// Byte offset of the 16-byte piece j of row r inside one operand block.
__host__ __device__ __forceinline__ uint32_t lg_swz(int r, int j) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((j ^ (r & 7)) << 4));
}

// ---------------------------------------------------------------------------
// the GEMM

// Two rings.  The copy ring holds what the producer brings from global
// memory a step (the activations' hi and lo blocks, the row blocks' codes and
// scales); a slot is refilled once the products that read its activations
// have committed.  The weight ring holds the dequantised hi and lo weight
// blocks; the dequant warps refill a slot once the products of the step two
// back have committed.  Four copy slots let the copies run ahead of the
// dequant and the products by four steps.
constexpr int LG_RSTAGES = 4, LG_BSTAGES = 2;
constexpr int LG_OP_BYTES = 128 * 64 * 2;       // one operand block: 128 rows x 64 columns of f16, 16 KB
constexpr int LG_A_BYTES = LG_OP_BYTES;         // activations, hi (then lo)
constexpr int LG_B_BYTES = LG_OP_BYTES;         // weights, hi (then lo)
constexpr int LG_RB = LG_N / 16;                // row blocks a tile
constexpr int LG_CODE_BYTES = LG_RB * 512;      // 4 KB
constexpr int LG_SCALE_BYTES = LG_RB * 64;      // 512 B
// a copy slot: A hi, A lo, codes, scales, rounded to 1 KB; a weight slot: B hi, B lo
constexpr int LG_OFF_CODES = 2 * LG_A_BYTES, LG_OFF_SCALES = LG_OFF_CODES + LG_CODE_BYTES;
constexpr int LG_RSLOT = (LG_OFF_SCALES + LG_SCALE_BYTES + 1023) / 1024 * 1024;  // 37 KB
constexpr int LG_BSLOT = 2 * LG_B_BYTES;                                          // 32 KB
constexpr int LG_RING_BYTES = LG_RSTAGES * LG_RSLOT + LG_BSTAGES * LG_BSLOT;
constexpr int LG_BAR_BYTES = 256;
constexpr int LG_SMEM = 1024 + LG_RING_BYTES + LG_BAR_BYTES;  // + alignment slack
constexpr int LG_DQ_WARPS = 8;  // warps that turn codes into weights (then run the epilogue)
constexpr int LG_THREADS = 64 + 32 * LG_DQ_WARPS;
constexpr int LG_TRIES = 1 << 22;  // polls a wait makes before it gives up

__global__ void __launch_bounds__(LG_THREADS, 1)
    lane_gemm_kernel(LaneGemmArgs a, const __grid_constant__ CUtensorMap tm_codes,
                     const __grid_constant__ CUtensorMap tm_scales) {
  extern __shared__ __align__(1024) uint8_t lg_raw[];
  uint8_t *base = lg_raw + ((1024 - (smem_u32(lg_raw) & 1023)) & 1023);
  uint8_t *bring = base + LG_RSTAGES * LG_RSLOT;
  uint64_t *bars = reinterpret_cast<uint64_t *>(base + LG_RING_BYTES);
  uint64_t *full = bars, *rempty = full + LG_RSTAGES, *bfull = rempty + LG_RSTAGES, *bempty = bfull + LG_BSTAGES,
           *accf = bempty + LG_BSTAGES;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(accf + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nt = blockIdx.x, mt = blockIdx.y, z = blockIdx.z;
  const int c_lo = (a.n_cc * z) / a.split, c_hi = (a.n_cc * (z + 1)) / a.split, nk = c_hi - c_lo;
  const int rb0 = nt * LG_RB, rbv = min(LG_RB, a.n_rb - rb0);  // row blocks this tile holds

  if (tid == 0) {
    for (int s = 0; s < LG_RSTAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&rempty[s], 1);
    }
    for (int s = 0; s < LG_BSTAGES; ++s) {
      mbar_init(&bfull[s], 32 * LG_DQ_WARPS);
      mbar_init(&bempty[s], 1);
    }
    mbar_init(accf, 1);
    mbar_init_fence();
  }
  if (warp == 1) {  // LG_N columns of tensor memory: one f32 accumulator a tile column
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_slot)),
                 "r"(LG_N)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool failed = false;
  // the next kernel may start its own set-up; it waits for this one to end
  // before it reads anything this one writes
  pdl_release();

  if (warp == 0) {
    // producer: the staged activations (a hi and a lo 16 KB block) and the 8
    // row blocks' codes (8 x 512 B) and scales (8 x 64 B) of the step, the
    // weights by one tensor load each (row blocks past the plane arrive as
    // zeros).  The weights of the first steps are requested before the wait
    // on the kernel ahead (the stage that writes the activations); nothing
    // else is.
    const uint64_t policy = l2_evict_last();  // the activations are read again by the other tiles
    auto weights = [&](int k) {
      const int s = k % LG_RSTAGES, c = c_lo + k;
      uint8_t *st = base + s * LG_RSLOT;
      if (lane == 0) {
        mbar_expect(&full[s], (uint32_t)(2 * LG_A_BYTES + LG_CODE_BYTES + LG_SCALE_BYTES));
        tma_load3(st + LG_OFF_CODES, &tm_codes, 0, c, rb0, &full[s]);
        tma_load3(st + LG_OFF_SCALES, &tm_scales, 0, c, rb0, &full[s]);
      }
      __syncwarp();
    };
    auto acts = [&](int k) {
      const int s = k % LG_RSTAGES, c = c_lo + k;
      uint8_t *st = base + s * LG_RSLOT;
      if (lane < 2) {  // the activations' hi and lo blocks of this step
        const uint4 *src = a.a_tiles + (((size_t)mt * a.n_cc + c) * 2 + lane) * (LG_A_BYTES / 16);
        bulk_load(st + lane * LG_A_BYTES, src, LG_A_BYTES, &full[s], policy);
      }
    };
    const int first = nk < LG_RSTAGES ? nk : LG_RSTAGES;
    for (int k = 0; k < first; ++k) weights(k);
    pdl_wait();
    for (int k = 0; k < first; ++k) acts(k);
    for (int k = first; k < nk; ++k) {
      const int s = k % LG_RSTAGES;
      const bool ok = mbar_wait(&rempty[s], (uint32_t)(((k / LG_RSTAGES) - 1) & 1), failed ? 1 : LG_TRIES);
      if (__any_sync(0xffffffffu, !ok)) failed = true;
      weights(k);
      acts(k);
    }
  } else if (warp == 1) {
    // the MMA issuer: twelve K=16 products a 64-column step
    for (int k = 0; k < nk; ++k) {
      const int r = k % LG_RSTAGES, b = k % LG_BSTAGES;
      bool ok = mbar_wait(&full[r], (uint32_t)((k / LG_RSTAGES) & 1), failed ? 1 : LG_TRIES);
      ok = mbar_wait(&bfull[b], (uint32_t)((k / LG_BSTAGES) & 1), (failed || !ok) ? 1 : LG_TRIES) && ok;
      if (__any_sync(0xffffffffu, !ok)) failed = true;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t ah = smem_u32(base + r * LG_RSLOT), al = ah + LG_A_BYTES;
        const uint32_t bh = smem_u32(bring + b * LG_BSLOT), bl = bh + LG_B_BYTES;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint32_t o = kk * 32;  // 16 columns further along K inside the swizzled rows
          tc_mma(tmem, lg_desc(ah + o), lg_desc(bh + o), (k > 0 || kk > 0) ? 1u : 0u);
          tc_mma(tmem, lg_desc(al + o), lg_desc(bh + o), 1u);
          tc_mma(tmem, lg_desc(ah + o), lg_desc(bl + o), 1u);
        }
        tc_commit(&rempty[r]);  // both slots are free once these products complete
        tc_commit(&bempty[b]);
      }
      __syncwarp();
    }
    if (lane == 0) tc_commit(accf);
    __syncwarp();
  } else {
    // warps 2-9: codes to f16 hi/lo weights in the operand layout (one
    // 16-byte thread slot of one row block's tile each), then the epilogue
    const int dt = tid - 64;  // 0..255: row block dt / 32, thread slot dt % 32
    for (int k = 0; k < nk; ++k) {
      const int rs = k % LG_RSTAGES, b = k % LG_BSTAGES;
      bool ok = mbar_wait(&full[rs], (uint32_t)((k / LG_RSTAGES) & 1), failed ? 1 : LG_TRIES);
      if (k >= LG_BSTAGES)  // the products of the step two back have read this weight slot
        ok = mbar_wait(&bempty[b], (uint32_t)(((k / LG_BSTAGES) - 1) & 1), (failed || !ok) ? 1 : LG_TRIES) && ok;
      if (__any_sync(0xffffffffu, !ok)) failed = true;
      uint8_t *st = base + rs * LG_RSLOT;
      uint8_t *bh = bring + b * LG_BSLOT, *bl = bh + LG_B_BYTES;
      const uint4 *codes = reinterpret_cast<const uint4 *>(st + LG_OFF_CODES);
      const uint2 *scs = reinterpret_cast<const uint2 *>(st + LG_OFF_SCALES);
      {
        const int rbl = dt >> 5, ts = dt & 31, g = ts >> 2, tq = ts & 3;
        const int n0 = rbl * 16 + g, n8 = n0 + 8;
        const bool have = rbl < rbv;
        const uint4 w = have ? codes[rbl * 32 + ts] : make_uint4(0x88888888u, 0x88888888u, 0x88888888u, 0x88888888u);
        const uint2 sc = have ? scs[rbl * 8 + g] : make_uint2(0u, 0u);
        const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int kb = 0; kb < 4; ++kb) {
          // register r of the product: rows g (r even) or g+8 (r odd), columns
          // (c, c+1) for r < 2 and (c+8, c+9) above, c = 16 kb + 2 tq
          uint32_t q[4];
          dequant_i4(words[kb], q);
          const uint32_t sg = kb < 2 ? sc.x : sc.y;  // f16 scales of rows g (low half) and g+8 (high half)
          const __half2 s2 = *reinterpret_cast<const __half2 *>(&sg);
          const __half2 sr[2] = {__low2half2(s2), __high2half2(s2)};
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            // hi = the product rounded to f16; lo = the exact remainder (a
            // 4-bit integer times an f16 needs at most 15 significant bits,
            // so the fused multiply-add's one rounding leaves it as it is)
            const __half2 c2 = *reinterpret_cast<const __half2 *>(&q[r]);
            const __half2 hi = __hmul2(c2, sr[r & 1]);
            const __half2 lo = __hfma2(c2, sr[r & 1], __hneg2(hi));
            const uint32_t off = lg_swz((r & 1) ? n8 : n0, 2 * kb + (r >> 1)) + 4 * tq;
            *reinterpret_cast<__half2 *>(bh + off) = hi;
            *reinterpret_cast<__half2 *>(bl + off) = lo;
          }
        }
      }
      fence_async_smem();  // the weights written here are read by the tensor core (async proxy)
      mbar_arrive(&bfull[b]);
    }
    // epilogue: this warp's quarter of the tile's lanes (the wait returns at
    // once: the accumulators needed the activations the kernel ahead wrote)
    {
      const bool ok = mbar_wait(accf, 0u, failed ? 1 : LG_TRIES);
      if (__any_sync(0xffffffffu, !ok)) failed = true;
    }
    pdl_wait();
    tc_fence_after();
    // a warp may read the tensor-memory lanes of its quarter (warp mod 4):
    // warps 2-5 take columns 0-63 of their lanes, warps 6-9 columns 64-127
    const int q = warp & 3, c_first = warp < 6 ? 0 : LG_N / 2;
    const int m_local = q * 32 + lane, m = mt * LG_M + m_local;
    const bool live = m < a.lanes;
    const float f = live ? a.factor[m] : 0.0f;
    const int n_rows = a.n_rb * 16;
    const bool argm = a.arg_val != nullptr;
    float best = -FLT_MAX;
    int best_i = 0x7fffffff;
    float *orow = a.out ? a.out + ((size_t)z * a.lanes + (live ? m : 0)) * a.out_stride : nullptr;
    for (int c0 = c_first; c0 < c_first + LG_N / 2; c0 += 32) {
      const int n0 = nt * LG_N + c0;
      if (n0 >= n_rows) break;  // warp-uniform
      float v[32];
      tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0, v);
      if (argm) {
        // app_core.c:11755 kern_logit_cap, then app_main.c:482's argmax
        // (rows in increasing order: a strict > keeps the first index)
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          float x = v[i] * f;
          if (a.cap > 0.0f) x = logit_cap(x, a.cap);
          v[i] = x;
          if (n0 + i < a.rows && x > best) {
            best = x;
            best_i = n0 + i;
          }
        }
      }
      if (live && orow) {
        if (argm) {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (n0 + i < a.rows) orow[n0 + i] = v[i];
        } else if (n0 + 32 <= n_rows) {
          float4 *o4 = reinterpret_cast<float4 *>(orow + n0);
#pragma unroll
          for (int i = 0; i < 8; ++i) o4[i] = make_float4(v[4 * i] * f, v[4 * i + 1] * f, v[4 * i + 2] * f, v[4 * i + 3] * f);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (n0 + i < n_rows) orow[n0 + i] = v[i] * f;
        }
      }
    }
    if (argm) {
      // the two warps of a lane quarter meet in shared memory (the ring is
      // idle now: every product has completed); the column half 0 warp keeps
      // the first index on a tie
      float *bv = reinterpret_cast<float *>(base);
      int *bi = reinterpret_cast<int *>(base + LG_M * sizeof(float));
      if (c_first != 0) {
        bv[m_local] = best;
        bi[m_local] = best_i;
      }
      named_sync(1, 32 * LG_DQ_WARPS);
      if (c_first == 0 && live) {
        const float ov = bv[m_local];
        const int oi = bi[m_local];
        if (ov > best || (ov == best && oi < best_i)) {
          best = ov;
          best_i = oi;
        }
        a.arg_val[(size_t)nt * a.lanes + m] = best;
        a.arg_idx[(size_t)nt * a.lanes + m] = best_i;
      }
    }
    tc_fence_before();
  }
  if (failed && lane == 0) atomicOr(a.err, 1);
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(LG_N) : "memory");
  }
}

// ---------------------------------------------------------------------------
// the row-wise stage between two products

__device__ __forceinline__ float block_sum(float v, float *red) {
  // fixed order: warps in order, lanes by the xor tree
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[warp] = v;
  __syncthreads();
  float t = 0.0f;
  for (int w = 0; w < nw; ++w) t += red[w];
  return t;
}

__device__ __forceinline__ float block_max(float v, float *red) {
  v = warp_max(v);
  const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[warp] = v;
  __syncthreads();
  float t = 0.0f;
  for (int w = 0; w < nw; ++w) t = fmaxf(t, red[w]);
  return t;
}

// Columns a thread of the stage takes a step (see lane_stage_kernel).
constexpr int LS_U = 4;

__global__ void __launch_bounds__(256) lane_stage_kernel(LaneStageArgs a) {
  extern __shared__ float ls_row[];  // the lane's staged values (cols floats), then the residual's
  __shared__ float red[32];
  pdl_release();
  pdl_wait();  // every input comes from kernels ahead; the operand blocks are still read by the one just ahead
  const int j = blockIdx.x, tid = threadIdx.x, nt = blockDim.x;
  float *y = ls_row;
  const int n = a.cols;
  // Each thread takes columns tid, tid + nt, tid + 2 nt, ..., LS_U of them a
  // step, with every global load of the step issued before any is used (the
  // loads of one lane's row are independent; issuing them together keeps
  // several in flight).  Each thread still adds its columns in increasing
  // order, so every sum is the one a column-at-a-time loop forms.
  constexpr int U = LS_U;
  if (a.mode == LS_PLAIN || a.mode == LS_NORM) {
    const float *xr = a.x + (size_t)j * a.x_stride;
    for (int i0 = tid; i0 < n; i0 += U * nt) {
      float v[U];
#pragma unroll
      for (int k = 0; k < U; ++k) v[k] = i0 + k * nt < n ? xr[i0 + k * nt] : 0.0f;
#pragma unroll
      for (int k = 0; k < U; ++k)
        if (i0 + k * nt < n) y[i0 + k * nt] = v[k];
    }
  } else if (a.mode == LS_GELU_PAIR) {
    // app_core.c:11673 gelu(gate) * up: the pair plane interleaves 16-row
    // blocks of gate and up rows
    for (int i0 = tid; i0 < n; i0 += U * nt) {
      float g[U], u[U];
#pragma unroll
      for (int k = 0; k < U; ++k) g[k] = u[k] = 0.0f;
      for (int z = 0; z < a.p_splits; ++z) {
        const float *pz = a.p + ((size_t)z * a.lanes + j) * a.p_stride;
        float gv[U], uv[U];
#pragma unroll
        for (int k = 0; k < U; ++k) {
          const int i = i0 + k * nt, gi = (i >> 4) * 32 + (i & 15);
          gv[k] = i < n ? pz[gi] : 0.0f;
          uv[k] = i < n ? pz[gi + 16] : 0.0f;
        }
#pragma unroll
        for (int k = 0; k < U; ++k) {
          g[k] += gv[k];
          u[k] += uv[k];
        }
      }
#pragma unroll
      for (int k = 0; k < U; ++k)
        if (i0 + k * nt < n) y[i0 + k * nt] = gelu_tanh(g[k]) * u[k];
    }
  } else if (a.mode == LS_GELU_MUL) {
    // app_core.c:11723: gelu(gate) times the layer's per-layer input
    const float *ar = a.aux + (size_t)j * a.aux_stride;
    for (int i0 = tid; i0 < n; i0 += U * nt) {
      float g[U], m[U];
#pragma unroll
      for (int k = 0; k < U; ++k) {
        g[k] = 0.0f;
        m[k] = i0 + k * nt < n ? ar[i0 + k * nt] : 0.0f;
      }
      for (int z = 0; z < a.p_splits; ++z) {
        const float *pz = a.p + ((size_t)z * a.lanes + j) * a.p_stride;
        float gv[U];
#pragma unroll
        for (int k = 0; k < U; ++k) gv[k] = i0 + k * nt < n ? pz[i0 + k * nt] : 0.0f;
#pragma unroll
        for (int k = 0; k < U; ++k) g[k] += gv[k];
      }
#pragma unroll
      for (int k = 0; k < U; ++k)
        if (i0 + k * nt < n) y[i0 + k * nt] = gelu_tanh(g[k]) * m[k];
    }
  } else {
    // LS_RESID, LS_RESID_NORM (app_core.c:11690-11740): x += norm(p) * w_res,
    // then the layer gain; the new stream is written back
    float *pr = ls_row + n;
    float ss = 0.0f;
    for (int i0 = tid; i0 < n; i0 += U * nt) {
      float v[U];
#pragma unroll
      for (int k = 0; k < U; ++k) v[k] = 0.0f;
      for (int z = 0; z < a.p_splits; ++z) {
        const float *pz = a.p + ((size_t)z * a.lanes + j) * a.p_stride;
        float pv[U];
#pragma unroll
        for (int k = 0; k < U; ++k) pv[k] = i0 + k * nt < n ? pz[i0 + k * nt] : 0.0f;
#pragma unroll
        for (int k = 0; k < U; ++k) v[k] += pv[k];
      }
#pragma unroll
      for (int k = 0; k < U; ++k)
        if (i0 + k * nt < n) {
          pr[i0 + k * nt] = v[k];
          ss += v[k] * v[k];
        }
    }
    const float sp = rms_shrink(block_sum(ss, red), n, a.eps);
    const float *xr = a.x + (size_t)j * a.x_stride;
    float *xo = a.x_out + (size_t)j * a.x_stride;
    for (int i0 = tid; i0 < n; i0 += U * nt) {
      float xv[U], wv[U];
#pragma unroll
      for (int k = 0; k < U; ++k) {
        const bool in = i0 + k * nt < n;
        xv[k] = in ? xr[i0 + k * nt] : 0.0f;
        wv[k] = in ? a.w_res[i0 + k * nt] : 0.0f;
      }
#pragma unroll
      for (int k = 0; k < U; ++k) {
        const int i = i0 + k * nt;
        if (i < n) {
          float v = xv[k] + pr[i] * sp * wv[k];
          if (a.gain != 1.0f) v *= a.gain;
          y[i] = v;
          xo[i] = v;
        }
      }
    }
  }
  if (a.mode == LS_NORM || a.mode == LS_RESID_NORM) {
    __syncthreads();
    float ss = 0.0f;
    for (int i = tid; i < n; i += nt) ss += y[i] * y[i];
    const float sh = rms_shrink(block_sum(ss, red), n, a.eps);
    for (int i = tid; i < n; i += nt) y[i] = y[i] * sh * a.w_in[i];
  }
  __syncthreads();
  if (a.row_out)
    for (int i = tid; i < n; i += nt) a.row_out[(size_t)j * a.row_stride + i] = y[i];
  if (!a.a_tiles) return;
  float mx = 0.0f;
  for (int i = tid; i < n; i += nt) mx = fmaxf(mx, fabsf(y[i]));
  const float sc = lane_scale(block_max(mx, red));
  if (tid == 0) a.factor[j] = a.out_scale / sc;
  // f16 hi and lo pieces of eight columns into the operand blocks of (lane
  // tile, step); columns past the row are zero
  const int mt = j / LG_M, r = j % LG_M, pieces = a.n_cc * 8;
  uint8_t *dst = reinterpret_cast<uint8_t *>(a.a_tiles);
  for (int p = tid; p < pieces; p += nt) {
    const int c0 = p * 8, cc = p >> 3, pj = p & 7;
    uint32_t wh[4], wl[4];
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const float v0 = c0 + 2 * h < n ? y[c0 + 2 * h] * sc : 0.0f;
      const float v1 = c0 + 2 * h + 1 < n ? y[c0 + 2 * h + 1] * sc : 0.0f;
      const __half2 hv = __floats2half2_rn(v0, v1);
      const __half2 lv = __floats2half2_rn(v0 - __low2float(hv), v1 - __high2float(hv));
      wh[h] = *reinterpret_cast<const uint32_t *>(&hv);
      wl[h] = *reinterpret_cast<const uint32_t *>(&lv);
    }
    uint8_t *blk = dst + ((size_t)mt * a.n_cc + cc) * 2 * LG_OP_BYTES + lg_swz(r, pj);
    *reinterpret_cast<uint4 *>(blk) = make_uint4(wh[0], wh[1], wh[2], wh[3]);
    *reinterpret_cast<uint4 *>(blk + LG_OP_BYTES) = make_uint4(wl[0], wl[1], wl[2], wl[3]);
  }
}

// The output head's argmax partials merged per lane (first index on a tie).
__global__ void lane_argmax_kernel(const float *val, const int *idx, int parts, int lanes, int32_t *top) {
  pdl_release();
  pdl_wait();
  const int j = blockIdx.x, tid = threadIdx.x;
  __shared__ float sv[256];
  __shared__ int si[256];
  float v = -FLT_MAX;
  int i = 0x7fffffff;
  for (int p = tid; p < parts; p += blockDim.x) {
    const float ov = val[(size_t)p * lanes + j];
    const int oi = idx[(size_t)p * lanes + j];
    if (ov > v || (ov == v && oi < i)) {
      v = ov;
      i = oi;
    }
  }
  sv[tid] = v;
  si[tid] = i;
  __syncthreads();
  for (int w = blockDim.x / 2; w > 0; w >>= 1) {
    if (tid < w) {
      const float ov = sv[tid + w];
      const int oi = si[tid + w];
      if (ov > sv[tid] || (ov == sv[tid] && oi < si[tid])) {
        sv[tid] = ov;
        si[tid] = oi;
      }
    }
    __syncthreads();
  }
  if (tid == 0) top[j] = si[0];
}

// A pass's new key and value rows, written to an owner layer's cache before
// its attention runs (app_core.c:11500-11512): one block a lane at position
// *p0 + lane; keys normed (k_norm) and turned, values normed with no weight,
// each side stored as floats or, where its scale is positive, as e4m3 codes
// of value / scale.  A warp a head row; a lane holds dimensions d and d +
// hd/2 for d = lane + 32 e.  With every row of the pass in the cache, the
// attention of all its 16-lane groups runs as one launch.  With `tab` set,
// lane j belongs to session j / per at position tab->pos[j / per] + j % per,
// with that session's caches and peaks.
struct KvTables {
  const int *pos;
  float *const *kc, *const *vc, *const *peak;
  int per;
};

__global__ void __launch_bounds__(256) lane_kv_kernel(const float *qkv, int qkv_stride, int heads, int kv_heads,
                                                      int hd, const float *k_norm, const float *cs_tab,
                                                      const float *sn_tab, float eps, const int *p0, float *kc,
                                                      float *vc, CacheStore cq, KvTables tab) {
  pdl_release();
  pdl_wait();
  const int j = blockIdx.x;
  int p;
  if (tab.pos) {
    const int z = j / tab.per;
    p = tab.pos[z] + (j - z * tab.per);
    kc = tab.kc[z];
    vc = tab.vc[z];
    cq.peak = tab.peak ? tab.peak[z] : nullptr;
  } else {
    p = *p0 + j;
  }
  const int half = hd / 2, kv_w = kv_heads * hd;
  const int warp = threadIdx.x >> 5, l = threadIdx.x & 31;
  const float *row = qkv + (size_t)j * qkv_stride + (size_t)heads * hd;
  const float *cs = cs_tab + (size_t)p * half, *sn = sn_tab + (size_t)p * half;
  for (int it = warp; it < 2 * kv_heads; it += blockDim.x >> 5) {
    const bool is_v = it >= kv_heads;
    const int kh = is_v ? it - kv_heads : it;
    const float *src = row + (is_v ? kv_w : 0) + (size_t)kh * hd;
    const size_t at = (size_t)p * kv_w + (size_t)kh * hd;
    const float q = is_v ? cq.vq : cq.kq;  // a byte side's scale, else 0
    float *dst = (is_v ? vc : kc) + at;
    uint8_t *dstb = reinterpret_cast<uint8_t *>(is_v ? vc : kc) + at;
    float lo[8], hi[8], ss = 0.0f, mx = 0.0f;  // heads up to 512: d = lane + 32 e < 256
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int d = l + 32 * e;
      lo[e] = d < half ? src[d] : 0.0f;
      hi[e] = d < half ? src[d + half] : 0.0f;
      ss += lo[e] * lo[e] + hi[e] * hi[e];
    }
    const float sh = rms_shrink(warp_sum(ss), hd, eps);  // app_core.c:4667 kern_norm_rms
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int d = l + 32 * e;
      if (d >= half) continue;
      float x = lo[e] * sh, y = hi[e] * sh;
      if (!is_v) {
        x *= k_norm[d];
        y *= k_norm[d + half];
        const float c = cs[d], sv = sn[d];  // app_core.c:5196 kern_rope_turn: pairs (d, d + hd/2)
        const float x2 = x * c - y * sv, y2 = y * c + x * sv;
        x = x2;
        y = y2;
      }
      mx = fmaxf(mx, fmaxf(fabsf(x), fabsf(y)));
      if (q > 0.0f) {
        dstb[d] = (uint8_t)cache_store8(x, q);
        dstb[d + half] = (uint8_t)cache_store8(y, q);
      } else {
        dst[d] = x;
        dst[d + half] = y;
      }
    }
    // the row's largest magnitude (app_core.c:11208 cache_lay's peak)
    mx = warp_max(mx);
    if (cq.peak && l == 0) atomicMax(reinterpret_cast<int *>(cq.peak) + (is_v ? 1 : 0), __float_as_int(mx));
  }
}

// Rows of a layer's byte cache sides decoded into float rows the attention
// kernel reads (app_core.c:11050 cache_grid_fill's table: each code's grid
// value times the side's scale): block row z covers one session, rows [lo,
// p0 + lanes) with lo = p0 - span + 1 on a sliding layer (not below 0) and
// 0 on a global one, 16 codes a thread and step.  A float side is skipped.
__global__ void __launch_bounds__(256) lane_widen_kernel(WidenArgs w) {
  pdl_release();
  pdl_wait();
  const int z = blockIdx.y;
  const uint8_t *kc = w.kc_tab ? reinterpret_cast<const uint8_t *>(w.kc_tab[z]) : w.kc;
  const uint8_t *vc = w.vc_tab ? reinterpret_cast<const uint8_t *>(w.vc_tab[z]) : w.vc;
  float *kf = w.kf_tab ? w.kf_tab[z] : w.kf, *vf = w.vf_tab ? w.vf_tab[z] : w.vf;
  const int p0 = w.pos_tab ? w.pos_tab[z] : *w.p0;
  const int lo = w.sliding ? max(0, p0 - w.span + 1) : 0;
  const size_t first = (size_t)lo * w.kv_w, n16 = (size_t)(p0 + w.lanes - lo) * w.kv_w / 16;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += (size_t)gridDim.x * blockDim.x) {
    const size_t at = first + 16 * i;
#pragma unroll
    for (int side = 0; side < 2; ++side) {
      const float q = side ? w.vq : w.kq;
      if (!(q > 0.0f)) continue;
      const uint4 c = *reinterpret_cast<const uint4 *>((side ? vc : kc) + at);
      float4 *o = reinterpret_cast<float4 *>((side ? vf : kf) + at);
      const uint32_t ws[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
      for (int k = 0; k < 4; ++k)
        o[k] = make_float4(cache_load8(ws[k] & 0xFFu, q), cache_load8((ws[k] >> 8) & 0xFFu, q),
                           cache_load8((ws[k] >> 16) & 0xFFu, q), cache_load8(ws[k] >> 24, q));
    }
  }
}

// app_core.c:1930 quant_step: a value onto the signed 8-bit grid of `step`,
// rounding ties to even
__device__ __forceinline__ float grid_step(float v, float step) {
  const float level = fminf(fmaxf(rintf(__fdiv_rn(v, step)), -128.0f), 127.0f);
  return level * step;
}

// A plain plane's row r: where its codes, scales or dense values start, and
// how a column finds its scale (a shift for groups of a power of two).
struct PlainRow {
  const uint8_t *codes;
  const float *scales;
  int shift;  // log2 of the group size, or -1 (divide), or -2 (one group)
};

__device__ __forceinline__ PlainRow plain_row(const PlainArgs &a, int r) {
  PlainRow p;
  p.codes = a.codes ? a.codes + (size_t)r * a.stride : nullptr;
  p.scales = a.codes ? a.scales + (size_t)r * a.groups : nullptr;
  p.shift = a.groups == 1 ? -2 : ((a.group_size & (a.group_size - 1)) == 0 ? __ffs(a.group_size) - 1 : -1);
  return p;
}

__device__ __forceinline__ float plain_weight(const PlainArgs &a, const PlainRow &p, int r, int c) {
  if (p.codes) {
    const int bit = c * a.bits;
    uint32_t w = p.codes[bit >> 3] >> (bit & 7);
    if ((bit & 7) + a.bits > 8) w |= (uint32_t)p.codes[(bit >> 3) + 1] << (8 - (bit & 7));
    const int code = (int)((w & ((1u << a.bits) - 1u)) ^ a.flip);
    const int g = p.shift == -2 ? 0 : (p.shift >= 0 ? c >> p.shift : c / a.group_size);
    return (float)(code - a.bias) * p.scales[g];
  }
  const size_t i = (size_t)r * a.cols + c;
  if (a.dense_type == 1) return reinterpret_cast<const float *>(a.dense)[i];
  const uint16_t h = reinterpret_cast<const uint16_t *>(a.dense)[i];
  return a.dense_type == 2 ? __half2float(__ushort_as_half(h)) : __uint_as_float((uint32_t)h << 16);
}

// Eight weights of a row from column c0 (a multiple of 8) in one load: the
// codes of 1, 2, 4 or 8 bits (1-8 bytes) and their group's scale, or eight
// dense values.
__device__ __forceinline__ void plain_weight8(const PlainArgs &a, const PlainRow &p, int r, int c0, float (&w)[8]) {
  if (p.codes) {
    const uint8_t *at = p.codes + (c0 * a.bits >> 3);
    uint64_t v;
    switch (a.bits) {
      case 1: v = *at; break;
      case 2: v = *reinterpret_cast<const uint16_t *>(at); break;
      case 4: v = *reinterpret_cast<const uint32_t *>(at); break;
      default: v = *reinterpret_cast<const uint64_t *>(at); break;
    }
    const int g = p.shift == -2 ? 0 : (p.shift >= 0 ? c0 >> p.shift : c0 / a.group_size);
    const float sc = p.scales[g];
    const uint32_t mask = (1u << a.bits) - 1u;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int code = (int)(((uint32_t)(v >> (k * a.bits)) & mask) ^ a.flip);
      w[k] = (float)(code - a.bias) * sc;
    }
    return;
  }
  const size_t i = (size_t)r * a.cols + c0;
  if (a.dense_type == 1) {
    const float4 x0 = *reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(a.dense) + i);
    const float4 x1 = *reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(a.dense) + i + 4);
    w[0] = x0.x; w[1] = x0.y; w[2] = x0.z; w[3] = x0.w;
    w[4] = x1.x; w[5] = x1.y; w[6] = x1.z; w[7] = x1.w;
    return;
  }
  const uint4 h = *reinterpret_cast<const uint4 *>(reinterpret_cast<const uint16_t *>(a.dense) + i);
  const uint32_t hw[4] = {h.x, h.y, h.z, h.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint16_t lo = (uint16_t)(hw[k] & 0xFFFFu), hi = (uint16_t)(hw[k] >> 16);
    w[2 * k] = a.dense_type == 2 ? __half2float(__ushort_as_half(lo)) : __uint_as_float((uint32_t)lo << 16);
    w[2 * k + 1] = a.dense_type == 2 ? __half2float(__ushort_as_half(hi)) : __uint_as_float((uint32_t)hi << 16);
  }
}

// A warp a row at a time (the block's rows r0 + warp, + 8, ...; 32 rows a
// block, so even a small plane spreads over the SMs), LN lanes at a time.
// Where the row allows (`vec`: columns in eights that share a scale, code
// rows and input rows aligned for it) thread t takes eight columns at a time
// from 8t, 8t + 256, ..., one load of weights and two of each lane's inputs;
// otherwise, or for the columns past the last 256, the columns t, t + 32, ....
// Each lane's sum then goes by one fixed shuffle tree; it depends neither on
// LN nor on the other lanes.  The head keeps, per lane, the largest of the
// block's values (first row on a tie, app_main.c:482).
constexpr int PL_ROWS = 32;
template <int LN>
__global__ void __launch_bounds__(256) plain_product_kernel(PlainArgs a) {
  __shared__ float best_v[8][LN];
  __shared__ int best_i[8][LN];
  pdl_release();
  pdl_wait();
  const int warp = threadIdx.x >> 5, l = threadIdx.x & 31;
  const int r0 = blockIdx.x * PL_ROWS, r1 = min(r0 + PL_ROWS, a.rows);
  for (int g0 = 0; g0 < a.lanes; g0 += LN) {
    const int gl = min(LN, a.lanes - g0);
    float keep_v[LN];
    int keep_i[LN];
#pragma unroll
    for (int j = 0; j < LN; ++j) {
      keep_v[j] = -FLT_MAX;
      keep_i[j] = 0x7fffffff;
    }
    for (int r = r0 + warp; r < r1; r += 8) {
      const PlainRow pr = plain_row(a, r);
      float acc[LN];
#pragma unroll
      for (int j = 0; j < LN; ++j) acc[j] = 0.0f;
      int c_from = l;
      if (a.vec) {
        const int n8 = a.cols >> 3;
#pragma unroll 2
        for (int q = l; q < n8; q += 32) {
          const int c0 = q << 3;
          float w[8];
          plain_weight8(a, pr, r, c0, w);
#pragma unroll
          for (int j = 0; j < LN; ++j)
            if (j < gl) {
              const float *xr = a.x + (size_t)(g0 + j) * a.x_stride + c0;
              const float4 x0 = *reinterpret_cast<const float4 *>(xr);
              const float4 x1 = *reinterpret_cast<const float4 *>(xr + 4);
              float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
              if (a.enter > 0.0f)
#pragma unroll
                for (int k = 0; k < 8; ++k) xv[k] = grid_step(xv[k], a.enter);
              float t = acc[j];
#pragma unroll
              for (int k = 0; k < 8; ++k) t = fmaf(w[k], xv[k], t);
              acc[j] = t;
            }
        }
        c_from = (n8 << 3) + l;
      }
#pragma unroll 4
      for (int c = c_from; c < a.cols; c += 32) {
        const float w = plain_weight(a, pr, r, c);
#pragma unroll
        for (int j = 0; j < LN; ++j)
          if (j < gl) {
            float x = a.x[(size_t)(g0 + j) * a.x_stride + c];
            if (a.enter > 0.0f) x = grid_step(x, a.enter);
            acc[j] = fmaf(w, x, acc[j]);
          }
      }
#pragma unroll
      for (int j = 0; j < LN; ++j) {
        float v = warp_sum(acc[j]);
        if (j >= gl) continue;
        if (a.leave > 0.0f) v = grid_step(v, a.leave);
        v *= a.out_scale;
        if (a.cap > 0.0f) v = logit_cap(v, a.cap);
        if (l == 0 && a.out) {
          const int orow = a.pair_half >= 0 ? (r >> 4) * 32 + a.pair_half * 16 + (r & 15) : a.out_row0 + r;
          a.out[(size_t)(g0 + j) * a.out_stride + orow] = v;
        }
        if (v > keep_v[j]) {  // rows rise, so the first row wins a tie
          keep_v[j] = v;
          keep_i[j] = r;
        }
      }
    }
    if (a.arg_val) {
      if (l == 0)
#pragma unroll
        for (int j = 0; j < LN; ++j) {
          best_v[warp][j] = keep_v[j];
          best_i[warp][j] = keep_i[j];
        }
      __syncthreads();
      if (threadIdx.x < gl) {
        const int j = threadIdx.x;
        float v = best_v[0][j];
        int i = best_i[0][j];
        for (int w = 1; w < 8; ++w)
          if (best_v[w][j] > v || (best_v[w][j] == v && best_i[w][j] < i)) {
            v = best_v[w][j];
            i = best_i[w][j];
          }
        a.arg_val[(size_t)blockIdx.x * a.lanes + g0 + j] = v;
        a.arg_idx[(size_t)blockIdx.x * a.lanes + g0 + j] = i;
      }
      __syncthreads();
    }
  }
}

// K-slice partials added in order: out[j][i] = sum_z p[z][j][i].
__global__ void lane_sum_kernel(const float *p, int splits, int lanes, int cols, int p_stride, float *out,
                                int out_stride) {
  pdl_release();
  pdl_wait();
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long)lanes * cols) return;
  const int j = (int)(idx / cols), i = (int)(idx - (long)j * cols);
  float s = 0.0f;
  for (int z = 0; z < splits; ++z) s += p[((size_t)z * lanes + j) * p_stride + i];
  out[(size_t)j * out_stride + i] = s;
}

}  // namespace igc

using namespace igc;

// A launch that may overlap the kernel ahead of it (programmatic dependent
// launch) while the calling thread has that turned on (igc_kernels_pdl);
// every kernel here waits for the one ahead before it reads its results.
template <typename... KArgs, typename... Args>
static cudaError_t lane_launch(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
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
  cfg.numAttrs = igc_kernels_pdl_get() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

extern "C" {

size_t igc_lane_stage_smem(int mode, int cols) {
  return sizeof(float) * (size_t)cols * ((mode == LS_RESID || mode == LS_RESID_NORM) ? 2 : 1);
}

constexpr int LS_SMEM_LIMIT = 160 * 1024;  // a stage row (and a residual's partner row) in shared memory

cudaError_t igc_lanes_configure(void) {
  cudaError_t e = cudaFuncSetAttribute(lane_stage_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, LS_SMEM_LIMIT);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(lane_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, LG_SMEM);
  return e;
}

cudaError_t igc_launch_lane_stage(const LaneStageArgs *a, cudaStream_t st) {
  if (a->lanes < 1 || a->cols < 1) return cudaErrorInvalidValue;
  if (a->a_tiles ? a->cols > a->n_cc * 64 : (!a->row_out || a->row_stride < a->cols)) return cudaErrorInvalidValue;
  const size_t smem = igc_lane_stage_smem(a->mode, a->cols);
  if (smem > LS_SMEM_LIMIT) return cudaErrorInvalidValue;
  return lane_launch(lane_stage_kernel, dim3(a->lanes), dim3(256), smem, st, *a);
}

// Positions of a prefill chunk's 16-lane attention groups: out[i] = p0 + 16 i.
__global__ void lane_positions_kernel(const int *p0, int groups, int *out) {
  pdl_release();
  pdl_wait();
  const int i = threadIdx.x;
  if (i < groups) out[i] = *p0 + 16 * i;
}

cudaError_t igc_launch_lane_positions(const int *p0, int groups, int *out, cudaStream_t st) {
  if (groups < 1 || groups > 1024) return cudaErrorInvalidValue;
  return lane_launch(lane_positions_kernel, dim3(1), dim3(1024), 0, st, p0, groups, out);
}



int igc_lane_gemm_split(int lanes, int n_rb, int n_cc, int sm_count) {
  // the split that minimises waves x (steps a block + a block's fixed cost,
  // about six steps' worth: set-up, pipeline fill, epilogue), at least two
  // steps a slice; ties keep the fewer slices
  const int tiles = ((n_rb + LG_RB - 1) / LG_RB) * ((lanes + LG_M - 1) / LG_M);
  int best = 1;
  long best_cost = -1;
  for (int split = 1; split <= 16 && split * 2 <= n_cc; ++split) {
    const long waves = ((long)tiles * split + sm_count - 1) / sm_count;
    const long cost = waves * ((n_cc + split - 1) / split + 6);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = split;
    }
  }
  return best;
}

int igc_lane_tmaps(const void *tiles, const void *scales, int n_rb, int n_cc, CUtensorMap *codes_map,
                   CUtensorMap *scales_map) {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = [] {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      fn = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }();
  if (!encode || !tiles || !scales || n_rb < 1 || n_cc < 1) return -1;
  const cuuint32_t ones[3] = {1, 1, 1};
  // codes: 128 words a tile, tiles `n_cc` apart in a row block
  const cuuint64_t cdim[3] = {128, (cuuint64_t)n_cc, (cuuint64_t)n_rb};
  const cuuint64_t cstride[2] = {512, (cuuint64_t)n_cc * 512};
  const cuuint32_t cbox[3] = {128, 1, (cuuint32_t)LG_RB};
  // scales: 16 words a (row block, step) record
  const cuuint64_t sdim[3] = {16, (cuuint64_t)n_cc, (cuuint64_t)n_rb};
  const cuuint64_t sstride[2] = {64, (cuuint64_t)n_cc * 64};
  const cuuint32_t sbox[3] = {16, 1, (cuuint32_t)LG_RB};
  CUresult r = encode(codes_map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<void *>(tiles), cdim, cstride, cbox,
                      ones, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r == CUDA_SUCCESS)
    r = encode(scales_map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<void *>(scales), sdim, sstride, sbox, ones,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -1;
}

cudaError_t igc_launch_lane_gemm(const LaneGemmArgs *a, const CUtensorMap *codes_map, const CUtensorMap *scales_map,
                                 cudaStream_t st) {
  if (a->lanes < 1 || a->split < 1 || a->split > a->n_cc || a->n_rb < 1 || !codes_map || !scales_map)
    return cudaErrorInvalidValue;
  if (a->arg_val && (a->split != 1 || !a->arg_idx)) return cudaErrorInvalidValue;
  dim3 grid((a->n_rb + LG_RB - 1) / LG_RB, (a->lanes + LG_M - 1) / LG_M, a->split);
  return lane_launch(lane_gemm_kernel, grid, dim3(LG_THREADS), (size_t)LG_SMEM, st, *a, *codes_map, *scales_map);
}

cudaError_t igc_launch_lane_kv(const float *qkv, int qkv_stride, int heads, int kv_heads, int hd, const float *k_norm,
                               const float *cs, const float *sn, float eps, const int *p0, int lanes, float *kc,
                               float *vc, const CacheStore *store, cudaStream_t st) {
  return igc_launch_lane_kv_many(qkv, qkv_stride, heads, kv_heads, hd, k_norm, cs, sn, eps, p0, lanes, kc, vc, store,
                                 nullptr, nullptr, nullptr, nullptr, 0, st);
}

cudaError_t igc_launch_lane_kv_many(const float *qkv, int qkv_stride, int heads, int kv_heads, int hd,
                                    const float *k_norm, const float *cs, const float *sn, float eps, const int *p0,
                                    int lanes, float *kc, float *vc, const CacheStore *store, const int *pos_tab,
                                    float *const *kc_tab, float *const *vc_tab, float *const *peak_tab, int per,
                                    cudaStream_t st) {
  if (lanes < 1 || hd % 32 || hd > 512 || kv_heads < 1) return cudaErrorInvalidValue;
  if (pos_tab ? (!kc_tab || !vc_tab || per < 1 || lanes % per) : (!p0 || !kc || !vc)) return cudaErrorInvalidValue;
  CacheStore cq = {};
  if (store) cq = *store;
  if (!(cq.kq >= 0.0f) || !(cq.vq >= 0.0f)) return cudaErrorInvalidValue;
  KvTables tab = {pos_tab, kc_tab, vc_tab, peak_tab, per};
  return lane_launch(lane_kv_kernel, dim3(lanes), dim3(256), 0, st, qkv, qkv_stride, heads, kv_heads, hd, k_norm, cs,
                     sn, eps, p0, kc, vc, cq, tab);
}

cudaError_t igc_launch_plain_product(const PlainArgs *a, int sm_count, int *blocks_out, cudaStream_t st) {
  (void)sm_count;
  if (!a || a->rows < 1 || a->cols < 1 || a->lanes < 1 || !a->x) return cudaErrorInvalidValue;
  if (a->codes ? (a->bits < 1 || a->bits > 8 || !a->scales || a->groups < 1 || a->group_size < 1)
               : (!a->dense || a->dense_type < 1 || a->dense_type > 3))
    return cudaErrorInvalidValue;
  if (a->arg_val && !a->arg_idx) return cudaErrorInvalidValue;
  const int blocks = igc_plain_blocks(a->rows);
  if (blocks_out) *blocks_out = blocks;
  PlainArgs v = *a;
  // eight columns a load where the rows and groups line up for it
  v.vec = (a->x_stride % 4 == 0) && (a->cols % 8 == 0) && ((size_t)a->x % 16 == 0) &&
          (a->codes ? ((a->bits == 1 || a->bits == 2 || a->bits == 4 || a->bits == 8) && a->group_size % 8 == 0 &&
                       a->stride % (size_t)a->bits == 0 && (size_t)a->codes % 8 == 0)
                    : ((size_t)a->dense % 16 == 0)) ? 1 : 0;
  a = &v;
  if (a->lanes <= 4) return lane_launch(plain_product_kernel<4>, dim3(blocks), dim3(256), 0, st, *a);
  return lane_launch(plain_product_kernel<16>, dim3(blocks), dim3(256), 0, st, *a);
}

int igc_plain_blocks(int rows) { return (rows + PL_ROWS - 1) / PL_ROWS; }

cudaError_t igc_launch_lane_widen(const WidenArgs *w, int batch, int rows_most, int sm_count, cudaStream_t st) {
  if (!w || batch < 1 || rows_most < 1 || w->kv_w < 16 || w->kv_w % 16 || w->lanes < 1) return cudaErrorInvalidValue;
  if (!(w->kq >= 0.0f) || !(w->vq >= 0.0f)) return cudaErrorInvalidValue;
  if (batch > 1 && (!w->pos_tab || !w->kc_tab || !w->vc_tab || !w->kf_tab || !w->vf_tab)) return cudaErrorInvalidValue;
  if (!w->pos_tab && !w->p0) return cudaErrorInvalidValue;
  // enough blocks for the most rows a launch can see, at most about two
  // waves of the GPU in all (each thread then strides)
  const long steps = ((long)rows_most * w->kv_w / 16 + 255) / 256;
  long x = steps < 1 ? 1 : steps;
  const long cap = (2L * sm_count * 4 + batch - 1) / batch;
  if (x > cap) x = cap < 1 ? 1 : cap;
  return lane_launch(lane_widen_kernel, dim3((unsigned)x, batch), dim3(256), 0, st, *w);
}

cudaError_t igc_launch_lane_argmax(const float *val, const int *idx, int parts, int lanes, int32_t *top,
                                   cudaStream_t st) {
  if (lanes < 1 || parts < 1) return cudaErrorInvalidValue;
  return lane_launch(lane_argmax_kernel, dim3(lanes), dim3(256), 0, st, val, idx, parts, lanes, top);
}

cudaError_t igc_launch_lane_sum(const float *p, int splits, int lanes, int cols, int p_stride, float *out,
                                int out_stride, cudaStream_t st) {
  const long n = (long)lanes * cols;
  return lane_launch(lane_sum_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, st, p, splits, lanes, cols,
                     p_stride, out, out_stride);
}

}  // extern "C"
