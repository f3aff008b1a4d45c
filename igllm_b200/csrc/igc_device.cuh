// igc_device.cuh - device-side building blocks shared by the kernels.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace igc {

// One m16n8k16 tensor-core product, f16 inputs, f32 accumulate.
// A: 16 weight rows x 16 input columns (4 regs of f16x2 per thread),
// B: 16 input columns x 8 lanes (2 regs), C/D: 16 rows x 8 lanes (4 floats).
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1, const float (&c)[4]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%10,%11,%12,%13};\n"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]),
        "f"(c[2]), "f"(c[3]));
}

// Eight 4-bit codes (one 32-bit word, laid out by the upload repack) to the
// four f16x2 A-fragment registers of one m16n8k16 product, each value being
// code - 8 exactly.  Register k takes nibbles k and k+4 (bits 4k and 4k+16).
// The lop3 masks put a nibble under the f16 exponent of 1024 (0x6400): the
// low nibble of each half reads 1024 + n, the high one 1024 + 16 n; one
// subtract or one fused multiply-add then leaves n - 8 with no rounding
// (the integer-to-float construction of Kim et al., "Who Says Elephants
// Can't Run", 2022).
__device__ __forceinline__ void dequant_i4(uint32_t w, uint32_t (&a)[4]) {
  const uint32_t lo_mask = 0x000f000fu, hi_mask = 0x00f000f0u, magic = 0x64006400u;
  uint32_t w8 = w >> 8;
  uint32_t t0, t1, t2, t3;
  // (x & mask) | magic in one lop3: immLut = (0xF0 & 0xCC) | 0xAA = 0xEA
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;\n" : "=r"(t0) : "r"(w), "r"(lo_mask), "r"(magic));
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;\n" : "=r"(t1) : "r"(w), "r"(hi_mask), "r"(magic));
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;\n" : "=r"(t2) : "r"(w8), "r"(lo_mask), "r"(magic));
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;\n" : "=r"(t3) : "r"(w8), "r"(hi_mask), "r"(magic));
  const uint32_t sub_lo = 0x64086408u;  // 1032 = 1024 + 8
  const uint32_t mul_hi = 0x2c002c00u;  // 1/16
  const uint32_t add_hi = 0xd480d480u;  // -72 = -(64 + 8)
  asm("sub.f16x2 %0, %1, %2;\n" : "=r"(a[0]) : "r"(t0), "r"(sub_lo));
  asm("fma.rn.f16x2 %0, %1, %2, %3;\n" : "=r"(a[1]) : "r"(t1), "r"(mul_hi), "r"(add_hi));
  asm("sub.f16x2 %0, %1, %2;\n" : "=r"(a[2]) : "r"(t2), "r"(sub_lo));
  asm("fma.rn.f16x2 %0, %1, %2, %3;\n" : "=r"(a[3]) : "r"(t3), "r"(mul_hi), "r"(add_hi));
}

// Streaming 16-byte load that does not allocate in L1: every weight byte is
// read exactly once per pass.
__device__ __forceinline__ uint4 ld_stream(const uint4 *p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ uint2 ld_stream2(const uint2 *p) {
  uint2 r;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];\n"
               : "=r"(r.x), "=r"(r.y)
               : "l"(p));
  return r;
}

// ---- bulk copies into shared memory, completed on an mbarrier -------------

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Makes the initialised barriers visible to the copy engine.
__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}

// Arms the barrier for `bytes` of copies and counts this thread's arrival.
__device__ __forceinline__ void mbar_expect(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try(uint64_t *bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Waits for the barrier's phase `parity` to complete, giving up after
// `tries` polls (each poll may suspend the thread for a short while).
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int tries) {
  for (int i = 0; i < tries; ++i)
    if (mbar_try(bar, parity)) return true;
  return false;
}

// An L2 policy that lets streamed weights leave L2 first, so activations,
// partial sums and the key/value caches stay resident.
__device__ __forceinline__ uint64_t l2_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;\n" : "=l"(pol));
  return pol;
}

// The opposite, for data read again soon (the key/value caches).
__device__ __forceinline__ uint64_t l2_evict_last() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;\n" : "=l"(pol));
  return pol;
}

// One bulk copy global -> shared (no multicast); `bytes` and both addresses
// are multiples of 16.
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                          uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
      "%4;\n" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Orders this thread's earlier shared-memory reads before later bulk copies
// into the same bytes.
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }

// ---- programmatic dependent launch -----------------------------------------
// A kernel launched with programmatic stream serialisation may start before
// the kernel ahead of it has finished; it must not read what that kernel
// writes, nor write anything, before pdl_wait() returns.  pdl_release() lets
// the next kernel start early (it still waits for this one in its pdl_wait).
// Both are no-ops for a kernel launched without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_release() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }

// ---- launch stamps ---------------------------------------------------------
// A stamped launch keeps two words: the earliest time any of its blocks got
// past its wait on the kernel ahead (when it could start its real work) and
// the latest time a block finished.  Their difference is the launch's span
// on the critical path of the pass, measured inside the graphed pass itself.
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
  return t;
}
__device__ __forceinline__ void stamp_begin(unsigned long long *st) {
  if (st && threadIdx.x == 0) atomicMin(st, global_ns());
}
// Every thread of the block calls it (it holds a block barrier).
__device__ __forceinline__ void stamp_end(unsigned long long *st) {
  if (st) {
    __syncthreads();
    if (threadIdx.x == 0) atomicMax(st + 1, global_ns());
  }
}

__device__ __forceinline__ void named_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(threads) : "memory");
}

// ---- thread-block clusters -------------------------------------------------
// All blocks of a cluster arrive, then wait; what each wrote to shared memory
// before it arrived is visible to the others after the wait.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}

// Stores (x, y) at `p` in the shared memory of cluster block `rank` (8-byte
// aligned); visible there after the next cluster barrier.
__device__ __forceinline__ void st_cluster2(float *p, int rank, float x, float y) {
  uint32_t a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(a) : "r"(smem_u32(p)), "r"(rank));
  asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};\n" ::"r"(a), "f"(x), "f"(y) : "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// app_core.c:5109 kern_gelu_tanh: x * t / (t + 1), t = e^{2y}, y the tanh
// argument; zero below the clamp, the clamp caps t above.
__device__ __forceinline__ float gelu_tanh(float x) {
  const float root = 0.7978845608028654f, bend = 0.044715f, reach = 30.0f;
  float cube = x * x * x;
  float turn = 2.0f * root * (x + bend * cube);
  if (!(turn > -reach)) return x * 0.0f;
  if (turn > reach) turn = reach;
  float rise = expf(turn);
  return x * (rise / (rise + 1.0f));
}

// app_core.c:5016 kern_logit_cap_one
__device__ __forceinline__ float logit_cap(float x, float cap) {
  float t = x * (1.0f / cap);
  t = fminf(fmaxf(t, -10.0f), 10.0f);
  return cap * (1.0f - 2.0f / (expf(t + t) + 1.0f));
}

// The byte cache's 8-bit float, e4m3 (app_core.c:10975-11035 cache_pack8,
// cache_code8, cache_real8): one sign bit, four exponent bits biased by 7,
// three significand bits.  Exponent field 0 counts steps of 2^-9 outright;
// any other field e holds (8 + significand) * 2^(e - 10).  Encoding rounds to
// nearest with ties to even, saturates at +-448 (code 0x7E, so the NaN code
// 0x7F never appears), stores a NaN as +448 and anything that rounds to zero
// as +0.  Worked from the format's
// definition on the float's exponent bits: a in [2^e, 2^(e+1)) has steps of
// 2^(e-3), and the rounded step count q in [8, 16] gives the code
// ((e + 7) << 3) + q - 8, a carry into the next exponent when q is 16.
__device__ __forceinline__ uint32_t cache_code8(float x) {
  const uint32_t sign = x < 0.0f ? 0x80u : 0u;
  const float a = fabsf(x);
  if (!(a < 448.0f)) return sign | 0x7Eu;
  if (a < 0.015625f) {
    const uint32_t q = (uint32_t)rintf(a * 512.0f);
    return q ? sign | q : 0u;  // a value that rounds to zero stores +0
  }
  const int e = (int)((__float_as_uint(a) >> 23) & 0xFFu) - 127;
  const float q = rintf(a * __uint_as_float((uint32_t)(127 + 3 - e) << 23));
  return sign | (uint32_t)(((e + 7) << 3) + (int)q - 8);
}

__device__ __forceinline__ float cache_real8(uint32_t code) {
  const uint32_t f = (code >> 3) & 15u, m = code & 7u;
  const float a = f == 0 ? (float)m * 0.001953125f : (float)(8u + m) * __uint_as_float((f + 127u - 10u) << 23);
  return (code & 0x80u) ? -a : a;
}

// A quantized embedding table as the export stores it (app_core.c:7886
// plane_bind_gemma, `embedding_quantized` + `embedding_scale`): codes of
// `bits` bits packed from the low bit, `stride` bytes a row, a value being
// the code minus 2^(bits-1), times the f16 scale of its 32-column group
// (`scales` [rows][g32]).  `codes` null: the table is bf16 instead.
struct EmbedCodes {
  const uint8_t *codes;
  size_t stride;
  int bits;
  const uint16_t *scales;
  int g32;
};

// The value of column c of row r of a code table (app_core.c:1826 plane_row).
__device__ __forceinline__ float embed_code(const EmbedCodes &t, size_t r, int c) {
  const size_t bit = (size_t)c * t.bits;  // 1, 2 or 4 bits: never across a byte
  const uint32_t v = (uint32_t)(t.codes[r * t.stride + (bit >> 3)] >> (bit & 7)) & ((1u << t.bits) - 1u);
  const float scale = __half2float(__ushort_as_half(t.scales[r * t.g32 + (c >> 5)]));
  return (float)((int)v - (1 << (t.bits - 1))) * scale;
}

// How a layer's key and value caches are stored, and where the largest
// magnitudes written go.  A side whose scale is 0 holds float rows; a
// positive scale makes it e4m3 bytes of value / scale (written by
// lane_kv_kernel, read back as float rows by lane_widen_kernel; the
// attention kernel itself reads float rows only).  `peak` ([key, value]) or,
// for a batched launch, peak_tab[block z] takes the running maximum of
// |value| over every row written (app_core.c:11208 cache_lay).
struct CacheStore {
  float kq, vq;
  float *peak;
  float *const *peak_tab;
};

// A stored value of a byte side: the decoded grid value times the side's
// scale, one rounding, as the reference's dequantizing table holds it
// (app_core.c:11050 cache_grid_fill).
__device__ __forceinline__ float cache_load8(uint32_t code, float scale) { return __fmul_rn(cache_real8(code), scale); }

// A value's code on a byte side: value / scale onto the grid (app_core.c:11205
// cache_lay divides by the scale, then cache_code8).
__device__ __forceinline__ uint32_t cache_store8(float x, float scale) { return cache_code8(__fdiv_rn(x, scale)); }

}  // namespace igc
