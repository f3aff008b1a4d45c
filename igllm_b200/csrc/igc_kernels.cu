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
template <int NT, int PAIR, int PRO, int EPI>
__global__ void __launch_bounds__(GEMV_THREADS) gemv_kernel(GemvArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  uint32_t *stage = reinterpret_cast<uint32_t *>(smem_raw);
  const size_t stage_bytes = gemv_stage_bytes(a.pl.n_cc, NT);
  float *red = reinterpret_cast<float *>(smem_raw + stage_bytes);  // [8 warps][32][8*NT]

  gemv_prologue<PRO>(a, stage, red, NT);

  const int warp = threadIdx.x >> 5, lane32 = threadIdx.x & 31;
  const int g = lane32 >> 2, t = lane32 & 3;
  const int S = a.split;
  const int per_iter = GEMV_WARPS / S;  // row-block units a CTA takes at once
  const int n_units = PAIR ? a.pl.n_rb / 2 : a.pl.n_rb;
  const int my_unit_off = warp / S, my_slice = warp % S;
  const int c_lo = (a.pl.n_cc * my_slice) / S, c_hi = (a.pl.n_cc * (my_slice + 1)) / S;

  // EPI_LOGITS running argmax per (nt, lane parity)
  float best_v[NT][2];
  int best_i[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    best_v[nt][0] = best_v[nt][1] = -FLT_MAX;
    best_i[nt][0] = best_i[nt][1] = 0x7fffffff;
  }

  for (int base = blockIdx.x * per_iter; base < n_units; base += gridDim.x * per_iter) {
    const int unit = base + my_unit_off;
    const bool active = unit < n_units;
    float tot[PAIR + 1][NT][4];
#pragma unroll
    for (int h = 0; h <= PAIR; ++h)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) tot[h][nt][i] = 0.0f;

    if (active) {
      constexpr int D = 4;  // chunks in flight per warp
      uint4 wbuf[PAIR + 1][D];
      uint2 sbuf[PAIR + 1][D];
      const int rb0 = PAIR ? unit * 2 : unit;
#pragma unroll
      for (int d = 0; d < D; ++d)
        if (c_lo + d < c_hi)
#pragma unroll
          for (int h = 0; h <= PAIR; ++h) {
            long tile = (long)(rb0 + h) * a.pl.n_cc + c_lo + d;
            wbuf[h][d] = ld_stream(a.pl.tiles + tile * 32 + lane32);
            sbuf[h][d] = ld_stream2(a.pl.scales + tile * 8 + g);
          }
      for (int c = c_lo; c < c_hi; c += D) {
#pragma unroll
        for (int d = 0; d < D; ++d) {
          if (c + d < c_hi) {
            uint4 w[PAIR + 1];
            uint2 s[PAIR + 1];
#pragma unroll
            for (int h = 0; h <= PAIR; ++h) {
              w[h] = wbuf[h][d];
              s[h] = sbuf[h][d];
            }
            const int cn = c + d + D;
            if (cn < c_hi)
#pragma unroll
              for (int h = 0; h <= PAIR; ++h) {
                long tile = (long)(rb0 + h) * a.pl.n_cc + cn;
                wbuf[h][d] = ld_stream(a.pl.tiles + tile * 32 + lane32);
                sbuf[h][d] = ld_stream2(a.pl.scales + tile * 8 + g);
              }
            uint4 b[NT][4];
            load_b<NT>(stage, c + d, lane32, b);
#pragma unroll
            for (int h = 0; h <= PAIR; ++h) chunk_product<NT>(w[h], s[h], b, tot[h]);
          }
        }
      }
    }

    // combine the S warps that shared this unit, in a fixed order
    if (S > 1) {
      float *mine = red + (warp * 32 + lane32) * (8 * NT);
#pragma unroll
      for (int h = 0; h <= PAIR; ++h)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int i = 0; i < 4; ++i) mine[(h * NT + nt) * 4 + i] = tot[h][nt][i];
      __syncthreads();
      if (my_slice == 0) {
        for (int o = 1; o < S; ++o) {
          const float *other = red + ((warp + o) * 32 + lane32) * (8 * NT);
#pragma unroll
          for (int h = 0; h <= PAIR; ++h)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
              for (int i = 0; i < 4; ++i) tot[h][nt][i] += other[(h * NT + nt) * 4 + i];
        }
      }
      __syncthreads();
    }

    if (active && my_slice == 0) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int row = unit * 16 + g + (i >= 2 ? 8 : 0);
          const int ln = nt * 8 + 2 * t + (i & 1);
          if (row >= a.pl.rows || ln >= a.lanes) continue;
          float v = tot[0][nt][i];
          if (EPI == EPI_STORE) {
            a.out[(size_t)ln * a.out_stride + row] = v * a.out_scale;
          } else if (EPI == EPI_GELU_PAIR) {
            a.out[(size_t)ln * a.out_stride + row] = gelu_tanh(v) * tot[PAIR][nt][i];
          } else if (EPI == EPI_GELU_MUL) {
            a.out[(size_t)ln * a.out_stride + row] =
                gelu_tanh(v) * a.aux[(size_t)ln * a.aux_stride + row];
          } else {  // EPI_LOGITS
            float cv = a.cap > 0.0f ? logit_cap(v, a.cap) : v;
            a.out[(size_t)ln * a.out_stride + row] = cv;
            const int k = i & 1;
            if (cv > best_v[nt][k] || (cv == best_v[nt][k] && row < best_i[nt][k])) {
              best_v[nt][k] = cv;
              best_i[nt][k] = row;
            }
          }
        }
    }
  }

  if (EPI == EPI_LOGITS) {
    // reduce across the 8 thread groups that hold the same lanes, then across
    // the warps of the block; block partials go to part_val / part_idx
    __shared__ float bv[GEMV_WARPS][16];
    __shared__ int bi[GEMV_WARPS][16];
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
    if (threadIdx.x < NT * 8) {
      float v = bv[0][threadIdx.x];
      int i = bi[0][threadIdx.x];
      for (int w = 1; w < GEMV_WARPS; ++w) {
        float ov = bv[w][threadIdx.x];
        int oi = bi[w][threadIdx.x];
        if (ov > v || (ov == v && oi < i)) {
          v = ov;
          i = oi;
        }
      }
      a.part_val[blockIdx.x * 16 + threadIdx.x] = v;
      a.part_idx[blockIdx.x * 16 + threadIdx.x] = i;
    }
  }
}

// ---------------------------------------------------------------------------
// embedding rows (app_core.c:11863-11874, :11886-11891)
__global__ void embed_kernel(const int32_t *ids, int lanes, const uint16_t *embed, int hidden,
                             float embed_gain, const uint16_t *ple_embed, int ple_vocab,
                             int ple_width, float ple_gain, float *x_out, float *seed_out) {
  int j = blockIdx.x;
  if (j >= lanes) return;
  int id = ids[j];
  const uint16_t *row = embed + (size_t)id * hidden;
  for (int i = threadIdx.x; i < hidden; i += blockDim.x)
    x_out[(size_t)j * hidden + i] = __uint_as_float((uint32_t)row[i] << 16) * embed_gain;
  if (ple_embed) {
    const uint16_t *srow = ple_embed + (size_t)(id % ple_vocab) * ple_width;
    for (int i = threadIdx.x; i < ple_width; i += blockDim.x)
      seed_out[(size_t)j * ple_width + i] = __uint_as_float((uint32_t)srow[i] << 16) * ple_gain;
  }
}

// app_core.c:11892-11903: each per-layer chunk normed with the shared weight,
// then (chunk + seed) / sqrt(2).  One block a (lane, chunk).
__global__ void ple_finish_kernel(const float *raw, const float *seed, int lanes, int layers,
                                  int ple_dim, const float *w, float eps, float blend, float *out) {
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
// attention, step 1: q heads normed and turned, and for an owner layer the
// new key and value rows normed, turned and written into the cache
// (app_core.c:11481-11512).  One block a lane, one warp a head.
__global__ void attn_prep_kernel(float *qkv, int qkv_stride, int heads, int kv_heads, int hd,
                                 const float *q_norm, const float *k_norm, const float *cs_tab,
                                 const float *sn_tab, int owner, float eps, const int *d_p0, int lanes,
                                 float *kc, float *vc) {
  int j = blockIdx.x;
  if (j >= lanes) return;
  int pos = *d_p0 + j;
  int warp = threadIdx.x >> 5, l32 = threadIdx.x & 31, nw = blockDim.x >> 5;
  int half = hd / 2;
  const float *cs = cs_tab + (size_t)pos * half;
  const float *sn = sn_tab + (size_t)pos * half;
  float *row = qkv + (size_t)j * qkv_stride;
  int n_q = heads, n_k = owner ? kv_heads : 0, n_v = owner ? kv_heads : 0;
  int kv_w = kv_heads * hd;
  for (int item = warp; item < n_q + n_k + n_v; item += nw) {
    float *v;
    const float *w;
    bool turn;
    float *cache = nullptr;
    if (item < n_q) {
      v = row + (size_t)item * hd;
      w = q_norm;
      turn = true;
    } else if (item < n_q + n_k) {
      int kh = item - n_q;
      v = row + (size_t)heads * hd + (size_t)kh * hd;
      w = k_norm;
      turn = true;
      cache = kc + (size_t)pos * kv_w + (size_t)kh * hd;
    } else {
      int vh = item - n_q - n_k;
      v = row + (size_t)heads * hd + kv_w + (size_t)vh * hd;
      w = nullptr;
      turn = false;
      cache = vc + (size_t)pos * kv_w + (size_t)vh * hd;
    }
    float s = 0.0f;
    for (int d = l32; d < hd; d += 32) s += v[d] * v[d];
    float sh = (float)(1.0 / sqrt((double)warp_sum(s) / (double)hd + (double)eps));
    __syncwarp();
    // normalise and turn, pairs (d, d + half) handled by one thread
    for (int d = l32; d < half; d += 32) {
      float lo = v[d] * sh, hi = v[d + half] * sh;
      if (w) {
        lo *= w[d];
        hi *= w[d + half];
      }
      if (turn) {
        float c = cs[d], si = sn[d];
        float nlo = lo * c - hi * si;
        float nhi = hi * c + lo * si;
        lo = nlo;
        hi = nhi;
      }
      v[d] = lo;
      v[d + half] = hi;
      if (cache) {
        cache[d] = lo;
        cache[d + half] = hi;
      }
    }
  }
}

// attention, step 2: one block a span chunk and a group of up to 8 lanes; the
// block's partial softmax (max, sum) and weighted value sum go to the
// partials, combined by attn_combine_kernel.  Score scale is 1.0
// (app_core.c:11314); sliding layers see [pos - span + 1, pos]
// (app_core.c:11515-11518).
constexpr int ATT_TILE = 16;
constexpr int ATT_LANES = 8;

__host__ __device__ inline size_t attn_smem_floats(int heads, int hd, int kv_w) {
  size_t pairs = (size_t)ATT_LANES * heads;
  return pairs * hd                    /* qs   */
         + (size_t)ATT_TILE * (kv_w + 1) /* ks   */
         + (size_t)ATT_TILE * kv_w       /* vs   */
         + pairs * ATT_TILE              /* sc   */
         + pairs                         /* fac  */
         + pairs * hd                    /* acc  */
         + 2 * pairs;                    /* m, l */
}

__global__ void __launch_bounds__(256) attn_chunk_kernel(const float *qkv, int qkv_stride, int heads,
                                                         int hd, const float *kc, const float *vc,
                                                         int kv_w, int group, int sliding, int span,
                                                         const int *d_p0, int lanes,
                                                         float *part_ml, float *part_acc) {
  extern __shared__ __align__(16) float sm[];
  const int chunk = blockIdx.x, lg = blockIdx.y;
  // The span every lane of the block reads, [lo_all, p0 + lanes), is cut into
  // gridDim.x chunks of a whole number of tiles; the chunk length follows the
  // position so one launch shape serves every position.
  const int p0 = *d_p0;
  const int lo_all = sliding ? max(0, p0 - span + 1) : 0;
  const int span_all = p0 + lanes - lo_all;
  const int per = ATT_TILE * (int)gridDim.x;
  const int chunk_len = ATT_TILE * ((span_all + per - 1) / per);
  if (chunk * chunk_len >= span_all) return;  // past the span: the combine never reads it
  const int j0 = lg * ATT_LANES;
  const int nl = min(ATT_LANES, lanes - j0);
  const int pairs = nl * heads;
  const int pmax = ATT_LANES * heads;
  float *qs = sm;                                  // [pmax][hd]
  float *ks = qs + (size_t)pmax * hd;              // [TILE][kv_w + 1]
  float *vs = ks + (size_t)ATT_TILE * (kv_w + 1);  // [TILE][kv_w]
  float *sc = vs + (size_t)ATT_TILE * kv_w;        // [pmax][TILE]
  float *fac = sc + (size_t)pmax * ATT_TILE;       // [pmax]
  float *acc = fac + pmax;                         // [pmax][hd]
  float *mrun = acc + (size_t)pmax * hd;           // [pmax]
  float *lrun = mrun + pmax;                       // [pmax]

  const int c_from = lo_all + chunk * chunk_len;
  const int c_upto = min(c_from + chunk_len, p0 + lanes);
  for (int i = threadIdx.x; i < pairs * hd; i += blockDim.x) {
    int pr = i / hd, d = i % hd;
    int j = j0 + pr / heads, h = pr % heads;
    qs[i] = qkv[(size_t)j * qkv_stride + (size_t)h * hd + d];
    acc[i] = 0.0f;
  }
  for (int i = threadIdx.x; i < pairs; i += blockDim.x) {
    mrun[i] = -FLT_MAX;
    lrun[i] = 0.0f;
  }
  for (int tb = c_from; tb < c_upto; tb += ATT_TILE) {
    const int tn = min(ATT_TILE, c_upto - tb);
    __syncthreads();
    for (int i = threadIdx.x; i < tn * kv_w; i += blockDim.x) {
      int r = i / kv_w, d = i % kv_w;
      ks[r * (kv_w + 1) + d] = kc[(size_t)(tb + r) * kv_w + d];
      vs[r * kv_w + d] = vc[(size_t)(tb + r) * kv_w + d];
    }
    __syncthreads();
    // scores: thread -> (pair, position)
    for (int i = threadIdx.x; i < pairs * ATT_TILE; i += blockDim.x) {
      int pr = i / ATT_TILE, r = i % ATT_TILE;
      int j = j0 + pr / heads, h = pr % heads;
      int pos = tb + r;
      float s = -FLT_MAX;
      int lo_j = sliding ? max(0, p0 + j - span + 1) : 0;
      if (r < tn && pos <= p0 + j && pos >= lo_j) {
        const float *kr = ks + r * (kv_w + 1) + (h / group) * hd;
        const float *q = qs + (size_t)pr * hd;
        float t = 0.0f;
        for (int d = 0; d < hd; ++d) t += kr[d] * q[d];
        s = t;
      }
      sc[pr * ATT_TILE + r] = s;
    }
    __syncthreads();
    // online softmax update, one thread a pair
    for (int pr = threadIdx.x; pr < pairs; pr += blockDim.x) {
      float m_old = mrun[pr], m_new = m_old;
      for (int r = 0; r < tn; ++r) m_new = fmaxf(m_new, sc[pr * ATT_TILE + r]);
      float f = (m_new == -FLT_MAX) ? 1.0f : ((m_old == -FLT_MAX) ? 0.0f : expf(m_old - m_new));
      float l = lrun[pr] * f;
      for (int r = 0; r < ATT_TILE; ++r) {
        float s = sc[pr * ATT_TILE + r];
        float e = (r < tn && s != -FLT_MAX) ? expf(s - m_new) : 0.0f;
        sc[pr * ATT_TILE + r] = e;
        l += e;
      }
      lrun[pr] = l;
      mrun[pr] = m_new;
      fac[pr] = f;
    }
    __syncthreads();
    // weighted values: thread -> (pair, dimension)
    for (int i = threadIdx.x; i < pairs * hd; i += blockDim.x) {
      int pr = i / hd, d = i % hd;
      int h = pr % heads;
      const float *vcol = vs + (h / group) * hd + d;
      float a = acc[i] * fac[pr];
      for (int r = 0; r < tn; ++r) a += sc[pr * ATT_TILE + r] * vcol[r * kv_w];
      acc[i] = a;
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < pairs * hd; i += blockDim.x) {
    int pr = i / hd, d = i % hd;
    int j = j0 + pr / heads, h = pr % heads;
    part_acc[(((size_t)chunk * 16 + j) * heads + h) * hd + d] = acc[i];
  }
  for (int pr = threadIdx.x; pr < pairs; pr += blockDim.x) {
    int j = j0 + pr / heads, h = pr % heads;
    part_ml[(((size_t)chunk * 16 + j) * heads + h) * 2 + 0] = mrun[pr];
    part_ml[(((size_t)chunk * 16 + j) * heads + h) * 2 + 1] = lrun[pr];
  }
}

// attention, step 3: the chunks' partials merged into each head's output,
// (sum_c acc_c e^{m_c - M}) / (sum_c l_c e^{m_c - M}).  One block a
// (lane, head); the chunk weights are formed once, then one thread a
// dimension sums the chunks with independent loads.
__global__ void attn_combine_kernel(const float *part_ml, const float *part_acc, int n_grid, int lanes,
                                    int heads, int hd, int sliding, int span, const int *d_p0, float *out,
                                    int out_stride) {
  __shared__ float wgt[1024];
  __shared__ float tot;
  int j = blockIdx.x / heads, h = blockIdx.x % heads;
  if (j >= lanes) return;
  const int p0 = *d_p0;
  const int lo_all = sliding ? max(0, p0 - span + 1) : 0;
  const int span_all = p0 + lanes - lo_all;
  const int per = ATT_TILE * n_grid;
  const int chunk_len = ATT_TILE * ((span_all + per - 1) / per);
  const int n_chunks = (span_all + chunk_len - 1) / chunk_len;
  if (threadIdx.x < 32) {
    float M = -FLT_MAX;
    for (int c = threadIdx.x; c < n_chunks; c += 32) M = fmaxf(M, part_ml[(((size_t)c * 16 + j) * heads + h) * 2]);
    M = warp_max(M);
    float L = 0.0f;
    for (int c = threadIdx.x; c < n_chunks; c += 32) {
      float m = part_ml[(((size_t)c * 16 + j) * heads + h) * 2];
      float w = (m == -FLT_MAX) ? 0.0f : expf(m - M);
      wgt[c] = w;
      L += part_ml[(((size_t)c * 16 + j) * heads + h) * 2 + 1] * w;
    }
    L = warp_sum(L);
    if (threadIdx.x == 0) tot = L;
  }
  __syncthreads();
  const float inv = 1.0f / tot;
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    float o = 0.0f;
#pragma unroll 8
    for (int c = 0; c < n_chunks; ++c) o += part_acc[(((size_t)c * 16 + j) * heads + h) * hd + d] * wgt[c];
    out[(size_t)j * out_stride + (size_t)h * hd + d] = o * inv;
  }
}

// argmax partials of the output head merged per lane (app_main.c:482: the
// first index of the largest value)
__global__ void argmax_final_kernel(const float *part_val, const int *part_idx, int parts, int lanes,
                                    int32_t *top_out) {
  int j = threadIdx.x;
  if (j >= lanes) return;
  float v = -FLT_MAX;
  int i = 0x7fffffff;
  for (int p = 0; p < parts; ++p) {
    float ov = part_val[p * 16 + j];
    int oi = part_idx[p * 16 + j];
    if (ov > v || (ov == v && oi < i)) {
      v = ov;
      i = oi;
    }
  }
  top_out[j] = i;
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

static size_t gemv_smem_nt(const GemvArgs &a, int NT) {
  size_t red = a.split > 1 ? (size_t)GEMV_WARPS * 32 * 8 * NT * 4 : 0;
  if (red < (size_t)GEMV_WARPS * 16 * 4) red = (size_t)GEMV_WARPS * 16 * 4;
  return gemv_stage_bytes(a.pl.n_cc, NT) + red;
}

template <int NT, int PAIR, int PRO, int EPI>
static cudaError_t launch_gemv_t(const GemvArgs &a, int grid, cudaStream_t st) {
  size_t smem = gemv_smem_nt(a, NT);
  gemv_kernel<NT, PAIR, PRO, EPI><<<grid, GEMV_THREADS, smem, st>>>(a);
  return cudaGetLastError();
}

template <int NT, int PAIR>
static cudaError_t launch_gemv_pe(const GemvArgs &a, int pro, int epi, int grid, cudaStream_t st) {
#define IGC_CASE(P, E) \
  if (pro == P && epi == E) return launch_gemv_t<NT, PAIR, P, E>(a, grid, st);
  if constexpr (PAIR) {
    IGC_CASE(PRO_RESID_NORM, EPI_GELU_PAIR)
    IGC_CASE(PRO_NORM, EPI_GELU_PAIR)
    IGC_CASE(PRO_F32, EPI_GELU_PAIR)
  } else {
    IGC_CASE(PRO_F32, EPI_STORE)
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
  return cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn > 0 ? dyn : 0);
}

template <int NT, int PAIR, int PRO, int EPI>
static cudaError_t allow_smem_t(int bytes) {
  return allow_smem_fn(gemv_kernel<NT, PAIR, PRO, EPI>, bytes);
}

template <int NT>
static cudaError_t allow_smem_nt(int bytes) {
  cudaError_t e = cudaSuccess;
#define IGC_ALLOW(PAIR, P, E) \
  if (e == cudaSuccess) e = allow_smem_t<NT, PAIR, P, E>(bytes);
  IGC_ALLOW(1, PRO_RESID_NORM, EPI_GELU_PAIR)
  IGC_ALLOW(1, PRO_NORM, EPI_GELU_PAIR)
  IGC_ALLOW(1, PRO_F32, EPI_GELU_PAIR)
  IGC_ALLOW(0, PRO_F32, EPI_STORE)
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
  e = allow_smem_nt<1>(bytes);
  if (e == cudaSuccess) e = allow_smem_nt<2>(bytes);
  if (e == cudaSuccess) e = allow_smem_fn(attn_chunk_kernel, bytes);
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

cudaError_t igc_launch_gemv(const GemvArgs *a, int pair, int pro, int epi, int grid, cudaStream_t st) {
  int NT = (a->lanes + 7) / 8;
  if (NT == 1) return pair ? launch_gemv_pe<1, 1>(*a, pro, epi, grid, st) : launch_gemv_pe<1, 0>(*a, pro, epi, grid, st);
  return pair ? launch_gemv_pe<2, 1>(*a, pro, epi, grid, st) : launch_gemv_pe<2, 0>(*a, pro, epi, grid, st);
}

size_t igc_gemv_smem(const GemvArgs *a) { return gemv_smem_nt(*a, (a->lanes + 7) / 8); }

cudaError_t igc_launch_embed(const int32_t *ids, int lanes, const uint16_t *embed, int hidden, float embed_gain,
                             const uint16_t *ple_embed, int ple_vocab, int ple_width, float ple_gain,
                             float *x_out, float *seed_out, cudaStream_t st) {
  embed_kernel<<<lanes, 256, 0, st>>>(ids, lanes, embed, hidden, embed_gain, ple_embed, ple_vocab, ple_width,
                                      ple_gain, x_out, seed_out);
  return cudaGetLastError();
}

cudaError_t igc_launch_ple_finish(const float *raw, const float *seed, int lanes, int layers, int ple_dim,
                                  const float *w, float eps, float blend, float *out, cudaStream_t st) {
  ple_finish_kernel<<<lanes * layers, 256, 0, st>>>(raw, seed, lanes, layers, ple_dim, w, eps, blend, out);
  return cudaGetLastError();
}

cudaError_t igc_launch_attn_prep(float *qkv, int qkv_stride, int heads, int kv_heads, int hd, const float *q_norm,
                                 const float *k_norm, const float *cs, const float *sn, int owner, float eps,
                                 const int *d_p0, int lanes, float *kc, float *vc, cudaStream_t st) {
  attn_prep_kernel<<<lanes, 256, 0, st>>>(qkv, qkv_stride, heads, kv_heads, hd, q_norm, k_norm, cs, sn, owner,
                                          eps, d_p0, lanes, kc, vc);
  return cudaGetLastError();
}

size_t igc_attn_smem(int heads, int hd, int kv_w) { return sizeof(float) * attn_smem_floats(heads, hd, kv_w); }

cudaError_t igc_launch_attn(const float *qkv, int qkv_stride, int heads, int hd, const float *kc, const float *vc,
                            int kv_w, int group, int sliding, int span, const int *d_p0, int lanes, int n_chunks,
                            float *part_ml, float *part_acc, float *out, int out_stride, cudaStream_t st) {
  size_t smem = igc_attn_smem(heads, hd, kv_w);
  dim3 grid(n_chunks, (lanes + ATT_LANES - 1) / ATT_LANES);
  attn_chunk_kernel<<<grid, 256, smem, st>>>(qkv, qkv_stride, heads, hd, kc, vc, kv_w, group, sliding, span, d_p0,
                                             lanes, part_ml, part_acc);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  attn_combine_kernel<<<lanes * heads, 256, 0, st>>>(part_ml, part_acc, n_chunks, lanes, heads, hd, sliding, span,
                                                     d_p0, out, out_stride);
  return cudaGetLastError();
}

cudaError_t igc_launch_argmax(const float *part_val, const int *part_idx, int parts, int lanes, int32_t *top,
                              cudaStream_t st) {
  argmax_final_kernel<<<1, 32, 0, st>>>(part_val, part_idx, parts, lanes, top);
  return cudaGetLastError();
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
