// Split-KV int8 attention of the verify step's full-attention layers (the
// spk_pre / spk_a / spk_c set of the reference: engine/spk_preqh.cu,
// engine/spk_g4hm.cu, engine/skv_split.cu K2S).  24 query heads, 4 KV heads
// (6 query heads each), head dim 256, rotary on dims 0..63, int8 KV cache with
// one fp16 scale per 32 dims:
//   kv [8][ctx][256] bytes (q + 128; heads 0..3 K, 4..7 V), sc [8][ctx][8] fp16.
//
// attn_pre_kernel    one CTA per (head unit, token): q heads -> RMS norm (rounded to
//                    fp16) x weight, rotary, x 1/16 -> qw16; KV heads -> the same for
//                    k, then k and the raw v quantised into the cache at pos + t.
//                    The per-row sum of squares is reduced in the reference's order
//                    (xor butterfly per warp, then over the 8 warp sums), so qw16 and
//                    the cache bytes equal the reference kernel's.
// attn_split_kernel  one CTA per (KV head, key range): the range [pos + T) / P is
//                    walked in 64-key tiles; scores S^T = K . Q^T with the keys as the
//                    mma M dimension and the 6 T query rows of the head group as N
//                    (66 rows -> 9 n-blocks of 8, not 5 m-blocks of 16), online
//                    softmax per row (causal: row t sees keys <= pos + t), O^T += V^T
//                    . P^T with the 256 dims as M (one 16-dim block per warp).  K / V
//                    are dequantised to fp16(q * scale) in shared memory (XOR-swizzled
//                    16-byte chunks, ldmatrix), the next tile's bytes prefetched into
//                    registers while the current one is computed.  Writes (max, sum,
//                    unnormalised output) per row.
// attn_combine_kernel one CTA per (head, token): merges the P partials of its row,
//                    times sigmoid of the gate half of the head's q projection row,
//                    fp16 out.
#include "tlx_internal.h"

#include <cuda_fp16.h>

#include <algorithm>

namespace tlx {
namespace {

constexpr int kHeads = 24, kKvHeads = 4, kGroup = 6, kHd = 256;
constexpr int kQRow = 2 * kHd * kHeads;   // 12288: per head 256 q then 256 gate
constexpr int kKRow = kHd * kKvHeads;     // 1024
constexpr int kMaxRows = 16;              // verify rows T
constexpr int kMaxR = kGroup * kMaxRows;  // 96 query rows per KV head
constexpr int kMaxNB = kMaxR / 8;         // 12 n-blocks
constexpr int kTile = 64;                 // keys per tile
constexpr int kWarps = 16, kThreads = kWarps * 32;

// ---------------------------------------------------------------- pre kernel
__device__ __forceinline__ float block_sumsq(float v, float* red) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float ss = v * v;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  if (warp == 0 && lane < 8) {
    float w = red[lane];
    for (int o = 4; o > 0; o >>= 1) w += __shfl_xor_sync(0xffu, w, o);
    if (lane == 0) red[8] = w;
  }
  __syncthreads();
  const float s = red[8];
  __syncthreads();
  return s;
}

// fp16(v * rsqrt(mean + eps)) * w, then rotary on dims 0..63 (pairs d, d + 32)
__device__ __forceinline__ float norm_rope(float v, float w, float cs, float sn, float* red, float* xch) {
  const int d = threadIdx.x;
  const float r = rsqrtf(block_sumsq(v, red) / 256.f + 1e-6f);
  const float x = __half2float(__float2half(v * r)) * w;
  xch[d] = x;
  __syncthreads();
  const float o = d < 32 ? x * cs - xch[d + 32] * sn : d < 64 ? x * cs + xch[d - 32] * sn : x;
  __syncthreads();
  return o;
}

// per 32-dim group (one warp): scale fp16(max|x| / 127) or 1e-8, byte rint(x / scale) + 128
__device__ __forceinline__ void quant8(float x, uint8_t* row, __half* srow) {
  float m = fabsf(x);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const __half s = __float2half(m > 0.f ? m * (1.f / 127.f) : 1e-8f);
  const int q = __float2int_rn(fminf(fmaxf(x / __half2float(s), -127.f), 127.f));
  const int d = threadIdx.x;
  row[d] = static_cast<uint8_t>(q + 128);
  if ((d & 31) == 0) srow[d >> 5] = s;
}

__global__ void __launch_bounds__(256) attn_pre_kernel(const __half* __restrict__ qrow, const __half* __restrict__ krow,
                                                       const __half* __restrict__ vrow, const float* __restrict__ qnw,
                                                       const float* __restrict__ knw, const float* __restrict__ freqs,
                                                       const int32_t* __restrict__ pos_slot, int64_t ctx,
                                                       uint8_t* __restrict__ kv, __half* __restrict__ sc,
                                                       __half* __restrict__ qw16) {
  __shared__ float red[9];
  __shared__ float xch[256];
  const int u = blockIdx.x, t = blockIdx.y, d = threadIdx.x;
  const int pos = pos_slot[0];
  const float ang = d < 64 ? static_cast<float>(pos + t) * freqs[d & 31] : 0.f;
  const float cs = cosf(ang), sn = sinf(ang);
  if (u < kHeads) {
    const float q = __half2float(qrow[static_cast<int64_t>(t) * kQRow + u * 2 * kHd + d]);
    const float o = norm_rope(q, qnw[d], cs, sn, red, xch);
    qw16[(static_cast<int64_t>(t) * kHeads + u) * kHd + d] = __float2half(o * 0.0625f);
    return;
  }
  const int g = u - kHeads;
  const float k = __half2float(krow[static_cast<int64_t>(t) * kKRow + g * kHd + d]);
  const float kf = __half2float(__float2half(norm_rope(k, knw[d], cs, sn, red, xch)));
  const float vf = __half2float(vrow[static_cast<int64_t>(t) * kKRow + g * kHd + d]);
  const int64_t l = static_cast<int64_t>(pos) + t;
  if (l < 0 || l >= ctx) return;   // outside the cache: nothing is written
  quant8(kf, kv + (static_cast<int64_t>(g) * ctx + l) * kHd, sc + (static_cast<int64_t>(g) * ctx + l) * 8);
  quant8(vf, kv + (static_cast<int64_t>(kKvHeads + g) * ctx + l) * kHd,
         sc + (static_cast<int64_t>(kKvHeads + g) * ctx + l) * 8);
}

// ---------------------------------------------------------------- split kernel
// shared memory (bytes): K tile, V tile, Q rows (fp16, 32 chunks of 16 B per row,
// chunk index XOR (row & 7)); S (fp32 [96][64]); P (fp16 [96][64], 8 chunks per row,
// swizzled); per-row correction
constexpr uint32_t kOffK = 0;
constexpr uint32_t kOffV = kOffK + kTile * 512;
constexpr uint32_t kOffQ = kOffV + kTile * 512;
constexpr uint32_t kOffS = kOffQ + kMaxR * 512;
// score rows are kSStride floats apart: the fragment writes (rows 2q, keys g) and
// the softmax reads (8 rows per 16-byte phase) then fall on distinct banks
constexpr int kSStride = kTile + 4;
constexpr uint32_t kOffP = kOffS + kMaxR * kSStride * 4;
constexpr uint32_t kOffCor = kOffP + kMaxR * kTile * 2;
constexpr uint32_t kSplitSmem = kOffCor + kMaxR * 4;

__device__ __forceinline__ uint32_t sw32(int row, int chunk) {   // rows of 32 chunks
  return static_cast<uint32_t>(row * 512 + ((chunk ^ (row & 7)) << 4));
}
__device__ __forceinline__ uint32_t sw8(int row, int chunk) {    // rows of 8 chunks
  return static_cast<uint32_t>(row * 128 + ((chunk ^ (row & 7)) << 4));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];\n" : "=r"(r0), "=r"(r1) : "r"(addr));
}
__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// 16 int8 cache bytes (q + 128) and their fp16 scale -> 16 fp16 fp16(q * scale)
__device__ __forceinline__ void dq16(const uint4 b, __half s, uint4& lo, uint4& hi) {
  const __half2 s2 = __half2half2(s);
  const __half2 c1152 = __float2half2_rn(1152.f);
  const uint32_t w[4] = {b.x, b.y, b.z, b.w};
  uint32_t o[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t p0 = __byte_perm(w[i], 0x64646464u, 0x5140u);   // bytes 0, 1 -> 1024 + b
    const uint32_t p1 = __byte_perm(w[i], 0x64646464u, 0x7362u);   // bytes 2, 3
    const __half2 h0 = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&p0), c1152), s2);
    const __half2 h1 = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&p1), c1152), s2);
    o[2 * i] = *reinterpret_cast<const uint32_t*>(&h0);
    o[2 * i + 1] = *reinterpret_cast<const uint32_t*>(&h1);
  }
  lo = make_uint4(o[0], o[1], o[2], o[3]);
  hi = make_uint4(o[4], o[5], o[6], o[7]);
}

struct SplitArgs {
  const uint8_t* kv;
  const __half* sc;
  const __half* qw16;
  const int32_t* pos_slot;
  int64_t ctx;
  int T, parts;
  float* pm;   // [4][parts][96]
  float* ps;
  float* pa;   // [4][parts][96][256]
};

__global__ void __launch_bounds__(kThreads, 1) attn_split_kernel(const SplitArgs a) {
  extern __shared__ __align__(128) uint8_t sm[];
  const int g = blockIdx.y, part = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int T = a.T, R = kGroup * T, NB = (R + 7) >> 3;
  const int pos = a.pos_slot[0];
  const int64_t total = std::min<int64_t>(static_cast<int64_t>(pos) + T, a.ctx);   // keys that exist
  // this CTA's key range, in whole tiles
  const int64_t ntiles_all = total > 0 ? (total + kTile - 1) / kTile : 0;
  const int64_t t0 = ntiles_all * part / a.parts, t1 = ntiles_all * (part + 1) / a.parts;
  const uint32_t sbase = static_cast<uint32_t>(__cvta_generic_to_shared(sm));
  const uint8_t* Kc = a.kv + static_cast<int64_t>(g) * a.ctx * kHd;
  const uint8_t* Vc = a.kv + static_cast<int64_t>(kKvHeads + g) * a.ctx * kHd;
  const __half* Ks = a.sc + static_cast<int64_t>(g) * a.ctx * 8;
  const __half* Vs = a.sc + static_cast<int64_t>(kKvHeads + g) * a.ctx * 8;

  // stage Q rows r = hl * T + t (zero rows up to NB * 8)
  for (int i = tid; i < NB * 8 * 32; i += kThreads) {
    const int r = i >> 5, c = i & 31;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (r < R) {
      const int hl = r / T, t = r - hl * T;
      v = *reinterpret_cast<const uint4*>(a.qw16 + (static_cast<int64_t>(t) * kHeads + g * kGroup + hl) * kHd + c * 8);
    }
    *reinterpret_cast<uint4*>(sm + kOffQ + sw32(r, c)) = v;
  }

  // row owner state: 4 threads per row, lanes l, l ^ 8, l ^ 16, l ^ 24 of a warp
  // (8 rows per warp), keys osub * 4 + 16 j + 0..3
  const int orow = (tid & 7) + 8 * (tid >> 5), osub = (tid >> 3) & 3;
  const bool owner = orow < R;
  const int ot = owner ? orow % T : 0;
  float m_run = -1e30f, l_run = 0.f;
  // PV accumulators: warp = 16-dim block, all n-blocks (rows)
  float acc[kMaxNB][4];
#pragma unroll
  for (int nb = 0; nb < kMaxNB; ++nb)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[nb][i] = 0.f;

  // staging map: 2048 16-byte chunks per tile (K then V, key-major), 4 per thread
  uint4 pre[4];
  __half pres[4];
  auto fetch = [&](int64_t tile) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = tid + j * kThreads;          // 0..2047
      const int isv = c >> 10, key = (c >> 4) & 63, ch = c & 15;
      const int64_t l = tile * kTile + key;
      if (l < total) {
        const uint8_t* src = (isv ? Vc : Kc) + l * kHd + ch * 16;
        pre[j] = __ldg(reinterpret_cast<const uint4*>(src));
        pres[j] = (isv ? Vs : Ks)[l * 8 + (ch >> 1)];
      } else {
        pre[j] = make_uint4(0x80808080u, 0x80808080u, 0x80808080u, 0x80808080u);   // q = 0
        pres[j] = __float2half(0.f);
      }
    }
  };
  auto store = [&]() {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = tid + j * kThreads;
      const int isv = c >> 10, key = (c >> 4) & 63, ch = c & 15;
      uint4 lo, hi;
      dq16(pre[j], pres[j], lo, hi);
      uint8_t* base = sm + (isv ? kOffV : kOffK);
      *reinterpret_cast<uint4*>(base + sw32(key, 2 * ch)) = lo;
      *reinterpret_cast<uint4*>(base + sw32(key, 2 * ch + 1)) = hi;
    }
  };

  if (t0 < t1) fetch(t0);
  for (int64_t tile = t0; tile < t1; ++tile) {
    __syncthreads();   // the previous tile's K / V / P are consumed
    store();
    __syncthreads();
    if (tile + 1 < t1) fetch(tile + 1);   // in flight during this tile's math

    // ---- scores S^T[key][row] = K . Q^T: items (key block mb, row block nb) ----
    for (int it = warp; it < 4 * NB; it += kWarps) {
      const int mb = it & 3, nb = it >> 2;
      float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int ks = 0; ks < 16; ++ks) {
        uint32_t a0, a1, a2, a3, b0, b1;
        const int arow = mb * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        ldsm_x4(sbase + kOffK + sw32(arow, 2 * ks + (lane >> 4)), a0, a1, a2, a3);
        const int brow = nb * 8 + (lane & 7);
        ldsm_x2(sbase + kOffQ + sw32(brow, 2 * ks + ((lane >> 3) & 1)), b0, b1);
        mma_f16(c, a0, a1, a2, a3, b0, b1);
      }
      // c0 / c1: key mb*16 + g, rows nb*8 + 2q, +1; c2 / c3: key + 8
      float* S = reinterpret_cast<float*>(sm + kOffS);
      const int key = mb * 16 + (lane >> 2), row = nb * 8 + 2 * (lane & 3);
      S[row * kSStride + key] = c[0];
      S[(row + 1) * kSStride + key] = c[1];
      S[row * kSStride + key + 8] = c[2];
      S[(row + 1) * kSStride + key + 8] = c[3];
    }
    __syncthreads();

    // ---- online softmax per row (4 threads x 16 keys) ----
    if (orow < NB * 8) {
      const float* S = reinterpret_cast<const float*>(sm + kOffS);
      const int64_t lim = std::min<int64_t>(total, static_cast<int64_t>(pos) + ot + 1);   // keys < lim
      float s[16];
      float mx = -1e30f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int k0 = osub * 4 + 16 * j;
        const float4 v = *reinterpret_cast<const float4*>(S + orow * kSStride + k0);
        const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const bool ok = owner && tile * kTile + k0 + i < lim;
          s[4 * j + i] = ok ? vv[i] : -1e30f;
          mx = fmaxf(mx, s[4 * j + i]);
        }
      }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
      const float mn = fmaxf(m_run, mx);
      const float cor = __expf(m_run - mn);
      float sum = 0.f;
      uint32_t ph[8];
#pragma unroll
      for (int i = 0; i < 16; i += 2) {
        const float p0 = s[i] > -1e29f ? __expf(s[i] - mn) : 0.f;
        const float p1 = s[i + 1] > -1e29f ? __expf(s[i + 1] - mn) : 0.f;
        sum += p0 + p1;
        const __half2 h = __floats2half2_rn(p0, p1);
        ph[i >> 1] = *reinterpret_cast<const uint32_t*>(&h);
      }
      sum += __shfl_xor_sync(0xffffffffu, sum, 8);
      sum += __shfl_xor_sync(0xffffffffu, sum, 16);
      l_run = l_run * cor + sum;
      m_run = mn;
#pragma unroll
      for (int j = 0; j < 4; ++j)   // keys osub * 4 + 16 j .. + 3: half of chunk 2 j + osub / 2
        *reinterpret_cast<uint2*>(sm + kOffP + sw8(orow, 2 * j + (osub >> 1)) + (osub & 1) * 8) =
            make_uint2(ph[2 * j], ph[2 * j + 1]);
      if (osub == 0) reinterpret_cast<float*>(sm + kOffCor)[orow] = cor;
    }
    __syncthreads();

    // ---- O^T[dim][row] = cor * O^T + V^T . P^T: warp = dims warp*16 .. +15 ----
    {
      const float* cor = reinterpret_cast<const float*>(sm + kOffCor);
      uint32_t va[4][4];
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {   // 16-key steps; A = V^T via transposed loads
        const int key = kk * 16 + (lane & 7) + (lane >> 4) * 8;
        ldsm_x4_t(sbase + kOffV + sw32(key, warp * 2 + ((lane >> 3) & 1)), va[kk][0], va[kk][1], va[kk][2],
                  va[kk][3]);
      }
#pragma unroll
      for (int nb = 0; nb < kMaxNB; ++nb) {
        if (nb < NB) {
          const float c0 = cor[nb * 8 + 2 * (lane & 3)], c1 = cor[nb * 8 + 2 * (lane & 3) + 1];
          acc[nb][0] *= c0;
          acc[nb][1] *= c1;
          acc[nb][2] *= c0;
          acc[nb][3] *= c1;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            uint32_t b0, b1;
            ldsm_x2(sbase + kOffP + sw8(nb * 8 + (lane & 7), 2 * kk + ((lane >> 3) & 1)), b0, b1);
            mma_f16(acc[nb], va[kk][0], va[kk][1], va[kk][2], va[kk][3], b0, b1);
          }
        }
      }
    }
  }

  // ---- partials: (max, sum) per row, unnormalised output [row][256] ----
  const int64_t pb = (static_cast<int64_t>(g) * a.parts + part) * kMaxR;
  if (owner && osub == 0) {
    a.pm[pb + orow] = m_run;
    a.ps[pb + orow] = l_run;
  }
#pragma unroll
  for (int nb = 0; nb < kMaxNB; ++nb) {
    if (nb < NB) {
      const int row = nb * 8 + 2 * (lane & 3), dim = warp * 16 + (lane >> 2);
      if (row < R) {
        a.pa[(pb + row) * kHd + dim] = acc[nb][0];
        a.pa[(pb + row) * kHd + dim + 8] = acc[nb][2];
      }
      if (row + 1 < R) {
        a.pa[(pb + row + 1) * kHd + dim] = acc[nb][1];
        a.pa[(pb + row + 1) * kHd + dim + 8] = acc[nb][3];
      }
    }
  }
}

// ---------------------------------------------------------------- combine kernel
__global__ void __launch_bounds__(256) attn_combine_kernel(const float* __restrict__ pm, const float* __restrict__ ps,
                                                           const float* __restrict__ pa, int parts, int T,
                                                           const __half* __restrict__ qrow, __half* __restrict__ ao) {
  const int h = blockIdx.x, t = blockIdx.y, d = threadIdx.x;
  const int g = h / kGroup, hl = h - g * kGroup;
  const int r = hl * T + t;
  const int64_t base = static_cast<int64_t>(g) * parts * kMaxR + r;
  float M = -1e30f;
  for (int p = 0; p < parts; ++p) M = fmaxf(M, pm[base + static_cast<int64_t>(p) * kMaxR]);
  float out = 0.f, ssum = 0.f;
  for (int p = 0; p < parts; ++p) {
    const int64_t b = base + static_cast<int64_t>(p) * kMaxR;
    const float e = __expf(pm[b] - M);
    ssum += ps[b] * e;
    out += pa[b * kHd + d] * e;
  }
  out /= ssum;
  const float gate = __half2float(qrow[static_cast<int64_t>(t) * kQRow + h * 2 * kHd + kHd + d]);
  ao[static_cast<int64_t>(t) * (kHeads * kHd) + h * kHd + d] = __float2half(out / (1.f + __expf(-gate)));
}

int parts_for(int sms) { return std::max(1, sms / kKvHeads); }

int sm_count_dev() {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms > 0 ? sms : 148;
}

}  // namespace

size_t attn_workspace_bytes(int rows) {
  if (rows < 1 || rows > kMaxRows) return 0;
  const size_t parts = static_cast<size_t>(parts_for(sm_count_dev()));
  return kKvHeads * parts * kMaxR * (2 + kHd) * sizeof(float);
}

int run_attn_pre(const void* qrow, const void* krow, const void* vrow, const float* qnw, const float* knw,
                 const float* freqs, const int32_t* pos_slot, int rows, int64_t ctx, void* kv, void* sc, void* qw16,
                 cudaStream_t stream) {
  if (!qrow || !krow || !vrow || !qnw || !knw || !freqs || !pos_slot || !kv || !sc || !qw16) return TLX_ERR_NULL;
  if (rows < 1 || rows > kMaxRows || ctx < 1) return TLX_ERR_SHAPE;
  attn_pre_kernel<<<dim3(kHeads + kKvHeads, rows), 256, 0, stream>>>(
      static_cast<const __half*>(qrow), static_cast<const __half*>(krow), static_cast<const __half*>(vrow), qnw, knw,
      freqs, pos_slot, ctx, static_cast<uint8_t*>(kv), static_cast<__half*>(sc), static_cast<__half*>(qw16));
  return cudaGetLastError() == cudaSuccess ? TLX_OK : TLX_ERR_LAUNCH;
}

static int split_args(const void* kv, const void* sc, const void* qw16, const int32_t* pos_slot, int rows,
                      int64_t ctx, void* ws, size_t ws_bytes, SplitArgs& a) {
  if (!kv || !sc || !qw16 || !pos_slot || !ws) return TLX_ERR_NULL;
  if (rows < 1 || rows > kMaxRows || ctx < 1) return TLX_ERR_SHAPE;
  if (ws_bytes < attn_workspace_bytes(rows)) return TLX_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(kv) & 15) || (reinterpret_cast<uintptr_t>(qw16) & 15) ||
      (reinterpret_cast<uintptr_t>(ws) & 15))
    return TLX_ERR_ALIGN;
  const int parts = parts_for(sm_count_dev());
  a.kv = static_cast<const uint8_t*>(kv);
  a.sc = static_cast<const __half*>(sc);
  a.qw16 = static_cast<const __half*>(qw16);
  a.pos_slot = pos_slot;
  a.ctx = ctx;
  a.T = rows;
  a.parts = parts;
  float* f = static_cast<float*>(ws);
  a.pm = f;
  a.ps = f + static_cast<size_t>(kKvHeads) * parts * kMaxR;
  a.pa = f + static_cast<size_t>(2) * kKvHeads * parts * kMaxR;
  return TLX_OK;
}

int run_attn_split(const void* kv, const void* sc, const void* qw16, const int32_t* pos_slot, int rows, int64_t ctx,
                   void* ws, size_t ws_bytes, cudaStream_t stream) {
  SplitArgs a;
  const int rc = split_args(kv, sc, qw16, pos_slot, rows, ctx, ws, ws_bytes, a);
  if (rc) return rc;
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(attn_split_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kSplitSmem)) != cudaSuccess)
      return TLX_ERR_LAUNCH;
    configured = true;
  }
  attn_split_kernel<<<dim3(a.parts, kKvHeads), kThreads, kSplitSmem, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? TLX_OK : TLX_ERR_LAUNCH;
}

int run_attn_combine(const void* ws, size_t ws_bytes, const void* qrow, int rows, void* ao, cudaStream_t stream) {
  if (!ws || !qrow || !ao) return TLX_ERR_NULL;
  if (rows < 1 || rows > kMaxRows) return TLX_ERR_SHAPE;
  if (ws_bytes < attn_workspace_bytes(rows)) return TLX_ERR_WORKSPACE;
  const int parts = parts_for(sm_count_dev());
  const float* f = static_cast<const float*>(ws);
  attn_combine_kernel<<<dim3(kHeads, rows), 256, 0, stream>>>(
      f, f + static_cast<size_t>(kKvHeads) * parts * kMaxR, f + static_cast<size_t>(2) * kKvHeads * parts * kMaxR,
      parts, rows, static_cast<const __half*>(qrow), static_cast<__half*>(ao));
  return cudaGetLastError() == cudaSuccess ? TLX_OK : TLX_ERR_LAUNCH;
}

}  // namespace tlx

extern "C" {

size_t tlx_attn_workspace_bytes(int rows) { return tlx::attn_workspace_bytes(rows); }

int tlx_attn_pre(const void* qrow, const void* krow, const void* vrow, const float* qnw, const float* knw,
                 const float* freqs, const int32_t* pos_slot, int rows, int64_t ctx, void* kv, void* sc, void* qw16,
                 void* stream) {
  return tlx::run_attn_pre(qrow, krow, vrow, qnw, knw, freqs, pos_slot, rows, ctx, kv, sc, qw16,
                           static_cast<cudaStream_t>(stream));
}

int tlx_attn_split(const void* kv, const void* sc, const void* qw16, const int32_t* pos_slot, int rows, int64_t ctx,
                   void* ws, size_t ws_bytes, void* stream) {
  return tlx::run_attn_split(kv, sc, qw16, pos_slot, rows, ctx, ws, ws_bytes, static_cast<cudaStream_t>(stream));
}

int tlx_attn_combine(const void* ws, size_t ws_bytes, const void* qrow, int rows, void* ao, void* stream) {
  return tlx::run_attn_combine(ws, ws_bytes, qrow, rows, ao, static_cast<cudaStream_t>(stream));
}

int tlx_attn_decode(const void* kv, const void* sc, const void* qw16, const void* qrow, const int32_t* pos_slot,
                    int rows, int64_t ctx, void* ao, void* ws, size_t ws_bytes, void* stream) {
  if (!qrow || !ao) return TLX_ERR_NULL;
  const int rc = tlx::run_attn_split(kv, sc, qw16, pos_slot, rows, ctx, ws, ws_bytes, static_cast<cudaStream_t>(stream));
  if (rc) return rc;
  return tlx::run_attn_combine(ws, ws_bytes, qrow, rows, ao, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
