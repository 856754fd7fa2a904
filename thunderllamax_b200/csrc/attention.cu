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
// attn_tc_kernel     one CTA per (KV head, key range): the range of [0, pos + T) is
//                    walked in 64-key tiles on tcgen05 (see below), online softmax
//                    per query row (causal: row t sees keys <= pos + t); writes (max,
//                    sum, unnormalised output) per row.
// attn_combine_kernel one CTA per (head, token): merges the P partials of its row,
//                    times sigmoid of the gate half of the head's q projection row,
//                    fp16 out.
#include <cuda_fp16.h>

#include "common.cuh"
#include "tlx_internal.h"

#include <algorithm>

namespace tlx {
namespace {

constexpr int kHeads = 24, kKvHeads = 4, kGroup = 6, kHd = 256;
constexpr int kQRow = 2 * kHd * kHeads;   // 12288: per head 256 q then 256 gate
constexpr int kKRow = kHd * kKvHeads;     // 1024
constexpr int kMaxRows = 16;              // verify rows T
constexpr int kMaxR = kGroup * kMaxRows;  // 96 query rows per KV head
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

// ---------------------------------------------------------------- tcgen05 split kernel
// One CTA (16 warps) per (KV head, key range), one per SM.  The scores S = Q . K^T
// of the 6 T query rows (M = 128 TMEM lanes, 66 used for T = 11) against a 64-key
// tile (N = 64, K = 256) and the output O += P . V (N = 256 dims, K = 64 keys) run
// as tcgen05 MMAs with fp32 accumulators in tensor memory: S double-buffered in
// columns 0..127, O in columns 128..383.  Operands are fp16 in shared memory,
// K-major with the 128-byte swizzle: Q [128 rows][256 dims] staged once, K [64
// keys][256 dims] and V^T [256 dims][64 keys] double-buffered, P [128 rows][64 keys].
//   warp 0 (one thread)   issues the MMAs: S(i+1) ahead of O += P(i) V(i)
//   warps 4..7            softmax: thread = query row = TMEM lane; the row's max and
//                         sum stay in the thread.  The reference max moves only when
//                         a tile's max exceeds it by more than 8 (e^8 keeps P in fp16
//                         range), and only then is the row of O rescaled in TMEM.
//   warps 8..15           producers: int8 K / V -> fp16(q * scale) into the next
//                         buffer (V transposed through registers), the tile after
//                         next prefetched into registers.
// Every wait is bounded; on a timeout the CTA raises the error word, the MMA thread
// drains every issued MMA and TMEM is freed before exit.
constexpr int kTcTile = 64;
constexpr int kTcRows = 128;
constexpr uint32_t kKAtom = kTcTile * 128;            // 8 KB: 64 keys x 64 dims
constexpr int kKvBufs = 3;                            // K / V tiles in flight
constexpr uint32_t kOffTK = 0;                        // kKvBufs buffers x 4 atoms
constexpr uint32_t kOffTV = kOffTK + kKvBufs * 4 * kKAtom;  // kKvBufs buffers x [256][64] (32 KB)
constexpr uint32_t kOffTP = kOffTV + kKvBufs * 256 * 128;   // [128][64] (16 KB)
constexpr uint32_t kOffTBar = kOffTP + kTcRows * 128;
constexpr uint32_t kTcSmem = kOffTBar + 128 + 1024;   // barriers, TMEM holder, abort flag; 1 KB alignment slack
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0, kColO = 128, kColQ = 384;   // Q: 256 fp16 per lane = 128 columns
// instruction descriptors (kind::f16: fp16 A / B K-major, fp32 D, M x N)
constexpr uint32_t kIdescQK = (1u << 4) | (static_cast<uint32_t>(kTcTile >> 3) << 17) | (static_cast<uint32_t>(kTcRows >> 4) << 24);
constexpr uint32_t kIdescPV = (1u << 4) | (static_cast<uint32_t>(256 >> 3) << 17) | (static_cast<uint32_t>(kTcRows >> 4) << 24);
constexpr float kLazy = 8.f;   // rescale O only when the row max grows by more than this

__device__ __forceinline__ uint32_t sw128(int r, int c) {   // (row, 16-byte chunk) in a K-major 128-B swizzled atom
  return static_cast<uint32_t>((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);   // start address
  d |= static_cast<uint64_t>(1u) << 16;                  // leading byte offset (unused: swizzled K-major)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;          // stride byte offset: next 8-row group
  d |= static_cast<uint64_t>(1u) << 46;                  // descriptor version
  d |= static_cast<uint64_t>(2u) << 61;                  // 128-byte swizzle
  return d;
}
__device__ __forceinline__ void tc_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(dst)), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tc_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
// D[tmem] (+)= A[tmem] . B[smem desc]^T (A: one row per lane, k packed two fp16 per column)
__device__ __forceinline__ void tc_mma_ts(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tc_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }
// 2^x on the SFU (ex2.approx: relative error ~2^-22; 2^-inf = 0)
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kMbarPollLimit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

struct TcArgs {
  const uint8_t* kv;
  const __half* sc;
  const __half* qw16;
  const int32_t* pos_slot;
  int64_t ctx;
  int T, parts;
  uint32_t* err;
  float* pm;   // [4][parts][96]
  float* ps;
  float* pa;   // [4][parts][96][256]
};

// fp16 pair (k, k + 1) of 8 dequantised values: bytes (q + 128) of one 8-byte word
__device__ __forceinline__ void dq8(uint2 w, __half2 s2, uint32_t (&o)[4]) {
  const __half2 c1152 = __float2half2_rn(1152.f);
  const uint32_t in[2] = {w.x, w.y};
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const uint32_t p0 = __byte_perm(in[i], 0x64646464u, 0x5140u);
    const uint32_t p1 = __byte_perm(in[i], 0x64646464u, 0x7362u);
    const __half2 h0 = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&p0), c1152), s2);
    const __half2 h1 = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&p1), c1152), s2);
    o[2 * i] = *reinterpret_cast<const uint32_t*>(&h0);
    o[2 * i + 1] = *reinterpret_cast<const uint32_t*>(&h1);
  }
}

__global__ void __launch_bounds__(kThreads, 1) attn_tc_kernel(const TcArgs a) {
  extern __shared__ __align__(1024) uint8_t smraw[];
  uint8_t* sm = smraw + ((1024u - (smem_u32(smraw) & 1023u)) & 1023u);
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + kOffTBar);
  uint64_t* kv_full = bar;                   // [kKvBufs] producers -> MMA
  uint64_t* kv_empty = bar + kKvBufs;        // [kKvBufs] PV commit -> producers
  uint64_t* s_full = bar + 2 * kKvBufs;      // [2] QK commit -> softmax
  uint64_t* s_free = s_full + 2;             // [2] softmax read S -> MMA
  uint64_t* p_full = s_full + 4;             // softmax wrote P -> MMA
  uint64_t* pv_done = s_full + 5;            // PV commit -> softmax
  uint64_t* done = s_full + 6;               // final drain
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(s_full + 7);
  static_assert((2 * kKvBufs + 7) * 8 + 8 <= 128, "barrier area");
  volatile uint32_t* abort_flag = tmem_holder + 1;

  const int g = blockIdx.y, part = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int T = a.T, R = kGroup * T;
  const int pos = a.pos_slot[0];
  const int64_t total = std::min<int64_t>(static_cast<int64_t>(pos) + T, a.ctx);
  const int64_t ntiles_all = total > 0 ? (total + kTcTile - 1) / kTcTile : 0;
  const int64_t t0 = ntiles_all * part / a.parts, t1 = ntiles_all * (part + 1) / a.parts;
  const int n = static_cast<int>(t1 - t0);
  const uint32_t sbase = smem_u32(sm);
  const uint8_t* Kc = a.kv + static_cast<int64_t>(g) * a.ctx * kHd;
  const uint8_t* Vc = a.kv + static_cast<int64_t>(kKvHeads + g) * a.ctx * kHd;
  const __half* Ks = a.sc + static_cast<int64_t>(g) * a.ctx * 8;
  const __half* Vs = a.sc + static_cast<int64_t>(kKvHeads + g) * a.ctx * 8;
  const int64_t pb = (static_cast<int64_t>(g) * a.parts + part) * kMaxR;

  if (tid == 0) {
    for (int i = 0; i < kKvBufs; ++i) {
      mbar_init(&kv_full[i], 8);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);
    }
    mbar_init(p_full, 4);
    mbar_init(pv_done, 1);
    mbar_init(done, 1);
    *abort_flag = 0u;
    mbar_fence_init();
  }
  if (warp == 0) tc_alloc(tmem_holder, kTmemCols);
  tc_before();
  __syncthreads();
  tc_after();
  const uint32_t tmem = *tmem_holder;
  if (warp >= 4 && warp < 8) {
    // Q into TMEM columns kColQ..: lane = query row r = hl * T + t (zero beyond R)
    const int r = (warp - 4) * 32 + lane;
    const uint4* src = nullptr;
    if (r < R) {
      const int hl = r / T, t = r - hl * T;
      src = reinterpret_cast<const uint4*>(a.qw16 + (static_cast<int64_t>(t) * kHeads + g * kGroup + hl) * kHd);
    }
#pragma unroll 1
    for (int c = 0; c < 8; ++c) {   // 32 dims = 16 columns per store
      uint32_t w[16];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 v = src ? src[c * 4 + j] : make_uint4(0u, 0u, 0u, 0u);
        w[4 * j] = v.x;
        w[4 * j + 1] = v.y;
        w[4 * j + 2] = v.z;
        w[4 * j + 3] = v.w;
      }
      tc_st16(tmem + (static_cast<uint32_t>((warp - 4) * 32) << 16) + kColQ + c * 16, w);
    }
    tc_wait_st();
  }
  tc_before();
  __syncthreads();
  tc_after();
  auto fail = [&]() {
    atomicOr(a.err, 1u);
    *abort_flag = 1u;
  };

  if (warp == 0) {
    // ------------------------------------------------------------- MMA issuer
    if (lane == 0 && n > 0) {
      auto issue_qk = [&](int j) -> bool {
        const int b = j & 1, kb_i = j % kKvBufs;
        const uint32_t u = static_cast<uint32_t>(j >> 1), ku = static_cast<uint32_t>(j / kKvBufs);
        if (!tc_wait(&kv_full[kb_i], ku & 1) || !tc_wait(&s_free[b], (u & 1) ^ 1)) return false;
        tc_after();
        const uint32_t kb = sbase + kOffTK + kb_i * 4 * kKAtom;
#pragma unroll
        for (int s = 0; s < 16; ++s) {
          const uint64_t bd = sw128_desc(kb + (s >> 2) * kKAtom + (s & 3) * 32);
          tc_mma_ts(tmem + kColS + b * kTcTile, tmem + kColQ + s * 8, bd, kIdescQK, s > 0 ? 1u : 0u);
        }
        tc_commit(&s_full[b]);
        return true;
      };
      bool ok = issue_qk(0);
      for (int i = 0; i < n && ok && !*abort_flag; ++i) {
        if (i + 1 < n && !(ok = issue_qk(i + 1))) break;
        if (!(ok = tc_wait(p_full, i & 1))) break;
        tc_after();
        const int b = i % kKvBufs;
        const uint32_t vb = sbase + kOffTV + b * 256 * 128;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tc_mma(tmem + kColO, sw128_desc(sbase + kOffTP + kk * 32), sw128_desc(vb + kk * 32), kIdescPV,
                 (i > 0 || kk > 0) ? 1u : 0u);
        tc_commit(pv_done);
        tc_commit(&kv_empty[b]);
      }
      if (!ok) fail();
      tc_commit(done);   // every issued MMA has completed before TMEM is released
      if (!tc_wait(done, 0)) fail();
    }
  } else if (warp >= 4 && warp < 8) {
    // --------------------------------------------------------------- softmax
    const int qd = warp - 4, row = qd * 32 + lane;
    const uint32_t lanebase = static_cast<uint32_t>(qd * 32) << 16;
    const bool valid = row < R;
    const int t = valid ? row % T : 0;
    const int64_t lim = std::min<int64_t>(total, static_cast<int64_t>(pos) + t + 1);   // keys < lim
    float m_ref = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int i = 0; i < n && ok && !*abort_flag; ++i) {
      const int b = i & 1;
      const uint32_t u = static_cast<uint32_t>(i >> 1);
      if (!(ok = tc_wait(&s_full[b], u & 1))) break;
      tc_after();
      // the tile's 64 scores of this row: four TMEM loads, one wait
      uint32_t r0[16], r1[16], r2[16], r3[16];
      tc_ld16(tmem + lanebase + kColS + b * kTcTile + 0, r0);
      tc_ld16(tmem + lanebase + kColS + b * kTcTile + 16, r1);
      tc_ld16(tmem + lanebase + kColS + b * kTcTile + 32, r2);
      tc_ld16(tmem + lanebase + kColS + b * kTcTile + 48, r3);
      tc_wait_ld();
      tc_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[b]);
      float s[kTcTile];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        s[j] = __uint_as_float(r0[j]);
        s[16 + j] = __uint_as_float(r1[j]);
        s[32 + j] = __uint_as_float(r2[j]);
        s[48 + j] = __uint_as_float(r3[j]);
      }
      // keys k0 + j exist for this row while j < rem (causal limit and cache end)
      const int64_t k0 = (t0 + i) * kTcTile;
      const int rem = valid ? static_cast<int>(std::max<int64_t>(0, std::min<int64_t>(kTcTile, lim - k0))) : 0;
      if (rem < kTcTile) {
#pragma unroll
        for (int j = 0; j < kTcTile; ++j)
          if (j >= rem) s[j] = -INFINITY;
      }
      float mx[8];   // 8 independent max chains, then a tree
#pragma unroll
      for (int j = 0; j < 8; ++j) mx[j] = s[j];
#pragma unroll
      for (int j = 8; j < kTcTile; ++j) mx[j & 7] = fmaxf(mx[j & 7], s[j]);
      const float mt = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])), fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
      // O (rows of earlier tiles) and P are free once the previous PV completed
      if (i > 0 && !(ok = tc_wait(pv_done, (i - 1) & 1))) break;
      tc_after();
      if (mt > m_ref + kLazy || (m_ref == -INFINITY && mt > -INFINITY)) {
        if (m_ref != -INFINITY && i > 0) {   // rescale this row of O and the running sum
          const float cor = __expf(m_ref - mt);
          l_run *= cor;
#pragma unroll 1
          for (int c = 0; c < 16; ++c) {
            uint32_t r[16];
            tc_ld16(tmem + lanebase + kColO + c * 16, r);
            tc_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j) r[j] = __float_as_uint(__uint_as_float(r[j]) * cor);
            tc_st16(tmem + lanebase + kColO + c * 16, r);
          }
          tc_wait_st();
        }
        m_ref = mt;
      }
      // p = e^(s - m) = 2^(s log2 e - m log2 e): one fma and one ex2 per key; a
      // missing key (-inf) gives 2^-inf = 0 (and a row without keys so far has all
      // scores -inf, so its offset is taken as 0)
      const float kLog2e = 1.4426950408889634f;
      const float off = m_ref == -INFINITY ? 0.f : -m_ref * kLog2e;
      float sums[4] = {0.f, 0.f, 0.f, 0.f};   // independent partial sums
#pragma unroll
      for (int c = 0; c < 8; ++c) {   // keys 8c .. 8c + 7 -> one 16-byte chunk of P
        uint32_t w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float p0 = ex2_approx(fmaf(s[8 * c + 2 * j], kLog2e, off));
          const float p1 = ex2_approx(fmaf(s[8 * c + 2 * j + 1], kLog2e, off));
          sums[j] += p0 + p1;
          const __half2 h = __floats2half2_rn(p0, p1);
          w[j] = *reinterpret_cast<const uint32_t*>(&h);
        }
        *reinterpret_cast<uint4*>(sm + kOffTP + sw128(row, c)) = make_uint4(w[0], w[1], w[2], w[3]);
      }
      l_run += (sums[0] + sums[1]) + (sums[2] + sums[3]);
      fence_proxy_async_smem();
      tc_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    if (!ok) fail();
    // partials: (max, sum) and the unnormalised output row
    if (n > 0 && ok && !*abort_flag && tc_wait(pv_done, (n - 1) & 1)) {
      tc_after();
#pragma unroll 1
      for (int c = 0; c < 16; ++c) {
        uint32_t r[16];
        tc_ld16(tmem + lanebase + kColO + c * 16, r);
        tc_wait_ld();
        if (valid) {
          float4* dst = reinterpret_cast<float4*>(a.pa + (pb + row) * kHd + c * 16);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            dst[j] = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                 __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
        }
      }
      if (valid) {
        a.pm[pb + row] = m_ref == -INFINITY ? -1e30f : m_ref;
        a.ps[pb + row] = l_run;
      }
    } else if (valid) {
      if (n > 0 && !*abort_flag) fail();
      a.pm[pb + row] = -1e30f;   // no key in this range (or an aborted CTA): contributes nothing
      a.ps[pb + row] = 0.f;
      for (int c = 0; c < kHd; c += 4) *reinterpret_cast<float4*>(a.pa + (pb + row) * kHd + c) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    tc_before();
  } else if (warp >= 8) {
    // -------------------------------------------------------------- producers
    const int ptid = tid - 256;
    const int vk = ptid & 7, vd = ptid >> 3;   // V unit: keys 8 vk .. +7, dims 8 vd .. +7
    uint4 kq[4];
    __half ks[4];
    uint2 vq[8];
    __half vsc[8];
    auto fetch = [&](int i) {
      const int64_t kbase = (t0 + i) * kTcTile;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = ptid + j * 256, key = c >> 4, ch = c & 15;
        const int64_t l = kbase + key;
        if (l < total) {
          kq[j] = __ldg(reinterpret_cast<const uint4*>(Kc + l * kHd + ch * 16));
          ks[j] = Ks[l * 8 + (ch >> 1)];
        } else {
          kq[j] = make_uint4(0x80808080u, 0x80808080u, 0x80808080u, 0x80808080u);
          ks[j] = __float2half(0.f);
        }
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int64_t l = kbase + vk * 8 + k;
        if (l < total) {
          vq[k] = __ldg(reinterpret_cast<const uint2*>(Vc + l * kHd + vd * 8));
          vsc[k] = Vs[l * 8 + (vd >> 2)];
        } else {
          vq[k] = make_uint2(0x80808080u, 0x80808080u);
          vsc[k] = __float2half(0.f);
        }
      }
    };
    bool ok = true;
    if (n > 0) fetch(0);
    for (int i = 0; i < n && ok && !*abort_flag; ++i) {
      const int b = i % kKvBufs;
      const uint32_t u = static_cast<uint32_t>(i / kKvBufs);
      uint4 kq_c[4];
      __half ks_c[4];
      uint2 vq_c[8];
      __half vsc_c[8];
#pragma unroll
      for (int j = 0; j < 4; ++j) { kq_c[j] = kq[j]; ks_c[j] = ks[j]; }
#pragma unroll
      for (int k = 0; k < 8; ++k) { vq_c[k] = vq[k]; vsc_c[k] = vsc[k]; }
      if (i + 1 < n) fetch(i + 1);   // in flight while this tile is written
      if (!(ok = tc_wait(&kv_empty[b], (u & 1) ^ 1))) break;
      uint8_t* kb = sm + kOffTK + b * 4 * kKAtom;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = ptid + j * 256, key = c >> 4, ch = c & 15;
        const __half2 s2 = __half2half2(ks_c[j]);
        uint32_t lo[4], hi[4];
        dq8(make_uint2(kq_c[j].x, kq_c[j].y), s2, lo);
        dq8(make_uint2(kq_c[j].z, kq_c[j].w), s2, hi);
        uint8_t* atom = kb + (ch >> 2) * kKAtom;   // dims 16 ch .. + 15 lie in atom ch / 4
        *reinterpret_cast<uint4*>(atom + sw128(key, (ch & 3) * 2)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        *reinterpret_cast<uint4*>(atom + sw128(key, (ch & 3) * 2 + 1)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
      }
      // V unit: 8 keys x 8 dims, transposed to V^T rows (one 16-byte chunk of 8 keys per dim)
      uint32_t vv[8][4];
#pragma unroll
      for (int k = 0; k < 8; ++k) dq8(vq_c[k], __half2half2(vsc_c[k]), vv[k]);
      uint8_t* vbuf = sm + kOffTV + b * 256 * 128;
#pragma unroll
      for (int d = 0; d < 8; ++d) {
        uint32_t w[4];
#pragma unroll
        for (int m = 0; m < 4; ++m)   // keys 2m, 2m + 1 of dim d
          w[m] = __byte_perm(vv[2 * m][d >> 1], vv[2 * m + 1][d >> 1], (d & 1) ? 0x7632u : 0x5410u);
        *reinterpret_cast<uint4*>(vbuf + sw128(vd * 8 + d, vk)) = make_uint4(w[0], w[1], w[2], w[3]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&kv_full[b]);
    }
    if (!ok) fail();
  }

  tc_before();
  __syncthreads();
  if (warp == 0) {
    tc_after();
    tc_dealloc(tmem, kTmemCols);
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
constexpr size_t kAttnErrBytes = 256;   // the workspace starts with the device error word

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
  return kAttnErrBytes + kKvHeads * parts * kMaxR * (2 + kHd) * sizeof(float);
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
                      int64_t ctx, void* ws, size_t ws_bytes, TcArgs& a) {
  if (!kv || !sc || !qw16 || !pos_slot || !ws) return TLX_ERR_NULL;
  if (rows < 1 || rows > kMaxRows || ctx < 1) return TLX_ERR_SHAPE;
  if (ws_bytes < attn_workspace_bytes(rows)) return TLX_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(kv) & 15) || (reinterpret_cast<uintptr_t>(qw16) & 15) ||
      (reinterpret_cast<uintptr_t>(ws) & 255))
    return TLX_ERR_ALIGN;
  const int parts = parts_for(sm_count_dev());
  a.kv = static_cast<const uint8_t*>(kv);
  a.sc = static_cast<const __half*>(sc);
  a.qw16 = static_cast<const __half*>(qw16);
  a.pos_slot = pos_slot;
  a.ctx = ctx;
  a.T = rows;
  a.parts = parts;
  a.err = static_cast<uint32_t*>(ws);
  float* f = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + kAttnErrBytes);
  a.pm = f;
  a.ps = f + static_cast<size_t>(kKvHeads) * parts * kMaxR;
  a.pa = f + static_cast<size_t>(2) * kKvHeads * parts * kMaxR;
  return TLX_OK;
}

int run_attn_split(const void* kv, const void* sc, const void* qw16, const int32_t* pos_slot, int rows, int64_t ctx,
                   void* ws, size_t ws_bytes, cudaStream_t stream) {
  TcArgs a;
  const int rc = split_args(kv, sc, qw16, pos_slot, rows, ctx, ws, ws_bytes, a);
  if (rc) return rc;
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kTcSmem)) != cudaSuccess)
      return TLX_ERR_LAUNCH;
    configured = true;
  }
  attn_tc_kernel<<<dim3(a.parts, kKvHeads), kThreads, kTcSmem, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? TLX_OK : TLX_ERR_LAUNCH;
}

int run_attn_combine(const void* ws, size_t ws_bytes, const void* qrow, int rows, void* ao, cudaStream_t stream) {
  if (!ws || !qrow || !ao) return TLX_ERR_NULL;
  if (rows < 1 || rows > kMaxRows) return TLX_ERR_SHAPE;
  if (ws_bytes < attn_workspace_bytes(rows)) return TLX_ERR_WORKSPACE;
  const int parts = parts_for(sm_count_dev());
  const float* f = reinterpret_cast<const float*>(static_cast<const uint8_t*>(ws) + kAttnErrBytes);
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
