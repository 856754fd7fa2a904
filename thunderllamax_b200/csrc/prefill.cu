// Prefill-sized FFN contraction (many tokens) on the 5th-generation tensor cores.
//
//   act[t][r] = silu(Wg x_t)[r] * (Wu x_t)[r]   IQ3_XXS gate and up, fp32 act
//   y[t][r]   = (W x_t)[r]                      Q6_K (the down projection), fp32 y
//
// The GEMM is computed transposed, D[row][token] = W . X^T, so the dequantised
// weights are the A operand (M = 128 rows per tile) and the tokens the B operand
// (N = 256 per tile): one dequantised weight tile feeds 256 tokens.  Per CTA
// (persistent, one per SM, tiles in row-major order so the CTAs working on one
// weight tile at a time share it through L2):
//
//   warp 0       TMA-loads the token tile (fp16, 128-byte swizzle) of every 64-k step;
//   warps 8..15  dequantise each 64-k step to fp16 (the decode of the matvec kernels:
//                exact integer part times the block scale, one fp16 rounding per
//                weight) and write it in the UMMA K-major 128-byte-swizzle layout;
//                each thread reads its decode lane's bytes of the packed chunk from
//                global memory one step ahead, so no staging buffer is needed;
//   warp 1       one thread issues tcgen05.mma (kind::f16, fp32 accumulators in
//                TMEM: gate at columns 0..255, up at 256..511) and commits each
//                stage back to the producers;
//   warps 4..7   read the accumulators (tcgen05.ld, one 32-lane quarter each),
//                apply silu(g) * u or store y.
//
// Every wait is bounded: on timeout a thread raises ERR_MBAR_TIMEOUT, the CTA
// abandons its remaining tiles, waits for its issued tensor-core work and frees
// its TMEM.  No cluster multicast.  Reference: the prefill GEMM pool of
// engine/pf_gemm3.cu:4-26, :219 and engine/pf_gemm3m.cu:184-229 (IQ3 dequant to
// fp16 shared memory, mma.sync m16n8k16, SiLU epilogue).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <type_traits>

#include "common.cuh"
#include "formats.cuh"
#include "tlx_internal.h"

namespace tlx {
namespace {

constexpr int kPfRows = 128;   // weight rows per tile (UMMA M)
constexpr int kPfTok = 256;    // tokens per tile (UMMA N)
constexpr int kKStep = 64;       // k per pipeline stage (one 128-byte swizzle atom)
constexpr int kWarps = 16;
constexpr int kDequantWarp0 = 8;  // warps 8..15
constexpr int kEpiWarp0 = 4;      // warps 4..7
constexpr uint32_t kPollLimit = kMbarPollLimit;

// ---------------------------------------------------------------- tcgen05 / TMA
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(dst)), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }

// D[tmem] (+)= A[smem desc] . B[smem desc]^T, kind::f16, fp32 accumulate
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n"
      " setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// arrive on `bar` once every tcgen05.mma issued so far by this thread has completed
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }

// 2-D tiled TMA load (no multicast) completing on an mbarrier
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// UMMA shared-memory descriptor: K-major, 128-byte swizzle, 8-row groups 1024 B apart
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);  // start address
  d |= static_cast<uint64_t>(1u) << 16;                // leading byte offset (unused for swizzled K-major)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;        // stride byte offset: next 8-row group
  d |= static_cast<uint64_t>(1u) << 46;                // descriptor version (Blackwell)
  d |= static_cast<uint64_t>(2u) << 61;                // layout: 128-byte swizzle
  return d;
}
// instruction descriptor, kind::f16: fp16 A and B (K-major), fp32 D, M x N
constexpr uint32_t kIdesc = (1u << 4) | (static_cast<uint32_t>(kPfTok >> 3) << 17) |
                            (static_cast<uint32_t>(kPfRows >> 4) << 24);

// byte offset of (row r, 16-byte chunk c) inside a K-major 128-byte-swizzled tile
__device__ __forceinline__ uint32_t sw128_off(int r, int c) {
  return static_cast<uint32_t>((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

__device__ __forceinline__ bool wait_bounded(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kPollLimit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}
// for long waits (the epilogue waits a whole tile): back off between polls so the
// waiting warps leave the issue slots to the dequantising warps (bounded: ~seconds)
__device__ __forceinline__ bool wait_bounded_sleepy(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < (kPollLimit >> 4); ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    __nanosleep(512);
  }
  return false;
}

// The part of one decode lane's bytes of a packed chunk (k in [64q, 64q + 64) of
// the block, rows g and g+8) that one dequantising thread needs, read from global
// memory two steps ahead of use.
//   IQ3_XXS, part p of 2: scale group p (mma steps 8p .. 8p+7)
//   Q6_K,    part j of 4: sub-block j (mma steps 4j .. 4j+3, groups 2j and 2j+1)
struct Iq3Part {
  uint2 q0, q1;      // grid indices of group p, row g / row g+8
  uint32_t sw0, sw1; // scale/sign word of group p, row g / row g+8
  uint32_t d;        // fp16 d of row g (lo) and g+8 (hi)
};
struct Q6Part {
  uint4 ua, ub;      // the lane's 16-byte units holding words 6j .. 6j+5
  uint32_t sc;       // biased sub-scales of sub-block j, row g (byte 0) / g+8 (byte 1)
  uint32_t d;
};
template <int QT>
using PartT = typename std::conditional<QT == QT_IQ3_XXS, Iq3Part, Q6Part>::type;

__device__ __forceinline__ void load_part(const uint8_t* ch, int vlane, int part, Iq3Part& r) {
  r.q0 = __ldg(reinterpret_cast<const uint2*>(ch + vlane * 16 + 8 * part));
  r.q1 = __ldg(reinterpret_cast<const uint2*>(ch + 512 + vlane * 16 + 8 * part));
  r.sw0 = __ldg(reinterpret_cast<const uint32_t*>(ch + 1024 + vlane * 16 + 4 * part));
  r.sw1 = __ldg(reinterpret_cast<const uint32_t*>(ch + 1024 + vlane * 16 + 8 + 4 * part));
  r.d = __ldg(reinterpret_cast<const uint32_t*>(ch + 1536 + (vlane >> 2) * 4));
}
__device__ __forceinline__ void load_part(const uint8_t* ch, int vlane, int part, Q6Part& r) {
  const int ua = (3 * part) >> 1;  // 6j / 4
  r.ua = __ldg(reinterpret_cast<const uint4*>(ch + (ua * 32 + vlane) * 16));
  r.ub = __ldg(reinterpret_cast<const uint4*>(ch + ((ua + 1) * 32 + vlane) * 16));
  r.sc = __ldg(reinterpret_cast<const uint16_t*>(ch + 3072 + vlane * 8 + 2 * part));
  r.d = __ldg(reinterpret_cast<const uint32_t*>(ch + 3328 + (vlane >> 2) * 4));
}

// rows r0, r1 of the swizzled A tile, 16-byte chunk c: 8 consecutive k per row
__device__ __forceinline__ void store_rows(uint8_t* adst, int r0, int r1, int c, const uint32_t (&a)[4],
                                           const uint32_t (&b)[4], uint32_t s0, uint32_t s1) {
  *reinterpret_cast<uint4*>(adst + sw128_off(r0, c)) =
      make_uint4(hmul2_u(a[0], s0), hmul2_u(a[2], s0), hmul2_u(b[0], s0), hmul2_u(b[2], s0));
  *reinterpret_cast<uint4*>(adst + sw128_off(r1, c)) =
      make_uint4(hmul2_u(a[1], s1), hmul2_u(a[3], s1), hmul2_u(b[1], s1), hmul2_u(b[3], s1));
}

// IQ3_XXS, group p: mma steps 8p .. 8p+7 (the decode of iq3_mma restricted to one group)
__device__ __forceinline__ void dequant_iq3_part(const Iq3Part& r, int part, const uint8_t* grid_lane, uint8_t* adst,
                                                 int r0, int r1, uint32_t magic) {
  uint32_t sg[2], m2[2];
  iq3_word(r.sw0, magic, sg[0], m2[0]);
  iq3_word(r.sw1, magic, sg[1], m2[1]);
  const __half2 dh = *reinterpret_cast<const __half2*>(&r.d);
  const float2 df = __half22float2(dh);
  const uint32_t s0 = h2_bits(__float2half2_rn(df.x * 0.25f)), s1 = h2_bits(__float2half2_rn(df.y * 0.25f));
  auto decode = [&](int ml, uint32_t (&a)[4]) {
    const int l = (ml >> 1) & 3, e = ml & 1;
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      const uint2 q = rr == 0 ? r.q0 : r.q1;
      const uint32_t word = ml < 4 ? q.x : q.y;
      const uint2 G = *reinterpret_cast<const uint2*>(grid_entry(grid_lane, word, ml & 3));
      a[rr] = hmul2_u(G.x, m2[rr]) ^ pair_signs(sg[rr], l, 2 * e);
      a[rr + 2] = hmul2_u(G.y, m2[rr]) ^ pair_signs(sg[rr], l, 2 * e + 1);
    }
  };
#pragma unroll
  for (int ml = 0; ml < 8; ml += 2) {
    uint32_t a[4], b[4];
    decode(ml, a);
    decode(ml + 1, b);
    store_rows(adst, r0, r1, 4 * part + (ml >> 1), a, b, s0, s1);
  }
}

// Q6_K, sub-block j: groups 2j and 2j+1 (q6_group restricted to one sub-block)
__device__ __forceinline__ void dequant_q6_part(const Q6Part& r, int part, uint8_t* adst, int r0, int r1,
                                                uint32_t magic) {
  uint32_t w[6];
  if (part & 1) {
    w[0] = r.ua.z; w[1] = r.ua.w; w[2] = r.ub.x; w[3] = r.ub.y; w[4] = r.ub.z; w[5] = r.ub.w;
  } else {
    w[0] = r.ua.x; w[1] = r.ua.y; w[2] = r.ua.z; w[3] = r.ua.w; w[4] = r.ub.x; w[5] = r.ub.y;
  }
  uint32_t sg[2], cg[2];
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    sg[rr] = hfma2_u(prmt(r.sc, 0x64646464u, 0x4040u | (rr << 8) | rr), kSixteenth, kMinus72);  // sc / 16
    cg[rr] = hmul2_u(sg[rr], kMinus1536);                                                       // -96 sc
  }
  const __half2 dh = *reinterpret_cast<const __half2*>(&r.d);
  const float2 df = __half22float2(dh);
  const uint32_t s0 = h2_bits(__float2half2_rn(df.x)), s1 = h2_bits(__float2half2_rn(df.y));
#pragma unroll
  for (int gg = 0; gg < 2; ++gg) {
    const uint32_t W0 = w[3 * gg], W1 = w[3 * gg + 1], W2 = w[3 * gg + 2];
    const uint32_t p0 = and_or<0x03F003F0u>(W0, magic);
    const uint32_t p1 = and_or<0x03F003F0u>(W0 >> 6, magic);
    const uint32_t p2 = and_or<0x03F003F0u>(W1, magic);
    const uint32_t p3 = and_or<0x03F003F0u>(W1 >> 6, magic);
    const uint32_t p4 = and_or<0x03F003F0u>(W2, magic);
    const uint32_t p5 = and_or<0x03F003F0u>(W2 >> 6, magic);
    const uint32_t p6 = and_or<0x00F000F0u>(W0 << 4, and_or<0x03000300u>(W2 << 8, magic));
    const uint32_t p7 = and_or<0x00F000F0u>(W1 << 4, and_or<0x03000300u>(W2 << 6, magic));
    uint32_t a[4], b[4];
    a[0] = hfma2_u(p0, sg[0], cg[0]);
    a[1] = hfma2_u(p1, sg[1], cg[1]);
    a[2] = hfma2_u(p2, sg[0], cg[0]);
    a[3] = hfma2_u(p3, sg[1], cg[1]);
    b[0] = hfma2_u(p4, sg[0], cg[0]);
    b[1] = hfma2_u(p5, sg[1], cg[1]);
    b[2] = hfma2_u(p6, sg[0], cg[0]);
    b[3] = hfma2_u(p7, sg[1], cg[1]);
    store_rows(adst, r0, r1, 2 * part + gg, a, b, s0, s1);
  }
}

struct PrefillParams {
  const uint8_t* w0;   // tiled weights (gate, or the single matrix)
  const uint8_t* w1;   // tiled up weights (gate/up mode)
  const uint32_t* grid;
  int M, N, K;         // tokens, weight rows, k
  void* out;           // fp32 act [M][ldo] (gate/up) or fp32 y [M][ldo]
  int64_t ldo;
  const float* row_scale;  // per-token power-of-two scale of the staged tokens (nullptr: 1)
  uint32_t* err;
  uint32_t fp16_magic;  // 0x64006400, passed at run time (and_or in formats.cuh)
  // work list: n_full whole tiles, then the last split_r tiles (the ones that would
  // leave most SMs idle in a final partial wave) as `pieces` k-ranges each; the
  // pieces write fp32 partial accumulators and the last one to finish sums them in
  // piece order (deterministic) and runs the epilogue
  int n_full, split_r, pieces;
  uint32_t* cnt;  // [split_r][2]: pieces arrived / departed (the last to depart re-arms both)
  float* part;    // [split_r][pieces][NMAT][kPfTok tokens][kPfRows rows]
};

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* q) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(q) : "memory");
  return v;
}

struct WorkItem {
  int tile, kt0, kt1;  // output tile and its k-step range
  int slot, piece;     // slot < 0: a whole tile
};

__device__ __forceinline__ WorkItem work_item(const PrefillParams& p, int item, int kt_per_tile) {
  WorkItem w;
  if (item < p.n_full) {
    w.tile = item;
    w.kt0 = 0;
    w.kt1 = kt_per_tile;
    w.slot = -1;
    w.piece = 0;
    return w;
  }
  const int j = item - p.n_full;
  w.slot = j / p.pieces;
  w.piece = j - w.slot * p.pieces;
  w.tile = p.n_full + w.slot;
  w.kt0 = w.piece * kt_per_tile / p.pieces;
  w.kt1 = (w.piece + 1) * kt_per_tile / p.pieces;
  return w;
}


template <int QT, int NMAT>
struct Smem {
  static constexpr uint32_t kA = NMAT * kPfRows * 128;  // dequantised weights per stage
  static constexpr uint32_t kB = kPfTok * 128;          // token tile per stage
  static constexpr uint32_t kStage = kA + kB;
  static constexpr int kStages = NMAT == 2 ? 3 : 4;
  static constexpr uint32_t kGrid = QT == QT_IQ3_XXS ? kGridTableBytes : 0u;
  static constexpr uint32_t kStagesOff = 0;
  static constexpr uint32_t kGridOff = kStagesOff + kStages * kStage;
  static constexpr uint32_t kBarOff = kGridOff + kGrid;
  // full[S], empty[S], acc_full, acc_empty, done, tmem holder + abort flag
  static constexpr uint32_t kBytes = kBarOff + (2 * kStages + 4) * 8 + 16;
  static constexpr uint32_t kAlloc = kBytes + 1024;  // slack to align the base to 1024
};

template <int QT, int NMAT>
__global__ void __launch_bounds__(kWarps * 32, 1)
    prefill_kernel(const __grid_constant__ CUtensorMap tok_map, const PrefillParams p) {
  using L = Smem<QT, NMAT>;
  constexpr int S = L::kStages;
  constexpr uint32_t kCols = NMAT * kPfTok;  // TMEM columns (fp32 accumulators)
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* full = bars;
  uint64_t* empty = bars + S;
  uint64_t* acc_full = bars + 2 * S;
  uint64_t* acc_empty = bars + 2 * S + 1;
  uint64_t* done = bars + 2 * S + 2;
  uint64_t* epi_sync = bars + 2 * S + 3;  // the four epilogue warps (split-tile pieces)
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 2 * S + 4);
  volatile uint32_t* abort_flag = tmem_holder + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = p.K >> 8;                       // 256-k blocks
  const int kt_per_tile = p.K / kKStep;
  const int row_tiles = p.N / kPfRows;
  const int tok_tiles = (p.M + kPfTok - 1) / kPfTok;
  const int n_tiles = row_tiles * tok_tiles;
  const int n_items = p.n_full + p.split_r * p.pieces;
  (void)n_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1 + (kWarps - kDequantWarp0));
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 4);
    mbar_init(done, 1);
    mbar_init(epi_sync, 4);
    *abort_flag = 0u;
    mbar_fence_init();
  }
  if constexpr (QT == QT_IQ3_XXS) {
    uint2* tab = reinterpret_cast<uint2*>(smem + L::kGridOff);
    if (threadIdx.x < 256) {
      const uint2 e = grid_pair_entry(__ldg(p.grid + threadIdx.x));
#pragma unroll
      for (int c = 0; c < kGridCopies; ++c) tab[threadIdx.x * kGridCopies + c] = e;
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, kCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  griddep_wait();
  griddep_launch_dependents();

  auto fail = [&]() {
    atomicOr(p.err, ERR_MBAR_TIMEOUT);
    *abort_flag = 1u;
  };

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    if (lane == 0) {
      uint32_t kt_global = 0;
      for (int item = blockIdx.x; item < n_items && !*abort_flag; item += gridDim.x) {
        const WorkItem wi = work_item(p, item, kt_per_tile);
        const int tt = wi.tile % tok_tiles;
        for (int kt = wi.kt0; kt < wi.kt1 && !*abort_flag; ++kt, ++kt_global) {
          const int s = static_cast<int>(kt_global % S);
          if (!wait_bounded(&empty[s], ((kt_global / S) & 1) ^ 1)) {
            fail();
            break;
          }
          mbar_arrive_expect_tx(&full[s], L::kB);
          tma_load_2d(smem + L::kStagesOff + s * L::kStage + L::kA, &tok_map, kt * kKStep, tt * kPfTok, &full[s]);
        }
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      uint32_t kt_global = 0, tiles_done = 0;
      for (int item = blockIdx.x; item < n_items && !*abort_flag; item += gridDim.x, ++tiles_done) {
        const WorkItem wi = work_item(p, item, kt_per_tile);
        if (!wait_bounded(acc_empty, (tiles_done & 1) ^ 1)) {
          fail();
          break;
        }
        tc_fence_after();
        for (int kt = wi.kt0; kt < wi.kt1 && !*abort_flag; ++kt, ++kt_global) {
          const int s = static_cast<int>(kt_global % S);
          if (!wait_bounded(&full[s], (kt_global / S) & 1)) {
            fail();
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(smem + L::kStagesOff + s * L::kStage);
          const uint32_t b0 = a0 + L::kA;
#pragma unroll
          for (int kk = 0; kk < kKStep / 16; ++kk) {
            const uint64_t bdesc = sw128_desc(b0 + kk * 32);
#pragma unroll
            for (int mat = 0; mat < NMAT; ++mat) {
              const uint64_t adesc = sw128_desc(a0 + mat * kPfRows * 128 + kk * 32);
              umma_f16(tmem + mat * kPfTok, adesc, bdesc, kIdesc, (kt > wi.kt0 || kk > 0) ? 1u : 0u);
            }
          }
          umma_commit(&empty[s]);  // the stage is free once these MMAs have read it
        }
        umma_commit(acc_full);     // accumulators complete
      }
      // every issued MMA has completed before TMEM is released
      umma_commit(done);
      if (!wait_bounded(done, 0)) fail();
    }
  } else if (warp >= kEpiWarp0 && warp < kEpiWarp0 + 4) {
    // ------------------------------------------------------------------- epilogue
    const int wq = warp & 3;  // TMEM lane quarter of this warp
    const int rowl = wq * 32 + lane;  // this thread's row within the tile (its TMEM lane)
    __shared__ uint32_t s_last;
    uint32_t tiles_done = 0, epi_phase = 0;
    // all four epilogue warps at one point (bounded, like every wait here)
    auto epi_bar = [&]() -> bool {
      __syncwarp();
      if (lane == 0) mbar_arrive(epi_sync);
      const bool ok = wait_bounded(epi_sync, epi_phase);
      epi_phase ^= 1u;
      return ok;
    };
    for (int item = blockIdx.x; item < n_items && !*abort_flag; item += gridDim.x, ++tiles_done) {
      const WorkItem wi = work_item(p, item, kt_per_tile);
      const int rt = wi.tile / tok_tiles, tt = wi.tile - rt * tok_tiles;
      if (!wait_bounded_sleepy(acc_full, tiles_done & 1)) {
        if (lane == 0) fail();
        break;
      }
      tc_fence_after();
      const int row = rt * kPfRows + rowl;
      const uint32_t tbase = tmem + (static_cast<uint32_t>(wq * 32) << 16);
      if (wi.slot < 0) {
        for (int c0 = 0; c0 < kPfTok; c0 += 16) {
          uint32_t g[16];
          tmem_ld16(tbase + c0, g);
          if constexpr (NMAT == 2) {
            uint32_t u[16];
            tmem_ld16(tbase + kPfTok + c0, u);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int tok = tt * kPfTok + c0 + j;
              if (tok < p.M) {
                const float sc = p.row_scale ? p.row_scale[tok] : 1.0f;
                const float gv = __uint_as_float(g[j]) * sc, uv = __uint_as_float(u[j]) * sc;
                static_cast<float*>(p.out)[tok * p.ldo + row] = __fdividef(gv, 1.0f + __expf(-gv)) * uv;
              }
            }
          } else {
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int tok = tt * kPfTok + c0 + j;
              if (tok < p.M) {
                const float sc = p.row_scale ? p.row_scale[tok] : 1.0f;
                static_cast<float*>(p.out)[tok * p.ldo + row] = __uint_as_float(g[j]) * sc;
              }
            }
          }
        }
      } else {
        // a piece: its fp32 partial accumulators to the workspace (all 256 token
        // columns; columns past M hold the zero-filled tokens' zeros)
        float* pp = p.part + static_cast<int64_t>(wi.slot * p.pieces + wi.piece) * NMAT * (kPfTok * kPfRows);
        for (int c0 = 0; c0 < kPfTok; c0 += 16) {
#pragma unroll
          for (int mat = 0; mat < NMAT; ++mat) {
            uint32_t g[16];
            tmem_ld16(tbase + mat * kPfTok + c0, g);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j)
              pp[(static_cast<int64_t>(mat) * kPfTok + c0 + j) * kPfRows + rowl] = __uint_as_float(g[j]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty);  // TMEM is free for the next item
      if (wi.slot >= 0) {
        // every piece of the tile runs in this final wave, one per CTA, all resident:
        // wait until all have written their partials, then each sums its own share of
        // the tile's token columns over the pieces in piece order (deterministic)
        uint32_t* arrive = p.cnt + 2 * wi.slot;
        uint32_t* depart = arrive + 1;
        __threadfence();
        if (!epi_bar()) {
          if (lane == 0) fail();
          break;
        }
        if (warp == kEpiWarp0 && lane == 0) {
          atomicAdd(arrive, 1u);
          bool all = false;
          for (uint32_t i = 0; i < (kPollLimit >> 4) && !all; ++i) {
            all = ld_acquire_gpu(arrive) >= static_cast<uint32_t>(p.pieces);
            if (!all) __nanosleep(256);
          }
          s_last = all ? 1u : 0u;
        }
        if (!epi_bar()) {
          if (lane == 0) fail();
          break;
        }
        if (!s_last) {
          if (lane == 0) fail();
          break;
        }
        __threadfence();
        const float* pb = p.part + static_cast<int64_t>(wi.slot * p.pieces) * NMAT * (kPfTok * kPfRows);
        const int c_lo = wi.piece * kPfTok / p.pieces, c_hi = (wi.piece + 1) * kPfTok / p.pieces;
        constexpr int kTokUnroll = 8;  // token columns whose partial loads are in flight together
        for (int c0 = c_lo; c0 < c_hi; c0 += kTokUnroll) {
          float acc[kTokUnroll][NMAT];
#pragma unroll
          for (int j = 0; j < kTokUnroll; ++j)
#pragma unroll
            for (int mat = 0; mat < NMAT; ++mat) acc[j][mat] = 0.f;
          for (int q = 0; q < p.pieces; ++q) {
            float v[kTokUnroll][NMAT];
#pragma unroll
            for (int j = 0; j < kTokUnroll; ++j)
#pragma unroll
              for (int mat = 0; mat < NMAT; ++mat)
                v[j][mat] = c0 + j < c_hi
                                ? __ldcg(pb + ((static_cast<int64_t>(q) * NMAT + mat) * kPfTok + c0 + j) * kPfRows + rowl)
                                : 0.f;
#pragma unroll
            for (int j = 0; j < kTokUnroll; ++j)
#pragma unroll
              for (int mat = 0; mat < NMAT; ++mat) acc[j][mat] += v[j][mat];
          }
#pragma unroll
          for (int j = 0; j < kTokUnroll; ++j) {
            const int tok = tt * kPfTok + c0 + j;
            if (c0 + j < c_hi && tok < p.M) {
              const float sc = p.row_scale ? p.row_scale[tok] : 1.0f;
              float o;
              if constexpr (NMAT == 2) {
                const float gv = acc[j][0] * sc, uv = acc[j][1] * sc;
                o = __fdividef(gv, 1.0f + __expf(-gv)) * uv;
              } else {
                o = acc[j][0] * sc;
              }
              static_cast<float*>(p.out)[tok * p.ldo + row] = o;
            }
          }
        }
        // the last piece to leave re-arms both counters for the next launch
        if (!epi_bar()) {
          if (lane == 0) fail();
          break;
        }
        if (warp == kEpiWarp0 && lane == 0 && atomicAdd(depart, 1u) == static_cast<uint32_t>(p.pieces - 1)) {
          *arrive = 0u;
          *depart = 0u;
        }
      }
    }
  } else if (warp >= kDequantWarp0) {
    // ----------------------------------------------------------------- dequantise
    // task = (matrix, 16-row tile t, row pair g) of the stage's 128 x 64 slice, split
    // in parts: IQ3_XXS (gate/up, 128 tasks) by scale group (2 parts), Q6_K (64 tasks)
    // by sub-block (4 parts); 256 threads either way
    static_assert((QT == QT_IQ3_XXS && NMAT == 2) || (QT == QT_Q6_K && NMAT == 1), "prefill combination");
    constexpr int kSplit = QT == QT_IQ3_XXS ? 2 : 4;
    const int dt = threadIdx.x - kDequantWarp0 * 32;
    const int task = dt / kSplit, part = dt - task * kSplit;
    const int mat = task >> 6, t16 = (task >> 3) & 7, g = task & 7;
    const uint8_t* grid_lane = smem + L::kGridOff + (lane % kGridCopies) * 8;
    const uint8_t* wmat = mat == 0 ? p.w0 : p.w1;
    const uint32_t chunk = chunk_bytes(QT);
    const int r0 = 16 * t16 + g, r1 = r0 + 8;
    // position in this CTA's k-step sequence: work item, its tile and k step (256-k
    // block kt / 4, quarter kt % 4 = decode lane 4g + q)
    struct Pos {
      int item, tile, kt, kt1;
    };
    auto start = [&](Pos& ps, int item) {
      ps.item = item;
      if (item < n_items) {
        const WorkItem wi = work_item(p, item, kt_per_tile);
        ps.tile = wi.tile;
        ps.kt = wi.kt0;
        ps.kt1 = wi.kt1;
      }
    };
    auto advance = [&](Pos& ps) {
      if (++ps.kt == ps.kt1) start(ps, ps.item + static_cast<int>(gridDim.x));
    };
    auto fetch = [&](const Pos& ps, PartT<QT>& r) {
      if (ps.item < n_items) {
        const int rt = ps.tile / tok_tiles;
        load_part(wmat + (static_cast<int64_t>(rt * 8 + t16) * nb + (ps.kt >> 2)) * chunk, 4 * g + (ps.kt & 3), part,
                  r);
      }
    };
    Pos cur;
    start(cur, static_cast<int>(blockIdx.x));
    Pos pre = cur;
    PartT<QT> bufA, bufB, bufC;
    fetch(pre, bufA);
    advance(pre);
    fetch(pre, bufB);
    advance(pre);
    uint32_t kt_global = 0;
    bool ok = true;
    // one step: decode `use` into the stage, prefetch two steps ahead into `fill`
    auto step = [&](const PartT<QT>& use, PartT<QT>& fill) -> bool {
      fetch(pre, fill);
      advance(pre);
      const int s = static_cast<int>(kt_global % S);
      if (!wait_bounded(&empty[s], ((kt_global / S) & 1) ^ 1)) return false;
      uint8_t* adst = smem + L::kStagesOff + s * L::kStage + mat * kPfRows * 128;
      if constexpr (QT == QT_IQ3_XXS) dequant_iq3_part(use, part, grid_lane, adst, r0, r1, p.fp16_magic);
      else dequant_q6_part(use, part, adst, r0, r1, p.fp16_magic);
      // generic-proxy writes -> visible to the tensor core (async proxy)
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&full[s]);
      advance(cur);
      ++kt_global;
      return true;
    };
    while (cur.item < n_items && ok && !*abort_flag) {
      ok = step(bufA, bufC);
      if (!ok || cur.item >= n_items || *abort_flag) break;
      ok = step(bufB, bufA);
      if (!ok || cur.item >= n_items || *abort_flag) break;
      ok = step(bufC, bufB);
    }
    if (!ok && lane == 0) fail();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kCols);
  }
}

// ---- bf16 / fp32 -> fp16 token staging with a power-of-two scale per token row ----
// Rows can hold values beyond the fp16 range (the fp32 gate/up act of large-weight
// inputs does).  One CTA per row: max |x| over the row, then s = max(0, E - 14) for
// max |x| in [2^E, 2^(E+1)), and the row is stored as fp16(x * 2^-s): a single fp16
// rounding (none for bf16, whose 8 significant bits fit), with the scaled values
// below 2^15; only entries more than 2^28 times smaller than the row's maximum lose
// bits as fp16 subnormals.  row_scale[t] = 2^s, which the GEMM epilogue multiplies
// back.  Rows whose maximum fits fp16 get s = 0 (the plain conversion).
template <bool F32>
__global__ void __launch_bounds__(256) to_f16_kernel(const void* __restrict__ xv, int64_t ldx, int M, int K,
                                                     __half* __restrict__ out, float* __restrict__ row_scale) {
  griddep_wait();
  griddep_launch_dependents();
  __shared__ uint32_t red[8];
  const int per = K >> 3;  // 8 values per step
  for (int t = blockIdx.x; t < M; t += gridDim.x) {
    // 8 values of the row as fp32
    auto load8 = [&](int i, float (&v)[8]) {
      if constexpr (F32) {
        const float4* r = reinterpret_cast<const float4*>(static_cast<const float*>(xv) + t * ldx + 8 * i);
        const float4 a = r[0], b = r[1];
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
      } else {
        const uint4 u = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(xv) + t * ldx + 8 * i);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          v[2 * j] = __uint_as_float(w[j] << 16);
          v[2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
        }
      }
    };
    uint32_t mx = 0;  // max |x| as fp32 magnitude bits (monotone; inf / NaN compare highest)
    for (int i = threadIdx.x; i < per; i += blockDim.x) {
      float v[8];
      load8(i, v);
#pragma unroll
      for (int j = 0; j < 8; ++j) mx = max(mx, __float_as_uint(v[j]) & 0x7FFFFFFFu);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = red[0];
#pragma unroll
    for (int w = 1; w < 8; ++w) mx = max(mx, red[w]);
    __syncthreads();
    const int e = static_cast<int>(mx >> 23) - 127;               // unbiased exponent of max |x|
    const int sh = (mx < 0x7F800000u && e > 14) ? e - 14 : 0;    // inf / NaN rows: no scale
    const float down = __uint_as_float(static_cast<uint32_t>(127 - sh) << 23);   // 2^-sh
    if (threadIdx.x == 0) row_scale[t] = __uint_as_float(static_cast<uint32_t>(127 + sh) << 23);
    __half* orow = out + static_cast<int64_t>(t) * K;
    for (int i = threadIdx.x; i < per; i += blockDim.x) {
      float v[8];
      load8(i, v);
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) o[j] = h2_bits(__floats2half2_rn(v[2 * j] * down, v[2 * j + 1] * down));
      *reinterpret_cast<uint4*>(orow + 8 * i) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

// ------------------------------------------------------------------------ host
// the driver's tensor-map encoder, looked up through the runtime (the library does
// not link the driver library, so it loads on machines without a GPU driver)
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

bool make_tok_map(CUtensorMap* map, const void* base, int M, int K, int64_t ld_elems) {
  const EncodeTiledFn enc = encode_tiled();
  if (!enc) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(M)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld_elems) * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kKStep), static_cast<cuuint32_t>(kPfTok)};
  const cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int launch_pdl_raw(const void* kern, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, void** args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelExC(&cfg, kern, args) == cudaSuccess ? TLX_OK : TLX_ERR_LAUNCH;
}

int sms() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

constexpr int kMinPieceSteps = 16;  // k steps (64 k each) of the shortest piece of a split tile

// split region of the workspace (after the token staging): two counters per split
// tile (fewer than ctas), then the partials of at most ctas pieces of two matrices
size_t split_cnt_bytes(int ctas) { return (static_cast<size_t>(ctas) * 8 + 255) & ~size_t(255); }
size_t split_bytes(int ctas) { return split_cnt_bytes(ctas) + static_cast<size_t>(ctas) * 2 * kPfTok * kPfRows * 4; }

template <int QT, int NMAT>
int launch_prefill(const CUtensorMap& map, const PrefillParams& p, int max_ctas, uint8_t* split_ws,
                   size_t split_ws_bytes, cudaStream_t stream) {
  using L = Smem<QT, NMAT>;
  auto kern = prefill_kernel<QT, NMAT>;
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(L::kAlloc)) !=
        cudaSuccess)
      return TLX_ERR_LAUNCH;
    configured = true;
  }
  const int tiles = (p.N / kPfRows) * ((p.M + kPfTok - 1) / kPfTok);
  int ctas = sms();
  if (max_ctas > 0 && max_ctas < ctas) ctas = max_ctas;
  PrefillParams q = p;
  // the tiles of a final partial wave are split into k pieces across the idle SMs
  q.n_full = tiles;
  q.split_r = 0;
  q.pieces = 1;
  q.cnt = nullptr;
  q.part = nullptr;
  const int rem = tiles % ctas;
  if (rem != 0 && split_ws && split_ws_bytes >= split_bytes(ctas)) {
    int pieces = ctas / rem;
    const int max_pieces = (p.K / kKStep) / kMinPieceSteps;
    if (pieces > max_pieces) pieces = max_pieces;
    if (pieces >= 2) {
      q.n_full = tiles - rem;
      q.split_r = rem;
      q.pieces = pieces;
      q.cnt = reinterpret_cast<uint32_t*>(split_ws);
      q.part = reinterpret_cast<float*>(split_ws + split_cnt_bytes(ctas));
    }
  }
  const int items = q.n_full + q.split_r * q.pieces;
  if (ctas > items) ctas = items;
  CUtensorMap m = map;
  void* args[] = {&m, &q};
  return launch_pdl_raw(reinterpret_cast<const void*>(kern), dim3(ctas), dim3(kWarps * 32), L::kAlloc, stream, args);
}

bool al16(const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; }

}  // namespace

// workspace after the error word: the fp16 tokens, then one float scale per token
size_t prefill_x_bytes(int m, int64_t k) {
  return ((static_cast<size_t>(m) * static_cast<size_t>(k) * 2 + 255) & ~size_t(255)) + static_cast<size_t>(m) * 4;
}
size_t prefill_scale_offset(int m, int64_t k) {
  return (static_cast<size_t>(m) * static_cast<size_t>(k) * 2 + 255) & ~size_t(255);
}

// act[m][n_rows] (fp32) = silu(Wg x) * (Wu x), or y[m][n_rows] (fp32) = W x
int run_prefill(int gate_up, int qt, const void* w0, const void* w1, const uint32_t* grid, const void* x,
                int x_dtype, int64_t ldx, int m, int64_t n_rows, int64_t k, void* out, int64_t ldo, void* ws,
                size_t ws_bytes, uint32_t* err, int max_ctas, cudaStream_t stream) {
  if (qt != QT_IQ3_XXS && qt != QT_Q6_K) return TLX_ERR_QTYPE;
  // gate/up: IQ3_XXS (the grid table and two matrices per stage); single matrix: Q6_K
  if ((gate_up && qt != QT_IQ3_XXS) || (!gate_up && qt != QT_Q6_K)) return TLX_ERR_QTYPE;
  if (!w0 || !x || !out || !err || (gate_up && !w1) || (qt == QT_IQ3_XXS && !grid)) return TLX_ERR_NULL;
  if (m < 1 || n_rows < kPfRows || n_rows % kPfRows || k < 256 || k % 256 || k > (1 << 20) ||
      n_rows > (1 << 20) || m > (1 << 20))
    return TLX_ERR_SHAPE;
  if (ldo < n_rows) return TLX_ERR_SHAPE;
  if (!al16(w0) || (w1 && !al16(w1)) || !al16(x)) return TLX_ERR_ALIGN;
  const void* xf16 = x;
  int64_t ldx16 = ldx;
  const float* row_scale = nullptr;
  if (x_dtype == DT_BF16 || x_dtype == DT_F32) {
    if (!ws || ws_bytes < prefill_x_bytes(m, k)) return TLX_ERR_WORKSPACE;
    if (ldx < k || ldx % 8 || !al16(ws)) return TLX_ERR_ALIGN;
    const int blocks = m < 65536 ? m : 65536;
    const void* xb = x;
    int mm = m, kk = static_cast<int>(k);
    __half* o = static_cast<__half*>(ws);
    float* sc = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + prefill_scale_offset(m, k));
    void* args[] = {&xb, &ldx, &mm, &kk, &o, &sc};
    const void* kern = x_dtype == DT_F32 ? reinterpret_cast<const void*>(to_f16_kernel<true>)
                                         : reinterpret_cast<const void*>(to_f16_kernel<false>);
    // an ordinary launch: overlapped with the persistent kernel before it (PDL), the
    // staging ran about 85 us slower at config 5
    const int rc = cudaLaunchKernel(kern, dim3(blocks), dim3(256), args, 0, stream) == cudaSuccess ? TLX_OK
                                                                                         : TLX_ERR_LAUNCH;
    if (rc) return rc;
    xf16 = ws;
    ldx16 = k;
    row_scale = sc;
  } else if (x_dtype == DT_F16) {
    if (ldx < k || ldx % 8) return TLX_ERR_ALIGN;
  } else {
    return TLX_ERR_DTYPE;
  }
  return prefill_on_f16(gate_up, w0, w1, grid, xf16, ldx16, row_scale, m, n_rows, k, out, ldo, ws, ws_bytes, err,
                        max_ctas, stream);
}

// the contraction on tokens already in fp16 (row_scale: the per-token power-of-two
// factor of the staged rows, or nullptr); ws: the workspace after the error word
int prefill_on_f16(int gate_up, const void* w0, const void* w1, const uint32_t* grid, const void* xf16,
                   int64_t ldx16, const float* row_scale, int m, int64_t n_rows, int64_t k, void* out, int64_t ldo,
                   void* ws, size_t ws_bytes, uint32_t* err, int max_ctas, cudaStream_t stream) {
  CUtensorMap map;
  if (!make_tok_map(&map, xf16, m, static_cast<int>(k), ldx16)) return TLX_ERR_ALIGN;
  PrefillParams p;
  p.w0 = static_cast<const uint8_t*>(w0);
  p.w1 = static_cast<const uint8_t*>(w1);
  p.grid = grid;
  p.M = m;
  p.N = static_cast<int>(n_rows);
  p.K = static_cast<int>(k);
  p.out = out;
  p.ldo = ldo;
  p.row_scale = row_scale;
  p.err = err;
  p.fp16_magic = kMagic;
  // the split region follows the token staging (present in a workspace sized by
  // tlx_prefill_workspace_bytes; a smaller one runs without splitting)
  uint8_t* split_ws = nullptr;
  size_t split_ws_bytes = 0;
  const size_t split_off = (prefill_x_bytes(m, k) + 255) & ~size_t(255);
  if (ws && ws_bytes > split_off && al16(ws)) {
    split_ws = static_cast<uint8_t*>(ws) + split_off;
    split_ws_bytes = ws_bytes - split_off;
  }
  if (gate_up) return launch_prefill<QT_IQ3_XXS, 2>(map, p, max_ctas, split_ws, split_ws_bytes, stream);
  return launch_prefill<QT_Q6_K, 1>(map, p, max_ctas, split_ws, split_ws_bytes, stream);
}

}  // namespace tlx

using namespace tlx;

namespace {
constexpr size_t kPfErrBytes = 256;  // the workspace starts with the device error word
}

extern "C" {

size_t tlx_prefill_workspace_bytes(int m, int64_t k) {
  if (m < 1 || k < 256 || k % 256) return 0;
  return kPfErrBytes + ((prefill_x_bytes(m, k) + 255) & ~size_t(255)) + split_bytes(sms());
}

int tlx_prefill_ffn_gate_up(int qtype, const void* w_gate, const void* w_up, const uint32_t* grid, const void* x,
                            int x_dtype, int64_t ldx, int m, int64_t n_rows, int64_t k, void* act, int64_t ld_act,
                            void* ws, size_t ws_bytes, void* stream) {
  if (!ws) return TLX_ERR_NULL;
  if (ws_bytes < kPfErrBytes) return TLX_ERR_WORKSPACE;
  uint8_t* w = static_cast<uint8_t*>(ws);
  return run_prefill(1, qtype, w_gate, w_up, grid, x, x_dtype, ldx, m, n_rows, k, act, ld_act, w + kPfErrBytes,
                     ws_bytes - kPfErrBytes, reinterpret_cast<uint32_t*>(w), 0, static_cast<cudaStream_t>(stream));
}

int tlx_prefill_gemm(int qtype, const void* w, const uint32_t* grid, const void* x, int x_dtype, int64_t ldx, int m,
                     int64_t n_rows, int64_t k, float* y, int64_t ldy, void* ws, size_t ws_bytes, void* stream) {
  if (!ws) return TLX_ERR_NULL;
  if (ws_bytes < kPfErrBytes) return TLX_ERR_WORKSPACE;
  uint8_t* wb = static_cast<uint8_t*>(ws);
  return run_prefill(0, qtype, w, nullptr, grid, x, x_dtype, ldx, m, n_rows, k, y, ldy, wb + kPfErrBytes,
                     ws_bytes - kPfErrBytes, reinterpret_cast<uint32_t*>(wb), 0, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
