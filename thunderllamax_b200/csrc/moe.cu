// MoE verify layer (P <= 8 positions) on B200: router, routed + shared IQ4_XS
// experts, combine.  Four launches chained with programmatic dependent launch:
//
//   moe_router_kernel   logits = W_r h (fp32) for all experts plus the shared-expert
//                       gate row (one warp per row), and h staged as the fp16
//                       activation image of the gate/up projection.
//   moe_gate_up_kernel  every CTA first picks the top-8 per position from the logits
//                       (8 masked-argmax passes, strict '>', ties to the lower id;
//                       gates = softmax over the 8; sg = sigmoid(w_sh . h)) and builds
//                       the SLOT list: one slot per distinct routed expert of this
//                       rank's range (ascending id) with the positions routed to it,
//                       then the shared expert.  All CTAs compute the same list (no
//                       serial step); CTA 0 publishes it.  Then per (slot, 16-row
//                       tile): gate and up for the slot's positions, act = silu(g) u
//                       in fp32 into the workspace.
//   moe_act_image_kernel  one CTA per (position, expert) pair: the pair's act as the
//                       fp16 activation image of the down projection with one
//                       power-of-two scale per pair (act can exceed the fp16 range; the
//                       scale keeps max |act| at 2^14), built once for every down CTA,
//                       which bulk-copies it into shared memory.
//   moe_down_kernel     per (slot, 16-row tile of the hidden dim): down over act into
//                       fp32 parts[pair][row] (scale undone exactly); the last slot to
//                       finish a tile combines it:
//                       y = hres + sum_r gates[r] part_r + sg * shared (r ascending).
//
// Reference chain engine/mm/MM_P7_lib.py:505-511: rt8e256 (engine/mm/MM_P1_rt8e256.cu:
// 14-62) -> shexp8 -> gx8e256up4 (engine/mm/MM_P2_gx8e256up4.cu:8-55) -> gx8e256dn
// (engine/mm/MM_P2_gx8e256dn.cu:9-45) -> cmbz2048 (engine/mm/MM_P34_cmbz2048.cu:6-29).
// The reference runs one CTA per (position, rank) pair and reads an expert chosen by
// two positions twice; here each distinct expert is read once for all its positions
// (the positions are the columns of one mma.m16n8k16 n-tile).
//
// Weights: IQ4_XS in the 16-row tile layout of formats.cuh (chunk = 16 rows x one
// 256-weight block, 2176 B).  Dequantisation: a 256-entry shared table maps one qs
// byte (two 4-bit IQ4_NL indices, weights j and j+16 of a sub-block) to the fp16 pair
// (kv[lo], kv[hi]); the table holds one copy per lane at stride 256 B, so the 32
// lookups of a warp hit 32 distinct banks and the address is a single byte permute.
// The pair is multiplied by the sub-block scale (ls - 32) in fp16 (exact whenever
// |kv * (ls - 32)| <= 2048, otherwise one rounding, <= 2^-11 relative); the block
// scale d multiplies the fp32 mma result.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "common.cuh"
#include "formats.cuh"
#include "tlx_internal.h"

namespace tlx {
namespace {

constexpr int kTopK = 8;
constexpr int kMaxPos = 8;
constexpr int kMaxExperts = 1024;
constexpr int kMaxSlots = kTopK * kMaxPos + 1;  // distinct routed experts <= 8 P, + shared
constexpr int kExpWarps = 16;                   // warps per expert-kernel CTA
constexpr int kRouterWarps = 4;                 // experts per router CTA
constexpr int kKeysPerLane = 8;                 // register-resident selection keys (E <= 256)
constexpr uint32_t kLutBytes = 256u * 256u;     // entry v at 256 v, lane word at + 4 lane
constexpr uint32_t kRow = 68;                   // uint2 entries per image row (64 + 4 pad)
constexpr uint32_t kRowBytes = kRow * 8u;
constexpr uint32_t kChunk = kChunkIq4;          // 2176
constexpr uint32_t kSmemLimit = 227u * 1024u;

struct MoeMeta {
  uint32_t router_done;  // CTAs of the router that finished (re-armed by the last)
  int32_t n_slots;       // routed slots + shared slot
  int32_t n_routed;
  int32_t pad0;
  int32_t ids[kMaxPos * kTopK];
  float gates[kMaxPos * kTopK];
  float sg[kMaxPos];
  int16_t slot_expert[kMaxSlots];  // -1: the shared expert
  uint8_t slot_count[kMaxSlots];
  uint8_t slot_tok[kMaxSlots][8];   // positions (columns) of the slot, ascending; unused = column 0
  uint8_t slot_pair[kMaxSlots][8];  // pair id of each column: 8 p + r, shared 8 P + p
};

// the slot list, cached in shared memory by the expert kernels
struct SlotCache {
  int16_t expert[kMaxSlots];
  uint8_t count[kMaxSlots];
  uint8_t tok[kMaxSlots][8];
  uint8_t pair[kMaxSlots][8];
  int n_slots;
};

__device__ __forceinline__ void load_slots(const MoeMeta* mt, SlotCache& sc) {
  // every entry is loaded whether or not it is in use, so that all loads are in flight
  // together (one L2 round trip); entries past n_slots are never read
  for (int i = threadIdx.x; i < kMaxSlots; i += blockDim.x) {
    sc.expert[i] = __ldcg(&mt->slot_expert[i]);
    sc.count[i] = __ldcg(&mt->slot_count[i]);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      sc.tok[i][c] = __ldcg(&mt->slot_tok[i][c]);
      sc.pair[i][c] = __ldcg(&mt->slot_pair[i][c]);
    }
  }
  if (threadIdx.x == 0) sc.n_slots = __ldcg(&mt->n_slots);
}

struct MoeParams {
  const float* wr;    // [E][H] fp32 router
  const float* wsh;   // [H] fp32 shared-expert gate
  const uint16_t* h;  // [P][ldh] bf16 bits
  int64_t ldh;
  const uint8_t* gate;  // tiled IQ4_XS [E][I x H], expert-major
  const uint8_t* up;
  const uint8_t* down;   // tiled IQ4_XS [E][H x I]
  const uint8_t* sgate;  // shared expert (nullptr: none)
  const uint8_t* sup;
  const uint8_t* sdown;
  const int8_t* kvalues;  // IQ4_NL table, 16 entries
  const float* hres;      // [P][ldr] or nullptr
  int64_t ldr;
  float* y;
  int64_t ldy;
  int32_t* ids_out;
  float* gates_out;
  float* sg_out;
  int P, E, H, I, e0, e1, with_shared, stages;
  int64_t gu_bytes, dn_bytes;  // tiled bytes of one expert matrix
  MoeMeta* meta;
  float* logits;   // [P][E + 1]
  uint32_t* cnt;   // [H / 16] combine counters
  uint32_t* err;
  uint2* ximg;     // [H/256][P][68]
  float* actf;     // [9P][I] fp32 act
  float* parts;    // [9P][H]
  uint2* aimg;     // [I/256][9P][68] fp16 act image of the down projection
  float* ainv;     // [9P] the image's power-of-two scale per pair (act = image * ainv)
};

// ---- activation image (IQ4 k order) ----
// mma m of lane quarter q takes the byte pair 2m, 2m+1 of the quarter's 32 qs bytes:
// sub-block 2q + (m >> 3), bytes j0 = 2 (m & 7), j0 + 1, i.e. the weights
// k0 = 64q + 32 (m >> 3) + 2 (m & 7) and k0 + 16 (lo / hi nibble of byte j0), k0 + 1
// and k0 + 17 (byte j0 + 1).  Entry (m, q) of a 256-k block and column holds fp16
// {x[k0], x[k0+16], x[k0+1], x[k0+17]}; rows of 64 entries padded to 68.

__device__ __forceinline__ float silu_f(float g) { return g / (1.0f + expf(-g)); }

__device__ __forceinline__ uint16_t f32_to_f16_bits(float v) { return __half_as_ushort(__float2half_rn(v)); }

// table word for one byte of w: address = 256 * byte + 4 * lane, one PRMT
__device__ __forceinline__ uint32_t lut_get(const uint8_t* lut, uint32_t w, uint32_t lane4, uint32_t sel) {
  return *reinterpret_cast<const uint32_t*>(lut + __byte_perm(w, lane4, sel));
}

struct Iq4Lane {
  uint32_t q[16];    // rows g (0..7) and g+8 (8..15): qs bytes 32q' .. 32q'+32
  uint32_t s[2][2];  // fp16x2 (ls - 32) of sub-blocks 2q', 2q'+1 for row g / g+8
  float d[2];
};

__device__ __forceinline__ void iq4_load(const uint8_t* chunk, int lane, Iq4Lane& L) {
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const uint4 v = lds128(chunk + (u * 32 + lane) * 16);
    L.q[4 * u + 0] = v.x;
    L.q[4 * u + 1] = v.y;
    L.q[4 * u + 2] = v.z;
    L.q[4 * u + 3] = v.w;
  }
  const uint4 hd = lds128(chunk + 2048 + (lane >> 2) * 16);
  const int qq = lane & 3;
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    const uint32_t dsh = rr ? hd.z : hd.x, sl = rr ? hd.w : hd.y;
    L.d[rr] = __half2float(__ushort_as_half(static_cast<unsigned short>(dsh & 0xFFFFu)));
    const uint32_t sh = dsh >> 16;
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const uint32_t ls = ((sl >> (8 * qq + 4 * hh)) & 15u) | (((sh >> (4 * qq + 2 * hh)) & 3u) << 4);
      // fp16 1024 + ls in both halves, minus 1056: (ls - 32), exact
      L.s[rr][hh] = hadd2_u((ls | (ls << 16)) | kMagic, kMinus1056);
    }
  }
}

// A fragment of mma m from the lane's qs words: a0/a2 row g, a1/a3 row g+8
__device__ __forceinline__ void iq4_a(const Iq4Lane& L, int m, const uint8_t* lut, uint32_t lane4,
                                      uint32_t (&a)[4]) {
  const int wi = m >> 1, hh = m >> 3;
  const uint32_t s0 = 0x7604u | (static_cast<uint32_t>(2 * (m & 1)) << 4);
  const uint32_t s1 = s0 + 0x10u;
  a[0] = hmul2_u(lut_get(lut, L.q[wi], lane4, s0), L.s[0][hh]);
  a[2] = hmul2_u(lut_get(lut, L.q[wi], lane4, s1), L.s[0][hh]);
  a[1] = hmul2_u(lut_get(lut, L.q[8 + wi], lane4, s0), L.s[1][hh]);
  a[3] = hmul2_u(lut_get(lut, L.q[8 + wi], lane4, s1), L.s[1][hh]);
}

// D(16 x 8) += A(16 rows x 256 k of one chunk) . B(image rows of this lane's column)
__device__ __forceinline__ void iq4_chunk_mma(const Iq4Lane& L, const uint2* xb, const uint8_t* lut, uint32_t lane4,
                                              float (&t)[4]) {
#pragma unroll
  for (int m = 0; m < 16; ++m) {
    const uint2 b = xb[m * 4];
    uint32_t a[4];
    iq4_a(L, m, lut, lane4, a);
    mma16816(t, a, b.x, b.y);
  }
}

// gate and up chunks of one block share the activation loads
__device__ __forceinline__ void iq4_pair_compute(const Iq4Lane& G, const Iq4Lane& U, const uint2* xb,
                                                 const uint8_t* lut, uint32_t lane4, float (&ag)[4], float (&au)[4]) {
  float tg[4] = {0.f, 0.f, 0.f, 0.f}, tu[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int m = 0; m < 16; ++m) {
    const uint2 b = xb[m * 4];
    uint32_t a[4];
    iq4_a(G, m, lut, lane4, a);
    mma16816(tg, a, b.x, b.y);
    iq4_a(U, m, lut, lane4, a);
    mma16816(tu, a, b.x, b.y);
  }
  ag[0] += G.d[0] * tg[0];
  ag[1] += G.d[0] * tg[1];
  ag[2] += G.d[1] * tg[2];
  ag[3] += G.d[1] * tg[3];
  au[0] += U.d[0] * tu[0];
  au[1] += U.d[0] * tu[1];
  au[2] += U.d[1] * tu[2];
  au[3] += U.d[1] * tu[3];
}

// the byte table: entry v -> fp16x2 (kv[v & 15], kv[v >> 4]), one copy per lane
__device__ __forceinline__ void build_lut(uint8_t* lut, const int8_t* kvalues) {
  for (int i = threadIdx.x; i < 256 * 32; i += blockDim.x) {
    const int v = i >> 5, c = i & 31;
    const __half lo = __int2half_rn(static_cast<int>(__ldg(kvalues + (v & 15))));
    const __half hi = __int2half_rn(static_cast<int>(__ldg(kvalues + (v >> 4))));
    const uint32_t word =
        static_cast<uint32_t>(__half_as_ushort(lo)) | (static_cast<uint32_t>(__half_as_ushort(hi)) << 16);
    *reinterpret_cast<uint32_t*>(lut + v * 256 + c * 4) = word;
  }
}

// ---------------------------------------------------------------------------- router
// Shared memory: [kRouterWarps][H] fp32 router rows | [P][H] bf16 h | barriers.
__host__ __device__ inline uint32_t router_smem_bytes(int P, int H) {
  return static_cast<uint32_t>(kRouterWarps * H * 4 + P * H * 2 + (kRouterWarps + 1) * 8);
}

__global__ void __launch_bounds__(kRouterWarps * 32) moe_router_kernel(const MoeParams p) {
  extern __shared__ __align__(128) uint8_t rsm[];
  const int P = p.P, H = p.H, E = p.E;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* rows = reinterpret_cast<float*>(rsm);
  uint16_t* hs = reinterpret_cast<uint16_t*>(rsm + kRouterWarps * H * 4);
  uint64_t* bars = reinterpret_cast<uint64_t*>(rsm + kRouterWarps * H * 4 + P * H * 2);
  uint64_t* hbar = bars + kRouterWarps;
  const int e = blockIdx.x * kRouterWarps + warp;  // this warp's row: an expert, or (e == E) the shared gate
  if (threadIdx.x == 0) {
    for (int w = 0; w <= kRouterWarps; ++w) mbar_init(&bars[w], 1);
    mbar_fence_init();
  }
  __syncthreads();
  // the router rows are constants: fetch them before waiting for the previous kernel
  if (lane == 0 && e <= E) {
    const float* row = e < E ? p.wr + static_cast<int64_t>(e) * H : p.wsh;
    mbar_arrive_expect_tx(&bars[warp], static_cast<uint32_t>(H * 4));
    bulk_g2s(rows + warp * H, row, static_cast<uint32_t>(H * 4), &bars[warp]);
  }
  griddep_wait();
  griddep_launch_dependents();

  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(hbar, static_cast<uint32_t>(P * H * 2));
    for (int t = 0; t < P; ++t) bulk_g2s(hs + t * H, p.h + t * p.ldh, static_cast<uint32_t>(H * 2), hbar);
  }
  bool ok = mbar_wait_bounded(hbar, 0, threadIdx.x == 0 ? p.err : nullptr);
  // this CTA's share of the fp16 activation image of h (bf16 -> fp16, exact in range)
  if (ok) {
    const int per_tok = H >> 2;
    auto f16 = [&](const uint16_t* q) {
      return static_cast<uint32_t>(f32_to_f16_bits(__uint_as_float(static_cast<uint32_t>(*q) << 16)));
    };
    for (int gi = blockIdx.x * blockDim.x + threadIdx.x; gi < P * per_tok; gi += gridDim.x * blockDim.x) {
      const int t = gi / per_tok, ei = gi - t * per_tok;
      const int b = ei >> 6, m = (ei & 63) >> 2, q = ei & 3;
      const uint16_t* hr = hs + t * H + 256 * b + 64 * q + 32 * (m >> 3) + 2 * (m & 7);
      p.ximg[(b * P + t) * kRow + m * 4 + q] = make_uint2(f16(hr) | (f16(hr + 16) << 16), f16(hr + 1) | (f16(hr + 17) << 16));
    }
  }
  // one router row per warp, fp32 FMAs in k order per lane, then a fixed shuffle tree
  const bool row_ok = e <= E && mbar_wait_bounded(&bars[warp], 0, lane == 0 ? p.err : nullptr);
  if (ok && row_ok) {
    const float* row = rows + warp * H;
    float acc[kMaxPos];
#pragma unroll
    for (int t = 0; t < kMaxPos; ++t) acc[t] = 0.f;
    for (int k = 4 * lane; k < H; k += 128) {
      const float4 w = *reinterpret_cast<const float4*>(row + k);
#pragma unroll
      for (int t = 0; t < kMaxPos; ++t)
        if (t < P) {
          const uint2 xb = *reinterpret_cast<const uint2*>(hs + t * H + k);
          acc[t] = fmaf(w.x, __uint_as_float(xb.x << 16), acc[t]);
          acc[t] = fmaf(w.y, __uint_as_float(xb.x & 0xFFFF0000u), acc[t]);
          acc[t] = fmaf(w.z, __uint_as_float(xb.y << 16), acc[t]);
          acc[t] = fmaf(w.w, __uint_as_float(xb.y & 0xFFFF0000u), acc[t]);
        }
    }
#pragma unroll
    for (int t = 0; t < kMaxPos; ++t)
      if (t < P) {
        float v = acc[t];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) p.logits[t * (E + 1) + e] = v;
      }
  }
}

// ------------------------------------------------------------------ expert selection
// Shared-memory scratch of the selection: logits [P][E + 1] fp32, then one word per
// expert: bit t = position t routed to it, bits 8 + 3t .. 10 + 3t = its rank there.
__host__ __device__ inline uint32_t sel_scratch_bytes(int P, int E) { return static_cast<uint32_t>((P * (E + 1) + E) * 4); }

// Top-8 of every position, gates and sg, then the slot list into `sc`: the shared
// expert first (slot 0; its weights are known before routing), then one slot per
// distinct routed expert of [e0, e1) in ascending id.  Called by every thread of the
// CTA; `publish` writes the routing and the slot list to the workspace and the
// caller's outputs.  Positions are independent warps; each of the 8 rounds is one
// masked argmax over the logits (two warp max-reductions of the packed key: the
// value bits, then the lowest index among equal values).
__device__ void select_experts(const MoeParams& p, uint8_t* scratch, SlotCache& sc, bool publish) {
  const int P = p.P, E = p.E;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  float* lgs = reinterpret_cast<float*>(scratch);
  uint32_t* info = reinterpret_cast<uint32_t*>(lgs + P * (E + 1));
  {
    // every logit is loaded before any is stored: one L2 round trip for up to
    // 4 x blockDim logits (the P <= 8 x 1025 of the largest shape take two)
    constexpr int kLd = 4;
    const int n = P * (E + 1);
    for (int base = threadIdx.x; base < n; base += kLd * blockDim.x) {
      float v[kLd];
#pragma unroll
      for (int j = 0; j < kLd; ++j) {
        const int i = base + j * static_cast<int>(blockDim.x);
        v[j] = i < n ? __ldcg(p.logits + i) : 0.f;
      }
#pragma unroll
      for (int j = 0; j < kLd; ++j) {
        const int i = base + j * static_cast<int>(blockDim.x);
        if (i < n) lgs[i] = v[j];
      }
    }
  }
  for (int i = threadIdx.x; i < E; i += blockDim.x) info[i] = 0u;
  __syncthreads();
  MoeMeta* mt = p.meta;
  for (int t = warp; t < P; t += nwarps) {
    float* l = lgs + t * (E + 1);
    int ids[kTopK];
    float vals[kTopK];
    if (E <= 32 * kKeysPerLane) {
      // keys of this lane's experts (lane + 32 j) stay in registers across the rounds
      uint64_t key[kKeysPerLane];
#pragma unroll
      for (int j = 0; j < kKeysPerLane; ++j) {
        const int x = lane + 32 * j;
        key[j] = x < E ? argmax_key(l[x], static_cast<uint32_t>(x)) : 0ull;
      }
#pragma unroll
      for (int r = 0; r < kTopK; ++r) {
        uint64_t best = key[0];
#pragma unroll
        for (int j = 1; j < kKeysPerLane; ++j) best = key[j] > best ? key[j] : best;
        const uint32_t hi = static_cast<uint32_t>(best >> 32), lo = static_cast<uint32_t>(best);
        const uint32_t mh = __reduce_max_sync(0xffffffffu, hi);
        const uint32_t ml = __reduce_max_sync(0xffffffffu, hi == mh ? lo : 0u);
        const uint64_t w = (static_cast<uint64_t>(mh) << 32) | ml;
#pragma unroll
        for (int j = 0; j < kKeysPerLane; ++j) key[j] = key[j] == w ? 0ull : key[j];  // never selected again
        ids[r] = key_index(w);
        vals[r] = key_value(w);
      }
    } else {
#pragma unroll 1
      for (int r = 0; r < kTopK; ++r) {
        uint64_t best = 0ull;
        for (int x = lane; x < E; x += 32) {
          const uint64_t k = argmax_key(l[x], static_cast<uint32_t>(x));
          best = k > best ? k : best;
        }
        const uint32_t hi = static_cast<uint32_t>(best >> 32), lo = static_cast<uint32_t>(best);
        const uint32_t mh = __reduce_max_sync(0xffffffffu, hi);
        const uint32_t ml = __reduce_max_sync(0xffffffffu, hi == mh ? lo : 0u);
        const uint64_t w = (static_cast<uint64_t>(mh) << 32) | ml;
        ids[r] = key_index(w);
        vals[r] = key_value(w);
        __syncwarp();
        if (lane == (ids[r] & 31)) l[ids[r]] = __uint_as_float(0x7FC00000u);  // NaN: never selected again
        __syncwarp();
      }
    }
    const float mx = vals[0];
    float ex[kTopK], s = 0.f;
#pragma unroll
    for (int r = 0; r < kTopK; ++r) {
      ex[r] = expf(vals[r] - mx);
      s += ex[r];
    }
    if (lane < kTopK) {  // lane r publishes rank r
      float g = 0.f;
      int id = 0;
#pragma unroll
      for (int r = 0; r < kTopK; ++r)
        if (r == lane) {
          g = ex[r] / s;
          id = ids[r];
        }
      if (id >= p.e0 && id < p.e1) atomicOr(&info[id], (1u << t) | (static_cast<uint32_t>(lane) << (8 + 3 * t)));
      if (publish) {
        mt->ids[t * kTopK + lane] = id;
        mt->gates[t * kTopK + lane] = g;
        if (p.ids_out) p.ids_out[t * kTopK + lane] = id;
        if (p.gates_out) p.gates_out[t * kTopK + lane] = g;
      }
    }
    if (lane == 0 && publish) {
      const float sgv = 1.0f / (1.0f + expf(-l[E]));
      mt->sg[t] = sgv;
      if (p.sg_out) p.sg_out[t] = sgv;
    }
  }
  __syncthreads();
  // slot list, built by warp 0: lane L owns experts [L per, (L + 1) per), a warp scan
  // gives each lane its first slot
  if (warp == 0) {
    const int first = p.with_shared ? 1 : 0;
    const int per = (E + 31) >> 5;
    const int x0 = lane * per, x1 = min(E, x0 + per);
    int c = 0;
    for (int x = x0; x < x1; ++x) c += info[x] ? 1 : 0;
    int incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    int u = first + incl - c;
    for (int x = x0; x < x1; ++x)
      if (info[x]) sc.expert[u++] = static_cast<int16_t>(x);
    const int nr = __shfl_sync(0xffffffffu, incl, 31);
    if (lane == 0) {
      if (p.with_shared) {
        sc.expert[0] = -1;
        sc.count[0] = static_cast<uint8_t>(P);
        for (int t = 0; t < 8; ++t) {
          const int tt = t < P ? t : 0;
          sc.tok[0][t] = static_cast<uint8_t>(tt);
          sc.pair[0][t] = static_cast<uint8_t>(kTopK * P + tt);
        }
      }
      sc.n_slots = nr + first;
    }
  }
  __syncthreads();
  // columns of every routed slot: positions ascending, unused columns repeat column 0
  for (int u = (p.with_shared ? 1 : 0) + threadIdx.x; u < sc.n_slots; u += blockDim.x) {
    const uint32_t in = info[sc.expert[u]];
    int n = 0;
    for (int t = 0; t < P; ++t)
      if (in & (1u << t)) {
        sc.tok[u][n] = static_cast<uint8_t>(t);
        sc.pair[u][n] = static_cast<uint8_t>(t * kTopK + ((in >> (8 + 3 * t)) & 7u));
        ++n;
      }
    sc.count[u] = static_cast<uint8_t>(n);
    for (int c2 = n; c2 < 8; ++c2) {
      sc.tok[u][c2] = sc.tok[u][0];
      sc.pair[u][c2] = sc.pair[u][0];
    }
  }
  __syncthreads();
  if (publish) {
    for (int i = threadIdx.x; i < sc.n_slots; i += blockDim.x) {
      mt->slot_expert[i] = sc.expert[i];
      mt->slot_count[i] = sc.count[i];
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        mt->slot_tok[i][c] = sc.tok[i][c];
        mt->slot_pair[i][c] = sc.pair[i][c];
      }
    }
    if (threadIdx.x == 0) mt->n_slots = sc.n_slots;
  }
}

// routing alone (tlx_moe_route): one CTA publishes ids / gates / sg and the slots
__global__ void __launch_bounds__(256) moe_select_kernel(const MoeParams p) {
  extern __shared__ __align__(16) uint8_t ssm[];
  __shared__ SlotCache sc;
  griddep_wait();
  griddep_launch_dependents();
  select_experts(p, ssm, sc, true);
}

// ------------------------------------------------------------- expert kernels (shared)
struct ExpLayout {
  uint32_t img, ring, bars, total;
};

__host__ __device__ inline ExpLayout exp_layout(uint32_t img_bytes, int stages) {
  ExpLayout L;
  L.img = kLutBytes;
  L.ring = L.img + ((img_bytes + 127u) & ~127u);
  L.bars = L.ring + static_cast<uint32_t>(kExpWarps * stages) * kChunk;
  L.total = L.bars + static_cast<uint32_t>(kExpWarps * stages + 1) * 8u;
  return L;
}

// Per-warp chunk ring.  The warp's items are i = cta + C (warp + W k); item i is
// slot i / tiles, tile i % tiles, and reads `per_item` consecutive chunks of one or
// two matrices (two: gate and up alternate).  Chunk number c (in the warp's order)
// lives in ring slot c % S; lane 0 issues chunks up to S ahead of the compute cursor.
struct Ring {
  uint8_t* ring;
  uint64_t* bars;
  int S;
  int in_flight;             // chunks issued and not yet handed back (lane 0's count)
  int i_slot;                // next stage to fill (lane 0)
  int c_slot;                // next stage to consume (every lane)
  uint32_t c_phase;
  int item, j, n_items, step, per_item, nmat;  // issue cursor
  const uint8_t* base0;                        // this item's matrices (tile offset included)
  const uint8_t* base1;
};

template <typename BaseFn>
__device__ __forceinline__ void ring_issue(Ring& R, BaseFn base_of) {
  while (R.item < R.n_items && R.in_flight < R.S) {
    if (R.j == 0) base_of(R.item, R.base0, R.base1);
    const int slot = R.i_slot;
    mbar_arrive_expect_tx(&R.bars[slot], kChunk);
    const bool second = R.nmat == 2 && (R.j & 1);
    const int blk = R.nmat == 2 ? (R.j >> 1) : R.j;
    bulk_g2s(R.ring + slot * kChunk, (second ? R.base1 : R.base0) + static_cast<int64_t>(blk) * kChunk, kChunk,
             &R.bars[slot]);
    if (++R.i_slot == R.S) R.i_slot = 0;
    ++R.in_flight;
    if (++R.j == R.per_item) {
      R.j = 0;
      R.item += R.step;
    }
  }
}

__device__ __forceinline__ bool ring_wait(const Ring& R, uint32_t* err) {
  return mbar_wait_bounded(&R.bars[R.c_slot], R.c_phase, err);
}

__device__ __forceinline__ void ring_pop(Ring& R) {
  if (++R.c_slot == R.S) {
    R.c_slot = 0;
    R.c_phase ^= 1u;
  }
}

// let every copy the warp issued land before the CTA can exit (lane 0 issued them)
__device__ __forceinline__ void ring_drain(Ring& R) {
  if ((threadIdx.x & 31) != 0) return;
  for (; R.in_flight > 0; --R.in_flight) {
    mbar_wait_bounded(&R.bars[R.c_slot], R.c_phase, nullptr);
    ring_pop(R);
  }
}

// ------------------------------------------------------------------- gate/up kernel
// Work split: the CTA's items are k = 0..Kc-1 (global item blockIdx.x + C k, i.e.
// slot i / tiles, tile i % tiles); their units (item, 256-block) are divided evenly
// over the 16 warps, so every warp streams about the same number of chunk pairs.  An
// item wholly inside one warp's range is finished by that warp; an item split across
// warps is summed (in warp order, deterministic) by the warp holding its last unit.
__global__ void __launch_bounds__(kExpWarps * 32, 1) moe_gate_up_kernel(const MoeParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ SlotCache sc;
  const int P = p.P, S = p.stages;
  const int nbh = p.H >> 8, tpe = p.I >> 4;
  const uint32_t img_bytes = static_cast<uint32_t>(nbh * P) * kRowBytes;
  const ExpLayout L = exp_layout(img_bytes, S);
  const uint8_t* lut = smem;
  uint2* xs = reinterpret_cast<uint2*>(smem + L.img);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint64_t* xbar = reinterpret_cast<uint64_t*>(smem + L.bars) + kExpWarps * S;
  uint8_t* ring = smem + L.ring + static_cast<uint32_t>(warp * S) * kChunk;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars) + warp * S;

  build_lut(smem, p.kvalues);
  if (lane == 0)
    for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
  if (threadIdx.x == 0) mbar_init(xbar, 1);
  mbar_fence_init();

  // everything above touches only constants; the slot list and the image come from
  // the router, so wait for it to complete
  griddep_wait();
  griddep_launch_dependents();
  // every warp waits for the activation image; copy it while the experts are selected
  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(xbar, img_bytes);
    const uint8_t* src = reinterpret_cast<const uint8_t*>(p.ximg);
    for (uint32_t off = 0; off < img_bytes; off += 32768u)
      bulk_g2s(reinterpret_cast<uint8_t*>(xs) + off, src + off, std::min(32768u, img_bytes - off), xbar);
  }
  // selection scratch: the weight rings (idle until the slot list exists)
  select_experts(p, smem + L.ring, sc, blockIdx.x == 0);
  fence_proxy_async_smem();  // the scratch is overwritten by bulk copies next
  __syncthreads();

  const int C = gridDim.x;
  const int n_items = sc.n_slots * tpe;
  const int Kc = static_cast<int>(blockIdx.x) < n_items ? (n_items - 1 - static_cast<int>(blockIdx.x)) / C + 1 : 0;
  const int Uc = Kc * nbh;
  const int v0 = warp * Uc / kExpWarps, v1 = (warp + 1) * Uc / kExpWarps;
  auto warp_of_unit = [&](int v) { return static_cast<int>((static_cast<int64_t>(v + 1) * kExpWarps - 1) / Uc); };

  // chunk stream of this warp: units v0..v1, each gate then up.  Producer state (lane
  // 0): the unit cursor, the next stage to fill and the chunks in flight; consumer
  // state (every lane): the next stage to read and its phase
  int iv = v0, ij = 0, ik = v0 / nbh, ib = v0 - (v0 / nbh) * nbh;
  int in_flight = 0, i_slot = 0, c_slot = 0;
  uint32_t c_phase = 0u;
  auto issue = [&]() {
    while (iv < v1 && in_flight < S) {
      const int i = static_cast<int>(blockIdx.x) + C * ik;
      const int u = i / tpe, tau = i - u * tpe;
      const int e = sc.expert[u];
      const uint8_t* base = ij == 0 ? (e >= 0 ? p.gate + static_cast<int64_t>(e) * p.gu_bytes : p.sgate)
                                    : (e >= 0 ? p.up + static_cast<int64_t>(e) * p.gu_bytes : p.sup);
      mbar_arrive_expect_tx(&bars[i_slot], kChunk);
      bulk_g2s(ring + i_slot * kChunk, base + (static_cast<int64_t>(tau) * nbh + ib) * kChunk, kChunk,
               &bars[i_slot]);
      if (++i_slot == S) i_slot = 0;
      ++in_flight;
      if (++ij == 2) {
        ij = 0;
        ++iv;
        if (++ib == nbh) {
          ib = 0;
          ++ik;
        }
      }
    }
  };
  auto next_stage = [&]() {
    if (++c_slot == S) {
      c_slot = 0;
      c_phase ^= 1u;
    }
  };
  if (lane == 0) issue();
  __syncwarp();

  // every warp waits for the image (the copy must land before the CTA exits)
  bool failed = !mbar_wait_bounded(xbar, 0, lane == 0 ? p.err : nullptr);

  const uint32_t lane4 = static_cast<uint32_t>(lane) * 4u;
  const int g = lane >> 2, qq = lane & 3;

  // item epilogue on complete sums: act = silu(g) * u (fp32; the down kernel scales
  // each pair's act into the fp16 range)
  auto epilogue = [&](int k, const float (&ag)[4], const float (&au)[4]) {
    const int i = static_cast<int>(blockIdx.x) + C * k;
    const int u = i / tpe, tau = i - u * tpe;
    const int cnt = sc.count[u];
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
      const int col = 2 * qq + h2;
      const float a0 = silu_f(ag[h2]) * au[h2];          // row g
      const float a1 = silu_f(ag[2 + h2]) * au[2 + h2];  // row g + 8
      if (col < cnt) {
        const int pair = sc.pair[u][col];
        float* dst = p.actf + static_cast<int64_t>(pair) * p.I + tau * 16 + g;
        dst[0] = a0;
        dst[8] = a1;
      }
    }
  };

  // partial pieces (items split across warps): [0] the warp's first item, [1] its last
  float stash0[8], stash1[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) stash0[e] = stash1[e] = 0.f;
  float ag[4] = {0.f, 0.f, 0.f, 0.f}, au[4] = {0.f, 0.f, 0.f, 0.f};
  int cur_k = -1, piece_v = v0;
  const uint2* xl = xs;
  auto finish_piece = [&](int k, int vs, int ve) {
    if (vs == k * nbh && ve == (k + 1) * nbh) {
      epilogue(k, ag, au);
    } else {
      if (k == v0 / nbh) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          stash0[e] = ag[e];
          stash0[4 + e] = au[e];
        }
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          stash1[e] = ag[e];
          stash1[4 + e] = au[e];
        }
      }
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) ag[e] = au[e] = 0.f;
  };
  for (int v = v0; v < v1 && !failed; ++v) {
    const int k = v / nbh, b = v - k * nbh;
    if (k != cur_k) {
      if (cur_k >= 0) finish_piece(cur_k, piece_v, v);
      cur_k = k;
      piece_v = v;
      const int i = static_cast<int>(blockIdx.x) + C * k;
      xl = xs + sc.tok[i / tpe][g] * kRow + qq;
    }
    Iq4Lane G, U;
    if (!mbar_wait_bounded(&bars[c_slot], c_phase, lane == 0 ? p.err : nullptr)) {
      failed = true;
      break;
    }
    iq4_load(ring + c_slot * kChunk, lane, G);
    next_stage();
    if (!mbar_wait_bounded(&bars[c_slot], c_phase, lane == 0 ? p.err : nullptr)) {
      if (lane == 0) --in_flight;  // the gate chunk's stage has landed: nothing to drain there
      failed = true;
      break;
    }
    iq4_load(ring + c_slot * kChunk, lane, U);
    next_stage();
    // both chunks are in registers: hand the stages back (after their last generic-proxy
    // reads) before computing on them
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      in_flight -= 2;
      issue();
    }
    iq4_pair_compute(G, U, xl + b * P * kRow, lut, lane4, ag, au);
  }
  if (failed) {
    // let every copy this warp issued land before the CTA can exit (lane 0 issued them;
    // the stages not yet consumed start at the consumer's position)
    if (lane == 0)
      for (; in_flight > 0; --in_flight) {
        mbar_wait_bounded(&bars[c_slot], c_phase, nullptr);
        next_stage();
      }
  } else if (cur_k >= 0) {
    finish_piece(cur_k, piece_v, v1);
  }
  // pieces of split items -> this warp's own (now idle) ring, then the owners sum them
  float* pieces = reinterpret_cast<float*>(ring);
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    pieces[e * 32 + lane] = stash0[e];
    pieces[(8 + e) * 32 + lane] = stash1[e];
  }
  __syncthreads();
  if (failed || Uc == 0) return;
  // the one split item this warp may finish: the item holding its first unit, when
  // that item starts in an earlier warp and ends inside this warp's range
  if (v0 < v1 && v0 % nbh != 0 && (v0 / nbh + 1) * nbh <= v1) {
    const int k = v0 / nbh;
    const int wf = warp_of_unit(k * nbh), wl = warp;
    float sg[4] = {0.f, 0.f, 0.f, 0.f}, su[4] = {0.f, 0.f, 0.f, 0.f};
    for (int w = wf; w <= wl; ++w) {
      const float* pw = reinterpret_cast<const float*>(smem + L.ring + static_cast<uint32_t>(w * S) * kChunk);
      const int a = (k == (w * Uc / kExpWarps) / nbh) ? 0 : 1;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        sg[e] += pw[(a * 8 + e) * 32 + lane];
        su[e] += pw[(a * 8 + 4 + e) * 32 + lane];
      }
    }
    epilogue(k, sg, su);
  }
}

// ------------------------------------------------------------------ act image kernel
// The down projection's B operand, built once per layer instead of in every down CTA:
// one CTA per (position, expert) pair takes the pair's fp32 act row, its max |act|,
// a power-of-two scale that keeps it at <= 2^14 (the synthetic act exceeds the fp16
// range; the scale is exact and undone on the fp32 result), and writes the fp16 image
// entries (the IQ4 k order above) and the scale to the workspace.  Entry (m, q) of
// block bi is written by one thread from two float2 loads; a warp's loads cover two
// contiguous 256-byte runs of the row.
__global__ void __launch_bounds__(128) moe_act_image_kernel(const MoeParams p) {
  griddep_wait();
  griddep_launch_dependents();
  __shared__ float red[4];
  const int pair = blockIdx.x, npair = 9 * p.P, I = p.I, nbi = I >> 8;
  const float* a = p.actf + static_cast<int64_t>(pair) * I;
  float mx = 0.f;
  for (int i = threadIdx.x * 4; i < I; i += blockDim.x * 4) {
    const float4 v = __ldcg(reinterpret_cast<const float4*>(a + i));
    mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  int ex = 0;
  if (mx > 0.f && mx == mx) frexpf(mx, &ex);
  const float inv = ldexpf(1.0f, ex - 14);
  const float scl = 1.0f / inv;  // exact: a power of two
  if (threadIdx.x == 0) p.ainv[pair] = inv;
  for (int e = threadIdx.x; e < nbi * 64; e += blockDim.x) {
    const int m = e & 15, q = (e >> 4) & 3, bi = e >> 6;
    const int k0 = 256 * bi + 64 * q + 32 * (m >> 3) + 2 * (m & 7);
    const float2 lo = __ldcg(reinterpret_cast<const float2*>(a + k0));
    const float2 hi = __ldcg(reinterpret_cast<const float2*>(a + k0 + 16));
    p.aimg[(bi * npair + pair) * kRow + m * 4 + q] =
        make_uint2(f32_to_f16_bits(lo.x * scl) | (static_cast<uint32_t>(f32_to_f16_bits(hi.x * scl)) << 16),
                   f32_to_f16_bits(lo.y * scl) | (static_cast<uint32_t>(f32_to_f16_bits(hi.y * scl)) << 16));
  }
}

// --------------------------------------------------------------- down + combine kernel
__global__ void __launch_bounds__(kExpWarps * 32, 1) moe_down_kernel(const MoeParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ SlotCache sc;
  __shared__ float s_inv[9 * kMaxPos];
  __shared__ float s_gate[9 * kMaxPos];
  const int P = p.P, S = p.stages, I = p.I;
  const int nbi = I >> 8, tpd = p.H >> 4;
  const int npair = 9 * P;
  const uint32_t img_bytes = static_cast<uint32_t>(nbi * npair) * kRowBytes;
  const ExpLayout L = exp_layout(img_bytes, S);
  const uint8_t* lut = smem;
  uint2* as = reinterpret_cast<uint2*>(smem + L.img);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  Ring R;
  R.ring = smem + L.ring + static_cast<uint32_t>(warp * S) * kChunk;
  R.bars = reinterpret_cast<uint64_t*>(smem + L.bars) + warp * S;
  R.S = S;
  uint64_t* ibar = reinterpret_cast<uint64_t*>(smem + L.bars) + kExpWarps * S;

  build_lut(smem, p.kvalues);
  if (lane == 0)
    for (int s = 0; s < S; ++s) mbar_init(&R.bars[s], 1);
  if (threadIdx.x == 0) mbar_init(ibar, 1);
  mbar_fence_init();
  __syncthreads();

  griddep_wait();
  griddep_launch_dependents();
  // the act image, built once for all CTAs by moe_act_image_kernel: bulk copies into
  // shared memory while the slot list and the combine weights are loaded
  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(ibar, img_bytes);
    const uint8_t* src = reinterpret_cast<const uint8_t*>(p.aimg);
    for (uint32_t off = 0; off < img_bytes; off += 32768u)
      bulk_g2s(reinterpret_cast<uint8_t*>(as) + off, src + off, std::min(32768u, img_bytes - off), ibar);
  }
  load_slots(p.meta, sc);
  for (int i = threadIdx.x; i < npair; i += blockDim.x) {
    // combine weight: the router gate of a routed pair whose expert is this rank's,
    // the shared gate of a shared pair (when the shared expert is here), else 0
    float gw = 0.f;
    if (i < kTopK * P) {
      const int id = __ldcg(&p.meta->ids[i]);
      const float g = __ldcg(&p.meta->gates[i]);
      gw = id >= p.e0 && id < p.e1 ? g : 0.f;
    } else if (p.with_shared) {
      gw = __ldcg(&p.meta->sg[i - kTopK * P]);
    }
    s_gate[i] = gw;
    s_inv[i] = __ldcg(p.ainv + i);
  }
  __syncthreads();
  const int n_slots = sc.n_slots;
  if (n_slots == 0) {
    // nothing routed to this rank's experts and no shared expert: y = hres (or 0)
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < P * p.H; i += gridDim.x * blockDim.x) {
      const int t = i / p.H, r = i - t * p.H;
      p.y[t * p.ldy + r] = p.hres ? p.hres[t * p.ldr + r] : 0.f;
    }
    mbar_wait_bounded(ibar, 0, threadIdx.x == 0 ? p.err : nullptr);  // the image copy lands before exit
    return;
  }
  const int n_items = n_slots * tpd;
  const int i_first = blockIdx.x + gridDim.x * warp;
  R.in_flight = R.i_slot = R.c_slot = 0;
  R.c_phase = 0u;
  R.item = i_first;
  R.j = 0;
  R.n_items = n_items;
  R.step = gridDim.x * kExpWarps;
  R.per_item = nbi;
  R.nmat = 1;
  auto base_of = [&](int item, const uint8_t*& b0, const uint8_t*& b1) {
    const int u = item / tpd, tau = item - u * tpd;
    const int e = sc.expert[u];
    b0 = (e >= 0 ? p.down + static_cast<int64_t>(e) * p.dn_bytes : p.sdown) + static_cast<int64_t>(tau) * nbi * kChunk;
    b1 = b0;
  };
  // weights do not depend on act: start streaming, then wait for the image
  if (lane == 0) ring_issue(R, base_of);
  bool failed = !mbar_wait_bounded(ibar, 0, threadIdx.x == 0 ? p.err : nullptr);
  const uint32_t lane4 = static_cast<uint32_t>(lane) * 4u;
  const int g = lane >> 2, qq = lane & 3;
  for (int item = i_first; item < n_items && !failed; item += R.step) {
    const int u = item / tpd, tau = item - u * tpd;
    const int cnt = sc.count[u];
    const uint2* xl = as + sc.pair[u][g] * kRow + qq;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int b = 0; b < nbi; ++b) {
      if (!ring_wait(R, lane == 0 ? p.err : nullptr)) {
        failed = true;
        break;
      }
      Iq4Lane W;
      iq4_load(R.ring + R.c_slot * kChunk, lane, W);
      ring_pop(R);
      // the chunk is in registers: hand the stage back before computing on it
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        --R.in_flight;
        ring_issue(R, base_of);
      }
      float t4[4] = {0.f, 0.f, 0.f, 0.f};
      iq4_chunk_mma(W, xl + b * npair * kRow, lut, lane4, t4);
      acc[0] += W.d[0] * t4[0];
      acc[1] += W.d[0] * t4[1];
      acc[2] += W.d[1] * t4[2];
      acc[3] += W.d[1] * t4[3];
    }
    if (failed) break;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int col = 2 * qq + (e & 1);
      if (col < cnt) {
        const int pair = sc.pair[u][col];
        const int row = tau * 16 + g + 8 * (e >> 1);
        p.parts[static_cast<int64_t>(pair) * p.H + row] = acc[e] * s_inv[pair];
      }
    }
  }
  if (failed) {
    ring_drain(R);
    return;
  }
  // one fence for all of this warp's parts, then per item: the last slot to finish
  // a 16-row tile combines it
  __threadfence();
  // the counters of up to 32 of the warp's items are bumped at once (lane j: the j-th
  // item), then the warp combines the tiles it completed
  for (int base = i_first; base < n_items; base += 32 * R.step) {
    const int mine = base + lane * R.step;
    uint32_t old = 0;
    if (mine < n_items) old = atomicAdd(p.cnt + mine % tpd, 1u);
    uint32_t last = __ballot_sync(0xffffffffu, mine < n_items && old == static_cast<uint32_t>(n_slots - 1));
    if (last) __threadfence();
    while (last) {
      const int tau = (base + (__ffs(last) - 1) * R.step) % tpd;
      last &= last - 1;
      // 16 rows x P positions per tile; every output's nine parts (and the residual)
      // are loaded for all of the lane's outputs before any is summed (one L2 round
      // trip per tile), then summed in a fixed order (routed ranks 0..7, then the
      // shared expert)
      constexpr int kIt = (16 * kMaxPos + 31) / 32, kBatch = 2;
#pragma unroll 1
      for (int it0 = 0; it0 < kIt && 32 * it0 < 16 * P; it0 += kBatch) {
        float pv[kBatch][kTopK + 2];
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
          const int idx = lane + 32 * (it0 + j);
          if (idx < 16 * P) {
            const int t = idx >> 4, row = tau * 16 + (idx & 15);
#pragma unroll
            for (int r = 0; r < kTopK; ++r)
              pv[j][r] = __ldcg(p.parts + static_cast<int64_t>(t * kTopK + r) * p.H + row);
            pv[j][kTopK] = __ldcg(p.parts + static_cast<int64_t>(kTopK * P + t) * p.H + row);
            pv[j][kTopK + 1] = p.hres ? p.hres[t * p.ldr + row] : 0.f;
          }
        }
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
          const int idx = lane + 32 * (it0 + j);
          if (idx < 16 * P) {
            const int t = idx >> 4, row = tau * 16 + (idx & 15);
            float a = 0.f;
#pragma unroll
            for (int r = 0; r < kTopK; ++r) {
              const float gw = s_gate[t * kTopK + r];
              if (gw != 0.f) a += gw * pv[j][r];
            }
            const float gs = s_gate[kTopK * P + t];
            if (gs != 0.f) a += gs * pv[j][kTopK];
            p.y[t * p.ldy + row] = pv[j][kTopK + 1] + a;
          }
        }
      }
      if (lane == 0) p.cnt[tau] = 0u;
    }
  }
  if (failed) ring_drain(R);
}

// ------------------------------------------------------------------------------ host
struct WsLayout {
  size_t meta, logits, cnt, err, ximg, actf, parts, aimg, ainv, total;
};

inline size_t up256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

bool moe_shape_ok(int P, int E, int H, int I) {
  return P >= 1 && P <= kMaxPos && E >= kTopK && E <= kMaxExperts && H >= 256 && H % 256 == 0 && I >= 256 &&
         I % 256 == 0 && H <= 16384 && I <= 4096;
}

WsLayout ws_layout(int P, int E, int H, int I) {
  WsLayout w;
  size_t o = 0;
  w.meta = o;
  o = up256(o + sizeof(MoeMeta));
  w.logits = o;
  o = up256(o + static_cast<size_t>(P) * (E + 1) * 4);
  w.cnt = o;
  o = up256(o + static_cast<size_t>(H / 16) * 4);
  w.err = o;
  o = up256(o + 4);
  w.ximg = o;
  o = up256(o + static_cast<size_t>(H / 256) * P * kRowBytes);
  w.actf = o;
  o = up256(o + static_cast<size_t>(9 * P) * I * 4);
  w.parts = o;
  o = up256(o + static_cast<size_t>(9 * P) * H * 4);
  w.aimg = o;
  o = up256(o + static_cast<size_t>(I / 256) * (9 * P) * kRowBytes);
  w.ainv = o;
  o = up256(o + static_cast<size_t>(9 * P) * 4);
  w.total = o;
  return w;
}

int stages_for(uint32_t img_bytes, int want) {
  // dynamic shared memory; the static slot cache and scales take the rest (< 4 KB)
  for (int s = want; s >= 2; --s)
    if (exp_layout(img_bytes, s).total <= kSmemLimit - 4096u) return s;
  return 0;
}

int launch_ex(const void* kern, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, const MoeParams& p) {
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
  void* args[] = {const_cast<MoeParams*>(&p)};
  return cudaLaunchKernelExC(&cfg, kern, args) == cudaSuccess ? TLX_OK : TLX_ERR_LAUNCH;
}

int sm_count() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

bool al(const void* q, size_t a) { return (reinterpret_cast<uintptr_t>(q) & (a - 1)) == 0; }

int setup(const MoeParams& in, int P, int E, int H, int I, int e0, int e1, void* ws, size_t ws_bytes, MoeParams& p) {
  if (!moe_shape_ok(P, E, H, I)) return TLX_ERR_SHAPE;
  if (e0 < 0 || e1 > E || e0 > e1) return TLX_ERR_SHAPE;
  if (!ws) return TLX_ERR_NULL;
  const WsLayout w = ws_layout(P, E, H, I);
  if (ws_bytes < w.total) return TLX_ERR_WORKSPACE;
  if (!al(ws, 256)) return TLX_ERR_ALIGN;
  p = in;
  p.P = P;
  p.E = E;
  p.H = H;
  p.I = I;
  p.e0 = e0;
  p.e1 = e1;
  uint8_t* b = static_cast<uint8_t*>(ws);
  p.meta = reinterpret_cast<MoeMeta*>(b + w.meta);
  p.logits = reinterpret_cast<float*>(b + w.logits);
  p.cnt = reinterpret_cast<uint32_t*>(b + w.cnt);
  p.err = reinterpret_cast<uint32_t*>(b + w.err);
  p.ximg = reinterpret_cast<uint2*>(b + w.ximg);
  p.actf = reinterpret_cast<float*>(b + w.actf);
  p.parts = reinterpret_cast<float*>(b + w.parts);
  p.aimg = reinterpret_cast<uint2*>(b + w.aimg);
  p.ainv = reinterpret_cast<float*>(b + w.ainv);
  p.gu_bytes = static_cast<int64_t>(I / 16) * (H / 256) * kChunk;
  p.dn_bytes = static_cast<int64_t>(H / 16) * (I / 256) * kChunk;
  return TLX_OK;
}

// raise a kernel's dynamic shared memory limit once (not per launch)
int ensure_smem(const void* kern, size_t bytes, size_t& configured) {
  if (bytes <= configured) return TLX_OK;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes)) != cudaSuccess)
    return TLX_ERR_LAUNCH;
  configured = bytes;
  return TLX_OK;
}
size_t g_router_smem = 0, g_select_smem = 0, g_gate_up_smem = 0, g_down_smem = 0;

int launch_router(const MoeParams& p, cudaStream_t stream) {
  const size_t smem = router_smem_bytes(p.P, p.H);
  if (smem > kSmemLimit - 4096u) return TLX_ERR_SHAPE;
  if (ensure_smem(reinterpret_cast<const void*>(moe_router_kernel), smem, g_router_smem)) return TLX_ERR_LAUNCH;
  const int ctas = (p.E + 1 + kRouterWarps - 1) / kRouterWarps;
  return launch_ex(reinterpret_cast<const void*>(moe_router_kernel), dim3(ctas), dim3(kRouterWarps * 32), smem,
                   stream, p);
}

int launch_select(const MoeParams& p, cudaStream_t stream) {
  const size_t smem = sel_scratch_bytes(p.P, p.E);
  if (ensure_smem(reinterpret_cast<const void*>(moe_select_kernel), smem, g_select_smem)) return TLX_ERR_LAUNCH;
  return launch_ex(reinterpret_cast<const void*>(moe_select_kernel), dim3(1), dim3(256), smem, stream, p);
}

int launch_experts(MoeParams p, cudaStream_t stream) {
  const int C = sm_count();
  {
    const uint32_t img = static_cast<uint32_t>((p.H / 256) * p.P) * kRowBytes;
    p.stages = stages_for(img, 4);
    if (p.stages == 0) return TLX_ERR_SHAPE;
    // the selection scratch lives in the (not yet used) weight rings
    if (sel_scratch_bytes(p.P, p.E) > static_cast<uint32_t>(kExpWarps * p.stages) * kChunk) return TLX_ERR_SHAPE;
    const uint32_t smem = exp_layout(img, p.stages).total;
    if (ensure_smem(reinterpret_cast<const void*>(moe_gate_up_kernel), smem, g_gate_up_smem)) return TLX_ERR_LAUNCH;
    const int rc = launch_ex(reinterpret_cast<const void*>(moe_gate_up_kernel), dim3(C), dim3(kExpWarps * 32), smem,
                             stream, p);
    if (rc) return rc;
  }
  {
    const int rc = launch_ex(reinterpret_cast<const void*>(moe_act_image_kernel), dim3(9 * p.P), dim3(128), 0, stream,
                             p);
    if (rc) return rc;
  }
  {
    const uint32_t img = static_cast<uint32_t>((p.I / 256) * 9 * p.P) * kRowBytes;
    p.stages = stages_for(img, 4);
    if (p.stages == 0) return TLX_ERR_SHAPE;
    const uint32_t smem = exp_layout(img, p.stages).total;
    if (ensure_smem(reinterpret_cast<const void*>(moe_down_kernel), smem, g_down_smem)) return TLX_ERR_LAUNCH;
    return launch_ex(reinterpret_cast<const void*>(moe_down_kernel), dim3(C), dim3(kExpWarps * 32), smem, stream, p);
  }
}

}  // namespace
}  // namespace tlx

using namespace tlx;

extern "C" {

size_t tlx_moe_workspace_bytes(int p, int n_experts, int hidden, int inner) {
  if (!moe_shape_ok(p, n_experts, hidden, inner)) return 0;
  return ws_layout(p, n_experts, hidden, inner).total;
}

}  // extern "C"

namespace {
// router logits (+ h image); with `select`, also the standalone selection launch
int route_impl(const float* w_router, const float* w_shared_gate, const void* h, int64_t ldh, int p, int n_experts,
               int hidden, int inner, int expert_begin, int expert_end, int with_shared, int32_t* ids, float* gates,
               float* sg, void* ws, size_t ws_bytes, void* stream, bool select) {
  if (!w_router || !w_shared_gate || !h) return TLX_ERR_NULL;
  MoeParams in = {};
  in.wr = w_router;
  in.wsh = w_shared_gate;
  in.h = static_cast<const uint16_t*>(h);
  in.ldh = ldh;
  in.ids_out = ids;
  in.gates_out = gates;
  in.sg_out = sg;
  in.with_shared = with_shared ? 1 : 0;
  MoeParams prm;
  int rc = setup(in, p, n_experts, hidden, inner, expert_begin, expert_end, ws, ws_bytes, prm);
  if (rc) return rc;
  if (ldh < hidden || (ldh & 7) || !al(h, 16) || !al(w_router, 16) || !al(w_shared_gate, 16)) return TLX_ERR_ALIGN;
  rc = launch_router(prm, static_cast<cudaStream_t>(stream));
  if (rc || !select) return rc;
  return launch_select(prm, static_cast<cudaStream_t>(stream));
}
}  // namespace

extern "C" {

int tlx_moe_route(const float* w_router, const float* w_shared_gate, const void* h, int64_t ldh, int p,
                  int n_experts, int hidden, int inner, int expert_begin, int expert_end, int with_shared,
                  int32_t* ids, float* gates, float* sg, void* ws, size_t ws_bytes, void* stream) {
  return route_impl(w_router, w_shared_gate, h, ldh, p, n_experts, hidden, inner, expert_begin, expert_end,
                    with_shared, ids, gates, sg, ws, ws_bytes, stream, true);
}

}  // extern "C"

namespace {
int experts_impl(const void* gate, const void* up, const void* down, const void* shared_gate, const void* shared_up,
                 const void* shared_down, const int8_t* kvalues, const float* hres, int64_t ldr, float* y, int64_t ldy,
                 int32_t* ids, float* gates, float* sg, int p, int n_experts, int hidden, int inner, int expert_begin,
                 int expert_end, void* ws, size_t ws_bytes, void* stream) {
  if (!kvalues || !y) return TLX_ERR_NULL;
  const bool shared = shared_gate != nullptr;
  if (shared && (!shared_up || !shared_down)) return TLX_ERR_NULL;
  if (expert_end > expert_begin && (!gate || !up || !down)) return TLX_ERR_NULL;
  MoeParams in = {};
  in.gate = static_cast<const uint8_t*>(gate);
  in.up = static_cast<const uint8_t*>(up);
  in.down = static_cast<const uint8_t*>(down);
  in.sgate = static_cast<const uint8_t*>(shared_gate);
  in.sup = static_cast<const uint8_t*>(shared_up);
  in.sdown = static_cast<const uint8_t*>(shared_down);
  in.kvalues = kvalues;
  in.hres = hres;
  in.ldr = ldr;
  in.y = y;
  in.ldy = ldy;
  in.ids_out = ids;
  in.gates_out = gates;
  in.sg_out = sg;
  in.with_shared = shared ? 1 : 0;
  MoeParams prm;
  int rc = setup(in, p, n_experts, hidden, inner, expert_begin, expert_end, ws, ws_bytes, prm);
  if (rc) return rc;
  for (const void* q : {gate, up, down, shared_gate, shared_up, shared_down})
    if (q && !al(q, 16)) return TLX_ERR_ALIGN;
  if (ldy < hidden || (hres && ldr < hidden)) return TLX_ERR_SHAPE;
  return launch_experts(prm, static_cast<cudaStream_t>(stream));
}
}  // namespace

extern "C" {

int tlx_moe_experts(const void* gate, const void* up, const void* down, const void* shared_gate,
                    const void* shared_up, const void* shared_down, const int8_t* kvalues, const float* hres,
                    int64_t ldr, float* y, int64_t ldy, int p, int n_experts, int hidden, int inner,
                    int expert_begin, int expert_end, void* ws, size_t ws_bytes, void* stream) {
  return experts_impl(gate, up, down, shared_gate, shared_up, shared_down, kvalues, hres, ldr, y, ldy, nullptr,
                      nullptr, nullptr, p, n_experts, hidden, inner, expert_begin, expert_end, ws, ws_bytes, stream);
}

int tlx_moe_verify(const float* w_router, const float* w_shared_gate, const void* gate, const void* up,
                   const void* down, const void* shared_gate, const void* shared_up, const void* shared_down,
                   const int8_t* kvalues, const void* h, int64_t ldh, const float* hres, int64_t ldr, float* y,
                   int64_t ldy, int32_t* ids, float* gates, float* sg, int p, int n_experts, int hidden, int inner,
                   int expert_begin, int expert_end, void* ws, size_t ws_bytes, void* stream) {
  int rc = route_impl(w_router, w_shared_gate, h, ldh, p, n_experts, hidden, inner, expert_begin, expert_end,
                      shared_gate != nullptr, ids, gates, sg, ws, ws_bytes, stream, false);
  if (rc) return rc;
  return experts_impl(gate, up, down, shared_gate, shared_up, shared_down, kvalues, hres, ldr, y, ldy, ids, gates, sg,
                      p, n_experts, hidden, inner, expert_begin, expert_end, ws, ws_bytes, stream);
}

int tlx_moe_workspace_error(const void* ws, int p, int n_experts, int hidden, int inner, uint32_t* err_out,
                            void* stream) {
  if (!ws || !err_out) return TLX_ERR_NULL;
  if (!moe_shape_ok(p, n_experts, hidden, inner)) return TLX_ERR_SHAPE;
  const WsLayout w = ws_layout(p, n_experts, hidden, inner);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(err_out, static_cast<const uint8_t*>(ws) + w.err, 4, cudaMemcpyDeviceToHost, s) != cudaSuccess)
    return TLX_ERR_LAUNCH;
  return cudaStreamSynchronize(s) == cudaSuccess ? TLX_OK : TLX_ERR_LAUNCH;
}

}  // extern "C"
