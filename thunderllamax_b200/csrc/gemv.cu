// K-row dequantised GEMV over IQ3_XXS / Q6_K tiles on sm_100a.
//
// One persistent launch covers the whole matrix.  Work item = (k-segment s,
// row tile t, block bb): 16 rows x 256 weights.  Items are dealt to warps as
// contiguous ranges ("stream-K"), so every warp streams the same number of
// weight bytes +-1 chunk regardless of how tiles divide into warps.  A tile
// whose k range was split between warps (or k-segments) is finished by the last
// piece to arrive: pieces write fragment-ordered fp32 partials to the
// workspace, bump a per-tile counter, and the last arriver adds all pieces in
// fixed k order (so results are bit-identical run to run) and runs the
// epilogue.
//
// Per warp: a STAGES-deep ring of chunks in shared memory filled by
// cp.async.bulk (lane 0 issues, completion on an mbarrier with tx count).
// Per CTA: the activations of its k-segment staged once as fp16 in mma B
// fragment order.  Inner loop: decode a chunk into exact-integer fp16 A
// fragments (formats.cuh), mma.sync.m16n8k16 into fp32, scale by the block's
// fp16 d after each 256-weight block.
//
// Epilogues: STORE  y[t][row] = acc (+ residual)       (down8nw32_11 / head8v11)
//            GATEUP y[t][row] = silu(gate) * up         (ffn8v11)
//            ARGMAX per-token (max, lowest index) over all rows, reduced across
//                   CTAs by the last CTA, which can also run greedy accept
//                   (h6kam + amred36 + acc36, fused)
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <mutex>

#include "common.cuh"
#include "formats.cuh"
#include "tlx_internal.h"

namespace tlx {

enum Epi : int { EPI_STORE = 0, EPI_GATEUP = 1, EPI_ARGMAX = 2 };

// Activation image.  Per 256-weight block b and column c one 512-byte row of 64
// uint2 entries; entry (mma step m, lane quarter q) holds the 4 halves
// x[c][256b + 64q + 4m + 0..3].  The entries of steps 2j and 2j+1 of one quarter are
// adjacent, so one 16-byte load gives the B fragments of two mma steps, and the
// 64-byte groups of pair j are swapped between even and odd columns (j ^ (c & 1)):
// the two columns that one 8-lane load phase reads (tokens g and g+1) then fall in
// different bank halves.  After the whole image, 4 entries per (block, column) hold
// the Q4_K / Q5_K sub-block sums (written by the staging kernel on request).
constexpr int kImageRow = 64;                       // uint2 entries per (block, column) row
constexpr uint32_t kImageRowBytes = kImageRow * 8u;   // 512
constexpr uint32_t kSumRowBytes = 32;                 // sums of one (block, column)

__host__ __device__ __forceinline__ int image_entry(int m, int q, int col) {
  return ((((m >> 1) ^ (col & 1))) << 3) | (q << 1) | (m & 1);
}
// uint2 index of the entry holding x[c][k..k+3], k % 4 == 0
__host__ __device__ __forceinline__ int64_t image_index(int64_t k, int col, int MC) {
  const int64_t b = k >> 8;
  const int kin = static_cast<int>(k & 255), q = kin >> 6, m = (kin & 63) >> 2;
  return (b * MC + col) * kImageRow + image_entry(m, q, col);
}
// uint2 index of the sums entry of (block b, column c, quarter q) in an image of NB blocks
__host__ __device__ __forceinline__ int64_t sums_index(int64_t b, int col, int q, int NB, int MC) {
  return static_cast<int64_t>(NB) * MC * kImageRow + (b * MC + col) * 4 + q;
}

// ---- peer exchange of the sharded verify step (one process per GPU, world > 1) ----
// Every rank owns one buffer of peer_buffer_bytes(world, m, ny); base[r] is rank r's
// buffer as mapped in this process.  A rank writes its results into its OWN buffer
// with ordinary stores and announces them with one release flag per kernel in every
// rank's buffer; the consumers then read the peers' buffers over NVLink (pull).  Only
// the flags cross NVLink as stores, so no system-scope fence waits behind a stream of
// remote stores.  Layout (bytes):
//   0     epoch: steps completed on this rank (local)
//   64    arrival counter of the down kernel's CTAs (local)
//   128   arrival counter of the finish kernel's CTAs (local)
//   256   down flags [2][kMaxPeers], 16 bytes apart: rank r's partial y of the step
//         with parity p is complete in rank r's buffer once flag [p][r] == epoch + 1
//   512   key flags  [2][kMaxPeers], the same for rank r's argmax keys
//   1024  keys [2][16] u64: this rank's per-token argmax keys
//   4096  y partial [2][m][ny] fp32: this rank's down partial
// Results are double-buffered by step parity: a rank can be at most one step ahead of
// another, because every step waits for all ranks' partials and keys.
constexpr uint32_t kPeerEpoch = 0, kPeerDownCnt = 64, kPeerFinishCnt = 128, kPeerDownFlags = 256,
                   kPeerKeyFlags = 512, kPeerKeys = 1024, kPeerY = 4096;

size_t peer_buffer_bytes(int world, int m, int64_t ny) {
  if (world < 2 || world > kMaxPeers || m < 1 || m > 16 || ny < 1) return 0;
  return kPeerY + 2ull * static_cast<size_t>(m) * static_cast<size_t>(ny) * 4ull;
}

__device__ __forceinline__ uint32_t* peer_flag(uint8_t* buf, uint32_t off, uint32_t par, int src) {
  return reinterpret_cast<uint32_t*>(buf + off + (par * kMaxPeers + src) * 16u);
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// bounded wait until a peer has set *flag to v (the flag lives in this rank's own
// buffer); on timeout raise ERR_PEER_TIMEOUT and go on (the step's results are then
// not valid, but nothing hangs)
__device__ __forceinline__ bool wait_peer_flag(const uint32_t* flag, uint32_t v, uint32_t* err) {
  for (uint32_t i = 0; i < kMbarPollLimit; ++i) {
    if (ld_acquire_sys(flag) == v) return true;
    __nanosleep(64);
  }
  if (err) atomicOr(err, ERR_PEER_TIMEOUT);
  return false;
}

struct GemvParams {
  const uint8_t* w0;
  const uint8_t* w1;
  const uint32_t* grid;
  const uint2* ximg;  // fp16 activation image (image_index / sums_index)
  int M;
  int MC;
  int CG;  // columns per token (1, or 3 for fp32 activations split into fp16 parts)
  int64_t n_rows;
  int T, NB, S, Bs, Cs, J;
  void* y;
  int y_f16;  // store y as fp16 instead of fp32
  int64_t ldy;
  uint2* y_img;  // GATEUP: write gact as an fp16 activation image for the consumer GEMV
  const float* residual;
  int64_t ldr;
  float* out_max;
  int32_t* out_idx;
  uint64_t* out_keys;
  int64_t row_offset;
  const int32_t* drafts;
  int n_drafts;
  int32_t* accept_out;
  float* partials;
  uint32_t* tile_cnt;
  unsigned long long* gkey;  // [16] running per-token argmax keys (zero between launches)
  uint32_t* done_cnt;
  uint32_t* err;
  PeerParams peer;           // world <= 1: no exchange
  uint32_t fp16_magic;       // 0x64006400, passed at run time (and_or in formats.cuh)
};

__host__ __device__ constexpr bool needs_sums(int qt) { return qt == QT_Q4_K || qt == QT_Q5_K; }



// ---- shared-memory layout (same arithmetic on host and device) ----
// A warp loads each chunk into registers and hands its ring stage back at once, so
// the epilogue works on registers; only fp32 activations (CG > 1: a token's value is
// the sum of several columns) need the per-warp scratch region `epi`.
struct SmemLayout {
  uint32_t xs, sums, grid, ring, bars, best, epi, total;
};

__host__ __device__ inline SmemLayout smem_layout(int qt, int nmat, int wpc, int stages, int Bs, int MC, int CG) {
  SmemLayout L;
  uint32_t off = 0;
  L.xs = off;
  off += static_cast<uint32_t>(Bs) * static_cast<uint32_t>(MC) * kImageRowBytes;
  L.sums = off;
  if (needs_sums(qt)) off += static_cast<uint32_t>(Bs) * static_cast<uint32_t>(MC) * kSumRowBytes;
  off = (off + 127u) & ~127u;
  L.grid = off;
  if (qt == QT_IQ3_XXS) off += kGridTableBytes;
  L.ring = off;
  off += static_cast<uint32_t>(wpc) * stages * chunk_bytes(qt) * nmat;
  off = (off + 15u) & ~15u;
  L.bars = off;
  off += static_cast<uint32_t>(wpc) * stages * 8u + 8u;  // + the activation-image barrier
  L.best = off;
  off += static_cast<uint32_t>(wpc) * 16u * 8u + 128u;  // + done flag and 16 final ids
  L.epi = off;
  if (CG > 1) off += static_cast<uint32_t>(wpc) * nmat * 1024u;
  L.total = off;
  return L;
}

// warp (segment-local) whose item range contains segment-local item f
__device__ __forceinline__ int warp_of(int64_t f, int64_t Fs, int Ws) {
  return static_cast<int>(((f + 1) * Ws - 1) / Fs);
}

__device__ __forceinline__ float silu_f(float g) { return g / (1.0f + expf(-g)); }

// ---- activation staging: x[M][K] (f32 / f16 / bf16) -> fp16 image ----
__global__ void stage_image_kernel(const void* __restrict__ x, int dtype, int64_t ldx, int M, int CG, int MC, int64_t K,
                                   uint2* __restrict__ img) {
  griddep_wait();
  griddep_launch_dependents();
  const int64_t per_tok = K >> 2;
  const int64_t total = static_cast<int64_t>(M) * per_tok;
  for (int64_t gi = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; gi < total;
       gi += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int t = static_cast<int>(gi / per_tok);
    const int64_t k = (gi - t * per_tok) * 4;
    const int64_t src = t * ldx + k;
    float v[4];
    if (dtype == DT_F32) {
      const float4 f = *reinterpret_cast<const float4*>(static_cast<const float*>(x) + src);
      v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
    } else {
      const uint2 raw = *reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(x) + src);
      const uint32_t h[2] = {raw.x, raw.y};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const uint32_t bits = (h[e >> 1] >> (16 * (e & 1))) & 0xFFFFu;
        v[e] = dtype == DT_BF16 ? __uint_as_float(bits << 16)
                                : __half2float(__ushort_as_half(static_cast<unsigned short>(bits)));
      }
    }
    for (int part = 0; part < CG; ++part) {
      // CG == 3: fp32 -> hi + mid + lo fp16 parts (33 significand bits >= 24)
      float hp[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        hp[e] = __half2float(__float2half_rn(v[e]));
        v[e] -= hp[e];
      }
      const __half2 h01 = __floats2half2_rn(hp[0], hp[1]);
      const __half2 h23 = __floats2half2_rn(hp[2], hp[3]);
      img[image_index(k, t * CG + part, MC)] = make_uint2(*reinterpret_cast<const uint32_t*>(&h01),
                                                          *reinterpret_cast<const uint32_t*>(&h23));
    }
  }
}

// Per-sub-block sums of the staged activations, for Q4_K's min term: sums entry q of
// (block b, column c) = {hi(S_2q), hi(S_2q+1), lo(S_2q), lo(S_2q+1)} where S_s = sum of
// x[c][256b + 32s .. +32) over the fp16 values in the image (summed in fp32) and
// hi / lo its two-fp16 split, so the min-term mma sees S to ~2^-22.
__global__ void stage_sums_kernel(int NB, int MC, uint2* __restrict__ img) {
  griddep_wait();
  griddep_launch_dependents();
  const int64_t total = static_cast<int64_t>(NB) * MC * 4;
  for (int64_t gi = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; gi < total;
       gi += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int q = static_cast<int>(gi & 3);
    const int64_t bc = gi >> 2;
    const int col = static_cast<int>(bc % MC);
    const int64_t b = bc / MC;
    const uint2* row = img + bc * kImageRow;
    float sum[2] = {0.f, 0.f};
#pragma unroll
    for (int m = 0; m < 16; ++m) {
      const uint2 e = row[image_entry(m, q, col)];
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&e.x));
      const float2 c = __half22float2(*reinterpret_cast<const __half2*>(&e.y));
      sum[m >> 3] += (a.x + a.y) + (c.x + c.y);
    }
    const __half h0 = __float2half_rn(sum[0]), h1 = __float2half_rn(sum[1]);
    const __half l0 = __float2half_rn(sum[0] - __half2float(h0)), l1 = __float2half_rn(sum[1] - __half2float(h1));
    const __half2 hh = __halves2half2(h0, h1), ll = __halves2half2(l0, l1);
    img[sums_index(b, col, q, NB, MC)] =
        make_uint2(*reinterpret_cast<const uint32_t*>(&hh), *reinterpret_cast<const uint32_t*>(&ll));
  }
}

// ---- one chunk set (NMAT chunks of one 16-row tile and 256-weight block) ----
// load_lane copies the calling lane's part of the chunks from the ring stage into
// registers (after which the stage can be refilled); compute_lane decodes them into
// exact-integer fp16 A fragments and runs the mma steps against the image rows.
template <int QT, int NMAT>
struct LaneData;
template <int NMAT>
struct LaneData<QT_Q6_K, NMAT> {
  Q6Lane s[NMAT];
};
template <int NMAT>
struct LaneData<QT_IQ3_XXS, NMAT> {
  Iq3Lane s[NMAT];
};
template <int NMAT>
struct LaneData<QT_Q4_K, NMAT> {
  Q4Lane s;
};
template <int NMAT>
struct LaneData<QT_Q5_K, NMAT> {
  Q4Lane s;
};
template <int NMAT>
struct LaneData<QT_Q8_0, NMAT> {
  Q8Lane s;
};

template <int QT, int NMAT>
__device__ __forceinline__ void load_lane(const uint8_t* stage, int lane, uint32_t magic, LaneData<QT, NMAT>& L) {
  constexpr uint32_t CH = chunk_bytes(QT);
  if constexpr (QT == QT_Q6_K) {
#pragma unroll
    for (int a = 0; a < NMAT; ++a) q6_load(stage + a * CH, lane, L.s[a]);
  } else if constexpr (QT == QT_IQ3_XXS) {
#pragma unroll
    for (int a = 0; a < NMAT; ++a) iq3_load(stage + a * CH, lane, magic, L.s[a]);
  } else if constexpr (QT == QT_Q8_0) {
    static_assert(NMAT == 1, "Q8_0 is read by the STORE epilogue only");
    q8_load(stage, lane, L.s);
  } else {
    static_assert(NMAT == 1, "Q4_K / Q5_K are read by the STORE epilogue only");
    q4_load<QT == QT_Q5_K>(stage, lane, L.s);
  }
}

// B fragments of mma steps 2j and 2j+1 for both token groups: xE / xO are this lane's
// image row addresses (shared space) for even / odd pairs j of the current block
template <int NT>
__device__ __forceinline__ void load_b_pair(const uint32_t (&xE)[NT], const uint32_t (&xO)[NT], int j,
                                            uint4 (&b)[NT]) {
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const uint32_t addr = ((j & 1) ? xO[nt] : xE[nt]) + static_cast<uint32_t>(j) * 64u;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(b[nt].x), "=r"(b[nt].y), "=r"(b[nt].z), "=r"(b[nt].w)
                 : "r"(addr));
  }
}

template <int QT, int NT, int NMAT>
__device__ __forceinline__ void compute_lane(const LaneData<QT, NMAT>& L, const uint32_t (&xE)[NT],
                                             const uint32_t (&xO)[NT], const uint32_t (&xsum)[NT],
                                             const uint8_t* grid_lane, uint32_t magic, float (&acc)[NMAT][NT][4]) {
  float tmp[NMAT][NT][4];
#pragma unroll
  for (int a = 0; a < NMAT; ++a)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) tmp[a][nt][i] = 0.f;
  if constexpr (QT == QT_Q6_K) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      uint4 b[NT];
      load_b_pair<NT>(xE, xO, j, b);
#pragma unroll
      for (int a = 0; a < NMAT; ++a) {
        uint32_t a0[4], a1[4];
        q6_group(L.s[a], j, magic, a0, a1);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          mma16816(tmp[a][nt], a0, b[nt].x, b[nt].y);
          mma16816(tmp[a][nt], a1, b[nt].z, b[nt].w);
        }
      }
    }
#pragma unroll
    for (int a = 0; a < NMAT; ++a) {
      const float2 sc = q6_block_scale(L.s[a]);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        acc[a][nt][0] = fmaf(sc.x, tmp[a][nt][0], acc[a][nt][0]);
        acc[a][nt][1] = fmaf(sc.x, tmp[a][nt][1], acc[a][nt][1]);
        acc[a][nt][2] = fmaf(sc.y, tmp[a][nt][2], acc[a][nt][2]);
        acc[a][nt][3] = fmaf(sc.y, tmp[a][nt][3], acc[a][nt][3]);
      }
    }
  } else if constexpr (QT == QT_IQ3_XXS) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      uint4 b[NT];
      load_b_pair<NT>(xE, xO, j, b);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
#pragma unroll
        for (int a = 0; a < NMAT; ++a) {
          uint32_t af[4];
          iq3_mma(L.s[a], grid_lane, 2 * j + h, af);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
            mma16816(tmp[a][nt], af, h ? b[nt].z : b[nt].x, h ? b[nt].w : b[nt].y);
        }
      }
    }
#pragma unroll
    for (int a = 0; a < NMAT; ++a) {
      const float2 sc = iq3_block_scale(L.s[a]);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        acc[a][nt][0] = fmaf(sc.x, tmp[a][nt][0], acc[a][nt][0]);
        acc[a][nt][1] = fmaf(sc.x, tmp[a][nt][1], acc[a][nt][1]);
        acc[a][nt][2] = fmaf(sc.y, tmp[a][nt][2], acc[a][nt][2]);
        acc[a][nt][3] = fmaf(sc.y, tmp[a][nt][3], acc[a][nt][3]);
      }
    }
  } else if constexpr (QT == QT_Q8_0) {
    // the fragments are the rounded weights fp16(d q)
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      uint4 b[NT];
      load_b_pair<NT>(xE, xO, j, b);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t af[4];
        q8_mma(L.s, 2 * j + h, magic, af);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma16816(acc[0][nt], af, h ? b[nt].z : b[nt].x, h ? b[nt].w : b[nt].y);
      }
    }
  } else {
    // Q4_K / Q5_K: acc += d * sum (sc q) x  -  dmin * sum_s mn_s xsum_s
    constexpr bool Q5 = QT == QT_Q5_K;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      uint4 b[NT];
      load_b_pair<NT>(xE, xO, j, b);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t af[4];
        q4_mma<Q5>(L.s, 2 * j + h, magic, af);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma16816(tmp[0][nt], af, h ? b[nt].z : b[nt].x, h ? b[nt].w : b[nt].y);
      }
    }
    // min term: A' = the lane's mins (sub-blocks 2q, 2q+1; k' and 8 + k' alike), B' =
    // the per-sub-block sums of x in two fp16 parts (sums entry q of the block)
    float tmin[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) tmin[nt][i] = 0.f;
    const uint32_t am[4] = {L.s.mn[0], L.s.mn[1], L.s.mn[0], L.s.mn[1]};
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      uint32_t s0, s1;
      asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];\n" : "=r"(s0), "=r"(s1) : "r"(xsum[nt]));
      mma16816(tmin[nt], am, s0, s1);
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      acc[0][nt][0] = fmaf(-L.s.dmin[0], tmin[nt][0], fmaf(L.s.d[0], tmp[0][nt][0], acc[0][nt][0]));
      acc[0][nt][1] = fmaf(-L.s.dmin[0], tmin[nt][1], fmaf(L.s.d[0], tmp[0][nt][1], acc[0][nt][1]));
      acc[0][nt][2] = fmaf(-L.s.dmin[1], tmin[nt][2], fmaf(L.s.d[1], tmp[0][nt][2], acc[0][nt][2]));
      acc[0][nt][3] = fmaf(-L.s.dmin[1], tmin[nt][3], fmaf(L.s.d[1], tmp[0][nt][3], acc[0][nt][3]));
    }
  }
}

// ---- epilogue of a complete 16-row tile from the fragment registers ----
// v[a][nt][e]: lane (g, q) holds rows g (e = 0, 1) and g + 8 (e = 2, 3) of columns
// 8 nt + 2q + (e & 1); here a column is a token.
template <int NT, int NMAT, int EPI>
__device__ __forceinline__ void tile_epilogue(const GemvParams& p, int64_t t, const float (&v)[NMAT][NT][4], int lane,
                                              uint64_t (&best)[2 * NT], uint32_t par) {
  const int g = lane >> 2, q = lane & 3;
  const int64_t row0 = t * kTileRows;
  if constexpr (EPI == EPI_ARGMAX) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int col = 8 * nt + 2 * q + (e & 1);
        const int64_t row = row0 + g + 8 * (e >> 1);
        if (col < p.M && row < p.n_rows) {
          const uint64_t key = argmax_key(v[0][nt][e], static_cast<uint32_t>(p.row_offset + row));
          uint64_t& b = best[2 * nt + (e & 1)];
          b = key > b ? key : b;
        }
      }
  } else if constexpr (EPI == EPI_GATEUP) {
    float o[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[nt][e] = silu_f(v[0][nt][e]) * v[1][nt][e];
    if (p.y_img) {
      // 4 consecutive rows of one token are one entry of the consumer's image: lanes
      // g = 4i .. 4i+3 (same q) hold them, and lane g = 4i gathers and stores
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float r1 = __shfl_down_sync(0xffffffffu, o[nt][e], 4);
          const float r2 = __shfl_down_sync(0xffffffffu, o[nt][e], 8);
          const float r3 = __shfl_down_sync(0xffffffffu, o[nt][e], 12);
          const int col = 8 * nt + 2 * q + (e & 1);
          if ((g & 3) == 0 && col < p.M) {
            const __half2 h01 = __floats2half2_rn(o[nt][e], r1), h23 = __floats2half2_rn(r2, r3);
            p.y_img[image_index(row0 + g + 8 * (e >> 1), col, p.M)] =
                make_uint2(*reinterpret_cast<const uint32_t*>(&h01), *reinterpret_cast<const uint32_t*>(&h23));
          }
        }
    } else {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int col = 8 * nt + 2 * q + (e & 1);
          const int64_t row = row0 + g + 8 * (e >> 1);
          if (col < p.M && row < p.n_rows) {
            if (p.y_f16)
              static_cast<__half*>(p.y)[col * p.ldy + row] = __float2half_rn(o[nt][e]);
            else
              static_cast<float*>(p.y)[col * p.ldy + row] = o[nt][e];
          }
        }
    }
  } else if (p.peer.world > 1) {
    // sharded down projection: this rank's partial of the tile goes to its own buffer
    // (parity slot); every rank's finish kernel reads it from there
    const PeerParams& pr = p.peer;
    float* part = reinterpret_cast<float*>(pr.base[pr.rank] + kPeerY) + static_cast<int64_t>(par) * pr.m * pr.ny;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int col = 8 * nt + 2 * q + (e & 1);
        const int64_t row = row0 + g + 8 * (e >> 1);
        if (col < p.M && row < p.n_rows) part[col * pr.ny + row] = v[0][nt][e];
      }
  } else {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int col = 8 * nt + 2 * q + (e & 1);
        const int64_t row = row0 + g + 8 * (e >> 1);
        if (col < p.M && row < p.n_rows) {
          float val = v[0][nt][e];
          if (p.residual) val += p.residual[col * p.ldr + row];
          if (p.y_f16)
            static_cast<__half*>(p.y)[col * p.ldy + row] = __float2half_rn(val);
          else
            static_cast<float*>(p.y)[col * p.ldy + row] = val;
        }
      }
  }
}

// fp32 activations (CG > 1 fp16 columns per token): sum each token's columns through
// the warp's scratch, then the token-column epilogue
template <int NT, int NMAT, int EPI>
__device__ __forceinline__ void tile_finish(const GemvParams& p, int64_t t, const float (&v)[NMAT][NT][4], int lane,
                                            float* epi, uint64_t (&best)[2 * NT], uint32_t par) {
  if (p.CG == 1) {
    tile_epilogue<NT, NMAT, EPI>(p, t, v, lane, best, par);
    return;
  }
  const int g = lane >> 2, q = lane & 3;
#pragma unroll
  for (int a = 0; a < NMAT; ++a)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int col = nt * 8 + 2 * q;
      *reinterpret_cast<float2*>(epi + a * 256 + g * 16 + col) = make_float2(v[a][nt][0], v[a][nt][1]);
      *reinterpret_cast<float2*>(epi + a * 256 + (g + 8) * 16 + col) = make_float2(v[a][nt][2], v[a][nt][3]);
    }
  __syncwarp();
  float vt[NMAT][NT][4];
#pragma unroll
  for (int a = 0; a < NMAT; ++a)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int tok = 8 * nt + 2 * q + (e & 1);
        const int row = g + 8 * (e >> 1);
        float s = 0.f;
        if (tok < p.M)
          for (int c = 0; c < p.CG; ++c) s += epi[a * 256 + row * 16 + tok * p.CG + c];
        vt[a][nt][e] = s;
      }
  __syncwarp();
  tile_epilogue<NT, NMAT, EPI>(p, t, vt, lane, best, par);
}

template <int QT, int NT, int EPI, int WPC, int STAGES>
__global__ void __launch_bounds__(WPC * 32, 1) tile_gemv_kernel(const GemvParams p) {
  constexpr int NMAT = EPI == EPI_GATEUP ? 2 : 1;
  constexpr uint32_t CH = chunk_bytes(QT);
  constexpr uint32_t STAGE_BYTES = CH * NMAT;
  extern __shared__ __align__(128) uint8_t smem[];
  const SmemLayout L = smem_layout(QT, NMAT, WPC, STAGES, p.Bs, p.MC, p.CG);
  uint32_t* grid_rep = reinterpret_cast<uint32_t*>(smem + L.grid);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* ring = smem + L.ring + static_cast<uint32_t>(warp) * STAGES * STAGE_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars) + warp * STAGES;
  uint64_t* xbar = reinterpret_cast<uint64_t*>(smem + L.bars) + WPC * STAGES;
  uint64_t* wbest = reinterpret_cast<uint64_t*>(smem + L.best);
  float* epi = reinterpret_cast<float*>(smem + L.epi) + warp * NMAT * 256;

  // ---- this warp's items: a contiguous range of (tile, block) of its k-segment ----
  const int seg = blockIdx.x / p.Cs;
  const int cta_in_seg = blockIdx.x - seg * p.Cs;
  const int64_t Fs = static_cast<int64_t>(p.T) * p.Bs;
  // warps beyond the item count idle, so every partition warp owns >= 1 item
  const int Ws = static_cast<int>(Fs < static_cast<int64_t>(p.Cs) * WPC ? Fs : static_cast<int64_t>(p.Cs) * WPC);
  const int wseg = cta_in_seg * WPC + warp;
  const bool active = wseg < Ws;
  const int64_t f0 = active ? static_cast<int64_t>(wseg) * Fs / Ws : 0;
  const int64_t f1 = active ? static_cast<int64_t>(wseg + 1) * Fs / Ws : 0;
  const int n_items = static_cast<int>(f1 - f0);
  int64_t t = f0 / p.Bs;
  int bb = static_cast<int>(f0 - t * p.Bs);

  // weight copy cursor (lane 0): the items of a tile are consecutive chunks; after the
  // segment's last block the next tile of the segment starts NB - Bs chunks further
  size_t woff = (static_cast<size_t>(t) * p.NB + static_cast<size_t>(seg) * p.Bs + bb) * CH;
  int w_left = p.Bs - bb;
  const size_t tile_skip = static_cast<size_t>(p.NB - p.Bs) * CH;
  auto issue = [&](int st) {
    mbar_arrive_expect_tx(&bars[st], STAGE_BYTES);
    bulk_g2s(ring + st * STAGE_BYTES, p.w0 + woff, CH, &bars[st]);
    if constexpr (NMAT == 2) bulk_g2s(ring + st * STAGE_BYTES + CH, p.w1 + woff, CH, &bars[st]);
    woff += CH;
    if (--w_left == 0) {
      w_left = p.Bs;
      woff += tile_skip;
    }
  };
  if (lane == 0) {
#pragma unroll
    for (int st = 0; st < STAGES; ++st) mbar_init(&bars[st], 1);
    mbar_fence_init();
    for (int st = 0; st < STAGES && st < n_items; ++st) issue(st);
  }
  __syncwarp();

  if constexpr (QT == QT_IQ3_XXS) {
    // one global load per entry, then kGridCopies shared copies of its fp16 pairs
    uint2* tab = reinterpret_cast<uint2*>(grid_rep);
    if (threadIdx.x < 256) {
      const uint2 e = grid_pair_entry(__ldg(p.grid + threadIdx.x));
#pragma unroll
      for (int c = 0; c < kGridCopies; ++c) tab[threadIdx.x * kGridCopies + c] = e;
    }
  }

  // Everything above touches only weights and constants.  With programmatic
  // dependent launch it overlaps the previous kernel's tail; from here on the
  // activations, outputs and workspace of the previous kernel in the stream are
  // read or written, so wait for it to complete.
  griddep_wait();
  griddep_launch_dependents();
  // sharded step: this step's number on this rank (it selects the parity slots)
  const uint32_t ep = p.peer.world > 1 ? *reinterpret_cast<volatile uint32_t*>(p.peer.base[p.peer.rank] + kPeerEpoch)
                                       : 0u;
  const uint32_t par = ep & 1u;

  // activations of this k-segment (and their sub-block sums): bulk copies of the
  // image slices
  const uint32_t xbytes = static_cast<uint32_t>(p.Bs) * static_cast<uint32_t>(p.MC) * kImageRowBytes;
  const uint32_t sbytes = needs_sums(QT) ? static_cast<uint32_t>(p.Bs) * static_cast<uint32_t>(p.MC) * kSumRowBytes : 0u;
  if (threadIdx.x == 0) {
    mbar_init(xbar, 1);
    mbar_fence_init();
    mbar_arrive_expect_tx(xbar, xbytes + sbytes);
    const uint8_t* src = reinterpret_cast<const uint8_t*>(p.ximg) + static_cast<size_t>(seg) * xbytes;
    for (uint32_t off = 0; off < xbytes; off += 32768u)
      bulk_g2s(smem + L.xs + off, src + off, xbytes - off < 32768u ? xbytes - off : 32768u, xbar);
    if constexpr (needs_sums(QT)) {
      const uint8_t* ssrc = reinterpret_cast<const uint8_t*>(p.ximg) +
                            static_cast<size_t>(p.NB) * p.MC * kImageRowBytes + static_cast<size_t>(seg) * sbytes;
      for (uint32_t off = 0; off < sbytes; off += 32768u)
        bulk_g2s(smem + L.sums + off, ssrc + off, sbytes - off < 32768u ? sbytes - off : 32768u, xbar);
    }
  }
  __syncthreads();
  bool failed = !mbar_wait_bounded(xbar, 0, threadIdx.x == 0 ? p.err : nullptr);

  // this lane's image rows (shared addresses): tokens g and g + 8, clamped to the last
  // valid column (clamped columns only feed accumulator columns that are never read);
  // pairs j of the 64-byte groups are swapped in odd columns
  const int g = lane >> 2, q = lane & 3;
  uint32_t xE[NT], xO[NT], xS[NT];
  {
    const uint32_t xs0 = smem_u32(smem + L.xs), ss0 = smem_u32(smem + L.sums);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int col = g + 8 * nt < p.MC ? g + 8 * nt : p.MC - 1;
      const uint32_t rowb = xs0 + static_cast<uint32_t>(col) * kImageRowBytes + q * 16u;
      xE[nt] = rowb + (col & 1) * 64u;
      xO[nt] = rowb - (col & 1) * 64u;
      xS[nt] = ss0 + (static_cast<uint32_t>(col) * 4u + q) * 8u;
    }
  }
  const uint32_t blk_stride = static_cast<uint32_t>(p.MC) * kImageRowBytes;
  const uint32_t sblk_stride = static_cast<uint32_t>(p.MC) * kSumRowBytes;
  const uint8_t* grid_lane = reinterpret_cast<const uint8_t*>(grid_rep) + (lane % kGridCopies) * 8;

  const uint32_t magic = p.fp16_magic;
  uint64_t best[2 * NT];
#pragma unroll
  for (int i = 0; i < 2 * NT; ++i) best[i] = 0ull;
  int slot = 0;
  uint32_t phase = 0;
  int done = 0, fail_at = 0;
  while (done < n_items && !failed) {
    const int run = n_items - done < p.Bs - bb ? n_items - done : p.Bs - bb;   // blocks of tile t in a row
    float acc[NMAT][NT][4];
#pragma unroll
    for (int a = 0; a < NMAT; ++a)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[a][nt][i] = 0.f;
    uint32_t bE[NT], bO[NT], bS[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      bE[nt] = xE[nt] + bb * blk_stride;
      bO[nt] = xO[nt] + bb * blk_stride;
      bS[nt] = xS[nt] + bb * sblk_stride;
    }
    for (int r = 0; r < run; ++r) {
      if (!mbar_wait_bounded(&bars[slot], phase, lane == 0 ? p.err : nullptr)) {
        failed = true;
        fail_at = done + r;
        break;
      }
      LaneData<QT, NMAT> Ld;
      load_lane<QT, NMAT>(ring + slot * STAGE_BYTES, lane, magic, Ld);
      // every lane's reads of the stage are ordered before the refill (warp barrier,
      // then the generic -> async proxy fence of the issuing lane)
      __syncwarp();
      if (lane == 0 && done + r + STAGES < n_items) {
        fence_proxy_async_smem();
        issue(slot);
      }
      if (++slot == STAGES) {
        slot = 0;
        phase ^= 1u;
      }
      compute_lane<QT, NT, NMAT>(Ld, bE, bO, bS, grid_lane, magic, acc);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        bE[nt] += blk_stride;
        bO[nt] += blk_stride;
        bS[nt] += sblk_stride;
      }
    }
    if (failed) break;

    // ---- blocks [bb, bb + run) of tile t are summed ----
    const bool whole = (p.S == 1) && (bb == 0) && (run == p.Bs);
    if (whole) {
      tile_finish<NT, NMAT, EPI>(p, t, acc, lane, epi, best, par);
    } else {
      // a piece of a split tile: fragment-ordered partials, the last arriver adds all
      // pieces in fixed k order (segment, piece) and runs the epilogue
      const int64_t run0 = t * p.Bs;
      const int w_first = warp_of(run0, Fs, Ws);
      const int w_last = warp_of(run0 + p.Bs - 1, Fs, Ws);
      const int pieces = w_last - w_first + 1;
      const int my_j = wseg - w_first;
      const int total = pieces * p.S;
      const int64_t slot_stride = static_cast<int64_t>(NMAT) * NT * 4 * 32;
      float* my_slot = p.partials + ((t * p.S + seg) * p.J + my_j) * slot_stride;
#pragma unroll
      for (int a = 0; a < NMAT; ++a)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) my_slot[((a * NT + nt) * 4 + e) * 32 + lane] = acc[a][nt][e];
      __threadfence();
      __syncwarp();
      uint32_t old = 0;
      if (lane == 0) old = atomicAdd(p.tile_cnt + t, 1u);
      old = __shfl_sync(0xffffffffu, old, 0);
      if (old == static_cast<uint32_t>(total - 1)) {
        __threadfence();
        float v[NMAT][NT][4];
#pragma unroll
        for (int a = 0; a < NMAT; ++a)
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) v[a][nt][e] = 0.f;
        // slot loads are issued in batches of UB slots ahead of the in-order adds (2
        // for the two-matrix gate/up, whose 4-slot batch would spill registers)
        constexpr int VN = NMAT * NT * 4;
        constexpr int UB = VN >= 16 ? 2 : 4;
        const int n_slots = p.S * pieces;
        const int my_slot_idx = seg * pieces + my_j;
        for (int base = 0; base < n_slots; base += UB) {
          float buf[UB][VN];
#pragma unroll
          for (int u = 0; u < UB; ++u) {
            const int sj = base + u;
            if (sj < n_slots && sj != my_slot_idx) {
              const int ss = sj / pieces, jj = sj - ss * pieces;
              const float* sl = p.partials + ((t * p.S + ss) * p.J + jj) * slot_stride + lane;
#pragma unroll
              for (int e = 0; e < VN; ++e) buf[u][e] = __ldcg(sl + e * 32);
            }
          }
#pragma unroll
          for (int u = 0; u < UB; ++u) {
            const int sj = base + u;
            if (sj < n_slots) {
#pragma unroll
              for (int a = 0; a < NMAT; ++a)
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                  for (int e = 0; e < 4; ++e)
                    v[a][nt][e] += sj == my_slot_idx ? acc[a][nt][e] : buf[u][(a * NT + nt) * 4 + e];
            }
          }
        }
        tile_finish<NT, NMAT, EPI>(p, t, v, lane, epi, best, par);
        if (lane == 0) p.tile_cnt[t] = 0u;
      }
    }
    done += run;
    bb += run;
    if (bb == p.Bs) {
      bb = 0;
      ++t;
    }
  }

  if (failed) {
    // let every copy this warp issued land before the CTA can exit: items fail_at ..
    // fail_at + STAGES - 1 (those that exist) were issued and not consumed
    for (int i = fail_at; i < n_items && i < fail_at + STAGES; ++i) {
      mbar_wait_bounded(&bars[slot], phase, nullptr);
      if (++slot == STAGES) {
        slot = 0;
        phase ^= 1u;
      }
    }
  }

  if constexpr (EPI == EPI_STORE) {
    if (p.peer.world > 1) {
      // the partials of this CTA's tiles are in this rank's buffer: order them before
      // the CTA count; the last CTA makes all of them visible at system scope and
      // raises this rank's down flag (slot [par][rank]) in every rank's buffer
      const PeerParams& pr = p.peer;
      __threadfence();
      __syncthreads();
      __shared__ uint32_t s_last;
      if (threadIdx.x == 0) {
        uint32_t* cnt = reinterpret_cast<uint32_t*>(pr.base[pr.rank] + kPeerDownCnt);
        s_last = atomicAdd(cnt, 1u) == gridDim.x - 1 ? 1u : 0u;
        if (s_last) *cnt = 0u;
      }
      __syncthreads();
      // the last CTA: thread r raises the flag in rank r's buffer, all ranks at once
      // (each thread's own system-scope fence, then its release store)
      if (s_last && threadIdx.x < pr.world) {
        __threadfence_system();
        st_release_sys(peer_flag(pr.base[threadIdx.x], kPeerDownFlags, par, pr.rank), ep + 1u);
      }
    }
  }

  if constexpr (EPI == EPI_ARGMAX) {
    // per-token keys: lanes -> warp (max over g of the lanes sharing q) -> CTA (shared)
    // -> all CTAs (atomicMax on the global keys; max is order-independent, so the
    // result is deterministic)
#pragma unroll
    for (int i = 0; i < 2 * NT; ++i)
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        const uint64_t o = __shfl_xor_sync(0xffffffffu, best[i], off);
        best[i] = o > best[i] ? o : best[i];
      }
    if (g == 0) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int tok = 8 * nt + 2 * q + j;
          if (tok < 16) wbest[warp * 16 + tok] = best[2 * nt + j];
        }
    }
    __syncthreads();
    uint32_t* flag = reinterpret_cast<uint32_t*>(wbest + WPC * 16);
    if (threadIdx.x < p.M) {
      uint64_t b = 0ull;
      for (int w = 0; w < WPC; ++w) {
        const uint64_t c = wbest[w * 16 + threadIdx.x];
        b = c > b ? c : b;
      }
      if (b) atomicMax(p.gkey + threadIdx.x, static_cast<unsigned long long>(b));
      __threadfence();
    }
    const PeerParams& pr = p.peer;
    __syncthreads();
    if (threadIdx.x == 0) {
      const uint32_t old = atomicAdd(p.done_cnt, 1u);
      flag[0] = old == gridDim.x - 1 ? 1u : 0u;
    }
    __syncthreads();
    if (flag[0]) {
      // the last CTA: every other CTA's atomicMax happened before its arrival
      __threadfence();
      int32_t* idx_s = reinterpret_cast<int32_t*>(flag + 2);
      uint64_t b = 0ull;
      if (threadIdx.x < p.M) b = atomicExch(p.gkey + threadIdx.x, 0ull);  // read and re-arm for the next launch
      if (pr.world > 1) {
        // this rank's keys into its own buffer (parity slot), one release flag in every
        // rank's buffer, then the merge of all ranks' keys read from their buffers
        // (max: the same result on every rank)
        if (threadIdx.x < p.M) reinterpret_cast<uint64_t*>(pr.base[pr.rank] + kPeerKeys)[par * 16 + threadIdx.x] = b;
        __syncthreads();
        // thread r raises the flag in rank r's buffer (its own fence, then its release
        // store: all ranks at once), then waits for rank r's flag in this buffer
        if (threadIdx.x < pr.world) {
          __threadfence_system();
          st_release_sys(peer_flag(pr.base[threadIdx.x], kPeerKeyFlags, par, pr.rank), ep + 1u);
          wait_peer_flag(peer_flag(pr.base[pr.rank], kPeerKeyFlags, par, threadIdx.x), ep + 1u, p.err);
        }
        __syncthreads();
        if (threadIdx.x < p.M) {
          // every rank's key is loaded before any is compared: one NVLink round trip
          uint64_t c[kMaxPeers];
#pragma unroll
          for (int r = 0; r < kMaxPeers; ++r)
            c[r] = r < pr.world ? __ldcv(reinterpret_cast<const unsigned long long*>(pr.base[r] + kPeerKeys) + par * 16 +
                                         threadIdx.x)
                                : 0ull;
#pragma unroll
          for (int r = 0; r < kMaxPeers; ++r) b = c[r] > b ? c[r] : b;
        }
      }
      if (threadIdx.x < p.M) {
        if (p.out_max) p.out_max[threadIdx.x] = key_value(b);
        if (p.out_idx) p.out_idx[threadIdx.x] = key_index(b);
        if (p.out_keys) p.out_keys[threadIdx.x] = b;
        idx_s[threadIdx.x] = key_index(b);
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        if (p.accept_out) {
          int m = 0;
          while (m < p.n_drafts && idx_s[m] == p.drafts[m]) ++m;
          p.accept_out[0] = m;
          p.accept_out[1] = idx_s[m];
        }
        *p.done_cnt = 0u;
      }
    }
  }
}

// ---- publish a partial for the peers (the exchange half of an all-reduce) ----
// Copies this rank's partial [m][ny] (pr.residual, row stride pr.ldr) into its own
// buffer (parity slot of the step), orders it before a CTA count, and the last CTA's
// threads raise this rank's down flag in every rank's buffer, one rank each.
// peer_finish_kernel then adds the ranks' partials.  The all-reduce of a layer whose
// producer writes an ordinary buffer (the expert-parallel MoE layer).
__global__ void __launch_bounds__(256) peer_publish_kernel(const PeerParams pr) {
  griddep_wait();
  griddep_launch_dependents();
  __shared__ uint32_t s_last;
  const uint32_t ep = *reinterpret_cast<volatile uint32_t*>(pr.base[pr.rank] + kPeerEpoch);
  const uint32_t par = ep & 1u;
  const int64_t total = static_cast<int64_t>(pr.m) * pr.ny;
  float* part = reinterpret_cast<float*>(pr.base[pr.rank] + kPeerY) + par * total;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t tok = i / pr.ny, row = i - tok * pr.ny;
    part[i] = pr.residual[tok * pr.ldr + row];
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t* cnt = reinterpret_cast<uint32_t*>(pr.base[pr.rank] + kPeerDownCnt);
    s_last = atomicAdd(cnt, 1u) == gridDim.x - 1 ? 1u : 0u;
    if (s_last) *cnt = 0u;
  }
  __syncthreads();
  if (s_last && threadIdx.x < pr.world) {
    __threadfence_system();
    st_release_sys(peer_flag(pr.base[threadIdx.x], kPeerDownFlags, par, pr.rank), ep + 1u);
  }
}

// ---- end of a sharded step: y = residual + the ranks' down partials, epoch + 1 ----
// Runs after the step's down and head kernels of this rank (stream order), so the only
// waits are on the other ranks' down flags.  The partials are read from every rank's
// buffer over NVLink and added in rank order, so every rank computes the same bits.
// The last CTA to finish advances the epoch.
__global__ void __launch_bounds__(256) peer_finish_kernel(const PeerParams pr, uint32_t* err) {
  griddep_wait();
  griddep_launch_dependents();
  __shared__ uint32_t last;
  const uint32_t ep = *reinterpret_cast<volatile uint32_t*>(pr.base[pr.rank] + kPeerEpoch);
  const uint32_t par = ep & 1u;
  if (threadIdx.x < pr.world)
    wait_peer_flag(peer_flag(pr.base[pr.rank], kPeerDownFlags, par, threadIdx.x), ep + 1u, err);
  __syncthreads();
  const int64_t total = static_cast<int64_t>(pr.m) * pr.ny;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t i0 = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  const bool vec = (pr.ny & 3) == 0 && (pr.ldy & 3) == 0 && (!pr.residual || (pr.ldr & 3) == 0) &&
                   (reinterpret_cast<uintptr_t>(pr.y) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(pr.residual) & 15) == 0;
  if (vec) {
    // 16-byte loads: one NVLink read of 16 bytes per rank and 4 outputs
    for (int64_t i = i0 * 4; i < total; i += stride * 4) {
      const int64_t tok = i / pr.ny, row = i - tok * pr.ny;
      float4 s = pr.residual ? *reinterpret_cast<const float4*>(pr.residual + tok * pr.ldr + row)
                             : make_float4(0.f, 0.f, 0.f, 0.f);
      // every rank's partial is loaded before any is added: one NVLink round trip
      float4 v[kMaxPeers];
#pragma unroll
      for (int r = 0; r < kMaxPeers; ++r)
        v[r] = r < pr.world ? __ldcv(reinterpret_cast<const float4*>(pr.base[r] + kPeerY) + (par * total + i) / 4)
                            : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int r = 0; r < kMaxPeers; ++r)
        if (r < pr.world) {
          s.x += v[r].x;
          s.y += v[r].y;
          s.z += v[r].z;
          s.w += v[r].w;
        }
      *reinterpret_cast<float4*>(pr.y + tok * pr.ldy + row) = s;
    }
  } else {
    for (int64_t i = i0; i < total; i += stride) {
      const int64_t tok = i / pr.ny, row = i - tok * pr.ny;
      float s = pr.residual ? pr.residual[tok * pr.ldr + row] : 0.f;
      float v[kMaxPeers];
#pragma unroll
      for (int r = 0; r < kMaxPeers; ++r)
        v[r] = r < pr.world ? __ldcv(reinterpret_cast<const float*>(pr.base[r] + kPeerY) + par * total + i) : 0.f;
#pragma unroll
      for (int r = 0; r < kMaxPeers; ++r)
        if (r < pr.world) s += v[r];
      pr.y[tok * pr.ldy + row] = s;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t* cnt = reinterpret_cast<uint32_t*>(pr.base[pr.rank] + kPeerFinishCnt);
    last = atomicAdd(cnt, 1u) == gridDim.x - 1 ? 1u : 0u;
    if (last) {
      *cnt = 0u;
      // every CTA has read the epoch; the step is complete on this rank
      *reinterpret_cast<volatile uint32_t*>(pr.base[pr.rank] + kPeerEpoch) = ep + 1u;
    }
  }
}

// ------------------------------------------------------------------------------------
// Host side: planning, workspace layout, dispatch
// ------------------------------------------------------------------------------------
struct Plan {
  int T, NB, S, Bs, C, Cs, J, MC, CG, NT, nmat, wpc, stages;
  size_t smem;
  size_t off_cnt, off_best, off_img, off_part, ws_bytes;
};

static int sm_count() {
  static int n = 0;
  static std::once_flag once;
  std::call_once(once, [] {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  });
  return n;
}

static int smem_optin() {
  static int n = 0;
  static std::once_flag once;
  std::call_once(once, [] {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess || n <= 0)
      n = 232448;  // sm_100: 227 KB
  });
  return n;
}

static constexpr uint32_t kXsBudget = 124u * 1024u;

// warps per CTA and ring depth per (format, epilogue), sized so the verify-step
// shapes (k = 5120 with 11 rows; k = 17408 in 4 segments) fit the 227 KB
// shared-memory opt-in without splitting k further
template <int QT, int EPI>
struct Cfg;
template <> struct Cfg<QT_Q6_K, EPI_STORE> { static constexpr int WPC = 16, STAGES = 2; };
template <> struct Cfg<QT_Q6_K, EPI_ARGMAX> { static constexpr int WPC = 12, STAGES = 2; };
template <> struct Cfg<QT_Q6_K, EPI_GATEUP> { static constexpr int WPC = 8, STAGES = 2; };
template <> struct Cfg<QT_IQ3_XXS, EPI_STORE> { static constexpr int WPC = 12, STAGES = 3; };
template <> struct Cfg<QT_Q4_K, EPI_STORE> { static constexpr int WPC = 12, STAGES = 3; };
template <> struct Cfg<QT_Q5_K, EPI_STORE> { static constexpr int WPC = 12, STAGES = 3; };
template <> struct Cfg<QT_Q8_0, EPI_STORE> { static constexpr int WPC = 12, STAGES = 3; };
template <> struct Cfg<QT_Q4_K, EPI_GATEUP> { static constexpr int WPC = 8, STAGES = 2; };   // (not launched)
template <> struct Cfg<QT_Q4_K, EPI_ARGMAX> { static constexpr int WPC = 16, STAGES = 2; };  // (not launched)
template <> struct Cfg<QT_IQ3_XXS, EPI_ARGMAX> { static constexpr int WPC = 12, STAGES = 3; };
template <> struct Cfg<QT_IQ3_XXS, EPI_GATEUP> { static constexpr int WPC = 12, STAGES = 2; };

static void cfg_for(int qt, int epi, int& wpc, int& stages) {
#define TLX_CFG(Q, E)            \
  if (qt == Q && epi == E) {     \
    wpc = Cfg<Q, E>::WPC;        \
    stages = Cfg<Q, E>::STAGES;  \
    return;                      \
  }
  TLX_CFG(QT_Q6_K, EPI_STORE)
  TLX_CFG(QT_Q6_K, EPI_ARGMAX)
  TLX_CFG(QT_Q6_K, EPI_GATEUP)
  TLX_CFG(QT_IQ3_XXS, EPI_STORE)
  TLX_CFG(QT_IQ3_XXS, EPI_ARGMAX)
  TLX_CFG(QT_IQ3_XXS, EPI_GATEUP)
  TLX_CFG(QT_Q4_K, EPI_STORE)
  TLX_CFG(QT_Q5_K, EPI_STORE)
  TLX_CFG(QT_Q8_0, EPI_STORE)
#undef TLX_CFG
  wpc = 8;
  stages = 2;
}

static int cols_per_token(int x_dtype) { return x_dtype == DT_F32 ? 3 : 1; }

static int make_plan(int qt, int epi, int64_t n_rows, int64_t k, int m, int x_dtype, int max_ctas, Plan& P) {
  if (qt != QT_Q6_K && qt != QT_IQ3_XXS && qt != QT_Q4_K && qt != QT_Q5_K && qt != QT_Q8_0) return TLX_ERR_QTYPE;
  // Q4_K / Q5_K / Q8_0: plain matvecs (v, GDN qkv and o-projection rows)
  if ((qt == QT_Q4_K || qt == QT_Q5_K || qt == QT_Q8_0) && epi != EPI_STORE) return TLX_ERR_QTYPE;
  if (n_rows <= 0 || k <= 0 || (k % kQK) != 0) return TLX_ERR_SHAPE;
  if (x_dtype != DT_F32 && x_dtype != DT_F16 && x_dtype != DT_BF16 && x_dtype != DT_IMAGE) return TLX_ERR_DTYPE;
  P.CG = cols_per_token(x_dtype);
  if (m < 1 || m * P.CG > 16) return TLX_ERR_SHAPE;
  if (n_rows > (int64_t(1) << 31) - 16 || k / kQK > (1 << 20)) return TLX_ERR_SHAPE;
  P.MC = m * P.CG;
  P.NT = P.MC <= 8 ? 1 : 2;
  P.nmat = epi == EPI_GATEUP ? 2 : 1;
  cfg_for(qt, epi, P.wpc, P.stages);
  P.T = static_cast<int>((n_rows + kTileRows - 1) / kTileRows);
  P.NB = static_cast<int>(k / kQK);
  // smallest k split whose activations fit the staging budget and whose whole
  // shared-memory layout fits the device's opt-in limit
  P.S = 0;
  const uint32_t smem_limit = static_cast<uint32_t>(smem_optin());
  for (int s = 1; s <= P.NB; ++s) {
    if (P.NB % s) continue;
    const uint32_t xs = static_cast<uint32_t>(P.NB / s) * P.MC * kImageRowBytes;
    const SmemLayout Ls = smem_layout(qt, P.nmat, P.wpc, P.stages, P.NB / s, P.MC, P.CG);
    if (xs <= kXsBudget && Ls.total <= smem_limit) {
      P.S = s;
      break;
    }
  }
  if (P.S == 0) return TLX_ERR_SHAPE;
  P.Bs = P.NB / P.S;
  int ctas = max_ctas > 0 ? max_ctas : sm_count();
  P.Cs = std::max(1, ctas / P.S);
  const int64_t Fs = static_cast<int64_t>(P.T) * P.Bs;
  // no more CTAs than needed to give every warp an item (the last CTA may idle warps)
  while (P.Cs > 1 && static_cast<int64_t>(P.Cs - 1) * P.wpc >= Fs) --P.Cs;
  P.C = P.Cs * P.S;
  const int64_t weff = std::min<int64_t>(Fs, static_cast<int64_t>(P.Cs) * P.wpc);
  const int64_t per_warp = Fs / weff;
  P.J = static_cast<int>(std::min<int64_t>(P.Bs, P.Bs / std::max<int64_t>(1, per_warp) + 2));
  const SmemLayout L = smem_layout(qt, P.nmat, P.wpc, P.stages, P.Bs, P.MC, P.CG);
  P.smem = L.total;
  size_t off = 256;
  P.off_cnt = off;
  off += (static_cast<size_t>(P.T) * 4 + 255) & ~size_t(255);
  P.off_best = off;  // end of the region that must be zero before a launch
  P.off_img = off;
  if (x_dtype != DT_IMAGE) off += (static_cast<size_t>(P.NB) * P.MC * (kImageRowBytes + kSumRowBytes) + 255) & ~size_t(255);
  P.off_part = off;
  off += static_cast<size_t>(P.T) * P.S * P.J * P.nmat * P.NT * 4 * 32 * sizeof(float);
  P.ws_bytes = off;
  return TLX_OK;
}

template <int QT, int NT, int EPI>
static int launch_t(const Plan& P, const GemvParams& gp, cudaStream_t stream) {
  constexpr int WPC = Cfg<QT, EPI>::WPC, STAGES = Cfg<QT, EPI>::STAGES;
  auto kern = tile_gemv_kernel<QT, NT, EPI, WPC, STAGES>;
  static size_t configured = 0;
  if (P.smem > configured) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(P.smem));
    if (e != cudaSuccess) return TLX_ERR_LAUNCH;
    configured = P.smem;
  }
  return launch_pdl(kern, dim3(P.C), dim3(WPC * 32), P.smem, stream, gp);
}

template <int EPI>
static int dispatch(int qt, const Plan& P, const GemvParams& gp, cudaStream_t s) {
  if constexpr (EPI == EPI_STORE) {
    if (qt == QT_Q4_K) return P.NT == 1 ? launch_t<QT_Q4_K, 1, EPI>(P, gp, s) : launch_t<QT_Q4_K, 2, EPI>(P, gp, s);
    if (qt == QT_Q5_K) return P.NT == 1 ? launch_t<QT_Q5_K, 1, EPI>(P, gp, s) : launch_t<QT_Q5_K, 2, EPI>(P, gp, s);
    if (qt == QT_Q8_0) return P.NT == 1 ? launch_t<QT_Q8_0, 1, EPI>(P, gp, s) : launch_t<QT_Q8_0, 2, EPI>(P, gp, s);
  }
  if (qt == QT_Q6_K) return P.NT == 1 ? launch_t<QT_Q6_K, 1, EPI>(P, gp, s) : launch_t<QT_Q6_K, 2, EPI>(P, gp, s);
  return P.NT == 1 ? launch_t<QT_IQ3_XXS, 1, EPI>(P, gp, s) : launch_t<QT_IQ3_XXS, 2, EPI>(P, gp, s);
}

// launch with programmatic stream serialization: the kernel may start while the
// previous kernel in the stream drains; it waits (griddepcontrol.wait) before
// touching anything that kernel produces
template <typename Kern, typename... Args>
static int launch_pdl(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, Args... args) {
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
  return cudaLaunchKernelEx(&cfg, kern, args...) == cudaSuccess ? TLX_OK : TLX_ERR_LAUNCH;
}

static bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

int peer_publish(const PeerParams& pr, cudaStream_t stream) {
  const int64_t total = static_cast<int64_t>(pr.m) * pr.ny;
  const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, 64));
  return launch_pdl(peer_publish_kernel, dim3(blocks), dim3(256), 0, stream, pr);
}

int peer_finish(const PeerParams& pr, uint32_t* err, cudaStream_t stream) {
  const int64_t total = static_cast<int64_t>(pr.m) * pr.ny;
  const int blocks = static_cast<int>(std::min<int64_t>((total / 4 + 255) / 256, 148));
  return launch_pdl(peer_finish_kernel, dim3(blocks), dim3(256), 0, stream, pr, err);
}


size_t activation_image_bytes(int m, int64_t k, int x_dtype) {
  if (m < 1 || k <= 0 || k % kQK) return 0;
  const int mc = m * cols_per_token(x_dtype);
  if (mc > 16) return 0;
  return static_cast<size_t>(k / kQK) * mc * (kImageRowBytes + kSumRowBytes);
}

static int stage_image(const void* x, int x_dtype, int64_t ldx, int m, int64_t k, void* image, bool sums,
                       cudaStream_t stream);

// the public staging entry: the image carries the Q4_K sub-block sums too, so any
// GEMV (Q4_K included) can read it
int stage_activations(const void* x, int x_dtype, int64_t ldx, int m, int64_t k, void* image, cudaStream_t stream) {
  return stage_image(x, x_dtype, ldx, m, k, image, true, stream);
}

static int stage_image(const void* x, int x_dtype, int64_t ldx, int m, int64_t k, void* image, bool sums,
                       cudaStream_t stream) {
  if (!x || !image) return TLX_ERR_NULL;
  if (x_dtype != DT_F32 && x_dtype != DT_F16 && x_dtype != DT_BF16) return TLX_ERR_DTYPE;
  if (activation_image_bytes(m, k, x_dtype) == 0) return TLX_ERR_SHAPE;
  const size_t xe = x_dtype == DT_F32 ? 4 : 2;
  if (!aligned(x, xe * 4) || ldx < k || (ldx % 4) != 0 || !aligned(image, 16)) return TLX_ERR_ALIGN;
  const int cg = cols_per_token(x_dtype);
  const int64_t groups = static_cast<int64_t>(m) * (k / 4);
  const int blocks = static_cast<int>(std::min<int64_t>((groups + 255) / 256, 4096));
  int rc = launch_pdl(stage_image_kernel, dim3(blocks), dim3(256), 0, stream, x, x_dtype, ldx, m, cg, m * cg, k,
                      static_cast<uint2*>(image));
  if (rc || !sums) return rc;
  const int nb = static_cast<int>(k / kQK);
  const int64_t items = static_cast<int64_t>(nb) * m * cg * 4;
  return launch_pdl(stage_sums_kernel, dim3(static_cast<unsigned>(std::min<int64_t>((items + 255) / 256, 1024))),
                    dim3(256), 0, stream, nb, m * cg, static_cast<uint2*>(image));
}

int run_gemv(int epi, int qt, const void* w0, const void* w1, const uint32_t* grid, const void* x, int x_dtype,
             int64_t ldx, int m, int64_t n_rows, int64_t k, const float* residual, int64_t ldr, void* y,
             int y_dtype, int64_t ldy, int64_t row_offset, float* out_max, int32_t* out_idx, uint64_t* out_keys,
             const int32_t* drafts, int n_drafts, int32_t* accept_out, void* ws, size_t ws_bytes, int max_ctas,
             cudaStream_t stream, const PeerParams* peer) {
  Plan P;
  int rc = make_plan(qt, epi, n_rows, k, m, x_dtype, max_ctas, P);
  if (rc) return rc;
  if (!w0 || !x || !ws) return TLX_ERR_NULL;
  if (epi == EPI_GATEUP && !w1) return TLX_ERR_NULL;
  if (qt == QT_IQ3_XXS && !grid) return TLX_ERR_NULL;
  if (epi != EPI_ARGMAX && !y && !(peer && epi == EPI_STORE)) return TLX_ERR_NULL;
  if (epi == EPI_STORE && y_dtype != DT_F32 && y_dtype != DT_F16) return TLX_ERR_DTYPE;
  if (epi == EPI_GATEUP && y_dtype != DT_F32 && y_dtype != DT_F16 && y_dtype != DT_IMAGE) return TLX_ERR_DTYPE;
  if (epi == EPI_GATEUP && y_dtype == DT_IMAGE && (n_rows % kQK) != 0) return TLX_ERR_SHAPE;
  if (ws_bytes < P.ws_bytes) return TLX_ERR_WORKSPACE;
  if (!aligned(w0, 16) || (w1 && !aligned(w1, 16)) || !aligned(ws, 256)) return TLX_ERR_ALIGN;
  if (x_dtype == DT_IMAGE) {
    if (!aligned(x, 16)) return TLX_ERR_ALIGN;
  } else {
    const size_t xe = x_dtype == DT_F32 ? 4 : 2;
    if (!aligned(x, xe * 4) || ldx < k || (ldx % 4) != 0) return TLX_ERR_ALIGN;
  }
  if (epi != EPI_ARGMAX && y_dtype != DT_IMAGE && ldy < n_rows) return TLX_ERR_SHAPE;
  if (epi == EPI_GATEUP && y_dtype == DT_IMAGE && !aligned(y, 16)) return TLX_ERR_ALIGN;
  if (residual && ldr < n_rows) return TLX_ERR_SHAPE;
  if (epi == EPI_ARGMAX && accept_out && (!drafts || n_drafts < 0 || n_drafts + 1 > m)) return TLX_ERR_SHAPE;
  if (epi == EPI_ARGMAX && (row_offset < 0 || row_offset + n_rows > (int64_t(1) << 32) - 1)) return TLX_ERR_SHAPE;
  if (peer) {
    // sharded step: the down projection (STORE, fp32 partial, no residual) or the head
    if (epi == EPI_GATEUP || peer->world < 2 || peer->world > kMaxPeers || peer->rank < 0 ||
        peer->rank >= peer->world || peer->m != m || peer->ny < 1 || (epi == EPI_ARGMAX && m > 16))
      return TLX_ERR_SHAPE;
    for (int r = 0; r < peer->world; ++r)
      if (!peer->base[r] || !aligned(peer->base[r], 256)) return TLX_ERR_ALIGN;
    if (epi == EPI_STORE && (peer->ny != n_rows || residual || y_dtype != DT_F32)) return TLX_ERR_SHAPE;

  }

  uint8_t* wsb = static_cast<uint8_t*>(ws);
  const uint2* ximg = static_cast<const uint2*>(x);
  if (x_dtype != DT_IMAGE) {
    rc = stage_image(x, x_dtype, ldx, m, k, wsb + P.off_img, qt == QT_Q4_K || qt == QT_Q5_K, stream);
    if (rc) return rc;
    ximg = reinterpret_cast<const uint2*>(wsb + P.off_img);
  }

  GemvParams gp{};
  gp.w0 = static_cast<const uint8_t*>(w0);
  gp.w1 = static_cast<const uint8_t*>(w1);
  gp.grid = grid;
  gp.ximg = ximg;
  gp.M = m;
  gp.MC = P.MC;
  gp.CG = P.CG;
  gp.n_rows = n_rows;
  gp.T = P.T;
  gp.NB = P.NB;
  gp.S = P.S;
  gp.Bs = P.Bs;
  gp.Cs = P.Cs;
  gp.J = P.J;
  gp.y = y_dtype == DT_IMAGE ? nullptr : y;
  gp.y_f16 = y_dtype == DT_F16 ? 1 : 0;
  gp.ldy = ldy;
  gp.y_img = y_dtype == DT_IMAGE ? static_cast<uint2*>(y) : nullptr;
  gp.residual = residual;
  gp.ldr = ldr;
  gp.out_max = out_max;
  gp.out_idx = out_idx;
  gp.out_keys = out_keys;
  gp.row_offset = row_offset;
  gp.drafts = drafts;
  gp.n_drafts = n_drafts;
  gp.accept_out = accept_out;
  gp.fp16_magic = kMagic;
  gp.err = reinterpret_cast<uint32_t*>(wsb);
  gp.done_cnt = reinterpret_cast<uint32_t*>(wsb + 4);
  gp.tile_cnt = reinterpret_cast<uint32_t*>(wsb + P.off_cnt);
  gp.gkey = reinterpret_cast<unsigned long long*>(wsb + 8);
  gp.partials = reinterpret_cast<float*>(wsb + P.off_part);
  if (peer) gp.peer = *peer;
  if (epi == EPI_STORE) return dispatch<EPI_STORE>(qt, P, gp, stream);
  if (epi == EPI_GATEUP) return dispatch<EPI_GATEUP>(qt, P, gp, stream);
  return dispatch<EPI_ARGMAX>(qt, P, gp, stream);
}

// ---- projections over one staged x: aq3k8v11 (q / k IQ3_XXS, v Q4_K) and q5g8v11
// (qkv Q5_K, gate IQ3_XXS).  Workspace: [image][ws of projection 0][ws 1]..., each
// region 256-byte aligned.
//
// The projections run side by side: after the staging kernel the stream forks into
// one side stream per projection (event record / wait, so a CUDA graph capture
// turns them into parallel branches) and joins again.  Each GEMV gets a share of
// the CTA budget in proportion to the rows it decodes (the GEMVs are bound by
// decode and issue, not by bytes; Q4_K rows count 1.47 times), so the small ones
// no longer pay a full-grid launch of their own one after the other.
static size_t al256(size_t n) { return (n + 255) & ~size_t(255); }

static int projection_ctas(int n, const Projection* pr, int64_t k, int max_ctas, int i) {
  const int total = max_ctas > 0 ? max_ctas : sm_count();
  if (n <= 1) return total;
  double all = 0.0, mine = 0.0;
  for (int j = 0; j < n; ++j) {
    // cost in IQ3_XXS-row equivalents (same k for all); the Q4_K factor is its byte
    // ratio to IQ3_XXS (144 / 98), which measured best for the 1024-row v projection
    const double b = static_cast<double>(pr[j].n_rows) * (pr[j].qt == QT_Q4_K ? 144.0 / 98.0 : 1.0);
    all += b;
    if (j == i) mine = b;
  }
  const int c = all > 0.0 ? static_cast<int>(total * mine / all) : 1;
  return std::max(1, std::min(total, c));
}

namespace {
constexpr int kMaxDevices = 16;
struct SideStreams {
  bool ok = false;
  cudaStream_t s[kMaxProjections];
  cudaEvent_t fork, join[kMaxProjections];
};
std::mutex g_side_mu;   // one fork / join sequence at a time (the events are shared)
SideStreams g_side[kMaxDevices];
std::once_flag g_side_once[kMaxDevices];

// this device's side streams, created on first use; nullptr if that failed (the
// projections then run one after the other on the caller's stream)
SideStreams* side_streams() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  SideStreams& ss = g_side[dev];
  std::call_once(g_side_once[dev], [&ss] {
    bool ok = cudaEventCreateWithFlags(&ss.fork, cudaEventDisableTiming) == cudaSuccess;
    for (int i = 0; i < kMaxProjections && ok; ++i)
      ok = cudaStreamCreateWithFlags(&ss.s[i], cudaStreamNonBlocking) == cudaSuccess &&
           cudaEventCreateWithFlags(&ss.join[i], cudaEventDisableTiming) == cudaSuccess;
    ss.ok = ok;
  });
  return ss.ok ? &ss : nullptr;
}
}  // namespace

size_t projections_workspace_bytes(int n, const Projection* pr, int m, int64_t k, int x_dtype, int max_ctas) {
  if (x_dtype != DT_F16 && x_dtype != DT_BF16) return 0;
  if (n < 1 || n > kMaxProjections) return 0;
  const size_t img = activation_image_bytes(m, k, x_dtype);
  if (!img) return 0;
  size_t total = al256(img);
  for (int i = 0; i < n; ++i) {
    const size_t w =
        gemv_workspace_bytes(EPI_STORE, pr[i].qt, pr[i].n_rows, k, m, DT_IMAGE, projection_ctas(n, pr, k, max_ctas, i));
    if (!w) return 0;
    total += al256(w);
  }
  return total;
}

int run_projections(int n, const Projection* pr, const uint32_t* grid, const void* x, int x_dtype, int64_t ldx, int m,
                    int64_t k, void* ws, size_t ws_bytes, int max_ctas, cudaStream_t stream) {
  if (!x || !ws) return TLX_ERR_NULL;
  for (int i = 0; i < n; ++i) {
    if (!pr[i].w || !pr[i].out) return TLX_ERR_NULL;
    if (pr[i].qt == QT_IQ3_XXS && !grid) return TLX_ERR_NULL;
  }
  if (x_dtype != DT_F16 && x_dtype != DT_BF16) return TLX_ERR_DTYPE;
  const size_t need = projections_workspace_bytes(n, pr, m, k, x_dtype, max_ctas);
  if (need == 0) return TLX_ERR_SHAPE;
  if (ws_bytes < need) return TLX_ERR_WORKSPACE;
  if (!aligned(ws, 256)) return TLX_ERR_ALIGN;
  bool sums = false;
  for (int i = 0; i < n; ++i) sums = sums || pr[i].qt == QT_Q4_K || pr[i].qt == QT_Q5_K;
  uint8_t* img = static_cast<uint8_t*>(ws);
  uint8_t* p = img + al256(activation_image_bytes(m, k, x_dtype));
  // x staged once (with the sub-block sums when a K-quant reads it); every
  // projection reads the image
  int rc = stage_image(x, x_dtype, ldx, m, k, img, sums, stream);
  if (rc) return rc;
  SideStreams* ss = n > 1 ? side_streams() : nullptr;
  std::unique_lock<std::mutex> lock(g_side_mu, std::defer_lock);
  if (ss) {
    lock.lock();
    if (cudaEventRecord(ss->fork, stream) != cudaSuccess) return TLX_ERR_LAUNCH;
  }
  for (int i = 0; i < n; ++i) {
    const int ctas = projection_ctas(n, pr, k, max_ctas, i);
    const size_t b = al256(gemv_workspace_bytes(EPI_STORE, pr[i].qt, pr[i].n_rows, k, m, DT_IMAGE, ctas));
    cudaStream_t st = stream;
    if (ss) {
      st = ss->s[i];
      if (cudaStreamWaitEvent(st, ss->fork, 0) != cudaSuccess) return TLX_ERR_LAUNCH;
    }
    rc = run_gemv(EPI_STORE, pr[i].qt, pr[i].w, nullptr, pr[i].qt == QT_IQ3_XXS ? grid : nullptr, img, DT_IMAGE, 0, m,
                  pr[i].n_rows, k, nullptr, 0, pr[i].out, DT_F16, pr[i].n_rows, 0, nullptr, nullptr, nullptr, nullptr,
                  0, nullptr, p, b, ctas, st);
    if (ss && (cudaEventRecord(ss->join[i], st) != cudaSuccess || cudaStreamWaitEvent(stream, ss->join[i], 0) != cudaSuccess))
      return TLX_ERR_LAUNCH;   // joined even after a failed launch, so no side branch is left open
    if (rc) return rc;
    p += b;
  }
  return TLX_OK;
}

// the projections' error words in their workspace (OR over the projections)
int projections_error(const void* ws, int n, const Projection* pr, int m, int64_t k, int x_dtype, int max_ctas,
                      uint32_t* err_out) {
  if (!ws || !err_out) return TLX_ERR_NULL;
  if (projections_workspace_bytes(n, pr, m, k, x_dtype, max_ctas) == 0) return TLX_ERR_SHAPE;
  const uint8_t* p = static_cast<const uint8_t*>(ws) + al256(activation_image_bytes(m, k, x_dtype));
  uint32_t e = 0;
  for (int i = 0; i < n; ++i) {
    uint32_t ei = 0;
    if (cudaMemcpy(&ei, p, 4, cudaMemcpyDeviceToHost) != cudaSuccess) return TLX_ERR_LAUNCH;
    e |= ei;
    p += al256(gemv_workspace_bytes(EPI_STORE, pr[i].qt, pr[i].n_rows, k, m, DT_IMAGE, projection_ctas(n, pr, k, max_ctas, i)));
  }
  *err_out = e;
  return TLX_OK;
}

size_t gemv_workspace_bytes(int epi, int qt, int64_t n_rows, int64_t k, int m, int x_dtype, int max_ctas) {
  Plan P;
  if (make_plan(qt, epi, n_rows, k, m, x_dtype, max_ctas, P)) return 0;
  return P.ws_bytes;
}

// bytes at the front of the workspace that must be zero before a launch (error
// word, done counter, per-tile arrival counters); the rest is written before read
size_t gemv_counter_bytes(int epi, int qt, int64_t n_rows, int64_t k, int m, int x_dtype, int max_ctas) {
  Plan P;
  if (make_plan(qt, epi, n_rows, k, m, x_dtype, max_ctas, P)) return 0;
  return P.off_best;
}

int gemv_plan_info(int epi, int qt, int64_t n_rows, int64_t k, int m, int x_dtype, int max_ctas, int32_t* info,
                   int n_info) {
  Plan P;
  int rc = make_plan(qt, epi, n_rows, k, m, x_dtype, max_ctas, P);
  if (rc) return rc;
  const int32_t v[] = {P.T, P.NB, P.S, P.Bs, P.C, P.Cs, P.J, P.MC, P.NT, P.wpc, P.stages, static_cast<int32_t>(P.smem)};
  for (int i = 0; i < n_info && i < static_cast<int>(sizeof(v) / sizeof(v[0])); ++i) info[i] = v[i];
  return TLX_OK;
}

}  // namespace tlx
