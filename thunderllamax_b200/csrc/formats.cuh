// B200 tile layouts for IQ3_XXS and Q6_K weights, and their device decoders.
//
// Rows are grouped in tiles of 16 (the M of one mma.sync.m16n8k16).  For tile t
// and 256-weight block b the layout holds one contiguous CHUNK of
// 16 * block_bytes bytes (IQ3_XXS: 16*98 = 1568, Q6_K: 16*210 = 3360), so the
// HBM footprint equals the GGUF footprint exactly and every chunk starts on a
// 16-byte boundary (chunk-major: offset (t*NB + b) * chunk_bytes).  Inside a
// chunk the bytes are permuted (and, for the Q6_K sub-scales, XOR-biased) so
// that lane l = 4g + q of a warp reads everything it needs with conflict-free
// 16-byte shared-memory loads and dequantises straight into the A fragment of
// mma.m16n8k16: rows g and g+8, block-local k in [64q, 64q+64).
//
// The k order inside an mma is free (a dot product is invariant under a
// consistent permutation of k), so every mma m (0..15) of lane quarter q takes
// weights k = 64q + 4m + {0,1,2,3} and the activations are staged to match:
// B fragment of (lane quarter q, mma m, token t) = x[t][256b + 64q + 4m + 0..3].
//
// Exactness: both decoders produce fp16 values that are exact small integers
// (IQ3_XXS: +-grid * (2s+1) <= 1922; Q6_K: (q-32) * sc, exact whenever
// |(q-32)*sc| <= 2048, i.e. always for |sc| <= 64; larger integer products are
// rounded to even, <= 2^-11 relative) and the remaining per-block
// scale (d/4 resp. d) is applied to the fp32 mma result, so products and sums
// are fp32-accurate.  References: the IQ3_XXS lane math of
// engine/ffn8v11.cu:103-116 and the Q6_K lane math of engine/aq6k8v11.cu:96-118 /
// engine/mm/MM_P6_h6kam.cu:45-56.
#pragma once
#include <cstdint>
#include <cstring>

#include "common.cuh"

namespace tlx {

enum QType : int { QT_Q8_0 = 8, QT_Q4_K = 12, QT_Q5_K = 13, QT_Q6_K = 14, QT_IQ3_XXS = 18, QT_IQ4_XS = 23 };

constexpr int kTileRows = 16;
constexpr int kQK = 256;
constexpr uint32_t kChunkQ6 = 16 * 210;     // 3360
constexpr uint32_t kChunkIq3 = 16 * 98;     // 1568
constexpr uint32_t kChunkIq4 = 16 * 136;    // 2176
constexpr uint32_t kChunkQ4 = 16 * 144;     // 2304
constexpr uint32_t kChunkQ5 = 16 * 176;     // 2816
constexpr uint32_t kChunkQ8 = 16 * 272;     // 4352

// bytes of one 256-weight group of a row in GGUF order (Q8_0: eight 34-byte blocks)
__host__ __device__ constexpr uint32_t block_bytes(int qt) {
  return qt == QT_Q6_K     ? 210u
         : qt == QT_IQ4_XS ? 136u
         : qt == QT_Q4_K   ? 144u
         : qt == QT_Q5_K   ? 176u
         : qt == QT_Q8_0   ? 272u
                           : 98u;
}
__host__ __device__ constexpr uint32_t chunk_bytes(int qt) { return 16u * block_bytes(qt); }

// ------------------------------------------------------------------------------------
// Host packers (plain C++; also used by the C-ABI tlx_pack_tiles).
// ------------------------------------------------------------------------------------

#if defined(__CUDACC__)
#define TLX_HD __host__ __device__
#else
#define TLX_HD
#endif

// 6-bit Q6_K quant of block-local weight i (0..255) of a GGUF block
TLX_HD inline uint32_t q6_value(const uint8_t* blk, int i) {
  const int h = i >> 7, j = (i >> 5) & 3, l = i & 31;
  const uint32_t lo = (blk[64 * h + 32 * (j & 1) + l] >> (4 * (j >> 1))) & 15u;
  const uint32_t hi = (blk[128 + 32 * h + l] >> (2 * j)) & 3u;
  return lo | (hi << 4);
}

// Q6_K chunk, the part owned by one lane: rows[r] = r-th row's GGUF block b
// (nullptr = zero row, stored as q = 32, sc = 0, d = 0)
TLX_HD inline void pack_q6_lane(const uint8_t* const rows[16], int lane, uint8_t* out) {
  const int g = lane >> 2, q = lane & 3;
  for (int gam = 0; gam < 8; ++gam) {
    uint32_t P[8][2];  // pair P -> (u, v)
    for (int p = 0; p < 8; ++p) {
      const int mu = p >> 2, r = p & 3;
      const int m = 2 * gam + mu;
      const uint8_t* blk = rows[g + 8 * (r & 1)];
      const int k = 64 * q + 4 * m + 2 * (r >> 1);
      P[p][0] = blk ? q6_value(blk, k) : 32u;
      P[p][1] = blk ? q6_value(blk, k + 1) : 32u;
    }
    // per half: field A at bits 4-9 (in place), field B at bits 10-15, spare bits 0-3
    uint32_t w[3];
    w[0] = (P[0][0] << 4) | (P[1][0] << 10) | (P[6][0] & 15u) | (P[0][1] << 20) | (P[1][1] << 26) |
           ((P[6][1] & 15u) << 16);
    w[1] = (P[2][0] << 4) | (P[3][0] << 10) | (P[7][0] & 15u) | (P[2][1] << 20) | (P[3][1] << 26) |
           ((P[7][1] & 15u) << 16);
    w[2] = (P[4][0] << 4) | (P[5][0] << 10) | (P[6][0] >> 4) | ((P[7][0] >> 4) << 2) | (P[4][1] << 20) |
           (P[5][1] << 26) | ((P[6][1] >> 4) << 16) | ((P[7][1] >> 4) << 18);
    for (int i3 = 0; i3 < 3; ++i3) {
      const int i = 3 * gam + i3;
      uint8_t* dst = out + ((i >> 2) * 32 + lane) * 16 + (i & 3) * 4;
      for (int bt = 0; bt < 4; ++bt) dst[bt] = static_cast<uint8_t>(w[i3] >> (8 * bt));
    }
  }
  for (int j = 0; j < 4; ++j)
    for (int rr = 0; rr < 2; ++rr) {
      const uint8_t* blk = rows[g + 8 * rr];
      const uint8_t sc = blk ? blk[192 + 4 * q + j] : 0;
      out[3072 + lane * 8 + j * 2 + rr] = static_cast<uint8_t>(sc ^ 0x80u);
    }
  if (q == 0)
    for (int rr = 0; rr < 2; ++rr) {
      const uint8_t* blk = rows[g + 8 * rr];
      out[3328 + g * 4 + rr * 2 + 0] = blk ? blk[208] : 0;
      out[3328 + g * 4 + rr * 2 + 1] = blk ? blk[209] : 0;
    }
}

// IQ3_XXS sign / scale word of one 32-weight sub-block, stored in pair order.  GGUF
// holds four 7-bit sign fields (field l: the signs of weights 8l .. 8l+6 of the
// sub-block; weight 8l+7 takes the field's parity) and the 4-bit scale at bits
// 28..31.  The tile word puts the even-weight sign of pair i (weights 8l+2i, 8l+2i+1)
// of field l at bit 4l + i and the odd-weight sign at bit 16 + 4l + i, so the fp16x2
// sign mask of a pair is ONE shift, (w << (15 - 4l - i)) & 0x80008000, and the four
// parities are computed for all fields at once.  The odd sign of pair 3 (the parity)
// is not stored: its slots 19 + 4j hold scale bit j.  32 bits, as in GGUF.
TLX_HD inline uint32_t iq3_sign_word(uint32_t v) {
  uint32_t u = 0;
  for (int l = 0; l < 4; ++l)
    for (int b = 0; b < 7; ++b)
      u |= ((v >> (7 * l + b)) & 1u) << ((b & 1) ? 16 + 4 * l + (b >> 1) : 4 * l + (b >> 1));
  for (int j = 0; j < 4; ++j) u |= ((v >> (28 + j)) & 1u) << (19 + 4 * j);
  return u;
}
TLX_HD inline uint32_t iq3_sign_word_inverse(uint32_t u) {
  uint32_t v = 0;
  for (int l = 0; l < 4; ++l)
    for (int b = 0; b < 7; ++b)
      v |= ((u >> ((b & 1) ? 16 + 4 * l + (b >> 1) : 4 * l + (b >> 1))) & 1u) << (7 * l + b);
  for (int j = 0; j < 4; ++j) v |= ((u >> (19 + 4 * j)) & 1u) << (28 + j);
  return v;
}

// IQ3_XXS chunk (GGUF block order d | qs[64] | scales[32]), the part owned by one lane
TLX_HD inline void pack_iq3_lane(const uint8_t* const rows[16], int lane, uint8_t* out) {
  const int g = lane >> 2, q = lane & 3;
  for (int rr = 0; rr < 2; ++rr) {
    const uint8_t* blk = rows[g + 8 * rr];
    for (int c = 0; c < 2; ++c) {
      const int ib = 2 * q + c;
      for (int j = 0; j < 8; ++j) out[rr * 512 + lane * 16 + c * 8 + j] = blk ? blk[2 + 8 * ib + j] : 0;
      uint32_t v = 0;
      if (blk)
        for (int j = 0; j < 4; ++j) v |= static_cast<uint32_t>(blk[66 + 4 * ib + j]) << (8 * j);
      const uint32_t u = iq3_sign_word(v);
      for (int j = 0; j < 4; ++j) out[1024 + lane * 16 + (rr * 2 + c) * 4 + j] = static_cast<uint8_t>(u >> (8 * j));
    }
  }
  if (q == 0)
    for (int rr = 0; rr < 2; ++rr) {
      const uint8_t* blk = rows[g + 8 * rr];
      out[1536 + g * 4 + rr * 2 + 0] = blk ? blk[0] : 0;
      out[1536 + g * 4 + rr * 2 + 1] = blk ? blk[1] : 0;
    }
}

// IQ4_XS chunk (GGUF block d f16 | scales_h u16 | scales_l[4] | qs[128]; the MoE
// expert weights).  Lane l = 4g + q owns sub-blocks 2q and 2q+1 of rows g and g+8,
// i.e. the 32 contiguous bytes qs[32q .. 32q+32) of each row, stored as four
// 16-byte units u = 2*rr + half at (u*32 + l)*16 (rr 0: row g, 1: row g+8), so each
// of the lane's four 16-byte loads is one contiguous 512-byte warp access.  The
// 8-byte block headers follow at 2048 + 16g (row g) and 2048 + 16g + 8 (row g+8),
// one 16-byte load for the four lanes of g.  Zero rows are all-zero (d = 0).
TLX_HD inline void pack_iq4_lane(const uint8_t* const rows[16], int lane, uint8_t* out) {
  const int g = lane >> 2, q = lane & 3;
  for (int rr = 0; rr < 2; ++rr) {
    const uint8_t* blk = rows[g + 8 * rr];
    for (int hf = 0; hf < 2; ++hf)
      for (int j = 0; j < 16; ++j)
        out[((2 * rr + hf) * 32 + lane) * 16 + j] = blk ? blk[8 + 32 * q + 16 * hf + j] : 0;
  }
  if (q == 0)
    for (int rr = 0; rr < 2; ++rr) {
      const uint8_t* blk = rows[g + 8 * rr];
      for (int i = 0; i < 8; ++i) out[2048 + g * 16 + rr * 8 + i] = blk ? blk[i] : 0;
    }
}

// Q4_K chunk (GGUF block d f16 | dmin f16 | scales[12] | qs[128]; the v rows of the
// attention projection).  Lane l = 4g + q owns sub-blocks 2q (low nibbles) and 2q+1
// (high nibbles) of rows g and g+8: the 32 bytes qs[32q .. 32q+32) of each row,
// stored as four 16-byte units u = 2*rr + half at (u*32 + l)*16 (the IQ4_XS lane
// placement).  Row r's 16-byte block header (d, dmin, the 12 packed scale/min
// bytes) follows at 2048 + 16r.  Zero rows are all-zero (d = dmin = 0).
TLX_HD inline void pack_q4k_lane(const uint8_t* const rows[16], int lane, uint8_t* out) {
  const int g = lane >> 2, q = lane & 3;
  for (int rr = 0; rr < 2; ++rr) {
    const uint8_t* blk = rows[g + 8 * rr];
    for (int hf = 0; hf < 2; ++hf)
      for (int j = 0; j < 16; ++j)
        out[((2 * rr + hf) * 32 + lane) * 16 + j] = blk ? blk[16 + 32 * q + 16 * hf + j] : 0;
  }
  if (q == 0)
    for (int rr = 0; rr < 2; ++rr) {
      const uint8_t* blk = rows[g + 8 * rr];
      for (int i = 0; i < 16; ++i) out[2048 + (g + 8 * rr) * 16 + i] = blk ? blk[i] : 0;
    }
}

// Q5_K chunk (GGUF block d f16 | dmin f16 | scales[12] | qh[32] | qs[128]; the GDN
// qkv rows).  The qs units are placed as in the Q4_K chunk (lane l = 4g + q: the 32
// bytes qs[32q .. 32q+32) of rows g and g+8 at ((2*rr + half)*32 + l)*16).  The fifth
// bits of the lane's weights, bit 2q (sub-block 2q, low nibbles) and bit 2q+1
// (sub-block 2q+1, high nibbles) of qh[e] for e = 0..31, are regrouped per 4-weight
// word i (e = 4i + j): one byte per (row, i) at 2048 + l*16 + rr*8 + i with bits
//   0: lo(j=1)  1: lo(3)  2: hi(1)  3: hi(3)  4: lo(0)  5: lo(2)  6: hi(0)  7: hi(2),
// the order in which q5_mma spreads them to the fp16 halves (a multiply by
// 0x00100001 and three shifts).  Row r's 16-byte header (d, dmin, scales) follows
// at 2560 + 16r.  Zero rows are all-zero.
TLX_HD inline uint8_t q5_hbyte(const uint8_t* qh, int q, int i) {
  auto lo = [&](int j) { return static_cast<uint32_t>((qh[4 * i + j] >> (2 * q)) & 1u); };
  auto hi = [&](int j) { return static_cast<uint32_t>((qh[4 * i + j] >> (2 * q + 1)) & 1u); };
  return static_cast<uint8_t>(lo(1) | lo(3) << 1 | hi(1) << 2 | hi(3) << 3 | lo(0) << 4 | lo(2) << 5 | hi(0) << 6 |
                              hi(2) << 7);
}

TLX_HD inline void pack_q5k_lane(const uint8_t* const rows[16], int lane, uint8_t* out) {
  const int g = lane >> 2, q = lane & 3;
  for (int rr = 0; rr < 2; ++rr) {
    const uint8_t* blk = rows[g + 8 * rr];
    for (int hf = 0; hf < 2; ++hf)
      for (int j = 0; j < 16; ++j)
        out[((2 * rr + hf) * 32 + lane) * 16 + j] = blk ? blk[48 + 32 * q + 16 * hf + j] : 0;
    for (int i = 0; i < 8; ++i) out[2048 + lane * 16 + rr * 8 + i] = blk ? q5_hbyte(blk + 16, q, i) : 0;
  }
  if (q == 0)
    for (int rr = 0; rr < 2; ++rr) {
      const uint8_t* blk = rows[g + 8 * rr];
      for (int i = 0; i < 16; ++i) out[2560 + (g + 8 * rr) * 16 + i] = blk ? blk[i] : 0;
    }
}

// Q8_0 chunk: a 256-weight group of a row is eight GGUF blocks (d f16 | qs[32] int8).
// Lane l = 4g + q owns blocks 2q and 2q+1 (k in [64q, 64q+64)) of rows g and g+8: the
// 64 quants of each row as four 16-byte units u = 4*rr + j (k = 64q + 16j + 0..15) at
// (u*32 + l)*16, then the lane's four scales {d(g, 2q), d(g, 2q+1), d(g+8, 2q),
// d(g+8, 2q+1)} as one 8-byte word at 4096 + 8l.  Zero rows are all-zero.
TLX_HD inline void pack_q8_lane(const uint8_t* const rows[16], int lane, uint8_t* out) {
  const int g = lane >> 2, q = lane & 3;
  for (int rr = 0; rr < 2; ++rr) {
    const uint8_t* grp = rows[g + 8 * rr];
    for (int j = 0; j < 4; ++j)
      for (int b = 0; b < 16; ++b) {
        const int e = 16 * j + b;  // 0..63 within the lane's two blocks
        out[((4 * rr + j) * 32 + lane) * 16 + b] = grp ? grp[34 * (2 * q + (e >> 5)) + 2 + (e & 31)] : 0;
      }
    for (int c = 0; c < 2; ++c)
      for (int i = 0; i < 2; ++i) out[4096 + lane * 8 + rr * 4 + c * 2 + i] = grp ? grp[34 * (2 * q + c) + i] : 0;
  }
}

TLX_HD inline void pack_lane(int qt, const uint8_t* const rows[16], int lane, uint8_t* out) {
  if (qt == QT_Q6_K) pack_q6_lane(rows, lane, out);
  else if (qt == QT_IQ4_XS) pack_iq4_lane(rows, lane, out);
  else if (qt == QT_Q4_K) pack_q4k_lane(rows, lane, out);
  else if (qt == QT_Q5_K) pack_q5k_lane(rows, lane, out);
  else if (qt == QT_Q8_0) pack_q8_lane(rows, lane, out);
  else pack_iq3_lane(rows, lane, out);
}

// ------------------------------------------------------------------------------------
// Device decoders.  Each works on one chunk in shared memory for the calling lane.
// A fragments: a[0] = row g k+0/1, a[1] = row g+8 k+0/1, a[2] = row g k+2/3,
// a[3] = row g+8 k+2/3 (k = 64q + 4m).
// ------------------------------------------------------------------------------------
#ifdef __CUDACC__

constexpr uint32_t kMagic = 0x64006400u;      // fp16x2 (1024, 1024)
constexpr uint32_t kMinus1056 = 0xE420E420u;  // fp16x2 (-1056, -1056) = -(1024 + 32)
constexpr uint32_t kMinus1536 = 0xE600E600u;  // fp16x2 (-1536, -1536) = -(1024 + 16 * 32)
constexpr uint32_t kMinus1152 = 0xE480E480u;  // fp16x2 (-1152, -1152) = -(1024 + 128)
constexpr uint32_t kMinus1024 = 0xE400E400u;  // fp16x2 (-1024, -1024)
constexpr uint32_t kSixteenth = 0x2C002C00u;  // fp16x2 (1/16, 1/16)
constexpr uint32_t kMinus72 = 0xD480D480u;    // fp16x2 (-72, -72)

// One-LOP3 bit assembly.  LOP3 takes a single immediate, so `(w & MASK) | 0x64006400`
// with both constants compiled in costs two LOP3 per decoded register (measured: 147
// against 83 LOP3 per Q6_K chunk).  The decoders therefore take the fp16 magic
// 0x64006400 as a run-time register value (`magic`, loaded from the kernel
// parameters, so the compiler can neither fold it nor split the operation) and
// assemble each register with one lop3.b32.
template <uint32_t M>
__device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t c) {   // (a & M) | c
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "n"(M), "r"(c));
  return d;
}
template <uint32_t M>
__device__ __forceinline__ uint32_t xor_or(uint32_t a, uint32_t c) {   // (a ^ M) | c
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xBE;" : "=r"(d) : "r"(a), "n"(M), "r"(c));
  return d;
}

// Q6_K: per-block lane state.  Every 6-bit field is decoded at mantissa offset 4 of
// an fp16 half (value 1024 + 16q) and turned into (q - 32) * sc by ONE fma:
// (1024 + 16q) * (sc/16) - 96 sc.  Both constants are exact in fp16 for every
// int8 sc (96 sc = 3 * 32 * sc needs <= 9 significand bits, |96 sc| <= 12288),
// so the result is the single rounding of the exact integer (q - 32) * sc.
struct Q6Lane {
  uint32_t w[24];
  uint32_t s16[4][2];  // fp16x2 (sc/16, sc/16) for sub-block 4q+j, row g / g+8
  uint32_t c96[4][2];  // fp16x2 (-96 sc, -96 sc)
  uint32_t d;          // fp16 d of row g (lo) and row g+8 (hi)
};

constexpr uint32_t kMinus96 = 0xD600D600u;  // fp16x2 (-96, -96)

// the lane's biased sub-scale bytes -> fp16x2 (sc/16) and (-96 sc) per sub-block / row
__device__ __forceinline__ void q6_scales(const uint2 sc, Q6Lane& s) {
  // biased byte b = sc + 128 -> fp16 1024 + b
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t word = j < 2 ? sc.x : sc.y;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const uint32_t bsel = 2u * (j & 1) + r;
      // (1024 + b) / 16 - 72 = (b - 128) / 16 = sc / 16, then sc / 16 * -1536 = -96 sc:
      // every intermediate is exact in fp16
      s.s16[j][r] = hfma2_u(prmt(word, 0x64646464u, 0x4040u | (bsel << 8) | bsel), kSixteenth, kMinus72);
      s.c96[j][r] = hmul2_u(s.s16[j][r], kMinus1536);
    }
  }
}

__device__ __forceinline__ void q6_load(const uint8_t* chunk, int lane, Q6Lane& s) {
#pragma unroll
  for (int p = 0; p < 6; ++p) {
    const uint4 v = *reinterpret_cast<const uint4*>(chunk + (p * 32 + lane) * 16);
    s.w[4 * p + 0] = v.x;
    s.w[4 * p + 1] = v.y;
    s.w[4 * p + 2] = v.z;
    s.w[4 * p + 3] = v.w;
  }
  q6_scales(*reinterpret_cast<const uint2*>(chunk + 3072 + lane * 8), s);
  s.d = *reinterpret_cast<const uint32_t*>(chunk + 3328 + (lane >> 2) * 4);
}

// decode group gam (mmas 2*gam, 2*gam+1).  Per half-word the packer stores field A
// at bits 4-9 (in place), field B at bits 10-15 (moved down by 6) and spare bits
// 0-3; the split pairs P6/P7 join a low nibble from the spare bits of W0/W1 with
// two high bits from the spare bits of W2.
__device__ __forceinline__ void q6_group(const Q6Lane& s, int gam, uint32_t magic, uint32_t (&a0)[4],
                                         uint32_t (&a1)[4]) {
  const uint32_t W0 = s.w[3 * gam], W1 = s.w[3 * gam + 1], W2 = s.w[3 * gam + 2];
  const int j = gam >> 1;
  const uint32_t sg = s.s16[j][0], sg8 = s.s16[j][1];
  const uint32_t cg = s.c96[j][0], cg8 = s.c96[j][1];
  const uint32_t p0 = and_or<0x03F003F0u>(W0, magic);
  const uint32_t p1 = and_or<0x03F003F0u>(W0 >> 6, magic);
  const uint32_t p2 = and_or<0x03F003F0u>(W1, magic);
  const uint32_t p3 = and_or<0x03F003F0u>(W1 >> 6, magic);
  const uint32_t p4 = and_or<0x03F003F0u>(W2, magic);
  const uint32_t p5 = and_or<0x03F003F0u>(W2 >> 6, magic);
  const uint32_t p6 = and_or<0x00F000F0u>(W0 << 4, and_or<0x03000300u>(W2 << 8, magic));
  const uint32_t p7 = and_or<0x00F000F0u>(W1 << 4, and_or<0x03000300u>(W2 << 6, magic));
  a0[0] = hfma2_u(p0, sg, cg);
  a0[1] = hfma2_u(p1, sg8, cg8);
  a0[2] = hfma2_u(p2, sg, cg);
  a0[3] = hfma2_u(p3, sg8, cg8);
  a1[0] = hfma2_u(p4, sg, cg);
  a1[1] = hfma2_u(p5, sg8, cg8);
  a1[2] = hfma2_u(p6, sg, cg);
  a1[3] = hfma2_u(p7, sg8, cg8);
}

__device__ __forceinline__ float2 q6_block_scale(const Q6Lane& s) {
  const __half2 h = *reinterpret_cast<const __half2*>(&s.d);
  return __half22float2(h);  // (row g, row g+8)
}

// IQ3_XXS grid table in shared memory: entry e holds its 4 magnitudes as two fp16x2
// (exact small integers), replicated kGridCopies times so lane l reads copy l % 16
// (one LDS.64 per grid entry, two wavefronts per warp, no bank conflicts)
constexpr int kGridCopies = 16;
constexpr uint32_t kGridTableBytes = 256u * kGridCopies * 8u;

__device__ __forceinline__ uint2 grid_pair_entry(uint32_t g) {
  uint2 e;
  e.x = hadd2_u(prmt(g, 0x64646464u, 0x4140u), kMinus1024);
  e.y = hadd2_u(prmt(g, 0x64646464u, 0x4342u), kMinus1024);
  return e;
}

// IQ3_XXS: per-block lane state
struct Iq3Lane {
  uint4 qs0, qs1;      // grid indices: row g / row g+8, groups 2q (bytes 0..7) and 2q+1 (8..15)
  uint32_t sg[2][2];   // sign words [row][group] in pair order, parities filled in
  uint32_t m2[2][2];   // fp16x2 (2s+1)
  uint32_t d;
};

constexpr uint32_t kTwo = 0x40004000u;          // fp16x2 (2, 2)
constexpr uint32_t kMinus2047 = 0xE7FFE7FFu;    // fp16x2 (-2047, -2047)

// one stored sign / scale word (iq3_sign_word) -> the full sign word and fp16x2 (2s+1)
__device__ __forceinline__ void iq3_word(uint32_t u, uint32_t magic, uint32_t& sg, uint32_t& m2) {
  // parity of field l = xor of its 7 stored bits (4l..4l+3, 16+4l..18+4l), at bit 4l
  const uint32_t y0 = u & 0x7777FFFFu;
  uint32_t y = y0 ^ (y0 >> 16);
  y ^= y >> 2;
  y ^= y >> 1;
  sg = and_or<0x88880000u>(y << 19, y0);
  // scale bits at 19 + 4j -> s at bits 12..15 and 28..31 (one multiply gathers them;
  // every partial product lands on a bit of its own) -> fp16 1024 + s -> 2 (1024 + s) - 2047
  const uint32_t gsc = ((u >> 19) & 0x1111u) * 0x12481248u;
  m2 = hfma2_u(and_or<0x000F000Fu>(gsc >> 12, magic), kTwo, kMinus2047);
}

// the lane's four stored words [row][group]
__device__ __forceinline__ void iq3_words(const uint4 sw, uint32_t magic, Iq3Lane& s) {
  iq3_word(sw.x, magic, s.sg[0][0], s.m2[0][0]);
  iq3_word(sw.y, magic, s.sg[0][1], s.m2[0][1]);
  iq3_word(sw.z, magic, s.sg[1][0], s.m2[1][0]);
  iq3_word(sw.w, magic, s.sg[1][1], s.m2[1][1]);
}

__device__ __forceinline__ void iq3_load(const uint8_t* chunk, int lane, uint32_t magic, Iq3Lane& s) {
  s.qs0 = *reinterpret_cast<const uint4*>(chunk + lane * 16);
  s.qs1 = *reinterpret_cast<const uint4*>(chunk + 512 + lane * 16);
  iq3_words(*reinterpret_cast<const uint4*>(chunk + 1024 + lane * 16), magic, s);
  s.d = *reinterpret_cast<const uint32_t*>(chunk + 1536 + (lane >> 2) * 4);
}

// fp16x2 sign mask of pair i (0..3) of field l from a sign word in pair order
__device__ __forceinline__ uint32_t pair_signs(uint32_t sg, int l, int i) {
  return (sg << (15 - 4 * l - i)) & 0x80008000u;
}

// grid entry address: byte k of a qs word picked by one PRMT, then idx * 128 + base
__device__ __forceinline__ const uint8_t* grid_entry(const uint8_t* grid_lane, uint32_t word, int k) {
  return grid_lane + prmt(word, 0u, 0x4440u | static_cast<uint32_t>(k)) * (kGridCopies * 8u);
}

// decode mma m (0..15) for both rows; grid_lane = table base + (lane % 16) * 8 bytes
__device__ __forceinline__ void iq3_mma(const Iq3Lane& s, const uint8_t* grid_lane, int m, uint32_t (&a)[4]) {
  const int c = m >> 3, l = (m >> 1) & 3, e = m & 1;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const uint4 qs = r == 0 ? s.qs0 : s.qs1;
    const uint32_t word = (m >> 2) == 0 ? qs.x : (m >> 2) == 1 ? qs.y : (m >> 2) == 2 ? qs.z : qs.w;
    const uint2 G = *reinterpret_cast<const uint2*>(grid_entry(grid_lane, word, m & 3));
    a[r] = hmul2_u(G.x, s.m2[r][c]) ^ pair_signs(s.sg[r][c], l, 2 * e);
    a[r + 2] = hmul2_u(G.y, s.m2[r][c]) ^ pair_signs(s.sg[r][c], l, 2 * e + 1);
  }
}

__device__ __forceinline__ float2 iq3_block_scale(const Iq3Lane& s) {
  const __half2 h = *reinterpret_cast<const __half2*>(&s.d);
  const float2 f = __half22float2(h);
  return make_float2(f.x * 0.25f, f.y * 0.25f);   // d * (2s+1)/4 = (d/4) * (2s+1)
}

// Q4_K: per-block lane state.  A low nibble v is decoded as the fp16 1024 + v and a
// high nibble as 1024 + 16v (mantissa offset 4); one fma per pair then gives the
// exact integer sc * v: (1024 + v) * sc - 1024 sc, resp. (1024 + 16v) * (sc/16) -
// 64 sc (sc, mn <= 63: every constant and product is an exact fp16 integer).  The
// min term -dmin * sum_s mn_s * sum_{k in s} x_k is one more mma per block: A' holds
// the lane's mins (k' = sub-block, duplicated for the two fp16 parts of each sum),
// B' the activation image's sub-block sums (entries 64..67 of each row).
struct Q4Lane {
  uint32_t w[2][8];    // qs words of rows g / g+8 (bytes 4i .. 4i+3 of the lane's 32)
  uint2 h[2];          // Q5_K only: fifth-bit bytes of rows g / g+8 (byte i: word i)
  uint32_t slo[2], clo[2], shi[2], chi[2];  // fp16x2 fma constants per row
  uint32_t mn[2];      // fp16x2 (mn_{2q}, mn_{2q+1}) per row
  float d[2], dmin[2];
};

// 6-bit (scale, min) of sub-block j from the 12 packed bytes in words h1..h3 (bytes
// 4..15 of the block header: h1 = scales[0..3], h2 = [4..7], h3 = [8..11])
__device__ __forceinline__ void q4_scale_min(uint32_t h1, uint32_t h2, uint32_t h3, int j, uint32_t& sc,
                                             uint32_t& mn) {
  const int jj = j & 3;
  const uint32_t b0 = (h1 >> (8 * jj)) & 0xFFu;   // scales[jj]
  const uint32_t b4 = (h2 >> (8 * jj)) & 0xFFu;   // scales[jj + 4]
  const uint32_t b8 = (h3 >> (8 * jj)) & 0xFFu;   // scales[jj + 8]
  if (j < 4) {
    sc = b0 & 63u;
    mn = b4 & 63u;
  } else {
    sc = (b8 & 0xFu) | ((b0 >> 6) << 4);
    mn = (b8 >> 4) | ((b4 >> 6) << 4);
  }
}

template <bool Q5 = false>
__device__ __forceinline__ void q4_load(const uint8_t* chunk, int lane, Q4Lane& s) {
  const int g = lane >> 2, q = lane & 3;
  constexpr uint32_t kHdr = Q5 ? 2560u : 2048u;
  if constexpr (Q5) {
    const uint4 hb = *reinterpret_cast<const uint4*>(chunk + 2048 + lane * 16);
    s.h[0] = make_uint2(hb.x, hb.y);
    s.h[1] = make_uint2(hb.z, hb.w);
  }
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const uint4 v = *reinterpret_cast<const uint4*>(chunk + ((2 * rr + hf) * 32 + lane) * 16);
      s.w[rr][4 * hf + 0] = v.x;
      s.w[rr][4 * hf + 1] = v.y;
      s.w[rr][4 * hf + 2] = v.z;
      s.w[rr][4 * hf + 3] = v.w;
    }
    const uint4 h = *reinterpret_cast<const uint4*>(chunk + kHdr + (g + 8 * rr) * 16);
    const __half2 dd = *reinterpret_cast<const __half2*>(&h.x);
    s.d[rr] = __low2float(dd);
    s.dmin[rr] = __high2float(dd);
    uint32_t sc0, mn0, sc1, mn1;
    q4_scale_min(h.y, h.z, h.w, 2 * q, sc0, mn0);
    q4_scale_min(h.y, h.z, h.w, 2 * q + 1, sc1, mn1);
    const __half f0 = __uint2half_rn(sc0), f1 = __uint2half_rn(sc1);
    s.slo[rr] = h2_bits(__halves2half2(f0, f0));
    s.clo[rr] = h2_bits(__halves2half2(__float2half_rn(-1024.0f * sc0), __float2half_rn(-1024.0f * sc0)));
    s.shi[rr] = h2_bits(__halves2half2(__float2half_rn(sc1 * 0.0625f), __float2half_rn(sc1 * 0.0625f)));
    s.chi[rr] = h2_bits(__halves2half2(__float2half_rn(-64.0f * sc1), __float2half_rn(-64.0f * sc1)));
    s.mn[rr] = h2_bits(__halves2half2(__uint2half_rn(mn0), __uint2half_rn(mn1)));
  }
}

// decode mma m (0..15): k = 64q + 4m + {0..3} = element 4(m & 7) + {0..3} of
// sub-block 2q (m < 8, low nibbles) or 2q+1 (m >= 8, high nibbles).  Q5_K adds the
// fifth bit h above the nibble: 1024 + v + 16h (low) resp. 1024 + 16(v + 16h)
// (high), still exact fp16 integers below 2048, so the same fma constants apply.
template <bool Q5 = false>
__device__ __forceinline__ void q4_mma(const Q4Lane& s, int m, uint32_t magic, uint32_t (&a)[4]) {
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    const uint32_t w = s.w[rr][m & 7];
    const uint32_t p01 = prmt(w, 0u, 0x4140u);  // bytes 0, 1 -> low bytes of the halves
    const uint32_t p23 = prmt(w, 0u, 0x4342u);
    uint32_t h01 = magic, h23 = magic;   // the fifth bits (Q5_K) with the fp16 magic
    if constexpr (Q5) {
      const int i = m & 7;
      const uint32_t word = i < 4 ? s.h[rr].x : s.h[rr].y;
      const uint32_t x = ((word >> (8 * (i & 3))) & 0xFFu) * 0x00100001u;  // byte at bits 0..7 and 20..27
      if (m < 8) {
        h01 = and_or<0x00100010u>(x, magic);        // bit 4 <- lo(0), bit 20 <- lo(1)
        h23 = and_or<0x00100010u>(x >> 1, magic);   // bit 4 <- lo(2), bit 20 <- lo(3)
      } else {
        h01 = and_or<0x01000100u>(x << 2, magic);   // bit 8 <- hi(0), bit 24 <- hi(1)
        h23 = and_or<0x01000100u>(x << 1, magic);   // bit 8 <- hi(2), bit 24 <- hi(3)
      }
    }
    if (m < 8) {
      a[rr] = hfma2_u(and_or<0x000F000Fu>(p01, h01), s.slo[rr], s.clo[rr]);
      a[rr + 2] = hfma2_u(and_or<0x000F000Fu>(p23, h23), s.slo[rr], s.clo[rr]);
    } else {
      a[rr] = hfma2_u(and_or<0x00F000F0u>(p01, h01), s.shi[rr], s.chi[rr]);
      a[rr + 2] = hfma2_u(and_or<0x00F000F0u>(p23, h23), s.shi[rr], s.chi[rr]);
    }
  }
}

// Q8_0: per-block lane state.  A weight is fp16(d * q), the value the reference's
// o-projection rounds to before its half multiply (engine/k3aonw32_11.cu:100-101):
// q + 128 is placed in an fp16 mantissa (1024 + q + 128), 1152 is subtracted
// (exact), and one fp16 multiply by d rounds the exact product once.
struct Q8Lane {
  uint4 u[2][4];       // quants of rows g / g+8: unit j = k 64q + 16j + 0..15
  uint32_t d[2][2];    // fp16x2 (d, d) of block 2q + c for rows g / g+8
};

__device__ __forceinline__ void q8_load(const uint8_t* chunk, int lane, Q8Lane& s) {
#pragma unroll
  for (int rr = 0; rr < 2; ++rr)
#pragma unroll
    for (int j = 0; j < 4; ++j) s.u[rr][j] = *reinterpret_cast<const uint4*>(chunk + ((4 * rr + j) * 32 + lane) * 16);
  const uint2 dd = *reinterpret_cast<const uint2*>(chunk + 4096 + lane * 8);
  s.d[0][0] = prmt(dd.x, 0u, 0x1010u);   // d(g, 2q) in both halves
  s.d[0][1] = prmt(dd.x, 0u, 0x3232u);   // d(g, 2q+1)
  s.d[1][0] = prmt(dd.y, 0u, 0x1010u);   // d(g+8, 2q)
  s.d[1][1] = prmt(dd.y, 0u, 0x3232u);   // d(g+8, 2q+1)
}

// decode mma m (0..15): k = 64q + 4m + {0..3}, block 2q + (m >> 3)
__device__ __forceinline__ void q8_mma(const Q8Lane& s, int m, uint32_t magic, uint32_t (&a)[4]) {
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    const uint4 u = s.u[rr][m >> 2];
    const uint32_t w = (m & 3) == 0 ? u.x : (m & 3) == 1 ? u.y : (m & 3) == 2 ? u.z : u.w;
    const uint32_t p01 = xor_or<0x00800080u>(prmt(w, 0u, 0x4140u), magic);   // 1024 + q + 128
    const uint32_t p23 = xor_or<0x00800080u>(prmt(w, 0u, 0x4342u), magic);
    const uint32_t dd = s.d[rr][m >> 3];
    a[rr] = hmul2_u(hadd2_u(p01, kMinus1152), dd);
    a[rr + 2] = hmul2_u(hadd2_u(p23, kMinus1152), dd);
  }
}

#endif  // __CUDACC__

}  // namespace tlx
