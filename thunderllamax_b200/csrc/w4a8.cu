// W4A8 prefill tier: int8 tokens times IQ3_XXS weights read through a linearised
// codebook, the reference's p8q8x + p8w4ffn7 pair (engine/pfk_q8.cu:24-59,
// engine/p8_w4ffn7.cu:4-12, 118-255; wired at engine/pf_prefill.py:1155-1158).
//
// tlx_act_quant_q8 restates the token quantiser bit for bit: half a warp per (token,
// 128-k chunk), s = max(max|x|, 1e-6) * (1/127) in fp32, q = clamp(rint(x / s)),
// the chunk's integer sum.
//
// The GEMM: each weight is level * sign * sdb, sdb = d (2s+1)/4 * 4.0507 per
// 32-weight group, and each token value is q * sx per 128-k chunk.  The reference
// multiplies int8 by int8 on IMMA and rescales the int32 sum after every 32 k, the
// only span one weight scale covers.  On tcgen05 that rescale would read the tensor
// memory accumulator back after every K = 32 MMA and spend two to three CUDA-core
// operations per output per 32 multiply-adds, which bounds an int8 kernel below the
// fp16 contraction it would replace.  So the tier runs on the fp16 tcgen05
// contraction of prefill.cu with the quantised operands: the weight tile decodes the
// levels through the same grid-table path (the lut8 bytes replace the grid
// magnitudes; (2s+1) * d/4 is the group scale), and the tokens are staged as
// fp16(q * sx * 4.0507 * 2^-e) with a power-of-two 2^e per token that the epilogue
// multiplies back.  Every level * (2s+1) product is exact in fp16; one fp16 rounding
// falls on each weight and each token value, the same as in the fp16 tier.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"
#include "tlx_internal.h"

namespace tlx {
namespace {

constexpr int kChunk = 128;           // tokens are quantised per 128-k chunk
constexpr float kLevelStep = 4.0507f;  // grid magnitude ~= step * level (engine/p8_w4ffn7.cu:42)

// Half a warp per (token, chunk): lane l of the half holds k = 8l .. 8l+7 (two 8-byte
// loads); each warp takes 2 * kQuantSteps chunks per pass and issues all their loads
// before the first reduction, so enough bytes are in flight to stream HBM.  The
// max and the integer sum do not depend on the reduction order.
constexpr int kQuantSteps = 2;

__global__ void __launch_bounds__(256) act_quant_q8_kernel(const __half* __restrict__ x, int64_t ldx, int m, int nch,
                                                           int8_t* __restrict__ xq, int64_t ldq,
                                                           float* __restrict__ sx, int32_t* __restrict__ rs) {
  const int lane = threadIdx.x & 31, half = lane >> 4, hl = lane & 15;
  const int64_t units = static_cast<int64_t>(m) * nch;
  const int64_t per_pass = static_cast<int64_t>(gridDim.x) * 8 * (2 * kQuantSteps);
  for (int64_t base = (static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5)) * (2 * kQuantSteps); base < units;
       base += per_pass) {
    uint2 h[kQuantSteps][2];
    int t[kQuantSteps], c[kQuantSteps];
    bool ok[kQuantSteps];
#pragma unroll
    for (int j = 0; j < kQuantSteps; ++j) {
      const int64_t u = base + 2 * j + half;
      ok[j] = u < units;
      t[j] = ok[j] ? static_cast<int>(u / nch) : 0;
      c[j] = ok[j] ? static_cast<int>(u - static_cast<int64_t>(t[j]) * nch) : 0;
      h[j][0] = h[j][1] = make_uint2(0u, 0u);
      if (ok[j]) {
        const uint2* src = reinterpret_cast<const uint2*>(x + t[j] * ldx + c[j] * kChunk + 8 * hl);
        h[j][0] = src[0];
        h[j][1] = src[1];
      }
    }
#pragma unroll
    for (int j = 0; j < kQuantSteps; ++j) {
      float f[8];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const uint32_t w = e == 0 ? h[j][0].x : e == 1 ? h[j][0].y : e == 2 ? h[j][1].x : h[j][1].y;
        const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&w));
        f[2 * e] = v.x;
        f[2 * e + 1] = v.y;
      }
      float am = 0.0f;
#pragma unroll
      for (int e = 0; e < 8; ++e) am = fmaxf(am, fabsf(f[e]));
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));   // within the half
      const float s = fmaxf(am, 1e-6f) * (1.0f / 127.0f);
      uint32_t packed[2] = {0u, 0u};
      int sum = 0;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int q = min(127, max(-127, __float2int_rn(__fdiv_rn(f[e], s))));   // IEEE quotient, ties to even
        packed[e >> 2] |= (static_cast<uint32_t>(q) & 0xFFu) << (8 * (e & 3));
        sum += q;
      }
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      if (ok[j]) {
        uint32_t* dst = reinterpret_cast<uint32_t*>(xq + t[j] * ldq + c[j] * kChunk + 8 * hl);
        dst[0] = packed[0];
        dst[1] = packed[1];
        if (hl == 0) {
          sx[static_cast<int64_t>(t[j]) * nch + c[j]] = s;
          rs[static_cast<int64_t>(t[j]) * nch + c[j]] = sum;
        }
      }
    }
  }
}

// One CTA per token row: the bound B = 127 * 4.0507 * max sx of the row gives the
// power-of-two e = exponent(B) - 14 (so every staged value stays below 2^15, and
// rows of small values are scaled up out of the fp16 subnormals); the row is stored
// as fp16(q * (sx * 4.0507 * 2^-e)) and row_scale[t] = 2^e.
__global__ void __launch_bounds__(256) w4a8_stage_kernel(const int8_t* __restrict__ xq, int64_t ldq,
                                                         const float* __restrict__ sx, int m, int k,
                                                         __half* __restrict__ out, float* __restrict__ row_scale) {
  __shared__ float red[8];
  const int nch = k / kChunk;
  for (int t = blockIdx.x; t < m; t += gridDim.x) {
    const float* srow = sx + static_cast<int64_t>(t) * nch;
    float mx = 0.0f;
    for (int c = threadIdx.x; c < nch; c += blockDim.x) mx = fmaxf(mx, fabsf(srow[c]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = red[0];
#pragma unroll
    for (int w = 1; w < 8; ++w) mx = fmaxf(mx, red[w]);
    __syncthreads();
    const uint32_t bits = __float_as_uint(mx * (127.0f * kLevelStep));
    int sh = 0;
    if (bits != 0u && bits < 0x7F800000u) sh = min(60, max(-60, static_cast<int>(bits >> 23) - 127 - 14));
    const float down = __uint_as_float(static_cast<uint32_t>(127 - sh) << 23);   // 2^-sh
    if (threadIdx.x == 0) row_scale[t] = __uint_as_float(static_cast<uint32_t>(127 + sh) << 23);
    const int8_t* qrow = xq + t * ldq;
    __half* orow = out + static_cast<int64_t>(t) * k;
    for (int i = threadIdx.x; i < (k >> 3); i += blockDim.x) {
      const uint2 v = *reinterpret_cast<const uint2*>(qrow + 8 * i);
      const float f = srow[(8 * i) / kChunk] * kLevelStep * down;
      const uint32_t w[2] = {v.x, v.y};
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t word = w[j >> 1] >> (16 * (j & 1));
        const float a = static_cast<float>(static_cast<int8_t>(word & 0xFFu));
        const float b = static_cast<float>(static_cast<int8_t>((word >> 8) & 0xFFu));
        o[j] = h2_bits(__floats2half2_rn(a * f, b * f));
      }
      *reinterpret_cast<uint4*>(orow + 8 * i) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

bool aligned(const void* q, uintptr_t a) { return (reinterpret_cast<uintptr_t>(q) & (a - 1)) == 0; }

}  // namespace
}  // namespace tlx

using namespace tlx;

namespace {
constexpr size_t kPfErrBytes = 256;  // the prefill workspace starts with the device error word
}

extern "C" {

int tlx_act_quant_q8(const void* x, int64_t ldx, int m, int64_t k, int8_t* xq, int64_t ldq, float* sx, int32_t* rs,
                     void* stream) {
  if (!x || !xq || !sx || !rs) return TLX_ERR_NULL;
  if (m < 1 || m > (1 << 20) || k < kChunk || k % kChunk || k > (1 << 20)) return TLX_ERR_SHAPE;
  if (ldx < k || ldq < k || ldx % 4 || ldq % 4 || !aligned(x, 8) || !aligned(xq, 4)) return TLX_ERR_ALIGN;
  const int nch = static_cast<int>(k / kChunk);
  const int64_t units = static_cast<int64_t>(m) * nch;
  const int64_t per_block = 8 * 2 * kQuantSteps;   // chunks one CTA takes per pass
  const int blocks = static_cast<int>((units + per_block - 1) / per_block < 148 * 16 ? (units + per_block - 1) / per_block
                                                                                     : 148 * 16);
  act_quant_q8_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<const __half*>(x), ldx, m,
                                                                             nch, xq, ldq, sx, rs);
  return cudaGetLastError() == cudaSuccess ? TLX_OK : TLX_ERR_LAUNCH;
}

int tlx_prefill_w4a8_gate_up(const void* w_gate, const void* w_up, const int8_t* lut8, const int8_t* xq, int64_t ldq,
                             const float* sx, int m, int64_t n_rows, int64_t k, float* act, int64_t ld_act, void* ws,
                             size_t ws_bytes, void* stream) {
  if (!w_gate || !w_up || !lut8 || !xq || !sx || !act || !ws) return TLX_ERR_NULL;
  if (m < 1 || n_rows < 128 || n_rows % 128 || k < 256 || k % 256 || k > (1 << 20) || n_rows > (1 << 20) ||
      m > (1 << 20) || ld_act < n_rows)
    return TLX_ERR_SHAPE;
  if (ldq < k || ldq % 8 || !aligned(xq, 8) || !aligned(lut8, 4) || !aligned(w_gate, 16) || !aligned(w_up, 16) ||
      !aligned(ws, 16))
    return TLX_ERR_ALIGN;
  if (ws_bytes < kPfErrBytes + prefill_x_bytes(m, k)) return TLX_ERR_WORKSPACE;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* base = static_cast<uint8_t*>(ws) + kPfErrBytes;
  __half* image = reinterpret_cast<__half*>(base);
  float* row_scale = reinterpret_cast<float*>(base + prefill_scale_offset(m, k));
  const int blocks = m < 65536 ? m : 65536;
  w4a8_stage_kernel<<<blocks, 256, 0, s>>>(xq, ldq, sx, m, static_cast<int>(k), image, row_scale);
  if (cudaGetLastError() != cudaSuccess) return TLX_ERR_LAUNCH;
  return prefill_on_f16(1, w_gate, w_up, reinterpret_cast<const uint32_t*>(lut8), image, k, row_scale, m, n_rows, k,
                        act, ld_act, base, ws_bytes - kPfErrBytes, static_cast<uint32_t*>(ws), 0, s);
}

}  // extern "C"
