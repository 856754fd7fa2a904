// n-gram draft proposal over the token history (the lookup{K+1}_nw32 family,
// engine/lookup11_nw32.cu:8-60 and its K = 4..9 siblings).
//
// Suffix s = hist[pos-8 .. pos-1].  Every start i in [0, pos - E] is scored by the
// length l (0..8) of the common prefix of hist[i .. i+7] and s; the winner is the
// largest (l, i) (longest match, then the most recent start).  On l = 8 the K
// tokens hist[i+8 .. i+8+K-1] become the drafts; l_hist[cyc] always records
// l + 1 (or 1000000 + pos when pos < E and the suffix / scan range is undefined).
//
// B200 layout: the scan is spread over a grid of CTAs (the history can be 100K+
// tokens; one CTA would walk it in ~100 dependent rounds).  Each thread compares
// four consecutive starts from one 16-byte load of hist[i .. i+3] (+ the rare
// continuation loads on a first-token hit), warps reduce with redux, a CTA with
// one shared atomic, the grid with one 64-bit atomicMax on the workspace key; the
// last CTA to finish (done counter) writes the outputs and re-arms the workspace.
// The key is (l << 32) | i, so histories past 2^20 tokens keep their order (the
// reference packs (l << 20) | i and is exact below that length).
#include "tlx_internal.h"

#include <algorithm>

namespace tlx {
namespace {

constexpr int kLookupThreads = 256;
constexpr int kStartsPerThread = 4;
constexpr int kStartsPerCta = kLookupThreads * kStartsPerThread;

struct LookupWs {
  unsigned long long key;  // best (l << 32) | i over the grid; 0 = none
  unsigned int done;       // CTAs finished
  unsigned int pad;
};

__device__ __forceinline__ int match_len(const int32_t* __restrict__ h, int i, const int (&s)[8]) {
  int l = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    if (h[i + j] != s[j]) break;
    ++l;
  }
  return l;
}

__global__ void __launch_bounds__(kLookupThreads) lookup_kernel(const int32_t* __restrict__ hist,
                                                                 const int32_t* __restrict__ pos_slot,
                                                                 const int32_t* __restrict__ cyc_slot,
                                                                 int32_t* __restrict__ drafts, int K, int E,
                                                                 int64_t hist_len, int32_t* __restrict__ l_hist,
                                                                 LookupWs* ws) {
  __shared__ unsigned long long cta_key;
  __shared__ unsigned int last;
  if (threadIdx.x == 0) cta_key = 0ull;
  __syncthreads();
  const int pos = pos_slot[0];
  const bool in_range = pos <= hist_len;   // the history holds pos tokens
  unsigned long long best = 0ull;
  if (in_range && pos >= E) {
    int s[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j] = __ldg(hist + pos - 8 + j);
    const int iend = pos - E;
    const int stride = gridDim.x * kStartsPerCta;
    for (int i0 = (blockIdx.x * kLookupThreads + threadIdx.x) * kStartsPerThread; i0 <= iend; i0 += stride) {
      int4 v;
      if (i0 + 3 <= iend) {
        v = __ldg(reinterpret_cast<const int4*>(hist + i0));   // i0 is a multiple of 4: 16-byte aligned
      } else {
        v.x = __ldg(hist + i0);
        v.y = i0 + 1 <= iend ? __ldg(hist + i0 + 1) : ~s[0];
        v.z = i0 + 2 <= iend ? __ldg(hist + i0 + 2) : ~s[0];
        v.w = ~s[0];
      }
      const int first[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int u = 0; u < kStartsPerThread; ++u) {
        if (first[u] == s[0]) {
          const int i = i0 + u;
          const int l = match_len(hist, i, s);
          const unsigned long long k = (static_cast<unsigned long long>(l) << 32) | static_cast<unsigned int>(i);
          best = k > best ? k : best;
        }
      }
    }
  }
  // warp max (as two 32-bit halves: l first, then i among the lanes with the top l)
  const unsigned int hi = static_cast<unsigned int>(best >> 32);
  const unsigned int top = __reduce_max_sync(0xffffffffu, hi);
  const unsigned int lo = __reduce_max_sync(0xffffffffu, hi == top ? static_cast<unsigned int>(best) : 0u);
  const unsigned long long wbest = (static_cast<unsigned long long>(top) << 32) | lo;
  if ((threadIdx.x & 31) == 0 && wbest) atomicMax(&cta_key, wbest);
  __syncthreads();
  if (threadIdx.x == 0) {
    if (cta_key) atomicMax(&ws->key, cta_key);
    __threadfence();
    last = atomicAdd(&ws->done, 1u) == gridDim.x - 1 ? 1u : 0u;
  }
  __syncthreads();
  if (!last || threadIdx.x != 0) return;
  // the last CTA: every other CTA's atomicMax happened before its arrival
  __threadfence();
  const unsigned long long key = atomicExch(&ws->key, 0ull);   // read and re-arm
  ws->done = 0u;
  const int l = static_cast<int>(key >> 32);
  if (!in_range) return;   // pos beyond the buffer: nothing is read or written
  l_hist[cyc_slot[0]] = pos < E ? 1000000 + pos : l + 1;
  if (l >= 8) {
    const int i = static_cast<int>(key & 0xFFFFFFFFull);
    for (int j = 0; j < K; ++j) drafts[j] = hist[i + 8 + j];
  }
}

}  // namespace

size_t lookup_workspace_bytes() { return 256; }

int run_lookup(const int32_t* hist, int64_t hist_len, const int32_t* pos_slot, const int32_t* cyc_slot,
               int32_t* drafts, int n_drafts, int scan_end, int32_t* l_hist, void* ws, size_t ws_bytes,
               cudaStream_t stream) {
  if (!hist || !pos_slot || !cyc_slot || !drafts || !l_hist || !ws) return TLX_ERR_NULL;
  if (n_drafts < 1 || n_drafts > 16 || scan_end < 8 + n_drafts) return TLX_ERR_SHAPE;
  if (hist_len < 1 || hist_len > 0x7FFFFFF0ll) return TLX_ERR_SHAPE;
  if (ws_bytes < lookup_workspace_bytes()) return TLX_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(hist) & 15) || (reinterpret_cast<uintptr_t>(ws) & 15)) return TLX_ERR_ALIGN;
  // the grid covers every start a history of hist_len tokens can have; CTAs past
  // the device-side pos return after the reduction handshake
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t need = (hist_len + kStartsPerCta - 1) / kStartsPerCta;
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(need, 2 * static_cast<int64_t>(sms))));
  lookup_kernel<<<grid, kLookupThreads, 0, stream>>>(hist, pos_slot, cyc_slot, drafts, n_drafts, scan_end, hist_len,
                                                     l_hist, static_cast<LookupWs*>(ws));
  return cudaGetLastError() == cudaSuccess ? TLX_OK : TLX_ERR_LAUNCH;
}

}  // namespace tlx

extern "C" {

size_t tlx_lookup_workspace_bytes(void) { return tlx::lookup_workspace_bytes(); }

int tlx_lookup(const int32_t* tok_hist, int64_t hist_len, const int32_t* pos_slot, const int32_t* cyc_slot,
               int32_t* drafts, int n_drafts, int scan_end, int32_t* l_hist, void* ws, size_t ws_bytes, void* stream) {
  return tlx::run_lookup(tok_hist, hist_len, pos_slot, cyc_slot, drafts, n_drafts, scan_end, l_hist, ws, ws_bytes,
                         static_cast<cudaStream_t>(stream));
}

}  // extern "C"
