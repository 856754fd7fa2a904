// Allocation-free variant of the fused LM-head argmax (tlx_head_argmax_noalloc).
//
// Who needs it: callers that cannot call cudaMalloc at the point where they run
// the head -- code that owns all device memory through its own fixed pool and
// forbids allocation after start-up (the reference engine preallocates every
// buffer once and bans reallocation in the request path), plug-ins embedded in
// a host that gives them no memory budget, and latency-critical loops where
// cudaMalloc's implicit device synchronisation is not acceptable.  The regular
// entry point needs a caller-owned workspace; this one uses a fixed scratch
// array compiled into the library instead.
//
// The scratch is a file-scope __device__ array of TLX_NOALLOC_SCRATCH_BYTES.
// Every GPU that loads the library holds it until the process exits.  In host
// code its name is only a host-side stand-in, never a device address, so its
// device address is looked up once per device with cudaGetSymbolAddress (with
// that device current) and that address is what the kernel receives.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "tlx_internal.h"

namespace {

constexpr size_t kScratchBytes = TLX_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;
constexpr int kEpiArgmax = 2;

__device__ __align__(256) uint8_t g_noalloc_scratch[kScratchBytes];

std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// device address of the scratch array for the current device (first call per
// device resolves it; no allocation happens here or anywhere in this file)
int scratch_for_current_device(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return TLX_ERR_DEVICE;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return TLX_ERR_DEVICE;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return TLX_OK;
}

}  // namespace

extern "C" int tlx_head_argmax_noalloc(int qtype, const void* w, const uint32_t* grid, const void* x, int x_dtype,
                                       int64_t ldx, int m, int64_t n_rows, int64_t k, int64_t row_offset,
                                       float* out_max, int32_t* out_idx, uint64_t* out_keys, const int32_t* drafts,
                                       int n_drafts, int32_t* accept_out, void* stream) {
  // the same grid as tlx_head_argmax: honour the tlx_set_max_ctas cap
  const int max_ctas = tlx::max_ctas_setting();
  const size_t need = tlx::gemv_workspace_bytes(kEpiArgmax, qtype, n_rows, k, m, x_dtype, max_ctas);
  if (need == 0) return TLX_ERR_SHAPE;
  if (need > kScratchBytes) return TLX_ERR_WORKSPACE;  // shape needs more than the built-in scratch
  void* ws = nullptr;
  int rc = scratch_for_current_device(&ws);
  if (rc != TLX_OK) return rc;
  // the array keeps whatever the previous call left: zero the arrival counters
  // and the error word (stream-ordered; partials are written before they are read)
  const size_t zero = tlx::gemv_counter_bytes(kEpiArgmax, qtype, n_rows, k, m, x_dtype, max_ctas);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(ws, 0, zero, s) != cudaSuccess) return TLX_ERR_LAUNCH;
  return tlx::run_gemv(kEpiArgmax, qtype, w, nullptr, grid, x, x_dtype, ldx, m, n_rows, k, nullptr, 0, nullptr,
                       TLX_DT_F32, 0, row_offset, out_max, out_idx, out_keys, drafts, n_drafts, accept_out, ws,
                       kScratchBytes, max_ctas, s);
}

// The error word of the current device's scratch (word 0): bit 0 = a bounded wait
// for a weight copy gave up, so that call's results are not to be trusted.  The
// next tlx_head_argmax_noalloc call on this device clears it, so read it in
// between.  Waits for `stream` to drain.
extern "C" int tlx_head_argmax_noalloc_error(uint32_t* err_out, void* stream) {
  if (!err_out) return TLX_ERR_NULL;
  void* ws = nullptr;
  int rc = scratch_for_current_device(&ws);
  if (rc != TLX_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(err_out, ws, 4, cudaMemcpyDeviceToHost, s) != cudaSuccess) return TLX_ERR_LAUNCH;
  return cudaStreamSynchronize(s) == cudaSuccess ? TLX_OK : TLX_ERR_LAUNCH;
}
