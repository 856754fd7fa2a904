// Peer memory between the GPUs of one node (one process per GPU).
//
// Each rank allocates one communication buffer (a torch tensor is fine: any
// cudaMalloc-backed device memory), exports it with tlx_ipc_handle, the handles are
// exchanged on the host (torch.distributed all_gather_object), and every rank opens
// every peer's buffer with tlx_ipc_open.  The fused verify kernels then write their
// partial results into their own buffer, raise per-rank release flags in every rank's
// buffer, and read the peers' results over NVLink / NVSwitch with ordinary loads once
// the flags are up (gemv.cu, PeerParams).  No TMA and no multicast touch peer memory.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "tlx_internal.h"

namespace {

using GetAddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

// cuMemGetAddressRange through the runtime's entry-point query (the library does not
// link the driver library directly)
GetAddressRangeFn address_range() {
  static GetAddressRangeFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<GetAddressRangeFn>(ptr);
  }
  return fn;
}

}  // namespace

extern "C" {

size_t tlx_ipc_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

int tlx_ipc_handle(const void* ptr, void* handle_out, uint64_t* offset_out) {
  if (!ptr || !handle_out || !offset_out) return TLX_ERR_NULL;
  const GetAddressRangeFn range = address_range();
  if (!range) return TLX_ERR_DEVICE;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) return TLX_ERR_DEVICE;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)) != cudaSuccess) return TLX_ERR_DEVICE;
  std::memcpy(handle_out, &h, sizeof(h));
  *offset_out = static_cast<uint64_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return TLX_OK;
}

int tlx_ipc_open(const void* handle, uint64_t offset, void** base_out, void** ptr_out) {
  if (!handle || !base_out || !ptr_out) return TLX_ERR_NULL;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  if (cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return TLX_ERR_DEVICE;
  *base_out = base;
  *ptr_out = static_cast<uint8_t*>(base) + offset;
  return TLX_OK;
}

int tlx_ipc_close(void* base) {
  if (!base) return TLX_ERR_NULL;
  return cudaIpcCloseMemHandle(base) == cudaSuccess ? TLX_OK : TLX_ERR_DEVICE;
}

// a communication buffer that is one allocation of its own (so its IPC handle names
// exactly this buffer), zeroed; set-up time only, never inside a step
int tlx_peer_buffer_alloc(size_t bytes, void** out) {
  if (!out) return TLX_ERR_NULL;
  if (bytes == 0) return TLX_ERR_SHAPE;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return TLX_ERR_DEVICE;
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(p);
    return TLX_ERR_DEVICE;
  }
  *out = p;
  return TLX_OK;
}

int tlx_peer_buffer_free(void* p) {
  if (!p) return TLX_ERR_NULL;
  return cudaFree(p) == cudaSuccess ? TLX_OK : TLX_ERR_DEVICE;
}

}  // extern "C"
