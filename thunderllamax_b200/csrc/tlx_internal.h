// Internal declarations shared by the library's translation units.
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "../../include/tlx_verify.h"

namespace tlx {

enum : int { DT_F32 = TLX_DT_F32, DT_F16 = TLX_DT_F16, DT_BF16 = TLX_DT_BF16, DT_IMAGE = TLX_DT_IMAGE };

int run_gemv(int epi, int qt, const void* w0, const void* w1, const uint32_t* grid, const void* x, int x_dtype,
             int64_t ldx, int m, int64_t n_rows, int64_t k, const float* residual, int64_t ldr, void* y,
             int y_dtype, int64_t ldy, int64_t row_offset, float* out_max, int32_t* out_idx, uint64_t* out_keys,
             const int32_t* drafts, int n_drafts, int32_t* accept_out, void* ws, size_t ws_bytes, int max_ctas,
             cudaStream_t stream);
size_t gemv_workspace_bytes(int epi, int qt, int64_t n_rows, int64_t k, int m, int x_dtype, int max_ctas);
size_t aq3k8v11_workspace_bytes(int m, int64_t k, int64_t nq, int64_t nk, int64_t nv, int x_dtype, int max_ctas);
int aq3k8v11_error(const void* ws, int m, int64_t k, int64_t nq, int64_t nk, int64_t nv, int x_dtype, int max_ctas,
                   uint32_t* err_out);
int run_aq3k8v11(const void* wq, const void* wk, const void* wv, const uint32_t* grid, const void* x, int x_dtype,
                 int64_t ldx, int m, int64_t k, int64_t nq, int64_t nk, int64_t nv, void* q_out, void* k_out,
                 void* v_out, void* ws, size_t ws_bytes, int max_ctas, cudaStream_t stream);
size_t activation_image_bytes(int m, int64_t k, int x_dtype);
int stage_activations(const void* x, int x_dtype, int64_t ldx, int m, int64_t k, void* image, cudaStream_t stream);
size_t gemv_counter_bytes(int epi, int qt, int64_t n_rows, int64_t k, int m, int x_dtype, int max_ctas);
int gemv_plan_info(int epi, int qt, int64_t n_rows, int64_t k, int m, int x_dtype, int max_ctas, int32_t* info,
                   int n_info);

}  // namespace tlx
