// Internal declarations shared by the library's translation units.
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "../../include/tlx_verify.h"

namespace tlx {

enum : int { DT_F32 = TLX_DT_F32, DT_F16 = TLX_DT_F16, DT_BF16 = TLX_DT_BF16, DT_IMAGE = TLX_DT_IMAGE };

// Peer exchange of the sharded verify step (one process per GPU): base[r] = rank r's
// communication buffer (peer_buffer_bytes) as mapped in this process.  The down
// projection (STORE) sends its partial y to every rank; the head (ARGMAX) adds the
// ranks' partials (+ residual) into y and merges the ranks' argmax keys.
constexpr int kMaxPeers = 8;
struct PeerParams {
  int world, rank;
  uint8_t* base[kMaxPeers];
  int m;                  // tokens of the y partials
  int64_t ny;             // y row length (the down projection's rows)
  const float* residual;  // head: y = residual + the ranks' partials in rank order
  int64_t ldr;
  float* y;
  int64_t ldy;
};
size_t peer_buffer_bytes(int world, int m, int64_t ny);
// end of a sharded step: y = residual + the ranks' down partials (rank order), epoch + 1
int peer_finish(const PeerParams& pr, uint32_t* err, cudaStream_t stream);
// a partial (pr.residual, row stride pr.ldr) into this rank's buffer + its flag everywhere
int peer_publish(const PeerParams& pr, cudaStream_t stream);

int run_gemv(int epi, int qt, const void* w0, const void* w1, const uint32_t* grid, const void* x, int x_dtype,
             int64_t ldx, int m, int64_t n_rows, int64_t k, const float* residual, int64_t ldr, void* y,
             int y_dtype, int64_t ldy, int64_t row_offset, float* out_max, int32_t* out_idx, uint64_t* out_keys,
             const int32_t* drafts, int n_drafts, int32_t* accept_out, void* ws, size_t ws_bytes, int max_ctas,
             cudaStream_t stream, const PeerParams* peer = nullptr);
size_t gemv_workspace_bytes(int epi, int qt, int64_t n_rows, int64_t k, int m, int x_dtype, int max_ctas);
// one matvec of a projection group: n_rows rows of qtype qt, fp16 output [m][n_rows]
struct Projection {
  int qt;
  const void* w;
  int64_t n_rows;
  void* out;
};
constexpr int kMaxProjections = 4;
size_t projections_workspace_bytes(int n, const Projection* pr, int m, int64_t k, int x_dtype, int max_ctas);
int run_projections(int n, const Projection* pr, const uint32_t* grid, const void* x, int x_dtype, int64_t ldx, int m,
                    int64_t k, void* ws, size_t ws_bytes, int max_ctas, cudaStream_t stream);
int projections_error(const void* ws, int n, const Projection* pr, int m, int64_t k, int x_dtype, int max_ctas,
                      uint32_t* err_out);
size_t activation_image_bytes(int m, int64_t k, int x_dtype);
int stage_activations(const void* x, int x_dtype, int64_t ldx, int m, int64_t k, void* image, cudaStream_t stream);
size_t gemv_counter_bytes(int epi, int qt, int64_t n_rows, int64_t k, int m, int x_dtype, int max_ctas);
// the CTA cap set by tlx_set_max_ctas (0 = one CTA per SM)
int max_ctas_setting();

// prefill contraction (prefill.cu).  Workspace after the error word: the fp16 token
// image [m][k] (256-byte aligned end), one float scale per token, then the split region.
size_t prefill_x_bytes(int m, int64_t k);
size_t prefill_scale_offset(int m, int64_t k);
// gate/up (gate_up = 1, IQ3_XXS tiles and a 256-entry grid table whose byte j of entry i
// is magnitude j) or the Q6_K GEMM on tokens already in fp16 (xf16 [m][ldx16]; row_scale:
// each token's power-of-two factor, or nullptr); shapes checked by the caller
int prefill_on_f16(int gate_up, const void* w0, const void* w1, const uint32_t* grid, const void* xf16,
                   int64_t ldx16, const float* row_scale, int m, int64_t n_rows, int64_t k, void* out, int64_t ldo,
                   void* ws, size_t ws_bytes, uint32_t* err, int max_ctas, cudaStream_t stream);
int gemv_plan_info(int epi, int qt, int64_t n_rows, int64_t k, int m, int x_dtype, int max_ctas, int32_t* info,
                   int n_info);

}  // namespace tlx
