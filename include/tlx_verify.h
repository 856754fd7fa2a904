/* ThunderLlamaX speculative-verify path on B200 (sm_100a) -- C ABI.
 *
 * Plain pointers and sizes only.  Every device entry point is stream-ordered,
 * allocates nothing, performs no host synchronisation (graph-capturable),
 * checks its arguments on the host before launching, and returns 0 or a
 * negative TLX_ERR_* code.  Device pointers are CUDA device addresses on the
 * current device; `stream` is a cudaStream_t (NULL = legacy default stream).
 *
 * Reference boundary being replaced: the per-kernel NVProgram call surface
 * prog(*device_buffers, global_size, local_size) of engine/engine0.py:99-106
 * with graph entries (prog, (bufs...), grid) of engine/gcycle.py:39-47; buffer
 * ownership per engine/engine0.py:65-95 (caller preallocates, kernels never
 * allocate).  Launch geometry is chosen here instead of being encoded in
 * kernel names (engine/gcycle.py:45).
 */
#ifndef TLX_VERIFY_H
#define TLX_VERIFY_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type ids (GGUF tensor types) */
#define TLX_Q8_0 8    /* STORE GEMV only (the GDN o-projection rows); one "block"
                        of the layout = 8 GGUF blocks (272 B per 256 weights) */
#define TLX_Q4_K 12   /* STORE GEMV only (the attention v rows) */
#define TLX_Q5_K 13   /* STORE GEMV only (the GDN qkv rows) */
#define TLX_Q6_K 14
#define TLX_IQ3_XXS 18
#define TLX_IQ4_XS 23
/* activation dtypes (ggml ids) */
#define TLX_DT_F32 0
#define TLX_DT_F16 1
#define TLX_DT_BF16 30
/* activations already staged as an fp16 activation image (tlx_stage_activations,
 * or tlx_ffn_gate_up with gact_dtype = TLX_DT_IMAGE): x points at the image, ldx
 * is ignored, one column per token */
#define TLX_DT_IMAGE 100
/* (Q4_K / Q5_K GEMVs also read the per-sub-block sums of x that
 * tlx_stage_activations writes into the image; an image written by tlx_ffn_gate_up
 * carries none, so give a Q4_K / Q5_K GEMV raw activations or a
 * tlx_stage_activations image.) */
/* gemv modes for tlx_gemv_workspace_bytes */
#define TLX_MODE_STORE 0
#define TLX_MODE_GATE_UP 1
#define TLX_MODE_ARGMAX 2

#define TLX_OK 0
#define TLX_ERR_SHAPE (-1)
#define TLX_ERR_ALIGN (-2)
#define TLX_ERR_DTYPE (-3)
#define TLX_ERR_QTYPE (-4)
#define TLX_ERR_WORKSPACE (-5)
#define TLX_ERR_LAUNCH (-6)
#define TLX_ERR_DEVICE (-7)
#define TLX_ERR_NULL (-8)

/* workspace error word bits (read with tlx_workspace_error) */
#define TLX_WS_ERR_MBAR_TIMEOUT 1u

const char* tlx_error_string(int code);
/* 0 if the current device is an sm_100 part this library was built for */
int tlx_device_check(void);
int tlx_version(void);
/* cap on CTAs per launch (0 = one per SM).  Tuning/testing knob: smaller values
 * force split tiles and k-segments on small shapes. */
void tlx_set_max_ctas(int n);

/* ---- weight layout ------------------------------------------------------------
 * GGUF rows (ggml block_iq3_xxs 98 B / block_q6_K 210 B / block_q4_K 144 B /
 * block_q5_K 176 B per 256 weights, block_q8_0 34 B per 32) ->
 * B200 tile layout (16-row tiles, one 16*block_bytes chunk per tile and block,
 * same byte count as GGUF plus zero rows up to a multiple of 16).  Replaces the
 * offline repackers engine/pack_w1c.py:18-45 (IQ3 row regions, Q6_K 212-B pad)
 * and engine/pack_w7.py (packed7 units). */
size_t tlx_tiled_bytes(int qtype, int64_t n_rows, int64_t k);
/* host -> host; src rows are src_row_stride bytes apart */
int tlx_pack_tiles(int qtype, const void* src, int64_t n_rows, int64_t k, int64_t src_row_stride, void* dst);
/* device -> device (same layout), stream-ordered */
int tlx_pack_tiles_device(int qtype, const void* src, int64_t n_rows, int64_t k, int64_t src_row_stride, void* dst,
                          void* stream);
/* inverse of tlx_pack_tiles (host), for round-trip checks */
int tlx_unpack_tiles(int qtype, const void* tiled, int64_t n_rows, int64_t k, void* dst);

/* ---- workspace -----------------------------------------------------------------
 * Caller-owned scratch for split-tile partial sums, per-tile arrival counters and
 * argmax partials.  Zero it once (tlx_workspace_init) before first use; every
 * successful launch leaves its counters at zero again.  One workspace must not be
 * used by two launches that can overlap on the GPU. */
size_t tlx_gemv_workspace_bytes(int mode, int qtype, int64_t n_rows, int64_t k, int m, int x_dtype);
int tlx_workspace_init(void* ws, size_t ws_bytes, void* stream);
/* launch plan for a shape: info[] = {tiles, blocks/row, k-segments, blocks/segment,
 * CTAs, CTAs/segment, max pieces/tile-segment, columns, n-tiles, warps/CTA,
 * ring stages, shared bytes} */
int tlx_gemv_plan(int mode, int qtype, int64_t n_rows, int64_t k, int m, int x_dtype, int32_t* info, int n_info);
/* synchronous read of the workspace error word (TLX_WS_ERR_* bits) */
int tlx_workspace_error(const void* ws, uint32_t* err_out);

/* ---- activation image --------------------------------------------------------------
 * The GEMV kernels read activations as an fp16 image in mma-fragment order
 * ([k/256][16][columns][4][4 halves]) that each CTA pulls into shared memory with
 * one bulk copy.  Raw bf16/fp16/fp32 activations are staged into the workspace by
 * each call; a caller that feeds the same activations to several GEMVs, or chains
 * gate/up -> down, can stage once and pass TLX_DT_IMAGE.  fp32 activations use 3
 * columns per token (exact hi+mid+lo fp16 split). */
size_t tlx_activation_image_bytes(int m, int64_t k, int x_dtype);
int tlx_stage_activations(const void* x, int x_dtype, int64_t ldx, int m, int64_t k, void* image, void* stream);

/* ---- K-row dequantised matvec ----------------------------------------------------
 * y[t][r] = sum_k W[r][k] * x[t][k] (+ residual[t][r]), t < m <= 16 (m <= 5 for
 * fp32 x), fp32 accumulate; y is fp32 or fp16 (y_dtype).  W tiled
 * (tlx_pack_tiles), grid = the 256 u32 IQ3_XXS grid entries (device; NULL for
 * Q6_K).  bf16/fp16 activations are carried as fp16 inside the kernel (exact for
 * |x| in [2^-24 * 2^7, 65504]); fp32 activations are split exactly into three
 * fp16 parts.
 * Replaces down8nw32_11(wd, gridf, gact, hh, y) engine/down8nw32_11.cu:88-126
 * (residual = hh), head8v11(w, xh, logits) engine/head8v11.cu:88-121 and the GDN
 * o-projections op38nw32_11(wo, gridf, z, attn_out) engine/op38nw32_11.cu:88-120
 * (IQ3_XXS) / k3aonw32_11(wq8, z, attn_out) engine/k3aonw32_11.cu:88-116 (Q8_0;
 * weights rounded to fp16(d q) as the reference does), fp16 z and output. */
int tlx_gemv(int qtype, const void* w, const uint32_t* grid, const void* x, int x_dtype, int64_t ldx, int m,
             int64_t n_rows, int64_t k, const float* residual, int64_t ldr, void* y, int y_dtype, int64_t ldy,
             void* ws, size_t ws_bytes, void* stream);

/* ---- fused gate/up + SiLU ------------------------------------------------------------
 * gact[t][r] = silu(Wg x_t)[r] * (Wu x_t)[r], stored fp32 or fp16 (gact_dtype), or
 * (gact_dtype = TLX_DT_IMAGE, n_rows % 256 == 0) directly as the fp16 activation
 * image a following GEMV over k = n_rows reads (the reference's fp16 gact feeding
 * down8; ldg ignored, gact must hold tlx_activation_image_bytes(m, n_rows, F16)).
 * Replaces ffn8v11(wg, wu, gridf, hhx, gact) engine/ffn8v11.cu:88-133 and the r7
 * twin engine/ffn8v11r7.cu:261. */
int tlx_ffn_gate_up(int qtype, const void* w_gate, const void* w_up, const uint32_t* grid, const void* x,
                    int x_dtype, int64_t ldx, int m, int64_t n_rows, int64_t k, void* gact, int gact_dtype,
                    int64_t ldg, void* ws, size_t ws_bytes, void* stream);

/* ---- LM head fused with per-row argmax (+ greedy accept) ---------------------------
 * For each token t: (max_r logit[t][r], lowest r attaining it) over the rows of W,
 * reported as global ids row_offset + r (vocab sharding).  No logits reach HBM.
 * out_keys[t] (optional) = the packed u64 key used for cross-shard merging.  If
 * accept_out != NULL: m = longest prefix with idx[s] == drafts[s] (s < n_drafts),
 * accept_out[0] = m, accept_out[1] = idx[m] (needs m_tokens >= n_drafts + 1).
 * Replaces head8v11 + amx3 (engine/head8v11.cu:88-121, engine/amx3.cu:117-142),
 * the fused h6kam_PP + amred36 (engine/mm/MM_P6_h6kam.cu:18-95,
 * engine/mm/MM_P6_amred36.cu:4-30) and acc36 (engine/mm/MM_P7_acc36.cu:11-25). */
int tlx_head_argmax(int qtype, const void* w, const uint32_t* grid, const void* x, int x_dtype, int64_t ldx, int m,
                    int64_t n_rows, int64_t k, int64_t row_offset, float* out_max, int32_t* out_idx,
                    uint64_t* out_keys, const int32_t* drafts, int n_drafts, int32_t* accept_out, void* ws,
                    size_t ws_bytes, void* stream);

/* ---- allocation-free head argmax --------------------------------------------------
 * Same computation and results as tlx_head_argmax, for callers that cannot call
 * cudaMalloc where they run the head (a runtime that owns all device memory in a
 * fixed pool and forbids allocation after start-up, a plug-in given no memory
 * budget, a loop that cannot afford cudaMalloc's implicit synchronisation).  No
 * reference counterpart: the reference's kernels take no workspace.
 * Scratch is a fixed array of TLX_NOALLOC_SCRATCH_BYTES inside the library, held
 * on every GPU that loads it until process exit; shapes needing more return
 * TLX_ERR_WORKSPACE (the full 151936 x 5120, 11-row head needs ~19.5 MB).  The
 * first call on a device looks the array's address up (make it before any stream
 * capture); every call clears the array's counters on `stream` and allocates
 * nothing.  All calls share the one array: calls that can overlap on the GPU
 * (different streams, concurrent graphs) race and must be serialised by the
 * caller.  The grid follows tlx_set_max_ctas like tlx_head_argmax's.  The array's
 * address is looked up once per device and kept: a cudaDeviceReset (or any other
 * reset of the device's primary context) is not supported afterwards. */
#define TLX_NOALLOC_SCRATCH_BYTES (24u << 20)
int tlx_head_argmax_noalloc(int qtype, const void* w, const uint32_t* grid, const void* x, int x_dtype, int64_t ldx,
                            int m, int64_t n_rows, int64_t k, int64_t row_offset, float* out_max, int32_t* out_idx,
                            uint64_t* out_keys, const int32_t* drafts, int n_drafts, int32_t* accept_out,
                            void* stream);
/* The error word of the last tlx_head_argmax_noalloc call on the current device
 * (what tlx_workspace_error reports for the regular entry point): 0 = fine,
 * TLX_WS_ERR_MBAR_TIMEOUT = a bounded wait gave up and the call's outputs are not
 * valid.  Read it before the next call on that device, which clears it.  Waits for
 * `stream`.  No reference counterpart. */
int tlx_head_argmax_noalloc_error(uint32_t* err_out, void* stream);

/* ---- argmax over materialised logits (amx3 / h_argmax) -----------------------------
 * amds[t] = argmax_v logits[t*ld + v] (fp32 or fp16 logits): the reference scan
 * from best = -1e30 with a strict '>', so the lowest index wins ties, NaN / -inf /
 * values <= -1e30 never win and a row without a candidate yields 0.
 * engine/amx3.cu:117-142. */
int tlx_argmax_rows(const void* logits, int dtype, int m, int64_t n, int64_t ld, int32_t* amds, void* stream);

/* h_argmax (T = 1): the same argmax of one row logits[0..n), then the decode-loop
 * side effects tok_slot[0] = idx, tok_hist[pos_slot[0]] = idx, pos_slot[0] += 1
 * (device ints, stream-ordered).  Replaces engine/h_argmax.cu:13-42 (there the
 * vocabulary is fixed at 248320 fp16 logits). */
int tlx_h_argmax(const void* logits, int dtype, int64_t n, int32_t* tok_slot, int32_t* pos_slot, int32_t* tok_hist,
                 void* stream);

/* merge per-shard argmax keys [n_shards][m] (after an all-gather) -> global
 * (max, idx) and optional accept, same rules as tlx_head_argmax. */
int tlx_argmax_merge(const uint64_t* keys, int n_shards, int m, float* out_max, int32_t* out_idx,
                     const int32_t* drafts, int n_drafts, int32_t* accept_out, void* stream);

/* ---- the sharded verify step over peer memory (one process per GPU) ---------------
 * Every rank owns one communication buffer of tlx_peer_buffer_bytes(world, m, ny)
 * bytes (tlx_peer_buffer_alloc: zeroed, an allocation of its own) and maps every other
 * rank's buffer into its process (tlx_ipc_handle on the owner, tlx_ipc_open on the
 * others); peer_bufs[r] is rank r's buffer as mapped in the calling process.  The step
 * replaces NCCL's all-reduce of the down partials and all-gather of the head keys (the
 * collectives of the row / k / vocabulary split):
 *   tlx_gemv_peer         the down projection shard (k split): its fp32 partial y goes
 *                         into this rank's own buffer, and its last CTA raises this
 *                         rank's flag in every rank's buffer (one release store each);
 *   tlx_head_argmax_peer  the vocabulary shard of the fused head; its last CTA puts the
 *                         11 argmax keys into this rank's buffer, raises its flag in
 *                         every rank's buffer, reads all ranks' keys over NVLink, merges
 *                         them and runs greedy accept (the same result on every rank);
 *   tlx_peer_finish       after both, on the same stream: y = residual + the ranks'
 *                         partials read from their buffers over NVLink, in rank order
 *                         (the same bits on every rank), and the step counter advances.
 * The FFN (gate/up, tlx_gemv_peer) and the head are independent and may run on two
 * streams at once with split CTA budgets (max_ctas > 0 caps a launch's grid; 0 = the
 * tlx_set_max_ctas setting); tlx_peer_finish must follow both.  Waits are only on other
 * GPUs' flags, never on another kernel of the same GPU, and are bounded: on timeout the
 * error word (workspace word 0, or err for tlx_peer_finish) gets
 * TLX_WS_ERR_PEER_TIMEOUT.  No reference counterpart: the reference runs on one GPU
 * (README.md:412-413). */
#define TLX_WS_ERR_PEER_TIMEOUT 4u
size_t tlx_peer_buffer_bytes(int world, int m, int64_t ny);
/* a zeroed communication buffer that is an allocation of its own (set-up time only) */
int tlx_peer_buffer_alloc(size_t bytes, void** out);
int tlx_peer_buffer_free(void* p);
size_t tlx_ipc_handle_bytes(void);
/* handle_out (tlx_ipc_handle_bytes) names the allocation holding ptr; offset_out = ptr
 * minus the allocation's base */
int tlx_ipc_handle(const void* ptr, void* handle_out, uint64_t* offset_out);
/* maps a peer's allocation (peer access enabled); *ptr_out = its base + offset */
int tlx_ipc_open(const void* handle, uint64_t offset, void** base_out, void** ptr_out);
int tlx_ipc_close(void* base);
int tlx_gemv_peer(int qtype, const void* w, const uint32_t* grid, const void* x, int x_dtype, int64_t ldx, int m,
                  int64_t n_rows, int64_t k, int world, int rank, void* const* peer_bufs, int max_ctas, void* ws,
                  size_t ws_bytes, void* stream);
int tlx_head_argmax_peer(int qtype, const void* w, const uint32_t* grid, const void* x, int x_dtype, int64_t ldx,
                         int m, int64_t n_rows, int64_t k, int64_t row_offset, float* out_max, int32_t* out_idx,
                         const int32_t* drafts, int n_drafts, int32_t* accept_out, int world, int rank,
                         void* const* peer_bufs, int max_ctas, void* ws, size_t ws_bytes, void* stream);
int tlx_peer_finish(int world, int rank, void* const* peer_bufs, int m, int64_t ny, const float* residual,
                    int64_t ldr, float* y, int64_t ldy, uint32_t* err, void* stream);
/* The same exchange for a partial an ordinary kernel wrote (the expert-parallel MoE
 * layer's output): copies part [m][ny] (row stride ldp) into this rank's buffer and
 * raises this rank's flag in every rank's buffer; tlx_peer_finish on the same stream
 * then sums all ranks' partials (an all-reduce without a collective library).  No
 * reference counterpart: the reference runs one GPU. */
int tlx_peer_publish(int world, int rank, void* const* peer_bufs, int m, int64_t ny, const float* part, int64_t ldp,
                     void* stream);

/* ---- greedy acceptance ------------------------------------------------------------
 * acc36: m = longest prefix amds[s] == drafts[s], s < k; mb[0] = m;
 * eb[0] = m, eb[1] = amds[m].  engine/mm/MM_P7_acc36.cu:11-25. */
int tlx_accept(const int32_t* amds, const int32_t* drafts, int k, int32_t* mb, int32_t* eb, void* stream);

/* accept11k with its commit side effects (engine/accept11k.cu:11-58): drafts[10]
 * replace the ten 1-int dring0..9 buffers; writes tok_hist[pos..pos+m],
 * cur_slot, pos_slot += m+1, m_slot, m_hist[cyc], emit[0..15], cyc_slot += 1,
 * h_seed = xA[m*dim ..], dhd_seed = m == 0 ? hd_d0 : hd_d1. */
int tlx_accept11k(const int32_t* amds, const int32_t* drafts, const float* xA, int32_t* m_slot, int32_t* m_hist,
                  int32_t* cyc_slot, int32_t* pos_slot, int32_t* cur_slot, int32_t* tok_hist, float* h_seed,
                  const float* hd_d0, const float* hd_d1, float* dhd_seed, int32_t* emit, const int32_t* l_hist,
                  int dim, void* stream);

/* aq3k8v11: the attention q / k / v projections of the probe trunk over m rows
 * (engine/aq3k8v11.cu:88-179): q = Wq x (IQ3_XXS, nq rows), k = Wk x (IQ3_XXS, nk
 * rows), v = Wv x (Q4_K, nv rows) for x [m][k] fp16 or bf16 (ld ldx); outputs fp16
 * [m][nq] / [m][nk] / [m][nv].  Weights tiled (tlx_pack_tiles).  x is staged once
 * and the three GEMVs share it.  Workspace: tlx_aq3k8v11_workspace_bytes, zeroed
 * once (tlx_workspace_init) and reused.  The reference shapes are nq = 12288,
 * nk = nv = 1024, k = 5120, m = 11.  After the staging the GEMVs run side by side
 * on internal side streams (one per projection, created once per device) forked
 * from `stream` by an event and joined back into it, so the call stays ordered on
 * `stream` and a CUDA graph capture records parallel branches; tlx_q5g8v11 does
 * the same. */
size_t tlx_aq3k8v11_workspace_bytes(int m, int64_t k, int64_t nq, int64_t nk, int64_t nv, int x_dtype);
int tlx_aq3k8v11(const void* wq, const void* wk, const void* wv, const uint32_t* grid, const void* x, int x_dtype,
                 int64_t ldx, int m, int64_t k, int64_t nq, int64_t nk, int64_t nv, void* q_out, void* k_out,
                 void* v_out, void* ws, size_t ws_bytes, void* stream);
/* the workspace's error bits (OR over the three GEMVs; synchronous read) */
int tlx_aq3k8v11_error(const void* ws, int m, int64_t k, int64_t nq, int64_t nk, int64_t nv, int x_dtype,
                       uint32_t* err_out);

/* q5g8v11: the GDN block's input projections of the probe trunk over m rows
 * (engine/q5g8v11.cu:68-150): qkv = Wqkv x (Q5_K, nqkv rows) and gate = Wg x
 * (IQ3_XXS, ngate rows) for x [m][k] fp16 or bf16 (ld ldx); outputs fp16 [m][nqkv]
 * and [m][ngate].  Weights tiled (tlx_pack_tiles, qtypes TLX_Q5_K / TLX_IQ3_XXS).
 * x is staged once for both GEMVs.  Workspace: tlx_q5g8v11_workspace_bytes, zeroed
 * once (tlx_workspace_init) and reused.  The reference shapes are nqkv = 10240,
 * ngate = 6144, k = 5120, m = 11. */
size_t tlx_q5g8v11_workspace_bytes(int m, int64_t k, int64_t nqkv, int64_t ngate, int x_dtype);
int tlx_q5g8v11(const void* wqkv, const void* wgate, const uint32_t* grid, const void* x, int x_dtype, int64_t ldx,
                int m, int64_t k, int64_t nqkv, int64_t ngate, void* qkv_out, void* gate_out, void* ws,
                size_t ws_bytes, void* stream);
/* the workspace's error bits (OR over the two GEMVs; synchronous read) */
int tlx_q5g8v11_error(const void* ws, int m, int64_t k, int64_t nqkv, int64_t ngate, int x_dtype, uint32_t* err_out);

/* n-gram draft proposal (lookup{K+1}_nw32, engine/lookup11_nw32.cu:8-60; the
 * K = 4..9 siblings engine/lookup5_nw32.cu .. lookup10_nw32.cu differ only in K
 * and scan_end).  With pos = pos_slot[0] and the suffix s = tok_hist[pos-8 ..
 * pos-1]: every start i in [0, pos - scan_end] is scored by the length l (0..8)
 * of the common prefix of tok_hist[i .. i+7] and s; the largest (l, i) wins
 * (longest, then most recent).  l_hist[cyc_slot[0]] = l + 1, or 1000000 + pos
 * when pos < scan_end; on l = 8, drafts[j] = tok_hist[i + 8 + j] for j <
 * n_drafts (the dring0..dring{K-1} buffers, contiguous here).  The reference's
 * scan_end is 8 + K for K <= 7 and 9 + K for K >= 8 (lookup11: K = 10,
 * scan_end = 19).  hist_len = tokens the buffer holds (16-byte aligned); a
 * device pos beyond it writes nothing.  Workspace: tlx_lookup_workspace_bytes,
 * zeroed once (tlx_workspace_init) and reused; one launch, stream-ordered. */
size_t tlx_lookup_workspace_bytes(void);
int tlx_lookup(const int32_t* tok_hist, int64_t hist_len, const int32_t* pos_slot, const int32_t* cyc_slot,
               int32_t* drafts, int n_drafts, int scan_end, int32_t* l_hist, void* ws, size_t ws_bytes, void* stream);

/* Split-KV int8 attention of the full-attention layers over `rows` verify rows
 * (engine/spk_preqh.cu:13-90, engine/spk_g4hm.cu, engine/skv_split.cu:176-199):
 * 24 query heads, 4 KV heads, head dim 256, rotary on dims 0..63.  The cache is
 * kv [8][ctx][256] bytes (int8 q + 128; heads 0..3 K, 4..7 V) with scales
 * sc [8][ctx][8] fp16 (one per 32 dims); pos = pos_slot[0] on the device.
 * tlx_attn_pre: qrow [rows][12288] fp16 (per head 256 q then 256 gate values),
 *   krow / vrow [rows][1024] fp16, qnw / knw [256] fp32 norm weights, freqs [32]
 *   fp32 rotary frequencies -> qw16 [rows][24][256] fp16 (normed, rotated, x 1/16)
 *   and the rows' K / V appended to the cache at pos .. pos + rows - 1 (positions
 *   outside [0, ctx) are not written).  Replaces spk_pre11 (its fp32 qw output is
 *   not produced; the attention reads qw16).
 * tlx_attn_split: per KV head and key range, online-softmax partials of the causal
 *   attention (row t sees keys 0 .. pos + t) into the workspace (spk_a11).
 * tlx_attn_combine: merge the partials, times sigmoid(gate), into ao [rows][6144]
 *   fp16 (spk_c11).  tlx_attn_decode = split + combine.
 * rows <= 16.  Workspace: tlx_attn_workspace_bytes(rows), 256-byte aligned, zeroed
 * once (tlx_workspace_init); its first word holds the error bits of the split
 * kernel's bounded waits (tlx_workspace_error). */
size_t tlx_attn_workspace_bytes(int rows);
int tlx_attn_pre(const void* qrow, const void* krow, const void* vrow, const float* qnw, const float* knw,
                 const float* freqs, const int32_t* pos_slot, int rows, int64_t ctx, void* kv, void* sc, void* qw16,
                 void* stream);
int tlx_attn_split(const void* kv, const void* sc, const void* qw16, const int32_t* pos_slot, int rows, int64_t ctx,
                   void* ws, size_t ws_bytes, void* stream);
int tlx_attn_combine(const void* ws, size_t ws_bytes, const void* qrow, int rows, void* ao, void* stream);
int tlx_attn_decode(const void* kv, const void* sc, const void* qw16, const void* qrow, const int32_t* pos_slot,
                    int rows, int64_t ctx, void* ao, void* ws, size_t ws_bytes, void* stream);

/* acceptsel11k: commit the accepted GDN state (engine/acceptsel11k.cu:8-40).
 * rec4 is [n_blocks][5][rec_elems] fp32 and conv4 [n_blocks][5][conv_elems] fp32,
 * slot 4 the live one; with m = m_slot[0] (device int, 0..10):
 *   rec4[b][4]  <- m <= 4 ? rec4[b][m]  : rec_x[m - 5][b]   (rec6x .. rec11x)
 *   conv4[b][4] <- m <= 3 ? conv4[b][m] : conv_x[m - 4][b]  (conv5x .. conv11x)
 * conv_x / rec_x are HOST arrays of 7 / 6 device pointers, each [n_blocks][elems].
 * The reference fixes n_blocks = 48, rec_elems = 786432, conv_elems = 30720.
 * An m outside 0..10 copies nothing. */
int tlx_acceptsel11k(float* rec4, float* conv4, const int32_t* m_slot, const float* const* conv_x,
                     const float* const* rec_x, int n_blocks, int64_t rec_elems, int64_t conv_elems, void* stream);

/* GDN state commit as a slot index (the index form of acceptsel11k; the reference
 * copies, engine/acceptsel11k.cu:15-39).  A slot table of tlx_gdn_slots_bytes(n_blocks)
 * bytes (device memory, 8-byte aligned) holds per GDN block b the device addresses of
 * the rec and conv buffers of the eleven draft positions and of the live state:
 * tab[(b * 2 + kind) * 12 + s], kind 0 = rec / 1 = conv, s = 0..10 the draft
 * positions, s = 11 the live state.  tlx_gdn_slots_init writes the reference's fixed
 * layout (the buffers of tlx_acceptsel11k; rec draft 4 is the live state itself).
 * tlx_acceptsel11k_flip reads m = m_slot[0] on the device and permutes the table: the
 * live entry then names the buffer holding draft m's state (what tlx_acceptsel11k
 * copies into the live slot) and draft m's entry the buffer that held the live state,
 * free for the next step's draft m.  It moves 8-byte addresses, not the 314 MB of
 * state; the GDN kernels that read and write the states do so through the table.
 * An m outside 0..10 changes nothing. */
size_t tlx_gdn_slots_bytes(int n_blocks);
int tlx_gdn_slots_init(uint64_t* tab, const float* rec4, const float* conv4, const float* const* conv_x,
                       const float* const* rec_x, int n_blocks, int64_t rec_elems, int64_t conv_elems, void* stream);
int tlx_acceptsel11k_flip(uint64_t* tab, const int32_t* m_slot, int n_blocks, void* stream);

/* ---- MoE verify layer (P <= 8 positions, top-8 of E <= 1024 experts + shared) ----
 * Router: logits = w_router[E][hidden] (fp32) . h[p] (bf16), top-8 by 8 masked-argmax
 * passes (strict '>', ties to the lower expert id), gates = exp(l - max) / sum over
 * the 8, sg = sigmoid(w_shared_gate . h[p]); ids / gates are [p][8] rank-major.
 * Replaces rt8e256 (engine/mm/MM_P1_rt8e256.cu:14-62).
 * Experts: IQ4_XS weights in the tile layout (tlx_pack_tiles, qtype 23), one expert
 * after another: gate / up [E][inner x hidden], down [E][hidden x inner]; the
 * shared expert has the same shapes (NULL shared_gate: no shared expert).
 * act = silu(gate h) * (up h), part = down act (fp32), and
 * y[p] = hres[p] + sum_r gates[p][r] part[p][r] + sg[p] shared[p] in that order.
 * Replaces shexp8 / gx8e256up4 / gx8e256dn / cmbz2048 (engine/mm/MM_P2_shexp8.cu:8,
 * engine/mm/MM_P2_gx8e256up4.cu:8-55, engine/mm/MM_P2_gx8e256dn.cu:9-45,
 * engine/mm/MM_P34_cmbz2048.cu:6-29); sequence engine/mm/MM_P7_lib.py:505-511.
 * Expert parallelism: only experts in [expert_begin, expert_end) are computed and
 * combined (pass the shared expert and hres on one rank only); summing y over the
 * ranks gives the full layer.  kvalues = the 16 IQ4_NL levels (gguf-py table).
 * The workspace (tlx_moe_workspace_bytes) must be zero-filled once before first
 * use; its counters re-arm themselves.  Four launches, no host sync, no allocation. */
size_t tlx_moe_workspace_bytes(int p, int n_experts, int hidden, int inner);
int tlx_moe_route(const float* w_router, const float* w_shared_gate, const void* h, int64_t ldh, int p,
                  int n_experts, int hidden, int inner, int expert_begin, int expert_end, int with_shared,
                  int32_t* ids, float* gates, float* sg, void* ws, size_t ws_bytes, void* stream);
int tlx_moe_experts(const void* gate, const void* up, const void* down, const void* shared_gate,
                    const void* shared_up, const void* shared_down, const int8_t* kvalues, const float* hres,
                    int64_t ldr, float* y, int64_t ldy, int p, int n_experts, int hidden, int inner,
                    int expert_begin, int expert_end, void* ws, size_t ws_bytes, void* stream);
int tlx_moe_verify(const float* w_router, const float* w_shared_gate, const void* gate, const void* up,
                   const void* down, const void* shared_gate, const void* shared_up, const void* shared_down,
                   const int8_t* kvalues, const void* h, int64_t ldh, const float* hres, int64_t ldr, float* y,
                   int64_t ldy, int32_t* ids, float* gates, float* sg, int p, int n_experts, int hidden, int inner,
                   int expert_begin, int expert_end, void* ws, size_t ws_bytes, void* stream);
/* device error word of a MoE workspace (bounded-wait timeouts), synchronising `stream` */
int tlx_moe_workspace_error(const void* ws, int p, int n_experts, int hidden, int inner, uint32_t* err_out,
                            void* stream);

/* ---- prefill-sized FFN contraction (tcgen05 tensor cores) ---------------------------
 * Many tokens at once: the GEMM runs as D[row][token] = W . X^T with the weights
 * dequantised to fp16 in shared memory (one fp16 rounding per weight: the exact
 * integer part times the block scale), tokens staged as fp16 by TMA, fp32
 * accumulators in tensor memory.  n_rows % 128 == 0, k % 256 == 0, any m >= 1;
 * x is fp16, bf16 or fp32 (ldx % 8 == 0).  bf16 and fp32 rows are staged to fp16 in
 * the workspace with a power-of-two scale per token row, so that rows beyond the
 * fp16 range (max |x| >= 2^15) are carried with one fp16 rounding (none for bf16);
 * the epilogue multiplies the scale back.  The workspace
 * (tlx_prefill_workspace_bytes; zero it once) holds a device error word, the fp16
 * copy of the tokens and their scales, and the split region: when the tiles do not
 * fill the last wave of SMs, the tiles of that wave run as k pieces on the idle SMs
 * and the last piece of each tile sums the pieces' fp32 partials in piece order
 * (deterministic); its counters are left zeroed.
 * act[t][r] = silu((Wg x_t)[r]) * (Wu x_t)[r] in fp32 for IQ3_XXS gate/up (fp32: the
 * product of two large projections can exceed the fp16 range; the down GEMM reads
 * it back through the scaled staging), and
 * y[t][r] = (W x_t)[r] (fp32) for Q6_K W (the down projection); other formats
 * return TLX_ERR_QTYPE.  Replaces pf_gemm3 / pf_gemm3m
 * (engine/pf_gemm3.cu:4-26, :219; engine/pf_gemm3m.cu:184-229). */
size_t tlx_prefill_workspace_bytes(int m, int64_t k);
int tlx_prefill_ffn_gate_up(int qtype, const void* w_gate, const void* w_up, const uint32_t* grid, const void* x,
                            int x_dtype, int64_t ldx, int m, int64_t n_rows, int64_t k, void* act, int64_t ld_act,
                            void* ws, size_t ws_bytes, void* stream);
int tlx_prefill_gemm(int qtype, const void* w, const uint32_t* grid, const void* x, int x_dtype, int64_t ldx, int m,
                     int64_t n_rows, int64_t k, float* y, int64_t ldy, void* ws, size_t ws_bytes, void* stream);

/* ---- W4A8 prefill tier (int8 tokens x linearised IQ3_XXS levels) ------------------
 * tlx_act_quant_q8: fp16 x[m][k] (k % 128 == 0; ldx % 4 == 0, x 8-byte aligned) ->
 * xq int8 [m][ldq] (ldq % 4 == 0, 4-byte aligned), sx fp32 [m][k/128] and rs int32
 * [m][k/128] (contiguous).  Per (token, 128-k chunk):
 * s = max(max|x|, 1e-6) * (1/127) in fp32, xq = clamp(rint(x / s), -127, 127) (IEEE
 * quotient, ties to even), rs = sum of the stored xq; bit-identical to the reference
 * quantiser.  Replaces p8q8x (engine/pfk_q8.cu:24-59, launched at
 * engine/pf_prefill.py:1156).
 * tlx_prefill_w4a8_gate_up: act[t][r] = silu(g) * u (fp32) with g = sum_k Wg[r][k] *
 * xq[t][k] * sx[t][k/128] on the weights' linearised codebook: lut8[4 i + j] is the
 * level (0..15) of IQ3_XXS grid entry i, magnitude j, and a 32-weight group's scale is
 * d * (0.5 + s) * 0.5 * 4.0507 (the reference builds lut8 as
 * clip(rint(grid / 4.0507), 0, 15), engine/pf_prefill.py:994).  w_gate / w_up are the
 * tiled IQ3_XXS weights of tlx_prefill_ffn_gate_up (no second copy of the weights);
 * n_rows % 128 == 0, k % 256 == 0, ldq % 8 == 0.  The workspace is the prefill
 * workspace (tlx_prefill_workspace_bytes(m, k), zeroed once).  The contraction runs on
 * the fp16 tcgen05 path with the quantised operands (each level * (2s+1) exact in fp16,
 * one fp16 rounding per weight and per token value); the output is fp32 where the
 * reference writes fp16.  Replaces p8w4ffn7 (engine/p8_w4ffn7.cu:118-255, launched at
 * engine/pf_prefill.py:1157). */
int tlx_act_quant_q8(const void* x, int64_t ldx, int m, int64_t k, int8_t* xq, int64_t ldq, float* sx, int32_t* rs,
                     void* stream);
int tlx_prefill_w4a8_gate_up(const void* w_gate, const void* w_up, const int8_t* lut8, const int8_t* xq, int64_t ldq,
                             const float* sx, int m, int64_t n_rows, int64_t k, float* act, int64_t ld_act, void* ws,
                             size_t ws_bytes, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* TLX_VERIFY_H */
