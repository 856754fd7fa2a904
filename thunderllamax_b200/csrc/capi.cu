// C ABI of the verify-path library (declarations in include/tlx_verify.h).
#include <cuda_runtime.h>

#include <cstdint>
#include <algorithm>
#include <cstring>
#include <vector>

#include <cooperative_groups.h>

#include "common.cuh"
#include "formats.cuh"
#include "tlx_internal.h"

using namespace tlx;

namespace {

constexpr int kEpiStore = 0, kEpiGateUp = 1, kEpiArgmax = 2;
int g_max_ctas = 0;  // 0 = one CTA per SM

inline cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

bool valid_qtype(int qt) {
  return qt == QT_Q6_K || qt == QT_IQ3_XXS || qt == QT_Q4_K || qt == QT_Q5_K || qt == QT_Q8_0;
}
// formats the tile packers know (IQ4_XS is read by the MoE kernels only)
bool valid_pack_qtype(int qt) { return valid_qtype(qt) || qt == QT_IQ4_XS; }

// ---- small kernels -----------------------------------------------------------------

// acc36 semantics (engine/mm/MM_P7_acc36.cu:18-24)
__global__ void accept_kernel(const int32_t* __restrict__ amds, const int32_t* __restrict__ drafts, int k,
                              int32_t* __restrict__ mb, int32_t* __restrict__ eb) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    int m = 0;
    while (m < k && amds[m] == drafts[m]) ++m;
    if (mb) mb[0] = m;
    if (eb) {
      eb[0] = m;
      eb[1] = amds[m];
    }
  }
}

// accept11k semantics (engine/accept11k.cu:23-57); the m ladder is a loop over the
// ten draft ids, the state copies are spread over the CTA
__global__ void accept11k_kernel(const int32_t* __restrict__ amds, const int32_t* __restrict__ drafts,
                                 const float* __restrict__ xA, int32_t* __restrict__ m_slot,
                                 int32_t* __restrict__ m_hist, int32_t* __restrict__ cyc_slot,
                                 int32_t* __restrict__ pos_slot, int32_t* __restrict__ cur_slot,
                                 int32_t* __restrict__ tok_hist, float* __restrict__ h_seed,
                                 const float* __restrict__ hd_d0, const float* __restrict__ hd_d1,
                                 float* __restrict__ dhd_seed, int32_t* __restrict__ emit,
                                 const int32_t* __restrict__ l_hist, int dim) {
  __shared__ int ms;
  if (threadIdx.x == 0) {
    int m = 0;
    while (m < 10 && amds[m] == drafts[m]) ++m;
    const int pos = pos_slot[0];
    for (int t = 0; t <= m; ++t) tok_hist[pos + t] = amds[t];
    cur_slot[0] = amds[m];
    pos_slot[0] = pos + m + 1;
    m_slot[0] = m;
    const int cyc = cyc_slot[0];
    m_hist[cyc] = m;
    emit[0] = pos + m + 1;
    emit[1] = m;
    for (int t = 0; t < 11; ++t) emit[2 + t] = amds[t];
    emit[13] = 0;
    emit[14] = cyc;
    emit[15] = l_hist[cyc];
    cyc_slot[0] = cyc + 1;
    ms = m;
  }
  __syncthreads();
  const int m = ms;
  const float* dh = m == 0 ? hd_d0 : hd_d1;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    if (h_seed && xA) h_seed[i] = xA[static_cast<int64_t>(m) * dim + i];
    if (dhd_seed && dh) dhd_seed[i] = dh[i];
  }
}

// acceptsel11k (engine/acceptsel11k.cu:8-40): the accepted GDN state slot m becomes
// the live slot 4.  rec: m <= 4 from rec4[b][m], m = 5..10 from rec{m+1}x[b]; conv:
// m <= 3 from conv4[b][m], m = 4..10 from conv{m+1}x[b].  An HBM-bound copy over
// all blocks at once (grid-stride, 16-byte vectors when every buffer allows).
struct SelPtrs {
  const float* conv_x[7];  // conv5x .. conv11x
  const float* rec_x[6];   // rec6x .. rec11x
};

template <typename V>
__global__ void acceptsel_kernel(float* __restrict__ rec4, float* __restrict__ conv4,
                                 const int32_t* __restrict__ m_slot, const SelPtrs src, int64_t rec_v,
                                 int64_t conv_v) {
  // blockIdx.y = GDN block b; blockIdx.x strides over that block's rec + conv vectors
  const int m = m_slot[0];
  if (m < 0 || m > 10) return;
  const int64_t b = blockIdx.y;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t t0 = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  // rec: slot m -> slot 4 (m == 4 is the live slot itself: nothing to copy)
  if (m != 4) {
    const V* s = m < 5 ? reinterpret_cast<const V*>(rec4) + (b * 5 + m) * rec_v
                       : reinterpret_cast<const V*>(src.rec_x[m - 5]) + b * rec_v;
    V* d = reinterpret_cast<V*>(rec4) + (b * 5 + 4) * rec_v;
    int64_t i = t0;
    for (; i + 3 * stride < rec_v; i += 4 * stride) {  // four loads in flight per thread
      const V v0 = s[i], v1 = s[i + stride], v2 = s[i + 2 * stride], v3 = s[i + 3 * stride];
      d[i] = v0;
      d[i + stride] = v1;
      d[i + 2 * stride] = v2;
      d[i + 3 * stride] = v3;
    }
    for (; i < rec_v; i += stride) d[i] = s[i];
  }
  const V* s = m < 4 ? reinterpret_cast<const V*>(conv4) + (b * 5 + m) * conv_v
                     : reinterpret_cast<const V*>(src.conv_x[m - 4]) + b * conv_v;
  V* d = reinterpret_cast<V*>(conv4) + (b * 5 + 4) * conv_v;
  for (int64_t i = t0; i < conv_v; i += stride) d[i] = s[i];
}

// GDN state commit as a slot index: the table of every GDN block holds the device
// addresses of the rec and conv buffers of the eleven draft positions (entries 0..10)
// and of the live state (entry 11): tab[(b * 2 + kind) * 12 + s], kind 0 = rec, 1 = conv.
// The flip permutes addresses instead of copying the state (acceptsel11k's 314 MB).
constexpr int kGdnSlots = 12, kGdnLive = 11;

struct GdnInit {
  const float* rec4;
  const float* conv4;
  const float* conv_x[7];  // conv5x .. conv11x
  const float* rec_x[6];   // rec6x .. rec11x
  int64_t rec_elems, conv_elems;
};

// the reference's fixed layout (engine/acceptsel11k.cu:15-39): rec draft m at
// rec4[b][m] for m <= 4 (slot 4 is also the live state) and rec{m+1}x[b] above; conv
// draft m at conv4[b][m] for m <= 3 and conv{m+1}x[b] above, live at conv4[b][4]
__global__ void gdn_slots_init_kernel(uint64_t* __restrict__ tab, const GdnInit in, int n_blocks) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= n_blocks) return;
  uint64_t* r = tab + static_cast<int64_t>(b) * 2 * kGdnSlots;
  uint64_t* c = r + kGdnSlots;
  for (int m = 0; m <= 10; ++m) {
    const float* rp = m <= 4 ? in.rec4 + (static_cast<int64_t>(b) * 5 + m) * in.rec_elems
                             : in.rec_x[m - 5] + static_cast<int64_t>(b) * in.rec_elems;
    const float* cp = m <= 3 ? in.conv4 + (static_cast<int64_t>(b) * 5 + m) * in.conv_elems
                             : in.conv_x[m - 4] + static_cast<int64_t>(b) * in.conv_elems;
    r[m] = reinterpret_cast<uint64_t>(rp);
    c[m] = reinterpret_cast<uint64_t>(cp);
  }
  r[kGdnLive] = reinterpret_cast<uint64_t>(in.rec4 + (static_cast<int64_t>(b) * 5 + 4) * in.rec_elems);
  c[kGdnLive] = reinterpret_cast<uint64_t>(in.conv4 + (static_cast<int64_t>(b) * 5 + 4) * in.conv_elems);
}

// accept m: the live entry takes draft m's buffer and draft m's entry the old live
// buffer (free for the next step's draft m).  rec draft 4 is the live state itself in
// this layout, so the rec flip keeps entries 4 and 11 equal (m == 4: nothing moves).
__global__ void gdn_flip_kernel(uint64_t* __restrict__ tab, const int32_t* __restrict__ m_slot, int n_blocks) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  const int m = m_slot[0];
  if (b >= n_blocks || m < 0 || m > 10) return;
  uint64_t* r = tab + static_cast<int64_t>(b) * 2 * kGdnSlots;
  uint64_t* c = r + kGdnSlots;
  if (m != 4) {
    const uint64_t live = r[kGdnLive];
    r[kGdnLive] = r[m];
    r[4] = r[m];
    r[m] = live;
  }
  const uint64_t live = c[kGdnLive];
  c[kGdnLive] = c[m];
  c[m] = live;
}

// argmax key of one row of materialised logits, reduced over the CTA (valid in
// thread 0): the amx3 / h_argmax scan rules through argmax_key
// Row argmax over materialised logits: one thread-block cluster of kArgmaxCluster
// CTAs per row.  Each CTA scans an interleaved share of the row with 16-byte loads
// (four in flight per thread) and reduces its key (argmax_key: candidates v >
// -1e30, lowest index on ties) through warp shuffles and shared memory; rank 0
// reads the other CTAs' keys from distributed shared memory.  No global scratch,
// so concurrent calls never share state.
constexpr int kArgmaxCluster = 8;
constexpr int kArgmaxThreads = 512;

template <typename T>
__device__ __forceinline__ uint64_t scan_keys(const T* __restrict__ row, int64_t n, int rank, bool vec) {
  constexpr int V = 16 / sizeof(T);
  uint64_t best = 0ull;
  const int64_t t = static_cast<int64_t>(rank) * kArgmaxThreads + threadIdx.x;
  const int64_t stride = static_cast<int64_t>(kArgmaxCluster) * kArgmaxThreads;
  auto take = [&](float v, int64_t i) {
    const uint64_t k = argmax_key(v, static_cast<uint32_t>(i));
    best = k > best ? k : best;
  };
  if (vec) {
    const int64_t nv = n / V;   // whole 16-byte vectors
#pragma unroll 4
    for (int64_t u = t; u < nv; u += stride) {
      const uint4 w = __ldg(reinterpret_cast<const uint4*>(row) + u);
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
      if constexpr (sizeof(T) == 2) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&ws[j]));
          take(f.x, u * V + 2 * j);
          take(f.y, u * V + 2 * j + 1);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) take(__uint_as_float(ws[j]), u * V + j);
      }
    }
    for (int64_t i = nv * V + t; i < n; i += stride) {
      if constexpr (sizeof(T) == 2) take(__half2float(row[i]), i);
      else take(row[i], i);
    }
  } else {
    for (int64_t i = t; i < n; i += stride) {
      if constexpr (sizeof(T) == 2) take(__half2float(row[i]), i);
      else take(row[i], i);
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const uint64_t k = __shfl_xor_sync(0xffffffffu, best, o);
    best = k > best ? k : best;
  }
  return best;
}

// the cluster's key for its row (valid in thread 0 of rank 0); every thread of the
// cluster must call it (it holds two cluster barriers)
template <typename T>
__device__ uint64_t cluster_row_key(const T* __restrict__ row, int64_t n, bool vec) {
  namespace cg = cooperative_groups;
  cg::cluster_group cl = cg::this_cluster();
  const int rank = static_cast<int>(cl.block_rank());
  __shared__ uint64_t wb[kArgmaxThreads / 32];
  __shared__ uint64_t cta_key;
  const uint64_t best = scan_keys(row, n, rank, vec);
  if ((threadIdx.x & 31) == 0) wb[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint64_t b = 0ull;
    for (int w = 0; w < kArgmaxThreads / 32; ++w) b = wb[w] > b ? wb[w] : b;
    cta_key = b;
  }
  cl.sync();   // every CTA's key is in its shared memory
  uint64_t b = 0ull;
  if (rank == 0 && threadIdx.x == 0)
    for (int r = 0; r < kArgmaxCluster; ++r) {
      const uint64_t k = *cl.map_shared_rank(&cta_key, r);
      b = k > b ? k : b;
    }
  cl.sync();   // rank 0 has read every CTA's key before any CTA exits
  return b;
}

// per-row argmax (engine/amx3.cu:117-142): cluster blockIdx.x / kArgmaxCluster = row
template <typename T>
__global__ void __launch_bounds__(kArgmaxThreads) argmax_rows_kernel(const T* __restrict__ logits, int64_t n,
                                                                     int64_t ld, bool vec,
                                                                     int32_t* __restrict__ amds) {
  const int row = blockIdx.x / kArgmaxCluster;
  const uint64_t b = cluster_row_key(logits + row * ld, n, vec);
  if (blockIdx.x % kArgmaxCluster == 0 && threadIdx.x == 0) amds[row] = key_index(b);
}

// h_argmax (T = 1, engine/h_argmax.cu:13-42): the argmax of one row, then the
// decode-loop side effects tok_slot = idx, tok_hist[pos] = idx, pos_slot = pos + 1
template <typename T>
__global__ void __launch_bounds__(kArgmaxThreads) h_argmax_kernel(const T* __restrict__ logits, int64_t n, bool vec,
                                                                  int32_t* __restrict__ tok_slot,
                                                                  int32_t* __restrict__ pos_slot,
                                                                  int32_t* __restrict__ tok_hist) {
  const uint64_t b = cluster_row_key(logits, n, vec);
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    const int32_t idx = key_index(b);
    const int32_t pos = pos_slot[0];
    tok_slot[0] = idx;
    tok_hist[pos] = idx;
    pos_slot[0] = pos + 1;
  }
}

template <typename Kern, typename... Args>
int launch_clusters(Kern kern, int rows, cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(rows * kArgmaxCluster));
  cfg.blockDim = dim3(kArgmaxThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kArgmaxCluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, args...) == cudaSuccess ? TLX_OK : TLX_ERR_LAUNCH;
}

__global__ void argmax_merge_kernel(const uint64_t* __restrict__ keys, int n_shards, int m,
                                    float* __restrict__ out_max, int32_t* __restrict__ out_idx,
                                    const int32_t* __restrict__ drafts, int n_drafts,
                                    int32_t* __restrict__ accept_out) {
  __shared__ int32_t ids[16];
  const int t = threadIdx.x;
  if (t < m) {
    uint64_t b = 0ull;
    for (int s = 0; s < n_shards; ++s) {
      const uint64_t k = keys[s * m + t];
      b = k > b ? k : b;
    }
    if (out_max) out_max[t] = key_value(b);
    if (out_idx) out_idx[t] = key_index(b);
    ids[t] = key_index(b);
  }
  __syncthreads();
  if (t == 0 && accept_out) {
    int mm = 0;
    while (mm < n_drafts && ids[mm] == drafts[mm]) ++mm;
    accept_out[0] = mm;
    accept_out[1] = ids[mm];
  }
}

// device packer: one CTA of 32 threads per (tile, block) chunk
__global__ void pack_tiles_kernel(int qt, const uint8_t* __restrict__ src, int64_t n_rows, int nb, int64_t stride,
                                  uint8_t* __restrict__ dst) {
  const int64_t chunk_id = blockIdx.x;
  const int64_t t = chunk_id / nb;
  const int b = static_cast<int>(chunk_id - t * nb);
  const uint32_t bb = block_bytes(qt);
  const uint8_t* rows[16];
  for (int r = 0; r < 16; ++r) {
    const int64_t row = t * 16 + r;
    rows[r] = row < n_rows ? src + row * stride + static_cast<int64_t>(b) * bb : nullptr;
  }
  uint8_t* out = dst + chunk_id * chunk_bytes(qt);
  pack_lane(qt, rows, threadIdx.x, out);
}

}  // namespace

namespace tlx {
// the CTA cap tlx_set_max_ctas set (0 = one CTA per SM), for the other entry points
int max_ctas_setting() { return g_max_ctas; }
}  // namespace tlx

extern "C" {

const char* tlx_error_string(int code) {
  switch (code) {
    case TLX_OK: return "ok";
    case TLX_ERR_SHAPE: return "unsupported or inconsistent shape";
    case TLX_ERR_ALIGN: return "pointer or stride misaligned";
    case TLX_ERR_DTYPE: return "unsupported activation dtype";
    case TLX_ERR_QTYPE: return "unsupported quantisation type";
    case TLX_ERR_WORKSPACE: return "workspace too small";
    case TLX_ERR_LAUNCH: return "CUDA launch failed";
    case TLX_ERR_DEVICE: return "no sm_100 device";
    case TLX_ERR_NULL: return "required pointer is NULL";
    default: return "unknown error";
  }
}

int tlx_version(void) { return 1; }

int tlx_device_check(void) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return TLX_ERR_DEVICE;
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  return (major == 10 && minor == 0) ? TLX_OK : TLX_ERR_DEVICE;
}

// 0 = one CTA per SM; tests lower it to force split tiles on small shapes
void tlx_set_max_ctas(int n) { g_max_ctas = n < 0 ? 0 : n; }

size_t tlx_tiled_bytes(int qtype, int64_t n_rows, int64_t k) {
  if (!valid_pack_qtype(qtype) || n_rows <= 0 || k <= 0 || k % kQK) return 0;
  const int64_t tiles = (n_rows + 15) / 16;
  return static_cast<size_t>(tiles) * (k / kQK) * chunk_bytes(qtype);
}

int tlx_pack_tiles(int qtype, const void* src, int64_t n_rows, int64_t k, int64_t src_row_stride, void* dst) {
  if (!valid_pack_qtype(qtype)) return TLX_ERR_QTYPE;
  if (!src || !dst) return TLX_ERR_NULL;
  if (n_rows <= 0 || k <= 0 || k % kQK) return TLX_ERR_SHAPE;
  const int nb = static_cast<int>(k / kQK);
  const uint32_t bb = block_bytes(qtype);
  if (src_row_stride < static_cast<int64_t>(nb) * bb) return TLX_ERR_SHAPE;
  const int64_t tiles = (n_rows + 15) / 16;
  const uint8_t* s = static_cast<const uint8_t*>(src);
  uint8_t* d = static_cast<uint8_t*>(dst);
  for (int64_t t = 0; t < tiles; ++t)
    for (int b = 0; b < nb; ++b) {
      const uint8_t* rows[16];
      for (int r = 0; r < 16; ++r) {
        const int64_t row = t * 16 + r;
        rows[r] = row < n_rows ? s + row * src_row_stride + static_cast<int64_t>(b) * bb : nullptr;
      }
      uint8_t* out = d + (t * nb + b) * static_cast<int64_t>(chunk_bytes(qtype));
      for (int lane = 0; lane < 32; ++lane) pack_lane(qtype, rows, lane, out);
    }
  return TLX_OK;
}

int tlx_pack_tiles_device(int qtype, const void* src, int64_t n_rows, int64_t k, int64_t src_row_stride, void* dst,
                          void* stream) {
  if (!valid_pack_qtype(qtype)) return TLX_ERR_QTYPE;
  if (!src || !dst) return TLX_ERR_NULL;
  if (n_rows <= 0 || k <= 0 || k % kQK) return TLX_ERR_SHAPE;
  const int nb = static_cast<int>(k / kQK);
  if (src_row_stride < static_cast<int64_t>(nb) * block_bytes(qtype)) return TLX_ERR_SHAPE;
  const int64_t chunks = (n_rows + 15) / 16 * nb;
  if (chunks > 0x7FFFFFFF) return TLX_ERR_SHAPE;
  pack_tiles_kernel<<<static_cast<unsigned>(chunks), 32, 0, as_stream(stream)>>>(
      qtype, static_cast<const uint8_t*>(src), n_rows, nb, src_row_stride, static_cast<uint8_t*>(dst));
  return cudaGetLastError() == cudaSuccess ? TLX_OK : TLX_ERR_LAUNCH;
}

int tlx_unpack_tiles(int qtype, const void* tiled, int64_t n_rows, int64_t k, void* dst) {
  if (!valid_pack_qtype(qtype)) return TLX_ERR_QTYPE;
  if (!tiled || !dst) return TLX_ERR_NULL;
  if (n_rows <= 0 || k <= 0 || k % kQK) return TLX_ERR_SHAPE;
  const int nb = static_cast<int>(k / kQK);
  const uint32_t bb = block_bytes(qtype), ch = chunk_bytes(qtype);
  const uint8_t* s = static_cast<const uint8_t*>(tiled);
  uint8_t* d = static_cast<uint8_t*>(dst);
  const int64_t row_bytes = static_cast<int64_t>(nb) * bb;
  for (int64_t row = 0; row < n_rows; ++row) {
    const int64_t t = row / 16;
    const int r = static_cast<int>(row % 16), g = r & 7, rr = r >> 3;
    for (int b = 0; b < nb; ++b) {
      const uint8_t* c = s + (t * nb + b) * static_cast<int64_t>(ch);
      uint8_t* blk = d + row * row_bytes + static_cast<int64_t>(b) * bb;
      if (qtype == QT_Q5_K) {
        for (int i = 0; i < 16; ++i) blk[i] = c[2560 + r * 16 + i];
        std::memset(blk + 16, 0, 32);
        for (int q = 0; q < 4; ++q) {
          const int lane = 4 * g + q;
          for (int hf = 0; hf < 2; ++hf)
            for (int j = 0; j < 16; ++j) blk[48 + 32 * q + 16 * hf + j] = c[((2 * rr + hf) * 32 + lane) * 16 + j];
          // the fifth-bit byte of word i: bit order as in pack_q5k_lane
          static const int kLoBit[4] = {4, 0, 5, 1}, kHiBit[4] = {6, 2, 7, 3};
          for (int i = 0; i < 8; ++i) {
            const uint8_t hb = c[2048 + lane * 16 + rr * 8 + i];
            for (int j = 0; j < 4; ++j) {
              blk[16 + 4 * i + j] |= static_cast<uint8_t>(((hb >> kLoBit[j]) & 1u) << (2 * q));
              blk[16 + 4 * i + j] |= static_cast<uint8_t>(((hb >> kHiBit[j]) & 1u) << (2 * q + 1));
            }
          }
        }
      } else if (qtype == QT_Q8_0) {
        for (int q = 0; q < 4; ++q) {
          const int lane = 4 * g + q;
          for (int e = 0; e < 64; ++e)
            blk[34 * (2 * q + (e >> 5)) + 2 + (e & 31)] = c[((4 * rr + (e >> 4)) * 32 + lane) * 16 + (e & 15)];
          for (int cc = 0; cc < 2; ++cc)
            for (int i = 0; i < 2; ++i) blk[34 * (2 * q + cc) + i] = c[4096 + lane * 8 + rr * 4 + cc * 2 + i];
        }
      } else if (qtype == QT_Q4_K) {
        for (int i = 0; i < 16; ++i) blk[i] = c[2048 + r * 16 + i];
        for (int q = 0; q < 4; ++q)
          for (int hf = 0; hf < 2; ++hf)
            for (int j = 0; j < 16; ++j)
              blk[16 + 32 * q + 16 * hf + j] = c[((2 * rr + hf) * 32 + 4 * g + q) * 16 + j];
      } else if (qtype == QT_IQ4_XS) {
        for (int i = 0; i < 8; ++i) blk[i] = c[2048 + g * 16 + rr * 8 + i];
        for (int q = 0; q < 4; ++q)
          for (int hf = 0; hf < 2; ++hf)
            for (int j = 0; j < 16; ++j)
              blk[8 + 32 * q + 16 * hf + j] = c[((2 * rr + hf) * 32 + 4 * g + q) * 16 + j];
      } else if (qtype == QT_IQ3_XXS) {
        blk[0] = c[1536 + g * 4 + rr * 2];
        blk[1] = c[1536 + g * 4 + rr * 2 + 1];
        for (int q = 0; q < 4; ++q) {
          const int lane = 4 * g + q;
          for (int cc = 0; cc < 2; ++cc) {
            const int ib = 2 * q + cc;
            for (int j = 0; j < 8; ++j) blk[2 + 8 * ib + j] = c[rr * 512 + lane * 16 + cc * 8 + j];
            uint32_t u = 0;
            for (int j = 0; j < 4; ++j) u |= static_cast<uint32_t>(c[1024 + lane * 16 + (rr * 2 + cc) * 4 + j]) << (8 * j);
            const uint32_t v = iq3_sign_word_inverse(u);
            for (int j = 0; j < 4; ++j) blk[66 + 4 * ib + j] = static_cast<uint8_t>(v >> (8 * j));
          }
        }
      } else {
        std::memset(blk, 0, 192);
        blk[208] = c[3328 + g * 4 + rr * 2];
        blk[209] = c[3328 + g * 4 + rr * 2 + 1];
        for (int q = 0; q < 4; ++q) {
          const int lane = 4 * g + q;
          for (int j = 0; j < 4; ++j) blk[192 + 4 * q + j] = c[3072 + lane * 8 + j * 2 + rr] ^ 0x80u;
          uint32_t w[24];
          for (int i = 0; i < 24; ++i) std::memcpy(&w[i], c + ((i >> 2) * 32 + lane) * 16 + (i & 3) * 4, 4);
          for (int gam = 0; gam < 8; ++gam) {
            const uint32_t W0 = w[3 * gam], W1 = w[3 * gam + 1], W2 = w[3 * gam + 2];
            uint32_t P[8][2];
            for (int h = 0; h < 2; ++h) {
              const int sh = 16 * h;
              P[0][h] = (W0 >> (sh + 4)) & 63u;
              P[1][h] = (W0 >> (sh + 10)) & 63u;
              P[2][h] = (W1 >> (sh + 4)) & 63u;
              P[3][h] = (W1 >> (sh + 10)) & 63u;
              P[4][h] = (W2 >> (sh + 4)) & 63u;
              P[5][h] = (W2 >> (sh + 10)) & 63u;
              P[6][h] = ((W0 >> sh) & 15u) | (((W2 >> sh) & 3u) << 4);
              P[7][h] = ((W1 >> sh) & 15u) | (((W2 >> (sh + 2)) & 3u) << 4);
            }
            for (int p = 0; p < 8; ++p) {
              const int mu = p >> 2, rsel = p & 3;
              if ((rsel & 1) != rr) continue;
              const int m = 2 * gam + mu;
              for (int h = 0; h < 2; ++h) {
                const int i = 64 * q + 4 * m + 2 * (rsel >> 1) + h;
                const uint32_t v = P[p][h];
                const int hh = i >> 7, j = (i >> 5) & 3, l = i & 31;
                blk[64 * hh + 32 * (j & 1) + l] |= static_cast<uint8_t>((v & 15u) << (4 * (j >> 1)));
                blk[128 + 32 * hh + l] |= static_cast<uint8_t>(((v >> 4) & 3u) << (2 * j));
              }
            }
          }
        }
      }
    }
  }
  return TLX_OK;
}

size_t tlx_gemv_workspace_bytes(int mode, int qtype, int64_t n_rows, int64_t k, int m, int x_dtype) {
  return gemv_workspace_bytes(mode, qtype, n_rows, k, m, x_dtype, g_max_ctas);
}

int tlx_gemv_plan(int mode, int qtype, int64_t n_rows, int64_t k, int m, int x_dtype, int32_t* info, int n_info) {
  return gemv_plan_info(mode, qtype, n_rows, k, m, x_dtype, g_max_ctas, info, n_info);
}

int tlx_workspace_init(void* ws, size_t ws_bytes, void* stream) {
  if (!ws) return TLX_ERR_NULL;
  return cudaMemsetAsync(ws, 0, ws_bytes, as_stream(stream)) == cudaSuccess ? TLX_OK : TLX_ERR_LAUNCH;
}

int tlx_workspace_error(const void* ws, uint32_t* err_out) {
  if (!ws || !err_out) return TLX_ERR_NULL;
  return cudaMemcpy(err_out, ws, 4, cudaMemcpyDeviceToHost) == cudaSuccess ? TLX_OK : TLX_ERR_LAUNCH;
}

size_t tlx_activation_image_bytes(int m, int64_t k, int x_dtype) {
  return activation_image_bytes(m, k, x_dtype);
}

int tlx_stage_activations(const void* x, int x_dtype, int64_t ldx, int m, int64_t k, void* image, void* stream) {
  return stage_activations(x, x_dtype, ldx, m, k, image, as_stream(stream));
}

int tlx_gemv(int qtype, const void* w, const uint32_t* grid, const void* x, int x_dtype, int64_t ldx, int m,
             int64_t n_rows, int64_t k, const float* residual, int64_t ldr, void* y, int y_dtype, int64_t ldy,
             void* ws, size_t ws_bytes, void* stream) {
  return run_gemv(kEpiStore, qtype, w, nullptr, grid, x, x_dtype, ldx, m, n_rows, k, residual, ldr, y, y_dtype, ldy, 0,
                  nullptr, nullptr, nullptr, nullptr, 0, nullptr, ws, ws_bytes, g_max_ctas, as_stream(stream));
}

int tlx_ffn_gate_up(int qtype, const void* w_gate, const void* w_up, const uint32_t* grid, const void* x,
                    int x_dtype, int64_t ldx, int m, int64_t n_rows, int64_t k, void* gact, int gact_dtype,
                    int64_t ldg, void* ws, size_t ws_bytes, void* stream) {
  return run_gemv(kEpiGateUp, qtype, w_gate, w_up, grid, x, x_dtype, ldx, m, n_rows, k, nullptr, 0, gact, gact_dtype,
                  ldg, 0,
                  nullptr, nullptr, nullptr, nullptr, 0, nullptr, ws, ws_bytes, g_max_ctas, as_stream(stream));
}

int tlx_head_argmax(int qtype, const void* w, const uint32_t* grid, const void* x, int x_dtype, int64_t ldx, int m,
                    int64_t n_rows, int64_t k, int64_t row_offset, float* out_max, int32_t* out_idx,
                    uint64_t* out_keys, const int32_t* drafts, int n_drafts, int32_t* accept_out, void* ws,
                    size_t ws_bytes, void* stream) {
  return run_gemv(kEpiArgmax, qtype, w, nullptr, grid, x, x_dtype, ldx, m, n_rows, k, nullptr, 0, nullptr,
                  TLX_DT_F32, 0, row_offset, out_max, out_idx, out_keys, drafts, n_drafts, accept_out, ws, ws_bytes, g_max_ctas,
                  as_stream(stream));
}

int tlx_acceptsel11k(float* rec4, float* conv4, const int32_t* m_slot, const float* const* conv_x,
                     const float* const* rec_x, int n_blocks, int64_t rec_elems, int64_t conv_elems, void* stream) {
  if (!rec4 || !conv4 || !m_slot || !conv_x || !rec_x) return TLX_ERR_NULL;
  if (n_blocks <= 0 || rec_elems <= 0 || conv_elems <= 0) return TLX_ERR_SHAPE;
  SelPtrs src;
  bool vec = (rec_elems % 4) == 0 && (conv_elems % 4) == 0 && (reinterpret_cast<uintptr_t>(rec4) & 15) == 0 &&
             (reinterpret_cast<uintptr_t>(conv4) & 15) == 0;
  for (int i = 0; i < 7; ++i) {
    if (!conv_x[i]) return TLX_ERR_NULL;
    src.conv_x[i] = conv_x[i];
    vec = vec && (reinterpret_cast<uintptr_t>(conv_x[i]) & 15) == 0;
  }
  for (int i = 0; i < 6; ++i) {
    if (!rec_x[i]) return TLX_ERR_NULL;
    src.rec_x[i] = rec_x[i];
    vec = vec && (reinterpret_cast<uintptr_t>(rec_x[i]) & 15) == 0;
  }
  if (n_blocks > 65535) return TLX_ERR_SHAPE;
  // ~ 8 CTAs per SM in total, spread over the blocks
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int per_block = std::max(1, (sms > 0 ? sms : 148) * 8 / n_blocks);
  const dim3 grid(static_cast<unsigned>(per_block), static_cast<unsigned>(n_blocks)), block(256);
  if (vec)
    acceptsel_kernel<float4><<<grid, block, 0, as_stream(stream)>>>(rec4, conv4, m_slot, src, rec_elems / 4,
                                                                     conv_elems / 4);
  else
    acceptsel_kernel<float><<<grid, block, 0, as_stream(stream)>>>(rec4, conv4, m_slot, src, rec_elems, conv_elems);
  return cudaGetLastError() == cudaSuccess ? TLX_OK : TLX_ERR_LAUNCH;
}

size_t tlx_gdn_slots_bytes(int n_blocks) {
  return n_blocks > 0 ? static_cast<size_t>(n_blocks) * 2 * kGdnSlots * sizeof(uint64_t) : 0;
}

int tlx_gdn_slots_init(uint64_t* tab, const float* rec4, const float* conv4, const float* const* conv_x,
                       const float* const* rec_x, int n_blocks, int64_t rec_elems, int64_t conv_elems, void* stream) {
  if (!tab || !rec4 || !conv4 || !conv_x || !rec_x) return TLX_ERR_NULL;
  if (n_blocks <= 0 || rec_elems <= 0 || conv_elems <= 0) return TLX_ERR_SHAPE;
  if (reinterpret_cast<uintptr_t>(tab) & 7) return TLX_ERR_ALIGN;
  GdnInit in;
  in.rec4 = rec4;
  in.conv4 = conv4;
  in.rec_elems = rec_elems;
  in.conv_elems = conv_elems;
  for (int i = 0; i < 7; ++i) {
    if (!conv_x[i]) return TLX_ERR_NULL;
    in.conv_x[i] = conv_x[i];
  }
  for (int i = 0; i < 6; ++i) {
    if (!rec_x[i]) return TLX_ERR_NULL;
    in.rec_x[i] = rec_x[i];
  }
  gdn_slots_init_kernel<<<(n_blocks + 127) / 128, 128, 0, as_stream(stream)>>>(tab, in, n_blocks);
  return cudaGetLastError() == cudaSuccess ? TLX_OK : TLX_ERR_LAUNCH;
}

int tlx_acceptsel11k_flip(uint64_t* tab, const int32_t* m_slot, int n_blocks, void* stream) {
  if (!tab || !m_slot) return TLX_ERR_NULL;
  if (n_blocks <= 0) return TLX_ERR_SHAPE;
  if (reinterpret_cast<uintptr_t>(tab) & 7) return TLX_ERR_ALIGN;
  gdn_flip_kernel<<<(n_blocks + 127) / 128, 128, 0, as_stream(stream)>>>(tab, m_slot, n_blocks);
  return cudaGetLastError() == cudaSuccess ? TLX_OK : TLX_ERR_LAUNCH;
}

static void aq3k8v11_set(Projection (&pr)[3], const void* wq, const void* wk, const void* wv, int64_t nq,
                         int64_t nk, int64_t nv, void* q_out, void* k_out, void* v_out) {
  pr[0] = {QT_IQ3_XXS, wq, nq, q_out};
  pr[1] = {QT_IQ3_XXS, wk, nk, k_out};
  pr[2] = {QT_Q4_K, wv, nv, v_out};
}

size_t tlx_aq3k8v11_workspace_bytes(int m, int64_t k, int64_t nq, int64_t nk, int64_t nv, int x_dtype) {
  Projection pr[3];
  aq3k8v11_set(pr, nullptr, nullptr, nullptr, nq, nk, nv, nullptr, nullptr, nullptr);
  return projections_workspace_bytes(3, pr, m, k, x_dtype, g_max_ctas);
}

int tlx_aq3k8v11_error(const void* ws, int m, int64_t k, int64_t nq, int64_t nk, int64_t nv, int x_dtype,
                       uint32_t* err_out) {
  Projection pr[3];
  aq3k8v11_set(pr, nullptr, nullptr, nullptr, nq, nk, nv, nullptr, nullptr, nullptr);
  return projections_error(ws, 3, pr, m, k, x_dtype, g_max_ctas, err_out);
}

int tlx_aq3k8v11(const void* wq, const void* wk, const void* wv, const uint32_t* grid, const void* x, int x_dtype,
                 int64_t ldx, int m, int64_t k, int64_t nq, int64_t nk, int64_t nv, void* q_out, void* k_out,
                 void* v_out, void* ws, size_t ws_bytes, void* stream) {
  Projection pr[3];
  aq3k8v11_set(pr, wq, wk, wv, nq, nk, nv, q_out, k_out, v_out);
  return run_projections(3, pr, grid, x, x_dtype, ldx, m, k, ws, ws_bytes, g_max_ctas, as_stream(stream));
}

static void q5g8v11_set(Projection (&pr)[2], const void* wqkv, const void* wgate, int64_t nqkv, int64_t ngate,
                        void* qkv_out, void* gate_out) {
  pr[0] = {QT_Q5_K, wqkv, nqkv, qkv_out};
  pr[1] = {QT_IQ3_XXS, wgate, ngate, gate_out};
}

size_t tlx_q5g8v11_workspace_bytes(int m, int64_t k, int64_t nqkv, int64_t ngate, int x_dtype) {
  Projection pr[2];
  q5g8v11_set(pr, nullptr, nullptr, nqkv, ngate, nullptr, nullptr);
  return projections_workspace_bytes(2, pr, m, k, x_dtype, g_max_ctas);
}

int tlx_q5g8v11_error(const void* ws, int m, int64_t k, int64_t nqkv, int64_t ngate, int x_dtype, uint32_t* err_out) {
  Projection pr[2];
  q5g8v11_set(pr, nullptr, nullptr, nqkv, ngate, nullptr, nullptr);
  return projections_error(ws, 2, pr, m, k, x_dtype, g_max_ctas, err_out);
}

int tlx_q5g8v11(const void* wqkv, const void* wgate, const uint32_t* grid, const void* x, int x_dtype, int64_t ldx,
                int m, int64_t k, int64_t nqkv, int64_t ngate, void* qkv_out, void* gate_out, void* ws,
                size_t ws_bytes, void* stream) {
  Projection pr[2];
  q5g8v11_set(pr, wqkv, wgate, nqkv, ngate, qkv_out, gate_out);
  return run_projections(2, pr, grid, x, x_dtype, ldx, m, k, ws, ws_bytes, g_max_ctas, as_stream(stream));
}

int tlx_h_argmax(const void* logits, int dtype, int64_t n, int32_t* tok_slot, int32_t* pos_slot, int32_t* tok_hist,
                 void* stream) {
  if (!logits || !tok_slot || !pos_slot || !tok_hist) return TLX_ERR_NULL;
  if (n <= 0 || n > 0xFFFFFFFFll) return TLX_ERR_SHAPE;
  const bool vec = (reinterpret_cast<uintptr_t>(logits) & 15) == 0;
  if (dtype == TLX_DT_F32)
    return launch_clusters(h_argmax_kernel<float>, 1, as_stream(stream), static_cast<const float*>(logits), n, vec,
                           tok_slot, pos_slot, tok_hist);
  if (dtype == TLX_DT_F16)
    return launch_clusters(h_argmax_kernel<__half>, 1, as_stream(stream), static_cast<const __half*>(logits), n, vec,
                           tok_slot, pos_slot, tok_hist);
  return TLX_ERR_DTYPE;
}

int tlx_argmax_rows(const void* logits, int dtype, int m, int64_t n, int64_t ld, int32_t* amds, void* stream) {
  if (!logits || !amds) return TLX_ERR_NULL;
  if (m <= 0 || n <= 0 || ld < n || n > 0xFFFFFFFFll || m > (1 << 24)) return TLX_ERR_SHAPE;
  const size_t es = dtype == TLX_DT_F32 ? 4 : 2;
  // 16-byte loads when every row starts on a 16-byte boundary
  const bool vec = (reinterpret_cast<uintptr_t>(logits) & 15) == 0 && (static_cast<size_t>(ld) * es) % 16 == 0;
  if (dtype == TLX_DT_F32)
    return launch_clusters(argmax_rows_kernel<float>, m, as_stream(stream), static_cast<const float*>(logits), n, ld,
                           vec, amds);
  if (dtype == TLX_DT_F16)
    return launch_clusters(argmax_rows_kernel<__half>, m, as_stream(stream), static_cast<const __half*>(logits), n,
                           ld, vec, amds);
  return TLX_ERR_DTYPE;
}

size_t tlx_peer_buffer_bytes(int world, int m, int64_t ny) { return peer_buffer_bytes(world, m, ny); }

// the PeerParams of a call: host array of the ranks' buffers as mapped here
static int make_peer(int world, int rank, void* const* bufs, int m, int64_t ny, PeerParams& pr) {
  if (!bufs) return TLX_ERR_NULL;
  if (world < 2 || world > kMaxPeers || rank < 0 || rank >= world) return TLX_ERR_SHAPE;
  pr = PeerParams{};
  pr.world = world;
  pr.rank = rank;
  for (int r = 0; r < world; ++r) pr.base[r] = static_cast<uint8_t*>(bufs[r]);
  pr.m = m;
  pr.ny = ny;
  return TLX_OK;
}

int tlx_gemv_peer(int qtype, const void* w, const uint32_t* grid, const void* x, int x_dtype, int64_t ldx, int m,
                  int64_t n_rows, int64_t k, int world, int rank, void* const* peer_bufs, int max_ctas, void* ws,
                  size_t ws_bytes, void* stream) {
  PeerParams pr;
  const int rc = make_peer(world, rank, peer_bufs, m, n_rows, pr);
  if (rc) return rc;
  if (!valid_qtype(qtype)) return TLX_ERR_QTYPE;
  return run_gemv(kEpiStore, qtype, w, nullptr, grid, x, x_dtype, ldx, m, n_rows, k, nullptr, 0, nullptr, TLX_DT_F32,
                  n_rows, 0, nullptr, nullptr, nullptr, nullptr, 0, nullptr, ws, ws_bytes,
                  max_ctas > 0 ? max_ctas : g_max_ctas, as_stream(stream), &pr);
}

int tlx_head_argmax_peer(int qtype, const void* w, const uint32_t* grid, const void* x, int x_dtype, int64_t ldx,
                         int m, int64_t n_rows, int64_t k, int64_t row_offset, float* out_max, int32_t* out_idx,
                         const int32_t* drafts, int n_drafts, int32_t* accept_out, int world, int rank,
                         void* const* peer_bufs, int max_ctas, void* ws, size_t ws_bytes, void* stream) {
  PeerParams pr;
  const int rc = make_peer(world, rank, peer_bufs, m, 1, pr);
  if (rc) return rc;
  if (!valid_qtype(qtype)) return TLX_ERR_QTYPE;
  return run_gemv(kEpiArgmax, qtype, w, nullptr, grid, x, x_dtype, ldx, m, n_rows, k, nullptr, 0, nullptr,
                  TLX_DT_F32, 0, row_offset, out_max, out_idx, nullptr, drafts, n_drafts, accept_out, ws, ws_bytes,
                  max_ctas > 0 ? max_ctas : g_max_ctas, as_stream(stream), &pr);
}

int tlx_peer_finish(int world, int rank, void* const* peer_bufs, int m, int64_t ny, const float* residual,
                    int64_t ldr, float* y, int64_t ldy, uint32_t* err, void* stream) {
  PeerParams pr;
  const int rc = make_peer(world, rank, peer_bufs, m, ny, pr);
  if (rc) return rc;
  if (!y || !err) return TLX_ERR_NULL;
  if (m < 1 || m > 16 || ny < 1 || ldy < ny || (residual && ldr < ny)) return TLX_ERR_SHAPE;
  for (int r = 0; r < world; ++r)
    if (!pr.base[r] || (reinterpret_cast<uintptr_t>(pr.base[r]) & 255)) return TLX_ERR_ALIGN;
  pr.residual = residual;
  pr.ldr = ldr;
  pr.y = y;
  pr.ldy = ldy;
  return peer_finish(pr, err, as_stream(stream));
}

int tlx_peer_publish(int world, int rank, void* const* peer_bufs, int m, int64_t ny, const float* part, int64_t ldp,
                     void* stream) {
  PeerParams pr;
  const int rc = make_peer(world, rank, peer_bufs, m, ny, pr);
  if (rc) return rc;
  if (!part) return TLX_ERR_NULL;
  if (m < 1 || m > 16 || ny < 1 || ldp < ny) return TLX_ERR_SHAPE;
  for (int r = 0; r < world; ++r)
    if (!pr.base[r] || (reinterpret_cast<uintptr_t>(pr.base[r]) & 255)) return TLX_ERR_ALIGN;
  pr.residual = part;
  pr.ldr = ldp;
  return peer_publish(pr, as_stream(stream));
}

int tlx_argmax_merge(const uint64_t* keys, int n_shards, int m, float* out_max, int32_t* out_idx,
                     const int32_t* drafts, int n_drafts, int32_t* accept_out, void* stream) {
  if (!keys) return TLX_ERR_NULL;
  if (n_shards <= 0 || m <= 0 || m > 16) return TLX_ERR_SHAPE;
  if (accept_out && (!drafts || n_drafts < 0 || n_drafts + 1 > m)) return TLX_ERR_SHAPE;
  argmax_merge_kernel<<<1, 32, 0, as_stream(stream)>>>(keys, n_shards, m, out_max, out_idx, drafts, n_drafts,
                                                       accept_out);
  return cudaGetLastError() == cudaSuccess ? TLX_OK : TLX_ERR_LAUNCH;
}

int tlx_accept(const int32_t* amds, const int32_t* drafts, int k, int32_t* mb, int32_t* eb, void* stream) {
  if (!amds || (k > 0 && !drafts)) return TLX_ERR_NULL;
  if (k < 0) return TLX_ERR_SHAPE;
  accept_kernel<<<1, 32, 0, as_stream(stream)>>>(amds, drafts, k, mb, eb);
  return cudaGetLastError() == cudaSuccess ? TLX_OK : TLX_ERR_LAUNCH;
}

int tlx_accept11k(const int32_t* amds, const int32_t* drafts, const float* xA, int32_t* m_slot, int32_t* m_hist,
                  int32_t* cyc_slot, int32_t* pos_slot, int32_t* cur_slot, int32_t* tok_hist, float* h_seed,
                  const float* hd_d0, const float* hd_d1, float* dhd_seed, int32_t* emit, const int32_t* l_hist,
                  int dim, void* stream) {
  if (!amds || !drafts || !m_slot || !m_hist || !cyc_slot || !pos_slot || !cur_slot || !tok_hist || !emit ||
      !l_hist)
    return TLX_ERR_NULL;
  if (dim < 0) return TLX_ERR_SHAPE;
  accept11k_kernel<<<1, 256, 0, as_stream(stream)>>>(amds, drafts, xA, m_slot, m_hist, cyc_slot, pos_slot, cur_slot,
                                                     tok_hist, h_seed, hd_d0, hd_d1, dhd_seed, emit, l_hist, dim);
  return cudaGetLastError() == cudaSuccess ? TLX_OK : TLX_ERR_LAUNCH;
}

}  // extern "C"
