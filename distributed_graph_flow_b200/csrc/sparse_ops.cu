// Sparse-matrix helpers around the SpMM (sm_100a):
//   * the GCN / GIN propagation matrices of the reference's sparse layers
//     (dgf/src/learning/jax/layers/homo_gnn_sparse_deferred.py:293, 526):
//     (A + A^T) plus a diagonal, optionally normalised symmetrically;
//   * CSR transposition support (row id of every entry) for the SpMM's
//     backward pass;
//   * the segment-sum backward (a scaled row gather) and segment counts;
//   * the merged sampled batch as a CSR (rows = sampled nodes, columns = the
//     neighbours they sampled, batch coordinates) for the mean aggregation
//     over a sampled subgraph.
// Each kernel is a single pass over its rows or entries; all are HBM-bound
// copies with one or two reads per entry.
#include <cuda_bf16.h>

#include "common.cuh"

namespace dgfx {
namespace {

unsigned grid_for_items(int64_t n, int threads) {
  const int64_t b = ceil_div(std::max<int64_t>(n, 1), threads);
  return static_cast<unsigned>(std::min<int64_t>(b, 148 * 32));
}

// One warp per row of the structure CSR (A + A^T, implicit values 1): copy
// the row's columns, append the diagonal entry, write the values
// (normalised: v / sqrt(d_r) / sqrt(d_c) with d = row sum of the matrix
// including the diagonal).
__global__ void add_diagonal_kernel(const int64_t* __restrict__ rowptr, const int32_t* __restrict__ col, int64_t rows,
                                    float diag, int normalize, int64_t* __restrict__ out_rowptr,
                                    int32_t* __restrict__ out_col, float* __restrict__ out_val) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t r = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; r < rows; r += warps) {
    const int64_t b = rowptr[r], e = rowptr[r + 1];
    const int64_t ob = b + r;  // rows before r each gained one diagonal entry
    const float dr = static_cast<float>(e - b) + diag;
    const float sr = normalize ? rsqrtf(dr) : 1.0f;
    for (int64_t j = b + lane; j < e; j += 32) {
      const int32_t c = col[j];
      float v = 1.0f;
      if (normalize) {
        const float dc = static_cast<float>(rowptr[c + 1] - rowptr[c]) + diag;
        v = sr * rsqrtf(dc);
      }
      out_col[ob + (j - b)] = c;
      out_val[ob + (j - b)] = v;
    }
    if (lane == 0) {
      out_col[ob + (e - b)] = static_cast<int32_t>(r);
      out_val[ob + (e - b)] = normalize ? diag * sr * sr : diag;
      out_rowptr[r] = ob;
      if (r == rows - 1) out_rowptr[rows] = e + rows;
    }
  }
}

// out[j] = row of entry j.
__global__ void row_ids_kernel(const int64_t* __restrict__ rowptr, int64_t rows, int64_t* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t r = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; r < rows; r += warps) {
    for (int64_t j = rowptr[r] + lane; j < rowptr[r + 1]; j += 32) out[j] = r;
  }
}

__global__ void segment_counts_kernel(const int64_t* __restrict__ ids, int64_t n, int64_t nseg,
                                      int32_t* __restrict__ cnt) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t s = ids[i];
    if (s >= 0 && s < nseg) atomicAdd(&cnt[s], 1);
  }
}

template <class T>
__device__ __forceinline__ float to_f(T x);
template <>
__device__ __forceinline__ float to_f<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <class T>
__device__ __forceinline__ T from_f(float x);
template <>
__device__ __forceinline__ float from_f<float>(float x) { return x; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

// out[i, :] = src[ids[i], :] * (cnt ? 1 / max(cnt[ids[i]], 1) : 1); zero rows
// for ids outside [0, nseg).
template <class T>
__global__ void gather_scaled_kernel(const T* __restrict__ src, const int64_t* __restrict__ ids, int64_t n,
                                     int64_t nseg, int64_t feat, const int32_t* __restrict__ cnt, T* __restrict__ out) {
  const int64_t total = n * feat;
  for (int64_t k = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; k < total;
       k += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t i = k / feat, f = k - i * feat;
    const int64_t s = ids[i];
    float v = 0.0f;
    if (s >= 0 && s < nseg) {
      v = to_f<T>(src[s * feat + f]);
      if (cnt != nullptr) v /= static_cast<float>(max(cnt[s], 1));
    }
    out[k] = from_f<T>(v);
  }
}

// Merged sampled batch (one node set, one edge set) as a CSR over batch
// nodes: row = the batch index of an edge's source, column = the batch
// index of its target. One warp per sample; a sample's edges are sorted by
// local source, so its rows are contiguous. Rows past the batch's node
// count (up to the capacity) are empty.
__global__ void batch_csr_kernel(const int64_t* __restrict__ node_off, const int64_t* __restrict__ edge_off,
                                 const int64_t* __restrict__ edge_src, const int64_t* __restrict__ edge_dst, int64_t B,
                                 int64_t node_cap, int64_t* __restrict__ rowptr, int32_t* __restrict__ col) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int64_t w0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  for (int64_t i = w0; i < B; i += warps) {
    const int64_t nb = node_off[i], nn = node_off[i + 1] - nb;
    const int64_t eb = edge_off[i], ne = edge_off[i + 1] - eb;
    for (int64_t l = lane; l < nn; l += 32) {  // first edge with local source >= l
      int64_t lo = 0, hi = ne;
      while (lo < hi) {
        const int64_t mid = (lo + hi) >> 1;
        if (edge_src[eb + mid] < l) lo = mid + 1;
        else hi = mid;
      }
      rowptr[nb + l] = eb + lo;
    }
    for (int64_t j = lane; j < ne; j += 32) col[eb + j] = static_cast<int32_t>(nb + edge_dst[eb + j]);
  }
  // Tail rows [total nodes, capacity]: empty.
  const int64_t total_n = node_off[B], total_e = edge_off[B];
  const int64_t threads = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t r = total_n + static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; r <= node_cap; r += threads) {
    rowptr[r] = total_e;
  }
}

// Mean aggregation over a merged sampled batch in one pass: one warp per
// batch node v. Its sample i comes from a binary search of the node
// offsets, its edges (a sample's edges are sorted by local source) from a
// binary search of the sample's sources; each lane owns 16-byte chunks of
// the feature row and sums the neighbours' chunks in edge order (fp32), four
// rows in flight. out[v] = that sum / max(count, 1). Rows past the batch's
// node count are not written.
template <class T>
__device__ __forceinline__ void chunk_add(const uint4& r, float* acc);
template <>
__device__ __forceinline__ void chunk_add<float>(const uint4& r, float* acc) {
  acc[0] += __uint_as_float(r.x);
  acc[1] += __uint_as_float(r.y);
  acc[2] += __uint_as_float(r.z);
  acc[3] += __uint_as_float(r.w);
}
template <>
__device__ __forceinline__ void chunk_add<__nv_bfloat16>(const uint4& r, float* acc) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&r);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float2 f = __bfloat1622float2(h[q]);
    acc[2 * q] += f.x;
    acc[2 * q + 1] += f.y;
  }
}
template <class T>
__device__ __forceinline__ uint4 chunk_pack(const float* acc, float scale);
template <>
__device__ __forceinline__ uint4 chunk_pack<float>(const float* acc, float scale) {
  return make_uint4(__float_as_uint(acc[0] * scale), __float_as_uint(acc[1] * scale), __float_as_uint(acc[2] * scale),
                    __float_as_uint(acc[3] * scale));
}
template <>
__device__ __forceinline__ uint4 chunk_pack<__nv_bfloat16>(const float* acc, float scale) {
  uint4 r;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&r);
#pragma unroll
  for (int q = 0; q < 4; ++q) h[q] = __floats2bfloat162_rn(acc[2 * q] * scale, acc[2 * q + 1] * scale);
  return r;
}

// One warp per sample: the sample's (src, dst) edges, sorted by src, are read
// 32 at a time into lanes and walked in order with shuffle broadcasts; lane
// ch sums 16-byte chunk ch of the destination rows (four rows loaded ahead),
// and a node's mean is written when its run of edges ends, zero rows for the
// nodes without edges in between. No per-node searches: a node's work is
// its own edges' row loads.
template <class T>
__device__ __forceinline__ void batch_mean_flush(uint4* __restrict__ out, int64_t nb, int64_t node_cap, int64_t chunks,
                                                 int64_t ch, bool on, int64_t cur, int64_t cnt, const float* acc,
                                                 int64_t* next) {
  if (cur >= 0) {  // the mean of node cur's run of edges
    if (on && nb + cur < node_cap) {
      out[(nb + cur) * chunks + ch] = chunk_pack<T>(acc, 1.0f / static_cast<float>(cnt > 1 ? cnt : 1));
    }
    *next = cur + 1;
  }
}

template <class T>
__global__ void batch_mean_kernel(const int64_t* __restrict__ node_off, const int64_t* __restrict__ edge_off,
                                  const int64_t* __restrict__ edge_src, const int64_t* __restrict__ edge_dst,
                                  int64_t B, int64_t node_cap, const uint4* __restrict__ feats, int64_t chunks,
                                  uint4* __restrict__ out) {
  constexpr int V = 16 / sizeof(T);
  constexpr int kAhead = 4;
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; i < B; i += warps) {
    const int64_t nb = node_off[i], nn = node_off[i + 1] - nb;
    const int64_t eb = edge_off[i], ne = edge_off[i + 1] - eb;
    for (int64_t c0 = 0; c0 < chunks; c0 += 32) {
      const int64_t ch = c0 + lane;
      const bool on = ch < chunks;
      int64_t cur = -1, cnt = 0, next = 0;
      float acc[V];
#pragma unroll
      for (int q = 0; q < V; ++q) acc[q] = 0.0f;
      for (int64_t k0 = 0; k0 < ne; k0 += 32) {
        const int m = static_cast<int>(ne - k0 < 32 ? ne - k0 : 32);
        const int64_t my_s = lane < m ? edge_src[eb + k0 + lane] : 0;
        const int64_t my_d = lane < m ? edge_dst[eb + k0 + lane] : 0;
        for (int j0 = 0; j0 < m; j0 += kAhead) {
          int64_t src[kAhead];
          uint4 r[kAhead];
#pragma unroll
          for (int u = 0; u < kAhead; ++u) {
            const int j = (j0 + u) & 31;
            src[u] = __shfl_sync(0xffffffffu, my_s, j);
            const int64_t d = __shfl_sync(0xffffffffu, my_d, j);
            r[u] = (on && j0 + u < m) ? __ldg(feats + (nb + d) * chunks + ch) : make_uint4(0, 0, 0, 0);
          }
#pragma unroll
          for (int u = 0; u < kAhead; ++u) {
            if (j0 + u >= m) break;  // uniform over the warp
            if (src[u] != cur) {
              batch_mean_flush<T>(out, nb, node_cap, chunks, ch, on, cur, cnt, acc, &next);
              for (int64_t z = next; z < src[u]; ++z) {  // nodes without edges before this run
                if (on && nb + z < node_cap) out[(nb + z) * chunks + ch] = make_uint4(0, 0, 0, 0);
              }
              next = src[u];
              cur = src[u];
              cnt = 0;
#pragma unroll
              for (int q = 0; q < V; ++q) acc[q] = 0.0f;
            }
            chunk_add<T>(r[u], acc);
            ++cnt;
          }
        }
      }
      batch_mean_flush<T>(out, nb, node_cap, chunks, ch, on, cur, cnt, acc, &next);
      for (int64_t z = next; z < nn; ++z) {  // trailing nodes without edges
        if (on && nb + z < node_cap) out[(nb + z) * chunks + ch] = make_uint4(0, 0, 0, 0);
      }
    }
  }
}

}  // namespace
}  // namespace dgfx

__global__ void publish_totals_kernel(const int64_t* __restrict__ a, const int64_t* __restrict__ b,
                                      int64_t* out2) {
  const int64_t x = *a, y = *b;
  out2[1] = y;
  out2[0] = x;
}

using namespace dgfx;

extern "C" int dgfx_publish_totals(const int64_t* d_node_total, const int64_t* d_edge_total, int64_t* out2,
                                   dgfx_stream stream_) {
  if (d_node_total == nullptr || d_edge_total == nullptr || out2 == nullptr) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_publish_totals: null pointer");
  }
  publish_totals_kernel<<<1, 1, 0, reinterpret_cast<cudaStream_t>(stream_)>>>(d_node_total, d_edge_total, out2);
  DGFX_CUDA_TRY(cudaGetLastError());
  return DGFX_OK;
}

extern "C" int dgfx_graph_launch_with_inputs(void* graph_exec, void* dst0, const void* src0, size_t bytes0,
                                             void* dst1, const void* src1, size_t bytes1, dgfx_stream stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (graph_exec == nullptr || (bytes0 > 0 && (dst0 == nullptr || src0 == nullptr)) ||
      (bytes1 > 0 && (dst1 == nullptr || src1 == nullptr))) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_graph_launch_with_inputs: bad arguments");
  }
  if (bytes0 > 0) DGFX_CUDA_TRY(cudaMemcpyAsync(dst0, src0, bytes0, cudaMemcpyDefault, stream));
  if (bytes1 > 0) DGFX_CUDA_TRY(cudaMemcpyAsync(dst1, src1, bytes1, cudaMemcpyDefault, stream));
  DGFX_CUDA_TRY(cudaGraphLaunch(reinterpret_cast<cudaGraphExec_t>(graph_exec), stream));
  return DGFX_OK;
}

extern "C" int dgfx_batch_mean(const int64_t* d_node_offsets, const int64_t* d_edge_offsets, const int64_t* d_edge_src,
                               const int64_t* d_edge_dst, int64_t num_seeds, int64_t node_capacity,
                               const void* d_feats, int dtype, int64_t feat, void* d_out, dgfx_stream stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (num_seeds < 0 || node_capacity < 0 || feat <= 0 || d_node_offsets == nullptr || d_edge_offsets == nullptr ||
      (dtype != DGFX_F32 && dtype != DGFX_BF16)) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_batch_mean: bad arguments");
  }
  const int64_t row_bytes = feat * (dtype == DGFX_F32 ? 4 : 2);
  if (row_bytes % 16 != 0 || reinterpret_cast<uintptr_t>(d_feats) % 16 != 0 ||
      reinterpret_cast<uintptr_t>(d_out) % 16 != 0) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_batch_mean: rows must be a multiple of 16 bytes, 16-byte aligned");
  }
  if (num_seeds == 0 || node_capacity == 0) return DGFX_OK;
  const int64_t chunks = row_bytes / 16;
  const unsigned g = grid_for_items(num_seeds * 32, 256);  // one warp per sample
  if (dtype == DGFX_F32) {
    batch_mean_kernel<float><<<g, 256, 0, stream>>>(d_node_offsets, d_edge_offsets, d_edge_src, d_edge_dst, num_seeds,
                                                    node_capacity, static_cast<const uint4*>(d_feats), chunks,
                                                    static_cast<uint4*>(d_out));
  } else {
    batch_mean_kernel<__nv_bfloat16><<<g, 256, 0, stream>>>(d_node_offsets, d_edge_offsets, d_edge_src, d_edge_dst,
                                                            num_seeds, node_capacity,
                                                            static_cast<const uint4*>(d_feats), chunks,
                                                            static_cast<uint4*>(d_out));
  }
  DGFX_CUDA_TRY(cudaGetLastError());
  return DGFX_OK;
}

extern "C" int dgfx_csr_add_diagonal(const int64_t* d_rowptr, const int32_t* d_col, int64_t num_rows, float diag,
                                     int32_t normalize_symmetric, int64_t* d_out_rowptr, int32_t* d_out_col,
                                     float* d_out_val, dgfx_stream stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (num_rows < 0 || d_rowptr == nullptr || d_out_rowptr == nullptr) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_csr_add_diagonal: bad arguments");
  }
  if (num_rows == 0) {
    DGFX_CUDA_TRY(cudaMemsetAsync(d_out_rowptr, 0, sizeof(int64_t), stream));
    return DGFX_OK;
  }
  if (normalize_symmetric && !(diag > 0.0f)) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_csr_add_diagonal: symmetric normalisation needs a positive diagonal");
  }
  add_diagonal_kernel<<<grid_for_items(num_rows * 32, 256), 256, 0, stream>>>(
      d_rowptr, d_col, num_rows, diag, normalize_symmetric, d_out_rowptr, d_out_col, d_out_val);
  DGFX_CUDA_TRY(cudaGetLastError());
  return DGFX_OK;
}

extern "C" int dgfx_csr_row_ids(const int64_t* d_rowptr, int64_t num_rows, int64_t* d_out, dgfx_stream stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (num_rows < 0 || d_rowptr == nullptr) return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_csr_row_ids: bad arguments");
  if (num_rows == 0) return DGFX_OK;
  row_ids_kernel<<<grid_for_items(num_rows * 32, 256), 256, 0, stream>>>(d_rowptr, num_rows, d_out);
  DGFX_CUDA_TRY(cudaGetLastError());
  return DGFX_OK;
}

extern "C" int dgfx_segment_counts(const int64_t* d_ids, int64_t n, int64_t num_segments, int32_t* d_counts,
                                   dgfx_stream stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (n < 0 || num_segments < 0) return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_segment_counts: bad arguments");
  if (num_segments > 0) DGFX_CUDA_TRY(cudaMemsetAsync(d_counts, 0, sizeof(int32_t) * num_segments, stream));
  if (n == 0) return DGFX_OK;
  segment_counts_kernel<<<grid_for_items(n, 256), 256, 0, stream>>>(d_ids, n, num_segments, d_counts);
  DGFX_CUDA_TRY(cudaGetLastError());
  return DGFX_OK;
}

extern "C" int dgfx_gather_rows_scaled(const void* d_src, int dtype, const int64_t* d_ids, int64_t n,
                                       int64_t num_segments, int64_t feat, const int32_t* d_counts, void* d_out,
                                       dgfx_stream stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (n < 0 || feat <= 0 || num_segments < 0 || (dtype != DGFX_F32 && dtype != DGFX_BF16)) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_gather_rows_scaled: bad arguments");
  }
  if (n == 0) return DGFX_OK;
  const unsigned g = grid_for_items(n * feat, 256);
  if (dtype == DGFX_F32) {
    gather_scaled_kernel<float><<<g, 256, 0, stream>>>(static_cast<const float*>(d_src), d_ids, n, num_segments, feat,
                                                       d_counts, static_cast<float*>(d_out));
  } else {
    gather_scaled_kernel<__nv_bfloat16><<<g, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(d_src), d_ids, n,
                                                               num_segments, feat, d_counts,
                                                               static_cast<__nv_bfloat16*>(d_out));
  }
  DGFX_CUDA_TRY(cudaGetLastError());
  return DGFX_OK;
}

extern "C" int dgfx_batch_csr(const int64_t* d_node_offsets, const int64_t* d_edge_offsets, const int64_t* d_edge_src,
                              const int64_t* d_edge_dst, int64_t num_seeds, int64_t node_capacity, int64_t* d_rowptr,
                              int32_t* d_col, dgfx_stream stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (num_seeds < 0 || node_capacity < 0 || d_node_offsets == nullptr || d_edge_offsets == nullptr ||
      d_rowptr == nullptr) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_batch_csr: bad arguments");
  }
  if (node_capacity >= (int64_t(1) << 31)) return fail(DGFX_ERR_UNSUPPORTED, "dgfx_batch_csr: more than 2^31 nodes");
  const int64_t work = std::max<int64_t>(num_seeds * 32, node_capacity + 1);
  batch_csr_kernel<<<grid_for_items(work, 256), 256, 0, stream>>>(d_node_offsets, d_edge_offsets, d_edge_src,
                                                                  d_edge_dst, num_seeds, node_capacity, d_rowptr,
                                                                  d_col);
  DGFX_CUDA_TRY(cudaGetLastError());
  return DGFX_OK;
}
