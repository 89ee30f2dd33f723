// Edge creation times from node creation times.
//
// Restates propagate_timestamp_to_edges (dgf/src/transform/temporal.py:95-103):
// edge_ts[e] = max(src_ts[src[e]], tgt_ts[tgt[e]]) when both endpoint node
// sets carry a creation time, else the one that does. One thread per edge;
// the ids are bounds-checked on the device (numpy indexing raises on an
// out-of-range index) and the first offending edge is reported.
#include <algorithm>
#include <string>

#include "common.cuh"

namespace dgfx {
namespace {

__global__ void edge_timestamps_kernel(const int64_t* __restrict__ src_ts, int64_t num_src,
                                       const int64_t* __restrict__ dst_ts, int64_t num_dst,
                                       const int64_t* __restrict__ src, const int64_t* __restrict__ dst,
                                       int64_t num_edges, int64_t* __restrict__ out,
                                       unsigned long long* __restrict__ first_bad) {
  for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < num_edges;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int64_t t = 0;
    bool ok = true;
    bool have = false;
    if (src_ts != nullptr) {
      const int64_t i = src[e];
      if (i < 0 || i >= num_src) {
        ok = false;
      } else {
        t = src_ts[i];
        have = true;
      }
    }
    if (dst_ts != nullptr) {
      const int64_t j = dst[e];
      if (j < 0 || j >= num_dst) {
        ok = false;
      } else {
        const int64_t u = dst_ts[j];
        t = have ? (u > t ? u : t) : u;
      }
    }
    if (!ok) atomicMin(first_bad, static_cast<unsigned long long>(e));
    out[e] = t;
  }
}

}  // namespace
}  // namespace dgfx

using namespace dgfx;

extern "C" int dgfx_edge_timestamps(const int64_t* d_src_ts, int64_t num_src, const int64_t* d_dst_ts,
                                    int64_t num_dst, const int64_t* d_src, const int64_t* d_dst, int64_t num_edges,
                                    int64_t* d_out, void* d_workspace, dgfx_stream stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (num_edges < 0 || num_src < 0 || num_dst < 0 || (d_src_ts == nullptr && d_dst_ts == nullptr) ||
      d_workspace == nullptr || (num_edges > 0 && (d_out == nullptr || (d_src_ts != nullptr && d_src == nullptr) ||
                                                   (d_dst_ts != nullptr && d_dst == nullptr)))) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_edge_timestamps: bad arguments");
  }
  if (num_edges == 0) return DGFX_OK;
  auto* first_bad = static_cast<unsigned long long*>(d_workspace);
  DGFX_CUDA_TRY(cudaMemsetAsync(first_bad, 0xFF, sizeof(unsigned long long), stream));
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t blocks = std::min<int64_t>(ceil_div(num_edges, int64_t(256)), int64_t(sms) * 16);
  edge_timestamps_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(d_src_ts, num_src, d_dst_ts, num_dst,
                                                                            d_src, d_dst, num_edges, d_out, first_bad);
  DGFX_CUDA_TRY(cudaGetLastError());
  unsigned long long bad = 0;
  DGFX_CUDA_TRY(cudaMemcpyAsync(&bad, first_bad, sizeof(bad), cudaMemcpyDeviceToHost, stream));
  DGFX_CUDA_TRY(cudaStreamSynchronize(stream));
  if (bad != ~0ull) {
    return fail(DGFX_ERR_INVALID_ARGUMENT,
                "dgfx_edge_timestamps: edge " + std::to_string(bad) + " has an endpoint index out of bounds");
  }
  return DGFX_OK;
}

// ---------------------------------------------------------------------------
// Merged-batch adjacency (dgf/src/transform/merge.py:165-197): the edges of
// edge set e of every sample, in sample order, shifted from per-sample local
// ids to merged ids (+ the sample's first node in the source / target node
// set), then padding edges (sentinel_src, sentinel_dst) up to num_out.
// node_offsets / edge_offsets follow the merged-batch layout: set-major, then
// sample, with a trailing total. One warp per sample; padding grid-stride.
// ---------------------------------------------------------------------------
namespace dgfx {
namespace {

__global__ void merge_edgeset_kernel(const int64_t* __restrict__ node_off, const int64_t* __restrict__ edge_off,
                                     const int64_t* __restrict__ esrc, const int64_t* __restrict__ edst, int64_t B,
                                     int32_t e, int32_t s_src, int32_t s_dst, int64_t num_out, int64_t sent_src,
                                     int64_t sent_dst, int64_t* __restrict__ out_src, int64_t* __restrict__ out_dst) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int64_t base = edge_off[e * B];
  const int64_t real = edge_off[(e + 1) * B] - base;
  for (int64_t i = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5; i < B; i += warps) {
    const int64_t a = edge_off[e * B + i], b = edge_off[e * B + i + 1];
    const int64_t so = node_off[s_src * B + i] - node_off[s_src * B];
    const int64_t dof = node_off[s_dst * B + i] - node_off[s_dst * B];
    for (int64_t j = a + lane; j < b; j += 32) {
      const int64_t k = j - base;
      if (k < num_out) {
        out_src[k] = esrc[j] + so;
        out_dst[k] = edst[j] + dof;
      }
    }
  }
  const int64_t tid = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  const int64_t nthreads = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t k = real + tid; k < num_out; k += nthreads) {
    out_src[k] = sent_src;
    out_dst[k] = sent_dst;
  }
}

}  // namespace
}  // namespace dgfx

extern "C" int dgfx_merge_edgeset(const int64_t* d_node_offsets, const int64_t* d_edge_offsets,
                                  const int64_t* d_edge_src, const int64_t* d_edge_dst, int64_t batch,
                                  int32_t edgeset, int32_t src_nodeset, int32_t dst_nodeset, int64_t num_out,
                                  int64_t sentinel_src, int64_t sentinel_dst, int64_t* d_out_src,
                                  int64_t* d_out_dst, dgfx_stream stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (batch < 0 || edgeset < 0 || src_nodeset < 0 || dst_nodeset < 0 || num_out < 0 || d_node_offsets == nullptr ||
      d_edge_offsets == nullptr || (num_out > 0 && (d_out_src == nullptr || d_out_dst == nullptr))) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_merge_edgeset: bad arguments");
  }
  if (num_out == 0) return DGFX_OK;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t work = std::max<int64_t>(batch * 32, num_out);
  const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>(ceil_div(work, int64_t(256)), int64_t(sms) * 16));
  merge_edgeset_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
      d_node_offsets, d_edge_offsets, d_edge_src, d_edge_dst, batch, edgeset, src_nodeset, dst_nodeset, num_out,
      sentinel_src, sentinel_dst, d_out_src, d_out_dst);
  DGFX_CUDA_TRY(cudaGetLastError());
  return DGFX_OK;
}
