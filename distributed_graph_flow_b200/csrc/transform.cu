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
