// Causal windows of per-node time series (sm_100a).
//
// Replaces the per-sample, per-node loop of filter_timeseries_by_timestamp
// (dgf/src/sampling/temporal.py:24-130), which keeps, for every sampled node,
// the entries of its is_timeseries features whose timestamps are <= the
// seed's timestamp (np.searchsorted(times, cutoff, side="right")), capped to
// the most recent max_timeseries_len entries. Series live in HBM as ragged
// arrays (row offsets + packed values). One thread per sampled node finds its
// window by binary search over its (sorted) timestamp row; a warp per window
// then copies the window's values of each feature into a packed output.
#include <string>

#include "common.cuh"

namespace dgfx {
namespace {

__global__ void ts_window_kernel(const int64_t* __restrict__ off, const int64_t* __restrict__ times,
                                 int64_t num_rows, const int64_t* __restrict__ rows,
                                 const int64_t* __restrict__ cutoffs, int64_t n, int64_t max_len,
                                 int64_t* __restrict__ rel_start, int64_t* __restrict__ len,
                                 unsigned long long* bad) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = rows[i];
    if (r < 0 || r >= num_rows) {
      atomicMin(bad, static_cast<unsigned long long>(i));
      rel_start[i] = 0;
      len[i] = 0;
      continue;
    }
    const int64_t b = off[r];
    const int64_t cut = cutoffs[i];
    int64_t lo = 0, hi = off[r + 1] - b;
    while (lo < hi) {  // first entry with time > cut
      const int64_t mid = (lo + hi) >> 1;
      if (times[b + mid] <= cut) lo = mid + 1;
      else hi = mid;
    }
    const int64_t start = (max_len >= 0 && lo > max_len) ? lo - max_len : 0;
    rel_start[i] = start;
    len[i] = lo - start;
  }
}

// out[out_off[i] .. + len[i]) = values[start[i] .. + len[i]) in elements of
// elem_bytes; a warp per segment, 4-byte words when everything is aligned.
__global__ void gather_segments_kernel(const uint8_t* __restrict__ values, int64_t elem_bytes,
                                       const int64_t* __restrict__ start, const int64_t* __restrict__ len,
                                       const int64_t* __restrict__ out_off, int64_t n, uint8_t* __restrict__ out,
                                       int words) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = int64_t(gridDim.x) * (blockDim.x >> 5);
  for (int64_t i = (blockIdx.x * int64_t(blockDim.x) + threadIdx.x) >> 5; i < n; i += warps) {
    const int64_t nbytes = len[i] * elem_bytes;
    const uint8_t* src = values + start[i] * elem_bytes;
    uint8_t* dst = out + out_off[i] * elem_bytes;
    if (words) {
      const uint32_t* s4 = reinterpret_cast<const uint32_t*>(src);
      uint32_t* d4 = reinterpret_cast<uint32_t*>(dst);
      for (int64_t k = lane; k < nbytes / 4; k += 32) d4[k] = s4[k];
    } else {
      for (int64_t k = lane; k < nbytes; k += 32) dst[k] = src[k];
    }
  }
}

unsigned blocks_for(int64_t n, int threads) {
  return static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(ceil_div(n, threads), 148 * 16)));
}

}  // namespace
}  // namespace dgfx

using namespace dgfx;

extern "C" int dgfx_timeseries_windows(const int64_t* d_row_offsets, const int64_t* d_times, int64_t num_rows,
                                       const int64_t* d_rows, const int64_t* d_cutoffs, int64_t n,
                                       int64_t max_len, int64_t* d_rel_start, int64_t* d_len, void* d_workspace,
                                       dgfx_stream stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (n < 0 || num_rows < 0 || d_workspace == nullptr ||
      (n > 0 && (d_row_offsets == nullptr || d_rows == nullptr || d_cutoffs == nullptr || d_rel_start == nullptr ||
                 d_len == nullptr))) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_timeseries_windows: bad arguments");
  }
  if (n == 0) return DGFX_OK;
  auto* bad = static_cast<unsigned long long*>(d_workspace);
  DGFX_CUDA_TRY(cudaMemsetAsync(bad, 0xFF, sizeof(unsigned long long), stream));
  ts_window_kernel<<<blocks_for(n, 256), 256, 0, stream>>>(d_row_offsets, d_times, num_rows, d_rows, d_cutoffs, n,
                                                           max_len, d_rel_start, d_len, bad);
  DGFX_CUDA_TRY(cudaGetLastError());
  unsigned long long b = 0;
  DGFX_CUDA_TRY(cudaMemcpyAsync(&b, bad, sizeof(b), cudaMemcpyDeviceToHost, stream));
  DGFX_CUDA_TRY(cudaStreamSynchronize(stream));
  if (b != ~0ull) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_timeseries_windows: row id at position " + std::to_string(b) +
                                               " is out of range");
  }
  return DGFX_OK;
}

extern "C" int dgfx_gather_segments(const void* d_values, int64_t elem_bytes, const int64_t* d_start,
                                    const int64_t* d_len, const int64_t* d_out_offsets, int64_t n, void* d_out,
                                    dgfx_stream stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (n < 0 || elem_bytes < 1 ||
      (n > 0 && (d_start == nullptr || d_len == nullptr || d_out_offsets == nullptr))) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_gather_segments: bad arguments");
  }
  if (n == 0) return DGFX_OK;
  const int words = (elem_bytes % 4 == 0 && reinterpret_cast<uintptr_t>(d_values) % 4 == 0 &&
                     reinterpret_cast<uintptr_t>(d_out) % 4 == 0)
                        ? 1
                        : 0;
  gather_segments_kernel<<<blocks_for(n * 32, 256), 256, 0, stream>>>(
      static_cast<const uint8_t*>(d_values), elem_bytes, d_start, d_len, d_out_offsets, n,
      static_cast<uint8_t*>(d_out), words);
  DGFX_CUDA_TRY(cudaGetLastError());
  return DGFX_OK;
}
