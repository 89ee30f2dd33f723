// Peer-memory feature gather for node-range-partitioned features.
//
// Every rank's feature partition is a plain cudaMalloc allocation whose CUDA
// IPC handle the other ranks open once (dgfx_ipc_*), so a rank holds device
// pointers to all partitions. dgfx_gather_rows_p2p then fetches each requested
// row from its owner in one kernel: local rows from this GPU's HBM, remote
// rows with ordinary 16-byte loads through NVLink / NVSwitch. No host
// synchronisation, no sort, no all-to-all; it replaces the halo exchange's
// partition + NCCL all-to-all + scatter sequence (driver.HaloFeatures) when
// peer access is available. Loads are plain ld.global (no TMA, no multicast).
#include <algorithm>
#include <cstring>
#include <string>

#include "common.cuh"

namespace dgfx {
namespace {

// out[i] = partition(owner)[row] for ids[*begin + i], owner = id / rows_per_rank.
// Each thread keeps U independent (id load -> row load) chains in flight to
// cover NVLink latency; 16-byte vectors per row = 1 << lvpr (row widths are
// powers of two here; other widths use the division path).
// Small CTAs (64 threads, <= 32 registers) so the gather can run beside a
// resident sampler kernel (it fills shared memory but leaves registers and
// threads for a few such CTAs per SM) when steps are pipelined.
constexpr int kGatherThreads = 64;

template <int U>
__global__ void __launch_bounds__(kGatherThreads, 32) gather_p2p_kernel(const uint4* const* __restrict__ tables, int32_t world,
                                                          uint32_t rows_per_rank, uint32_t num_nodes, int64_t vpr,
                                                          int lvpr, const int64_t* __restrict__ ids,
                                                          const int64_t* __restrict__ begin,
                                                          const int64_t* __restrict__ end, int64_t max_rows,
                                                          uint4* __restrict__ out) {
  const int64_t lo = *begin;
  int64_t n = *end - lo;
  n = n < max_rows ? n : max_rows;
  const int64_t total = n * vpr;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t base = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; base < total;
       base += stride * U) {
    uint4 x[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t v = base + u * stride;
      x[u] = make_uint4(0, 0, 0, 0);
      if (v < total) {
        const int64_t i = lvpr >= 0 ? (v >> lvpr) : v / vpr;
        const int64_t c = v - i * vpr;
        const int64_t id = ids[lo + i];
        if (id >= 0 && id < num_nodes) {
          const uint32_t o = static_cast<uint32_t>(id) / rows_per_rank;
          if (o < static_cast<uint32_t>(world)) {
            x[u] = __ldg(tables[o] + (static_cast<int64_t>(static_cast<uint32_t>(id) - o * rows_per_rank) * vpr + c));
          }
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t v = base + u * stride;
      if (v < total) out[v] = x[u];
    }
  }
}

}  // namespace
}  // namespace dgfx

using namespace dgfx;

extern "C" int dgfx_device_alloc(size_t bytes, void** d_ptr) {
  if (d_ptr == nullptr) return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_device_alloc: null output");
  *d_ptr = nullptr;
  DGFX_CUDA_TRY(cudaMalloc(d_ptr, bytes == 0 ? 256 : bytes));
  return DGFX_OK;
}

extern "C" int dgfx_device_free(void* d_ptr) {
  if (d_ptr != nullptr) DGFX_CUDA_TRY(cudaFree(d_ptr));
  return DGFX_OK;
}

extern "C" int dgfx_ipc_get_handle(const void* d_ptr, void* handle64) {
  if (d_ptr == nullptr || handle64 == nullptr) return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_ipc_get_handle: null");
  cudaIpcMemHandle_t h;
  DGFX_CUDA_TRY(cudaIpcGetMemHandle(&h, const_cast<void*>(d_ptr)));
  static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
  std::memcpy(handle64, &h, sizeof(h));
  return DGFX_OK;
}

extern "C" int dgfx_ipc_open(const void* handle64, void** d_ptr) {
  if (d_ptr == nullptr || handle64 == nullptr) return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_ipc_open: null");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle64, sizeof(h));
  *d_ptr = nullptr;
  DGFX_CUDA_TRY(cudaIpcOpenMemHandle(d_ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return DGFX_OK;
}

extern "C" int dgfx_ipc_close(void* d_ptr) {
  if (d_ptr != nullptr) DGFX_CUDA_TRY(cudaIpcCloseMemHandle(d_ptr));
  return DGFX_OK;
}

extern "C" int dgfx_gather_rows_p2p(const void* const* d_tables, int32_t world, int64_t rows_per_rank,
                                    int64_t num_nodes, int64_t row_bytes, const int64_t* d_row_ids,
                                    const int64_t* d_begin, const int64_t* d_end, int64_t max_rows, void* d_out,
                                    dgfx_stream stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (d_tables == nullptr || world < 1 || rows_per_rank < 1 || num_nodes < 0 || row_bytes <= 0 ||
      row_bytes % 16 != 0 || max_rows < 0 || d_begin == nullptr || d_end == nullptr) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_gather_rows_p2p: bad arguments");
  }
  if (max_rows == 0) return DGFX_OK;
  if (num_nodes >= (int64_t(1) << 32) || rows_per_rank >= (int64_t(1) << 32)) {
    return fail(DGFX_ERR_UNSUPPORTED, "dgfx_gather_rows_p2p: more than 2^32 - 1 nodes");
  }
  const int64_t vpr = row_bytes / 16;
  int lvpr = -1;
  for (int b = 0; b < 31; ++b) {
    if ((int64_t(1) << b) == vpr) lvpr = b;
  }
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  constexpr int U = 3;
  const int64_t blocks =
      std::min<int64_t>(ceil_div(max_rows * vpr, kGatherThreads * U), static_cast<int64_t>(sms) * 24);
  gather_p2p_kernel<U><<<static_cast<unsigned>(std::max<int64_t>(blocks, 1)), kGatherThreads, 0, stream>>>(
      reinterpret_cast<const uint4* const*>(d_tables), world, static_cast<uint32_t>(rows_per_rank),
      static_cast<uint32_t>(num_nodes), vpr, lvpr, d_row_ids, d_begin, d_end, max_rows, static_cast<uint4*>(d_out));
  DGFX_CUDA_TRY(cudaGetLastError());
  return DGFX_OK;
}
