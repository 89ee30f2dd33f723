// Halo feature exchange helpers for node-range-partitioned features.
//
// The exchange itself is one NCCL all-to-all of ids and one of rows (issued by
// the host driver); these kernels prepare and consume it:
//   * partition: a stable sort of the requested ids by owner rank
//     (owner = id / rows_per_rank), the permutation back to request order and
//     the per-owner counts;
//   * local gather at the owner (ids shifted by the owner's first node);
//   * scatter of received rows back into request order.
// This replaces the reference's Beam CoGroupByKey feature joins
// (dgf/src/sampling/beam_semi_distributed_sampler_v2.py:271-387).
#include <string>

#include "common.cuh"
#include "primitives.cuh"

namespace dgfx {
namespace {

__global__ void owner_keys_kernel(const int64_t* __restrict__ ids, int64_t n, int64_t rows_per_rank, int32_t world,
                                  uint64_t* __restrict__ keys, uint32_t* __restrict__ vals, int64_t* __restrict__ counts) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int64_t o = ids[i] / rows_per_rank;
    o = o < 0 ? 0 : (o >= world ? world - 1 : o);
    keys[i] = static_cast<uint64_t>(o);
    vals[i] = static_cast<uint32_t>(i);
    atomicAdd(reinterpret_cast<unsigned long long*>(&counts[o]), 1ull);
  }
}

__global__ void permute_ids_kernel(const int64_t* __restrict__ ids, const uint32_t* __restrict__ perm, int64_t n,
                                   int64_t* __restrict__ out) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    out[i] = ids[perm[i]];
  }
}

__global__ void gather_local_kernel(const uint4* __restrict__ table, int64_t rows, int64_t vpr,
                                    const int64_t* __restrict__ ids, int64_t n, int64_t id_base,
                                    uint4* __restrict__ out) {
  const int64_t total = n * vpr;
  for (int64_t v = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; v < total;
       v += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t i = v / vpr, c = v - i * vpr;
    const int64_t r = ids[i] - id_base;
    out[v] = (r >= 0 && r < rows) ? __ldg(table + r * vpr + c) : make_uint4(0, 0, 0, 0);
  }
}

__global__ void scatter_rows_kernel(const uint4* __restrict__ rows, int64_t n, int64_t vpr,
                                    const uint32_t* __restrict__ perm, uint4* __restrict__ out) {
  const int64_t total = n * vpr;
  for (int64_t v = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; v < total;
       v += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t i = v / vpr, c = v - i * vpr;
    out[static_cast<int64_t>(perm[i]) * vpr + c] = rows[v];
  }
}

unsigned blocks_for(int64_t n) {
  const int64_t b = ceil_div(std::max<int64_t>(n, 1), 256);
  return static_cast<unsigned>(std::min<int64_t>(b, 148 * 32));
}

void carve(Arena& a, int64_t n, uint64_t** k0, uint32_t** v0, uint64_t** k1) {
  *k0 = a.take<uint64_t>(static_cast<size_t>(n));
  *v0 = a.take<uint32_t>(static_cast<size_t>(n));
  *k1 = a.take<uint64_t>(static_cast<size_t>(n));
}

}  // namespace
}  // namespace dgfx

using namespace dgfx;

extern "C" int dgfx_halo_partition_workspace_size(int64_t n, int32_t world, size_t* bytes) {
  if (bytes == nullptr || n < 0 || world < 1) return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_halo_partition_workspace_size");
  Arena a(nullptr, 0);
  uint64_t *k0, *k1;
  uint32_t* v0;
  carve(a, n, &k0, &v0, &k1);
  *bytes = a.used + radix_sort_workspace_bytes(n) + 1024;
  return DGFX_OK;
}

extern "C" int dgfx_halo_partition(const int64_t* d_ids, int64_t n, int64_t rows_per_rank, int32_t world,
                                   int64_t* d_sorted_ids, uint32_t* d_perm, int64_t* d_counts, void* d_workspace,
                                   size_t workspace_bytes, dgfx_stream stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (n < 0 || rows_per_rank < 1 || world < 1 || world > 256 || d_counts == nullptr) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_halo_partition: bad arguments");
  }
  if (n >= (int64_t(1) << 32)) return fail(DGFX_ERR_UNSUPPORTED, "dgfx_halo_partition: too many ids");
  size_t need = 0;
  DGFX_TRY(dgfx_halo_partition_workspace_size(n, world, &need));
  if (d_workspace == nullptr || workspace_bytes < need) return fail(DGFX_ERR_WORKSPACE, "dgfx_halo_partition: workspace");
  DGFX_CUDA_TRY(cudaMemsetAsync(d_counts, 0, sizeof(int64_t) * world, stream));
  if (n == 0) return DGFX_OK;
  Arena arena(d_workspace, workspace_bytes);
  uint64_t *k0, *k1;
  uint32_t* v0;
  carve(arena, n, &k0, &v0, &k1);
  owner_keys_kernel<<<blocks_for(n), 256, 0, stream>>>(d_ids, n, rows_per_rank, world, k0, v0, d_counts);
  DGFX_CUDA_TRY(cudaGetLastError());
  bool in1 = false;
  DGFX_TRY(radix_sort_pairs(k0, v0, k1, d_perm, n, 0, std::max(1, bit_length(static_cast<uint64_t>(world - 1))), &in1,
                            arena, stream));
  const uint32_t* perm = in1 ? d_perm : v0;
  if (!in1) DGFX_CUDA_TRY(cudaMemcpyAsync(d_perm, v0, sizeof(uint32_t) * n, cudaMemcpyDeviceToDevice, stream));
  permute_ids_kernel<<<blocks_for(n), 256, 0, stream>>>(d_ids, perm, n, d_sorted_ids);
  DGFX_CUDA_TRY(cudaGetLastError());
  return DGFX_OK;
}

extern "C" int dgfx_gather_rows_local(const void* d_table, int64_t local_rows, int64_t row_bytes,
                                      const int64_t* d_ids, int64_t n, int64_t id_base, void* d_out,
                                      dgfx_stream stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (row_bytes <= 0 || row_bytes % 16 != 0 || n < 0 || local_rows < 0) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_gather_rows_local: bad arguments");
  }
  if (n == 0) return DGFX_OK;
  const int64_t vpr = row_bytes / 16;
  gather_local_kernel<<<blocks_for(n * vpr), 256, 0, stream>>>(static_cast<const uint4*>(d_table), local_rows, vpr,
                                                               d_ids, n, id_base, static_cast<uint4*>(d_out));
  DGFX_CUDA_TRY(cudaGetLastError());
  return DGFX_OK;
}

extern "C" int dgfx_scatter_rows(const void* d_rows, int64_t n, int64_t row_bytes, const uint32_t* d_perm,
                                 void* d_out, dgfx_stream stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (row_bytes <= 0 || row_bytes % 16 != 0 || n < 0) return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_scatter_rows");
  if (n == 0) return DGFX_OK;
  const int64_t vpr = row_bytes / 16;
  scatter_rows_kernel<<<blocks_for(n * vpr), 256, 0, stream>>>(static_cast<const uint4*>(d_rows), n, vpr, d_perm,
                                                               static_cast<uint4*>(d_out));
  DGFX_CUDA_TRY(cudaGetLastError());
  return DGFX_OK;
}
