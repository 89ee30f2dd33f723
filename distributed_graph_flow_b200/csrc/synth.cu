// Seeded synthetic graphs and features (the stand-ins for the benchmark
// datasets), generated on the device so billion-edge inputs take seconds.
//
// Graph: out-degrees follow a discrete power law P(d) ~ d^-alpha (inverse
// transform of a Pareto draw, floor(u^(-1/(alpha-1))), capped: the largest
// k <= max_degree with k^-(alpha-1) >= u, found by binary search in a table
// of those thresholds computed once on the host, so a host restatement of
// the generator gives the same degrees bit for bit), rescaled
// exactly to num_edges by row pointers rowptr[v] = floor(cum_v * E / S) over
// the raw degree prefix sums cum (S = total raw degree). Targets follow a
// power-law popularity: rank r = floor(N * u^3) mapped through the affine
// permutation v = (a * r + b) mod N (gcd(a, N) = 1), so in-degrees are skewed
// and hubs are spread over the id range. Every draw is Philox4x32-10 keyed by
// (seed, stream) with the node or edge index as counter, so the graph is a
// pure function of its parameters.
//
// Features: N(0, 1) by the Box-Muller transform of two Philox uniforms, keyed
// by (seed, node, column) so any node-range partition regenerates identical
// rows.
#include <cuda_bf16.h>

#include <cmath>
#include <string>
#include <vector>

#include "common.cuh"
#include "primitives.cuh"

namespace dgfx {
namespace {

__device__ __forceinline__ double u01(uint32_t hi, uint32_t lo) {
  // 53-bit uniform in [0, 1).
  const uint64_t x = (static_cast<uint64_t>(hi) << 32 | lo) >> 11;
  return static_cast<double>(x) * (1.0 / 9007199254740992.0);
}

// thr[k - 1] = k^-(alpha - 1) for k = 1 .. max_deg (thr[0] = 1 >= u).
__global__ void raw_degree_kernel(int64_t n, const double* __restrict__ thr, int64_t max_deg, uint32_t k0, uint32_t k1,
                                  int64_t* __restrict__ deg) {
  for (int64_t v = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; v < n;
       v += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const U4 r = philox4x32_10(U4{static_cast<uint32_t>(v), static_cast<uint32_t>(v >> 32), 0x5eedu, 1u}, k0, k1);
    const double u = 1.0 - u01(r.x, r.y);  // (0, 1]
    int64_t lo = 1, hi = max_deg;
    while (lo < hi) {
      const int64_t mid = (lo + hi + 1) >> 1;
      if (__ldg(thr + mid - 1) >= u) lo = mid;
      else hi = mid - 1;
    }
    deg[v] = lo;
  }
}

// rowptr[v] = floor(cum[v] * E / S) with cum the exclusive prefix of the raw
// degrees (cum[n] = S, passed separately because rowptr is rewritten).
__global__ void scale_rowptr_kernel(int64_t* __restrict__ rowptr, int64_t n, int64_t E, const int64_t* __restrict__ total) {
  const unsigned __int128 S = static_cast<unsigned __int128>(*total);
  for (int64_t v = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; v <= n;
       v += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const unsigned __int128 c = static_cast<unsigned __int128>(rowptr[v]);
    rowptr[v] = S == 0 ? 0 : static_cast<int64_t>((c * static_cast<unsigned __int128>(E)) / S);
  }
}

// Edge list in source-major order: src[j] = row of j, dst[j] = popular node
// among m targets (rank m * u^3 through an affine permutation of [0, m)).
__global__ void edges_kernel(const int64_t* __restrict__ rowptr, int64_t n, int64_t m, uint64_t perm_a,
                             uint64_t perm_b, uint32_t k0, uint32_t k1, int64_t* __restrict__ src,
                             int64_t* __restrict__ dst) {
  for (int64_t v = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; v < n;
       v += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t b = rowptr[v], e = rowptr[v + 1];
    for (int64_t j = b; j < e; ++j) {
      const U4 r = philox4x32_10(U4{static_cast<uint32_t>(j), static_cast<uint32_t>(j >> 32), 0xd57u, 2u}, k0, k1);
      const double u = u01(r.x, r.y);
      int64_t rank = static_cast<int64_t>(static_cast<double>(m) * u * u * u);
      rank = rank < m ? rank : m - 1;
      const unsigned __int128 t = static_cast<unsigned __int128>(perm_a) * static_cast<uint64_t>(rank) + perm_b;
      src[j] = v;
      dst[j] = static_cast<int64_t>(t % static_cast<uint64_t>(m));
    }
  }
}

__global__ void uniform_int_kernel(int64_t n, int64_t lo, int64_t hi, uint32_t k0, uint32_t k1, uint32_t stream,
                                   int64_t* __restrict__ out) {
  const uint64_t range = static_cast<uint64_t>(hi - lo);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const U4 r = philox4x32_10(U4{static_cast<uint32_t>(i), static_cast<uint32_t>(i >> 32), stream, 3u}, k0, k1);
    out[i] = lo + static_cast<int64_t>(bounded64(static_cast<uint64_t>(r.y) << 32 | r.x, range));
  }
}

template <class T>
__device__ __forceinline__ T from_float(float x);
template <>
__device__ __forceinline__ float from_float<float>(float x) { return x; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_float<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

template <class T>
__global__ void normal_features_kernel(int64_t node_begin, int64_t count, int64_t dim, uint32_t k0, uint32_t k1,
                                       T* __restrict__ out) {
  const int64_t pairs = (dim + 1) / 2;
  const int64_t total = count * pairs;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / pairs, p = i - row * pairs;
    const int64_t v = node_begin + row;
    const U4 r = philox4x32_10(U4{static_cast<uint32_t>(v), static_cast<uint32_t>(v >> 32), static_cast<uint32_t>(p), 4u},
                               k0, k1);
    const double u1 = 1.0 - u01(r.x, r.y);  // (0, 1]
    const double u2 = u01(r.z, r.w);
    const double rad = sqrt(-2.0 * log(u1));
    const double a = 6.283185307179586 * u2;
    out[row * dim + 2 * p] = from_float<T>(static_cast<float>(rad * cos(a)));
    if (2 * p + 1 < dim) out[row * dim + 2 * p + 1] = from_float<T>(static_cast<float>(rad * sin(a)));
  }
}

// Rows of the same N(0, 1) table for an arbitrary list of node ids.
template <class T>
__global__ void normal_rows_kernel(const int64_t* __restrict__ ids, int64_t count, int64_t dim, uint32_t k0, uint32_t k1,
                                   T* __restrict__ out) {
  const int64_t pairs = (dim + 1) / 2;
  const int64_t total = count * pairs;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / pairs, p = i - row * pairs;
    const int64_t v = ids[row];
    const U4 r = philox4x32_10(U4{static_cast<uint32_t>(v), static_cast<uint32_t>(v >> 32), static_cast<uint32_t>(p), 4u},
                               k0, k1);
    const double u1 = 1.0 - u01(r.x, r.y);
    const double u2 = u01(r.z, r.w);
    const double rad = sqrt(-2.0 * log(u1));
    const double a = 6.283185307179586 * u2;
    out[row * dim + 2 * p] = from_float<T>(static_cast<float>(rad * cos(a)));
    if (2 * p + 1 < dim) out[row * dim + 2 * p + 1] = from_float<T>(static_cast<float>(rad * sin(a)));
  }
}

unsigned blocks_for(int64_t n) {
  const int64_t b = ceil_div(std::max<int64_t>(n, 1), 256);
  return static_cast<unsigned>(std::min<int64_t>(b, 148 * 64));
}

uint64_t gcd64(uint64_t a, uint64_t b) {
  while (b) {
    const uint64_t t = a % b;
    a = b;
    b = t;
  }
  return a;
}

}  // namespace
}  // namespace dgfx

using namespace dgfx;

extern "C" int dgfx_synth_graph_workspace_size(int64_t num_nodes, int64_t max_degree, size_t* bytes) {
  if (bytes == nullptr || num_nodes < 1 || max_degree < 1) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_synth_graph_workspace_size");
  }
  *bytes = align_up(sizeof(int64_t) * (num_nodes + 1), 256) + 256 + scan_workspace_bytes(num_nodes + 1) +
           align_up(sizeof(double) * static_cast<size_t>(max_degree), 256) + 1024;
  return DGFX_OK;
}

namespace {
int synth_graph(int64_t num_src, int64_t num_dst, int64_t num_edges, double alpha, int64_t max_degree, uint64_t seed,
                int64_t* d_rowptr, int64_t* d_src, int64_t* d_dst, void* d_workspace, size_t workspace_bytes,
                cudaStream_t stream) {
  if (num_src < 1 || num_dst < 1 || num_edges < 0 || !(alpha > 1.0) || max_degree < 1 || d_rowptr == nullptr) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_synth_graph: bad arguments");
  }
  size_t need = 0;
  DGFX_TRY(dgfx_synth_graph_workspace_size(num_src, max_degree, &need));
  if (d_workspace == nullptr || workspace_bytes < need) return fail(DGFX_ERR_WORKSPACE, "dgfx_synth_graph: workspace");
  Arena arena(d_workspace, workspace_bytes);
  int64_t* deg = arena.take<int64_t>(static_cast<size_t>(num_src + 1));
  double* thr = arena.take<double>(static_cast<size_t>(max_degree));
  {
    std::vector<double> h(static_cast<size_t>(max_degree));
    for (int64_t k = 1; k <= max_degree; ++k) h[k - 1] = std::pow(static_cast<double>(k), -(alpha - 1.0));
    // Pageable source: the copy has been staged when the call returns.
    DGFX_CUDA_TRY(cudaMemcpyAsync(thr, h.data(), h.size() * sizeof(double), cudaMemcpyHostToDevice, stream));
  }
  const uint32_t k0 = static_cast<uint32_t>(seed), k1 = static_cast<uint32_t>(seed >> 32);
  raw_degree_kernel<<<blocks_for(num_src), 256, 0, stream>>>(num_src, thr, max_degree, k0, k1, deg);
  DGFX_CUDA_TRY(cudaGetLastError());
  int64_t* total = arena.take<int64_t>(1);
  DGFX_TRY(exclusive_scan<int64_t>(deg, d_rowptr, num_src, true, arena, stream));
  DGFX_CUDA_TRY(cudaMemcpyAsync(total, d_rowptr + num_src, sizeof(int64_t), cudaMemcpyDeviceToDevice, stream));
  scale_rowptr_kernel<<<blocks_for(num_src + 1), 256, 0, stream>>>(d_rowptr, num_src, num_edges, total);
  DGFX_CUDA_TRY(cudaGetLastError());
  if (d_src != nullptr && d_dst != nullptr) {
    // Affine permutation multiplier coprime with the target count.
    const uint64_t m = static_cast<uint64_t>(num_dst);
    uint64_t a = (0x9E3779B97F4A7C15ull ^ seed) % m;
    if (a < 2) a = 2;
    while (gcd64(a, m) != 1) ++a;
    const uint64_t b = (seed * 0xD1B54A32D192ED03ull) % m;
    edges_kernel<<<blocks_for(num_src), 256, 0, stream>>>(d_rowptr, num_src, num_dst, a, b, k0, k1, d_src, d_dst);
    DGFX_CUDA_TRY(cudaGetLastError());
  }
  return DGFX_OK;
}
}  // namespace

extern "C" int dgfx_synth_graph(int64_t num_nodes, int64_t num_edges, double alpha, int64_t max_degree, uint64_t seed,
                                int64_t* d_rowptr, int64_t* d_src, int64_t* d_dst, void* d_workspace,
                                size_t workspace_bytes, dgfx_stream stream_) {
  return synth_graph(num_nodes, num_nodes, num_edges, alpha, max_degree, seed, d_rowptr, d_src, d_dst, d_workspace,
                     workspace_bytes, reinterpret_cast<cudaStream_t>(stream_));
}

extern "C" int dgfx_synth_bipartite(int64_t num_src, int64_t num_dst, int64_t num_edges, double alpha,
                                    int64_t max_degree, uint64_t seed, int64_t* d_rowptr, int64_t* d_src,
                                    int64_t* d_dst, void* d_workspace, size_t workspace_bytes, dgfx_stream stream_) {
  return synth_graph(num_src, num_dst, num_edges, alpha, max_degree, seed, d_rowptr, d_src, d_dst, d_workspace,
                     workspace_bytes, reinterpret_cast<cudaStream_t>(stream_));
}

extern "C" int dgfx_synth_uniform_int(int64_t n, int64_t lo, int64_t hi, uint64_t seed, uint32_t stream_id,
                                      int64_t* d_out, dgfx_stream stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (n < 0 || hi <= lo || (n > 0 && d_out == nullptr)) return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_synth_uniform_int");
  if (n == 0) return DGFX_OK;
  uniform_int_kernel<<<blocks_for(n), 256, 0, stream>>>(n, lo, hi, static_cast<uint32_t>(seed),
                                                        static_cast<uint32_t>(seed >> 32), stream_id, d_out);
  DGFX_CUDA_TRY(cudaGetLastError());
  return DGFX_OK;
}

extern "C" int dgfx_synth_normal_features(int64_t node_begin, int64_t count, int64_t dim, uint64_t seed, int dtype,
                                          void* d_out, dgfx_stream stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (count < 0 || dim < 1 || (dtype != DGFX_F32 && dtype != DGFX_BF16)) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_synth_normal_features: bad arguments");
  }
  if (count == 0) return DGFX_OK;
  const uint32_t k0 = static_cast<uint32_t>(seed), k1 = static_cast<uint32_t>(seed >> 32);
  const int64_t work = count * ((dim + 1) / 2);
  if (dtype == DGFX_F32) {
    normal_features_kernel<float><<<blocks_for(work), 256, 0, stream>>>(node_begin, count, dim, k0, k1,
                                                                        static_cast<float*>(d_out));
  } else {
    normal_features_kernel<__nv_bfloat16><<<blocks_for(work), 256, 0, stream>>>(node_begin, count, dim, k0, k1,
                                                                                static_cast<__nv_bfloat16*>(d_out));
  }
  DGFX_CUDA_TRY(cudaGetLastError());
  return DGFX_OK;
}

extern "C" int dgfx_synth_normal_rows(const int64_t* d_ids, int64_t count, int64_t dim, uint64_t seed, int dtype,
                                      void* d_out, dgfx_stream stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (count < 0 || dim < 1 || (dtype != DGFX_F32 && dtype != DGFX_BF16)) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_synth_normal_rows: bad arguments");
  }
  if (count == 0) return DGFX_OK;
  const uint32_t k0 = static_cast<uint32_t>(seed), k1 = static_cast<uint32_t>(seed >> 32);
  const int64_t work = count * ((dim + 1) / 2);
  if (dtype == DGFX_F32) {
    normal_rows_kernel<float><<<blocks_for(work), 256, 0, stream>>>(d_ids, count, dim, k0, k1, static_cast<float*>(d_out));
  } else {
    normal_rows_kernel<__nv_bfloat16><<<blocks_for(work), 256, 0, stream>>>(d_ids, count, dim, k0, k1,
                                                                            static_cast<__nv_bfloat16*>(d_out));
  }
  DGFX_CUDA_TRY(cudaGetLastError());
  return DGFX_OK;
}
