// Device CSR builder: one direction of one edgeset.
//
// Same result as AdjacencyIndex::CreateFromEdgeList (dgf/src/sampling/
// in_memory_sampler.cc:220-257) behind BuildAdjacencyIndex (dgf/src/sampling/
// in_memory_sampler_ext.cc:1020-1093): the edges of each source are ordered by
// (timestamp, target) — by target only for non-temporal edgesets — and
// duplicates are kept. The sort is a stable LSD radix sort, so equal edges
// keep their input order.
//
// Key layout: when bits(src) + bits(ts range) + bits(dst) <= 64 one 64-bit
// key (src | ts - ts_min | dst) is sorted once; otherwise the three fields are
// sorted as successive stable passes (dst, then ts, then src).
#include <limits>
#include <string>

#include "common.cuh"
#include "primitives.cuh"

namespace dgfx {
namespace {

constexpr int kThreads = 256;

inline unsigned grid_for(int64_t n, int threads = kThreads) {
  const int64_t b = ceil_div(n, threads);
  return static_cast<unsigned>(b < 1 ? 1 : (b > (1ll << 30) ? (1ll << 30) : b));
}

__global__ void validate_kernel(const int64_t* __restrict__ s, const int64_t* __restrict__ d, int64_t n,
                                int64_t num_src, int64_t num_dst, unsigned long long* first_bad) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t a = s[i], b = d[i];
    if (a < 0 || a >= num_src || b < 0 || b >= num_dst) atomicMin(first_bad, static_cast<unsigned long long>(i));
  }
}

__global__ void minmax_kernel(const int64_t* __restrict__ ts, int64_t n, long long* mn, long long* mx) {
  long long lo = 0x7fffffffffffffffll, hi = -0x7fffffffffffffffll - 1;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const long long v = ts[i];
    lo = v < lo ? v : lo;
    hi = v > hi ? v : hi;
  }
  for (int o = 16; o > 0; o >>= 1) {
    const long long l2 = __shfl_xor_sync(0xffffffffu, lo, o), h2 = __shfl_xor_sync(0xffffffffu, hi, o);
    lo = l2 < lo ? l2 : lo;
    hi = h2 > hi ? h2 : hi;
  }
  if ((threadIdx.x & 31) == 0) {
    atomicMin(mn, lo);
    atomicMax(mx, hi);
  }
}

// key = s << (bt + bd) | (ts - ts_min) << bd | d ; val = edge index.
__global__ void pack_keys_kernel(const int64_t* __restrict__ s, const int64_t* __restrict__ d,
                                 const int64_t* __restrict__ ts, int64_t n, int bt, int bd, long long ts_min,
                                 uint64_t* __restrict__ keys, uint32_t* __restrict__ vals) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    uint64_t k = static_cast<uint64_t>(s[i]) << (bt + bd);
    if (ts != nullptr) k |= (static_cast<uint64_t>(ts[i]) - static_cast<uint64_t>(ts_min)) << bd;
    k |= static_cast<uint64_t>(d[i]);
    keys[i] = k;
    vals[i] = static_cast<uint32_t>(i);
  }
}

// keys[i] = field[perm[i]] (optionally minus an offset, as unsigned).
__global__ void gather_field_kernel(const int64_t* __restrict__ field, const uint32_t* __restrict__ perm, int64_t n,
                                    long long offset, uint64_t* __restrict__ keys) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint32_t e = perm == nullptr ? static_cast<uint32_t>(i) : perm[i];
    keys[i] = static_cast<uint64_t>(field[e]) - static_cast<uint64_t>(offset);
  }
}

__global__ void iota_kernel(uint32_t* __restrict__ v, int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    v[i] = static_cast<uint32_t>(i);
  }
}

__global__ void count_kernel(const int64_t* __restrict__ s, int64_t n, int32_t* __restrict__ counts) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    atomicAdd(&counts[s[i]], 1);
  }
}

__global__ void fill_kernel(const uint32_t* __restrict__ perm, const int64_t* __restrict__ d,
                            const int64_t* __restrict__ ts, int64_t n, int32_t* __restrict__ col,
                            int64_t* __restrict__ ts_out, int64_t* __restrict__ edge_pos) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint32_t e = perm[i];
    col[i] = static_cast<int32_t>(d[e]);
    if (ts_out != nullptr) ts_out[i] = ts[e];
    if (edge_pos != nullptr) edge_pos[e] = i;
  }
}

struct BuildPlan {
  int64_t n, num_src;
  bool has_ts;
};

// Lays out (or, with a null base, sizes) the builder's workspace.
struct BuildBufs {
  unsigned long long* first_bad = nullptr;
  long long* ts_minmax = nullptr;
  uint64_t* k0 = nullptr;
  uint64_t* k1 = nullptr;
  uint32_t* v0 = nullptr;
  uint32_t* v1 = nullptr;
  int32_t* counts = nullptr;
};

void carve(Arena& a, const BuildPlan& p, BuildBufs* b) {
  b->first_bad = a.take<unsigned long long>(1);
  b->ts_minmax = a.take<long long>(2);
  b->k0 = a.take<uint64_t>(static_cast<size_t>(p.n));
  b->k1 = a.take<uint64_t>(static_cast<size_t>(p.n));
  b->v0 = a.take<uint32_t>(static_cast<size_t>(p.n));
  b->v1 = a.take<uint32_t>(static_cast<size_t>(p.n));
  b->counts = a.take<int32_t>(static_cast<size_t>(p.num_src));
}

size_t build_ws_bytes(int64_t n, int64_t num_src, bool has_ts) {
  Arena a(nullptr, 0);
  BuildBufs b;
  carve(a, BuildPlan{n, num_src, has_ts}, &b);
  const size_t fixed = a.used;
  return fixed + std::max(radix_sort_workspace_bytes(n), scan_workspace_bytes(num_src + 1)) + 1024;
}

}  // namespace
}  // namespace dgfx

using namespace dgfx;

extern "C" int dgfx_csr_build_workspace_size(int64_t num_edges, int64_t num_src, int64_t num_dst, int has_ts,
                                             size_t* bytes) {
  if (bytes == nullptr || num_edges < 0 || num_src < 0 || num_dst < 0) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_csr_build_workspace_size: bad arguments");
  }
  // Reversal swaps the roles; size for the larger side.
  *bytes = build_ws_bytes(num_edges, std::max(num_src, num_dst), has_ts != 0);
  return DGFX_OK;
}

extern "C" int dgfx_csr_build(const int64_t* d_src, const int64_t* d_dst, const int64_t* d_ts, int64_t num_edges,
                              int64_t num_src, int64_t num_dst, int reversed, int64_t* d_rowptr, int32_t* d_col,
                              int64_t* d_ts_out, int64_t* d_edge_pos, void* d_workspace, size_t workspace_bytes,
                              dgfx_stream stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (num_edges < 0 || num_src < 0 || num_dst < 0 || d_rowptr == nullptr) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_csr_build: bad arguments");
  }
  if (num_edges > 0 && (d_src == nullptr || d_dst == nullptr || d_col == nullptr)) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_csr_build: null edge arrays");
  }
  if (num_edges >= (int64_t(1) << 32)) {
    return fail(DGFX_ERR_UNSUPPORTED, "dgfx_csr_build: more than 2^32 - 1 edges in one edgeset");
  }
  if (num_src >= (int64_t(1) << 31) || num_dst >= (int64_t(1) << 31)) {
    return fail(DGFX_ERR_UNSUPPORTED, "dgfx_csr_build: more than 2^31 - 1 nodes in one nodeset");
  }
  const int64_t* s = d_src;
  const int64_t* d = d_dst;
  if (reversed) {
    std::swap(num_src, num_dst);
    std::swap(s, d);
  }
  const int64_t n = num_edges;
  const bool has_ts = d_ts != nullptr;
  Arena arena(d_workspace, workspace_bytes);
  if (d_workspace == nullptr || workspace_bytes < build_ws_bytes(n, num_src, has_ts)) {
    return fail(DGFX_ERR_WORKSPACE, "dgfx_csr_build: workspace too small");
  }
  BuildBufs b;
  carve(arena, BuildPlan{n, num_src, has_ts}, &b);

  // 1. Validate ids; report the first invalid edge like the reference.
  if (n > 0) {
    const unsigned long long none = ~0ull;
    DGFX_CUDA_TRY(cudaMemcpyAsync(b.first_bad, &none, sizeof(none), cudaMemcpyHostToDevice, stream));
    validate_kernel<<<grid_for(n), kThreads, 0, stream>>>(s, d, n, num_src, num_dst, b.first_bad);
    DGFX_CUDA_TRY(cudaGetLastError());
    unsigned long long bad = 0;
    DGFX_CUDA_TRY(cudaMemcpyAsync(&bad, b.first_bad, sizeof(bad), cudaMemcpyDeviceToHost, stream));
    DGFX_CUDA_TRY(cudaStreamSynchronize(stream));
    if (bad != none) {
      int64_t a = 0, c = 0;
      DGFX_CUDA_TRY(cudaMemcpy(&a, s + bad, sizeof(a), cudaMemcpyDeviceToHost));
      DGFX_CUDA_TRY(cudaMemcpy(&c, d + bad, sizeof(c), cudaMemcpyDeviceToHost));
      if (a < 0 || a >= num_src) {
        return fail(DGFX_ERR_INVALID_ARGUMENT, "Invalid source node index " + std::to_string(a) +
                                                   ". The node index should be between 0 and " +
                                                   std::to_string(num_src) + ".");
      }
      return fail(DGFX_ERR_INVALID_ARGUMENT, "Invalid target node index " + std::to_string(c) +
                                                 ". The node index should be between 0 and " +
                                                 std::to_string(num_dst) + ".");
    }
  }

  // 2. Row pointers from per-source counts.
  if (num_src > 0) DGFX_CUDA_TRY(cudaMemsetAsync(b.counts, 0, sizeof(int32_t) * num_src, stream));
  if (n > 0) {
    count_kernel<<<grid_for(n), kThreads, 0, stream>>>(s, n, b.counts);
    DGFX_CUDA_TRY(cudaGetLastError());
  }
  {
    Arena scan_ws = arena;
    DGFX_TRY(exclusive_scan<int32_t>(b.counts, d_rowptr, num_src, true, scan_ws, stream));
  }
  if (n == 0) return DGFX_OK;

  // 3. Sort.
  long long ts_min = 0;
  int bt = 0;
  if (has_ts) {
    long long init[2] = {std::numeric_limits<long long>::max(), std::numeric_limits<long long>::min()};
    DGFX_CUDA_TRY(cudaMemcpyAsync(b.ts_minmax, init, sizeof(init), cudaMemcpyHostToDevice, stream));
    minmax_kernel<<<grid_for(n), kThreads, 0, stream>>>(d_ts, n, b.ts_minmax, b.ts_minmax + 1);
    DGFX_CUDA_TRY(cudaGetLastError());
    long long mm[2];
    DGFX_CUDA_TRY(cudaMemcpyAsync(mm, b.ts_minmax, sizeof(mm), cudaMemcpyDeviceToHost, stream));
    DGFX_CUDA_TRY(cudaStreamSynchronize(stream));
    ts_min = mm[0];
    bt = bit_length(static_cast<uint64_t>(mm[1]) - static_cast<uint64_t>(mm[0]));
  }
  const int bs = bit_length(static_cast<uint64_t>(num_src > 0 ? num_src - 1 : 0));
  const int bd = bit_length(static_cast<uint64_t>(num_dst > 0 ? num_dst - 1 : 0));
  const uint32_t* perm = nullptr;
  Arena sort_ws = arena;
  if (bs + bt + bd <= 64) {
    pack_keys_kernel<<<grid_for(n), kThreads, 0, stream>>>(s, d, has_ts ? d_ts : nullptr, n, bt, bd, ts_min, b.k0,
                                                           b.v0);
    DGFX_CUDA_TRY(cudaGetLastError());
    bool in1 = false;
    DGFX_TRY(radix_sort_pairs(b.k0, b.v0, b.k1, b.v1, n, 0, bs + bt + bd, &in1, sort_ws, stream));
    perm = in1 ? b.v1 : b.v0;
  } else {
    // Successive stable passes, least significant field first.
    uint64_t* ka = b.k0;
    uint32_t* va = b.v0;
    uint64_t* kb = b.k1;
    uint32_t* vb = b.v1;
    iota_kernel<<<grid_for(n), kThreads, 0, stream>>>(va, n);
    DGFX_CUDA_TRY(cudaGetLastError());
    struct Field {
      const int64_t* data;
      long long offset;
      int bits;
    } fields[3] = {{d, 0, bd}, {d_ts, ts_min, bt}, {s, 0, bs}};
    for (const Field& f : fields) {
      if (f.data == nullptr || f.bits == 0) continue;
      gather_field_kernel<<<grid_for(n), kThreads, 0, stream>>>(f.data, va, n, f.offset, ka);
      DGFX_CUDA_TRY(cudaGetLastError());
      bool in1 = false;
      sort_ws = arena;
      DGFX_TRY(radix_sort_pairs(ka, va, kb, vb, n, 0, f.bits, &in1, sort_ws, stream));
      if (in1) {
        std::swap(ka, kb);
        std::swap(va, vb);
      }
    }
    perm = va;
  }

  // 4. Columns, timestamps and the edge -> position map.
  fill_kernel<<<grid_for(n), kThreads, 0, stream>>>(perm, d, has_ts ? d_ts : nullptr, n, d_col,
                                                    has_ts ? d_ts_out : nullptr, d_edge_pos);
  DGFX_CUDA_TRY(cudaGetLastError());
  return DGFX_OK;
}
