// Sparse neighbour aggregation and feature gather (sm_100a).
//
// CSR SpMM, row-split: every row becomes ceil(nnz / kChunk) warp tasks (at
// least one). A task accumulates its nnz range in fp32 registers: the warp
// broadcasts (col, val) pairs by shuffle and each lane loads 16-byte slices
// of the gathered X rows (a 256-wide fp32 row is 1 KB: two fully coalesced
// 512-byte warp loads). Rows with one task write Y directly; longer rows
// write fp32 partials that a fixup kernel sums in task order, so results are
// deterministic. This is the HBM-bound gather form of the aggregation
// (sum_j val_j * X[col_j]), which has ~0.5 flop per byte and stays off the
// tensor cores.
//
// References: mean pooling as jax.ops.segment_sum / max(count, 1)
// (dgf/src/learning/jax/layers/hetero_gnn.py:283-295); SparseMatrix @ dense
// (dgf/src/learning/jax/layers/homo_gnn_sparse_deferred.py:138-161, matrix
// built in dgf/src/learning/jax/message_passing.py:24-38); feature gather
// full_feature_value[node_idxs] (dgf/src/sampling/in_memory_sampler.py:
// 338-346).
#include <cuda_bf16.h>

#include <algorithm>
#include <string>

#include "common.cuh"
#include "primitives.cuh"

namespace dgfx {
namespace {

constexpr int kChunk = 256;        // nnz per SpMM task
constexpr int kWarpsPerBlock = 8;  // 256-thread blocks

__device__ __forceinline__ void load_vec(const float* p, float* o) {
  const float4 v = __ldg(reinterpret_cast<const float4*>(p));
  o[0] = v.x;
  o[1] = v.y;
  o[2] = v.z;
  o[3] = v.w;
}
__device__ __forceinline__ void load_vec(const __nv_bfloat16* p, float* o) {
  const uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    o[2 * i] = f.x;
    o[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void store_vec(float* p, const float* o) {
  *reinterpret_cast<float4*>(p) = make_float4(o[0], o[1], o[2], o[3]);
}
__device__ __forceinline__ void store_vec(__nv_bfloat16* p, const float* o) {
  uint4 v;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(o[2 * i], o[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = v;
}

// Stores V consecutive fp32 accumulators as YT (V = 4 or 8).
template <int V>
__device__ __forceinline__ void store_span(float* p, const float* o) {
#pragma unroll
  for (int q = 0; q < V; q += 4) store_vec(p + q, o + q);
}
template <int V>
__device__ __forceinline__ void store_span(__nv_bfloat16* p, const float* o) {
  if constexpr (V == 8) {
    store_vec(p, o);
  } else {
    uint2 v;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&v);
    h[0] = __floats2bfloat162_rn(o[0], o[1]);
    h[1] = __floats2bfloat162_rn(o[2], o[3]);
    *reinterpret_cast<uint2*>(p) = v;
  }
}

template <class T> struct Vec;
template <> struct Vec<float> { static constexpr int n = 4; };
template <> struct Vec<__nv_bfloat16> { static constexpr int n = 8; };

// ---- task planning --------------------------------------------------------
__global__ void spmm_count_kernel(const int64_t* __restrict__ rowptr, int64_t rows, int32_t* __restrict__ cnt,
                                  int32_t* __restrict__ split_cnt) {
  for (int64_t r = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; r < rows;
       r += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t nnz = rowptr[r + 1] - rowptr[r];
    const int64_t c = nnz <= kChunk ? 1 : (nnz + kChunk - 1) / kChunk;
    cnt[r] = static_cast<int32_t>(c);
    split_cnt[r] = c > 1 ? static_cast<int32_t>(c) : 0;
  }
}

__global__ void spmm_fill_kernel(const int64_t* __restrict__ task_off, int64_t rows, int32_t* __restrict__ task_row,
                                 unsigned long long* __restrict__ next_task = nullptr, int num_counters = 1) {
  if (next_task != nullptr && blockIdx.x == 0) {
    for (int i = threadIdx.x; i < num_counters; i += blockDim.x) next_task[i] = 0;  // counters of the launches that follow
  }
  for (int64_t r = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; r < rows;
       r += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    for (int64_t t = task_off[r]; t < task_off[r + 1]; ++t) task_row[t] = static_cast<int32_t>(r);
  }
}

// ---- main kernel ----------------------------------------------------------
// CPL = 16-byte chunks per lane (feature slice per warp = 32 * CPL * VEC);
// U = gathered rows kept in flight per warp. Chunks stay raw (uint4) in
// registers until their FMA so U * CPL loads fit in 64 registers, which keeps
// four 256-thread CTAs (32 warps) resident per SM. The next 32 (col, val)
// pairs are fetched while the current ones are consumed.
__device__ __forceinline__ void unpack(const uint4& r, float* o, const float*) {
  o[0] = __uint_as_float(r.x);
  o[1] = __uint_as_float(r.y);
  o[2] = __uint_as_float(r.z);
  o[3] = __uint_as_float(r.w);
}
__device__ __forceinline__ void unpack(const uint4& r, float* o, const __nv_bfloat16*) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    o[2 * i] = f.x;
    o[2 * i + 1] = f.y;
  }
}

template <class XT, class YT, int CPL, int U>
__global__ void __launch_bounds__(kWarpsPerBlock * 32, 3)
spmm_kernel(const int64_t* __restrict__ rowptr, const int32_t* __restrict__ col, const float* __restrict__ val,
            const XT* __restrict__ X, YT* __restrict__ Y, int64_t feat, int64_t f0, int64_t fw,
            const int64_t* __restrict__ task_off, const int32_t* __restrict__ task_row,
            const int64_t* __restrict__ split_off, float* __restrict__ partial, int64_t rows, int normalize,
            int64_t num_cols, unsigned long long* __restrict__ next_task) {
  constexpr int V = Vec<XT>::n;
  const int lane = threadIdx.x & 31;
  const int64_t ntasks = task_off[rows];
  const int nchunks = static_cast<int>(fw / V);
  auto fetch = [&](int64_t base, int64_t e, int32_t& c, float& w) {
    const int64_t idx = base + lane;
    const bool ok = idx < e;
    c = ok ? (col != nullptr ? col[idx] : static_cast<int32_t>(idx)) : 0;
    w = ok ? (val != nullptr ? val[idx] : 1.f) : 0.f;
    if (c < 0 || c >= num_cols) {  // out-of-range column: no contribution
      c = 0;
      w = 0.f;
    }
  };
  // Tasks (1 to kChunk nonzeros) are taken from a counter, the next index
  // fetched while the current task runs: a static split of power-law rows
  // over the persistent grid leaves warps idle.
  unsigned long long claim = lane == 0 ? atomicAdd(next_task, 1ull) : 0ull;
  for (int64_t t = static_cast<int64_t>(__shfl_sync(0xffffffffu, claim, 0)); t < ntasks;
       t = static_cast<int64_t>(__shfl_sync(0xffffffffu, claim, 0))) {
    claim = lane == 0 ? atomicAdd(next_task, 1ull) : 0ull;
    const int64_t r = task_row[t];
    const int64_t j = t - task_off[r];
    const int64_t rb = rowptr[r], re = rowptr[r + 1];
    const int64_t b = rb + j * kChunk;
    const int64_t e = min(re, b + kChunk);
    float acc[CPL][V];
#pragma unroll
    for (int c = 0; c < CPL; ++c)
#pragma unroll
      for (int i = 0; i < V; ++i) acc[c][i] = 0.f;
    int32_t my_col;
    float my_val;
    fetch(b, e, my_col, my_val);
    for (int64_t base = b; base < e; base += 32) {
      const int m = static_cast<int>(e - base < 32 ? e - base : 32);
      int32_t nx_col;
      float nx_val;
      fetch(base + 32, e, nx_col, nx_val);
      for (int i = 0; i < m; i += U) {
        uint4 raw[U][CPL];
        float wv[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int src = (i + u) & 31;
          const int64_t cc = __shfl_sync(0xffffffffu, my_col, src);
          wv[u] = __shfl_sync(0xffffffffu, my_val, src);
          if (i + u < m) {
            const uint4* row = reinterpret_cast<const uint4*>(X + cc * feat + f0);
#pragma unroll
            for (int c = 0; c < CPL; ++c) {
              const int ch = lane + 32 * c;
              if (ch < nchunks) raw[u][c] = __ldg(row + ch);
            }
          }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          if (i + u < m) {
#pragma unroll
            for (int c = 0; c < CPL; ++c) {
              const int ch = lane + 32 * c;
              if (ch < nchunks) {
                float x[V];
                unpack(raw[u][c], x, X);
#pragma unroll
                for (int q = 0; q < V; ++q) acc[c][q] = fmaf(wv[u], x[q], acc[c][q]);
              }
            }
          }
        }
      }
      my_col = nx_col;
      my_val = nx_val;
    }
    const int64_t ntask_r = task_off[r + 1] - task_off[r];
    if (ntask_r == 1) {
      float scale = 1.f;
      if (normalize) scale = 1.f / static_cast<float>((re - rb > 1 ? re - rb : 1));
      YT* out = Y + r * feat + f0;
#pragma unroll
      for (int c = 0; c < CPL; ++c) {
        const int ch = lane + 32 * c;
        if (ch < nchunks) {
          float o[V];
#pragma unroll
          for (int q = 0; q < V; ++q) o[q] = acc[c][q] * scale;
          store_span<V>(out + ch * V, o);
        }
      }
    } else {
      float* out = partial + (split_off[r] + j) * fw;
#pragma unroll
      for (int c = 0; c < CPL; ++c) {
        const int ch = lane + 32 * c;
        if (ch < nchunks) {
#pragma unroll
          for (int q = 0; q < V; q += 4) store_vec(out + ch * V + q, &acc[c][q]);
        }
      }
    }
  }
}

// Sums the partials of split rows in task order: one warp per row.
template <class YT>
__global__ void spmm_fixup_kernel(const int64_t* __restrict__ rowptr, const int64_t* __restrict__ split_off,
                                  const float* __restrict__ partial, YT* __restrict__ Y, int64_t rows, int64_t feat,
                                  int64_t f0, int64_t fw, int normalize) {
  constexpr int V = Vec<YT>::n;
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t r = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5; r < rows; r += warps) {
    const int64_t s0 = split_off[r], s1 = split_off[r + 1];
    if (s1 - s0 == 0) continue;
    float scale = 1.f;
    if (normalize) scale = 1.f / static_cast<float>((rowptr[r + 1] - rowptr[r] > 1 ? rowptr[r + 1] - rowptr[r] : 1));
    for (int64_t ch = lane; ch < fw / V; ch += 32) {
      float acc[V];
#pragma unroll
      for (int q = 0; q < V; ++q) acc[q] = 0.f;
      for (int64_t s = s0; s < s1; ++s) {
        const float* src = partial + s * fw + ch * V;
#pragma unroll
        for (int q = 0; q < V; q += 4) {
          const float4 v = *reinterpret_cast<const float4*>(src + q);
          acc[q] += v.x;
          acc[q + 1] += v.y;
          acc[q + 2] += v.z;
          acc[q + 3] += v.w;
        }
      }
#pragma unroll
      for (int q = 0; q < V; ++q) acc[q] *= scale;
      store_vec(Y + r * feat + f0 + ch * V, acc);
    }
  }
}

// ---- segment_sum helpers --------------------------------------------------
// rowptr[s] = first item with id >= s (ids sorted ascending), s in [0, nseg].
__global__ void sorted_bounds_kernel(const int64_t* __restrict__ ids, int64_t n, int64_t nseg,
                                     int64_t* __restrict__ rowptr) {
  for (int64_t s = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; s <= nseg;
       s += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int64_t lo = 0, hi = n;
    while (lo < hi) {
      const int64_t mid = (lo + hi) >> 1;
      if (ids[mid] < s) lo = mid + 1;
      else hi = mid;
    }
    rowptr[s] = lo;
  }
}

template <class XT>
__global__ void segment_atomic_kernel(const XT* __restrict__ data, const int64_t* __restrict__ ids, int64_t n,
                                      int64_t feat, int64_t nseg, float* __restrict__ acc, int32_t* __restrict__ cnt) {
  constexpr int V = Vec<XT>::n;
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t i = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5; i < n; i += warps) {
    const int64_t s = ids[i];
    if (s < 0 || s >= nseg) continue;
    if (lane == 0 && cnt != nullptr) atomicAdd(&cnt[s], 1);
    for (int64_t ch = lane; ch < feat / V; ch += 32) {
      float x[V];
      load_vec(data + i * feat + ch * V, x);
#pragma unroll
      for (int q = 0; q < V; q += 4) {
        atomicAdd(reinterpret_cast<float4*>(acc + s * feat + ch * V + q), make_float4(x[q], x[q + 1], x[q + 2], x[q + 3]));
      }
    }
  }
}

template <class YT>
__global__ void segment_finish_kernel(const float* __restrict__ acc, const int32_t* __restrict__ cnt, int64_t nseg,
                                      int64_t feat, YT* __restrict__ out) {
  constexpr int V = Vec<YT>::n;
  const int64_t nvec = nseg * (feat / V);
  for (int64_t v = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; v < nvec;
       v += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t s = v / (feat / V);
    float scale = 1.f;
    if (cnt != nullptr) scale = 1.f / static_cast<float>(max(cnt[s], 1));
    float o[V];
#pragma unroll
    for (int q = 0; q < V; ++q) o[q] = acc[v * V + q] * scale;
    store_vec(out + v * V, o);
  }
}

// ---- gather ---------------------------------------------------------------
__global__ void gather_rows_kernel(const uint4* __restrict__ table, int64_t num_table_rows, int64_t vec_per_row,
                                   const int64_t* __restrict__ ids, int64_t n, uint4* __restrict__ out) {
  const int64_t total = n * vec_per_row;
  for (int64_t v = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; v < total;
       v += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t i = v / vec_per_row, c = v - i * vec_per_row;
    const int64_t r = ids[i];
    uint4 x = make_uint4(0, 0, 0, 0);
    if (r >= 0 && r < num_table_rows) x = __ldg(table + r * vec_per_row + c);
    out[v] = x;
  }
}

// Rows [*begin, *end) of ids (bounds read on the device, at most max_rows):
// out[i] = table[ids[*begin + i]].
__global__ void gather_rows_ranged_kernel(const uint4* __restrict__ table, int64_t num_table_rows, int64_t vec_per_row,
                                          const int64_t* __restrict__ ids, const int64_t* __restrict__ begin,
                                          const int64_t* __restrict__ end, int64_t max_rows, uint4* __restrict__ out) {
  const int64_t lo = *begin;
  int64_t n = *end - lo;
  n = n < max_rows ? n : max_rows;
  const int64_t total = n * vec_per_row;
  for (int64_t v = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; v < total;
       v += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t i = v / vec_per_row, c = v - i * vec_per_row;
    const int64_t r = ids[lo + i];
    uint4 x = make_uint4(0, 0, 0, 0);
    if (r >= 0 && r < num_table_rows) x = __ldg(table + r * vec_per_row + c);
    out[v] = x;
  }
}

int sm_count() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

// ---- segment softmax aggregation (attention) ------------------------------
// out[t, h, :] = sum_e w[e, h] * msg[e, h, :] over the items e of segment t,
// w[e, h] = exp(l[e, h] - m[t, h]) / (sum_e' exp(l[e', h] - m[t, h]) + 1e-9),
// m[t, h] = max_e l[e, h]: the relation attention of
// dgf/src/learning/jax/layers/hetero_graph_attention_network.py:242-263.
// One warp per segment over its items in CSR order (perm[j] = item of slot j,
// nullptr = identity); lane l owns the 16-byte slices v = l + 32 i of the
// H x D message row, each inside one head. Online softmax: per slice a running
// (max, sum, weighted sum), rescaled once per group of four rows to the
// group's new max, so every message row is read once and no [E, H] weight
// array is materialised.
template <class MT>
__device__ __forceinline__ void unpack16(const uint4& x, float* f);
template <>
__device__ __forceinline__ void unpack16<float>(const uint4& x, float* f) {
  f[0] = __uint_as_float(x.x);
  f[1] = __uint_as_float(x.y);
  f[2] = __uint_as_float(x.z);
  f[3] = __uint_as_float(x.w);
}
template <>
__device__ __forceinline__ void unpack16<__nv_bfloat16>(const uint4& x, float* f) {
  const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

// Online-softmax state of one 16-byte message slice: running max, running
// sum of exp(l - max) and running weighted sum of the slice's elements.
template <int EPV>
struct SoftmaxState {
  float m, s, acc[EPV];
  __device__ __forceinline__ void init() {
    m = -INFINITY;
    s = 0.0f;
#pragma unroll
    for (int k = 0; k < EPV; ++k) acc[k] = 0.0f;
  }
  __device__ __forceinline__ void add(float l, const float* x) {
    const float mn = fmaxf(m, l);
    if (mn == -INFINITY) return;  // every logit so far is -inf
    const float sc = __expf(m - mn);
    const float p = __expf(l - mn);
    s = s * sc + p;
#pragma unroll
    for (int k = 0; k < EPV; ++k) acc[k] = acc[k] * sc + p * x[k];
    m = mn;
  }
  // U rows at once: one rescale to the group's new max, then U plain
  // accumulations (rows past the segment carry l = -inf, x = 0).
  template <int U>
  __device__ __forceinline__ void add_group(const float* l, const float (*x)[EPV]) {
    float mg = l[0];
#pragma unroll
    for (int u = 1; u < U; ++u) mg = fmaxf(mg, l[u]);
    const float mn = fmaxf(m, mg);
    if (mn == -INFINITY) return;  // every logit so far is -inf
    const float sc = __expf(m - mn);
    s *= sc;
#pragma unroll
    for (int k = 0; k < EPV; ++k) acc[k] *= sc;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const float p = __expf(l[u] - mn);
      s += p;
#pragma unroll
      for (int k = 0; k < EPV; ++k) acc[k] = fmaf(p, x[u][k], acc[k]);
    }
    m = mn;
  }
  __device__ __forceinline__ void merge(float m2, float s2, const float* acc2) {
    const float mn = fmaxf(m, m2);
    if (mn == -INFINITY) return;
    const float a = __expf(m - mn), b = __expf(m2 - mn);
    s = s * a + s2 * b;
#pragma unroll
    for (int k = 0; k < EPV; ++k) acc[k] = acc[k] * a + acc2[k] * b;
    m = mn;
  }
};

// One warp per task: a chunk of at most kChunk items of one segment (the
// SpMM task plan), four message rows in flight. A segment of one task writes
// its output; chunks of a split segment write their states (per slice: max,
// sum, EPV weighted sums) for segment_softmax_fixup_kernel.
template <class MT, class OT, int VPL>
__global__ void __launch_bounds__(256, (VPL == 1 && sizeof(MT) == 2) ? 5 : 1) segment_softmax_kernel(
    const int64_t* __restrict__ rowptr, const int64_t* __restrict__ task_off, const int64_t* __restrict__ split_off,
    const int32_t* __restrict__ task_row, const int64_t* __restrict__ num_tasks, const uint32_t* __restrict__ perm,
    const float* __restrict__ logits, int heads, const uint4* __restrict__ msg, int64_t vpr, int head_dim,
    float* __restrict__ partial, OT* __restrict__ out) {
  constexpr int EPV = 16 / sizeof(MT);
  constexpr int kU = 4;
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  int head[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) head[i] = static_cast<int>(((lane + 32 * i) * EPV) / head_dim);
  const int64_t ntot = *num_tasks;  // task_off[nseg]: the exact plan size
  for (int64_t t = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5; t < ntot; t += warps) {
    const int64_t r = task_row[t];
    const int64_t c = t - task_off[r];
    const int64_t ntask = task_off[r + 1] - task_off[r];
    const int64_t lo = rowptr[r] + c * kChunk;
    const int64_t hi = min(rowptr[r + 1], lo + kChunk);
    SoftmaxState<EPV> st[VPL];
#pragma unroll
    for (int i = 0; i < VPL; ++i) st[i].init();
    for (int64_t j0 = lo; j0 < hi; j0 += kU) {
      float l[kU][VPL];
      uint4 x[kU][VPL];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int64_t j = j0 + u;
        const int64_t e = j < hi ? (perm != nullptr ? static_cast<int64_t>(perm[j]) : j) : -1;
#pragma unroll
        for (int i = 0; i < VPL; ++i) {
          const int64_t v = lane + 32 * i;
          l[u][i] = -INFINITY;
          x[u][i] = make_uint4(0, 0, 0, 0);
          if (e >= 0 && v < vpr) {
            l[u][i] = __ldg(logits + e * heads + head[i]);
            x[u][i] = __ldg(msg + e * vpr + v);
          }
        }
      }
#pragma unroll
      for (int i = 0; i < VPL; ++i) {
        if (lane + 32 * i < vpr) {
          float f[kU][EPV];
          float lg[kU];
#pragma unroll
          for (int u = 0; u < kU; ++u) {
            unpack16<MT>(x[u][i], f[u]);
            lg[u] = l[u][i];
          }
          st[i].template add_group<kU>(lg, f);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int64_t v = lane + 32 * i;
      if (v >= vpr) continue;
      if (ntask == 1) {
        const float inv = 1.0f / (st[i].s + 1e-9f);
        OT* o = out + (r * vpr + v) * EPV;
#pragma unroll
        for (int k = 0; k < EPV; ++k) o[k] = static_cast<OT>(st[i].acc[k] * inv);
      } else {
        float* p = partial + ((split_off[r] + c) * vpr + v) * (2 + EPV);
        p[0] = st[i].m;
        p[1] = st[i].s;
#pragma unroll
        for (int k = 0; k < EPV; ++k) p[2 + k] = st[i].acc[k];
      }
    }
  }
}

// Sorted items (no permutation), heads dividing 32, at most one 16-byte slice
// per lane (H x D <= 32 slices). A chunk's logits are rows lo..hi of [E, H],
// contiguous, so the warp first reads them coalesced and reduces the chunk's
// maximum per head (lane i holds head i % H); the weighted sum then needs no
// running rescale: per row one exponential, one add and EPV FMAs. The next
// four message rows are loaded while the current four are consumed, and the
// first four are in flight during the maximum. Chunk states have the layout
// of segment_softmax_kernel's, so the same fix-up merges split segments.
template <class OT, int EPV>
__device__ __forceinline__ void store_slice(OT* o, const float* acc, float scale);
template <>
__device__ __forceinline__ void store_slice<float, 4>(float* o, const float* a, float sc) {
  *reinterpret_cast<float4*>(o) = make_float4(a[0] * sc, a[1] * sc, a[2] * sc, a[3] * sc);
}
template <>
__device__ __forceinline__ void store_slice<float, 8>(float* o, const float* a, float sc) {
  reinterpret_cast<float4*>(o)[0] = make_float4(a[0] * sc, a[1] * sc, a[2] * sc, a[3] * sc);
  reinterpret_cast<float4*>(o)[1] = make_float4(a[4] * sc, a[5] * sc, a[6] * sc, a[7] * sc);
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}
template <>
__device__ __forceinline__ void store_slice<__nv_bfloat16, 4>(__nv_bfloat16* o, const float* a, float sc) {
  *reinterpret_cast<uint2*>(o) = make_uint2(pack_bf16x2(a[0] * sc, a[1] * sc), pack_bf16x2(a[2] * sc, a[3] * sc));
}
template <>
__device__ __forceinline__ void store_slice<__nv_bfloat16, 8>(__nv_bfloat16* o, const float* a, float sc) {
  *reinterpret_cast<uint4*>(o) = make_uint4(pack_bf16x2(a[0] * sc, a[1] * sc), pack_bf16x2(a[2] * sc, a[3] * sc),
                                            pack_bf16x2(a[4] * sc, a[5] * sc), pack_bf16x2(a[6] * sc, a[7] * sc));
}

template <int U>
__device__ __forceinline__ void load_rows(uint4 (&x)[U], float (&l)[U], const uint4* __restrict__ mp,
                                          const float* __restrict__ lp, int j0, int n, int vpr, int heads,
                                          bool active) {
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int j = j0 + u;
    if (active && j < n) {
      x[u] = __ldg(mp + j * vpr);
      l[u] = __ldg(lp + j * heads);
    } else {
      x[u] = make_uint4(0, 0, 0, 0);
      l[u] = -INFINITY;
    }
  }
}

template <class MT, class OT>
__global__ void __launch_bounds__(256, 4) segment_softmax_sorted_kernel(
    const int64_t* __restrict__ rowptr, const int64_t* __restrict__ task_off, const int64_t* __restrict__ split_off,
    const int32_t* __restrict__ task_row, const int64_t* __restrict__ num_tasks, const float* __restrict__ logits,
    int heads, const uint4* __restrict__ msg, int vpr, int head_dim, float* __restrict__ partial,
    OT* __restrict__ out, unsigned long long* __restrict__ next_task) {
  constexpr int EPV = 16 / sizeof(MT);
  constexpr int kU = 4;
  const int lane = threadIdx.x & 31;
  const bool active = lane < vpr;
  const int head = active ? (lane * EPV) / head_dim : 0;
  const int64_t ntot = *num_tasks;
  // Tasks are taken from a counter (a persistent grid; chunks hold 1 to
  // kChunk rows, so a static split leaves warps idle), the next one fetched
  // while the current one is processed.
  unsigned long long claim = lane == 0 ? atomicAdd(next_task, 1ull) : 0ull;
  for (int64_t t = static_cast<int64_t>(__shfl_sync(0xffffffffu, claim, 0)); t < ntot;
       t = static_cast<int64_t>(__shfl_sync(0xffffffffu, claim, 0))) {
    claim = lane == 0 ? atomicAdd(next_task, 1ull) : 0ull;
    const int64_t r = task_row[t];
    const int64_t c = t - task_off[r];
    const int64_t ntask = task_off[r + 1] - task_off[r];
    const int64_t lo = rowptr[r] + c * kChunk;
    const int n = static_cast<int>(min(rowptr[r + 1], lo + kChunk) - lo);
    const uint4* mp = msg + lo * vpr + lane;
    const float* lp = logits + lo * heads + head;
    uint4 x[kU];
    float l[kU];
    load_rows<kU>(x, l, mp, lp, 0, n, vpr, heads, active);
    // The chunk's maximum per head.
    const float* lc = logits + lo * heads;
    const int nl = n * heads;
    float m = -INFINITY;
    for (int k = lane; k < nl; k += 32) m = fmaxf(m, __ldg(lc + k));
    for (int off = heads; off < 32; off <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    m = __shfl_sync(0xffffffffu, m, head);
    const float mb = m == -INFINITY ? 0.0f : m;  // a head whose logits are all -inf gets weight 0
    float s = 0.0f, acc[EPV];
#pragma unroll
    for (int k = 0; k < EPV; ++k) acc[k] = 0.0f;
    for (int j0 = 0; j0 < n; j0 += kU) {
      uint4 xn[kU];
      float ln[kU];
      load_rows<kU>(xn, ln, mp, lp, j0 + kU, n, vpr, heads, active);
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const float p = __expf(l[u] - mb);
        s += p;
        float f[EPV];
        unpack16<MT>(x[u], f);
#pragma unroll
        for (int k = 0; k < EPV; ++k) acc[k] = fmaf(p, f[k], acc[k]);
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        x[u] = xn[u];
        l[u] = ln[u];
      }
    }
    if (active && ntask == 1) {
      store_slice<OT, EPV>(out + (r * vpr + lane) * EPV, acc, 1.0f / (s + 1e-9f));
    } else if (active) {
      float* p = partial + ((split_off[r] + c) * vpr + lane) * (2 + EPV);
      p[0] = m;
      p[1] = s;
#pragma unroll
      for (int k = 0; k < EPV; ++k) p[2 + k] = acc[k];
    }
  }
}

// Split segments: merge their chunk states in chunk order (deterministic).
template <class MT, class OT, int VPL>
__global__ void __launch_bounds__(256) segment_softmax_fixup_kernel(const int64_t* __restrict__ task_off,
                                                                    const int64_t* __restrict__ split_off,
                                                                    int64_t nseg, int64_t vpr,
                                                                    const float* __restrict__ partial,
                                                                    OT* __restrict__ out) {
  constexpr int EPV = 16 / sizeof(MT);
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t r = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5; r < nseg; r += warps) {
    const int64_t ntask = task_off[r + 1] - task_off[r];
    if (ntask <= 1) continue;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int64_t v = lane + 32 * i;
      if (v >= vpr) continue;
      SoftmaxState<EPV> st;
      st.init();
      for (int64_t c = 0; c < ntask; ++c) {
        const float* p = partial + ((split_off[r] + c) * vpr + v) * (2 + EPV);
        st.merge(p[0], p[1], p + 2);
      }
      const float inv = 1.0f / (st.s + 1e-9f);
      OT* o = out + (r * vpr + v) * EPV;
#pragma unroll
      for (int k = 0; k < EPV; ++k) o[k] = static_cast<OT>(st.acc[k] * inv);
    }
  }
}

__global__ void softmax_sort_input_kernel(const int64_t* __restrict__ ids, int64_t n, int64_t nseg,
                                          uint64_t* __restrict__ keys, uint32_t* __restrict__ vals) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t id = ids[i];
    keys[i] = (id >= 0 && id < nseg) ? static_cast<uint64_t>(id) : static_cast<uint64_t>(nseg);
    vals[i] = static_cast<uint32_t>(i);
  }
}

unsigned grid_for(int64_t work, int threads) {
  const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
  const int64_t b = ceil_div(std::max<int64_t>(work, 1), threads);
  return static_cast<unsigned>(std::min(b, cap));
}

struct SpmmBufs {
  int32_t* cnt;
  int32_t* split_cnt;
  int64_t* task_off;
  int64_t* split_off;
  int32_t* task_row;
  float* partial;
  unsigned long long* next_task;  // one task counter per feature block
};

int64_t max_tasks(int64_t rows, int64_t nnz) { return rows + nnz / kChunk + 1; }
int64_t max_split_tasks(int64_t nnz) { return 2 * (nnz / kChunk) + 2; }
// Feature columns handled per launch (fp32 partial slice width).
int64_t feat_block(int64_t feat, int dtype) {
  const int64_t cap = dtype == DGFX_BF16 ? 1024 : 512;
  return std::min(feat, cap);
}
// Launches per SpMM at most (the smallest feature block is 512 columns).
int64_t spmm_feature_blocks(int64_t feat) { return ceil_div(std::max<int64_t>(feat, 1), int64_t(512)); }

void carve_spmm(Arena& a, int64_t rows, int64_t nnz, int64_t feat, SpmmBufs* b) {
  b->cnt = a.take<int32_t>(static_cast<size_t>(rows));
  b->split_cnt = a.take<int32_t>(static_cast<size_t>(rows));
  b->task_off = a.take<int64_t>(static_cast<size_t>(rows + 1));
  b->split_off = a.take<int64_t>(static_cast<size_t>(rows + 1));
  b->task_row = a.take<int32_t>(static_cast<size_t>(max_tasks(rows, nnz)));
  b->partial = a.take<float>(static_cast<size_t>(max_split_tasks(nnz) * std::min<int64_t>(feat, 1024)));
  b->next_task = a.take<unsigned long long>(static_cast<size_t>(spmm_feature_blocks(feat)));
}

size_t spmm_ws(int64_t rows, int64_t nnz, int64_t feat) {
  Arena a(nullptr, 0);
  SpmmBufs b;
  carve_spmm(a, rows, nnz, feat, &b);
  return a.used + scan_workspace_bytes(rows + 1) + 1024;
}

template <class XT, class YT>
int launch_spmm(const int64_t* rowptr, const int32_t* col, const float* val, int64_t rows, int64_t num_cols,
                const void* x, void* y, int64_t feat, int normalize, const SpmmBufs& b, cudaStream_t stream, int xdtype) {
  constexpr int V = Vec<XT>::n;
  const int64_t fb = feat_block(feat, xdtype);
  const unsigned grid = static_cast<unsigned>(sm_count() * 3);  // persistent: 3 resident CTAs per SM
  for (int64_t f0 = 0; f0 < feat; f0 += fb) {
    unsigned long long* next_task = b.next_task + f0 / fb;
    const int64_t fw = std::min(fb, feat - f0);
    const int64_t chunks = fw / V;
    const XT* X = static_cast<const XT*>(x);
    YT* Y = static_cast<YT*>(y);
    if (chunks <= 32) {
      spmm_kernel<XT, YT, 1, 8><<<grid, kWarpsPerBlock * 32, 0, stream>>>(rowptr, col, val, X, Y, feat, f0, fw,
                                                                           b.task_off, b.task_row, b.split_off,
                                                                           b.partial, rows, normalize, num_cols, next_task);
    } else if (chunks <= 64) {
      spmm_kernel<XT, YT, 2, 4><<<grid, kWarpsPerBlock * 32, 0, stream>>>(rowptr, col, val, X, Y, feat, f0, fw,
                                                                           b.task_off, b.task_row, b.split_off,
                                                                           b.partial, rows, normalize, num_cols, next_task);
    } else {
      spmm_kernel<XT, YT, 4, 2><<<grid, kWarpsPerBlock * 32, 0, stream>>>(rowptr, col, val, X, Y, feat, f0, fw,
                                                                           b.task_off, b.task_row, b.split_off,
                                                                           b.partial, rows, normalize, num_cols, next_task);
    }
    DGFX_CUDA_TRY(cudaGetLastError());
    spmm_fixup_kernel<YT><<<grid_for(rows * 32, 256), 256, 0, stream>>>(rowptr, b.split_off, b.partial, Y, rows,
                                                                         feat, f0, fw, normalize);
    DGFX_CUDA_TRY(cudaGetLastError());
  }
  return DGFX_OK;
}

int check_dtype(int t) { return t == DGFX_F32 || t == DGFX_BF16; }

}  // namespace
}  // namespace dgfx

using namespace dgfx;

extern "C" int dgfx_gather_rows(const void* d_table, int64_t num_table_rows, int64_t row_bytes,
                                const int64_t* d_row_ids, int64_t num_rows, void* d_out, dgfx_stream stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (row_bytes <= 0 || row_bytes % 16 != 0 || num_rows < 0 || num_table_rows < 0) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_gather_rows: row_bytes must be a positive multiple of 16");
  }
  if (num_rows == 0) return DGFX_OK;
  if (reinterpret_cast<uintptr_t>(d_table) % 16 != 0 || reinterpret_cast<uintptr_t>(d_out) % 16 != 0) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_gather_rows: table and out must be 16-byte aligned");
  }
  const int64_t vpr = row_bytes / 16;
  gather_rows_kernel<<<grid_for(num_rows * vpr, 256), 256, 0, stream>>>(
      static_cast<const uint4*>(d_table), num_table_rows, vpr, d_row_ids, num_rows, static_cast<uint4*>(d_out));
  DGFX_CUDA_TRY(cudaGetLastError());
  return DGFX_OK;
}

extern "C" int dgfx_gather_rows_ranged(const void* d_table, int64_t num_table_rows, int64_t row_bytes,
                                       const int64_t* d_row_ids, const int64_t* d_begin, const int64_t* d_end,
                                       int64_t max_rows, void* d_out, dgfx_stream stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (row_bytes <= 0 || row_bytes % 16 != 0 || max_rows < 0 || num_table_rows < 0 || d_begin == nullptr ||
      d_end == nullptr) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_gather_rows_ranged: bad arguments");
  }
  if (max_rows == 0) return DGFX_OK;
  if (reinterpret_cast<uintptr_t>(d_table) % 16 != 0 || reinterpret_cast<uintptr_t>(d_out) % 16 != 0) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_gather_rows_ranged: table and out must be 16-byte aligned");
  }
  const int64_t vpr = row_bytes / 16;
  gather_rows_ranged_kernel<<<grid_for(max_rows * vpr, 256), 256, 0, stream>>>(
      static_cast<const uint4*>(d_table), num_table_rows, vpr, d_row_ids, d_begin, d_end, max_rows,
      static_cast<uint4*>(d_out));
  DGFX_CUDA_TRY(cudaGetLastError());
  return DGFX_OK;
}

extern "C" int dgfx_spmm_workspace_size(int64_t num_rows, int64_t nnz, int64_t feat, size_t* bytes) {
  if (bytes == nullptr || num_rows < 0 || nnz < 0 || feat <= 0) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_spmm_workspace_size: bad arguments");
  }
  *bytes = spmm_ws(num_rows, nnz, feat);
  return DGFX_OK;
}

namespace {
int spmm_impl(const int64_t* rowptr, const int32_t* col, const float* val, int64_t rows, int64_t nnz,
              int64_t num_cols, const void* x, int xt, void* y, int yt, int64_t feat, int normalize, void* ws,
              size_t ws_bytes, cudaStream_t stream) {
  Arena arena(ws, ws_bytes);
  if (ws == nullptr || ws_bytes < spmm_ws(rows, nnz, feat)) return fail(DGFX_ERR_WORKSPACE, "spmm: workspace too small");
  SpmmBufs b;
  carve_spmm(arena, rows, nnz, feat, &b);
  spmm_count_kernel<<<grid_for(rows, 256), 256, 0, stream>>>(rowptr, rows, b.cnt, b.split_cnt);
  DGFX_CUDA_TRY(cudaGetLastError());
  const size_t mark = arena.used;
  DGFX_TRY(exclusive_scan<int32_t>(b.cnt, b.task_off, rows, true, arena, stream));
  arena.used = mark;
  DGFX_TRY(exclusive_scan<int32_t>(b.split_cnt, b.split_off, rows, true, arena, stream));
  spmm_fill_kernel<<<grid_for(rows, 256), 256, 0, stream>>>(b.task_off, rows, b.task_row, b.next_task,
                                                            static_cast<int>(spmm_feature_blocks(feat)));
  DGFX_CUDA_TRY(cudaGetLastError());
  if (xt == DGFX_F32 && yt == DGFX_F32) return launch_spmm<float, float>(rowptr, col, val, rows, num_cols, x, y, feat, normalize, b, stream, xt);
  if (xt == DGFX_F32 && yt == DGFX_BF16) return launch_spmm<float, __nv_bfloat16>(rowptr, col, val, rows, num_cols, x, y, feat, normalize, b, stream, xt);
  if (xt == DGFX_BF16 && yt == DGFX_F32) return launch_spmm<__nv_bfloat16, float>(rowptr, col, val, rows, num_cols, x, y, feat, normalize, b, stream, xt);
  return launch_spmm<__nv_bfloat16, __nv_bfloat16>(rowptr, col, val, rows, num_cols, x, y, feat, normalize, b, stream, xt);
}
}  // namespace

extern "C" int dgfx_spmm_csr(const int64_t* d_rowptr, const int32_t* d_col, const float* d_val, int64_t num_rows,
                             int64_t num_cols, int64_t nnz, const void* d_x, int x_dtype, void* d_y, int y_dtype,
                             int64_t feat, int32_t normalize, void* d_workspace, size_t workspace_bytes,
                             dgfx_stream stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (!check_dtype(x_dtype) || !check_dtype(y_dtype)) return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_spmm_csr: dtype");
  if (num_rows < 0 || num_cols < 0 || nnz < 0 || feat <= 0 || d_rowptr == nullptr || d_y == nullptr) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_spmm_csr: bad arguments");
  }
  if (feat % 8 != 0) return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_spmm_csr: feat must be a multiple of 8");
  if (num_cols >= (int64_t(1) << 31)) return fail(DGFX_ERR_UNSUPPORTED, "dgfx_spmm_csr: more than 2^31 - 1 columns");
  if (reinterpret_cast<uintptr_t>(d_x) % 16 != 0 || reinterpret_cast<uintptr_t>(d_y) % 16 != 0) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_spmm_csr: X and Y must be 16-byte aligned");
  }
  if (num_rows == 0) return DGFX_OK;
  if (nnz > 0 && d_col == nullptr) return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_spmm_csr: null col");
  return spmm_impl(d_rowptr, d_col, d_val, num_rows, nnz, num_cols, d_x, x_dtype, d_y, y_dtype, feat, normalize,
                   d_workspace, workspace_bytes, stream);
}

extern "C" int dgfx_segment_sum_workspace_size(int64_t num_items, int64_t feat, int64_t num_segments, size_t* bytes) {
  if (bytes == nullptr || num_items < 0 || feat <= 0 || num_segments < 0) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_segment_sum_workspace_size: bad arguments");
  }
  const size_t sorted = align_up(sizeof(int64_t) * (num_segments + 1), 256) + spmm_ws(num_segments, num_items, feat);
  const size_t atomic = align_up(sizeof(float) * num_segments * feat, 256) + align_up(sizeof(int32_t) * num_segments, 256);
  *bytes = std::max(sorted, atomic) + 1024;
  return DGFX_OK;
}

extern "C" int dgfx_segment_sum(const void* d_data, int data_dtype, const int64_t* d_ids, int64_t n, int64_t feat,
                                int64_t nseg, int32_t mean, int32_t sorted, void* d_out, int out_dtype,
                                void* d_workspace, size_t workspace_bytes, dgfx_stream stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (!check_dtype(data_dtype) || !check_dtype(out_dtype)) return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_segment_sum: dtype");
  if (n < 0 || feat <= 0 || nseg < 0 || feat % 8 != 0) return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_segment_sum: bad arguments");
  if (n >= (int64_t(1) << 31)) return fail(DGFX_ERR_UNSUPPORTED, "dgfx_segment_sum: more than 2^31 - 1 items");
  if (nseg == 0) return DGFX_OK;
  size_t need = 0;
  DGFX_TRY(dgfx_segment_sum_workspace_size(n, feat, nseg, &need));
  if (d_workspace == nullptr || workspace_bytes < need) return fail(DGFX_ERR_WORKSPACE, "dgfx_segment_sum: workspace too small");
  Arena arena(d_workspace, workspace_bytes);
  if (sorted) {
    int64_t* rowptr = arena.take<int64_t>(static_cast<size_t>(nseg + 1));
    sorted_bounds_kernel<<<grid_for(nseg + 1, 256), 256, 0, stream>>>(d_ids, n, nseg, rowptr);
    DGFX_CUDA_TRY(cudaGetLastError());
    // Items are gathered in place: X row j = data row j (identity columns).
    return spmm_impl(rowptr, nullptr, nullptr, nseg, n, n, d_data, data_dtype, d_out, out_dtype, feat, mean,
                     arena.base + arena.used, workspace_bytes - arena.used, stream);
  }
  float* acc = arena.take<float>(static_cast<size_t>(nseg * feat));
  int32_t* cnt = mean ? arena.take<int32_t>(static_cast<size_t>(nseg)) : nullptr;
  DGFX_CUDA_TRY(cudaMemsetAsync(acc, 0, sizeof(float) * nseg * feat, stream));
  if (cnt != nullptr) DGFX_CUDA_TRY(cudaMemsetAsync(cnt, 0, sizeof(int32_t) * nseg, stream));
  if (n > 0) {
    if (data_dtype == DGFX_F32) {
      segment_atomic_kernel<float><<<grid_for(n * 32, 256), 256, 0, stream>>>(
          static_cast<const float*>(d_data), d_ids, n, feat, nseg, acc, cnt);
    } else {
      segment_atomic_kernel<__nv_bfloat16><<<grid_for(n * 32, 256), 256, 0, stream>>>(
          static_cast<const __nv_bfloat16*>(d_data), d_ids, n, feat, nseg, acc, cnt);
    }
    DGFX_CUDA_TRY(cudaGetLastError());
  }
  if (out_dtype == DGFX_F32) {
    segment_finish_kernel<float><<<grid_for(nseg * feat / 4, 256), 256, 0, stream>>>(acc, cnt, nseg, feat,
                                                                                     static_cast<float*>(d_out));
  } else {
    segment_finish_kernel<__nv_bfloat16><<<grid_for(nseg * feat / 8, 256), 256, 0, stream>>>(
        acc, cnt, nseg, feat, static_cast<__nv_bfloat16*>(d_out));
  }
  DGFX_CUDA_TRY(cudaGetLastError());
  return DGFX_OK;
}

namespace dgfx {
namespace {
size_t softmax_ws(int64_t n, int64_t nseg, bool sorted, int64_t vpr, int64_t epv) {
  Arena a(nullptr, 0);
  a.take<int64_t>(static_cast<size_t>(nseg + 1));  // rowptr
  if (!sorted) {
    a.take<uint64_t>(static_cast<size_t>(std::max<int64_t>(n, 1)));
    a.take<uint32_t>(static_cast<size_t>(std::max<int64_t>(n, 1)));
    a.take<uint64_t>(static_cast<size_t>(std::max<int64_t>(n, 1)));
    a.take<uint32_t>(static_cast<size_t>(std::max<int64_t>(n, 1)));
  }
  a.take<int32_t>(static_cast<size_t>(nseg));                       // cnt
  a.take<int32_t>(static_cast<size_t>(nseg));                       // split_cnt
  a.take<int64_t>(static_cast<size_t>(nseg + 1));                   // task_off
  a.take<int64_t>(static_cast<size_t>(nseg + 1));                   // split_off
  a.take<int32_t>(static_cast<size_t>(max_tasks(nseg, n)));         // task_row
  a.take<float>(static_cast<size_t>(max_split_tasks(n) * vpr * (2 + epv)));  // chunk states
  a.take<unsigned long long>(1);                                              // task counter
  return a.used + std::max(scan_workspace_bytes(nseg + 1), sorted ? size_t(0) : radix_sort_workspace_bytes(n)) +
         2048;
}

template <class MT, class OT>
int launch_softmax(const int64_t* rowptr, const uint32_t* perm, int64_t nseg, int64_t n, const float* logits,
                   int heads, const void* msg, int64_t vpr, int head_dim, void* out, Arena& arena,
                   cudaStream_t stream) {
  constexpr int64_t EPV = 16 / sizeof(MT);
  int32_t* cnt = arena.take<int32_t>(static_cast<size_t>(nseg));
  int32_t* split_cnt = arena.take<int32_t>(static_cast<size_t>(nseg));
  int64_t* task_off = arena.take<int64_t>(static_cast<size_t>(nseg + 1));
  int64_t* split_off = arena.take<int64_t>(static_cast<size_t>(nseg + 1));
  int32_t* task_row = arena.take<int32_t>(static_cast<size_t>(max_tasks(nseg, n)));
  float* partial = arena.take<float>(static_cast<size_t>(max_split_tasks(n) * vpr * (2 + EPV)));
  auto* next_task = arena.take<unsigned long long>(1);
  spmm_count_kernel<<<grid_for(nseg, 256), 256, 0, stream>>>(rowptr, nseg, cnt, split_cnt);
  DGFX_CUDA_TRY(cudaGetLastError());
  const size_t mark = arena.used;
  DGFX_TRY(exclusive_scan<int32_t>(cnt, task_off, nseg, true, arena, stream));
  arena.used = mark;
  DGFX_TRY(exclusive_scan<int32_t>(split_cnt, split_off, nseg, true, arena, stream));
  spmm_fill_kernel<<<grid_for(nseg, 256), 256, 0, stream>>>(task_off, nseg, task_row, next_task);
  DGFX_CUDA_TRY(cudaGetLastError());
  // Grid sized for the largest possible plan; the kernel reads the exact task
  // count (task_off[nseg]) on the device.
  const int64_t tasks = max_tasks(nseg, n);
  const unsigned blocks = grid_for(tasks * 32, 256);
  auto m = static_cast<const uint4*>(msg);
  auto o = static_cast<OT*>(out);
  const int vpl = static_cast<int>(ceil_div(vpr, int64_t(32)));
#define DGFX_SOFTMAX_LAUNCH(V)                                                                                \
  segment_softmax_kernel<MT, OT, V><<<blocks, 256, 0, stream>>>(rowptr, task_off, split_off, task_row,         \
                                                                 task_off + nseg, perm, logits, heads, m, vpr,  \
                                                                 head_dim, partial, o);                        \
  DGFX_CUDA_TRY(cudaGetLastError());                                                                           \
  segment_softmax_fixup_kernel<MT, OT, V><<<grid_for(nseg * 32, 256), 256, 0, stream>>>(task_off, split_off,   \
                                                                                        nseg, vpr, partial, o);
  if (perm == nullptr && vpr <= 32 && 32 % heads == 0 && reinterpret_cast<uintptr_t>(out) % 16 == 0) {
    // Persistent: four 256-thread CTAs of 64 registers fill an SM.
    const unsigned pblocks = std::min<unsigned>(blocks, static_cast<unsigned>(sm_count()) * 4);
    segment_softmax_sorted_kernel<MT, OT><<<pblocks, 256, 0, stream>>>(rowptr, task_off, split_off, task_row,
                                                                       task_off + nseg, logits, heads, m,
                                                                       static_cast<int>(vpr), head_dim, partial, o,
                                                                       next_task);
    DGFX_CUDA_TRY(cudaGetLastError());
    segment_softmax_fixup_kernel<MT, OT, 1><<<grid_for(nseg * 32, 256), 256, 0, stream>>>(task_off, split_off, nseg,
                                                                                          vpr, partial, o);
  } else if (vpl <= 1) {
    DGFX_SOFTMAX_LAUNCH(1)
  } else if (vpl == 2) {
    DGFX_SOFTMAX_LAUNCH(2)
  } else {
    DGFX_SOFTMAX_LAUNCH(4)
  }
#undef DGFX_SOFTMAX_LAUNCH
  DGFX_CUDA_TRY(cudaGetLastError());
  return DGFX_OK;
}
}  // namespace
}  // namespace dgfx

extern "C" int dgfx_segment_softmax_workspace_size(int64_t num_items, int64_t num_segments, int32_t heads,
                                                   int64_t head_dim, int msg_dtype, int32_t sorted, size_t* bytes) {
  if (bytes == nullptr || num_items < 0 || num_segments < 0 || heads < 1 || head_dim < 1 || !check_dtype(msg_dtype)) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_segment_softmax_workspace_size: bad arguments");
  }
  const int64_t epv = msg_dtype == DGFX_F32 ? 4 : 8;
  *bytes = softmax_ws(num_items, num_segments, sorted != 0, ceil_div(heads * head_dim, epv), epv);
  return DGFX_OK;
}

extern "C" int dgfx_segment_softmax(const float* d_logits, int32_t heads, const void* d_messages, int msg_dtype,
                                    int64_t head_dim, const int64_t* d_ids, int64_t n, int64_t nseg, int32_t sorted,
                                    void* d_out, int out_dtype, void* d_workspace, size_t workspace_bytes,
                                    dgfx_stream stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (!check_dtype(msg_dtype) || !check_dtype(out_dtype)) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_segment_softmax: dtype");
  }
  const int64_t epv = msg_dtype == DGFX_F32 ? 4 : 8;
  if (n < 0 || nseg < 0 || heads < 1 || head_dim < 1 || head_dim % epv != 0 ||
      (n > 0 && (d_logits == nullptr || d_messages == nullptr || d_ids == nullptr)) ||
      (nseg > 0 && d_out == nullptr)) {
    return fail(DGFX_ERR_INVALID_ARGUMENT,
                "dgfx_segment_softmax: bad arguments (head_dim must be a multiple of 4 for fp32, 8 for bf16 messages)");
  }
  const int64_t vpr = heads * head_dim / epv;
  if (vpr > 128 || n >= (int64_t(1) << 31)) {
    return fail(DGFX_ERR_UNSUPPORTED, "dgfx_segment_softmax: heads * head_dim rows above 2 KB or 2^31 items");
  }
  if (nseg == 0) return DGFX_OK;
  if (d_workspace == nullptr || workspace_bytes < softmax_ws(n, nseg, sorted != 0, vpr, epv)) {
    return fail(DGFX_ERR_WORKSPACE, "dgfx_segment_softmax: workspace too small");
  }
  Arena arena(d_workspace, workspace_bytes);
  int64_t* rowptr = arena.take<int64_t>(static_cast<size_t>(nseg + 1));
  const uint32_t* perm = nullptr;
  if (sorted || n == 0) {
    sorted_bounds_kernel<<<grid_for(nseg + 1, 256), 256, 0, stream>>>(d_ids, n, nseg, rowptr);
  } else {
    uint64_t* k0 = arena.take<uint64_t>(static_cast<size_t>(n));
    uint32_t* v0 = arena.take<uint32_t>(static_cast<size_t>(n));
    uint64_t* k1 = arena.take<uint64_t>(static_cast<size_t>(n));
    uint32_t* v1 = arena.take<uint32_t>(static_cast<size_t>(n));
    softmax_sort_input_kernel<<<grid_for(n, 256), 256, 0, stream>>>(d_ids, n, nseg, k0, v0);
    DGFX_CUDA_TRY(cudaGetLastError());
    bool in1 = false;
    DGFX_TRY(radix_sort_pairs(k0, v0, k1, v1, n, 0, std::max(1, bit_length(static_cast<uint64_t>(nseg))), &in1,
                              arena, stream));
    const uint64_t* ks = in1 ? k1 : k0;
    perm = in1 ? v1 : v0;
    sorted_bounds_kernel<<<grid_for(nseg + 1, 256), 256, 0, stream>>>(reinterpret_cast<const int64_t*>(ks), n, nseg,
                                                                       rowptr);
  }
  DGFX_CUDA_TRY(cudaGetLastError());
  const int hd = static_cast<int>(head_dim);
  if (msg_dtype == DGFX_F32) {
    return out_dtype == DGFX_F32
               ? launch_softmax<float, float>(rowptr, perm, nseg, n, d_logits, heads, d_messages, vpr, hd, d_out,
                                              arena, stream)
               : launch_softmax<float, __nv_bfloat16>(rowptr, perm, nseg, n, d_logits, heads, d_messages, vpr, hd,
                                                      d_out, arena, stream);
  }
  return out_dtype == DGFX_F32
             ? launch_softmax<__nv_bfloat16, float>(rowptr, perm, nseg, n, d_logits, heads, d_messages, vpr, hd,
                                                    d_out, arena, stream)
             : launch_softmax<__nv_bfloat16, __nv_bfloat16>(rowptr, perm, nseg, n, d_logits, heads, d_messages, vpr,
                                                            hd, d_out, arena, stream);
}
