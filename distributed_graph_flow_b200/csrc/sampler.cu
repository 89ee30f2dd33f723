// Per-seed k-hop sampler (sm_100a).
//
// Semantics follow DGF's SampleBuilder::RecursiveGrow / Grow and
// Sampler::Sample (dgf/src/sampling/in_memory_sampler_ext.cc:231-370,
// 418-533) with the per-node samplers of dgf/src/sampling/
// in_memory_sampler.cc:22-364.
//
// Design. The sampling plan is unrolled on the host into a padded expansion
// tree: every plan node instance gets a fixed "position" in depth-first
// pre-order, with hop_width slots reserved per plan edge, so a plan node's
// padded subtree has Z(p) = 1 + sum_c hop_width(c) * Z(child(c)) positions and
// one seed's tree has T = Z(root). The reference's depth-first traversal
// visits instances in exactly this position order (plan edges in order, the
// picked neighbours of one edge in pick order), so:
//   * "first discovery" of a node = its smallest position,
//   * the reference's local id = number of first discoveries of the same
//     nodeset at smaller positions (a scan),
// and no recursion or ordered map is needed. One CTA samples one seed:
//   1. level-synchronous expansion: a task per (position, plan edge) reads the
//      row, applies the timestamp cutoff (upper_bound on the time-sorted row)
//      and the masked edge, and writes the picked neighbours into the child
//      slots (-1 marks an empty slot);
//   2. relabel: hash table keyed by (nodeset, node) keeps the minimum position
//      (atomicMin), then a block scan numbers first discoveries per nodeset
//      (with_replacement: every occupied position is a new node);
//   3. edges: one key (edgeset | src_local | dst_local) per occupied non-root
//      position, sorted by a block-level stable LSD radix sort (8 bits per
//      pass, ceil((bits(#edgesets) + 2 * bits(T)) / 8) passes) and
//      deduplicated; this equals the reference's btree_set iteration order;
//   4. per-seed results go to a scratch slice; two scans and a compaction
//      kernel produce the merged batch.
// Arrays live in shared memory when the tree is small enough (T <= 8192),
// otherwise in a per-CTA slice of the workspace.
//
// Random mode draws from Philox4x32-10 keyed by the sampler seed with counter
// (tree position, plan edge | draw block, seed slot, call index) and picks k
// of n with Floyd's algorithm (Bentley & Floyd, "Programming pearls: a sample
// of brilliance", CACM 1987), output in adjacency order. This is a different
// generator from the reference's std::mt19937_64, so random-mode results
// match the reference in distribution (uniform k-subsets of the valid row),
// not bit for bit; FIRST and MOST_RECENT modes and fanout >= degree are exact.
#include <algorithm>
#include <cstring>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <type_traits>
#include <vector>

#include "common.cuh"
#include "primitives.cuh"
#include "walk_plan.cuh"

namespace dgfx {
namespace {

constexpr uint64_t kEmptyKey = ~0ull;
constexpr int kMaxNodesets = 64;
constexpr int kMaxEdgesets = 256;
constexpr int kMaxSmemPositions = 8192;
constexpr int64_t kMaxPositions = int64_t(1) << 24;

struct EdgeDev {
  const int64_t* rowptr;
  const int32_t* col;
  const int64_t* ts;
  const int64_t* edge_pos;
  int64_t num_edges;
  int32_t k;        // hop width
  int32_t stride;   // Z(child)
  int32_t edgeset;
  int32_t reversed;
  int32_t rel_off;  // first child slot relative to the parent's position
  int32_t child;    // plan node the edge leads to
};

// Plan node as the warp sampler walks it.
struct PlanNodeDev {
  int32_t first_edge, num_edges, nodeset, in_edge;  // in_edge: the plan edge into this node (-1 at the root)
};

struct Params {
  const EdgeDev* edges;
  const int4* tasks;       // (parent position, plan edge, first child slot, 0)
  const int32_t* level;    // tasks of depth d: [level[d], level[d+1])
  const int32_t* children; // child slots of the depth-d tasks: [clevel[d], clevel[d+1])
  const int32_t* clevel;
  int32_t depth;           // number of expansion levels
  const int2* pos_info;    // (parent position, plan edge << 8 | nodeset)
  int32_t T, N2, H, log2H;
  int32_t num_nodesets, num_edgesets;
  int32_t root_has_children;
  int64_t root_num_src;
  int32_t with_replacement, mode, mask_edgeset;
  const int64_t* seeds;
  const int64_t* seed_ts;
  const int64_t* masks;
  int64_t B;
  uint32_t key0, key1, call_lo, call_hi;
  unsigned long long* call_dev;  // non-null: the call index is this device word (advanced by compact_kernel)
  int32_t* scratch_nodes;    // [B][T]
  uint64_t* scratch_edges;   // [B][T]
  int32_t* node_cnt;         // [NS][B]
  int32_t* edge_cnt;         // [ES][B]
  char* global_work;         // per-CTA arrays when not in shared memory
  size_t work_stride;
  unsigned long long* status;  // [0] first bad seed slot, [1] ts missing, [2] table overflow,
                               // [3..5] expanded rows, sampled neighbours, timestamp probes
  int32_t pbits;               // bits of a local id (local ids < T <= 2^pbits)
  int32_t keybits;             // bits of an edge sort key (edgeset | src | dst)
  uint32_t ns_key_base[kMaxNodesets];  // node set offsets of the 32-bit dedup keys
  // Warp sampler (one warp per seed over occupied positions only).
  const PlanNodeDev* pnodes;
  int32_t warp_cap;            // entries per warp in shared memory (power of two)
  int32_t max_edges_per_node;  // tasks per entry and level
  int32_t warp_bytes;          // shared memory per warp
  unsigned int* overflow_count;  // [0] seeds for the padded kernel, [1] next seed of the warp kernel
  int32_t* overflow_list;        // seeds with more entries than any warp slot holds
  // Large-tree warp tier: seeds that outgrew warp_cap, redone by one warp
  // each with big_cap entries (runtime capacity) before the padded sampler.
  int32_t big_cap;               // 0: no large-tree tier
  int32_t big_bytes;             // shared memory of one large-tree warp
  unsigned int* mid_count;       // [0] seeds listed for the large-tree tier, [1] next of them
  int32_t* mid_list;
};

// Per-CTA working arrays (shared or global memory). The dedup table packs
// (key << 32 | minimum position) into one 64-bit word per slot; after the
// relabel the same words hold the edge sort keys and their sort buffer
// (2 * T <= H words).
struct Work {
  unsigned long long* slot;  // [H]
  int32_t* node;             // [T]
  int32_t* local;            // [T]
};

__host__ __device__ inline size_t work_bytes(int T, int H) {
  return static_cast<size_t>(H) * 8 + static_cast<size_t>(T) * 8 + 64;
}

__device__ inline Work carve_work(char* base, int T, int H) {
  Work w;
  w.slot = reinterpret_cast<unsigned long long*>(base);
  w.node = reinterpret_cast<int32_t*>(base + static_cast<size_t>(H) * 8);
  w.local = w.node + T;
  return w;
}

// Shared memory of one CTA: radix-sort counters, then (if the tree fits)
// the working arrays.
__host__ __device__ inline size_t counter_bytes(int threads) {
  return static_cast<size_t>(threads / 32) * 256 * 4 + 256 * 4;
}

// One expansion task, first half: choose up to k neighbours of node v over
// plan edge e and record their CSR positions (int64, -1 = empty) in the
// child slots base + j * stride (j < k) of the pick array `at`. The column
// loads happen afterwards, one child slot per thread (load_children), so a
// task costs one dependent global load (its row bounds), not k.
// stats[0..2] (shared) count expanded rows, sampled neighbours and timestamp
// probes of this CTA.
__device__ void expand_task(const Params& p, long long* at, int32_t q, int32_t e, int32_t base, int64_t v,
                            bool has_ts, int64_t seed_ts, int64_t mask, uint32_t slot, uint2 call, int32_t pre_n,
                            unsigned int* stats) {
  const EdgeDev E = p.edges[e];
  const int32_t k = E.k, stride = E.stride;
  int32_t cnt = 0;
  if (v >= 0) {
    const int64_t rb = E.rowptr[v];
    const int64_t re = E.rowptr[v + 1];
    int64_t n = re - rb;
    const bool temporal = has_ts && E.ts != nullptr;
    if (!has_ts && E.ts != nullptr) {
      // SampleRandomUniform / SampleFirst on a temporal index fail
      // (in_memory_sampler.cc:26-30, 168-172).
      atomicOr(&p.status[1], 1ull);
      n = 0;
    }
    if (temporal && n > 0 && pre_n >= 0) {
      n = pre_n;  // cutoff found by the cooperative pre-pass
    } else if (temporal && n > 0) {
      // upper_bound(ts[rb..re), seed_ts): first position with ts > seed_ts.
      int64_t lo = 0, hi = n;
      unsigned int probes = 0;
      while (lo < hi) {
        const int64_t mid = (lo + hi) >> 1;
        if (E.ts[rb + mid] <= seed_ts) lo = mid + 1;
        else hi = mid;
        ++probes;
      }
      n = lo;
      atomicAdd(&stats[2], probes);
    }
    int64_t moff = -1;
    if (!temporal && mask >= 0 && E.edgeset == p.mask_edgeset && E.edge_pos != nullptr && mask < E.num_edges) {
      const int64_t pos = E.edge_pos[mask];
      if (pos >= rb && pos < rb + n) moff = pos - rb;
    }
    const int64_t nv = n - (moff >= 0 ? 1 : 0);
    cnt = static_cast<int32_t>(nv < k ? nv : k);
    atomicAdd(&stats[0], 1u);
    atomicAdd(&stats[1], static_cast<unsigned int>(cnt));
    const int mode = (p.mode == DGFX_MODE_MOST_RECENT && !temporal) ? DGFX_MODE_RANDOM : p.mode;
    if (cnt > 0) {
      if (mode == DGFX_MODE_RANDOM && cnt < nv) {
        // Floyd: for j = nv-cnt .. nv-1 pick t in [0, j]; take t unless
        // already taken, else take j. Chosen offsets go to the child slots.
        int32_t taken = 0;
        U4 block{};  // draws m and m + 1 are the two halves of one Philox block
        for (int64_t j = nv - cnt; j < nv; ++j) {
          if ((taken & 1) == 0) {
            const U4 c{static_cast<uint32_t>(q), static_cast<uint32_t>(e) | ((static_cast<uint32_t>(taken) >> 1) << 16),
                       slot, call.x};
            block = philox4x32_10(c, p.key0 ^ call.y, p.key1);
          }
          const uint64_t r = (taken & 1) ? (static_cast<uint64_t>(block.w) << 32 | block.z)
                                         : (static_cast<uint64_t>(block.y) << 32 | block.x);
          int64_t t = static_cast<int64_t>(bounded64(r, static_cast<uint64_t>(j + 1)));
          for (int32_t i = 0; i < taken; ++i) {
            if (at[base + i * stride] == t) {
              t = j;
              break;
            }
          }
          at[base + taken * stride] = t;
          ++taken;
        }
        // Adjacency order (insertion sort over the slots).
        for (int32_t i = 1; i < cnt; ++i) {
          const long long x = at[base + i * stride];
          int32_t j = i - 1;
          while (j >= 0 && at[base + j * stride] > x) {
            at[base + (j + 1) * stride] = at[base + j * stride];
            --j;
          }
          at[base + (j + 1) * stride] = x;
        }
        for (int32_t i = 0; i < cnt; ++i) {
          long long off = at[base + i * stride];
          if (moff >= 0 && off >= moff) ++off;
          at[base + i * stride] = rb + off;
        }
      } else {
        const int64_t first = (mode == DGFX_MODE_MOST_RECENT) ? nv - cnt : 0;
        for (int32_t i = 0; i < cnt; ++i) {
          int64_t off = first + i;
          if (moff >= 0 && off >= moff) ++off;
          at[base + i * stride] = rb + off;
        }
      }
    }
  }
  for (int32_t i = cnt; i < k; ++i) at[base + i * stride] = -1;
}

// Temporal cutoff of every task of one level, eight lanes per task: each
// round the group probes 8 pivots of the remaining interval of the
// time-sorted row (a 9-ary search; rows of <= 8 remaining entries are read
// whole), so a row of d edges costs ceil(log9(d)) dependent loads instead of
// log2(d). cut[t - t0] = number of row entries with ts <= seed_ts, or -1
// when the task's edge set has no timestamps / the node is absent.
__device__ void cutoff_prepass(const Params& p, const Work& w, int32_t* cut, int t0, int t1, int64_t seed_ts,
                               unsigned int* stats) {
  const int gl = threadIdx.x & 7;
  const int ngroups = blockDim.x >> 3;
  const int shift = threadIdx.x & 24;
  const unsigned gmask = 0xFFu << shift;
  for (int t = t0 + (threadIdx.x >> 3); t < t1; t += ngroups) {
    const int4 task = p.tasks[t];
    const int32_t v = w.node[task.x];
    const EdgeDev& E = p.edges[task.y];
    int32_t res = -1;
    if (v >= 0 && E.ts != nullptr) {
      const int64_t rb = E.rowptr[v];
      const int64_t* ts = E.ts + rb;
      int64_t lo = 0, hi = E.rowptr[v + 1] - rb;
      unsigned int probes = 0;
      while (lo < hi) {
        const int64_t len = hi - lo;
        if (len <= 8) {
          const bool le = gl < len && ts[lo + gl] <= seed_ts;
          lo += __popc(__ballot_sync(gmask, le));
          probes += static_cast<unsigned int>(len);
          break;
        }
        const bool le = ts[lo + ((gl + 1) * len) / 9] <= seed_ts;
        const int c = __popc((__ballot_sync(gmask, le) >> shift) & 0xFFu);  // pivots <= cut form a prefix
        const int64_t base = lo;
        if (c > 0) lo = base + (c * len) / 9 + 1;
        if (c < 8) hi = base + ((c + 1) * len) / 9;
        probes += 8;
      }
      res = static_cast<int32_t>(lo);
      if (gl == 0) atomicAdd(&stats[2], probes);
    }
    if (gl == 0) cut[t - t0] = res;
  }
}

// Expansion, second half: node[q] = col[at[q]] for the child slots
// children[c0..c1), four independent loads in flight per thread.
__device__ void load_children(const Params& p, const Work& w, const long long* at, int c0, int c1) {
  constexpr int kIlp = 4;
  const int bd = blockDim.x;
  for (int i0 = c0 + threadIdx.x; i0 < c1; i0 += kIlp * bd) {
    int32_t q[kIlp];
    int32_t v[kIlp];
#pragma unroll
    for (int u = 0; u < kIlp; ++u) {
      const int i = i0 + u * bd;
      q[u] = i < c1 ? p.children[i] : -1;
      v[u] = -1;
      if (q[u] >= 0) {
        const long long a = at[q[u]];
        if (a >= 0) v[u] = p.edges[p.pos_info[q[u]].y >> 8].col[a];
      }
    }
#pragma unroll
    for (int u = 0; u < kIlp; ++u) {
      if (q[u] >= 0) w.node[q[u]] = v[u];
    }
  }
}

// Exclusive scan over items [0, n) of a block: value(i) is read twice (must
// not depend on what sink writes), sink(i, prefix) receives each prefix.
template <class V, class S>
__device__ uint64_t block_scan_items(int n, V value, S sink, uint64_t* smem33) {
  const int per = (n + static_cast<int>(blockDim.x) - 1) / static_cast<int>(blockDim.x);
  const int lo = min(n, static_cast<int>(threadIdx.x) * per);
  const int hi = min(n, lo + per);
  uint64_t s = 0;
  for (int i = lo; i < hi; ++i) s += value(i);
  uint64_t total = 0;
  uint64_t pre = block_exclusive_scan<uint64_t>(s, smem33, &total);
  for (int i = lo; i < hi; ++i) {
    const uint64_t v = value(i);
    sink(i, pre);
    pre += v;
  }
  __syncthreads();
  return total;
}

// Stable LSD radix sort of n 64-bit keys (bits [0, nbits)) by one CTA, 8 bits
// per pass. Warp w owns items [w * chunk, (w + 1) * chunk), visited in rounds
// of 32 consecutive items, so (warp, round, lane) order is input order; ranks
// within a round come from __match_any_sync. cnt has (blockDim.x / 32) * 256
// entries and dbase 256. Returns the buffer holding the sorted keys.
__device__ unsigned long long* block_radix_sort(unsigned long long* a, unsigned long long* b, int n, int nbits,
                                                int32_t* cnt, int32_t* dbase) {
  const int nw = blockDim.x >> 5, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int chunk = (n + nw - 1) / nw;
  const int lo = min(n, warp * chunk), hi = min(n, lo + chunk);
  const uint32_t lt = (1u << lane) - 1u;
  for (int shift = 0; shift < nbits; shift += 8) {
    for (int i = threadIdx.x; i < nw * 256; i += blockDim.x) cnt[i] = 0;
    __syncthreads();
    for (int base = lo; base < hi; base += 32) {
      const int i = base + lane;
      const bool v = i < hi;
      const uint32_t d = v ? static_cast<uint32_t>(a[i] >> shift) & 255u : 256u;
      const uint32_t peers = __match_any_sync(0xffffffffu, d);
      if (v && (peers & lt) == 0) cnt[warp * 256 + d] += __popc(peers);
    }
    __syncthreads();
    for (int d = threadIdx.x; d < 256; d += blockDim.x) {
      int s = 0;
      for (int w = 0; w < nw; ++w) s += cnt[w * 256 + d];
      dbase[d] = s;
    }
    __syncthreads();
    if (warp == 0) {
      int v[8];
      int s = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        v[j] = dbase[lane * 8 + j];
        s += v[j];
      }
      int pre = warp_inclusive_scan(s) - s;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        dbase[lane * 8 + j] = pre;
        pre += v[j];
      }
    }
    __syncthreads();
    for (int d = threadIdx.x; d < 256; d += blockDim.x) {
      int run = dbase[d];
      for (int w = 0; w < nw; ++w) {
        const int c = cnt[w * 256 + d];
        cnt[w * 256 + d] = run;
        run += c;
      }
    }
    __syncthreads();
    for (int base = lo; base < hi; base += 32) {
      const int i = base + lane;
      const bool v = i < hi;
      const unsigned long long k = v ? a[i] : 0ull;
      const uint32_t d = v ? static_cast<uint32_t>(k >> shift) & 255u : 256u;
      const uint32_t peers = __match_any_sync(0xffffffffu, d);
      const int rank = __popc(peers & lt);
      int start = 0;
      if (v) start = cnt[warp * 256 + d];
      __syncwarp();
      if (v) {
        b[start + rank] = k;
        if (rank == 0) cnt[warp * 256 + d] = start + __popc(peers);
      }
      __syncwarp();
    }
    __syncthreads();
    unsigned long long* t = a;
    a = b;
    b = t;
  }
  return a;
}

__device__ __forceinline__ void sample_one(const Params& p, const int64_t sample) {
  extern __shared__ __align__(16) char smem_dyn[];
  __shared__ uint64_t scan_tmp[33];
  __shared__ int32_t ns_count[kMaxNodesets];
  __shared__ int32_t ns_base[kMaxNodesets];
  __shared__ int32_t es_count[kMaxEdgesets];
  __shared__ unsigned int stats[3];
  __shared__ int32_t wtot[8];
  __shared__ int lbits_s;

  const int T = p.T;
  int32_t* cnt = reinterpret_cast<int32_t*>(smem_dyn);
  int32_t* dbase = cnt + (blockDim.x >> 5) * 256;
  char* base = p.global_work != nullptr ? p.global_work + static_cast<size_t>(sample) * p.work_stride
                                        : smem_dyn + counter_bytes(blockDim.x);
  const Work w = carve_work(base, T, p.H);
  const uint32_t slot = static_cast<uint32_t>(sample);

  __shared__ uint2 call_s;
  const int64_t seed = p.seeds[sample];
  const bool has_ts = p.seed_ts != nullptr;
  const int64_t sts = has_ts ? p.seed_ts[sample] : 0;
  const int64_t mask = p.masks != nullptr ? p.masks[sample] : -1;

  for (int i = threadIdx.x; i < p.num_nodesets; i += blockDim.x) ns_count[i] = 0;
  for (int i = threadIdx.x; i < p.num_edgesets; i += blockDim.x) es_count[i] = 0;
  if (threadIdx.x < 3) stats[threadIdx.x] = 0;
  if (threadIdx.x == 0) {
    const unsigned long long cidx =
        p.call_dev != nullptr ? *p.call_dev : ((static_cast<unsigned long long>(p.call_hi) << 32) | p.call_lo);
    call_s = make_uint2(static_cast<uint32_t>(cidx), static_cast<uint32_t>(cidx >> 32));
    bool ok = true;
    if (p.root_has_children && (seed < 0 || seed >= p.root_num_src)) {
      atomicMin(&p.status[0], static_cast<unsigned long long>(sample));
      ok = false;
    }
    w.node[0] = ok ? static_cast<int32_t>(seed) : -1;
  }
  __syncthreads();

  // 1. Level-synchronous expansion: picks (CSR positions, in the dedup
  //    table's words, which are free until the relabel), then the column
  //    loads of all picks of the level in parallel.
  long long* at = reinterpret_cast<long long*>(w.slot);
  const uint2 call = call_s;
  for (int d = 0; d < p.depth; ++d) {
    const int t0 = p.level[d], t1 = p.level[d + 1];
    // Temporal cutoffs first (local ids are not numbered yet: their array
    // is free and holds one cutoff per task of the level).
    const bool pre = has_ts && (t1 - t0) <= T;
    if (pre) {
      cutoff_prepass(p, w, w.local, t0, t1, sts, stats);
      __syncthreads();
    }
    for (int t = t0 + threadIdx.x; t < t1; t += blockDim.x) {
      const int4 task = p.tasks[t];
      expand_task(p, at, task.x, task.y, task.z, w.node[task.x], has_ts, sts, mask, slot, call,
                  pre ? w.local[t - t0] : -1, stats);
    }
    __syncthreads();
    load_children(p, w, at, p.clevel[d], p.clevel[d + 1]);
    __syncthreads();
  }

  // 2. Relabel. Dedup slot word = (node key << 32) | smallest position;
  //    after numbering, the low word holds 0x80000000 | local id (never a
  //    position, so later first-discovery tests fail for every position).
  if (p.with_replacement) {
    for (int q = threadIdx.x; q < T; q += blockDim.x) w.local[q] = -1;
    __syncthreads();
  } else {
    for (int i = threadIdx.x; i < p.H; i += blockDim.x) w.slot[i] = kEmptyKey;
    __syncthreads();
    const uint32_t hmask = static_cast<uint32_t>(p.H - 1);
    for (int q = threadIdx.x; q < T; q += blockDim.x) {
      const int32_t v = w.node[q];
      int32_t slot_q = -1;
      if (v >= 0) {
        const int ns = p.num_nodesets == 1 ? 0 : (p.pos_info[q].y & 0xFF);
        const uint32_t key = p.ns_key_base[ns] + static_cast<uint32_t>(v);
        const unsigned long long entry = (static_cast<unsigned long long>(key) << 32) | static_cast<uint32_t>(q);
        uint32_t h = ((key * 0x9E3779B1u) >> (32 - p.log2H)) & hmask;
        for (int probe = 0; probe < p.H; ++probe) {
          const unsigned long long prev = atomicCAS(&w.slot[h], kEmptyKey, entry);
          if (prev == kEmptyKey) {
            slot_q = static_cast<int32_t>(h);
            break;
          }
          if (static_cast<uint32_t>(prev >> 32) == key) {
            atomicMin(&w.slot[h], entry);
            slot_q = static_cast<int32_t>(h);
            break;
          }
          h = (h + 1) & hmask;
        }
        if (slot_q < 0) atomicOr(&p.status[2], 1ull);
      }
      w.local[q] = slot_q;
    }
    __syncthreads();
  }
  // Number first discoveries per nodeset in position order. Warps own
  // contiguous position ranges (rounds of 32); pass 1 counts first
  // discoveries per (warp, nodeset), pass 2 ranks them: rank = first
  // discoveries of the nodeset in earlier warps + earlier rounds + earlier
  // lanes. A position is a first discovery iff the dedup word of its node
  // still holds it as the minimum position (the rank written by pass 2 has
  // bit 31 set, so it never equals a position).
  const int nw = blockDim.x >> 5, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t lt = (1u << lane) - 1u;
  const int NS = p.num_nodesets;
  int32_t* wcnt = cnt;  // [nw][NS]; the radix-sort counters are free here
  const int pchunk = ((T + nw - 1) / nw + 31) & ~31;
  const int plo = min(T, warp * pchunk), phi = min(T, plo + pchunk);
  auto first_ns = [&](int q) -> int {
    if (q >= phi) return -1;
    if (p.with_replacement) {
      if (w.node[q] < 0) return -1;
    } else {
      const int32_t sl = w.local[q];
      if (sl < 0 || static_cast<uint32_t>(w.slot[sl]) != static_cast<uint32_t>(q)) return -1;
    }
    return NS == 1 ? 0 : (p.pos_info[q].y & 0xFF);
  };
  for (int i = threadIdx.x; i < nw * NS; i += blockDim.x) wcnt[i] = 0;
  __syncthreads();
  for (int b = plo; b < phi; b += 32) {
    const int ns = first_ns(b + lane);
    const uint32_t peers = __match_any_sync(0xffffffffu, ns);
    if (ns >= 0 && (peers & lt) == 0) wcnt[warp * NS + ns] += __popc(peers);
  }
  __syncthreads();
  for (int g = threadIdx.x; g < NS; g += blockDim.x) {
    int32_t run = 0;
    for (int v = 0; v < nw; ++v) {
      const int32_t c = wcnt[v * NS + g];
      wcnt[v * NS + g] = run;
      run += c;
    }
    ns_count[g] = run;
  }
  __syncthreads();
  for (int b = plo; b < phi; b += 32) {
    const int q = b + lane;
    const int ns = first_ns(q);
    const uint32_t peers = __match_any_sync(0xffffffffu, ns);
    if (ns >= 0) {
      const uint32_t rank = static_cast<uint32_t>(wcnt[warp * NS + ns]) + __popc(peers & lt);
      if (p.with_replacement) {
        w.local[q] = static_cast<int32_t>(rank);
      } else {
        const int32_t sl = w.local[q];
        w.slot[sl] = (w.slot[sl] & 0xFFFFFFFF00000000ull) | (0x80000000u | rank);
      }
    }
    __syncwarp();
    if (ns >= 0 && (peers & lt) == 0) wcnt[warp * NS + ns] += __popc(peers);
    __syncwarp();
  }
  __syncthreads();
  if (!p.with_replacement) {
    for (int q = threadIdx.x; q < T; q += blockDim.x) {
      const int32_t sl = w.local[q];
      w.local[q] = sl >= 0 ? static_cast<int32_t>(static_cast<uint32_t>(w.slot[sl]) & 0x7FFFFFFFu) : -1;
    }
  }
  if (threadIdx.x == 0) {
    int32_t acc = 0, most = 1;
    for (int g = 0; g < NS; ++g) {
      ns_base[g] = acc;
      acc += ns_count[g];
      most = ns_count[g] > most ? ns_count[g] : most;
    }
    lbits_s = max(1, 32 - __clz(most - 1));
  }
  __syncthreads();

  // Nodes of this seed, per nodeset in local-id order. Every occurrence of a
  // node writes the same value to its local slot.
  int32_t* out_nodes = p.scratch_nodes + sample * static_cast<int64_t>(T);
  for (int q = threadIdx.x; q < T; q += blockDim.x) {
    const int32_t v = w.node[q];
    if (v < 0) continue;
    const int ns = NS == 1 ? 0 : (p.pos_info[q].y & 0xFF);
    const int32_t l = w.local[q];
    if (l >= 0) out_nodes[ns_base[ns] + l] = v;
  }

  // 3. Edge keys (edgeset | src_local | dst_local), local ids in lb bits (the
  //    widest local id of this sample), one per occupied non-root position,
  //    compacted in position order by warp ballots, radix-sorted (stable)
  //    and deduplicated. The dedup table's words are free again.
  const int lb = lbits_s;
  const int esbits = p.keybits - 2 * p.pbits;
  unsigned long long* keys = w.slot;
  unsigned long long* tmp = w.slot + T;
  auto edge_key = [&](int q, unsigned long long* key) -> bool {
    if (q < 1 || q >= phi || w.node[q] < 0 || w.local[q] < 0) return false;
    const int2 info = p.pos_info[q];
    const EdgeDev& E = p.edges[info.y >> 8];
    const unsigned long long a = static_cast<uint32_t>(w.local[info.x]);
    const unsigned long long b = static_cast<uint32_t>(w.local[q]);
    const unsigned long long src = E.reversed ? b : a, dst = E.reversed ? a : b;
    *key = (static_cast<unsigned long long>(E.edgeset) << (2 * lb)) | (src << lb) | dst;
    return true;
  };
  // Pass 1 computes each position's key once (staged by position in the
  // sort's spare half; a real key is < 2^56, ~0 marks none) and counts them
  // per warp; pass 2 compacts the staged keys in position order.
  unsigned long long* staged = tmp;
  int32_t wsum = 0;
#pragma unroll 4
  for (int b = plo; b < phi; b += 32) {
    const int q = b + lane;
    unsigned long long key = ~0ull;
    const bool ok = edge_key(q, &key);
    if (q < phi) staged[q] = ok ? key : ~0ull;
    wsum += __popc(__ballot_sync(0xffffffffu, ok));
  }
  if (lane == 0) wtot[warp] = wsum;
  __syncthreads();
  int32_t wbase = 0, n_keys = 0;
  for (int v = 0; v < nw; ++v) {
    wbase += v < warp ? wtot[v] : 0;
    n_keys += wtot[v];
  }
  for (int b = plo; b < phi; b += 32) {
    const int q = b + lane;
    const unsigned long long key = q < phi ? staged[q] : ~0ull;
    const bool ok = key != ~0ull;
    const uint32_t m = __ballot_sync(0xffffffffu, ok);
    if (ok) keys[wbase + __popc(m & lt)] = key;
    wbase += __popc(m);
  }
  __syncthreads();
  const unsigned long long* ek;
  if (n_keys <= static_cast<int>(blockDim.x)) {
    // Few keys (the usual case): one key per thread, stable rank = keys
    // smaller, or equal at a smaller index; one pass, no digit passes.
    if (static_cast<int>(threadIdx.x) < n_keys) {
      const int me = static_cast<int>(threadIdx.x);
      const unsigned long long k = keys[me];
      int rank = 0;
      for (int j = 0; j < n_keys; ++j) {
        const unsigned long long kj = keys[j];
        rank += (kj < k || (kj == k && j < me)) ? 1 : 0;
      }
      tmp[rank] = k;
    }
    __syncthreads();
    ek = tmp;
  } else {
    ek = block_radix_sort(keys, tmp, n_keys, esbits + 2 * lb, cnt, dbase);
  }
  uint64_t* out_edges = p.scratch_edges + sample * static_cast<int64_t>(T);
  const unsigned long long lmask = (1ull << lb) - 1;
  auto is_new = [&](int i) -> uint64_t { return (i == 0 || ek[i - 1] != ek[i]) ? 1ull : 0ull; };
  auto put = [&](int i, uint64_t pre) {
    const unsigned long long k = ek[i];
    if (i == 0 || ek[i - 1] != k) {
      const unsigned long long es = k >> (2 * lb);
      out_edges[pre] = (es << 48) | (((k >> lb) & lmask) << 24) | (k & lmask);
      atomicAdd(&es_count[static_cast<int>(es)], 1);
    }
  };
  block_scan_items(n_keys, is_new, put, scan_tmp);

  for (int s = threadIdx.x; s < p.num_nodesets; s += blockDim.x) p.node_cnt[s * p.B + sample] = ns_count[s];
  for (int e = threadIdx.x; e < p.num_edgesets; e += blockDim.x) p.edge_cnt[e * p.B + sample] = es_count[e];
  if (threadIdx.x < 3) atomicAdd(&p.status[3 + threadIdx.x], static_cast<unsigned long long>(stats[threadIdx.x]));
}

// Padded sampler: one CTA per seed. Without an overflow list it samples seed
// blockIdx.x; with one (after the warp sampler) its CTAs take the listed
// seeds in turn.
__global__ void __launch_bounds__(256) sample_kernel(Params p) {
  if (p.overflow_list == nullptr) {
    sample_one(p, blockIdx.x);
    return;
  }
  const unsigned int n = *p.overflow_count;
  for (unsigned int i = blockIdx.x; i < n; i += gridDim.x) {
    sample_one(p, p.overflow_list[i]);
    __syncthreads();  // the next seed re-initialises the CTA's shared state
  }
}

// ===========================================================================
// Warp sampler: one warp per seed over the occupied tree positions only.
//
// The padded tree has T positions, but on power-law graphs only a few
// percent of them are occupied (rows shorter than the hop width, empty
// rows). The warp sampler keeps one compact entry per occupied position
// (node id, padded position, parent entry, plan node) in shared memory,
// level by level, so every phase costs the entries a seed really has:
//   1. expansion: the tasks (entry, plan edge) of a level go to the lanes,
//      one round of 32 at a time: each lane loads its row bounds, finds a
//      temporal cutoff with an 8-pivot search (ceil(log9(d)) dependent
//      loads), and the round's Philox blocks (same counters as the padded
//      sampler: tree position, plan edge, seed slot, call) are computed
//      lane-parallel before each lane runs its task's Floyd steps (a 64-bit
//      mask for rows of at most 64 valid entries); a warp scan gives each
//      task its place among the next level's entries; then the lanes load
//      the picked columns, four in flight each;
//   2. numbering: an entry's rank in depth-first order is the number of
//      entries with a smaller padded position (all pairs, broadcast loads);
//      a hash table keeps each node's smallest rank (atomicMin) and a walk
//      over the entries in rank order numbers first discoveries per node set
//      (__match_any_sync), exactly the reference's first-discovery order;
//   3. edges: one 32-bit key (edgeset | src | dst) per non-root entry,
//      sorted by a bitonic network over registers and lane shuffles,
//      deduplicated by a ballot scan.
// Results go to the same per-seed scratch slices as the padded sampler's,
// so the compaction is shared and every tier gives identical batches. Tiers:
// the warp sampler proper (4 warps per CTA, 32..128 entries) takes every
// seed; a seed whose tree outgrows it is listed for the large-tree tier (one
// CTA of four warps per seed, up to 512 entries), and a seed beyond that for
// the padded sampler. Each starts the seed again with
// the same random stream.
// ===========================================================================
constexpr int kWarpCapMax = 128;  // 4 entries per lane: ranks and edge sorts by one all-pairs pass
constexpr int kWarpsPerCta = 4;
constexpr int kCtaWarps = 4;  // warps of one large-tree CTA
constexpr int kMaxWarpDepth = 30;

__host__ __device__ inline int warp_region_bytes(int cap, int ns, int es, int depth) {
  const int b = 24 * cap + 4 * (ns + es + depth + 2);
  return (b + 15) & ~15;
}

// upper_bound(ts[0, n), cut): entries with ts <= cut. Eight pivots per round,
// all loads of a round in flight; rows of <= 8 entries take one round.
__device__ __forceinline__ int64_t upper_bound_9ary(const int64_t* __restrict__ ts, int64_t n, int64_t cut,
                                                    unsigned int* probes) {
  int64_t lo = 0, hi = n;
  while (hi - lo > 8) {
    const int64_t len = hi - lo;
    int64_t v[8];
#pragma unroll
    for (int g = 0; g < 8; ++g) v[g] = __ldg(ts + lo + ((g + 1) * len) / 9);
    int c = 0;
#pragma unroll
    for (int g = 0; g < 8; ++g) c += v[g] <= cut ? 1 : 0;  // pivots <= cut form a prefix
    const int64_t base = lo;
    if (c > 0) lo = base + (c * len) / 9 + 1;
    if (c < 8) hi = base + ((c + 1) * len) / 9;
    *probes += 8;
  }
  const int64_t len = hi - lo;
  int64_t v[8];
#pragma unroll
  for (int g = 0; g < 8; ++g) v[g] = g < len ? __ldg(ts + lo + g) : 0;
  int c = 0;
#pragma unroll
  for (int g = 0; g < 8; ++g) c += (g < len && v[g] <= cut) ? 1 : 0;
  *probes += static_cast<unsigned int>(len);
  return lo + c;
}

constexpr int kRegPicks = 16;  // register-resident Floyd picks (power of two)

// Philox block of draw pair m >> 1 of one expansion task (the padded
// sampler's counters: tree position, plan edge | block index, seed slot,
// call index).
__device__ __forceinline__ U4 task_block(uint32_t key0, uint32_t key1, int32_t q, int32_t e, int32_t m, uint32_t slot,
                                         uint2 call) {
  const U4 c{static_cast<uint32_t>(q), static_cast<uint32_t>(e) | ((static_cast<uint32_t>(m) >> 1) << 16), slot, call.x};
  return philox4x32_10(c, key0 ^ call.y, key1);
}

// Picks of one round of tasks (one task per lane; all lanes call): into
// at[0, cnt) of each lane's task, CSR positions in adjacency order. Random
// mode: Floyd's k-subset of the valid row. The Philox blocks of the whole
// round (counters: tree position, plan edge | block index, seed slot, call
// index; two 64-bit draws per block, as in the padded sampler) are computed
// lane-parallel into `stage` (stage_blocks blocks at a time), then each lane
// runs its task's Floyd steps over its draws: rows of at most 64 valid
// entries keep the chosen set as a 64-bit mask (O(1) duplicate test, the set
// bits come out in adjacency order), longer rows use the task's own array.
// FIRST / MOST_RECENT (and random with cnt == nv): the first / last cnt
// valid entries.
template <bool kReg>
__device__ __forceinline__ void warp_round_picks(uint32_t key0, uint32_t key1, long long* at, int32_t cnt, int64_t rb,
                                                 int64_t nv, int64_t moff, int mode, int32_t q, int32_t e,
                                                 uint32_t slot, uint2 call, unsigned long long* stage,
                                                 int stage_blocks) {
  constexpr unsigned FULL = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  const bool rnd = mode == DGFX_MODE_RANDOM && cnt > 0 && cnt < nv;
  if (!rnd && cnt > 0) {
    const int64_t first = (mode == DGFX_MODE_MOST_RECENT) ? nv - cnt : 0;
    for (int32_t i = 0; i < cnt; ++i) {
      int64_t off = first + i;
      if (moff >= 0 && off >= moff) ++off;
      at[i] = rb + off;
    }
  }
  const int nb = rnd ? (cnt + 1) >> 1 : 0;
  const int incl = warp_inclusive_scan(nb);
  const int total = __shfl_sync(FULL, incl, 31);
  if (total == 0) return;
  const int off = incl - nb;
  const bool small = nv <= 64;
  // kReg: rows longer than 64 with at most kRegPicks picks keep the chosen
  // offsets in registers (unrolled duplicate test, sorting network; more
  // code, shorter dependent chains, for the latency-bound large-tree tier);
  // otherwise the task's own array.
  const bool reg = kReg && !small && cnt <= kRegPicks && nv <= 0x7FFFFFFF;
  uint32_t ch[kRegPicks];
#pragma unroll
  for (int i = 0; i < kRegPicks; ++i) ch[i] = 0xFFFFFFFFu;  // never an offset (nv <= 2^31 - 1)
  unsigned long long chosen = 0;
  int32_t m = 0;
  for (int base = 0; base < total; base += stage_blocks) {
    const int end = min(total, base + stage_blocks);
    for (int b0 = base; b0 < end; b0 += 32) {
      const int b = b0 + lane;
      // Owner of block b: the last lane whose first block is <= b.
      int L = 0;
#pragma unroll
      for (int step = 16; step > 0; step >>= 1) {
        const int oc = __shfl_sync(FULL, off, min(L + step, 31));
        if (L + step <= 31 && oc <= b) L += step;
      }
      const int32_t qo = __shfl_sync(FULL, q, L);
      const int32_t eo = __shfl_sync(FULL, e, L);
      const int offo = __shfl_sync(FULL, off, L);
      if (b < end) {
        const U4 r = task_block(key0, key1, qo, eo, 2 * (b - offo), slot, call);
        stage[2 * (b - base)] = static_cast<unsigned long long>(r.y) << 32 | r.x;
        stage[2 * (b - base) + 1] = static_cast<unsigned long long>(r.w) << 32 | r.z;
      }
    }
    __syncwarp();
    if (rnd) {
      for (; m < cnt && off + (m >> 1) < end; ++m) {
        const uint64_t r = stage[2 * (off + (m >> 1) - base) + (m & 1)];
        const int64_t j = nv - cnt + m;
        int64_t t = static_cast<int64_t>(bounded64(r, static_cast<uint64_t>(j + 1)));
        if (small) {
          if ((chosen >> t) & 1ull) t = j;
          chosen |= 1ull << t;
        } else if (reg) {
          bool dup = false;
#pragma unroll
          for (int i = 0; i < kRegPicks; ++i) dup |= ch[i] == static_cast<uint32_t>(t);
          if (dup) t = j;
#pragma unroll
          for (int i = 0; i < kRegPicks; ++i) ch[i] = i == m ? static_cast<uint32_t>(t) : ch[i];
        } else {
          for (int32_t i = 0; i < m; ++i) {
            if (at[i] == t) {
              t = j;
              break;
            }
          }
          at[m] = t;
        }
      }
    }
    __syncwarp();
  }
  if (!rnd) return;
  if (small) {
    for (int32_t i = 0; i < cnt; ++i) {
      long long o = __ffsll(static_cast<long long>(chosen)) - 1;
      chosen &= chosen - 1;
      if (moff >= 0 && o >= moff) ++o;
      at[i] = rb + o;
    }
    return;
  }
  if (reg) {  // adjacency order: bitonic network (unused slots sort last)
#pragma unroll
    for (int k = 2; k <= kRegPicks; k <<= 1) {
#pragma unroll
      for (int j = k >> 1; j > 0; j >>= 1) {
#pragma unroll
        for (int i = 0; i < kRegPicks; ++i) {
          const int l = i ^ j;
          if (l > i) {
            const uint32_t a = ch[i], b = ch[l];
            const bool swap = (a > b) == ((i & k) == 0);
            ch[i] = swap ? b : a;
            ch[l] = swap ? a : b;
          }
        }
      }
    }
#pragma unroll
    for (int i = 0; i < kRegPicks; ++i) {
      if (i < cnt) {
        long long o = ch[i];
        if (moff >= 0 && o >= moff) ++o;
        at[i] = rb + o;
      }
    }
    return;
  }
  for (int32_t i = 1; i < cnt; ++i) {  // adjacency order
    const long long x = at[i];
    int32_t j = i - 1;
    while (j >= 0 && at[j] > x) {
      at[j + 1] = at[j];
      --j;
    }
    at[j + 1] = x;
  }
  for (int32_t i = 0; i < cnt; ++i) {
    long long o = at[i];
    if (moff >= 0 && o >= moff) ++o;
    at[i] = rb + o;
  }
}

// Per-warp shared arrays (capacity C entries).
struct WarpArrays {
  long long* at;     // [C] CSR positions of picks; then the dedup table; then edge keys
  int32_t* node;     // [C] node ids; with pos, the sorted edge keys at the end
  int32_t* pos;      // [C] padded positions; then dedup slots
  int32_t* meta;     // [C] parent entry << 8 | plan node
  uint16_t* order;   // [C] entry of each depth-first rank
  uint16_t* local;   // [C] rank, then local id
  int32_t* ns_cnt;   // [NS]
  int32_t* es_cnt;   // [ES]
  int32_t* lv;       // [depth + 2] level boundaries
};

// Bitonic sort (ascending) of G * R keys held R per thread in blocked order:
// element e = t * R + r, t the thread's index in its group of G threads
// (one warp, or with kCta a CTA of kCtaWarps warps whose cross-warp stages
// exchange through `xchg`, G * R words of shared memory, between barriers).
// Stages within a thread swap registers, stages across lanes use shuffles.
template <int R, bool kCta>
__device__ __forceinline__ void bitonic_sort_blocked(uint32_t (&v)[R], int t, uint32_t* xchg) {
  constexpr int G = kCta ? kCtaWarps * 32 : 32;
  constexpr int P = G * R;
  const int lane = threadIdx.x & 31;
  auto ce = [&](int a, int b, int k) {  // a < b, both in this thread
    const bool up = ((t * R + a) & k) == 0;
    const uint32_t x = v[a], y = v[b];
    const bool swap = (x > y) == up;
    v[a] = swap ? y : x;
    v[b] = swap ? x : y;
  };
  for (int k = 2; k <= P; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      if (j < R) {
        if constexpr (R >= 2) {
          if (j == 1) {
            ce(0, 1, k);
            if constexpr (R == 4) ce(2, 3, k);
          } else if constexpr (R == 4) {
            ce(0, 2, k);
            ce(1, 3, k);
          }
        }
      } else if (j < 32 * R) {
        const int d = j / R;  // lane distance
        const bool lower = (lane & d) == 0;
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const uint32_t o = __shfl_xor_sync(0xffffffffu, v[r], d);
          const bool up = ((t * R + r) & k) == 0;
          v[r] = (lower == up) ? min(v[r], o) : max(v[r], o);
        }
      } else if constexpr (kCta) {
#pragma unroll
        for (int r = 0; r < R; ++r) xchg[t * R + r] = v[r];
        __syncthreads();
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const int e = t * R + r;
          const uint32_t o = xchg[e ^ j];
          const bool lower = (e & j) == 0;
          const bool up = (e & k) == 0;
          v[r] = (lower == up) ? min(v[r], o) : max(v[r], o);
        }
        __syncthreads();
      }
    }
  }
}

// Deduplication table of the compact samplers: 32-bit words (rank << 16 |
// entry), the smallest rank of each node kept by atomicMin; a slot's node is
// read through the entry it holds. Empty slots hold ~0 (ranks stay below
// 2^15). Returns the slot, or -1 if the table is full (cannot happen: H > n).
constexpr uint32_t kEmptyWord = 0xFFFFFFFFu;
__device__ __forceinline__ int dedup_insert(const Params& p, uint32_t* tab, int H, int log2H, uint32_t key,
                                            uint32_t word, const int32_t* node, const int32_t* meta, int NS) {
  uint32_t h = (key * 0x9E3779B1u) >> (32 - log2H);
  for (int probe = 0; probe < H; ++probe) {
    const uint32_t prev = atomicCAS(&tab[h], kEmptyWord, word);
    if (prev == kEmptyWord) return static_cast<int>(h);
    const int j = static_cast<int>(prev & 0xFFFFu);
    const int nsj = NS == 1 ? 0 : p.pnodes[meta[j] & 0xFF].nodeset;
    if (p.ns_key_base[nsj] + static_cast<uint32_t>(node[j]) == key) {
      atomicMin(&tab[h], word);
      return static_cast<int>(h);
    }
    h = (h + 1) & static_cast<uint32_t>(H - 1);
  }
  return -1;
}

// Samples one seed with arrays of capacity C = 32 * K (K entries per lane
// in the all-pairs passes); returns false (nothing written) if the tree has
// more than C occupied positions.
template <int K>
__device__ __forceinline__ bool warp_sample_one(const Params& p, const WarpArrays& w, const int64_t sample,
                                                uint2 call) {
  constexpr int C = 32 * K;
  constexpr unsigned FULL = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  const uint32_t lt = (1u << lane) - 1u;
  const int NS = p.num_nodesets, ES = p.num_edgesets, D = p.depth;
  long long* at = w.at;
  int32_t* node = w.node;
  int32_t* pos = w.pos;
  int32_t* meta = w.meta;
  uint16_t* order = w.order;
  uint16_t* local = w.local;
  int32_t* ns_cnt = w.ns_cnt;
  int32_t* es_cnt = w.es_cnt;
  int32_t* lv = w.lv;

  const uint32_t slot = static_cast<uint32_t>(sample);
  const bool has_ts = p.seed_ts != nullptr;
  const int64_t sts = has_ts ? p.seed_ts[sample] : 0;
  const int64_t mask = p.masks != nullptr ? p.masks[sample] : -1;
  const int64_t seed = p.seeds[sample];
  const bool ok = !(p.root_has_children && (seed < 0 || seed >= p.root_num_src));
  if (!ok && lane == 0) atomicMin(&p.status[0], static_cast<unsigned long long>(sample));
  for (int i = lane; i < NS; i += 32) ns_cnt[i] = 0;
  for (int i = lane; i < ES; i += 32) es_cnt[i] = 0;
  if (lane == 0) {
    node[0] = static_cast<int32_t>(seed);
    pos[0] = 0;
    meta[0] = 0;  // plan node 0, no parent
    lv[0] = 0;
    lv[1] = ok ? 1 : 0;
  }
  __syncwarp();
  unsigned int st_rows = 0, st_picks = 0, st_probes = 0;

  // 1. Expansion, level by level; tasks in chunks of two rounds.
  bool overflow = false;
  const int maxm = p.max_edges_per_node;
  for (int d = 0; d < D; ++d) {
    const int l0 = lv[d], l1 = lv[d + 1];
    int fill = l1;
    const int ntask = (l1 - l0) * maxm;
    for (int t0 = 0; t0 < ntask; t0 += 32) {
      const int t = t0 + lane;
      int32_t cnt = 0, pe = -1, q = 0, ent = 0;
      int64_t rb = 0, nv = 0, moff = -1;
      int md = p.mode;
      if (t < ntask) {
        const int e = l0 + t / maxm, j = t - (t / maxm) * maxm;
        const PlanNodeDev P = p.pnodes[meta[e] & 0xFF];
        if (j < P.num_edges) {
          pe = P.first_edge + j;
          ent = e;
          q = pos[e];
          const EdgeDev& E = p.edges[pe];
          const int32_t v = node[e];
          rb = __ldg(E.rowptr + v);
          int64_t n = __ldg(E.rowptr + v + 1) - rb;
          const bool temporal = has_ts && E.ts != nullptr;
          if (!has_ts && E.ts != nullptr) {
            // SampleRandomUniform / SampleFirst on a temporal index fail
            // (in_memory_sampler.cc:26-30, 168-172).
            atomicOr(&p.status[1], 1ull);
            n = 0;
          }
          if (temporal && n > 0) n = upper_bound_9ary(E.ts + rb, n, sts, &st_probes);
          if (!temporal && mask >= 0 && E.edgeset == p.mask_edgeset && E.edge_pos != nullptr && mask < E.num_edges) {
            const int64_t ps = E.edge_pos[mask];
            if (ps >= rb && ps < rb + n) moff = ps - rb;
          }
          nv = n - (moff >= 0 ? 1 : 0);
          cnt = static_cast<int32_t>(nv < E.k ? nv : E.k);
          md = (p.mode == DGFX_MODE_MOST_RECENT && !temporal) ? DGFX_MODE_RANDOM : p.mode;
          ++st_rows;
          st_picks += static_cast<unsigned int>(cnt);
        }
      }
      const int32_t inc = warp_inclusive_scan(cnt);
      const int32_t tot = __shfl_sync(FULL, inc, 31);
      if (fill + tot > C) {
        overflow = true;
        break;
      }
      const int32_t out = fill + inc - cnt;
      warp_round_picks<false>(p.key0, p.key1, at + out, cnt, rb, nv, moff, md, q, pe, slot, call,
                              reinterpret_cast<unsigned long long*>(order), C / 4);
      if (cnt > 0) {
        const EdgeDev& E = p.edges[pe];
        const int32_t base = q + E.rel_off;
        const int32_t mt = (ent << 8) | E.child;
        for (int32_t i = 0; i < cnt; ++i) {
          pos[out + i] = base + i * E.stride;
          meta[out + i] = mt;
        }
      }
      fill += tot;
    }
    if (overflow) break;
    __syncwarp();
    // Columns of the new entries, four loads in flight per lane.
    for (int i0 = l1 + lane; i0 < fill; i0 += 32 * 4) {
      int32_t v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + 32 * u;
        v[u] = -1;
        if (i < fill) v[u] = __ldg(p.edges[p.pnodes[meta[i] & 0xFF].in_edge].col + at[i]);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (i0 + 32 * u < fill) node[i0 + 32 * u] = v[u];
      }
    }
    if (lane == 0) lv[d + 2] = fill;
    __syncwarp();
  }
  if (overflow) {  // redone with larger arrays (its work is counted there)
    __syncwarp();
    return false;
  }
  st_rows = warp_reduce_sum(st_rows);
  st_picks = warp_reduce_sum(st_picks);
  st_probes = warp_reduce_sum(st_probes);
  if (lane == 0) {
    atomicAdd(&p.status[3], static_cast<unsigned long long>(st_rows));
    atomicAdd(&p.status[4], static_cast<unsigned long long>(st_picks));
    atomicAdd(&p.status[5], static_cast<unsigned long long>(st_probes));
  }
  const int n = lv[D + 1];

  // 2. Numbering. Rank in depth-first order = number of entries with a
  //    smaller position (up to 32 entries: all pairs by broadcast loads).
  if (n <= 32) {
    const int32_t pk = lane < n ? pos[lane] : 0x7FFFFFFF;
    int rk = 0;
    for (int j = 0; j < n; ++j) rk += pos[j] < pk ? 1 : 0;
    if (lane < n) {
      local[lane] = static_cast<uint16_t>(rk);
      order[rk] = static_cast<uint16_t>(lane);
    }
  } else {
    // More entries: the entries of a level are in position order, so the
    // rank is the index within the own level plus a binary search in each
    // other level (fewer instructions than all pairs).
    for (int i = lane; i < n; i += 32) {
      const int32_t pi = pos[i];
      int r = 0;
      for (int L = 0; L <= D; ++L) {
        const int lo = lv[L], hi = lv[L + 1];
        if (i >= lo && i < hi) {
          r += i - lo;
          continue;
        }
        int a = lo, b = hi;
        while (a < b) {
          const int m = (a + b) >> 1;
          if (pos[m] < pi) a = m + 1;
          else b = m;
        }
        r += a - lo;
      }
      local[i] = static_cast<uint16_t>(r);
      order[r] = static_cast<uint16_t>(i);
    }
  }
  __syncwarp();
  uint32_t* tab = reinterpret_cast<uint32_t*>(at);  // 2 C words
  if (!p.with_replacement) {
    int H = 2;
    while (H < 2 * n && H < 2 * C) H <<= 1;
    const int log2H = 31 - __clz(H);
    for (int i = lane; i < H; i += 32) tab[i] = kEmptyWord;
    __syncwarp();
    for (int i = lane; i < n; i += 32) {
      const int ns = NS == 1 ? 0 : p.pnodes[meta[i] & 0xFF].nodeset;
      const uint32_t key = p.ns_key_base[ns] + static_cast<uint32_t>(node[i]);
      const int where = dedup_insert(p, tab, H, log2H, key, (static_cast<uint32_t>(local[i]) << 16) | i, node,
                                     meta, NS);
      if (where < 0) atomicOr(&p.status[2], 1ull);
      pos[i] = where;  // positions are not needed any more
    }
    __syncwarp();
  }
  // First discoveries in rank order, numbered per node set; with
  // replacement every entry is a new node.
  for (int r0 = 0; r0 < n; r0 += 32) {
    const int r = r0 + lane;
    int ns = -1, i = -1;
    if (r < n) {
      i = order[r];
      const bool first = p.with_replacement || (pos[i] >= 0 && (tab[pos[i]] >> 16) == static_cast<uint32_t>(r));
      if (first) ns = NS == 1 ? 0 : p.pnodes[meta[i] & 0xFF].nodeset;
    }
    const uint32_t peers = __match_any_sync(FULL, ns);
    int base = 0;
    if (ns >= 0) base = ns_cnt[ns];
    __syncwarp();
    if (ns >= 0) {
      const uint32_t l = static_cast<uint32_t>(base) + __popc(peers & lt);
      if (p.with_replacement) local[i] = static_cast<uint16_t>(l);
      else tab[pos[i]] = 0x80000000u | l;
      if ((peers & lt) == 0) ns_cnt[ns] = base + __popc(peers);
    }
    __syncwarp();
  }
  if (!p.with_replacement) {
    for (int i = lane; i < n; i += 32) {
      local[i] = pos[i] >= 0 ? static_cast<uint16_t>(tab[pos[i]] & 0x7FFFFFFFu) : 0;
    }
  }
  __syncwarp();
  // Nodes per node set in local-id order (every occurrence of a node writes
  // the same value).
  int most = 1;
  for (int g = 0; g < NS; ++g) most = max(most, ns_cnt[g]);
  const int lb = max(1, 32 - __clz(most - 1));
  int32_t* out_nodes = p.scratch_nodes + sample * static_cast<int64_t>(p.T);
  for (int i = lane; i < n; i += 32) {
    const int ns = NS == 1 ? 0 : p.pnodes[meta[i] & 0xFF].nodeset;
    int b = 0;
    for (int g = 0; g < ns; ++g) b += ns_cnt[g];
    out_nodes[b + local[i]] = node[i];
  }
  __syncwarp();

  // 3. Edges: a 32-bit key (edgeset | src | dst) per non-root entry,
  //    sorted, deduplicated.
  const int nk = n > 0 ? n - 1 : 0;
  auto edge_key = [&](int c) -> uint32_t {
    const int par = meta[c] >> 8;
    const EdgeDev& E = p.edges[p.pnodes[meta[c] & 0xFF].in_edge];
    const uint32_t a = local[par], b = local[c];
    const uint32_t src = E.reversed ? b : a, dst = E.reversed ? a : b;
    return (static_cast<uint32_t>(E.edgeset) << (2 * lb)) | (src << lb) | dst;
  };
  // Sorted by a register bitonic sort over 32 * KC keys (KC per lane: 1
  // for up to 32 keys, else K; two variants keep the hot code small; ~0
  // padding sorts last; equal keys are equal edges, so stability does not
  // matter).
  auto sort_keys = [&](auto kc_tag) {
    constexpr int KC = decltype(kc_tag)::value;
    uint32_t v[KC];
#pragma unroll
    for (int r = 0; r < KC; ++r) {
      const int e = lane * KC + r;
      v[r] = e < nk ? edge_key(e + 1) : ~0u;
    }
    bitonic_sort_blocked<KC, false>(v, lane, nullptr);
    uint32_t* sorted = reinterpret_cast<uint32_t*>(node);
#pragma unroll
    for (int r = 0; r < KC; ++r) {
      if (lane * KC + r < nk) sorted[lane * KC + r] = v[r];
    }
  };
  if (K == 1 || nk <= 32) sort_keys(std::integral_constant<int, 1>{});
  else sort_keys(std::integral_constant<int, K>{});
  const uint32_t* ek = reinterpret_cast<const uint32_t*>(node);
  __syncwarp();
  uint64_t* out_edges = p.scratch_edges + sample * static_cast<int64_t>(p.T);
  const uint32_t lmask = (1u << lb) - 1;
  int wbase = 0;
  for (int i0 = 0; i0 < nk; i0 += 32) {
    const int i = i0 + lane;
    const uint32_t k = i < nk ? ek[i] : ~0u;
    const bool fresh = i < nk && (i == 0 || ek[i - 1] != k);
    const uint32_t m = __ballot_sync(FULL, fresh);
    if (fresh) {
      const unsigned long long es = k >> (2 * lb);
      out_edges[wbase + __popc(m & lt)] = (es << 48) | (static_cast<unsigned long long>((k >> lb) & lmask) << 24) |
                                          (k & lmask);
      atomicAdd(&es_cnt[static_cast<int>(es)], 1);
    }
    wbase += __popc(m);
  }
  __syncwarp();
  for (int g = lane; g < NS; g += 32) p.node_cnt[g * p.B + sample] = ns_cnt[g];
  for (int g = lane; g < ES; g += 32) p.edge_cnt[g * p.B + sample] = es_cnt[g];
  __syncwarp();
  return true;
}

__device__ __forceinline__ WarpArrays carve_warp(char* base, int C, int32_t* counters, int NS, int ES) {
  WarpArrays w;
  w.at = reinterpret_cast<long long*>(base);
  w.node = reinterpret_cast<int32_t*>(base + 8 * static_cast<size_t>(C));
  w.pos = w.node + C;
  w.meta = w.pos + C;
  w.order = reinterpret_cast<uint16_t*>(w.meta + C);
  w.local = w.order + C;
  w.ns_cnt = counters;
  w.es_cnt = counters + NS;
  w.lv = counters + NS + ES;
  return w;
}

// Persistent warps: each takes the next seed from a counter in turn, so a
// warp whose seed has a large tree does not hold back the others. A seed
// that outgrows the capacity (32 K entries) is listed for the large-tree
// tier (if the sampler has one) or the padded sampler.
template <int K>
__global__ void __launch_bounds__(kWarpsPerCta * 32, 8) warp_sample_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(16) char smem_warp[];
  const int lane = threadIdx.x & 31;
  constexpr int C = 32 * K;
  const int NS = p.num_nodesets, ES = p.num_edgesets;
  char* wb = smem_warp + static_cast<size_t>(threadIdx.x >> 5) * p.warp_bytes;
  int32_t* counters = reinterpret_cast<int32_t*>(wb + 24 * static_cast<size_t>(C));  // always in shared memory
  const WarpArrays w = carve_warp(wb, C, counters, NS, ES);
  uint2 call;
  {
    const unsigned long long cidx =
        p.call_dev != nullptr ? *p.call_dev : ((static_cast<unsigned long long>(p.call_hi) << 32) | p.call_lo);
    call = make_uint2(static_cast<uint32_t>(cidx), static_cast<uint32_t>(cidx >> 32));
  }
  for (;;) {
    unsigned int s = 0;
    if (lane == 0) s = atomicAdd(p.overflow_count + 1, 1u);
    s = __shfl_sync(0xffffffffu, s, 0);
    if (static_cast<int64_t>(s) >= p.B) break;
    if (warp_sample_one<K>(p, w, static_cast<int64_t>(s), call)) {
      if (lane == 0) atomicAdd(&p.status[7], 1ull);
      continue;
    }
    // The tree outgrew the warp's arrays: a larger tier redoes it (with the
    // same random stream).
    if (lane == 0) {
      if (p.big_cap > 0) {
        p.mid_list[atomicAdd(p.mid_count, 1u)] = static_cast<int32_t>(s);
      } else {
        p.overflow_list[atomicAdd(p.overflow_count, 1u)] = static_cast<int32_t>(s);
        atomicAdd(&p.status[8], 1ull);
      }
    }
    __syncwarp();
  }
}

using WarpKernel = void (*)(const Params);
WarpKernel warp_kernel_for(int cap) {
  return cap <= 32 ? warp_sample_kernel<1> : (cap <= 64 ? warp_sample_kernel<2> : warp_sample_kernel<4>);
}
// ===========================================================================
// Large-tree tier: one CTA of kCtaWarps warps per seed over the occupied
// positions, for the seeds whose trees outgrew the warp sampler. The same
// compact entries and phases as warp_sample_one, with every per-entry loop
// spread over the CTA's threads (the tier exists because a single warp's
// per-seed latency, not throughput, bounds these seeds):
//   - expansion: tasks in rounds of blockDim; a block scan places each task's
//     picks among the next level's entries (position order, as in the warp
//     sampler); each warp draws its tasks' Philox blocks into its own
//     staging quarter;
//   - numbering: the entries of a level are in position order (children are
//     appended by parent, plan edge and pick, and a parent's subtree holds
//     its children's positions), so an entry's depth-first rank is its index
//     within its level plus one binary search per other level; the hash
//     table keeps each node's smallest rank; first discoveries are numbered
//     per node set over contiguous rank ranges, one per warp (counts per
//     warp, prefix over warps, then a walk per warp);
//   - edges: a bitonic sort of the 32-bit keys (registers, shuffles, and
//     shared memory for the cross-warp stages), deduplication by block scans
//     of the first-of-run flags.
// Capacity C entries (power of two, at most kLargeCapMax = 512: 12 KB of
// shared memory per CTA, so that nine CTAs fit an SM by both registers and
// shared memory and a batch's large trees (about a sixth of 8192 seeds on
// power-law graphs) take one wave; local ids in 9 bits keep an edge key
// within 32 bits).
// ===========================================================================
constexpr int kLargeCapMax = 512;

__host__ __device__ inline int cta_region_bytes(int cap, int ns, int es, int depth) {
  const int b = 24 * cap + 4 * (ns + es + depth + 2 + kCtaWarps * ns + 2 * kCtaWarps + 40);
  return (b + 15) & ~15;
}

// Exclusive scan of one int per thread over the CTA (kCtaWarps warps);
// `wsum` holds kCtaWarps ints. Two barriers; call from every thread.
__device__ __forceinline__ int cta_exclusive_scan(int v, int* wsum, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int inc = warp_inclusive_scan(v);
  if (lane == 31) wsum[warp] = inc;
  __syncthreads();
  int base = 0, tot = 0;
#pragma unroll
  for (int w = 0; w < kCtaWarps; ++w) {
    const int x = wsum[w];
    base += w < warp ? x : 0;
    tot += x;
  }
  __syncthreads();
  *total = tot;
  return base + inc - v;
}

// Samples one seed; returns false (nothing written) if the tree has more
// than C occupied positions. All threads of the CTA call it.
__device__ __forceinline__ bool cta_sample_one(const Params& p, const WarpArrays& w, int32_t* wcnt, int32_t* wsum,
                                            const int64_t sample, uint2 call, const int C) {
  constexpr unsigned FULL = 0xffffffffu;
  constexpr int NT = kCtaWarps * 32;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t lt = (1u << lane) - 1u;
  const int NS = p.num_nodesets, ES = p.num_edgesets, D = p.depth;
  long long* at = w.at;
  int32_t* node = w.node;
  int32_t* pos = w.pos;
  int32_t* meta = w.meta;
  uint16_t* order = w.order;
  uint16_t* local = w.local;
  int32_t* ns_cnt = w.ns_cnt;
  int32_t* es_cnt = w.es_cnt;
  int32_t* lv = w.lv;

  const uint32_t slot = static_cast<uint32_t>(sample);
  const bool has_ts = p.seed_ts != nullptr;
  const int64_t sts = has_ts ? p.seed_ts[sample] : 0;
  const int64_t mask = p.masks != nullptr ? p.masks[sample] : -1;
  const int64_t seed = p.seeds[sample];
  const bool ok = !(p.root_has_children && (seed < 0 || seed >= p.root_num_src));
  for (int i = tid; i < NS; i += NT) ns_cnt[i] = 0;
  for (int i = tid; i < ES; i += NT) es_cnt[i] = 0;
  if (tid == 0) {
    if (!ok) atomicMin(&p.status[0], static_cast<unsigned long long>(sample));
    node[0] = static_cast<int32_t>(seed);
    pos[0] = 0;
    meta[0] = 0;
    lv[0] = 0;
    lv[1] = ok ? 1 : 0;
  }
  __syncthreads();
  unsigned int st_rows = 0, st_picks = 0, st_probes = 0;
  // Each warp's Philox staging: a quarter of the order + local arrays.
  const int stage_blocks = C / (4 * kCtaWarps);
  unsigned long long* stage = reinterpret_cast<unsigned long long*>(order) + 2 * stage_blocks * warp;

  // 1. Expansion.
  bool overflow = false;
  const int maxm = p.max_edges_per_node;
  for (int d = 0; d < D && !overflow; ++d) {
    const int l0 = lv[d], l1 = lv[d + 1];
    int fill = l1;
    const int ntask = (l1 - l0) * maxm;
    for (int t0 = 0; t0 < ntask; t0 += NT) {
      const int t = t0 + tid;
      int32_t cnt = 0, pe = -1, q = 0, ent = 0;
      int64_t rb = 0, nv = 0, moff = -1;
      int md = p.mode;
      if (t < ntask) {
        const int e = l0 + t / maxm, j = t - (t / maxm) * maxm;
        const PlanNodeDev P = p.pnodes[meta[e] & 0xFF];
        if (j < P.num_edges) {
          pe = P.first_edge + j;
          ent = e;
          q = pos[e];
          const EdgeDev& E = p.edges[pe];
          const int32_t v = node[e];
          rb = __ldg(E.rowptr + v);
          int64_t n = __ldg(E.rowptr + v + 1) - rb;
          const bool temporal = has_ts && E.ts != nullptr;
          if (!has_ts && E.ts != nullptr) {
            // SampleRandomUniform / SampleFirst on a temporal index fail
            // (in_memory_sampler.cc:26-30, 168-172).
            atomicOr(&p.status[1], 1ull);
            n = 0;
          }
          if (temporal && n > 0) n = upper_bound_9ary(E.ts + rb, n, sts, &st_probes);
          if (!temporal && mask >= 0 && E.edgeset == p.mask_edgeset && E.edge_pos != nullptr && mask < E.num_edges) {
            const int64_t ps = E.edge_pos[mask];
            if (ps >= rb && ps < rb + n) moff = ps - rb;
          }
          nv = n - (moff >= 0 ? 1 : 0);
          cnt = static_cast<int32_t>(nv < E.k ? nv : E.k);
          md = (p.mode == DGFX_MODE_MOST_RECENT && !temporal) ? DGFX_MODE_RANDOM : p.mode;
          ++st_rows;
          st_picks += static_cast<unsigned int>(cnt);
        }
      }
      int tot = 0;
      const int32_t out = fill + cta_exclusive_scan(cnt, wsum, &tot);
      if (fill + tot > C) {  // uniform: every thread sees the same total
        overflow = true;
        break;
      }
      warp_round_picks<true>(p.key0, p.key1, at + out, cnt, rb, nv, moff, md, q, pe, slot, call, stage, stage_blocks);
      if (cnt > 0) {
        const EdgeDev& E = p.edges[pe];
        const int32_t base = q + E.rel_off;
        const int32_t mt = (ent << 8) | E.child;
        for (int32_t i = 0; i < cnt; ++i) {
          pos[out + i] = base + i * E.stride;
          meta[out + i] = mt;
        }
      }
      fill += tot;
    }
    if (overflow) break;
    __syncthreads();
    // Columns of the new entries, four loads in flight per thread.
    for (int i0 = l1 + tid; i0 < fill; i0 += NT * 4) {
      int32_t v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + NT * u;
        v[u] = -1;
        if (i < fill) v[u] = __ldg(p.edges[p.pnodes[meta[i] & 0xFF].in_edge].col + at[i]);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (i0 + NT * u < fill) node[i0 + NT * u] = v[u];
      }
    }
    if (tid == 0) lv[d + 2] = fill;
    __syncthreads();
  }
  if (overflow) {  // redone by the padded sampler (its work is counted there)
    __syncthreads();
    return false;
  }
  st_rows = warp_reduce_sum(st_rows);
  st_picks = warp_reduce_sum(st_picks);
  st_probes = warp_reduce_sum(st_probes);
  if (lane == 0) {
    atomicAdd(&p.status[3], static_cast<unsigned long long>(st_rows));
    atomicAdd(&p.status[4], static_cast<unsigned long long>(st_picks));
    atomicAdd(&p.status[5], static_cast<unsigned long long>(st_probes));
  }
  const int n = lv[D + 1];

  // 2. Numbering: depth-first rank by binary searches over the levels.
  for (int i = tid; i < n; i += NT) {
    const int32_t pi = pos[i];
    int r = 0;
    for (int L = 0; L <= D; ++L) {
      const int lo = lv[L], hi = lv[L + 1];
      if (i >= lo && i < hi) {
        r += i - lo;
        continue;
      }
      int a = lo, b = hi;  // first entry of level L at or after pi
      while (a < b) {
        const int m = (a + b) >> 1;
        if (pos[m] < pi) a = m + 1;
        else b = m;
      }
      r += a - lo;
    }
    local[i] = static_cast<uint16_t>(r);
    order[r] = static_cast<uint16_t>(i);
  }
  __syncthreads();
  uint32_t* tab = reinterpret_cast<uint32_t*>(at);  // 2 C words
  if (!p.with_replacement) {
    int H = 2;
    while (H < 2 * n && H < 2 * C) H <<= 1;
    const int log2H = 31 - __clz(H);
    for (int i = tid; i < H; i += NT) tab[i] = kEmptyWord;
    __syncthreads();
    for (int i = tid; i < n; i += NT) {
      const int ns = NS == 1 ? 0 : p.pnodes[meta[i] & 0xFF].nodeset;
      const uint32_t key = p.ns_key_base[ns] + static_cast<uint32_t>(node[i]);
      const int where = dedup_insert(p, tab, H, log2H, key, (static_cast<uint32_t>(local[i]) << 16) | i, node,
                                     meta, NS);
      if (where < 0) atomicOr(&p.status[2], 1ull);
      pos[i] = where;  // positions are not needed any more
    }
    __syncthreads();
  }
  // First discoveries in rank order, numbered per node set. Warp v walks
  // ranks [v * span, (v + 1) * span): pass 1 counts per node set, the
  // counts become per-warp starting offsets, pass 2 numbers.
  const int span = ((n + kCtaWarps - 1) / kCtaWarps + 31) & ~31;
  const int rlo = min(n, warp * span), rhi = min(n, rlo + span);
  auto first_ns = [&](int r, int* ent) -> int {
    *ent = -1;
    if (r >= rhi) return -1;
    const int i = order[r];
    *ent = i;
    const bool first = p.with_replacement || (pos[i] >= 0 && (tab[pos[i]] >> 16) == static_cast<uint32_t>(r));
    return first ? (NS == 1 ? 0 : p.pnodes[meta[i] & 0xFF].nodeset) : -1;
  };
  for (int i = tid; i < kCtaWarps * NS; i += NT) wcnt[i] = 0;
  __syncthreads();
  for (int r0 = rlo; r0 < rhi; r0 += 32) {
    int ent;
    const int ns = first_ns(r0 + lane, &ent);
    const uint32_t peers = __match_any_sync(FULL, ns);
    if (ns >= 0 && (peers & lt) == 0) wcnt[warp * NS + ns] += __popc(peers);
    __syncwarp();
  }
  __syncthreads();
  for (int g = tid; g < NS; g += NT) {
    int32_t run = 0;
    for (int v = 0; v < kCtaWarps; ++v) {
      const int32_t c = wcnt[v * NS + g];
      wcnt[v * NS + g] = run;
      run += c;
    }
    ns_cnt[g] = run;
  }
  __syncthreads();
  for (int r0 = rlo; r0 < rhi; r0 += 32) {
    int i;
    const int ns = first_ns(r0 + lane, &i);
    const uint32_t peers = __match_any_sync(FULL, ns);
    int base = 0;
    if (ns >= 0) base = wcnt[warp * NS + ns];
    __syncwarp();
    if (ns >= 0) {
      const uint32_t l = static_cast<uint32_t>(base) + __popc(peers & lt);
      if (p.with_replacement) local[i] = static_cast<uint16_t>(l);
      else tab[pos[i]] = 0x80000000u | l;
      if ((peers & lt) == 0) wcnt[warp * NS + ns] = base + __popc(peers);
    }
    __syncwarp();
  }
  __syncthreads();
  if (!p.with_replacement) {
    for (int i = tid; i < n; i += NT) {
      local[i] = pos[i] >= 0 ? static_cast<uint16_t>(tab[pos[i]] & 0x7FFFFFFFu) : 0;
    }
  }
  __syncthreads();
  int most = 1;
  for (int g = 0; g < NS; ++g) most = max(most, ns_cnt[g]);
  const int lb = max(1, 32 - __clz(most - 1));
  int32_t* out_nodes = p.scratch_nodes + sample * static_cast<int64_t>(p.T);
  for (int i = tid; i < n; i += NT) {
    const int ns = NS == 1 ? 0 : p.pnodes[meta[i] & 0xFF].nodeset;
    int b = 0;
    for (int g = 0; g < ns; ++g) b += ns_cnt[g];
    out_nodes[b + local[i]] = node[i];
  }

  // 3. Edges: the 32-bit keys sorted by a bitonic sort over the CTA
  //    (registers, shuffles, and shared memory across warps), then
  //    deduplication.
  const int nk = n > 0 ? n - 1 : 0;
  auto edge_key = [&](int c) -> uint32_t {
    const int par = meta[c] >> 8;
    const EdgeDev& E = p.edges[p.pnodes[meta[c] & 0xFF].in_edge];
    const uint32_t a = local[par], b = local[c];
    const uint32_t src = E.reversed ? b : a, dst = E.reversed ? a : b;
    return (static_cast<uint32_t>(E.edgeset) << (2 * lb)) | (src << lb) | dst;
  };
  uint32_t* sorted = reinterpret_cast<uint32_t*>(node);
  uint32_t* xchg = reinterpret_cast<uint32_t*>(at);  // 2 C words >= 128 * 4
  auto sort_keys = [&](auto kc_tag) {
    constexpr int KC = decltype(kc_tag)::value;
    uint32_t v[KC];
#pragma unroll
    for (int r = 0; r < KC; ++r) {
      const int e = tid * KC + r;
      v[r] = e < nk ? edge_key(e + 1) : ~0u;
    }
    __syncthreads();  // xchg overlays the dedup table read above
    bitonic_sort_blocked<KC, true>(v, tid, xchg);
#pragma unroll
    for (int r = 0; r < KC; ++r) {
      if (tid * KC + r < nk) sorted[tid * KC + r] = v[r];
    }
  };
  if (nk <= NT) sort_keys(std::integral_constant<int, 1>{});
  else if (nk <= 2 * NT) sort_keys(std::integral_constant<int, 2>{});
  else sort_keys(std::integral_constant<int, 4>{});
  __syncthreads();
  uint64_t* out_edges = p.scratch_edges + sample * static_cast<int64_t>(p.T);
  const uint32_t lmask = (1u << lb) - 1;
  int obase = 0;
  for (int i0 = 0; i0 < nk; i0 += NT) {
    const int i = i0 + tid;
    const uint32_t k = i < nk ? sorted[i] : ~0u;
    const bool fresh = i < nk && (i == 0 || sorted[i - 1] != k);
    int tot = 0;
    const int o = obase + cta_exclusive_scan(fresh ? 1 : 0, wsum, &tot);
    if (fresh) {
      const unsigned long long es = k >> (2 * lb);
      out_edges[o] = (es << 48) | (static_cast<unsigned long long>((k >> lb) & lmask) << 24) | (k & lmask);
      atomicAdd(&es_cnt[static_cast<int>(es)], 1);
    }
    obase += tot;
  }
  __syncthreads();
  for (int g = tid; g < NS; g += NT) p.node_cnt[g * p.B + sample] = ns_cnt[g];
  for (int g = tid; g < ES; g += NT) p.edge_cnt[g * p.B + sample] = es_cnt[g];
  __syncthreads();  // the next seed re-initialises the shared arrays
  return true;
}

// Persistent CTAs over the seeds the warp sampler listed; seeds beyond the
// capacity go to the padded sampler.
__global__ void __launch_bounds__(kCtaWarps * 32, 9) large_tree_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(16) char smem_large[];
  __shared__ unsigned int next_s;
  const int C = p.big_cap;
  const int NS = p.num_nodesets, ES = p.num_edgesets;
  int32_t* counters = reinterpret_cast<int32_t*>(smem_large + 24 * static_cast<size_t>(C));
  const WarpArrays w = carve_warp(smem_large, C, counters, NS, ES);
  int32_t* wcnt = counters + NS + ES + p.depth + 2;  // [kCtaWarps][NS]
  int32_t* wsum = wcnt + kCtaWarps * NS;             // [kCtaWarps]
  uint2 call;
  {
    const unsigned long long cidx =
        p.call_dev != nullptr ? *p.call_dev : ((static_cast<unsigned long long>(p.call_hi) << 32) | p.call_lo);
    call = make_uint2(static_cast<uint32_t>(cidx), static_cast<uint32_t>(cidx >> 32));
  }
  const unsigned int listed = p.mid_count[0];  // written by the warp sampler's kernel
  for (;;) {
    if (threadIdx.x == 0) {
      const unsigned int i = atomicAdd(p.mid_count + 1, 1u);
      next_s = i < listed ? static_cast<unsigned int>(p.mid_list[i]) : 0xFFFFFFFFu;
    }
    __syncthreads();
    const unsigned int s = next_s;
    __syncthreads();  // next_s is rewritten at the next turn
    if (s == 0xFFFFFFFFu || static_cast<int64_t>(s) >= p.B) break;
    if (cta_sample_one(p, w, wcnt, wsum, static_cast<int64_t>(s), call, C)) {
      if (threadIdx.x == 0) atomicAdd(&p.status[7], 1ull);
      continue;
    }
    if (threadIdx.x == 0) {
      p.overflow_list[atomicAdd(p.overflow_count, 1u)] = static_cast<int32_t>(s);
      atomicAdd(&p.status[8], 1ull);
    }
  }
}

// Largest row length of an index (the cap on useful slots per plan edge).
__global__ void max_degree_kernel(const int64_t* __restrict__ rowptr, int64_t n, unsigned long long* out) {
  unsigned long long m = 0;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const unsigned long long d = static_cast<unsigned long long>(rowptr[i + 1] - rowptr[i]);
    m = d > m ? d : m;
  }
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long x = __shfl_xor_sync(0xffffffffu, m, o);
    m = x > m ? x : m;
  }
  if ((threadIdx.x & 31) == 0) atomicMax(out, m);
}

// Start of a call: status word 0 (first bad seed slot) to ~0, words 1..5
// (flags, work counters) and 7..8 (seeds per tier) to 0; word 6 (the device
// call index) is kept. The tiers' seed counters to 0.
__global__ void reset_kernel(unsigned long long* status, unsigned int* overflow_count, unsigned int* mid_count) {
  const int i = threadIdx.x;
  if (i == 0) status[0] = ~0ull;
  if (i >= 1 && i <= 5) status[i] = 0;
  if (i == 7 || i == 8) status[i] = 0;
  if (i < 2) {
    overflow_count[i] = 0;
    mid_count[i] = 0;
  }
}

// Merged batch from the per-seed scratch: one warp per seed.
__global__ void compact_kernel(Params p, const int64_t* __restrict__ node_off, const int64_t* __restrict__ edge_off,
                               int root_ns, int64_t* __restrict__ node_ids, int64_t* __restrict__ edge_src,
                               int64_t* __restrict__ edge_dst) {
  const int64_t warp = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  // Every sample_kernel CTA has read the call index by now.
  if (p.call_dev != nullptr && blockIdx.x == 0 && threadIdx.x == 0) atomicAdd(p.call_dev, 1ull);
  if (warp >= p.B) return;
  const int64_t i = warp;
  const int32_t* src_nodes = p.scratch_nodes + i * static_cast<int64_t>(p.T);
  const uint64_t* src_edges = p.scratch_edges + i * static_cast<int64_t>(p.T);
  if (p.num_nodesets == 1 && p.num_edgesets == 1) {
    // One node set and one edge set: all four offsets, then the node and
    // edge chunks, loaded before any store (one dependent round trip each).
    const int64_t no = node_off[i], nc = node_off[i + 1] - no;
    const int64_t eo = edge_off[i], ec = edge_off[i + 1] - eo;
    const int64_t seed = p.seeds[i];
    for (int64_t j = lane; j < nc || j < ec; j += 32) {
      const int64_t v = j < nc ? static_cast<int64_t>(src_nodes[j]) : 0;
      const uint64_t k = j < ec ? src_edges[j] : 0;
      if (j < nc) node_ids[no + j] = (root_ns == 0 && j == 0) ? seed : v;
      if (j < ec) {
        edge_src[eo + j] = static_cast<int64_t>((k >> 24) & 0xFFFFFFull);
        edge_dst[eo + j] = static_cast<int64_t>(k & 0xFFFFFFull);
      }
    }
    return;
  }
  int64_t acc = 0;
  for (int s = 0; s < p.num_nodesets; ++s) {
    const int64_t o = node_off[s * p.B + i];
    const int64_t c = node_off[s * p.B + i + 1] - o;
    for (int64_t j = lane; j < c; j += 32) {
      int64_t v = src_nodes[acc + j];
      if (s == root_ns && j == 0) v = p.seeds[i];
      node_ids[o + j] = v;
    }
    acc += c;
  }
  acc = 0;
  for (int e = 0; e < p.num_edgesets; ++e) {
    const int64_t o = edge_off[e * p.B + i];
    const int64_t c = edge_off[e * p.B + i + 1] - o;
    for (int64_t j = lane; j < c; j += 32) {
      const uint64_t k = src_edges[acc + j];
      edge_src[o + j] = static_cast<int64_t>((k >> 24) & 0xFFFFFFull);
      edge_dst[o + j] = static_cast<int64_t>(k & 0xFFFFFFull);
    }
    acc += c;
  }
}

}  // namespace
}  // namespace dgfx

// ===========================================================================
// Host side
// ===========================================================================
using namespace dgfx;

struct dgfx_sampler {
  // Plan, unrolled.
  int32_t T = 0, N2 = 1, H = 2, log2H = 1, depth = 0;
  int32_t num_nodesets = 0, num_edgesets = 0, root_ns = 0, root_has_children = 0;
  int64_t root_num_src = 0;
  int32_t with_replacement = 0, mode = 0, mask_edgeset = -1;
  uint64_t seed = 0;
  bool use_smem = true;
  // Warp sampler (0 capacity: not eligible; kernel_kind 1 forces the padded
  // sampler).
  int32_t warp_cap = 0, max_edges_per_node = 1, warp_bytes = 0;
  int32_t kernel_kind = 0;
  int32_t padded_blocks = 0;  // CTAs of the padded sampler when it serves overflow seeds
  int32_t warp_blocks = 0;    // resident CTAs of the (persistent) warp sampler
  // Large-tree warp tier (0 capacity: none): seeds that outgrow warp_cap.
  int32_t big_cap = 0, big_bytes = 0, big_blocks = 0;
  int32_t sms = 148;
  PlanNodeDev* d_pnodes = nullptr;
  // Split calls (dgfx_sampler_sample_split): the first kernel's completion
  // and this handle's last tail, so the next call on this handle waits for
  // the previous tail before it reuses the workspace.
  cudaEvent_t ev_warp = nullptr, ev_tail = nullptr;
  bool tail_pending = false;
  unsigned long long tail_capture = 0;  // capture sequence that recorded ev_tail (0: recorded eagerly)
  int threads = 256;
  size_t smem_bytes = 0;
  int32_t pbits = 1, keybits = 2;
  uint32_t ns_key_base[kMaxNodesets] = {};
  // Device tables (one allocation).
  void* d_tables = nullptr;
  EdgeDev* d_edges = nullptr;
  int4* d_tasks = nullptr;
  int32_t* d_level = nullptr;
  int32_t* d_children = nullptr;
  int32_t* d_clevel = nullptr;
  int2* d_pos = nullptr;
  unsigned long long* d_status = nullptr;
  int64_t last_B = 0;
  const int64_t* last_seeds = nullptr;
  std::vector<EdgeDev> h_edges;
  WalkPlan walk;  // for random-walk negative sampling
};

const dgfx::WalkPlan* dgfx_sampler_walk_plan(const dgfx_sampler* s) { return s == nullptr ? nullptr : &s->walk; }

namespace {

// Host-side reads of the status words after a split call: `stream` waits
// for the call's tail first (eagerly recorded tails only; a tail recorded
// in a captured graph is ordered by that graph's replays on their stream).
int wait_tail(dgfx_sampler* s, cudaStream_t stream) {
  if (s->tail_pending && s->tail_capture == 0) DGFX_CUDA_TRY(cudaStreamWaitEvent(stream, s->ev_tail, 0));
  s->tail_pending = false;
  return DGFX_OK;
}

int pow2_at_least(int64_t x) {
  int64_t p = 1;
  while (p < x) p <<= 1;
  return static_cast<int>(p);
}

struct SampleBufs {
  int32_t* scratch_nodes;
  uint64_t* scratch_edges;
  int32_t* node_cnt;
  int32_t* edge_cnt;
  char* global_work;
  unsigned int* overflow_count;
  int32_t* overflow_list;
  unsigned int* mid_count;
  int32_t* mid_list;
};

void carve_sample(Arena& a, const dgfx_sampler* s, int64_t B, SampleBufs* b) {
  b->scratch_nodes = a.take<int32_t>(static_cast<size_t>(B * s->T));
  b->scratch_edges = a.take<uint64_t>(static_cast<size_t>(B * s->T));
  b->node_cnt = a.take<int32_t>(static_cast<size_t>(B * s->num_nodesets));
  b->edge_cnt = a.take<int32_t>(static_cast<size_t>(B * s->num_edgesets));
  b->global_work = s->use_smem ? nullptr : a.take<char>(static_cast<size_t>(B) * work_bytes(s->T, s->H));
  b->overflow_count = a.take<unsigned int>(2);  // [0] overflowed seeds, [1] next seed of the warp sampler
  b->overflow_list = a.take<int32_t>(static_cast<size_t>(std::max<int64_t>(B, 1)));
  b->mid_count = a.take<unsigned int>(2);  // [0] seeds listed for the large-tree tier, [1] next of them
  b->mid_list = a.take<int32_t>(static_cast<size_t>(std::max<int64_t>(B, 1)));
}

size_t sample_ws_bytes(const dgfx_sampler* s, int64_t B) {
  Arena a(nullptr, 0);
  SampleBufs b;
  carve_sample(a, s, B, &b);
  const int64_t n = std::max<int64_t>(B * s->num_nodesets, B * s->num_edgesets) + 1;
  return a.used + scan_workspace_bytes(n) + 1024;
}

}  // namespace

extern "C" int dgfx_sampler_create(int32_t num_plan_nodes, const int32_t* node_nodeset,
                                   const int32_t* node_first_edge, const int32_t* node_num_edges,
                                   int32_t num_plan_edges, const int32_t* edge_edgeset,
                                   const int32_t* edge_reversed, const int32_t* edge_hop_width,
                                   const int32_t* edge_child, int32_t with_replacement, int32_t num_nodesets,
                                   const int64_t* num_nodes, int32_t num_edgesets, const dgfx_csr_view* forward,
                                   const dgfx_csr_view* backward, int32_t mode, int32_t edgeset_to_mask,
                                   uint64_t seed, dgfx_sampler** out) {
  if (out == nullptr) return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_sampler_create: out is null");
  *out = nullptr;
  if (num_plan_nodes < 1 || num_plan_edges < 0 || num_nodesets < 1 || num_edgesets < 0) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_sampler_create: empty plan or schema");
  }
  if (num_nodesets > kMaxNodesets || num_edgesets > kMaxEdgesets) {
    return fail(DGFX_ERR_UNSUPPORTED, "dgfx_sampler_create: at most 64 nodesets and 256 edgesets");
  }
  if (mode < DGFX_MODE_RANDOM || mode > DGFX_MODE_MOST_RECENT) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_sampler_create: unknown mode");
  }
  for (int32_t i = 0; i < num_plan_nodes; ++i) {
    if (node_nodeset[i] < 0 || node_nodeset[i] >= num_nodesets || node_num_edges[i] < 0 ||
        node_first_edge[i] < 0 || node_first_edge[i] + node_num_edges[i] > num_plan_edges) {
      return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_sampler_create: malformed plan node " + std::to_string(i));
    }
  }
  for (int32_t j = 0; j < num_plan_edges; ++j) {
    if (edge_edgeset[j] < 0 || edge_edgeset[j] >= num_edgesets || edge_child[j] <= 0 ||
        edge_child[j] >= num_plan_nodes || edge_hop_width[j] < 0) {
      return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_sampler_create: malformed plan edge " + std::to_string(j));
    }
    const dgfx_csr_view& v = edge_reversed[j] ? backward[edge_edgeset[j]] : forward[edge_edgeset[j]];
    if (v.rowptr == nullptr) return fail(DGFX_ERR_INVALID_ARGUMENT, "Check failed edges.has_value()");
  }
  auto s = std::make_unique<dgfx_sampler>();
  s->num_nodesets = num_nodesets;
  s->num_edgesets = num_edgesets;
  s->with_replacement = with_replacement != 0;
  s->mode = mode;
  s->mask_edgeset = edgeset_to_mask;
  s->seed = seed;
  s->root_ns = node_nodeset[0];

  // Slots per plan edge: hop_width capped by the largest row of the index it
  // walks (no row can yield more), which keeps wide fanouts compact.
  std::vector<int32_t> slots(num_plan_edges);
  {
    std::map<const int64_t*, int64_t> max_deg;
    unsigned long long* d_max = nullptr;
    for (int j = 0; j < num_plan_edges; ++j) {
      const dgfx_csr_view& v = edge_reversed[j] ? backward[edge_edgeset[j]] : forward[edge_edgeset[j]];
      auto it = max_deg.find(v.rowptr);
      if (it == max_deg.end()) {
        if (d_max == nullptr) DGFX_CUDA_TRY(cudaMalloc(&d_max, sizeof(unsigned long long)));
        DGFX_CUDA_TRY(cudaMemset(d_max, 0, sizeof(unsigned long long)));
        if (v.num_src > 0) {
          const int64_t blocks = std::min<int64_t>(ceil_div(v.num_src, 256), 148 * 16);
          max_degree_kernel<<<static_cast<unsigned>(blocks), 256>>>(v.rowptr, v.num_src, d_max);
          DGFX_CUDA_TRY(cudaGetLastError());
        }
        unsigned long long m = 0;
        DGFX_CUDA_TRY(cudaMemcpy(&m, d_max, sizeof(m), cudaMemcpyDeviceToHost));
        it = max_deg.emplace(v.rowptr, static_cast<int64_t>(m)).first;
      }
      slots[j] = static_cast<int32_t>(std::min<int64_t>(edge_hop_width[j], it->second));
    }
    if (d_max != nullptr) cudaFree(d_max);
  }

  // Padded subtree sizes Z(p): memoised recursion with a cycle guard.
  std::vector<int64_t> Z(num_plan_nodes, -1);
  std::vector<int> state(num_plan_nodes, 0);
  std::function<int64_t(int)> size_of = [&](int pn) -> int64_t {
    if (Z[pn] >= 0) return Z[pn];
    if (state[pn] == 1) return -1;
    state[pn] = 1;
    int64_t z = 1;
    for (int c = 0; c < node_num_edges[pn]; ++c) {
      const int j = node_first_edge[pn] + c;
      const int64_t zc = size_of(edge_child[j]);
      if (zc < 0) return -1;
      z += static_cast<int64_t>(slots[j]) * zc;
      if (z > kMaxPositions) return -1;
    }
    state[pn] = 2;
    return Z[pn] = z;
  };
  const int64_t T = size_of(0);
  if (T < 0) {
    return fail(DGFX_ERR_UNSUPPORTED, "dgfx_sampler_create: sampling plan expands to more than 2^24 tree positions "
                                      "per seed (or is cyclic)");
  }
  s->T = static_cast<int32_t>(T);
  s->N2 = pow2_at_least(std::max<int64_t>(T, 2));
  s->H = pow2_at_least(2 * T);
  s->log2H = 0;
  while ((1 << s->log2H) < s->H) ++s->log2H;
  s->use_smem = T <= kMaxSmemPositions;

  // Pre-order positions and expansion tasks by depth.
  std::vector<int2> pos(static_cast<size_t>(T));
  std::vector<std::vector<int4>> tasks_by_depth;
  std::function<void(int, int64_t, int64_t, int, int)> place = [&](int pn, int64_t q, int64_t parent, int pedge,
                                                                   int depth) {
    pos[q] = make_int2(static_cast<int>(parent), (pedge < 0 ? 0 : pedge << 8) | node_nodeset[pn]);
    int64_t off = q + 1;
    for (int c = 0; c < node_num_edges[pn]; ++c) {
      const int j = node_first_edge[pn] + c;
      const int64_t zc = Z[edge_child[j]];
      if (static_cast<int>(tasks_by_depth.size()) <= depth) tasks_by_depth.resize(depth + 1);
      tasks_by_depth[depth].push_back(make_int4(static_cast<int>(q), j, static_cast<int>(off), 0));
      for (int k = 0; k < slots[j]; ++k) place(edge_child[j], off + k * zc, q, j, depth + 1);
      off += static_cast<int64_t>(slots[j]) * zc;
    }
  };
  place(0, 0, -1, -1, 0);
  if (num_plan_edges >= (1 << 23)) return fail(DGFX_ERR_UNSUPPORTED, "dgfx_sampler_create: too many plan edges");
  std::vector<int4> tasks;
  std::vector<int32_t> level{0};
  std::vector<int32_t> children;
  std::vector<int32_t> clevel{0};
  for (auto& v : tasks_by_depth) {
    tasks.insert(tasks.end(), v.begin(), v.end());
    level.push_back(static_cast<int32_t>(tasks.size()));
    for (const int4& t : v) {
      const int32_t zc = static_cast<int32_t>(Z[edge_child[t.y]]);
      for (int k = 0; k < slots[t.y]; ++k) children.push_back(t.z + k * zc);
    }
    clevel.push_back(static_cast<int32_t>(children.size()));
  }
  s->depth = static_cast<int32_t>(tasks_by_depth.size());
  s->root_has_children = node_num_edges[0] > 0;
  if (s->root_has_children) {
    const int j = node_first_edge[0];
    const dgfx_csr_view& v = edge_reversed[j] ? backward[edge_edgeset[j]] : forward[edge_edgeset[j]];
    s->root_num_src = v.num_src;
  }
  s->h_edges.resize(num_plan_edges);
  for (int j = 0; j < num_plan_edges; ++j) {
    const dgfx_csr_view& v = edge_reversed[j] ? backward[edge_edgeset[j]] : forward[edge_edgeset[j]];
    EdgeDev& E = s->h_edges[j];
    E.rowptr = v.rowptr;
    E.col = v.col;
    E.ts = v.ts;
    E.edge_pos = (edge_edgeset[j] == edgeset_to_mask) ? v.edge_pos : nullptr;
    E.num_edges = v.num_edges;
    E.k = slots[j];
    E.stride = static_cast<int32_t>(Z[edge_child[j]]);
    E.edgeset = edge_edgeset[j];
    E.reversed = edge_reversed[j] != 0;
    E.child = edge_child[j];
  }
  // Warp sampler tables: per plan node its edges, node set and incoming
  // edge; per plan edge the first child slot relative to the parent.
  std::vector<PlanNodeDev> pnodes(num_plan_nodes);
  for (int pn = 0; pn < num_plan_nodes; ++pn) {
    pnodes[pn] = PlanNodeDev{node_first_edge[pn], node_num_edges[pn], node_nodeset[pn], -1};
    int64_t off = 1;
    for (int c = 0; c < node_num_edges[pn]; ++c) {
      const int j = node_first_edge[pn] + c;
      s->h_edges[j].rel_off = static_cast<int32_t>(off);
      off += static_cast<int64_t>(slots[j]) * Z[edge_child[j]];
      s->max_edges_per_node = std::max(s->max_edges_per_node, node_num_edges[pn]);
    }
  }
  for (int j = 0; j < num_plan_edges; ++j) pnodes[edge_child[j]].in_edge = j;
  // Dedup keys: node ids of all node sets laid end to end in 32 bits.
  {
    uint64_t acc = 0;
    for (int i = 0; i < num_nodesets; ++i) {
      s->ns_key_base[i] = static_cast<uint32_t>(acc);
      acc += static_cast<uint64_t>(num_nodes[i] < 0 ? 0 : num_nodes[i]);
    }
    if (acc >= 0xFFFFFFFFull) {
      return fail(DGFX_ERR_UNSUPPORTED, "dgfx_sampler_create: more than 2^32 - 2 nodes over all node sets");
    }
  }
  s->pbits = std::max(1, bit_length(static_cast<uint64_t>(T - 1)));
  s->keybits = bit_length(static_cast<uint64_t>(num_edgesets)) + 2 * s->pbits;

  // One device allocation for all tables.
  const size_t b_edges = align_up(sizeof(EdgeDev) * std::max<size_t>(1, s->h_edges.size()), 256);
  const size_t b_tasks = align_up(sizeof(int4) * std::max<size_t>(1, tasks.size()), 256);
  const size_t b_level = align_up(sizeof(int32_t) * level.size(), 256);
  const size_t b_pos = align_up(sizeof(int2) * pos.size(), 256);
  const size_t b_children = align_up(sizeof(int32_t) * std::max<size_t>(1, children.size()), 256);
  const size_t b_clevel = align_up(sizeof(int32_t) * clevel.size(), 256);
  const size_t b_status = 256;
  const size_t b_pnodes = align_up(sizeof(PlanNodeDev) * pnodes.size(), 256);
  char* d = nullptr;
  DGFX_CUDA_TRY(cudaMalloc(&d, b_edges + b_tasks + b_level + b_pos + b_children + b_clevel + b_status + b_pnodes));
  s->d_pnodes = reinterpret_cast<PlanNodeDev*>(d + b_edges + b_tasks + b_level + b_pos + b_children + b_clevel +
                                               b_status);
  DGFX_CUDA_TRY(cudaMemcpy(s->d_pnodes, pnodes.data(), sizeof(PlanNodeDev) * pnodes.size(), cudaMemcpyHostToDevice));
  s->d_tables = d;
  s->d_edges = reinterpret_cast<EdgeDev*>(d);
  s->d_tasks = reinterpret_cast<int4*>(d + b_edges);
  s->d_level = reinterpret_cast<int32_t*>(d + b_edges + b_tasks);
  s->d_pos = reinterpret_cast<int2*>(d + b_edges + b_tasks + b_level);
  s->d_children = reinterpret_cast<int32_t*>(d + b_edges + b_tasks + b_level + b_pos);
  s->d_clevel = reinterpret_cast<int32_t*>(d + b_edges + b_tasks + b_level + b_pos + b_children);
  s->d_status =
      reinterpret_cast<unsigned long long*>(d + b_edges + b_tasks + b_level + b_pos + b_children + b_clevel);
  if (!s->h_edges.empty()) {
    DGFX_CUDA_TRY(cudaMemcpy(s->d_edges, s->h_edges.data(), sizeof(EdgeDev) * s->h_edges.size(), cudaMemcpyHostToDevice));
  }
  if (!tasks.empty()) DGFX_CUDA_TRY(cudaMemcpy(s->d_tasks, tasks.data(), sizeof(int4) * tasks.size(), cudaMemcpyHostToDevice));
  DGFX_CUDA_TRY(cudaMemcpy(s->d_level, level.data(), sizeof(int32_t) * level.size(), cudaMemcpyHostToDevice));
  DGFX_CUDA_TRY(cudaMemcpy(s->d_pos, pos.data(), sizeof(int2) * pos.size(), cudaMemcpyHostToDevice));
  if (!children.empty()) {
    DGFX_CUDA_TRY(cudaMemcpy(s->d_children, children.data(), sizeof(int32_t) * children.size(), cudaMemcpyHostToDevice));
  }
  DGFX_CUDA_TRY(cudaMemcpy(s->d_clevel, clevel.data(), sizeof(int32_t) * clevel.size(), cudaMemcpyHostToDevice));
  // Status: first bad seed, ts missing, table overflow, 3 stats, device call
  // index, seeds finished by the warp sampler, seeds it handed to the padded
  // sampler.
  const unsigned long long init[9] = {~0ull, 0ull, 0ull, 0ull, 0ull, 0ull, 0ull, 0ull, 0ull};
  DGFX_CUDA_TRY(cudaMemcpy(s->d_status, init, sizeof(init), cudaMemcpyHostToDevice));

  // The plan as random walks see it (plan nodes, plan edges with their CSR,
  // forward indices and endpoints per edge set).
  {
    WalkPlan& w = s->walk;
    w.num_nodesets = num_nodesets;
    w.num_edgesets = num_edgesets;
    w.seed = seed;
    w.node_nodeset.assign(node_nodeset, node_nodeset + num_plan_nodes);
    w.node_first_edge.assign(node_first_edge, node_first_edge + num_plan_nodes);
    w.node_num_edges.assign(node_num_edges, node_num_edges + num_plan_nodes);
    w.edge_edgeset.assign(edge_edgeset, edge_edgeset + num_plan_edges);
    w.edge_reversed.assign(edge_reversed, edge_reversed + num_plan_edges);
    w.edge_child.assign(edge_child, edge_child + num_plan_edges);
    w.num_nodes.assign(num_nodes, num_nodes + num_nodesets);
    w.forward.assign(forward, forward + num_edgesets);
    w.es_src.assign(num_edgesets, -1);
    w.es_dst.assign(num_edgesets, -1);
    std::vector<WalkNode> hn(num_plan_nodes);
    std::vector<WalkEdge> he(std::max(1, num_plan_edges));
    for (int i = 0; i < num_plan_nodes; ++i) {
      hn[i] = WalkNode{node_nodeset[i], node_first_edge[i], node_num_edges[i], 0};
      for (int c = 0; c < node_num_edges[i]; ++c) {
        const int j = node_first_edge[i] + c;
        const int here = node_nodeset[i], there = node_nodeset[edge_child[j]];
        w.es_src[edge_edgeset[j]] = edge_reversed[j] ? there : here;
        w.es_dst[edge_edgeset[j]] = edge_reversed[j] ? here : there;
      }
    }
    for (int j = 0; j < num_plan_edges; ++j) {
      const dgfx_csr_view& v = edge_reversed[j] ? backward[edge_edgeset[j]] : forward[edge_edgeset[j]];
      he[j] = WalkEdge{v.rowptr, v.col, edge_child[j], node_nodeset[edge_child[j]]};
    }
    const size_t b_nodes = align_up(sizeof(WalkNode) * hn.size(), 256);
    char* dw = nullptr;
    DGFX_CUDA_TRY(cudaMalloc(&dw, b_nodes + sizeof(WalkEdge) * he.size()));
    w.d_nodes = reinterpret_cast<WalkNode*>(dw);
    w.d_edges = reinterpret_cast<WalkEdge*>(dw + b_nodes);
    DGFX_CUDA_TRY(cudaMemcpy(w.d_nodes, hn.data(), sizeof(WalkNode) * hn.size(), cudaMemcpyHostToDevice));
    DGFX_CUDA_TRY(cudaMemcpy(w.d_edges, he.data(), sizeof(WalkEdge) * he.size(), cudaMemcpyHostToDevice));
  }

  // Threads per CTA: about one per eight tree positions, 32..256.
  s->threads = std::min(256, std::max(32, s->N2 / 8));
  s->smem_bytes = counter_bytes(s->threads) + (s->use_smem ? work_bytes(s->T, s->H) : 0);
  if (s->smem_bytes > 48 * 1024) {
    DGFX_CUDA_TRY(cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(s->smem_bytes)));
  }
  // Warp sampler: capacity = the tree size rounded up to a power of two,
  // at most kWarpCapMax entries (larger trees go to the padded sampler when
  // they outgrow it). Plan node ids and parent entries are packed in 8 and
  // 24 bits.
  if (num_plan_nodes <= 256 && s->depth <= kMaxWarpDepth) {
    int cap = 32;  // 32, 64 or 128 entries: 1, 2 or 4 per lane
    while (cap < T && cap < kWarpCapMax) cap <<= 1;
    const int bytes = warp_region_bytes(cap, num_nodesets, num_edgesets, s->depth);
    if (bytes * kWarpsPerCta <= 200 * 1024) {
      s->warp_cap = cap;
      s->warp_bytes = bytes;
      if (bytes * kWarpsPerCta > 48 * 1024) {
        DGFX_CUDA_TRY(cudaFuncSetAttribute(reinterpret_cast<const void*>(warp_kernel_for(cap)),
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, bytes * kWarpsPerCta));
      }
    }
    // Large-tree tier: the tree size rounded up to a power of two, at most
    // kLargeCapMax entries (trees beyond it go to the padded sampler).
    if (s->warp_cap > 0 && T > s->warp_cap) {
      const int big = std::min(pow2_at_least(T), kLargeCapMax);
      const int bb = cta_region_bytes(big, num_nodesets, num_edgesets, s->depth);
      if (big > s->warp_cap && bb <= 200 * 1024) {
        s->big_cap = big;
        s->big_bytes = bb;
        if (bb > 48 * 1024) {
          DGFX_CUDA_TRY(cudaFuncSetAttribute(reinterpret_cast<const void*>(large_tree_kernel),
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, bb));
        }
      }
    }
  }
  {
    int dev = 0, sms = 148, per_sm = 1;
    DGFX_CUDA_TRY(cudaGetDevice(&dev));
    DGFX_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    DGFX_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, sample_kernel, s->threads, s->smem_bytes));
    s->padded_blocks = std::max(1, sms * std::max(1, per_sm));
    s->sms = sms;
    if (s->warp_cap > 0) {
      int wper = 1;
      DGFX_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&wper, reinterpret_cast<const void*>(warp_kernel_for(s->warp_cap)),
                                                                 kWarpsPerCta * 32,
                                                                 static_cast<size_t>(s->warp_bytes) * kWarpsPerCta));
      s->warp_blocks = std::max(1, sms * std::max(1, wper));
    }
    if (s->big_cap > 0) {
      int bper = 1;
      DGFX_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&bper, reinterpret_cast<const void*>(large_tree_kernel),
                                                                 kCtaWarps * 32, static_cast<size_t>(s->big_bytes)));
      s->big_blocks = std::max(1, sms * std::max(1, bper));
    }
  }
  *out = s.release();
  return DGFX_OK;
}

extern "C" void dgfx_sampler_destroy(dgfx_sampler* s) {
  if (s == nullptr) return;
  if (s->ev_warp != nullptr) cudaEventDestroy(s->ev_warp);
  if (s->ev_tail != nullptr) cudaEventDestroy(s->ev_tail);
  if (s->d_tables != nullptr) cudaFree(s->d_tables);
  if (s->walk.d_nodes != nullptr) cudaFree(s->walk.d_nodes);
  delete s;
}

extern "C" int dgfx_sampler_set_kernel(dgfx_sampler* s, int32_t kind) {
  if (s == nullptr || kind < 0 || kind > 2) return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_sampler_set_kernel: bad arguments");
  s->kernel_kind = kind;
  return DGFX_OK;
}

extern "C" int dgfx_sampler_kernel_info(const dgfx_sampler* s, int32_t* warp_capacity, int32_t* large_capacity) {
  if (s == nullptr || warp_capacity == nullptr) return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_sampler_kernel_info: null");
  *warp_capacity = s->kernel_kind != 1 ? s->warp_cap : 0;
  if (large_capacity != nullptr) *large_capacity = s->kernel_kind == 0 ? s->big_cap : 0;
  return DGFX_OK;
}

extern "C" int dgfx_sampler_kernel_stats(dgfx_sampler* s, dgfx_stream stream_, int64_t* out2) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (s == nullptr || out2 == nullptr) return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_sampler_kernel_stats: null argument");
  unsigned long long st[2];
  DGFX_TRY(wait_tail(s, stream));
  DGFX_CUDA_TRY(cudaMemcpyAsync(st, s->d_status + 7, sizeof(st), cudaMemcpyDeviceToHost, stream));
  DGFX_CUDA_TRY(cudaStreamSynchronize(stream));
  out2[0] = static_cast<int64_t>(st[0]);
  out2[1] = static_cast<int64_t>(st[1]);
  return DGFX_OK;
}

extern "C" int dgfx_sampler_tree_size(const dgfx_sampler* s, int64_t* positions) {
  if (s == nullptr || positions == nullptr) return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_sampler_tree_size: null");
  *positions = s->T;
  return DGFX_OK;
}

extern "C" int dgfx_sampler_workspace_size(const dgfx_sampler* s, int64_t num_seeds, size_t* bytes) {
  if (s == nullptr || bytes == nullptr || num_seeds < 0) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_sampler_workspace_size: bad arguments");
  }
  *bytes = sample_ws_bytes(s, num_seeds);
  return DGFX_OK;
}

extern "C" int dgfx_sampler_output_capacity(const dgfx_sampler* s, int64_t num_seeds, int64_t* max_nodes,
                                            int64_t* max_edges) {
  if (s == nullptr || max_nodes == nullptr || max_edges == nullptr || num_seeds < 0) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_sampler_output_capacity: bad arguments");
  }
  *max_nodes = num_seeds * s->T;
  *max_edges = num_seeds * std::max(0, s->T - 1);
  return DGFX_OK;
}

namespace {
// One sampling call. Everything runs on `stream` when tail == stream. With a
// separate tail stream, the first sampling kernel runs on `stream` and the
// rest (the padded kernel for large trees, the offset scans, the
// compaction) on `tail` after it; the batch is complete in `tail` order.
int sample_impl(dgfx_sampler* s, const int64_t* d_seeds, const int64_t* d_seed_ts, const int64_t* d_masked_edges,
                int64_t B, uint64_t call_index, const dgfx_sample_out* out, void* d_workspace, size_t workspace_bytes,
                cudaStream_t stream, cudaStream_t tail) {
  const bool split = tail != stream;
  if (s == nullptr || out == nullptr || B < 0) return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_sampler_sample: bad arguments");
  if (B > 0 && d_seeds == nullptr) return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_sampler_sample: null seeds");
  if (B >= (int64_t(1) << 31)) return fail(DGFX_ERR_UNSUPPORTED, "dgfx_sampler_sample: more than 2^31 - 1 seeds");
  if (d_masked_edges != nullptr && s->mask_edgeset < 0) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "masked_edge_idxs provided but no edgeset to mask configured.");
  }
  if (d_workspace == nullptr || workspace_bytes < sample_ws_bytes(s, B)) {
    return fail(DGFX_ERR_WORKSPACE, "dgfx_sampler_sample: workspace too small");
  }
  if (split) {
    if (s->ev_warp == nullptr) DGFX_CUDA_TRY(cudaEventCreateWithFlags(&s->ev_warp, cudaEventDisableTiming));
    if (s->ev_tail == nullptr) DGFX_CUDA_TRY(cudaEventCreateWithFlags(&s->ev_tail, cudaEventDisableTiming));
  }
  cudaStreamCaptureStatus cst = cudaStreamCaptureStatusNone;
  unsigned long long cid = 0;
  DGFX_CUDA_TRY(cudaStreamGetCaptureInfo(stream, &cst, &cid));
  const bool capturing = cst == cudaStreamCaptureStatusActive;
  if (s->tail_pending) {  // the last split call's tail must end before the workspace is reused
    if (!capturing && s->tail_capture == 0) {
      DGFX_CUDA_TRY(cudaStreamWaitEvent(stream, s->ev_tail, 0));
    } else if (capturing && s->tail_capture == cid) {
      DGFX_CUDA_TRY(cudaStreamWaitEvent(stream, s->ev_tail, 0));  // recorded earlier in this capture
    } else if (capturing) {
      return fail(DGFX_ERR_FAILED_PRECONDITION,
                  "dgfx_sampler_sample: a split call's tail is pending from outside this stream capture; "
                  "call dgfx_sampler_check before capturing");
    }
    // else: recorded in a capture that has ended; its graph's replays are ordered on their stream.
    s->tail_pending = false;
  }
  s->last_B = B;
  s->last_seeds = d_seeds;
  Arena arena(d_workspace, workspace_bytes);
  SampleBufs b;
  carve_sample(arena, s, B, &b);
  // Status words and the tiers' seed counters in one launch (kernels only,
  // so the call can be captured in a CUDA graph).
  reset_kernel<<<1, 32, 0, stream>>>(s->d_status, b.overflow_count, b.mid_count);
  DGFX_CUDA_TRY(cudaGetLastError());
  if (B == 0) {
    if (split) {
      DGFX_CUDA_TRY(cudaEventRecord(s->ev_warp, stream));
      DGFX_CUDA_TRY(cudaStreamWaitEvent(tail, s->ev_warp, 0));
    }
    DGFX_CUDA_TRY(cudaMemsetAsync(out->node_offsets, 0, sizeof(int64_t), tail));
    DGFX_CUDA_TRY(cudaMemsetAsync(out->edge_offsets, 0, sizeof(int64_t), tail));
    if (split) {
      DGFX_CUDA_TRY(cudaEventRecord(s->ev_tail, tail));
      s->tail_pending = true;
      s->tail_capture = capturing ? cid : 0;
    }
    return DGFX_OK;
  }
  Params p{};
  p.edges = s->d_edges;
  p.tasks = s->d_tasks;
  p.level = s->d_level;
  p.children = s->d_children;
  p.clevel = s->d_clevel;
  p.depth = s->depth;
  p.pos_info = s->d_pos;
  p.T = s->T;
  p.N2 = s->N2;
  p.H = s->H;
  p.log2H = s->log2H;
  p.num_nodesets = s->num_nodesets;
  p.num_edgesets = s->num_edgesets;
  p.root_has_children = s->root_has_children;
  p.root_num_src = s->root_num_src;
  p.with_replacement = s->with_replacement;
  p.mode = s->mode;
  p.mask_edgeset = s->mask_edgeset;
  p.seeds = d_seeds;
  p.seed_ts = d_seed_ts;
  p.masks = d_masked_edges;
  p.B = B;
  p.key0 = static_cast<uint32_t>(s->seed);
  p.key1 = static_cast<uint32_t>(s->seed >> 32);
  p.call_lo = static_cast<uint32_t>(call_index);
  p.call_hi = static_cast<uint32_t>(call_index >> 32);
  p.call_dev = call_index == ~0ull ? s->d_status + 6 : nullptr;
  p.scratch_nodes = b.scratch_nodes;
  p.scratch_edges = b.scratch_edges;
  p.node_cnt = b.node_cnt;
  p.edge_cnt = b.edge_cnt;
  p.global_work = b.global_work;
  p.work_stride = work_bytes(s->T, s->H);
  p.status = s->d_status;
  p.pbits = s->pbits;
  p.keybits = s->keybits;
  for (int i = 0; i < kMaxNodesets; ++i) p.ns_key_base[i] = s->ns_key_base[i];
  p.pnodes = s->d_pnodes;
  p.warp_cap = s->warp_cap;
  p.max_edges_per_node = s->max_edges_per_node;
  p.warp_bytes = s->warp_bytes;
  p.overflow_count = b.overflow_count;
  p.overflow_list = nullptr;
  const bool big = s->big_cap > 0 && s->kernel_kind == 0;
  p.big_cap = big ? s->big_cap : 0;
  p.big_bytes = s->big_bytes;
  p.mid_count = b.mid_count;
  p.mid_list = b.mid_list;
  const size_t smem = s->smem_bytes;
  if (s->warp_cap > 0 && s->kernel_kind != 1) {
    p.overflow_list = b.overflow_list;
    const int64_t blocks = std::min<int64_t>(ceil_div(B, kWarpsPerCta), s->warp_blocks);
    warp_kernel_for(s->warp_cap)<<<static_cast<unsigned>(blocks), kWarpsPerCta * 32,
                         static_cast<size_t>(s->warp_bytes) * kWarpsPerCta, stream>>>(p);
    DGFX_CUDA_TRY(cudaGetLastError());
    if (split) {
      DGFX_CUDA_TRY(cudaEventRecord(s->ev_warp, stream));
      DGFX_CUDA_TRY(cudaStreamWaitEvent(tail, s->ev_warp, 0));
    }
    if (big) {  // seeds whose trees outgrew warp_cap: one CTA each with big_cap entries
      const int64_t bb = std::min<int64_t>(B, s->big_blocks);
      large_tree_kernel<<<static_cast<unsigned>(bb), kCtaWarps * 32, static_cast<size_t>(s->big_bytes), tail>>>(p);
      DGFX_CUDA_TRY(cudaGetLastError());
    }
    if (s->T > (big ? s->big_cap : s->warp_cap)) {  // trees beyond every warp tier's capacity
      // Behind the large-tree tier only the rare trees of more than big_cap
      // entries remain: one CTA per SM (persistent over the list).
      const int64_t pb = std::min<int64_t>(B, big ? s->sms : s->padded_blocks);
      sample_kernel<<<static_cast<unsigned>(pb), s->threads, smem, tail>>>(p);
      DGFX_CUDA_TRY(cudaGetLastError());
    }
  } else {
    sample_kernel<<<static_cast<unsigned>(B), s->threads, smem, stream>>>(p);
    DGFX_CUDA_TRY(cudaGetLastError());
    if (split) {
      DGFX_CUDA_TRY(cudaEventRecord(s->ev_warp, stream));
      DGFX_CUDA_TRY(cudaStreamWaitEvent(tail, s->ev_warp, 0));
    }
  }
  DGFX_TRY(exclusive_scan_pair<int32_t>(b.node_cnt, out->node_offsets, B * s->num_nodesets, b.edge_cnt,
                                        out->edge_offsets, B * s->num_edgesets, arena, tail));
  const int64_t threads = 256;
  const int64_t blocks = ceil_div(B * 32, threads);
  compact_kernel<<<static_cast<unsigned>(blocks), static_cast<unsigned>(threads), 0, tail>>>(
      p, out->node_offsets, out->edge_offsets, s->root_ns, out->node_ids, out->edge_src, out->edge_dst);
  DGFX_CUDA_TRY(cudaGetLastError());
  if (split) {
    DGFX_CUDA_TRY(cudaEventRecord(s->ev_tail, tail));
    s->tail_pending = true;
    s->tail_capture = capturing ? cid : 0;
  }
  return DGFX_OK;
}
}  // namespace

extern "C" int dgfx_sampler_sample(dgfx_sampler* s, const int64_t* d_seeds, const int64_t* d_seed_ts,
                                   const int64_t* d_masked_edges, int64_t B, uint64_t call_index,
                                   const dgfx_sample_out* out, void* d_workspace, size_t workspace_bytes,
                                   dgfx_stream stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  return sample_impl(s, d_seeds, d_seed_ts, d_masked_edges, B, call_index, out, d_workspace, workspace_bytes, stream,
                     stream);
}

extern "C" int dgfx_sampler_sample_split(dgfx_sampler* s, const int64_t* d_seeds, const int64_t* d_seed_ts,
                                         const int64_t* d_masked_edges, int64_t B, uint64_t call_index,
                                         const dgfx_sample_out* out, void* d_workspace, size_t workspace_bytes,
                                         dgfx_stream stream_, dgfx_stream tail_stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  cudaStream_t tail = reinterpret_cast<cudaStream_t>(tail_stream_);
  if (tail == stream) return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_sampler_sample_split: tail stream == stream");
  return sample_impl(s, d_seeds, d_seed_ts, d_masked_edges, B, call_index, out, d_workspace, workspace_bytes, stream,
                     tail);
}

extern "C" int dgfx_sampler_check(dgfx_sampler* s, dgfx_stream stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (s == nullptr) return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_sampler_check: null sampler");
  unsigned long long st[3];
  DGFX_TRY(wait_tail(s, stream));
  DGFX_CUDA_TRY(cudaMemcpyAsync(st, s->d_status, sizeof(st), cudaMemcpyDeviceToHost, stream));
  DGFX_CUDA_TRY(cudaStreamSynchronize(stream));
  if (st[0] != ~0ull) {
    int64_t seed = 0;
    DGFX_CUDA_TRY(cudaMemcpy(&seed, s->last_seeds + st[0], sizeof(seed), cudaMemcpyDeviceToHost));
    return fail(DGFX_ERR_INVALID_ARGUMENT, "The source node idx " + std::to_string(static_cast<uint64_t>(seed)) +
                                               " is out of bounds. Should be lower than " +
                                               std::to_string(s->root_num_src));
  }
  if (st[1] != 0) {
    return fail(DGFX_ERR_FAILED_PRECONDITION,
                "Cannot use SampleRandomUniform when timestamps are available. Use "
                "SampleRandomUniformWithTimestamp instead.");
  }
  if (st[2] != 0) return fail(DGFX_ERR_INTERNAL, "sampler: dedup table overflow");
  return DGFX_OK;
}

extern "C" int dgfx_sampler_stats(dgfx_sampler* s, dgfx_stream stream_, int64_t* out3) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (s == nullptr || out3 == nullptr) return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_sampler_stats: null argument");
  unsigned long long st[6];
  DGFX_TRY(wait_tail(s, stream));
  DGFX_CUDA_TRY(cudaMemcpyAsync(st, s->d_status, sizeof(st), cudaMemcpyDeviceToHost, stream));
  DGFX_CUDA_TRY(cudaStreamSynchronize(stream));
  for (int i = 0; i < 3; ++i) out3[i] = static_cast<int64_t>(st[3 + i]);
  return DGFX_OK;
}

// ===========================================================================
// Allocation-free sampling entry point.
//
// Some callers cannot allocate device memory at the point where they sample:
// code running under a framework that owns the whole device memory pool
// (a JAX/XLA process that preallocates HBM, a serving runtime with a fixed
// arena) or a plugin invoked where allocation is forbidden. They cannot
// provide dgfx_sampler_sample's workspace, so this variant takes its scratch
// from one file-scope device array instead. The array is fixed at
// kNoAllocScratchBytes (64 MiB) and every GPU that loads this library holds
// it until the process exits. Its device address is looked up with
// cudaGetSymbolAddress once per device, on the first call made with that
// device current; make that first call before any stream capture. The
// address is kept for the life of the process, so a device reset
// (cudaDeviceReset) invalidates it: the entry point must not be called
// again after one in the same process.
// All calls share the array and it keeps the previous call's contents; the
// sampler writes every scratch word it later reads, so nothing needs
// clearing. Calls whose executions overlap on the GPU (two streams, or two
// host threads) race on the array and must be serialised by the caller.
// ===========================================================================
namespace {
constexpr size_t kNoAllocScratchBytes = size_t(64) << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};

int noalloc_scratch(void** out) {
  int dev = 0;
  DGFX_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(DGFX_ERR_UNSUPPORTED, "dgfx_sampler_sample_noalloc: device id");
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      return fail(DGFX_ERR_CUDA, std::string("dgfx_sampler_sample_noalloc: cudaGetSymbolAddress failed: ") +
                                     cudaGetErrorString(e));
    }
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return DGFX_OK;
}
}  // namespace

extern "C" int dgfx_sampler_sample_noalloc(dgfx_sampler* s, const int64_t* d_seeds, const int64_t* d_seed_ts,
                                           const int64_t* d_masked_edges, int64_t B, uint64_t call_index,
                                           const dgfx_sample_out* out, dgfx_stream stream) {
  if (s == nullptr || B < 0) return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_sampler_sample_noalloc: bad arguments");
  const size_t need = sample_ws_bytes(s, B);
  if (need > kNoAllocScratchBytes) {
    return fail(DGFX_ERR_INVALID_ARGUMENT,
                "dgfx_sampler_sample_noalloc: " + std::to_string(B) + " seeds need " + std::to_string(need) +
                    " bytes of scratch, more than the fixed " + std::to_string(kNoAllocScratchBytes) +
                    " bytes; use fewer seeds per call or dgfx_sampler_sample with a workspace");
  }
  void* scratch = nullptr;
  DGFX_TRY(noalloc_scratch(&scratch));
  return dgfx_sampler_sample(s, d_seeds, d_seed_ts, d_masked_edges, B, call_index, out, scratch,
                             kNoAllocScratchBytes, stream);
}
