// Random-walk negative sampling for link prediction (sm_100a).
//
// Semantics follow RandomWalkNegativeSamplerHelper::SampleForSeed and
// Sampler::RandomWalkNegativeSampling (dgf/src/sampling/
// in_memory_sampler_ext.cc:774-948). For each seed, num_walks walks go down
// the sampler's plan from the root: at a plan node one of its plan edges is
// chosen uniformly, then one uniform neighbour of the current node over that
// edge's index (all of the row: no timestamp cutoff, no masking); a node
// without neighbours ends the walk. Every node reached on a plan node of the
// target edge set's target node set counts one visit, except the seed itself
// when the edge set is homogeneous (the walk goes on). Visited nodes that the
// seed already links to in the target edge set (the forward index's HasEdge)
// are dropped; the most visited of the rest fill the row, most visits first;
// the remaining slots are uniform draws over the target node set, never the
// seed of a homogeneous edge set, with no other exclusion.
//
// Design. A persistent grid; one CTA owns one seed at a time. Its threads run
// the walks in parallel and count visits in an open-addressing table of
// (node << 32 | visits) words (shared memory when small, else a per-CTA slice
// of the workspace; sized for twice the most nodes the walks can reach, so it
// never fills). Then each occupied slot is filtered by HasEdge and packed into
// a (~visits << 32 | node) key, the keys are ranked by a bitonic sort
// (ascending = most visits first, ties to the smaller node id: the reference
// leaves ties in its hash map's iteration order) and the row is written.
//
// HasEdge is the reference's std::binary_search over the forward row: lower
// bound by halving, then an equality test. On a temporal index the rows are
// sorted by (timestamp, target), and the same search over the same order
// gives the same answer as the reference.
//
// Random stream: Philox4x32-10 keyed by the sampler seed with key1 xor a
// domain tag (independent of the sampling calls' stream), counter (walk,
// step, seed slot, call index). One draw per walk step: the low 64 bits pick
// the plan edge, the high 64 bits the neighbour (multiply-high reduction).
// Fallback slot j draws with counter (attempt, 2^31 | j, seed slot, call
// index). The generator differs from the reference's std::mt19937_64, so
// results agree in distribution, not bit for bit.
#include <algorithm>
#include <functional>
#include <string>
#include <vector>

#include "common.cuh"
#include "walk_plan.cuh"

namespace dgfx {
namespace {

constexpr unsigned long long kEmptySlot = ~0ull;
constexpr uint32_t kWalkDomain = 0x52574E53u;  // key1 tag of the walk stream
constexpr uint32_t kMaxFallbackDraws = 64;
constexpr int kSmemTableBytes = 96 * 1024;  // dynamic shared memory opt-in limit used here
constexpr int kMaxGlobalCtas = 148 * 8;

struct RwParams {
  const WalkNode* nodes;
  const WalkEdge* edges;
  const int64_t* fwd_rowptr;  // forward index of the target edge set
  const int32_t* fwd_col;
  int64_t fwd_num_src;
  const int64_t* seeds;
  int64_t num_seeds;
  int64_t root_num_nodes;
  int64_t num_target;
  int32_t target_ns, homogeneous, num_walks, k, max_steps;
  int32_t H, log2H;
  uint32_t key0, key1, call_lo, call_hi;
  int64_t* out;                          // [num_seeds, k]
  unsigned long long* global_tables;     // per-CTA [H + H/2] words, or null (shared memory)
  unsigned long long* status;            // [0] first bad seed slot, [1] table overflow, [2] fallback exhausted
};

__device__ __forceinline__ U4 walk_draw(const RwParams& p, uint32_t c0, uint32_t c1, uint32_t slot) {
  return philox4x32_10(U4{c0, c1, slot, p.call_lo}, p.key0 ^ p.call_hi, p.key1 ^ kWalkDomain);
}

// Adds one visit of `node`; false if the table is full.
__device__ __forceinline__ bool count_visit(unsigned long long* table, int H, int log2H, uint32_t node) {
  uint32_t s = (node * 0x9E3779B1u) >> (32 - log2H);
  const unsigned long long fresh = (static_cast<unsigned long long>(node) << 32) | 1ull;
  for (int i = 0; i < H; ++i) {
    unsigned long long w = *reinterpret_cast<volatile unsigned long long*>(&table[s]);
    if (w == kEmptySlot) {
      const unsigned long long prev = atomicCAS(&table[s], kEmptySlot, fresh);
      if (prev == kEmptySlot) return true;
      w = prev;
    }
    if (static_cast<uint32_t>(w >> 32) == node) {
      atomicAdd(&table[s], 1ull);
      return true;
    }
    s = (s + 1) & static_cast<uint32_t>(H - 1);
  }
  return false;
}

// std::binary_search(row.begin(), row.end(), target) over the forward row of
// src (AdjacencyIndex::HasEdge, in_memory_sampler.h:111-114).
__device__ __forceinline__ bool has_edge(const RwParams& p, int64_t src, int32_t target) {
  if (p.fwd_rowptr == nullptr || src < 0 || src >= p.fwd_num_src) return false;
  int64_t first = p.fwd_rowptr[src];
  const int64_t last = p.fwd_rowptr[src + 1];
  int64_t len = last - first;
  while (len > 0) {
    const int64_t half = len >> 1;
    const int64_t mid = first + half;
    if (p.fwd_col[mid] < target) {
      first = mid + 1;
      len -= half + 1;
    } else {
      len = half;
    }
  }
  return first < last && !(target < p.fwd_col[first]);
}

__global__ void __launch_bounds__(256) random_walk_negatives_kernel(RwParams p) {
  extern __shared__ unsigned long long rw_smem[];
  __shared__ int n_cand;
  const int H = p.H;
  unsigned long long* table =
      p.global_tables != nullptr ? p.global_tables + static_cast<size_t>(blockIdx.x) * (H + H / 2) : rw_smem;
  unsigned long long* cand = table + H;  // H / 2 words
  const int tid = threadIdx.x, nt = blockDim.x;
  for (int64_t slot = blockIdx.x; slot < p.num_seeds; slot += gridDim.x) {
    const int64_t seed = p.seeds[slot];
    int64_t* row = p.out + slot * p.k;
    if (seed < 0 || seed >= p.root_num_nodes) {
      if (tid == 0) atomicMin(&p.status[0], static_cast<unsigned long long>(slot));
      for (int j = tid; j < p.k; j += nt) row[j] = -1;
      continue;  // uniform across the CTA: every thread reads the same seed
    }
    for (int i = tid; i < H; i += nt) table[i] = kEmptySlot;
    if (tid == 0) n_cand = 0;
    __syncthreads();

    // Phase 1: walks (ext.cc:788-819).
    const uint32_t sl = static_cast<uint32_t>(slot);
    for (int w = tid; w < p.num_walks; w += nt) {
      int64_t cur = seed;
      int32_t pn = 0;
      for (int32_t step = 0; step < p.max_steps; ++step) {
        const WalkNode nd = p.nodes[pn];
        if (nd.num_edges <= 0) break;
        const U4 r = walk_draw(p, static_cast<uint32_t>(w), static_cast<uint32_t>(step), sl);
        const int32_t j = nd.first_edge +
                          static_cast<int32_t>(bounded64(static_cast<uint64_t>(r.y) << 32 | r.x,
                                                         static_cast<uint64_t>(nd.num_edges)));
        const WalkEdge E = p.edges[j];
        const int64_t rb = E.rowptr[cur];
        const int64_t n = E.rowptr[cur + 1] - rb;
        if (n <= 0) break;
        cur = E.col[rb + static_cast<int64_t>(bounded64(static_cast<uint64_t>(r.w) << 32 | r.z,
                                                        static_cast<uint64_t>(n)))];
        pn = E.child;
        if (E.child_nodeset == p.target_ns) {
          if (p.homogeneous && cur == seed) continue;
          if (!count_visit(table, H, p.log2H, static_cast<uint32_t>(cur))) atomicAdd(&p.status[1], 1ull);
        }
      }
    }
    __syncthreads();

    // Phase 2: drop nodes the seed already links to (ext.cc:821-834).
    for (int i = tid; i < H; i += nt) {
      const unsigned long long w = table[i];
      if (w == kEmptySlot) continue;
      const uint32_t node = static_cast<uint32_t>(w >> 32);
      const uint32_t visits = static_cast<uint32_t>(w);
      if (has_edge(p, seed, static_cast<int32_t>(node))) continue;
      const int c = atomicAdd(&n_cand, 1);
      if (c < H / 2) cand[c] = (static_cast<unsigned long long>(~visits) << 32) | node;
      else atomicAdd(&p.status[1], 1ull);
    }
    __syncthreads();

    // Phase 3: rank (ext.cc:836-853). Keys are distinct (one per node).
    const int nc = min(n_cand, H / 2);
    int P = 1;
    while (P < nc) P <<= 1;
    for (int i = nc + tid; i < P; i += nt) cand[i] = kEmptySlot;
    __syncthreads();
    for (int size = 2; size <= P; size <<= 1) {
      for (int stride = size >> 1; stride > 0; stride >>= 1) {
        for (int i = tid; i < P; i += nt) {
          const int partner = i ^ stride;
          if (partner > i) {
            const unsigned long long a = cand[i], b = cand[partner];
            const bool up = (i & size) == 0;
            if ((a > b) == up) {
              cand[i] = b;
              cand[partner] = a;
            }
          }
        }
        __syncthreads();
      }
    }

    // Phase 3 output and phase 4 fallback (ext.cc:855-870).
    const int take = min(nc, p.k);
    for (int j = tid; j < p.k; j += nt) {
      if (j < take) {
        row[j] = static_cast<int64_t>(static_cast<uint32_t>(cand[j]));
        continue;
      }
      int64_t v = -1;
      for (uint32_t a = 0; a < kMaxFallbackDraws; ++a) {
        const U4 r = walk_draw(p, a, 0x80000000u | static_cast<uint32_t>(j), sl);
        const int64_t c = static_cast<int64_t>(
            bounded64(static_cast<uint64_t>(r.y) << 32 | r.x, static_cast<uint64_t>(p.num_target)));
        if (p.homogeneous && c == seed) continue;
        v = c;
        break;
      }
      if (v < 0) atomicAdd(&p.status[2], 1ull);
      row[j] = v;
    }
    __syncthreads();  // the table and keys are reused by the next seed
  }
}

// Most nodes of the target node set one walk can count: the largest number
// of plan nodes of that set on a root-to-leaf path (the root excluded). The
// plan is a tree (the sampler rejects cyclic plans).
int64_t visits_per_walk(const WalkPlan& w, int32_t target_ns) {
  std::vector<int64_t> memo(w.node_nodeset.size(), -1);
  std::function<int64_t(int)> best = [&](int i) -> int64_t {
    if (memo[i] >= 0) return memo[i];
    int64_t b = 0;
    for (int c = 0; c < w.node_num_edges[i]; ++c) {
      const int child = w.edge_child[w.node_first_edge[i] + c];
      b = std::max(b, best(child) + (w.node_nodeset[child] == target_ns ? 1 : 0));
    }
    return memo[i] = b;
  };
  return best(0);
}

struct RwLayout {
  int H = 64, log2H = 6, threads = 64;
  bool smem = true;
  int64_t grid = 1;
  size_t status_bytes = 256, table_bytes = 0;
};

int rw_layout(const WalkPlan& w, int64_t num_seeds, int32_t target_edgeset, int32_t num_walks, RwLayout* L) {
  const int32_t tns = w.es_dst[target_edgeset];
  const int64_t per_walk = visits_per_walk(w, tns);
  const int64_t visits = static_cast<int64_t>(num_walks) * per_walk;
  if (visits >= (int64_t(1) << 31)) {
    return fail(DGFX_ERR_UNSUPPORTED, "dgfx_random_walk_negatives: num_walks * visits per walk must stay below 2^31");
  }
  const int64_t distinct = std::min<int64_t>(visits, w.num_nodes[tns]);
  int64_t H = 64;
  while (H < 2 * distinct) H <<= 1;
  if (H > (int64_t(1) << 30)) return fail(DGFX_ERR_UNSUPPORTED, "dgfx_random_walk_negatives: visit table too large");
  L->H = static_cast<int>(H);
  L->log2H = 0;
  while ((int64_t(1) << L->log2H) < H) ++L->log2H;
  int threads = 32;
  while (threads < num_walks && threads < 256) threads <<= 1;
  L->threads = threads;
  const size_t words = static_cast<size_t>(H + H / 2);
  L->smem = words * 8 <= static_cast<size_t>(kSmemTableBytes);
  int64_t grid = std::max<int64_t>(1, num_seeds);
  if (!L->smem) {
    // A slice per CTA; at most 4 GiB of tables.
    const int64_t fit = std::max<int64_t>(1, (int64_t(4) << 30) / static_cast<int64_t>(words * 8));
    grid = std::min<int64_t>({grid, int64_t(kMaxGlobalCtas), fit});
  } else {
    grid = std::min<int64_t>(grid, int64_t(148) * (2048 / threads));
  }
  L->grid = grid;
  L->table_bytes = L->smem ? 0 : static_cast<size_t>(grid) * words * 8;
  return DGFX_OK;
}

int rw_validate(const dgfx_sampler* s, const WalkPlan** wp, int32_t target_edgeset, int32_t num_walks,
                int32_t num_negatives) {
  const WalkPlan* w = dgfx_sampler_walk_plan(s);
  if (w == nullptr) return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_random_walk_negatives: null sampler");
  if (target_edgeset < 0 || target_edgeset >= w->num_edgesets) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "Invalid target_edgeset_idx");
  }
  if (w->forward[target_edgeset].rowptr == nullptr || w->es_dst[target_edgeset] < 0) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "Edgeset " + std::to_string(target_edgeset) +
                                               " does not have a forward index. Ensure it is traversed forward in "
                                               "the SamplingPlan.");
  }
  if (num_walks < 0 || num_negatives < 0) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_random_walk_negatives: negative num_walks or num_negatives_per_seed");
  }
  *wp = w;
  return DGFX_OK;
}

}  // namespace
}  // namespace dgfx

using namespace dgfx;

extern "C" int dgfx_random_walk_negatives_workspace_size(const dgfx_sampler* s, int64_t num_seeds,
                                                         int32_t target_edgeset, int32_t num_walks,
                                                         int32_t num_negatives_per_seed, size_t* bytes) {
  if (bytes == nullptr || num_seeds < 0) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_random_walk_negatives_workspace_size: bad arguments");
  }
  const WalkPlan* w = nullptr;
  DGFX_TRY(rw_validate(s, &w, target_edgeset, num_walks, num_negatives_per_seed));
  RwLayout L;
  DGFX_TRY(rw_layout(*w, num_seeds, target_edgeset, num_walks, &L));
  *bytes = L.status_bytes + L.table_bytes;
  return DGFX_OK;
}

extern "C" int dgfx_random_walk_negatives(dgfx_sampler* s, const int64_t* d_seeds, int64_t num_seeds,
                                          int32_t target_edgeset, int32_t num_walks, int32_t num_negatives_per_seed,
                                          uint64_t call_index, int64_t* d_out, void* d_workspace,
                                          size_t workspace_bytes, dgfx_stream stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (num_seeds < 0 || (num_seeds > 0 && d_seeds == nullptr) ||
      (num_seeds > 0 && num_negatives_per_seed > 0 && d_out == nullptr) || d_workspace == nullptr) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_random_walk_negatives: bad arguments");
  }
  if (num_seeds >= (int64_t(1) << 31)) {
    return fail(DGFX_ERR_UNSUPPORTED, "dgfx_random_walk_negatives: more than 2^31 - 1 seeds");
  }
  const WalkPlan* w = nullptr;
  DGFX_TRY(rw_validate(s, &w, target_edgeset, num_walks, num_negatives_per_seed));
  RwLayout L;
  DGFX_TRY(rw_layout(*w, num_seeds, target_edgeset, num_walks, &L));
  if (workspace_bytes < L.status_bytes + L.table_bytes) {
    return fail(DGFX_ERR_WORKSPACE, "dgfx_random_walk_negatives: workspace too small");
  }
  const int32_t tns = w->es_dst[target_edgeset];
  const int64_t num_target = w->num_nodes[tns];
  const bool homogeneous = w->es_src[target_edgeset] == tns;
  // Slots left after the ranked candidates are filled by draws over the
  // target node set; with no node to draw (or only the seed itself) the
  // reference's fallback loop never ends.
  if (num_seeds > 0 && num_negatives_per_seed > 0 && (num_target < 1 || (homogeneous && num_target < 2))) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_random_walk_negatives: the target node set has no node to draw "
                                           "for the fallback slots");
  }
  auto* status = reinterpret_cast<unsigned long long*>(d_workspace);
  DGFX_CUDA_TRY(cudaMemsetAsync(status, 0xFF, 8, stream));
  DGFX_CUDA_TRY(cudaMemsetAsync(status + 1, 0, 16, stream));
  if (num_seeds == 0 || num_negatives_per_seed == 0) return DGFX_OK;
  RwParams p{};
  p.nodes = w->d_nodes;
  p.edges = w->d_edges;
  const dgfx_csr_view& f = w->forward[target_edgeset];
  p.fwd_rowptr = f.rowptr;
  p.fwd_col = f.col;
  p.fwd_num_src = f.num_src;
  p.seeds = d_seeds;
  p.num_seeds = num_seeds;
  p.root_num_nodes = w->num_nodes[w->node_nodeset[0]];
  p.num_target = num_target;
  p.target_ns = tns;
  p.homogeneous = homogeneous ? 1 : 0;
  p.num_walks = num_walks;
  p.k = num_negatives_per_seed;
  p.max_steps = static_cast<int32_t>(w->node_nodeset.size());
  p.H = L.H;
  p.log2H = L.log2H;
  p.key0 = static_cast<uint32_t>(w->seed);
  p.key1 = static_cast<uint32_t>(w->seed >> 32);
  p.call_lo = static_cast<uint32_t>(call_index);
  p.call_hi = static_cast<uint32_t>(call_index >> 32);
  p.out = d_out;
  p.global_tables = L.smem ? nullptr
                           : reinterpret_cast<unsigned long long*>(static_cast<char*>(d_workspace) + L.status_bytes);
  p.status = status;
  const size_t smem = L.smem ? static_cast<size_t>(L.H + L.H / 2) * 8 : 0;
  if (smem > 0) {
    DGFX_CUDA_TRY(cudaFuncSetAttribute(random_walk_negatives_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       kSmemTableBytes));
  }
  random_walk_negatives_kernel<<<static_cast<unsigned>(L.grid), L.threads, smem, stream>>>(p);
  DGFX_CUDA_TRY(cudaGetLastError());
  return DGFX_OK;
}

extern "C" int dgfx_random_walk_negatives_check(const void* d_workspace, dgfx_stream stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (d_workspace == nullptr) return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_random_walk_negatives_check: null workspace");
  unsigned long long st[3];
  DGFX_CUDA_TRY(cudaMemcpyAsync(st, d_workspace, sizeof(st), cudaMemcpyDeviceToHost, stream));
  DGFX_CUDA_TRY(cudaStreamSynchronize(stream));
  if (st[0] != ~0ull) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_random_walk_negatives: seed at position " + std::to_string(st[0]) +
                                               " is not a node of the plan's root node set");
  }
  if (st[1] != 0) return fail(DGFX_ERR_INTERNAL, "dgfx_random_walk_negatives: visit table overflow");
  if (st[2] != 0) return fail(DGFX_ERR_INTERNAL, "dgfx_random_walk_negatives: fallback draws exhausted");
  return DGFX_OK;
}
