// Subgraph extraction as the union of per-seed samples.
//
// Restates the numbering and edge set of SubGraphExtractor
// (dgf/src/sampling/in_memory_sampler_ext.cc:600-772) on a merged batch of
// per-seed samples (one sample per seed, the sampler's output layout):
//   * the seeds are the first nodes of the root node set, ids 0..B-1 in seed
//     order (ExtractSubGraph registers every seed first, duplicates included;
//     a repeated seed node maps to its last seed id);
//   * every other node gets the next id of its node set in order of its
//     first occurrence, i.e. of (seed index, local id in that seed's sample):
//     the reference's depth-first traversal visits seed after seed, and a
//     sample's local ids are its first-discovery order;
//   * edges are every sample's edges mapped to these ids, deduplicated and
//     sorted by (source, target) per edge set (the btree_set iteration).
// With deterministic expansion (oldest-first, or hop_width >= degree) this is
// exactly the reference's result: a (node, plan step) pair it skips because
// it was expanded before yields, when expanded again, only nodes and edges
// already present.
//
// Device steps: occurrence keys (node set, node) sorted stably (their input
// order is (seed, local)), group heads and the first occurrence of each
// group, a second sort of the non-seed groups by (node set, first
// occurrence) for the ids, then edge keys (edge set, src id, dst id) sorted
// and deduplicated. Sizes come back to the host three times (group counts,
// per-node-set counts, per-edge-set counts).
#include <algorithm>
#include <string>
#include <vector>

#include "common.cuh"
#include "primitives.cuh"

namespace dgfx {
namespace {

constexpr int kMaxSets = 64;

unsigned grid1d(int64_t work) {
  return static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(ceil_div(std::max<int64_t>(work, 1), 256),
                                                                      int64_t(148) * 32)));
}

// Occurrence o of (node set s, sample i, local l): key = s << 32 | node,
// order = i << 24 | l, seed = i when it is sample i's seed (root set, l = 0).
__global__ void occ_keys_kernel(const int64_t* __restrict__ node_ids, const int64_t* __restrict__ node_off,
                                int64_t B, int32_t NS, int32_t root, uint64_t* __restrict__ keys,
                                uint32_t* __restrict__ vals, uint64_t* __restrict__ order,
                                int32_t* __restrict__ seed_of) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t w = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5; w < NS * B; w += warps) {
    const int64_t s = w / B, i = w - s * B;
    const int64_t a = node_off[w], b = node_off[w + 1];
    for (int64_t o = a + lane; o < b; o += 32) {
      const int64_t l = o - a;
      keys[o] = (static_cast<uint64_t>(s) << 32) | static_cast<uint32_t>(node_ids[o]);
      vals[o] = static_cast<uint32_t>(o);
      order[o] = (static_cast<uint64_t>(i) << 24) | static_cast<uint64_t>(l);
      seed_of[o] = (s == root && l == 0) ? static_cast<int32_t>(i) : -1;
    }
  }
}

__global__ void head_flags_kernel(const uint64_t* __restrict__ ks, int64_t n, int32_t* __restrict__ head) {
  for (int64_t p = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; p < n;
       p += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    head[p] = (p == 0 || ks[p] != ks[p - 1]) ? 1 : 0;
  }
}

// Per sorted position: its group (scan of heads), the group's key and first
// occurrence order (the head, by stability), the occurrence's group, and the
// group's last seed id (atomicMax; -1 when no seed occurrence).
__global__ void groups_kernel(const uint64_t* __restrict__ ks, const uint32_t* __restrict__ vs,
                              const int32_t* __restrict__ head, const int64_t* __restrict__ gscan, int64_t n,
                              const uint64_t* __restrict__ order, const int32_t* __restrict__ seed_of,
                              uint64_t* __restrict__ gkey, uint64_t* __restrict__ gfirst,
                              int32_t* __restrict__ gseed, int32_t* __restrict__ occ_group) {
  for (int64_t p = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; p < n;
       p += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t g = gscan[p] + head[p] - 1;
    const uint32_t o = vs[p];
    if (head[p]) {
      gkey[g] = ks[p];
      gfirst[g] = order[o];
    }
    occ_group[o] = static_cast<int32_t>(g);
    if (seed_of[o] >= 0) atomicMax(&gseed[g], seed_of[o]);
  }
}

__global__ void fill_kernel(int32_t* __restrict__ p, int64_t n, int32_t v) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    p[i] = v;
  }
}

// Non-seed groups sorted by (node set, first occurrence); seed groups last.
__global__ void rank_keys_kernel(const uint64_t* __restrict__ gkey, const uint64_t* __restrict__ gfirst,
                                 const int32_t* __restrict__ gseed, int64_t G, uint64_t* __restrict__ k,
                                 uint32_t* __restrict__ v) {
  for (int64_t g = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; g < G;
       g += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint64_t s = gkey[g] >> 32;
    k[g] = gseed[g] >= 0 ? ~0ull : ((s << 56) | gfirst[g]);
    v[g] = static_cast<uint32_t>(g);
  }
}

// start[s] = first sorted position of node set s (lower bound of s << 56).
__global__ void set_bounds_kernel(const uint64_t* __restrict__ k, int64_t G, int32_t NS, int64_t* __restrict__ start) {
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s > NS) return;
  const uint64_t t = s == NS ? ~0ull : (static_cast<uint64_t>(s) << 56);
  int64_t lo = 0, hi = G;
  while (lo < hi) {
    const int64_t mid = (lo + hi) >> 1;
    if (k[mid] < t) lo = mid + 1;
    else hi = mid;
  }
  start[s] = lo;
}

struct SetBases {
  int64_t base[kMaxSets];    // first output slot of node set s
  int64_t first_id[kMaxSets];  // id of the first non-seed node of set s
  int64_t start[kMaxSets];   // first sorted position of set s
};

__global__ void assign_ids_kernel(const uint64_t* __restrict__ k, const uint32_t* __restrict__ v,
                                  const uint64_t* __restrict__ gkey, const int32_t* __restrict__ gseed, int64_t G,
                                  SetBases sb, int64_t* __restrict__ gid, int64_t* __restrict__ out_nodes) {
  for (int64_t p = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; p < G;
       p += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint32_t g = v[p];
    if (gseed[g] >= 0) {
      gid[g] = gseed[g];
      continue;
    }
    const int s = static_cast<int>(k[p] >> 56);
    const int64_t id = sb.first_id[s] + (p - sb.start[s]);
    gid[g] = id;
    out_nodes[sb.base[s] + id] = static_cast<int64_t>(static_cast<uint32_t>(gkey[g]));
  }
}

__global__ void seed_nodes_kernel(const int64_t* __restrict__ node_ids, const int64_t* __restrict__ node_off,
                                  int64_t B, int32_t root, int64_t base, int64_t* __restrict__ out_nodes) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < B;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    out_nodes[base + i] = node_ids[node_off[root * B + i]];
  }
}

struct EdgeSets {
  int32_t src_ns[256];
  int32_t dst_ns[256];
};

// Edge key = edge set << 56 | src id << 28 | dst id.
__global__ void edge_keys_kernel(const int64_t* __restrict__ esrc, const int64_t* __restrict__ edst,
                                 const int64_t* __restrict__ edge_off, const int64_t* __restrict__ node_off, int64_t B,
                                 int32_t ES, EdgeSets es, const int32_t* __restrict__ occ_group,
                                 const int64_t* __restrict__ gid, uint64_t* __restrict__ keys,
                                 uint32_t* __restrict__ vals) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t w = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5; w < ES * B; w += warps) {
    const int64_t e = w / B, i = w - e * B;
    const int64_t so = node_off[es.src_ns[e] * B + i], dof = node_off[es.dst_ns[e] * B + i];
    for (int64_t j = edge_off[w] + lane; j < edge_off[w + 1]; j += 32) {
      const uint64_t a = static_cast<uint64_t>(gid[occ_group[so + esrc[j]]]);
      const uint64_t b = static_cast<uint64_t>(gid[occ_group[dof + edst[j]]]);
      keys[j] = (static_cast<uint64_t>(e) << 56) | (a << 28) | b;
      vals[j] = 0;
    }
  }
}

__global__ void unique_out_kernel(const uint64_t* __restrict__ ks, const int32_t* __restrict__ head,
                                  const int64_t* __restrict__ pos, int64_t m, int64_t* __restrict__ out_src,
                                  int64_t* __restrict__ out_dst, int64_t* __restrict__ out_es) {
  for (int64_t p = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; p < m;
       p += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    if (!head[p]) continue;
    const uint64_t k = ks[p];
    const int64_t q = pos[p];
    out_src[q] = static_cast<int64_t>((k >> 28) & ((1ull << 28) - 1));
    out_dst[q] = static_cast<int64_t>(k & ((1ull << 28) - 1));
    out_es[q] = static_cast<int64_t>(k >> 56);
  }
}

struct UnionBufs {
  uint64_t *k0, *k1, *order, *gkey, *gfirst, *rk0, *rk1;
  uint32_t *v0, *v1, *rv0, *rv1;
  int32_t *seed_of, *head, *occ_group, *gseed;
  int64_t *gscan, *gid, *start, *ekey_pos, *out_es;
};

void carve_union(Arena& a, int64_t n, int64_t m, UnionBufs* b) {
  const int64_t nm = std::max<int64_t>(std::max<int64_t>(n, m), 1);
  const size_t N = static_cast<size_t>(std::max<int64_t>(n, 1)), M = static_cast<size_t>(nm);
  b->k0 = a.take<uint64_t>(M);
  b->k1 = a.take<uint64_t>(M);
  b->v0 = a.take<uint32_t>(M);
  b->v1 = a.take<uint32_t>(M);
  b->order = a.take<uint64_t>(N);
  b->seed_of = a.take<int32_t>(N);
  b->head = a.take<int32_t>(M);
  b->gscan = a.take<int64_t>(M + 1);
  b->occ_group = a.take<int32_t>(N);
  b->gkey = a.take<uint64_t>(N);
  b->gfirst = a.take<uint64_t>(N);
  b->gseed = a.take<int32_t>(N);
  b->gid = a.take<int64_t>(N);
  b->rk0 = a.take<uint64_t>(N);
  b->rk1 = a.take<uint64_t>(N);
  b->rv0 = a.take<uint32_t>(N);
  b->rv1 = a.take<uint32_t>(N);
  b->start = a.take<int64_t>(kMaxSets + 1);
  b->ekey_pos = a.take<int64_t>(M + 1);
  b->out_es = a.take<int64_t>(M);
}

size_t union_ws(int64_t n, int64_t m) {
  Arena a(nullptr, 0);
  UnionBufs b;
  carve_union(a, n, m, &b);
  const int64_t nm = std::max(n, m) + 1;
  return a.used + std::max(radix_sort_workspace_bytes(nm), scan_workspace_bytes(nm)) + 4096;
}

}  // namespace
}  // namespace dgfx

using namespace dgfx;

extern "C" int dgfx_subgraph_union_workspace_size(int64_t total_nodes, int64_t total_edges, size_t* bytes) {
  if (bytes == nullptr || total_nodes < 0 || total_edges < 0) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_subgraph_union_workspace_size: bad arguments");
  }
  *bytes = union_ws(total_nodes, total_edges);
  return DGFX_OK;
}

extern "C" int dgfx_subgraph_union(const int64_t* d_node_ids, const int64_t* d_node_offsets,
                                   const int64_t* d_edge_src, const int64_t* d_edge_dst,
                                   const int64_t* d_edge_offsets, int64_t batch, int32_t num_nodesets,
                                   int32_t num_edgesets, int32_t root_nodeset, const int32_t* edge_src_nodeset,
                                   const int32_t* edge_dst_nodeset, int64_t total_nodes, int64_t total_edges,
                                   int64_t* d_out_node_ids, int64_t* out_node_counts, int64_t* d_out_src,
                                   int64_t* d_out_dst, int64_t* out_edge_counts, void* d_workspace,
                                   size_t workspace_bytes, dgfx_stream stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  const int32_t NS = num_nodesets, ES = num_edgesets;
  if (batch < 0 || NS < 1 || NS > kMaxSets || ES < 0 || ES > 256 || root_nodeset < 0 || root_nodeset >= NS ||
      total_nodes < 0 || total_edges < 0 || out_node_counts == nullptr || out_edge_counts == nullptr ||
      (ES > 0 && (edge_src_nodeset == nullptr || edge_dst_nodeset == nullptr))) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_subgraph_union: bad arguments");
  }
  if (batch >= (int64_t(1) << 31) || total_nodes >= (int64_t(1) << 28) || total_edges >= (int64_t(1) << 31)) {
    return fail(DGFX_ERR_UNSUPPORTED, "dgfx_subgraph_union: more than 2^28 sampled nodes or 2^31 edges");
  }
  if (d_workspace == nullptr || workspace_bytes < union_ws(total_nodes, total_edges)) {
    return fail(DGFX_ERR_WORKSPACE, "dgfx_subgraph_union: workspace too small");
  }
  for (int32_t s = 0; s < NS; ++s) out_node_counts[s] = 0;
  for (int32_t e = 0; e < ES; ++e) out_edge_counts[e] = 0;
  const int64_t n = total_nodes, m = total_edges;
  if (n == 0 || batch == 0) return DGFX_OK;
  Arena arena(d_workspace, workspace_bytes);
  UnionBufs b;
  carve_union(arena, n, m, &b);
  const size_t mark = arena.used;

  // 1. Occurrences grouped by (node set, node), input order kept.
  occ_keys_kernel<<<grid1d(NS * batch * 32), 256, 0, stream>>>(d_node_ids, d_node_offsets, batch, NS, root_nodeset,
                                                               b.k0, b.v0, b.order, b.seed_of);
  DGFX_CUDA_TRY(cudaGetLastError());
  bool in1 = false;
  DGFX_TRY(radix_sort_pairs(b.k0, b.v0, b.k1, b.v1, n, 0, 32 + bit_length(static_cast<uint64_t>(NS)), &in1, arena,
                            stream));
  arena.used = mark;
  const uint64_t* ks = in1 ? b.k1 : b.k0;
  const uint32_t* vs = in1 ? b.v1 : b.v0;
  head_flags_kernel<<<grid1d(n), 256, 0, stream>>>(ks, n, b.head);
  DGFX_TRY(exclusive_scan<int32_t>(b.head, b.gscan, n, true, arena, stream));
  arena.used = mark;
  int64_t G = 0;
  DGFX_CUDA_TRY(cudaMemcpyAsync(&G, b.gscan + n, sizeof(G), cudaMemcpyDeviceToHost, stream));
  DGFX_CUDA_TRY(cudaStreamSynchronize(stream));
  fill_kernel<<<grid1d(G), 256, 0, stream>>>(b.gseed, G, -1);
  groups_kernel<<<grid1d(n), 256, 0, stream>>>(ks, vs, b.head, b.gscan, n, b.order, b.seed_of, b.gkey, b.gfirst,
                                               b.gseed, b.occ_group);
  DGFX_CUDA_TRY(cudaGetLastError());

  // 2. Ids: seeds 0..B-1 of the root set, the rest by first occurrence.
  rank_keys_kernel<<<grid1d(G), 256, 0, stream>>>(b.gkey, b.gfirst, b.gseed, G, b.rk0, b.rv0);
  DGFX_CUDA_TRY(cudaGetLastError());
  DGFX_TRY(radix_sort_pairs(b.rk0, b.rv0, b.rk1, b.rv1, G, 0, 64, &in1, arena, stream));
  arena.used = mark;
  const uint64_t* rks = in1 ? b.rk1 : b.rk0;
  const uint32_t* rvs = in1 ? b.rv1 : b.rv0;
  set_bounds_kernel<<<1, 128, 0, stream>>>(rks, G, NS, b.start);
  DGFX_CUDA_TRY(cudaGetLastError());
  std::vector<int64_t> start(NS + 1);
  DGFX_CUDA_TRY(cudaMemcpyAsync(start.data(), b.start, sizeof(int64_t) * (NS + 1), cudaMemcpyDeviceToHost, stream));
  DGFX_CUDA_TRY(cudaStreamSynchronize(stream));
  SetBases sb{};
  int64_t acc = 0;
  for (int32_t s = 0; s < NS; ++s) {
    const int64_t fresh = start[s + 1] - start[s];
    const int64_t seeds = s == root_nodeset ? batch : 0;
    sb.base[s] = acc;
    sb.first_id[s] = seeds;
    sb.start[s] = start[s];
    out_node_counts[s] = seeds + fresh;
    acc += seeds + fresh;
  }
  seed_nodes_kernel<<<grid1d(batch), 256, 0, stream>>>(d_node_ids, d_node_offsets, batch, root_nodeset,
                                                       sb.base[root_nodeset], d_out_node_ids);
  assign_ids_kernel<<<grid1d(G), 256, 0, stream>>>(rks, rvs, b.gkey, b.gseed, G, sb, b.gid, d_out_node_ids);
  DGFX_CUDA_TRY(cudaGetLastError());

  // 3. Edges mapped to ids, sorted and deduplicated.
  if (m == 0 || ES == 0) return DGFX_OK;
  EdgeSets es{};
  for (int32_t e = 0; e < ES; ++e) {
    es.src_ns[e] = edge_src_nodeset[e];
    es.dst_ns[e] = edge_dst_nodeset[e];
  }
  edge_keys_kernel<<<grid1d(ES * batch * 32), 256, 0, stream>>>(d_edge_src, d_edge_dst, d_edge_offsets,
                                                                 d_node_offsets, batch, ES, es, b.occ_group, b.gid,
                                                                 b.k0, b.v0);
  DGFX_CUDA_TRY(cudaGetLastError());
  DGFX_TRY(radix_sort_pairs(b.k0, b.v0, b.k1, b.v1, m, 0, 56 + bit_length(static_cast<uint64_t>(ES)), &in1, arena,
                            stream));
  arena.used = mark;
  const uint64_t* eks = in1 ? b.k1 : b.k0;
  head_flags_kernel<<<grid1d(m), 256, 0, stream>>>(eks, m, b.head);
  DGFX_TRY(exclusive_scan<int32_t>(b.head, b.ekey_pos, m, true, arena, stream));
  arena.used = mark;
  unique_out_kernel<<<grid1d(m), 256, 0, stream>>>(eks, b.head, b.ekey_pos, m, d_out_src, d_out_dst, b.out_es);
  DGFX_CUDA_TRY(cudaGetLastError());
  int64_t U = 0;
  DGFX_CUDA_TRY(cudaMemcpyAsync(&U, b.ekey_pos + m, sizeof(U), cudaMemcpyDeviceToHost, stream));
  DGFX_CUDA_TRY(cudaStreamSynchronize(stream));
  std::vector<int64_t> es_of(static_cast<size_t>(U));
  if (U > 0) {
    DGFX_CUDA_TRY(cudaMemcpyAsync(es_of.data(), b.out_es, sizeof(int64_t) * U, cudaMemcpyDeviceToHost, stream));
    DGFX_CUDA_TRY(cudaStreamSynchronize(stream));
  }
  for (int64_t q = 0; q < U; ++q) ++out_edge_counts[es_of[static_cast<size_t>(q)]];
  return DGFX_OK;
}
