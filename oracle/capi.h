// ORACLE — test infrastructure only (see grow.h).
//
// extern "C" surface shared by the two oracle builds:
//   * liboracle.so  — grow.h over the oracle's restated AdjacencyIndex
//   * _ref/libdgf_ref.so — grow.h over the reference's own AdjacencyIndex,
//     compiled from dgf/src/sampling/in_memory_sampler.cc
// Both export the same symbols so one ctypes wrapper (oracle/oracle.py)
// drives either. Before including this header the translation unit defines
//   using OracleIndex = ...;                         // index type
//   dgf_oracle::Status OracleCreate(...);            // CreateFromEdgeList
//   std::string OracleIndexString(const OracleIndex&);
#pragma once

#include <cstdint>
#include <cstring>
#include <atomic>
#include <memory>
#include <string_view>
#include <thread>
#include <unordered_map>
#include <string>
#include <vector>

#include "grow.h"
#include "synth_cpu.h"

namespace {
thread_local std::string g_oracle_error;

struct OracleHandle {
  dgf_oracle::Sampler<OracleIndex> sampler;
  std::vector<dgf_oracle::Sample> results;
};

struct IndexHandle {
  OracleIndex index;
};

auto CreateFn() {
  return [](const std::vector<dgf_oracle::InputIdx>& s,
            const std::vector<dgf_oracle::InputIdx>& t, const std::int64_t* ts,
            bool populate_edge_idxs, std::size_t num_src, std::size_t num_dst,
            OracleIndex* out) -> dgf_oracle::Status {
    return OracleCreate(s, t, ts, populate_edge_idxs, num_src, num_dst, out);
  };
}
}  // namespace

extern "C" {

const char* oracle_last_error() { return g_oracle_error.c_str(); }

// Plan: node i has nodeset node_nodeset[i] and plan edges
// [node_first_edge[i], node_first_edge[i] + node_num_edges[i]). Graph:
// edgeset e has num_edges[e] edges (src[e][i], dst[e][i]) and optional ts[e].
// Returns nullptr on error (message in oracle_last_error()).
void* oracle_sampler_create(int n_nodesets, const std::int64_t* num_nodes,
                            int n_edgesets, const std::int64_t* const* src,
                            const std::int64_t* const* dst,
                            const std::int64_t* const* ts,
                            const std::int64_t* num_edges, int n_plan_nodes,
                            const int* node_nodeset, const int* node_first_edge,
                            const int* node_num_edges, int n_plan_edges,
                            const int* edge_edgeset, const int* edge_reversed,
                            const int* edge_hop_width, const int* edge_child,
                            int with_replacement, int mode, int num_threads,
                            std::int64_t seed, int edgeset_to_mask,
                            int has_temporal) {
  auto h = std::make_unique<OracleHandle>();
  auto& s = h->sampler;
  s.plan.with_replacement = with_replacement != 0;
  for (int i = 0; i < n_plan_nodes; ++i) {
    dgf_oracle::PlanNode n;
    n.nodeset = node_nodeset[i];
    for (int j = 0; j < node_num_edges[i]; ++j) n.edges.push_back(node_first_edge[i] + j);
    s.plan.nodes.push_back(n);
  }
  for (int i = 0; i < n_plan_edges; ++i) {
    s.plan.edges.push_back({edge_edgeset[i], edge_reversed[i] != 0, edge_hop_width[i], edge_child[i]});
  }
  s.num_nodes.assign(num_nodes, num_nodes + n_nodesets);
  s.mask_edgeset = edgeset_to_mask;
  s.mode = mode;
  s.has_temporal = has_temporal != 0;
  s.num_threads = num_threads;
  std::vector<dgf_oracle::EdgeList> lists(n_edgesets);
  for (int e = 0; e < n_edgesets; ++e) {
    lists[e].src = src[e];
    lists[e].dst = dst[e];
    lists[e].ts = ts != nullptr ? ts[e] : nullptr;
    lists[e].num_edges = static_cast<std::size_t>(num_edges[e]);
  }
  dgf_oracle::Status st = s.Init(lists, seed, CreateFn());
  if (!st.ok()) {
    g_oracle_error = st.msg;
    return nullptr;
  }
  return h.release();
}

// Same as oracle_sampler_create, but the plan's indices are given as
// prebuilt CSR arrays (rowptr int64[n+1], col int32[E], optional ts
// int64[E]) per edgeset and direction (NULL rowptr: not walked). Used to
// time the CPU sampler on graphs too large to sort on the host; the arrays
// must already be in CreateFromEdgeList order.
void* oracle_sampler_create_csr(int n_nodesets, const std::int64_t* num_nodes, int n_edgesets,
                                const std::int64_t* const* fwd_rowptr, const std::int32_t* const* fwd_col,
                                const std::int64_t* const* fwd_ts, const std::int64_t* const* bwd_rowptr,
                                const std::int32_t* const* bwd_col, const std::int64_t* const* bwd_ts,
                                const std::int64_t* num_edges, int n_plan_nodes, const int* node_nodeset,
                                const int* node_first_edge, const int* node_num_edges, int n_plan_edges,
                                const int* edge_edgeset, const int* edge_reversed, const int* edge_hop_width,
                                const int* edge_child, int with_replacement, int mode, int num_threads,
                                std::int64_t seed, int has_temporal, int fill_threads) {
  auto h = std::make_unique<OracleHandle>();
  auto& s = h->sampler;
  s.plan.with_replacement = with_replacement != 0;
  for (int i = 0; i < n_plan_nodes; ++i) {
    dgf_oracle::PlanNode n;
    n.nodeset = node_nodeset[i];
    for (int j = 0; j < node_num_edges[i]; ++j) n.edges.push_back(node_first_edge[i] + j);
    s.plan.nodes.push_back(n);
  }
  for (int i = 0; i < n_plan_edges; ++i) {
    s.plan.edges.push_back({edge_edgeset[i], edge_reversed[i] != 0, edge_hop_width[i], edge_child[i]});
  }
  s.num_nodes.assign(num_nodes, num_nodes + n_nodesets);
  s.mode = mode;
  s.has_temporal = has_temporal != 0;
  s.num_threads = num_threads;
  s.num_steps = s.plan.nodes.size();
  s.edgesets.assign(n_edgesets, {});
  const int nt = std::max(1, fill_threads);
  auto fill = [&](const std::int64_t* rp, const std::int32_t* col, const std::int64_t* ts, std::size_t nrows,
                  std::size_t ne) {
    OracleIndex idx;
    idx.source_blocks.resize(nrows + 1);
    idx.target_node_idxs.resize(ne);
    if (ts != nullptr) idx.timestamps.resize(ne);
    std::vector<std::thread> pool;
    for (int t = 0; t < nt; ++t) {
      pool.emplace_back([&, t]() {
        const std::size_t lo = ne * t / nt, hi = ne * (t + 1) / nt;
        for (std::size_t i = lo; i < hi; ++i) idx.target_node_idxs[i] = static_cast<dgf_oracle::InputIdx>(col[i]);
        if (ts != nullptr) {
          for (std::size_t i = lo; i < hi; ++i) idx.timestamps[i] = ts[i];
        }
        const std::size_t rlo = (nrows + 1) * t / nt, rhi = (nrows + 1) * (t + 1) / nt;
        for (std::size_t i = rlo; i < rhi; ++i) idx.source_blocks[i] = static_cast<dgf_oracle::InputIdx>(rp[i]);
      });
    }
    for (auto& th : pool) th.join();
    return idx;
  };
  for (int e = 0; e < n_edgesets; ++e) {
    auto& es = s.edgesets[e];
    for (const auto& pe : s.plan.edges) {
      if (pe.edgeset != e) continue;
      (pe.reversed ? es.need_bwd : es.need_fwd) = true;
    }
    // Row counts come from the plan's node sets.
    for (int i = 0; i < n_plan_nodes; ++i) {
      for (int j : s.plan.nodes[i].edges) {
        const auto& pe = s.plan.edges[j];
        if (pe.edgeset != e) continue;
        const int here = s.plan.nodes[i].nodeset, there = s.plan.nodes[pe.child].nodeset;
        es.src_ns = pe.reversed ? there : here;
        es.dst_ns = pe.reversed ? here : there;
      }
    }
    const std::size_t ne = static_cast<std::size_t>(num_edges[e]);
    if (es.need_fwd) {
      if (fwd_rowptr == nullptr || fwd_rowptr[e] == nullptr) {
        g_oracle_error = "missing forward CSR";
        return nullptr;
      }
      es.fwd = fill(fwd_rowptr[e], fwd_col[e], fwd_ts != nullptr ? fwd_ts[e] : nullptr, s.num_nodes[es.src_ns], ne);
    }
    if (es.need_bwd) {
      if (bwd_rowptr == nullptr || bwd_rowptr[e] == nullptr) {
        g_oracle_error = "missing backward CSR";
        return nullptr;
      }
      es.bwd = fill(bwd_rowptr[e], bwd_col[e], bwd_ts != nullptr ? bwd_ts[e] : nullptr, s.num_nodes[es.dst_ns], ne);
    }
  }
  if (seed >= 0) s.rng.seed(static_cast<std::uint64_t>(seed));
  else s.rng.seed(std::random_device()());
  return h.release();
}

// A sampler over one homogeneous synthetic edge set (synth_cpu.h: the
// library's power-law generator restated on the host, optional uniform
// integer edge timestamps), indexed by OracleCreate — on the reference
// build, the reference's own AdjacencyIndex::CreateFromEdgeList — with no
// GPU involved. The edge list is cut into contiguous source-node ranges and
// each range is indexed by its own CreateFromEdgeList call (sources
// renumbered from the range start) on build_threads host threads; because
// the index sorts by source first, concatenating the ranges' rows gives the
// index one call over the whole list would build. Returns nullptr on error.
void* oracle_sampler_create_synth(std::int64_t num_nodes, std::int64_t num_edges, double alpha,
                                  std::int64_t max_degree, std::uint64_t graph_seed, int has_ts, std::int64_t ts_lo,
                                  std::int64_t ts_hi, std::uint64_t ts_seed, std::uint32_t ts_stream,
                                  int n_plan_nodes, const int* node_first_edge, const int* node_num_edges,
                                  int n_plan_edges, const int* edge_hop_width, const int* edge_child,
                                  int with_replacement, int mode, int num_threads, std::int64_t seed,
                                  int build_threads) {
  auto h = std::make_unique<OracleHandle>();
  auto& s = h->sampler;
  s.plan.with_replacement = with_replacement != 0;
  for (int i = 0; i < n_plan_nodes; ++i) {
    dgf_oracle::PlanNode n;
    n.nodeset = 0;
    for (int j = 0; j < node_num_edges[i]; ++j) n.edges.push_back(node_first_edge[i] + j);
    s.plan.nodes.push_back(n);
  }
  for (int i = 0; i < n_plan_edges; ++i) s.plan.edges.push_back({0, false, edge_hop_width[i], edge_child[i]});
  s.num_nodes.assign(1, num_nodes);
  s.mode = mode;
  s.has_temporal = has_ts != 0;
  s.num_threads = num_threads;
  s.num_steps = s.plan.nodes.size();
  s.edgesets.assign(1, {});
  auto& es = s.edgesets[0];
  es.need_fwd = true;
  es.src_ns = es.dst_ns = 0;

  const int nt = std::max(1, build_threads);
  std::vector<std::int64_t> rowptr(static_cast<std::size_t>(num_nodes) + 1);
  dgf_synth::graph_rowptr(num_nodes, num_edges, alpha, max_degree, graph_seed, rowptr.data(), nt);
  std::uint64_t pa = 0, pb = 0;
  dgf_synth::target_permutation(static_cast<std::uint64_t>(num_nodes), graph_seed, &pa, &pb);
  const std::uint32_t k0 = static_cast<std::uint32_t>(graph_seed), k1 = static_cast<std::uint32_t>(graph_seed >> 32);
  // Source ranges of about equal edge counts (4 per thread for balance).
  const int nchunks = 4 * nt;
  std::vector<std::int64_t> cut(nchunks + 1, num_nodes);
  cut[0] = 0;
  for (int c = 1; c < nchunks; ++c) {
    const std::int64_t want = num_edges / nchunks * c;
    cut[c] = std::upper_bound(rowptr.begin(), rowptr.end() - 1, want) - rowptr.begin() - 1;
    cut[c] = std::max(cut[c], cut[c - 1]);
  }
  std::vector<OracleIndex> parts(nchunks);
  std::vector<dgf_oracle::Status> errs(nchunks);
  std::atomic<int> next{0};
  std::vector<std::thread> pool;
  for (int t = 0; t < nt; ++t) {
    pool.emplace_back([&]() {
      for (int c = next++; c < nchunks; c = next++) {
        const std::int64_t lo = cut[c], hi = cut[c + 1];
        const std::int64_t e0 = rowptr[lo], e1 = rowptr[hi];
        std::vector<dgf_oracle::InputIdx> src(static_cast<std::size_t>(e1 - e0)), dst(src.size());
        std::vector<std::int64_t> ts;
        for (std::int64_t v = lo; v < hi; ++v) {
          for (std::int64_t j = rowptr[v]; j < rowptr[v + 1]; ++j) {
            src[j - e0] = static_cast<dgf_oracle::InputIdx>(v - lo);
            dst[j - e0] = static_cast<dgf_oracle::InputIdx>(dgf_synth::edge_target(j, num_nodes, pa, pb, k0, k1));
          }
        }
        if (has_ts) {
          // Edge j's timestamp is element j of the uniform stream.
          ts.resize(src.size());
          const std::uint32_t t0 = static_cast<std::uint32_t>(ts_seed), t1 = static_cast<std::uint32_t>(ts_seed >> 32);
          const std::uint64_t range = static_cast<std::uint64_t>(ts_hi - ts_lo);
          for (std::int64_t j = e0; j < e1; ++j) {
            const dgf_synth::U4 r = dgf_synth::philox4x32_10(
                dgf_synth::U4{static_cast<std::uint32_t>(j), static_cast<std::uint32_t>(j >> 32), ts_stream, 3u}, t0, t1);
            ts[j - e0] = ts_lo + static_cast<std::int64_t>(
                                     dgf_synth::bounded64(static_cast<std::uint64_t>(r.y) << 32 | r.x, range));
          }
        }
        errs[c] = OracleCreate(src, dst, has_ts ? ts.data() : nullptr, false, static_cast<std::size_t>(hi - lo),
                               static_cast<std::size_t>(num_nodes), &parts[c]);
      }
    });
  }
  for (auto& th : pool) th.join();
  for (const auto& st : errs) {
    if (!st.ok()) {
      g_oracle_error = st.msg;
      return nullptr;
    }
  }
  OracleIndex idx;
  idx.source_blocks.resize(static_cast<std::size_t>(num_nodes) + 1);
  idx.target_node_idxs.resize(static_cast<std::size_t>(num_edges));
  if (has_ts) idx.timestamps.resize(static_cast<std::size_t>(num_edges));
  pool.clear();
  for (int t = 0; t < nt; ++t) {
    pool.emplace_back([&, t]() {
      for (int c = t; c < nchunks; c += nt) {
        const std::int64_t lo = cut[c], hi = cut[c + 1], e0 = rowptr[lo];
        const OracleIndex& p = parts[c];
        for (std::int64_t i = 0; i < hi - lo; ++i) idx.source_blocks[lo + i] = e0 + p.source_blocks[i];
        std::copy(p.target_node_idxs.begin(), p.target_node_idxs.end(), idx.target_node_idxs.begin() + e0);
        if (has_ts) std::copy(p.timestamps.begin(), p.timestamps.end(), idx.timestamps.begin() + e0);
        parts[c] = OracleIndex();
      }
    });
  }
  for (auto& th : pool) th.join();
  idx.source_blocks[num_nodes] = static_cast<dgf_oracle::InputIdx>(num_edges);
  es.fwd = std::move(idx);
  if (seed >= 0) s.rng.seed(static_cast<std::uint64_t>(seed));
  else s.rng.seed(std::random_device()());
  return h.release();
}

// Switches the sampling mode of a sampler handle (kRandom / kFirst /
// kMostRecent), so one index serves a deterministic parity batch and the
// timed random-mode baseline.
void oracle_sampler_set_mode(void* hv, int mode) { static_cast<OracleHandle*>(hv)->sampler.mode = mode; }

// CSR arrays of the sampler's forward index of edge set e (rowptr int64[n+1],
// col int64[E], ts int64[E] if temporal); sizes via oracle_index_sizes on
// the sampler's index. Returns 0, or -1 if the edge set has no forward index.
int oracle_sampler_fwd_csr(void* hv, int e, std::int64_t* rowptr, std::int64_t* col, std::int64_t* ts) {
  auto* h = static_cast<OracleHandle*>(hv);
  if (e < 0 || e >= static_cast<int>(h->sampler.edgesets.size()) || !h->sampler.edgesets[e].fwd) return -1;
  const OracleIndex& x = *h->sampler.edgesets[e].fwd;
  if (rowptr) for (std::size_t i = 0; i < x.source_blocks.size(); ++i) rowptr[i] = static_cast<std::int64_t>(x.source_blocks[i]);
  if (col) for (std::size_t i = 0; i < x.target_node_idxs.size(); ++i) col[i] = static_cast<std::int64_t>(x.target_node_idxs[i]);
  if (ts) for (std::size_t i = 0; i < x.timestamps.size(); ++i) ts[i] = x.timestamps[i];
  return 0;
}

// Random-walk negatives for n seeds into out[n * k] (see
// dgf_oracle::RandomWalkNegatives; kind 0 = the reference's generator, 1 =
// the device's Philox stream for sampler_seed / call_index). Returns 0 or the
// status code (message in oracle_last_error()).
int oracle_random_walk_negatives(void* hv, const std::int64_t* seeds, std::int64_t n, int target_edgeset,
                                 int num_walks, int k, int kind, std::uint64_t sampler_seed,
                                 std::uint64_t call_index, int threads, std::int64_t* out) {
  auto* h = static_cast<OracleHandle*>(hv);
  dgf_oracle::Status st = dgf_oracle::RandomWalkNegatives(h->sampler, seeds, static_cast<std::size_t>(n),
                                                          target_edgeset, num_walks, k, kind, sampler_seed,
                                                          call_index, threads, out);
  if (!st.ok()) {
    g_oracle_error = st.msg;
    return st.code;
  }
  return 0;
}

// Raw id -> index (ByteIdToIdxMapper / PairMapping, dgf/src/io/io_ext.cc:
// 26-170): index_ids are n fixed-width byte rows of width wi, queries m rows
// of width wq; a byte id is its bytes without trailing zero bytes; a repeated
// index id maps to its last position; unknown ids map to -1. The query loop
// is split into blocks over `threads` threads like PairMapping; *mismatch is
// the largest unknown position (-1 if none).
void oracle_bytes_map(const char* index_ids, std::int64_t n, std::int64_t wi, const char* queries, std::int64_t m,
                      std::int64_t wq, int threads, std::int64_t* out, std::int64_t* mismatch) {
  auto view = [](const char* base, std::int64_t i, std::int64_t w) {
    std::int64_t len = w;
    const char* p = base + i * w;
    while (len > 0 && p[len - 1] == 0) --len;
    return std::string_view(p, static_cast<std::size_t>(len));
  };
  std::unordered_map<std::string_view, std::int64_t> index;
  index.reserve(static_cast<std::size_t>(n) * 2);
  for (std::int64_t i = 0; i < n; ++i) index[view(index_ids, i, wi)] = i;
  std::atomic<std::int64_t> last{-1};
  const int nt = std::max(1, threads);
  std::vector<std::thread> pool;
  for (int t = 0; t < nt; ++t) {
    pool.emplace_back([&, t]() {
      const std::int64_t lo = m * t / nt, hi = m * (t + 1) / nt;
      std::int64_t local = -1;
      for (std::int64_t i = lo; i < hi; ++i) {
        auto it = index.find(view(queries, i, wq));
        if (it == index.end()) {
          out[i] = -1;
          local = i;
        } else {
          out[i] = it->second;
        }
      }
      std::int64_t cur = last.load();
      while (local > cur && !last.compare_exchange_weak(cur, local)) {
      }
    });
  }
  for (auto& th : pool) th.join();
  *mismatch = last.load();
}

void oracle_sampler_free(void* h) { delete static_cast<OracleHandle*>(h); }

// Samples n seeds; keeps the results in the handle. Returns 0 on success,
// else the status code (message in oracle_last_error()).
int oracle_sample(void* hv, const std::int64_t* seeds, const std::int64_t* ts,
                  const std::int64_t* masks, std::int64_t n, int threads) {
  auto* h = static_cast<OracleHandle*>(hv);
  dgf_oracle::Status st = h->sampler.SampleBatch(seeds, ts, masks, static_cast<std::size_t>(n), threads, &h->results);
  if (!st.ok()) {
    g_oracle_error = st.msg;
    h->results.clear();
    return st.code;
  }
  return 0;
}

// node_counts[n * n_nodesets], edge_counts[n * n_edgesets] (sample-major).
void oracle_result_counts(void* hv, std::int64_t* node_counts, std::int64_t* edge_counts) {
  auto* h = static_cast<OracleHandle*>(hv);
  std::size_t a = 0, b = 0;
  for (const auto& s : h->results) {
    for (const auto& v : s.nodes) node_counts[a++] = static_cast<std::int64_t>(v.size());
    for (const auto& v : s.edges) edge_counts[b++] = static_cast<std::int64_t>(v.size());
  }
}

// Concatenated in (sample, nodeset) / (sample, edgeset) order.
void oracle_result_copy(void* hv, std::int64_t* nodes, std::int64_t* esrc, std::int64_t* edst) {
  auto* h = static_cast<OracleHandle*>(hv);
  for (const auto& s : h->results) {
    for (const auto& v : s.nodes) {
      for (auto x : v) *nodes++ = static_cast<std::int64_t>(x);
    }
    for (const auto& v : s.edges) {
      for (const auto& p : v) {
        *esrc++ = p.first;
        *edst++ = p.second;
      }
    }
  }
}

// ---- single index access (CSR parity and per-node known-answer tests) ----

void* oracle_index_build(const std::int64_t* src, const std::int64_t* dst,
                         const std::int64_t* ts, std::int64_t num_edges,
                         std::int64_t num_src, std::int64_t num_dst,
                         int reversed, int populate_edge_idxs) {
  auto h = std::make_unique<IndexHandle>();
  dgf_oracle::EdgeList el{src, dst, ts, static_cast<std::size_t>(num_edges)};
  dgf_oracle::Status st = dgf_oracle::BuildIndex(el, reversed != 0, static_cast<std::size_t>(num_src),
                                                 static_cast<std::size_t>(num_dst), populate_edge_idxs != 0,
                                                 &h->index, CreateFn());
  if (!st.ok()) {
    g_oracle_error = st.msg;
    return nullptr;
  }
  return h.release();
}

void oracle_index_free(void* h) { delete static_cast<IndexHandle*>(h); }

// sizes[0] = len(source_blocks), [1] = len(targets), [2] = len(timestamps),
// [3] = len(edge_idxs).
void oracle_index_sizes(void* hv, std::int64_t* sizes) {
  const auto& x = static_cast<IndexHandle*>(hv)->index;
  sizes[0] = static_cast<std::int64_t>(x.source_blocks.size());
  sizes[1] = static_cast<std::int64_t>(x.target_node_idxs.size());
  sizes[2] = static_cast<std::int64_t>(x.timestamps.size());
  sizes[3] = static_cast<std::int64_t>(x.edge_idxs.size());
}

void oracle_index_copy(void* hv, std::int64_t* blocks, std::int64_t* targets,
                       std::int64_t* timestamps, std::int64_t* edge_idxs) {
  const auto& x = static_cast<IndexHandle*>(hv)->index;
  for (std::size_t i = 0; i < x.source_blocks.size(); ++i) blocks[i] = static_cast<std::int64_t>(x.source_blocks[i]);
  for (std::size_t i = 0; i < x.target_node_idxs.size(); ++i) targets[i] = static_cast<std::int64_t>(x.target_node_idxs[i]);
  for (std::size_t i = 0; i < x.timestamps.size(); ++i) timestamps[i] = x.timestamps[i];
  for (std::size_t i = 0; i < x.edge_idxs.size(); ++i) edge_idxs[i] = static_cast<std::int64_t>(x.edge_idxs[i]);
}

// Writes the index's debug string into buf (truncated to cap); returns its
// full length.
std::int64_t oracle_index_string(void* hv, char* buf, std::int64_t cap) {
  const std::string s = OracleIndexString(static_cast<IndexHandle*>(hv)->index);
  if (cap > 0) {
    const std::size_t n = std::min<std::size_t>(s.size(), static_cast<std::size_t>(cap - 1));
    std::memcpy(buf, s.data(), n);
    buf[n] = 0;
  }
  return static_cast<std::int64_t>(s.size());
}

// One per-node sampler call. kind: 0 SampleRandomUniform, 1 SampleFirst,
// 2 SampleRandomUniformWithTimestamp, 3 SampleFirstWithTimestamp.
// rng_seed seeds a fresh std::mt19937_64. Returns the number of targets
// written to out (<= cap), or -1 on error.
std::int64_t oracle_index_sample(void* hv, int kind, std::int64_t source,
                                 std::int64_t k, std::int64_t seed_ts,
                                 std::int64_t masked, std::uint64_t rng_seed,
                                 std::int64_t* out, std::int64_t cap) {
  const auto& x = static_cast<IndexHandle*>(hv)->index;
  std::mt19937_64 rng(rng_seed);
  std::vector<dgf_oracle::InputIdx> res;
  const auto src = static_cast<dgf_oracle::InputIdx>(source);
  const auto m = static_cast<dgf_oracle::InputIdx>(masked);
  dgf_oracle::Status st;
  switch (kind) {
    case 0: st = dgf_oracle::ToStatus(x.SampleRandomUniform(src, k, &res, &rng, m)); break;
    case 1: st = dgf_oracle::ToStatus(x.SampleFirst(src, k, &res, m)); break;
    case 2: st = dgf_oracle::ToStatus(x.SampleRandomUniformWithTimestamp(src, seed_ts, k, &res, &rng)); break;
    default: st = dgf_oracle::ToStatus(x.SampleFirstWithTimestamp(src, seed_ts, k, &res)); break;
  }
  if (!st.ok()) {
    g_oracle_error = st.msg;
    return -1;
  }
  const std::int64_t n = std::min<std::int64_t>(cap, static_cast<std::int64_t>(res.size()));
  for (std::int64_t i = 0; i < n; ++i) out[i] = static_cast<std::int64_t>(res[i]);
  return static_cast<std::int64_t>(res.size());
}

// CPU restatement of the synthetic generators (synth_cpu.h).
void oracle_synth_rowptr(std::int64_t n_src, std::int64_t num_edges, double alpha, std::int64_t max_degree,
                         std::uint64_t seed, std::int64_t* rowptr, int threads) {
  dgf_synth::graph_rowptr(n_src, num_edges, alpha, max_degree, seed, rowptr, threads);
}

void oracle_synth_edges(const std::int64_t* rowptr, std::int64_t n_src, std::int64_t n_dst, std::uint64_t seed,
                        std::int64_t* src, std::int64_t* dst, int threads) {
  dgf_synth::graph_edges(rowptr, n_src, n_dst, seed, src, dst, threads);
}

void oracle_synth_uniform_int(std::int64_t n, std::int64_t lo, std::int64_t hi, std::uint64_t seed,
                              std::uint32_t stream, std::int64_t* out, int threads) {
  dgf_synth::uniform_int(n, lo, hi, seed, stream, out, threads);
}

void oracle_synth_normal_features(std::int64_t node_begin, std::int64_t count, std::int64_t dim, std::uint64_t seed,
                                  int bf16, void* out, int threads) {
  dgf_synth::normal_features(node_begin, count, dim, seed, bf16, out, threads);
}

}  // extern "C"
