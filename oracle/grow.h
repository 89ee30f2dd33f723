// ORACLE — test infrastructure only. Nothing in the product
// (distributed_graph_flow_b200/) may include, link or call this file; only
// tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use it, and
// only as the checker or the timed CPU baseline.
//
// CPU restatement of DGF's per-seed sampling driver:
//   * SampleBuilder::RecursiveGrow / Grow
//       dgf/src/sampling/in_memory_sampler_ext.cc:231-370
//   * Sampler::IndexEdgeSets (plan scan, forward/backward index needs)
//       dgf/src/sampling/in_memory_sampler_ext.cc:1095-1214
//   * BuildAdjacencyIndex (id validation, reversed swap)
//       dgf/src/sampling/in_memory_sampler_ext.cc:1020-1093
//   * Sampler::Sample (argument checks, mt19937_64 seeding of the builder
//     pool and of every seed)  dgf/src/sampling/in_memory_sampler_ext.cc:418-533
//   * RandomWalkNegativeSamplerHelper / Sampler::RandomWalkNegativeSampling
//       dgf/src/sampling/in_memory_sampler_ext.cc:774-948
//
// The driver is a template over the adjacency-index type so that the same
// restatement runs on top of (a) the oracle's own restated AdjacencyIndex
// (dgf_oracle.cc) and (b) the reference's AdjacencyIndex compiled from its
// unmodified sources (ref_harness.cc, built into oracle/_ref/). Comparing the
// two pins the restated per-node samplers bit-exactly, random mode included
// (both draw from std::mt19937_64 through the same libstdc++ calls).
//
// Ordered containers (std::map / std::set) stand in for absl::btree_map /
// absl::btree_set; both iterate in key order, which is all the reference
// relies on (first-discovery numbering and lexicographically sorted edges).
#pragma once

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <functional>
#include <map>
#include <optional>
#include <random>
#include <set>
#include <string>
#include <thread>
#include <utility>
#include <vector>

namespace dgf_oracle {

using InputIdx = std::size_t;
using SampleIdx = std::uint32_t;
using Timestamp = std::int64_t;
constexpr InputIdx kNoMask = static_cast<InputIdx>(-1);

// Sampling modes. kRandom and kFirst are the reference's two modes
// (debug_sampling=False / True). kMostRecent is an extension with no
// reference counterpart: the newest k edges of the valid (ts <= seed_ts)
// prefix, in adjacency order; non-temporal edgesets fall back to kRandom.
enum Mode : int { kRandom = 0, kFirst = 1, kMostRecent = 2 };

struct Status {
  int code = 0;  // 0 ok, 3 invalid argument, 9 failed precondition
  std::string msg;
  bool ok() const { return code == 0; }
  static Status Ok() { return {}; }
  static Status Invalid(std::string m) { return {3, std::move(m)}; }
  static Status Precondition(std::string m) { return {9, std::move(m)}; }
};

struct PlanEdge {
  int edgeset;
  bool reversed;
  int hop_width;
  int child;  // index into Plan::nodes
};
struct PlanNode {
  int nodeset;
  std::vector<int> edges;  // indices into Plan::edges, in plan order
};
struct Plan {
  std::vector<PlanNode> nodes;  // nodes[0] is the root
  std::vector<PlanEdge> edges;
  bool with_replacement = false;
};

struct EdgeList {
  const std::int64_t* src = nullptr;
  const std::int64_t* dst = nullptr;
  const std::int64_t* ts = nullptr;  // nullable: non-temporal edgeset
  std::size_t num_edges = 0;
};

// One sampled subgraph: node ids per nodeset (index = local id) and the
// deduplicated, lexicographically sorted (src_local, dst_local) edges per
// edgeset.
struct Sample {
  std::vector<std::vector<InputIdx>> nodes;
  std::vector<std::vector<std::pair<SampleIdx, SampleIdx>>> edges;
};

// Validates ids and builds one direction of an edgeset index.
// Follows BuildAdjacencyIndex, in_memory_sampler_ext.cc:1020-1093.
template <class Index, class Create>
Status BuildIndex(const EdgeList& el, bool reversed, std::size_t num_src,
                  std::size_t num_dst, bool populate_edge_idxs, Index* out,
                  Create&& create) {
  if (reversed) std::swap(num_src, num_dst);
  std::vector<InputIdx> s(el.num_edges), t(el.num_edges);
  for (std::size_t i = 0; i < el.num_edges; ++i) {
    std::int64_t a = el.src[i], b = el.dst[i];
    if (reversed) std::swap(a, b);
    if (a < 0 || static_cast<std::size_t>(a) >= num_src) {
      return Status::Invalid("Invalid source node index " + std::to_string(a) +
                             ". The node index should be between 0 and " +
                             std::to_string(num_src) + ".");
    }
    if (b < 0 || static_cast<std::size_t>(b) >= num_dst) {
      return Status::Invalid("Invalid target node index " + std::to_string(b) +
                             ". The node index should be between 0 and " +
                             std::to_string(num_dst) + ".");
    }
    s[i] = static_cast<InputIdx>(a);
    t[i] = static_cast<InputIdx>(b);
  }
  return create(s, t, el.ts, populate_edge_idxs, num_src, num_dst, out);
}

// Newest-k of the valid prefix (extension mode, no reference counterpart).
template <class Index>
Status SampleLastWithTimestamp(const Index& idx, InputIdx src, Timestamp ts,
                               std::size_t k, std::vector<InputIdx>* out) {
  out->clear();
  if (src + 1 >= idx.source_blocks.size()) {
    return Status::Invalid("The source node idx " + std::to_string(src) +
                           " is out of bounds. Should be lower than " +
                           std::to_string(idx.source_blocks.size() - 1));
  }
  const InputIdx b = idx.source_blocks[src], e = idx.source_blocks[src + 1];
  const auto first = idx.timestamps.begin() + b;
  const InputIdx valid = std::upper_bound(first, idx.timestamps.begin() + e, ts) - first;
  const InputIdx take = std::min<InputIdx>(k, valid);
  for (InputIdx i = valid - take; i < valid; ++i) out->push_back(idx.target_node_idxs[b + i]);
  return Status::Ok();
}

// Adapter turning the index's own status type into the oracle Status.
template <class S> Status ToStatus(const S& s) {
  if (s.ok()) return Status::Ok();
  const int code = static_cast<int>(s.code());
  return Status{code == 0 ? 13 : code, std::string(s.message())};
}
inline Status ToStatus(const Status& s) { return s; }

template <class Index>
class Sampler {
 public:
  struct EdgeSetInfo {
    int src_ns = -1, dst_ns = -1;
    bool need_fwd = false, need_bwd = false;
    std::optional<Index> fwd, bwd;
  };

  Plan plan;
  std::vector<std::size_t> num_nodes;  // per nodeset
  std::vector<EdgeSetInfo> edgesets;
  int mask_edgeset = -1;
  int mode = kRandom;
  bool has_temporal = false;
  int num_threads = 0;
  std::mt19937_64 rng;
  std::size_t builder_pool = 0;  // size of the reference's SampleBuilder pool
  std::size_t num_steps = 0;

  // Follows Sampler::IndexEdgeSets (ext.cc:1095-1214) and CreateSampler
  // (ext.cc:1216-1246).
  template <class Create>
  Status Init(const std::vector<EdgeList>& lists, std::int64_t seed, Create&& create) {
    edgesets.assign(lists.size(), {});
    num_steps = plan.nodes.size();
    // Depth-first scan of the plan, in plan order.
    std::function<Status(int)> scan = [&](int n) -> Status {
      for (int ei : plan.nodes[n].edges) {
        const PlanEdge& pe = plan.edges[ei];
        EdgeSetInfo& es = edgesets[pe.edgeset];
        const int here = plan.nodes[n].nodeset, there = plan.nodes[pe.child].nodeset;
        const int s = pe.reversed ? there : here, t = pe.reversed ? here : there;
        if (!(es.src_ns == -1 || es.src_ns == s)) return Status::Invalid("Check failed source nodeset");
        if (!(es.dst_ns == -1 || es.dst_ns == t)) return Status::Invalid("Check failed target nodeset");
        es.src_ns = s;
        es.dst_ns = t;
        (pe.reversed ? es.need_bwd : es.need_fwd) = true;
        Status st = scan(pe.child);
        if (!st.ok()) return st;
      }
      return Status::Ok();
    };
    Status st = scan(0);
    if (!st.ok()) return st;
    for (std::size_t e = 0; e < lists.size(); ++e) {
      EdgeSetInfo& es = edgesets[e];
      const bool masked = static_cast<int>(e) == mask_edgeset;
      if (es.need_fwd) {
        Index idx;
        st = BuildIndex(lists[e], false, num_nodes[es.src_ns], num_nodes[es.dst_ns], masked, &idx, create);
        if (!st.ok()) return st;
        es.fwd = std::move(idx);
      }
      if (es.need_bwd) {
        Index idx;
        st = BuildIndex(lists[e], true, num_nodes[es.src_ns], num_nodes[es.dst_ns], masked, &idx, create);
        if (!st.ok()) return st;
        es.bwd = std::move(idx);
      }
    }
    if (seed >= 0) rng.seed(static_cast<std::uint64_t>(seed));
    else rng.seed(std::random_device()());
    return Status::Ok();
  }

  struct Builder {
    std::vector<std::vector<InputIdx>> nodes;
    std::vector<std::map<InputIdx, SampleIdx>> local;
    std::vector<std::set<std::pair<SampleIdx, SampleIdx>>> edges;
    std::vector<std::vector<InputIdx>> cache;
    std::mt19937_64 rng;
  };

  // Follows SampleBuilder::RecursiveGrow, ext.cc:231-331.
  Status Grow(Builder& b, int pnode, InputIdx src, SampleIdx src_local,
              const std::optional<Timestamp>& ts, InputIdx mask, int depth) const {
    if (!(static_cast<std::size_t>(depth) < b.cache.size())) return Status::Invalid("Check failed depth < recursion_cache.size()");
    std::vector<InputIdx>& picked = b.cache[depth];
    picked.clear();
    for (int ei : plan.nodes[pnode].edges) {
      const PlanEdge& pe = plan.edges[ei];
      const EdgeSetInfo& es = edgesets[pe.edgeset];
      const std::optional<Index>& idx = pe.reversed ? es.bwd : es.fwd;
      if (!idx.has_value()) return Status::Invalid("Check failed edges.has_value()");
      Status st;
      if (ts.has_value()) {
        if (mask_edgeset != -1) return Status::Invalid("Check failed sampler.edgeset_to_mask_idx_ == -1");
        if (mode == kFirst) {
          st = ToStatus(idx->SampleFirstWithTimestamp(src, *ts, pe.hop_width, &picked));
        } else if (mode == kMostRecent && !idx->timestamps.empty()) {
          st = SampleLastWithTimestamp(*idx, src, *ts, pe.hop_width, &picked);
        } else {
          st = ToStatus(idx->SampleRandomUniformWithTimestamp(src, *ts, pe.hop_width, &picked, &b.rng));
        }
      } else {
        const InputIdx m = (pe.edgeset == mask_edgeset) ? mask : kNoMask;
        if (mode == kFirst) {
          st = ToStatus(idx->SampleFirst(src, pe.hop_width, &picked, m));
        } else {
          st = ToStatus(idx->SampleRandomUniform(src, pe.hop_width, &picked, &b.rng, m));
        }
      }
      if (!st.ok()) return st;

      const int child = pe.child;
      const int cns = plan.nodes[child].nodeset;
      for (const InputIdx target : picked) {
        SampleIdx tl;
        if (!plan.with_replacement) {
          auto [it, fresh] = b.local[cns].try_emplace(target, static_cast<SampleIdx>(b.local[cns].size()));
          tl = it->second;
          if (fresh) b.nodes[cns].push_back(target);
        } else {
          tl = static_cast<SampleIdx>(b.nodes[cns].size());
          b.nodes[cns].push_back(target);
        }
        if (!pe.reversed) b.edges[pe.edgeset].insert({src_local, tl});
        else b.edges[pe.edgeset].insert({tl, src_local});
        st = Grow(b, child, target, tl, ts, mask, depth + 1);
        if (!st.ok()) return st;
      }
    }
    return Status::Ok();
  }

  // Follows SampleBuilder::Grow, ext.cc:333-370.
  Status GrowSeed(Builder& b, InputIdx seed, const std::optional<Timestamp>& ts, InputIdx mask) const {
    b.cache.resize(std::max(b.cache.size(), num_steps));
    b.nodes.assign(num_nodes.size(), {});
    b.local.assign(num_nodes.size(), {});
    b.edges.assign(edgesets.size(), {});
    const int root_ns = plan.nodes[0].nodeset;
    b.nodes[root_ns].push_back(seed);
    if (!plan.with_replacement) b.local[root_ns][seed] = 0;
    return Grow(b, 0, seed, 0, ts, mask, 0);
  }

  // Follows Sampler::Sample, ext.cc:418-533. `threads` only parallelises the
  // oracle's own loop over seeds (results do not depend on it); the RNG
  // accounting mirrors the reference's builder pool of `num_threads`.
  Status SampleBatch(const std::int64_t* seeds, const std::int64_t* ts,
                     const std::int64_t* masks, std::size_t n, int threads,
                     std::vector<Sample>* out) {
    if (ts != nullptr && !has_temporal) {
      return Status::Invalid(
          "seed_timestamps provided but no temporal edgesets configured. Set "
          "the 'edgeset_timestamp_features' field in the sampling plan.");
    }
    if (masks != nullptr && mask_edgeset == -1) {
      return Status::Invalid("masked_edge_idxs provided but no edgeset to mask configured.");
    }
    // Builder pool pre-fill: one draw per missing builder (ext.cc:450-455).
    while (builder_pool < static_cast<std::size_t>(num_threads)) {
      rng();
      ++builder_pool;
    }
    // One draw per seed, sequentially (ext.cc:465-468).
    std::vector<std::uint64_t> per_seed(n);
    for (std::size_t i = 0; i < n; ++i) per_seed[i] = rng();
    // Tasks beyond the pool size create a builder, drawing once each
    // (ext.cc:400-406); builders are only returned after export.
    while (builder_pool < n) {
      rng();
      ++builder_pool;
    }

    out->assign(n, {});
    std::vector<Status> status(n);
    std::atomic<std::size_t> next{0};
    auto worker = [&]() {
      Builder b;
      for (;;) {
        const std::size_t lo = next.fetch_add(16);
        if (lo >= n) break;
        const std::size_t hi = std::min(n, lo + 16);
        for (std::size_t i = lo; i < hi; ++i) {
          b.rng.seed(per_seed[i]);
          std::optional<Timestamp> t;
          if (ts != nullptr) t = ts[i];
          const InputIdx m = masks != nullptr ? static_cast<InputIdx>(masks[i]) : kNoMask;
          status[i] = GrowSeed(b, static_cast<InputIdx>(seeds[i]), t, m);
          Sample& s = (*out)[i];
          s.nodes = b.nodes;
          s.edges.resize(b.edges.size());
          for (std::size_t e = 0; e < b.edges.size(); ++e) s.edges[e].assign(b.edges[e].begin(), b.edges[e].end());
        }
      }
    };
    const int nt = std::max(1, threads);
    if (nt == 1) {
      worker();
    } else {
      std::vector<std::thread> pool;
      for (int t = 0; t < nt; ++t) pool.emplace_back(worker);
      for (auto& t : pool) t.join();
    }
    for (const Status& s : status) {
      if (!s.ok()) return s;
    }
    return Status::Ok();
  }
};

// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as
// easy as 1, 2, 3", SC'11; published round multipliers and Weyl key
// increments) and the multiply-high reduction to [0, range) (Lemire 2019).
// Used to replay the device's random stream draw for draw.
struct Philox4 {
  std::uint32_t v[4];
};
inline Philox4 Philox4x32_10(Philox4 c, std::uint32_t k0, std::uint32_t k1) {
  for (int r = 0; r < 10; ++r) {
    const std::uint64_t p0 = static_cast<std::uint64_t>(0xD2511F53u) * c.v[0];
    const std::uint64_t p1 = static_cast<std::uint64_t>(0xCD9E8D57u) * c.v[2];
    c = Philox4{{static_cast<std::uint32_t>(p1 >> 32) ^ c.v[1] ^ k0, static_cast<std::uint32_t>(p1),
                 static_cast<std::uint32_t>(p0 >> 32) ^ c.v[3] ^ k1, static_cast<std::uint32_t>(p0)}};
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return c;
}
inline std::uint64_t MulHiRange(std::uint64_t r, std::uint64_t range) {
  return static_cast<std::uint64_t>((static_cast<unsigned __int128>(r) * range) >> 64);
}

// Random-walk negatives. kind 0 draws exactly as the reference does (one
// std::mt19937_64 per seed seeded from the sampler's generator, in seed order;
// uniform_int_distribution for the plan edge, the neighbour and the fallback
// node). kind 1 replays the device's stream instead: Philox4x32-10 with key
// (seed_lo ^ call_hi, seed_hi ^ 0x52574E53) and counter (walk, step, seed
// slot, call_lo) per step, (attempt, 2^31 | slot j, seed slot, call_lo) per
// fallback draw, at most 64 fallback attempts. Visit counts are kept in
// node order and ranked by a stable sort on the count, so ties go to the
// smaller node id; the reference's order among equal counts is its hash
// map's iteration order.
template <class Index>
bool OracleHasEdge(const Index& idx, InputIdx src, InputIdx tgt) {
  if (src + 1 >= idx.source_blocks.size()) return false;
  if constexpr (requires { idx.HasEdge(src, tgt); }) {
    return idx.HasEdge(src, tgt);  // the reference's own (ref build)
  } else {
    const auto b = idx.target_node_idxs.begin() + idx.source_blocks[src];
    const auto e = idx.target_node_idxs.begin() + idx.source_blocks[src + 1];
    return std::binary_search(b, e, tgt);
  }
}

template <class Index>
Status RandomWalkNegatives(Sampler<Index>& s, const std::int64_t* seeds, std::size_t n, int target_edgeset,
                           int num_walks, int k, int kind, std::uint64_t sampler_seed, std::uint64_t call_index,
                           int threads, std::int64_t* out) {
  if (target_edgeset < 0 || target_edgeset >= static_cast<int>(s.edgesets.size())) {
    return Status::Invalid("Invalid target_edgeset_idx");
  }
  const auto& es = s.edgesets[target_edgeset];
  if (!es.fwd.has_value()) {
    return Status::Invalid("Edgeset " + std::to_string(target_edgeset) +
                           " does not have a forward index. Ensure it is traversed forward in the SamplingPlan.");
  }
  const int tns = es.dst_ns;
  const std::size_t num_target = s.num_nodes[tns];
  const bool homogeneous = es.src_ns == es.dst_ns;
  if (n > 0 && k > 0 && (num_target < 1 || (homogeneous && num_target < 2))) {
    return Status::Invalid("the target node set has no node to draw for the fallback slots");
  }
  const std::size_t root_nodes = s.num_nodes[s.plan.nodes[0].nodeset];
  for (std::size_t i = 0; i < n; ++i) {
    if (seeds[i] < 0 || static_cast<std::size_t>(seeds[i]) >= root_nodes) {
      return Status::Invalid("seed at position " + std::to_string(i) + " is not a node of the plan's root node set");
    }
  }
  std::vector<std::uint64_t> per_seed(n);
  if (kind == 0) {
    for (std::size_t i = 0; i < n; ++i) per_seed[i] = s.rng();
  }
  const std::uint32_t k0 = static_cast<std::uint32_t>(sampler_seed) ^ static_cast<std::uint32_t>(call_index >> 32);
  const std::uint32_t k1 = static_cast<std::uint32_t>(sampler_seed >> 32) ^ 0x52574E53u;
  const std::uint32_t call_lo = static_cast<std::uint32_t>(call_index);
  std::vector<Status> status(n);

  auto one = [&](std::size_t slot) {
    const InputIdx seed = static_cast<InputIdx>(seeds[slot]);
    std::int64_t* row = out + slot * static_cast<std::size_t>(k);
    std::mt19937_64 rng(per_seed[slot]);
    std::map<InputIdx, int> visits;
    for (int w = 0; w < num_walks; ++w) {
      InputIdx cur = seed;
      int pn = 0;
      for (std::uint32_t step = 0; !s.plan.nodes[pn].edges.empty(); ++step) {
        const auto& node = s.plan.nodes[pn];
        std::size_t ei, pick_r = 0;
        Philox4 r{};
        if (kind == 0) {
          std::uniform_int_distribution<std::size_t> e_dist(0, node.edges.size() - 1);
          ei = e_dist(rng);
        } else {
          r = Philox4x32_10(Philox4{{static_cast<std::uint32_t>(w), step, static_cast<std::uint32_t>(slot), call_lo}},
                            k0, k1);
          ei = MulHiRange(static_cast<std::uint64_t>(r.v[1]) << 32 | r.v[0], node.edges.size());
        }
        const PlanEdge& pe = s.plan.edges[node.edges[ei]];
        const auto& ces = s.edgesets[pe.edgeset];
        const std::optional<Index>& idx = pe.reversed ? ces.bwd : ces.fwd;
        if (!idx.has_value()) {
          status[slot] = Status::Invalid("Edgeset does not have the required index.");
          return;
        }
        const std::size_t b = idx->source_blocks[cur], e = idx->source_blocks[cur + 1];
        if (e == b) break;
        if (kind == 0) {
          std::uniform_int_distribution<std::size_t> n_dist(0, e - b - 1);
          pick_r = n_dist(rng);
        } else {
          pick_r = MulHiRange(static_cast<std::uint64_t>(r.v[3]) << 32 | r.v[2], e - b);
        }
        cur = idx->target_node_idxs[b + pick_r];
        pn = pe.child;
        if (s.plan.nodes[pn].nodeset == tns) {
          if (homogeneous && cur == seed) continue;
          ++visits[cur];
        }
      }
    }
    std::vector<std::pair<InputIdx, int>> cand;
    for (const auto& [node, count] : visits) {
      if (!OracleHasEdge(*es.fwd, seed, node)) cand.emplace_back(node, count);
    }
    std::stable_sort(cand.begin(), cand.end(), [](const auto& a, const auto& b) { return a.second > b.second; });
    const int take = std::min<int>(static_cast<int>(cand.size()), k);
    for (int j = 0; j < take; ++j) row[j] = static_cast<std::int64_t>(cand[j].first);
    for (int j = take; j < k; ++j) {
      if (kind == 0) {
        std::uniform_int_distribution<InputIdx> t_dist(0, num_target - 1);
        for (;;) {
          const InputIdx c = t_dist(rng);
          if (homogeneous && c == seed) continue;
          row[j] = static_cast<std::int64_t>(c);
          break;
        }
      } else {
        row[j] = -1;
        for (std::uint32_t a = 0; a < 64; ++a) {
          const Philox4 r = Philox4x32_10(
              Philox4{{a, 0x80000000u | static_cast<std::uint32_t>(j), static_cast<std::uint32_t>(slot), call_lo}}, k0,
              k1);
          const InputIdx c = MulHiRange(static_cast<std::uint64_t>(r.v[1]) << 32 | r.v[0], num_target);
          if (homogeneous && c == seed) continue;
          row[j] = static_cast<std::int64_t>(c);
          break;
        }
      }
    }
  };

  const int nt = std::max(1, threads);
  std::atomic<std::size_t> next{0};
  auto worker = [&]() {
    for (;;) {
      const std::size_t i = next.fetch_add(1);
      if (i >= n) break;
      one(i);
    }
  };
  if (nt == 1) {
    worker();
  } else {
    std::vector<std::thread> pool;
    for (int t = 0; t < nt; ++t) pool.emplace_back(worker);
    for (auto& t : pool) t.join();
  }
  for (const Status& st : status) {
    if (!st.ok()) return st;
  }
  return Status::Ok();
}

}  // namespace dgf_oracle
