// ORACLE — test infrastructure only (see grow.h). Built into
// oracle/liboracle.so by oracle/Makefile; never linked by the product.
//
// CPU restatement of DGF's adjacency index and per-node neighbour samplers,
// written from the reference's behaviour (dgf/src/sampling/in_memory_sampler.h
// and in_memory_sampler.cc), with the same field names because tests compare
// the two field by field:
//   * CreateFromEdgeList    in_memory_sampler.cc:220-257  (sort by
//                           (source, timestamp, target); duplicates kept)
//   * SampleRandomUniform   in_memory_sampler.cc:22-162   (k >= n: all; small
//                           k: rejection with duplicate check; else
//                           std::sample; masked-edge variants incl. reservoir)
//   * SampleFirst           in_memory_sampler.cc:164-202
//   * SampleRandomUniformWithTimestamp  in_memory_sampler.cc:302-333
//   * SampleFirstWithTimestamp          in_memory_sampler.cc:335-364
//   * AdjacencyIndex::to_string         in_memory_sampler.h:117-132
// Random draws go through std::mt19937_64 / std::uniform_int_distribution /
// std::sample in the same order as the reference, so with libstdc++ the
// outputs are identical for the same generator state.

#include <algorithm>
#include <cstdint>
#include <iterator>
#include <random>
#include <sstream>
#include <string>
#include <vector>

#include "grow.h"

namespace dgf_oracle {

struct OIndex {
  std::vector<InputIdx> source_blocks;
  std::vector<InputIdx> target_node_idxs;
  std::vector<Timestamp> timestamps;
  std::vector<InputIdx> edge_idxs;

  Status Bounds(InputIdx src) const {
    if (src + 1 >= source_blocks.size()) {
      return Status::Invalid("The source node idx " + std::to_string(src) +
                             " is out of bounds. Should be lower than " +
                             std::to_string(source_blocks.size() - 1));
    }
    return Status::Ok();
  }

  static Status TimestampsPresent() {
    return Status::Precondition(
        "Cannot use SampleRandomUniform when timestamps are available. Use "
        "SampleRandomUniformWithTimestamp instead.");
  }

  // k distinct positions of [0, n) by repeated draws, rejecting repeats and
  // (optionally) the masked edge; output in draw order.
  template <class Accept>
  void RejectionDraws(InputIdx b, std::size_t k, std::uniform_int_distribution<std::size_t>& dist,
                      std::mt19937_64* rng, Accept&& accept, std::vector<InputIdx>* out) const {
    std::size_t chosen[16];
    for (std::size_t i = 0; i < k; ++i) {
      for (;;) {
        const std::size_t pos = dist(*rng);
        if (!accept(pos)) continue;
        bool seen = false;
        for (std::size_t j = 0; j < i && !seen; ++j) seen = chosen[j] == pos;
        if (seen) continue;
        chosen[i] = pos;
        out->push_back(target_node_idxs[b + pos]);
        break;
      }
    }
  }

  Status SampleRandomUniform(InputIdx src, std::size_t k, std::vector<InputIdx>* out,
                             std::mt19937_64* rng, InputIdx masked = kNoMask) const {
    if (!timestamps.empty()) return TimestampsPresent();
    Status st = Bounds(src);
    if (!st.ok()) return st;
    out->clear();
    const InputIdx b = source_blocks[src], e = source_blocks[src + 1];
    const InputIdx n = e - b;
    std::uniform_int_distribution<std::size_t> dist(0, n - 1);
    if (n == 0) return Status::Ok();

    bool row_has_mask = false;
    if (masked != kNoMask) {
      if (edge_idxs.empty()) return Status::Invalid("Check failed !edge_idxs.empty()");
      for (InputIdx i = b; i < e && !row_has_mask; ++i) row_has_mask = edge_idxs[i] == masked;
    }
    if (!row_has_mask) {
      if (k >= n) {
        out->insert(out->end(), target_node_idxs.begin() + b, target_node_idxs.begin() + e);
      } else if (k < 16 && 2 * k < n) {
        RejectionDraws(b, k, dist, rng, [](std::size_t) { return true; }, out);
      } else {
        std::sample(target_node_idxs.begin() + b, target_node_idxs.begin() + e,
                    std::back_inserter(*out), k, *rng);
      }
      return Status::Ok();
    }

    std::size_t valid = 0;
    for (InputIdx i = b; i < e; ++i) valid += edge_idxs[i] != masked;
    if (valid == 0) return Status::Ok();
    if (k >= valid) {
      for (InputIdx i = b; i < e; ++i) {
        if (edge_idxs[i] != masked) out->push_back(target_node_idxs[i]);
      }
    } else if (k < 16 && 2 * k < valid) {
      RejectionDraws(b, k, dist, rng, [&](std::size_t pos) { return edge_idxs[b + pos] != masked; }, out);
    } else {
      // Reservoir over the unmasked edges.
      const std::size_t base = out->size();
      std::size_t seen = 0;
      for (InputIdx i = b; i < e; ++i) {
        if (edge_idxs[i] == masked) continue;
        ++seen;
        if (out->size() - base < k) {
          out->push_back(target_node_idxs[i]);
        } else {
          std::uniform_int_distribution<std::size_t> pick(0, seen - 1);
          const std::size_t r = pick(*rng);
          if (r < k) (*out)[base + r] = target_node_idxs[i];
        }
      }
    }
    return Status::Ok();
  }

  Status SampleFirst(InputIdx src, std::size_t k, std::vector<InputIdx>* out,
                     InputIdx masked = kNoMask) const {
    if (!timestamps.empty()) return TimestampsPresent();
    Status st = Bounds(src);
    if (!st.ok()) return st;
    out->clear();
    const InputIdx b = source_blocks[src], e = source_blocks[src + 1];
    if (masked != kNoMask && !edge_idxs.empty()) {
      for (InputIdx i = b; i < e && out->size() < k; ++i) {
        if (edge_idxs[i] != masked) out->push_back(target_node_idxs[i]);
      }
    } else {
      const InputIdx take = std::min<InputIdx>(k, e - b);
      out->insert(out->end(), target_node_idxs.begin() + b, target_node_idxs.begin() + b + take);
    }
    return Status::Ok();
  }

  InputIdx ValidPrefix(InputIdx b, InputIdx e, Timestamp ts) const {
    return std::upper_bound(timestamps.begin() + b, timestamps.begin() + e, ts) - (timestamps.begin() + b);
  }

  Status SampleRandomUniformWithTimestamp(InputIdx src, Timestamp ts, std::size_t k,
                                          std::vector<InputIdx>* out,
                                          std::mt19937_64* rng) const {
    Status st = Bounds(src);
    if (!st.ok()) return st;
    out->clear();
    if (timestamps.empty()) return SampleRandomUniform(src, k, out, rng);
    const InputIdx b = source_blocks[src];
    const InputIdx valid = ValidPrefix(b, source_blocks[src + 1], ts);
    const auto first = target_node_idxs.begin() + b;
    if (k >= valid) out->insert(out->end(), first, first + valid);
    else std::sample(first, first + valid, std::back_inserter(*out), k, *rng);
    return Status::Ok();
  }

  Status SampleFirstWithTimestamp(InputIdx src, Timestamp ts, std::size_t k,
                                  std::vector<InputIdx>* out) const {
    Status st = Bounds(src);
    if (!st.ok()) return st;
    out->clear();
    if (timestamps.empty()) return SampleFirst(src, k, out);
    const InputIdx b = source_blocks[src];
    const InputIdx take = std::min<InputIdx>(k, ValidPrefix(b, source_blocks[src + 1], ts));
    out->insert(out->end(), target_node_idxs.begin() + b, target_node_idxs.begin() + b + take);
    return Status::Ok();
  }
};

}  // namespace dgf_oracle

using OracleIndex = dgf_oracle::OIndex;

// Sorts the edge list by (source, timestamp, target) and fills the blocks.
dgf_oracle::Status OracleCreate(const std::vector<dgf_oracle::InputIdx>& s,
                                const std::vector<dgf_oracle::InputIdx>& t,
                                const std::int64_t* ts, bool populate_edge_idxs,
                                std::size_t num_src, std::size_t /*num_dst*/,
                                OracleIndex* out) {
  using dgf_oracle::InputIdx;
  struct E {
    InputIdx src, dst;
    std::int64_t ts;
    InputIdx idx;
  };
  std::vector<E> edges(s.size());
  for (std::size_t i = 0; i < s.size(); ++i) edges[i] = {s[i], t[i], ts != nullptr ? ts[i] : 0, i};
  const bool temporal = ts != nullptr;
  std::sort(edges.begin(), edges.end(), [temporal](const E& a, const E& b) {
    if (a.src != b.src) return a.src < b.src;
    if (temporal && a.ts != b.ts) return a.ts < b.ts;
    return a.dst < b.dst;
  });
  OracleIndex& x = *out;
  x.source_blocks.assign(num_src + 1, 0);
  x.target_node_idxs.clear();
  x.timestamps.clear();
  x.edge_idxs.clear();
  for (const E& e : edges) {
    ++x.source_blocks[e.src + 1];
    x.target_node_idxs.push_back(e.dst);
    if (temporal) x.timestamps.push_back(e.ts);
    if (populate_edge_idxs && !temporal) x.edge_idxs.push_back(e.idx);
  }
  for (std::size_t i = 0; i < num_src; ++i) x.source_blocks[i + 1] += x.source_blocks[i];
  return dgf_oracle::Status::Ok();
}

namespace {
template <class V> std::string Cropped(const V& v) {
  std::ostringstream os;
  const std::size_t n = std::min<std::size_t>(v.size(), 10);
  for (std::size_t i = 0; i < n; ++i) os << (i ? ", " : "") << v[i];
  if (v.size() > 10) os << ", ...";
  return os.str();
}
}  // namespace

std::string OracleIndexString(const OracleIndex& x) {
  std::ostringstream os;
  os << "AdjacencyIndex(source_blocks=(" << x.source_blocks.size() << ")[" << Cropped(x.source_blocks)
     << "], target_node_idxs=(" << x.target_node_idxs.size() << ")[" << Cropped(x.target_node_idxs) << "])";
  return os.str();
}

#include "capi.h"
