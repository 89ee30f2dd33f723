// ORACLE — test infrastructure only (see grow.h). Built into
// oracle/_ref/libdgf_ref.so by oracle/Makefile, together with the reference's
// own, unmodified dgf/src/sampling/in_memory_sampler.cc (compiled where it
// lies, against the abseil stand-ins in oracle/ref_shim/).
//
// It runs the restated per-seed driver (grow.h) on top of the reference's
// AdjacencyIndex and its per-node samplers, so these use the reference's
// compiled code: CreateFromEdgeList (in_memory_sampler.cc:220-257) and the
// four Sample* functions (in_memory_sampler.cc:22-202, 302-364).

#include <string>
#include <utility>
#include <vector>

#include "dgf/src/sampling/in_memory_sampler.h"
#include "grow.h"

using OracleIndex = dgf::sampling::in_memory_sampler::AdjacencyIndex;

namespace {
namespace ims = dgf::sampling::in_memory_sampler;

template <bool T, bool I>
dgf_oracle::Status Build(const std::vector<dgf_oracle::InputIdx>& s,
                         const std::vector<dgf_oracle::InputIdx>& t,
                         const std::int64_t* ts, std::size_t num_src,
                         std::size_t num_dst, OracleIndex* out) {
  std::vector<ims::Edge<T, I>> edges(s.size());
  for (std::size_t i = 0; i < s.size(); ++i) {
    edges[i].source = s[i];
    edges[i].target = t[i];
    if constexpr (T) edges[i].timestamp = ts[i];
    if constexpr (I) edges[i].edge_idx = i;
  }
  auto r = OracleIndex::CreateFromEdgeList<T, I>(std::move(edges), num_src, num_dst);
  if (!r.ok()) return dgf_oracle::ToStatus(r.status());
  *out = std::move(r).value();
  return dgf_oracle::Status::Ok();
}
}  // namespace

dgf_oracle::Status OracleCreate(const std::vector<dgf_oracle::InputIdx>& s,
                                const std::vector<dgf_oracle::InputIdx>& t,
                                const std::int64_t* ts, bool populate_edge_idxs,
                                std::size_t num_src, std::size_t num_dst,
                                OracleIndex* out) {
  if (ts != nullptr) return Build<true, false>(s, t, ts, num_src, num_dst, out);
  if (populate_edge_idxs) return Build<false, true>(s, t, ts, num_src, num_dst, out);
  return Build<false, false>(s, t, ts, num_src, num_dst, out);
}

std::string OracleIndexString(const OracleIndex& x) { return x.to_string(); }

#include "capi.h"
