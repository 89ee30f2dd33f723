// The sampling plan as random walks see it, kept by every dgfx_sampler.
//
// RandomWalkNegativeSamplerHelper (dgf/src/sampling/in_memory_sampler_ext.cc:
// 774-872) walks the sampler's own plan: at a plan node it takes one of the
// node's plan edges uniformly, then one uniform neighbour over that edge's
// index. The device tables below hold exactly that: per plan node its first
// plan edge and edge count, per plan edge the CSR it walks and the plan node
// (and node set) it leads to.
#pragma once

#include <cstdint>
#include <vector>

#include "../../include/dgfx.h"

namespace dgfx {

struct WalkNode {
  int32_t nodeset;
  int32_t first_edge;
  int32_t num_edges;
  int32_t pad;
};

struct WalkEdge {
  const int64_t* rowptr;
  const int32_t* col;
  int32_t child;          // plan node reached
  int32_t child_nodeset;  // its node set
};

struct WalkPlan {
  int32_t num_nodesets = 0;
  int32_t num_edgesets = 0;
  std::vector<int32_t> node_nodeset, node_first_edge, node_num_edges;
  std::vector<int32_t> edge_edgeset, edge_reversed, edge_child;
  std::vector<int64_t> num_nodes;       // per node set
  std::vector<dgfx_csr_view> forward;   // per edge set (rowptr NULL: no forward index)
  std::vector<int32_t> es_src, es_dst;  // endpoints of each walked edge set (-1: not in the plan)
  uint64_t seed = 0;
  WalkNode* d_nodes = nullptr;          // device tables, one allocation owned by the sampler
  WalkEdge* d_edges = nullptr;
};

}  // namespace dgfx

// The walk plan of a sampler (defined with the sampler).
const dgfx::WalkPlan* dgfx_sampler_walk_plan(const dgfx_sampler* s);
