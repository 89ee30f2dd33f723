"""Known-answer cases transcribed from the reference's own sampler tests.

Each case cites the reference test it comes from (paths within the DGF
project). The graphs are the tests' fixtures; the expected outputs are the
tests' asserted values. These pin the oracle and, through it, the GPU path.
"""

import numpy as np

# ---------------------------------------------------------------------------
# Toy 3-edgeset graph: dgf/src/sampling/in_memory_sampler_test.py:35-82.
# ---------------------------------------------------------------------------
TOY_NODESETS = {"n1": 2, "n2": 3}
TOY_EDGESETS = {
    # name: (source, target, adjacency)
    "e11": ("n1", "n1", [[1], [0]]),
    "e12": ("n1", "n2", [[0, 0, 0], [0, 1, 2]]),
    "e22": ("n2", "n2", [[0], [2]]),
}
TOY_FEATURES = {"n1": {"f1": np.array([10, 11])}, "n2": {"f2": np.array([20.0, 21.0, 22.0])}}

# Sampler.__str__ of SimpleSamplingConfig(seed_nodeset="n1", num_hops=2)
# (hop_width=5, reverse=True): in_memory_sampler_test.py:84-134.
TOY_SAMPLER_STR = """\
Sampler(
  plan=SamplingPlan(root=
Node(nodeset_idx=0, children=[
  Edge(edgeset_idx=0, reversed=0, hop_width=5, node=
    Node(nodeset_idx=0, children=[
      Edge(edgeset_idx=0, reversed=0, hop_width=5, node=
        Node(nodeset_idx=0, children=[])),
      Edge(edgeset_idx=0, reversed=1, hop_width=5, node=
        Node(nodeset_idx=0, children=[])),
      Edge(edgeset_idx=1, reversed=0, hop_width=5, node=
        Node(nodeset_idx=1, children=[]))
    ])),
  Edge(edgeset_idx=0, reversed=1, hop_width=5, node=
    Node(nodeset_idx=0, children=[
      Edge(edgeset_idx=0, reversed=0, hop_width=5, node=
        Node(nodeset_idx=0, children=[])),
      Edge(edgeset_idx=0, reversed=1, hop_width=5, node=
        Node(nodeset_idx=0, children=[])),
      Edge(edgeset_idx=1, reversed=0, hop_width=5, node=
        Node(nodeset_idx=1, children=[]))
    ])),
  Edge(edgeset_idx=1, reversed=0, hop_width=5, node=
    Node(nodeset_idx=1, children=[
      Edge(edgeset_idx=1, reversed=1, hop_width=5, node=
        Node(nodeset_idx=0, children=[])),
      Edge(edgeset_idx=2, reversed=0, hop_width=5, node=
        Node(nodeset_idx=1, children=[])),
      Edge(edgeset_idx=2, reversed=1, hop_width=5, node=
        Node(nodeset_idx=1, children=[]))
    ]))
]),
  with_replacement=0
),
  nodeset_index={n1: 0, n2: 1},
  edgeset_index={e11: 0, e12: 1, e22: 2},
  nodesets=[{idx=0, num_nodes=2}, {idx=1, num_nodes=3}]
)"""

# BuildAdjacencyIndex string goldens: in_memory_sampler_test.py:136-195.
# (adjacency, reversed, num_source_nodes, num_target_nodes, expected)
INDEX_STRING_CASES = [
    ([[], []], False, 2, 2, "AdjacencyIndex(source_blocks=(3)[0, 0, 0], target_node_idxs=(0)[])"),
    ([[0, 0, 0], [0, 1, 2]], False, 2, 3,
     "AdjacencyIndex(source_blocks=(3)[0, 3, 3], target_node_idxs=(3)[0, 1, 2])"),
    ([[0, 0, 0], [0, 1, 2]], True, 2, 3,
     "AdjacencyIndex(source_blocks=(4)[0, 1, 2, 3], target_node_idxs=(3)[0, 0, 0])"),
    ([[0, 0, 1, 1], [0, 1, 0, 1]], False, 2, 2,
     "AdjacencyIndex(source_blocks=(3)[0, 2, 4], target_node_idxs=(4)[0, 1, 0, 1])"),
]

# Deterministic (debug_sampling=True) sample goldens on the toy graph.
# Each: (description, config kwargs, seeds, masked, edgeset_to_mask,
#        expected per seed: ({nodeset: #idx}, {edgeset: adjacency})).
TOY_SAMPLE_CASES = [
    (
        "1-hop deterministic, in_memory_sampler_test.py:255-297",
        dict(seed_nodeset="n1", num_hops=1, hop_width=2),
        [0], None, None,
        [({"n1": [0, 1], "n2": [0, 1]}, {"e11": [[1], [0]], "e12": [[0, 0], [0, 1]], "e22": [[], []]})],
    ),
    (
        "2-hop deterministic, in_memory_sampler_test.py:299-343",
        dict(seed_nodeset="n1", num_hops=2, hop_width=2),
        [0], None, None,
        [({"n1": [0, 1], "n2": [0, 2, 1]}, {"e11": [[1], [0]], "e12": [[0, 0], [0, 2]], "e22": [[0], [1]]})],
    ),
    (
        "2-hop deterministic with replacement, in_memory_sampler_test.py:345-389",
        dict(seed_nodeset="n1", num_hops=2, hop_width=2, with_replacement=True),
        [0], None, None,
        [({"n1": [0, 1, 0, 0, 0], "n2": [0, 2, 1]},
          {"e11": [[1, 1], [0, 2]], "e12": [[0, 0, 3, 4], [0, 2, 0, 2]], "e22": [[0], [1]]})],
    ),
    (
        "multi-seed deterministic, in_memory_sampler_test.py:472-540",
        dict(seed_nodeset="n1", num_hops=1, hop_width=2),
        [0, 1], None, None,
        [({"n1": [0, 1], "n2": [0, 1]}, {"e11": [[1], [0]], "e12": [[0, 0], [0, 1]], "e22": [[], []]}),
         ({"n1": [1, 0], "n2": []}, {"e11": [[0], [1]], "e12": [[], []], "e22": [[], []]})],
    ),
    (
        "0-hop, in_memory_sampler_test.py:197-219",
        dict(seed_nodeset="n1", num_hops=0, hop_width=2),
        [0], None, None,
        [({"n1": [0], "n2": []}, {"e11": [[], []], "e12": [[], []], "e22": [[], []]})],
    ),
]

# Masking goldens (only the node sets the tests assert).
# in_memory_sampler_test.py:391-418 and :443-470.
TOY_MASK_CASES = [
    ("mask forward", dict(seed_nodeset="n1", num_hops=1, hop_width=2), 0, 1, "e12", {"n2": [0, 2]}),
    ("mask reverse", dict(seed_nodeset="n2", num_hops=1, hop_width=2, reverse=True), 0, 0, "e12", {"n1": []}),
]

# ---------------------------------------------------------------------------
# Temporal graph: dgf/src/util/gen_test_graph.py:2179-2250 (include_e2=True).
# ---------------------------------------------------------------------------
TEMPORAL_NODES = {"n1": 4}
TEMPORAL_NODE_TS = np.array([10, 20, 30, 40], np.int64)
TEMPORAL_NODE_FEAT = np.array([[1.0, 1.0], [2.0, 2.0], [3.0, 3.0], [4.0, 4.0]], np.float32)
TEMPORAL_E1 = ([[0, 0, 1], [1, 2, 3]], np.array([15, 25, 35], np.int64))
TEMPORAL_E2 = [[2, 3], [0, 1]]

# test_temporal_sampling, in_memory_sampler_test.py:980-1086: plan
# SimpleSamplingConfig(n1, num_hops=2, hop_width=2, reverse=False,
# temporal_sampling=True), debug_sampling=True, seed node 0.
TEMPORAL_CASES = {
    10: ({"n1": [0]}, {"e1": [[], []], "e2": [[], []]}, [10], [[1.0, 1.0]]),
    20: ({"n1": [0, 1]}, {"e1": [[0], [1]], "e2": [[], []]}, [10, 20], [[1.0, 1.0], [2.0, 2.0]]),
    25: ({"n1": [0, 1, 2]}, {"e1": [[0, 0], [1, 2]], "e2": [[2], [0]]}, [10, 20, 30],
         [[1.0, 1.0], [2.0, 2.0], [3.0, 3.0]]),
    40: ({"n1": [0, 1, 3, 2]}, {"e1": [[0, 0, 1], [1, 3, 2]], "e2": [[3], [0]]}, [10, 20, 40, 30],
         [[1.0, 1.0], [2.0, 2.0], [4.0, 4.0], [3.0, 3.0]]),
}

# ---------------------------------------------------------------------------
# AdjacencyIndex known answers: dgf/src/sampling/in_memory_sampler_test.cc.
# ---------------------------------------------------------------------------
# (edges [(src, dst[, ts])], num_src, num_dst, source_blocks, targets, timestamps)
CSR_CASES = [
    ("BasicCase :93-102", [(0, 0), (0, 1), (2, 3)], 3, 4, [0, 2, 2, 3], [0, 1, 3], None),
    ("EmptyEdges :104-111", [], 2, 2, [0, 0, 0], [], None),
    ("SourceWithNoOutgoingEdges :113-121", [(0, 1), (2, 3)], 4, 4, [0, 1, 1, 2, 2], [1, 3], None),
    ("DuplicateEdgesKept :123-132", [(0, 1), (0, 1), (0, 2)], 1, 3, [0, 3], [1, 1, 2], None),
    ("EdgesOutOfOrder :134-143", [(2, 3), (0, 1), (0, 0)], 3, 4, [0, 2, 2, 3], [0, 1, 3], None),
    ("Temporal :163-174", [(0, 1, 15), (0, 2, 25), (1, 3, 35)], 4, 4, [0, 2, 3, 3, 3], [1, 2, 3], [15, 25, 35]),
]

# Per-node sampler known answers on CreateTestIndex = {{0,3,3,5},
# {10,11,12,20,21}} (in_memory_sampler_test.cc:24-82) and the masking /
# temporal ones (:176-287). kind: 0 random, 1 first, 2 random+ts, 3 first+ts.
PER_NODE_FIRST = [
    ("SampleFirst_LessThanAvailable :35-40", 0, 2, [10, 11]),
    ("SampleFirst_MoreThanAvailable :42-47", 0, 5, [10, 11, 12]),
    ("SampleFirst_NoNeighbors :49-54", 1, 1, []),
]
PER_NODE_RANDOM = [
    # (name, source, k, expected size, allowed superset)
    ("SampleRandomUniform_LessThanAvailable :56-64", 0, 2, 2, [10, 11, 12]),
    ("SampleRandomUniform_MoreThanAvailable :66-73", 0, 5, 3, [10, 11, 12]),
    ("SampleRandomUniform_NoNeighbors :75-82", 1, 1, 0, []),
]
# Masked index: edges 0->1 (e0), 0->2 (e1), 0->3 (e2) (:194-268), and
# 0->1..5 (e0..e4) for MoreCandidates (:270-287).
MASK_FIRST = ("SampleFirst_WithMasking :194-206", 2, 1, [1, 3])
MASK_RANDOM = [
    # (name, targets, edge_idxs, k, masked, expected size, allowed)
    ("WithMasking :208-222", [1, 2, 3], [0, 1, 2], 2, 1, 2, [1, 3]),
    ("AllMasked :224-237", [1, 2, 3], [5, 5, 5], 2, 5, 0, []),
    ("NoneMasked :239-253", [1, 2, 3], [0, 1, 2], 2, 5, 2, [1, 2, 3]),
    ("NumSamplesLargerThanAvailable :255-268", [1, 2, 3], [0, 1, 2], 5, 1, 2, [1, 3]),
    ("MoreCandidates :270-287", [1, 2, 3, 4, 5], [0, 1, 2, 3, 4], 2, 2, 2, [1, 2, 4, 5]),
]
# SampleWithTimestamp_FiltersFutureEdges :176-190.
TEMPORAL_FILTER = ([(0, 1, 15), (0, 2, 25), (1, 3, 35)], 4, 4, 0, 20, 2, [1])

# ---------------------------------------------------------------------------
# propagate_timestamp_to_edges: dgf/src/transform/temporal_test.py:27-238.
# (name, n1 node ts or None, n2 node ts or None, adjacency, target_feature,
#  expected edge ts or the ValueError message fragment)
# ---------------------------------------------------------------------------
EDGE_TS_CASES = [
    ("basic :27-81", ("timestamps", [10, 20]), ("timestamps", [5, 25]), [[0, 1], [1, 0]], "timestamps", [25, 20]),
    ("single_node_timestamp :83-119", ("timestamps", [10, 20]), None, [[0, 1], [1, 0]], "timestamps", [10, 20]),
    ("custom_names :145-199", ("time", [10, 20]), ("ts", [5, 25]), [[0, 1], [1, 0]], "edge_ts", [25, 20]),
    ("fail_no_timestamps :121-143", None, None, [[0, 1], [1, 0]], "timestamps", "Neither source nodeset"),
]

# ---------------------------------------------------------------------------
# merge_graphs: dgf/src/transform/merge_test.py:30-224 on two copies of
# gen_test_graph.generate_in_memory_graph(False, False) (:1259-1337) with
# generate_schema(False, False, variable_length=False) (:98-190).
# ---------------------------------------------------------------------------
MERGE_GRAPH = {
    "nodes": {"n1": 2, "n2": 2},
    "features": {
        "n1": {"f2": np.array([[0.0, 1.0], [2.0, 3.0]], np.float32), "f1": np.array([[b"blue"], [b"red"]])},
        "n2": {"f3": np.array([4, 5], np.int64), "f4": np.array([10, 11], np.int64)},
    },
    "edges": {"e1": ("n1", "n1", [[0, 0], [0, 1]]), "e2": ("n1", "n2", [[0, 0], [0, 1]])},
}
MERGE_PADDING = {"nodes": {"n1": 6, "n2": 7}, "edges": {"e1": 5, "e2": 6}}
MERGE_EXPECTED_PADDED = {
    "offsets": {"n1": [0, 2, 4], "n2": [0, 2, 4]},
    "num_nodes": {"n1": 6, "n2": 7},
    "features": {
        "n1": {"f1": [[b"blue"], [b"red"], [b"blue"], [b"red"], [b""], [b""]],
               "f2": [[0.0, 1.0], [2.0, 3.0], [0.0, 1.0], [2.0, 3.0], [0.0, 0.0], [0.0, 0.0]]},
        "n2": {"f3": [4, 5, 4, 5, 0, 0, 0], "f4": [10, 11, 10, 11, 0, 0, 0]},
    },
    "adjacency": {"e1": [[0, 0, 2, 2, 5], [0, 1, 2, 3, 5]], "e2": [[0, 0, 2, 2, 5, 5], [0, 1, 2, 3, 6, 6]]},
}
MERGE_EXPECTED_UNPADDED = {
    "offsets": {"n1": [0, 2, 4], "n2": [0, 2, 4]},
    "num_nodes": {"n1": 4, "n2": 4},
    "adjacency": {"e1": [[0, 0, 2, 2], [0, 1, 2, 3]], "e2": [[0, 0, 2, 2], [0, 1, 2, 3]]},
}
# test_batch_padding_too_small (:156-180): n1 padded to 4 (no room for the sentinel).
MERGE_TOO_SMALL_MESSAGE = r"Required at least 5 nodes \(including the sentinel node\), but the padder only defines 4."

# ---------------------------------------------------------------------------
# SubGraph / MultiSubGraphs on the toy graph: in_memory_sampler_test.py:
# 614-830 (SimpleSamplingConfig(seed_nodeset, num_hops=depth, hop_width=100),
# reverse=True by default). Each case: (name, seed nodeset, depth, seeds,
# ({nodeset: #idx}, {edgeset: adjacency})).
# ---------------------------------------------------------------------------
SUBGRAPH_CASES = [
    ("depth0 n1 [0,1] :616-642", "n1", 0, [0, 1],
     ({"n1": [0, 1], "n2": []}, {"e11": [[], []], "e12": [[], []], "e22": [[], []]})),
    ("depth1 n1 [0,1] :643-669", "n1", 1, [0, 1],
     ({"n1": [0, 1], "n2": [0, 1, 2]}, {"e11": [[1], [0]], "e12": [[0, 0, 0], [0, 1, 2]], "e22": [[], []]})),
    ("depth2 n1 [0,1] :670-702", "n1", 2, [0, 1],
     ({"n1": [0, 1], "n2": [0, 2, 1]}, {"e11": [[1], [0]], "e12": [[0, 0, 0], [0, 1, 2]], "e22": [[0], [1]]})),
    ("depth2 n2 [2,0] :703-735", "n2", 2, [2, 0],
     ({"n1": [0, 1], "n2": [2, 0, 1]}, {"e11": [[1], [0]], "e12": [[0, 0, 0], [0, 1, 2]], "e22": [[1], [0]]})),
]
# multisubgraph([0, 1]) with num_hops=1, hop_width=100 (:764-830).
MULTISUBGRAPH_CASE = ("n1", 1, [0, 1], [
    ({"n1": [0, 1], "n2": [0, 1, 2]}, {"e11": [[1], [0]], "e12": [[0, 0, 0], [0, 1, 2]], "e22": [[], []]}),
    ({"n1": [1, 0], "n2": []}, {"e11": [[0], [1]], "e12": [[], []], "e22": [[], []]}),
])
# test_subgraph_line (:883-978): one n1 node with a self loop, one n2 node,
# plan n1 -e11-> n1 -e11-> n1 -e12-> n2 (hop_width 5), seed [0].
SUBGRAPH_LINE = ({"n1": 1, "n2": 1}, {"e11": ("n1", "n1", [[0], [0]]), "e12": ("n1", "n2", [[0], [0]])},
                 ({"n1": [0], "n2": [0]}, {"e11": [[0], [0]], "e12": [[0], [0]]}))
# test_ego_sampling_matches_subgraph (:832-881): 8 nodes, 18 directed edges;
# 2 hops, hop_width 20: sample(0) == subgraph([0]).
EGO_EDGES = [[0, 0, 0, 1, 1, 1, 2, 2, 3, 4, 4, 4, 4, 5, 6, 6, 6, 7],
             [1, 4, 6, 0, 2, 3, 1, 4, 1, 0, 2, 5, 6, 4, 0, 4, 7, 6]]

# ---------------------------------------------------------------------------
# Random-walk negative sampling: in_memory_sampler_test.py:1171-1277 and
# dgf/src/generate/edge_neighbor_generator_test.py:48-131, on the
# recommender-like graph of dgf/src/util/gen_test_graph.py:2253-2329
# (n1: 3 nodes, n2: 6 nodes, e2: n1 -> n2 with edges 0->0, 0->1, 1->1, 1->2).
# Plans: "walk3" = n1 -e2-> n2 -e2(rev)-> n1 -e2-> n2 (all hop_width 1);
# "walk2" = n1 -e2-> n2 -e2(rev)-> n1. Each case: (name, plan, seeds,
# num_walks, k, {row: expected first entry}); every entry must be a node of
# n2 (0..5).
# ---------------------------------------------------------------------------
RECOMMENDER_NODES = {"n1": 3, "n2": 6}
RECOMMENDER_E2 = [[0, 0, 1, 1], [0, 1, 1, 2]]
RW_NEGATIVE_CASES = [
    ("random walk top-1 :1171-1225", "walk3", [0], 500, 3, {0: 2}),
    ("fallback with 0 walks :1227-1277", "walk2", [0], 0, 3, {}),
    ("generator seeds of edges 0 and 2 :85-119", "walk3", [0, 1], 500, 3, {0: 2, 1: 0}),
    ("generator seed without edges :121-131", "walk3", [2], 500, 3, {}),
]

# ---------------------------------------------------------------------------
# Raw id -> index: dgf/src/io/io_cc_test.py:24-85. Each case: (name, index
# ids, query ids, expected indices, expected last-mismatch position).
# ---------------------------------------------------------------------------
ID_MAP_CASES = [
    ("with_all_matches", [b"X", b"Y"], [b"Y", b"X", b"Y"], [1, 0, 1], -1),
    ("with_missing_match", [b"X", b"Y"], [b"Y", b"X", b"Z"], [1, 0, -1], 2),
    ("empty_index", [], [], [], -1),
    ("empty_value", [b"X", b""], [b"", b"X", b"Z"], [1, 0, -1], 2),
]
# PairMapping (:87-103): mappers over [X, Y] and [Z, X].
PAIR_MAP_CASE = ([b"X", b"Y"], [b"Z", b"X"], [b"Y", b"X", b"_"], [b"Z", b"Z", b"X"],
                 [[1, 0, -1], [0, 0, 1]], 2, -1)

# ---------------------------------------------------------------------------
# GF graph fixture: dgf/src/util/gen_test_graph.py:345-466 (generate_gf_graph,
# edge_ids=True) and the in-memory graph it must load as (:1259-1330,
# node_ids=True, edge_ids=True); checked by dgf/src/io/graph_in_memory_test.py:
# 28-177. n1 ids are bytes (one shard), n2 ids int64 (two shards); e2's
# targets are n2's integer ids; with dangling edges e2's second source is
# b"missing" ("Node ID 'missing' not found in nodeset 'n1'", one e2 edge left
# when removed).
# ---------------------------------------------------------------------------
GF_N1 = {"#id": [b"1", b"2"], "f1": [[b"blue"], [b"red"]], "f2": [[0.0, 1.0], [2.0, 3.0]]}
GF_N2_SHARDS = [
    {"#id": [1], "f3": [4], "f4": [10], "f5": [[11, 12]], "f6": [[[11, 12], [13, 14]]]},
    {"#id": [2], "f3": [5], "f4": [11], "f5": [[12, 13, 14]], "f6": [[[15, 16], [17, 18], [19, 20]]]},
]
GF_E1 = {"#source": [b"1", b"1"], "#target": [b"1", b"2"], "#id": [b"a", b"b"]}
GF_E2 = {"#source": [b"1", b"1"], "#target": [1, 2], "#id": [b"A", b"B"]}
GF_ADJACENCY = {"e1": [[0, 0], [0, 1]], "e2": [[0, 0], [0, 1]]}

# ---------------------------------------------------------------------------
# Causal timeseries slicing: dgf/src/sampling/temporal_test.py:67-298 and
# in_memory_sampler_test.py:1279-1460. Each case: (name, {feature: rows},
# groups [(timestamp feature, [features])], target, max_len, expected
# {feature: rows}).
# ---------------------------------------------------------------------------
TS_FILTER_CASES = [
    ("scalar target 28, max 2 :67-131",
     {"time": [[10, 20, 30, 40, 50], [5, 15, 25, 35]], "signal": [[1.0, 2.0, 3.0, 4.0, 5.0], [0.5, 1.5, 2.5, 3.5]]},
     [("time", ["time", "signal"])], 28, 2,
     {"time": [[10, 20], [15, 25]], "signal": [[1.0, 2.0], [1.5, 2.5]]}),
    ("group without timestamps left alone :133-183",
     {"time": [[10, 20, 30, 40]], "signal": [[1.0, 2.0, 3.0, 4.0]], "waveform": [[0.1, 0.2, 0.3, 0.4]]},
     [("time", ["time", "signal"]), (None, ["waveform"])], 25, None,
     {"time": [[10, 20]], "signal": [[1.0, 2.0]], "waveform": [[0.1, 0.2, 0.3, 0.4]]}),
    ("edge set target 20 :185-240",
     {"timestamps": [[10, 20, 30, 40]], "edge_sig": [[1.0, 2.0, 3.0, 4.0]]},
     [("timestamps", ["timestamps", "edge_sig"])], 20, None,
     {"timestamps": [[10, 20]], "edge_sig": [[1.0, 2.0]]}),
    ("cache and filter target 30 :262-294",
     {"time": [[10, 20, 30, 40, 50]], "signal": [[1.0, 2.0, 3.0, 4.0, 5.0]]},
     [("time", ["time", "signal"])], 30, None,
     {"time": [[10, 20, 30]], "signal": [[1.0, 2.0, 3.0]]}),
]
# Sampler level (in_memory_sampler_test.py:1279-1400): alerts (#creation_time
# 30, 60) <- hardware (one node, time 10..70, signal 1..7), one hop reversed,
# temporal sampling, max_timeseries_len 3, seeds [0, 1] at [30, 60].
TS_SAMPLER_TIME = [10, 20, 30, 40, 50, 60, 70]
TS_SAMPLER_EXPECTED = [([10, 20, 30], [1.0, 2.0, 3.0]), ([40, 50, 60], [4.0, 5.0, 6.0])]
