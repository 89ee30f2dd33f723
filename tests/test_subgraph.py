"""SubGraph / MultiSubGraphs (in_memory_sampler_ext.cc:600-1017,
in_memory_sampler.py:176-261).

CPU: the oracle's restatement of SubGraphExtractor against the reference's
own test vectors (in_memory_sampler_test.py:614-978). GPU: the sampler's
subgraph / multisubgraph against the same vectors and against the oracle on
random heterogeneous graphs in the deterministic modes (debug sampling and
hop_width >= degree), duplicate seeds included.
"""

import numpy as np
import pytest

from golden import reference_cases as rc
from helpers import assert_sample_equal, random_hetero_graph, toy_graph


def _plan(schema, seed_nodeset, depth, hop_width=100):
    from distributed_graph_flow_b200.sampling import config as cfg

    return cfg.simple_sampling_config_to_sampling_plan(
        cfg.SimpleSamplingConfig(seed_nodeset=seed_nodeset, num_hops=depth, hop_width=hop_width), schema)


def _oracle_subgraph(graph, schema, plan, seeds):
    from oracle import oracle as O

    return O.subgraph(graph, plan, seeds, sorted(schema.node_sets), sorted(schema.edge_sets), schema)


def _line_graph():
    from distributed_graph_flow_b200.data import in_memory_graph as img
    from distributed_graph_flow_b200.data import schema as sl
    from distributed_graph_flow_b200.sampling import config as cfg

    nodes, edges, _ = rc.SUBGRAPH_LINE
    graph = img.InMemoryGraph(node_sets={n: img.InMemoryNodeSet(num_nodes=c) for n, c in nodes.items()},
                              edge_sets={e: img.InMemoryEdgeSet(adjacency=np.array(a)) for e, (_, _, a) in edges.items()})
    schema = sl.GraphSchema(node_sets={n: sl.NodeSchema() for n in nodes},
                            edge_sets={e: sl.EdgeSchema(source=s, target=t) for e, (s, t, _) in edges.items()})
    leaf = cfg.PlanNode("n2")
    n3 = cfg.PlanNode("n1", [cfg.PlanEdge(edgeset="e12", reversed=False, node=leaf, hop_width=5)])
    n2 = cfg.PlanNode("n1", [cfg.PlanEdge(edgeset="e11", reversed=False, node=n3, hop_width=5)])
    root = cfg.PlanNode("n1", [cfg.PlanEdge(edgeset="e11", reversed=False, node=n2, hop_width=5)])
    return graph, schema, cfg.SamplingPlan(root=root)


def _ego_graph():
    from distributed_graph_flow_b200.data import in_memory_graph as img
    from distributed_graph_flow_b200.data import schema as sl

    graph = img.InMemoryGraph(node_sets={"n1": img.InMemoryNodeSet(num_nodes=8)},
                              edge_sets={"e11": img.InMemoryEdgeSet(adjacency=np.array(rc.EGO_EDGES))})
    schema = sl.GraphSchema(node_sets={"n1": sl.NodeSchema()},
                            edge_sets={"e11": sl.EdgeSchema(source="n1", target="n1")})
    return graph, schema


@pytest.mark.parametrize("case", rc.SUBGRAPH_CASES, ids=[c[0] for c in rc.SUBGRAPH_CASES])
def test_oracle_subgraph_goldens(case):
    _, seed_ns, depth, seeds, (exp_nodes, exp_edges) = case
    graph, schema = toy_graph()
    nodes, edges = _oracle_subgraph(graph, schema, _plan(schema, seed_ns, depth), seeds)
    assert_sample_equal(nodes, edges, exp_nodes, exp_edges, case[0])


def test_oracle_multisubgraph_and_line_and_ego():
    from oracle import oracle as O

    graph, schema = toy_graph()
    seed_ns, depth, seeds, expected = rc.MULTISUBGRAPH_CASE
    for sd, (en, ee) in zip(seeds, expected):
        nodes, edges = _oracle_subgraph(graph, schema, _plan(schema, seed_ns, depth), [sd])
        assert_sample_equal(nodes, edges, en, ee, f"multisubgraph seed {sd}")
    g2, s2, plan = _line_graph()
    nodes, edges = _oracle_subgraph(g2, s2, plan, [0])
    assert_sample_equal(nodes, edges, rc.SUBGRAPH_LINE[2][0], rc.SUBGRAPH_LINE[2][1], "line")
    # test_ego_sampling_matches_subgraph: sample(0) == subgraph([0]).
    g3, s3 = _ego_graph()
    plan3 = _plan(s3, "n1", 2, hop_width=20)
    nodes, edges = _oracle_subgraph(g3, s3, plan3, [0])
    [(sn, se)] = O.OracleSampler(g3, plan3, s3, debug_sampling=True).sample([0])
    assert_sample_equal(nodes, edges, sn, se, "ego")


def _gpu_sampler(graph, schema, plan, debug=True):
    from distributed_graph_flow_b200 import sampling

    return sampling.create_sampler(graph, plan, schema, debug_sampling=debug, return_features=False,
                                   return_node_idxs=True, batch_size=8)


def _arrays(g):
    return ({n: g.node_sets[n].features["#idx"] for n in g.node_sets},
            {n: g.edge_sets[n].adjacency for n in g.edge_sets})


@pytest.mark.gpu
@pytest.mark.parametrize("case", rc.SUBGRAPH_CASES, ids=[c[0] for c in rc.SUBGRAPH_CASES])
def test_gpu_subgraph_goldens(cuda, case):
    _, seed_ns, depth, seeds, (exp_nodes, exp_edges) = case
    graph, schema = toy_graph()
    # Random mode with hop_width >= degree, as in the reference test.
    s = _gpu_sampler(graph, schema, _plan(schema, seed_ns, depth), debug=False)
    nodes, edges = _arrays(s.subgraph(seeds))
    assert_sample_equal(nodes, edges, exp_nodes, exp_edges, case[0])


@pytest.mark.gpu
def test_gpu_multisubgraph_line_ego(cuda):
    graph, schema = toy_graph()
    seed_ns, depth, seeds, expected = rc.MULTISUBGRAPH_CASE
    s = _gpu_sampler(graph, schema, _plan(schema, seed_ns, depth), debug=False)
    out = s.multisubgraph(seeds)
    assert len(out) == len(expected)
    for g, (en, ee) in zip(out, expected):
        nodes, edges = _arrays(g)
        assert_sample_equal(nodes, edges, en, ee, "multisubgraph")
    g2, s2, plan = _line_graph()
    nodes, edges = _arrays(_gpu_sampler(g2, s2, plan).subgraph([0]))
    assert_sample_equal(nodes, edges, rc.SUBGRAPH_LINE[2][0], rc.SUBGRAPH_LINE[2][1], "line")
    g3, s3 = _ego_graph()
    s = _gpu_sampler(g3, s3, _plan(s3, "n1", 2, hop_width=20))
    a = _arrays(s.sample(0))
    b = _arrays(s.subgraph([0]))
    assert_sample_equal(b[0], b[1], a[0], a[1], "ego")


@pytest.mark.gpu
@pytest.mark.parametrize("gseed", [0, 1, 2])
@pytest.mark.parametrize("hop_width", [2, 3, 1000])
def test_gpu_subgraph_matches_oracle(cuda, gseed, hop_width):
    graph, schema = random_hetero_graph(gseed, temporal=False)
    plan = _plan(schema, "a", 2, hop_width=hop_width)
    s = _gpu_sampler(graph, schema, plan, debug=True)
    rng = np.random.default_rng(gseed)
    for seeds in (rng.integers(0, 40, 1).tolist(), rng.integers(0, 40, 7).tolist(), [3, 5, 3, 9, 5], []):
        nodes, edges = _arrays(s.subgraph(seeds))
        exp_nodes, exp_edges = _oracle_subgraph(graph, schema, plan, seeds)
        assert_sample_equal(nodes, edges, exp_nodes, exp_edges, f"seeds {seeds}")
        for n in exp_nodes:
            assert len(nodes[n]) == len(exp_nodes[n]), f"seeds {seeds} nodeset {n}"
