"""propagate_timestamp_to_edges (dgf/src/transform/temporal.py:24-131).

CPU: the oracle against the reference's own test vectors, and every error
path of the API (raised before any device work). GPU: the API on the same
vectors, a large random case against the oracle, out-of-range ids.
"""

import numpy as np
import pytest

from golden.reference_cases import EDGE_TS_CASES


def _case_graph(n1_ts, n2_ts, adjacency):
    from distributed_graph_flow_b200.data import in_memory_graph as img
    from distributed_graph_flow_b200.data import schema as sl

    def ns(ts):
        if ts is None:
            return img.InMemoryNodeSet(num_nodes=2, features={}), sl.NodeSchema(features={})
        name, vals = ts
        return (img.InMemoryNodeSet(num_nodes=2, features={name: np.array(vals, np.int64)}),
                sl.NodeSchema(features={name: sl.FeatureSchema(format=sl.FeatureFormat.INTEGER_64,
                                                               semantic=sl.FeatureSemantic.TIMESTAMP,
                                                               is_creation_time=True)}))

    g1, s1 = ns(n1_ts)
    g2, s2 = ns(n2_ts)
    graph = img.InMemoryGraph(node_sets={"n1": g1, "n2": g2},
                              edge_sets={"e1": img.InMemoryEdgeSet(adjacency=np.array(adjacency))})
    schema = sl.GraphSchema(node_sets={"n1": s1, "n2": s2}, edge_sets={"e1": sl.EdgeSchema(source="n1", target="n2")})
    return graph, schema


@pytest.mark.parametrize("case", EDGE_TS_CASES, ids=[c[0] for c in EDGE_TS_CASES])
def test_oracle_matches_reference_vectors(case):
    from oracle import oracle

    _, n1, n2, adj, _, expected = case
    if isinstance(expected, str):
        return
    got = oracle.edge_timestamps(None if n1 is None else np.array(n1[1]), None if n2 is None else np.array(n2[1]),
                                 np.array(adj))
    np.testing.assert_array_equal(got, np.array(expected))


def test_error_paths():
    """Both ValueErrors of the reference, raised before any device work."""
    from distributed_graph_flow_b200.data import in_memory_graph as img
    from distributed_graph_flow_b200.data import schema as sl
    from distributed_graph_flow_b200.transform import temporal

    graph, schema = _case_graph(None, None, [[0, 1], [1, 0]])
    with pytest.raises(ValueError, match="Neither source nodeset"):
        temporal.propagate_timestamp_to_edges(graph, schema)
    # temporal_test.py:201-238: the edge set already has the target feature.
    g = img.InMemoryGraph(
        node_sets={"n1": img.InMemoryNodeSet(num_nodes=2, features={"timestamps": np.array([10, 20])})},
        edge_sets={"e1": img.InMemoryEdgeSet(adjacency=np.array([[0, 1]]), features={"timestamps": np.array([1])})})
    s = sl.GraphSchema(
        node_sets={"n1": sl.NodeSchema(features={"timestamps": sl.FeatureSchema(format=sl.FeatureFormat.INTEGER_64)})},
        edge_sets={"e1": sl.EdgeSchema(source="n1", target="n1",
                                       features={"timestamps": sl.FeatureSchema(format=sl.FeatureFormat.INTEGER_64)})})
    with pytest.raises(ValueError, match="already exists in edgeset"):
        temporal.propagate_timestamp_to_edges(g, s)
    # Edge sets outside target_edgesets are left alone (no error for them).
    out_graph, out_schema = temporal.propagate_timestamp_to_edges(graph, schema, target_edgesets=["other"])
    assert out_graph.edge_sets["e1"].features == {} and out_schema.edge_sets["e1"].features == {}


@pytest.mark.gpu
@pytest.mark.parametrize("case", EDGE_TS_CASES, ids=[c[0] for c in EDGE_TS_CASES])
def test_reference_vectors_gpu(cuda, case):
    from distributed_graph_flow_b200.data import schema as sl
    from distributed_graph_flow_b200.transform import temporal

    _, n1, n2, adj, feature, expected = case
    graph, schema = _case_graph(n1, n2, adj)
    if isinstance(expected, str):
        with pytest.raises(ValueError, match=expected):
            temporal.propagate_timestamp_to_edges(graph, schema, target_feature=feature)
        return
    new_graph, new_schema = temporal.propagate_timestamp_to_edges(graph, schema, target_feature=feature)
    got = new_graph.edge_sets["e1"].features[feature]
    assert got.dtype == np.int64
    np.testing.assert_array_equal(got, np.array(expected))
    fs = new_schema.edge_sets["e1"].features[feature]
    assert fs.is_creation_time and fs.semantic == sl.FeatureSemantic.TIMESTAMP
    assert fs.format == sl.FeatureFormat.INTEGER_64
    np.testing.assert_array_equal(new_graph.edge_sets["e1"].adjacency, np.array(adj))


@pytest.mark.gpu
def test_large_random_against_oracle(cuda):
    import torch

    from distributed_graph_flow_b200.transform import temporal
    from oracle import oracle

    rng = np.random.default_rng(5)
    ns, nt, e = 100_003, 7_001, 2_000_011
    sts = rng.integers(-(2**40), 2**40, ns)
    tts = rng.integers(0, 2**62, nt)
    adj = np.stack([rng.integers(0, ns, e), rng.integers(0, nt, e)])
    dev = torch.device("cuda", 0)
    for s_ts, t_ts in ((sts, tts), (sts, None), (None, tts)):
        got = temporal.edge_timestamps(None if s_ts is None else torch.from_numpy(s_ts).to(dev),
                                       None if t_ts is None else torch.from_numpy(t_ts).to(dev),
                                       torch.from_numpy(adj[0]).to(dev), torch.from_numpy(adj[1]).to(dev))
        np.testing.assert_array_equal(got.cpu().numpy(), oracle.edge_timestamps(s_ts, t_ts, adj))
    # int32 node times: numpy keeps int32 for the result, so does the API.
    graph, schema = _case_graph(("timestamps", [10, 20]), ("timestamps", [5, 25]), [[0, 1], [1, 0]])
    graph.node_sets["n1"].features["timestamps"] = np.array([10, 20], np.int32)
    graph.node_sets["n2"].features["timestamps"] = np.array([5, 25], np.int32)
    out, _ = temporal.propagate_timestamp_to_edges(graph, schema)
    assert out.edge_sets["e1"].features["timestamps"].dtype == np.int32
    np.testing.assert_array_equal(out.edge_sets["e1"].features["timestamps"], [25, 20])


@pytest.mark.gpu
def test_out_of_range_ids(cuda):
    from distributed_graph_flow_b200.transform import temporal

    graph, schema = _case_graph(("timestamps", [10, 20]), ("timestamps", [5, 25]), [[0, 1, 2], [1, 0, 0]])
    with pytest.raises(IndexError, match="edge 2"):
        temporal.propagate_timestamp_to_edges(graph, schema)
