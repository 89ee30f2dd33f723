"""merge_graphs / merge_batch (dgf/src/transform/merge.py:33-232).

CPU: the padding errors (raised from host metadata before any device work).
GPU: the reference's test vectors (padded, unpadded, without the sentinel
offset) and merge_batch on a sampled batch against merge_graphs of the same
samples exported to host graphs.
"""

import numpy as np
import pytest

from golden import reference_cases as rc


def _graph_and_schema():
    from distributed_graph_flow_b200.data import in_memory_graph as img
    from distributed_graph_flow_b200.data import schema as sl

    g = rc.MERGE_GRAPH
    graph = img.InMemoryGraph(
        node_sets={n: img.InMemoryNodeSet(num_nodes=c, features={k: v.copy() for k, v in g["features"][n].items()})
                   for n, c in g["nodes"].items()},
        edge_sets={e: img.InMemoryEdgeSet(adjacency=np.array(adj)) for e, (_, _, adj) in g["edges"].items()},
    )
    schema = sl.GraphSchema(
        node_sets={
            "n1": sl.NodeSchema(features={"f2": sl.FeatureSchema(format=sl.FeatureFormat.FLOAT_32, shape=(2,)),
                                          "f1": sl.FeatureSchema(format=sl.FeatureFormat.BYTES, shape=(1,))}),
            "n2": sl.NodeSchema(features={"f3": sl.FeatureSchema(format=sl.FeatureFormat.INTEGER_64),
                                          "f4": sl.FeatureSchema(format=sl.FeatureFormat.INTEGER_64, shape=())}),
        },
        edge_sets={e: sl.EdgeSchema(source=s, target=t) for e, (s, t, _) in g["edges"].items()},
    )
    return graph, schema


def _padding(nodes, edges):
    from distributed_graph_flow_b200.data import padding as pl

    return pl.Padding(node_sets={k: pl.NodeSetPadding(num_nodes=v) for k, v in nodes.items()},
                      edge_sets={k: pl.EdgeSetPadding(num_edges=v) for k, v in edges.items()})


def test_padding_too_small():
    from distributed_graph_flow_b200.transform import merge

    graph, schema = _graph_and_schema()
    pad = _padding({"n1": 4, "n2": 7}, {"e1": 5, "e2": 6})
    with pytest.raises(merge.InsufficientPaddingError, match=rc.MERGE_TOO_SMALL_MESSAGE):
        merge.merge_graphs([graph, graph], schema, pad)
    pad = _padding({"n1": 6, "n2": 7}, {"e1": 3, "e2": 6})
    with pytest.raises(merge.InsufficientPaddingError, match="Required at least 4 edges, but the padder only defines 3"):
        merge.merge_graphs([graph, graph], schema, pad)
    assert merge.merge_graphs([], schema, pad)[1] == {}


@pytest.mark.gpu
@pytest.mark.parametrize("padded", [True, False])
@pytest.mark.parametrize("sentinel_offset", [True, False])
def test_reference_vectors(cuda, padded, sentinel_offset):
    from distributed_graph_flow_b200.transform import merge

    graph, schema = _graph_and_schema()
    pad = _padding(rc.MERGE_PADDING["nodes"], rc.MERGE_PADDING["edges"]) if padded else None
    merged, offsets = merge.merge_graphs([graph, graph], schema, pad, sentinel_offset=sentinel_offset)
    exp = rc.MERGE_EXPECTED_PADDED if padded else rc.MERGE_EXPECTED_UNPADDED
    for n, off in exp["offsets"].items():
        np.testing.assert_array_equal(offsets[n], off if sentinel_offset else off[:-1])
    for n, c in exp["num_nodes"].items():
        assert merged.node_sets[n].num_nodes == c
    for e, adj in exp["adjacency"].items():
        np.testing.assert_array_equal(merged.edge_sets[e].adjacency, np.array(adj))
    if padded:
        for n, feats in exp["features"].items():
            for f, v in feats.items():
                np.testing.assert_array_equal(merged.node_sets[n].features[f], np.array(v))


@pytest.mark.gpu
@pytest.mark.parametrize("padded", [True, False])
def test_merge_batch_matches_merge_graphs(cuda, padded):
    """Sampled batch merged on the device == merge_graphs of its exported graphs."""
    import torch

    from distributed_graph_flow_b200 import sampling
    from distributed_graph_flow_b200.sampling import _in_memory_sampler_ext as ext
    from distributed_graph_flow_b200.transform import merge
    from helpers import random_hetero_graph

    graph, schema = random_hetero_graph(3, temporal=False)
    s = sampling.create_sampler(graph, sampling.SimpleSamplingConfig(seed_nodeset="a", num_hops=2, hop_width=4),
                                schema, debug_sampling=True, return_features=False, return_node_idxs=True,
                                batch_size=64)
    native = s._cc_sampler
    seeds = torch.arange(0, 40, dtype=torch.int64, device="cuda") % graph.node_sets["a"].num_nodes
    batch = native.sample_merged(seeds)
    graphs = ext.export_graphs(batch)
    pad = None
    if padded:
        pad = _padding({n: int(sum(g.node_sets[n].num_nodes for g in graphs)) + 3 for n in schema.node_sets},
                       {e: int(sum(g.edge_sets[e].adjacency.shape[1] for g in graphs)) + 2 for e in schema.edge_sets})
    ns_schema = {n: type(schema.node_sets[n])(features={}) for n in schema.node_sets}
    hschema = type(schema)(node_sets=ns_schema, edge_sets=schema.edge_sets)
    exp_graph, exp_off = merge.merge_graphs(graphs, hschema, pad)
    node_ids, adjacency, offsets = merge.merge_batch(batch, schema, pad)
    for e in schema.edge_sets:
        np.testing.assert_array_equal(adjacency[e].cpu().numpy(), exp_graph.edge_sets[e].adjacency)
    for n in schema.node_sets:
        np.testing.assert_array_equal(offsets[n].cpu().numpy(), exp_off[n])
        exp_ids = np.concatenate([g.node_sets[n].features["#idx"] for g in graphs])
        got = node_ids[n].cpu().numpy()
        np.testing.assert_array_equal(got[:len(exp_ids)], exp_ids)
        assert len(got) == exp_graph.node_sets[n].num_nodes
