"""Shared test fixtures: graphs built from the reference tests' fixtures and
seeded synthetic graphs."""

import numpy as np

from distributed_graph_flow_b200.data import in_memory_graph as img
from distributed_graph_flow_b200.data import schema as sch
from golden import reference_cases as rc


def toy_graph():
    schema = sch.GraphSchema(
        node_sets={
            "n1": sch.NodeSchema(features={"f1": sch.FeatureSchema(format=sch.FeatureFormat.INTEGER_64)}),
            "n2": sch.NodeSchema(features={"f2": sch.FeatureSchema(format=sch.FeatureFormat.BYTES)}),
        },
        edge_sets={name: sch.EdgeSchema(source=s, target=t) for name, (s, t, _) in rc.TOY_EDGESETS.items()},
    )
    graph = img.InMemoryGraph(
        node_sets={n: img.InMemoryNodeSet(num_nodes=c, features=dict(rc.TOY_FEATURES[n])) for n, c in rc.TOY_NODESETS.items()},
        edge_sets={name: img.InMemoryEdgeSet(adjacency=np.array(adj)) for name, (_, _, adj) in rc.TOY_EDGESETS.items()},
    )
    return graph, schema


def temporal_graph():
    ts_feat = sch.FeatureSchema(
        format=sch.FeatureFormat.INTEGER_64, semantic=sch.FeatureSemantic.TIMESTAMP, is_creation_time=True
    )
    schema = sch.GraphSchema(
        node_sets={
            "n1": sch.NodeSchema(
                features={
                    "timestamp": ts_feat,
                    "feat": sch.FeatureSchema(format=sch.FeatureFormat.FLOAT_32, shape=(2,)),
                }
            )
        },
        edge_sets={
            "e1": sch.EdgeSchema(source="n1", target="n1", features={"timestamp": ts_feat}),
            "e2": sch.EdgeSchema(source="n1", target="n1", features={}),
        },
    )
    graph = img.InMemoryGraph(
        node_sets={
            "n1": img.InMemoryNodeSet(
                num_nodes=4, features={"timestamp": rc.TEMPORAL_NODE_TS.copy(), "feat": rc.TEMPORAL_NODE_FEAT.copy()}
            )
        },
        edge_sets={
            "e1": img.InMemoryEdgeSet(
                adjacency=np.array(rc.TEMPORAL_E1[0], np.int64), features={"timestamp": rc.TEMPORAL_E1[1].copy()}
            ),
            "e2": img.InMemoryEdgeSet(adjacency=np.array(rc.TEMPORAL_E2, np.int64)),
        },
    )
    return graph, schema


def random_hetero_graph(seed=0, sizes=None, edges=None, temporal=True, max_ts=50):
    """Small heterogeneous graph: node sets a/b/c, edge sets with duplicates,
    self loops and empty rows; int64 timestamps with many ties."""
    rng = np.random.default_rng(seed)
    sizes = sizes or {"a": 40, "b": 25, "c": 7}
    edges = edges or {"ab": ("a", "b", 300), "aa": ("a", "a", 200), "bc": ("b", "c", 60), "ca": ("c", "a", 30)}
    ts_feat = sch.FeatureSchema(format=sch.FeatureFormat.INTEGER_64, is_creation_time=True)
    node_sets = {}
    for n, c in sizes.items():
        node_sets[n] = img.InMemoryNodeSet(
            num_nodes=c, features={"x": rng.standard_normal((c, 8)).astype(np.float32)}
        )
    edge_sets = {}
    es_schema = {}
    for name, (s, t, m) in edges.items():
        # Power-law-ish sources so some rows are long and some empty.
        src = np.minimum((rng.pareto(1.2, m) * 2).astype(np.int64), sizes[s] - 1)
        dst = rng.integers(0, sizes[t], m)
        feats = {}
        if temporal:
            feats["timestamp"] = rng.integers(0, max_ts, m).astype(np.int64)
        edge_sets[name] = img.InMemoryEdgeSet(adjacency=np.stack([src, dst]).astype(np.int64), features=feats)
        es_schema[name] = sch.EdgeSchema(source=s, target=t, features={"timestamp": ts_feat} if temporal else {})
    schema = sch.GraphSchema(node_sets={n: sch.NodeSchema() for n in sizes}, edge_sets=es_schema)
    return img.InMemoryGraph(node_sets=node_sets, edge_sets=edge_sets), schema


def assert_sample_equal(got_nodes, got_edges, exp_nodes, exp_edges, msg=""):
    for k, v in exp_nodes.items():
        np.testing.assert_array_equal(np.asarray(got_nodes[k]), np.asarray(v, np.int64), err_msg=f"{msg} nodeset {k}")
    for k, v in exp_edges.items():
        exp = np.asarray(v, np.int64).reshape(2, -1)
        got = np.asarray(got_edges[k]).reshape(2, -1)
        np.testing.assert_array_equal(got, exp, err_msg=f"{msg} edgeset {k}")
