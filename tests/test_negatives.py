"""Random-walk negative sampling (in_memory_sampler_ext.cc:774-948) and the
link-prediction generator around it (generate/edge_neighbor_generator.py).

CPU: the oracle restatement (and its twin over the reference's compiled
AdjacencyIndex / HasEdge) against the reference tests' assertions
(in_memory_sampler_test.py:1171-1277, edge_neighbor_generator_test.py), the
walk invariants on random graphs, and the error messages. GPU: the same
reference assertions through the product API, bit-exact rows against the
oracle replaying the device's Philox stream (shared-memory and global visit
tables, homogeneous / bipartite / temporal edge sets, fallback-only and
k > candidates), a chi-square test of the fallback draws, and the errors.
"""

import numpy as np
import pytest

from golden import reference_cases as rc
from helpers import random_hetero_graph


def _recommender():
    from distributed_graph_flow_b200.data import in_memory_graph as img
    from distributed_graph_flow_b200.data import schema as sl

    graph = img.InMemoryGraph(
        node_sets={n: img.InMemoryNodeSet(num_nodes=c) for n, c in rc.RECOMMENDER_NODES.items()},
        edge_sets={"e2": img.InMemoryEdgeSet(adjacency=np.array(rc.RECOMMENDER_E2, np.int64))})
    schema = sl.GraphSchema(node_sets={n: sl.NodeSchema() for n in rc.RECOMMENDER_NODES},
                            edge_sets={"e2": sl.EdgeSchema(source="n1", target="n2")})
    return graph, schema


def _walk_plan(name):
    from distributed_graph_flow_b200.sampling import config as cfg

    if name == "walk3":
        tail = cfg.PlanNode("n1", [cfg.PlanEdge(edgeset="e2", reversed=False, hop_width=1, node=cfg.PlanNode("n2"))])
    else:
        tail = cfg.PlanNode("n1")
    mid = cfg.PlanNode("n2", [cfg.PlanEdge(edgeset="e2", reversed=True, hop_width=1, node=tail)])
    return cfg.SamplingPlan(root=cfg.PlanNode("n1", [cfg.PlanEdge(edgeset="e2", reversed=False, hop_width=1,
                                                                  node=mid)]))


def _backward_only_plan():
    """n2 -e2(rev)-> n1: e2 has no forward index."""
    from distributed_graph_flow_b200.sampling import config as cfg

    return cfg.SamplingPlan(root=cfg.PlanNode("n2", [cfg.PlanEdge(edgeset="e2", reversed=True, hop_width=2,
                                                                  node=cfg.PlanNode("n1"))]))


def _check_case(rows, case):
    name, _, seeds, _, k, first = case
    assert rows.shape == (len(seeds), k), name
    for r, v in first.items():
        assert rows[r, 0] == v, f"{name}: row {r} = {rows[r]}"
    assert np.all((rows >= 0) & (rows < rc.RECOMMENDER_NODES["n2"])), name


def _oracle(graph, schema, plan, ref=False, seed=1234, ets=None):
    from oracle import oracle as O

    if ref and not O.available(ref=True):
        pytest.skip("reference twin not built")
    return O.OracleSampler(graph, plan, schema, seed=seed, edgeset_timestamp_features=ets, ref=ref)


@pytest.mark.parametrize("ref", [False, True])
@pytest.mark.parametrize("case", rc.RW_NEGATIVE_CASES, ids=[c[0] for c in rc.RW_NEGATIVE_CASES])
def test_oracle_reference_cases(case, ref):
    graph, schema = _recommender()
    o = _oracle(graph, schema, _walk_plan(case[1]), ref=ref)
    for kind in (0, 1):
        _check_case(o.random_walk_negatives(case[2], 0, case[3], case[4], kind=kind, sampler_seed=99), case)


def _homogeneous(seed, n=60, m=400, temporal=False):
    from distributed_graph_flow_b200.data import in_memory_graph as img
    from distributed_graph_flow_b200.data import schema as sl

    rng = np.random.default_rng(seed)
    src = np.minimum((rng.pareto(1.1, m) * 3).astype(np.int64), n - 1)
    dst = rng.integers(0, n, m)
    feats = {"ts": rng.integers(0, 50, m).astype(np.int64)} if temporal else {}
    ts_feat = sl.FeatureSchema(format=sl.FeatureFormat.INTEGER_64, is_creation_time=True)
    graph = img.InMemoryGraph(node_sets={"v": img.InMemoryNodeSet(num_nodes=n)},
                              edge_sets={"e": img.InMemoryEdgeSet(adjacency=np.stack([src, dst]), features=feats)})
    schema = sl.GraphSchema(node_sets={"v": sl.NodeSchema()},
                            edge_sets={"e": sl.EdgeSchema("v", "v", features={"ts": ts_feat} if temporal else {})})
    return graph, schema


def _hop_plan(nodeset, edgeset, widths):
    from distributed_graph_flow_b200 import sampling

    return sampling.explicit_plan(nodeset, edgeset, widths)


def _neighbours(graph, edgeset, v):
    adj = np.asarray(graph.edge_sets[edgeset].adjacency)
    return set(adj[1][adj[0] == v].tolist())


@pytest.mark.parametrize("gseed", [0, 1])
def test_oracle_invariants_homogeneous(gseed):
    """Ranked negatives are walk-reachable non-neighbours, never the seed;
    the restated HasEdge agrees with the reference's own (ref twin), on a
    temporal index (rows sorted by time) too."""
    for temporal in (False, True):
        graph, schema = _homogeneous(gseed, temporal=temporal)
        plan = _hop_plan("v", "e", [3, 2])
        ets = {"e": "ts"} if temporal else None
        o = _oracle(graph, schema, plan, ets=ets)
        seeds = np.arange(60)
        rows = o.random_walk_negatives(seeds, 0, 40, 6, kind=1, sampler_seed=5)
        from oracle import oracle as O

        if O.available(ref=True):
            r = _oracle(graph, schema, plan, ref=True, ets=ets)
            np.testing.assert_array_equal(r.random_walk_negatives(seeds, 0, 40, 6, kind=1, sampler_seed=5), rows)
            np.testing.assert_array_equal(r.random_walk_negatives(seeds, 0, 40, 6, kind=0),
                                          o.random_walk_negatives(seeds, 0, 40, 6, kind=0))
        for s, row in zip(seeds, rows):
            assert s not in row
            assert np.all((row >= 0) & (row < 60))


def test_oracle_errors():
    from oracle import oracle as O

    graph, schema = _recommender()
    o = _oracle(graph, schema, _walk_plan("walk3"))
    with pytest.raises(O.OracleError, match="Invalid target_edgeset_idx"):
        o.random_walk_negatives([0], 1, 5, 3)
    o2 = _oracle(graph, schema, _backward_only_plan())
    with pytest.raises(O.OracleError, match="does not have a forward index"):
        o2.random_walk_negatives([0], 0, 5, 3)


# ---------------------------------------------------------------------------
# GPU
# ---------------------------------------------------------------------------
def _gpu(graph, schema, plan, seed=1234, ets=None):
    from distributed_graph_flow_b200 import sampling

    if ets:
        plan.edgeset_timestamp_features = ets
    return sampling.create_sampler(graph, plan, schema, batch_size=1, seed=seed)


@pytest.mark.gpu
@pytest.mark.parametrize("case", rc.RW_NEGATIVE_CASES, ids=[c[0] for c in rc.RW_NEGATIVE_CASES])
def test_gpu_reference_cases(cuda, case):
    graph, schema = _recommender()
    s = _gpu(graph, schema, _walk_plan(case[1]))
    e = s._cc_sampler.EdgesetNameToEdgesetIdx("e2")
    rows = s._cc_sampler.RandomWalkNegativeSampling(seed_node_idxs=np.array(case[2], np.int64), target_edgeset_idx=e,
                                                     num_walks=case[3], num_negatives_per_seed=case[4])
    _check_case(rows, case)


@pytest.mark.gpu
def test_gpu_edge_neighbor_generator(cuda):
    from distributed_graph_flow_b200.generate import edge_neighbor_generator as eng

    graph, schema = _recommender()
    s = _gpu(graph, schema, _walk_plan("walk3"))
    rw = eng.RandomWalkNegativeSampler(graph=graph, schema=schema, target_edgeset="e2", num_negative_neighbors=3,
                                       sampler=s, num_walks=500)
    neg = rw.sample(np.array([0, 2], np.int64))
    assert neg.shape == (2, 3) and neg[0, 0] == 2 and neg[1, 0] == 0
    assert np.all((neg >= 0) & (neg < 6))
    gen = eng.EdgeNeighborGenerator(graph, schema, "e2", 3, sampler=s,
                                    config=eng.RandomWalkEdgeNeighborGeneratorConfig(num_walks_per_negative=100))
    out = gen.generate(np.array([0, 1], np.int64))
    np.testing.assert_array_equal(out.pos_src_node_idxs, [0, 0])
    np.testing.assert_array_equal(out.pos_trg_node_idxs, [0, 1])
    assert out.neg_trg_node_idxs.shape == (2, 3) and np.all(out.neg_trg_node_idxs[:, 0] == 2)
    rnd = eng.EdgeNeighborGenerator(graph, schema, "e2", 3).generate(np.array([0, 1], np.int64))
    assert rnd.neg_trg_node_idxs.shape == (2, 3) and np.all((rnd.neg_trg_node_idxs >= 0) & (rnd.neg_trg_node_idxs < 6))
    with pytest.raises(ValueError, match="A sampler must be provided"):
        eng.EdgeNeighborGenerator(graph, schema, "e2", 3, config=eng.RandomWalkEdgeNeighborGeneratorConfig())


def _compare(cuda, graph, schema, plan, target, seeds, walks, k, ets=None, calls=2):
    s = _gpu(graph, schema, plan, seed=77, ets=ets)
    cc = s._cc_sampler
    o = _oracle(graph, schema, plan, ets=ets)
    e = cc.EdgesetNameToEdgesetIdx(target)
    d_seeds = cuda.as_tensor(np.asarray(seeds, np.int64), device="cuda")
    for call in range(calls):
        got = cc.random_walk_negatives(d_seeds, e, walks, k, call_index=call).cpu().numpy()
        exp = o.random_walk_negatives(seeds, e, walks, k, kind=1, sampler_seed=cc._seed, call_index=call)
        np.testing.assert_array_equal(got, exp, err_msg=f"{target} walks={walks} k={k} call={call}")
    return got


@pytest.mark.gpu
@pytest.mark.parametrize("walks,k", [(0, 4), (1, 3), (7, 5), (50, 40), (300, 8)])
def test_gpu_matches_oracle_homogeneous(cuda, walks, k):
    for temporal in (False, True):
        graph, schema = _homogeneous(3, temporal=temporal)
        rng = np.random.default_rng(walks)
        seeds = rng.integers(0, 60, 97)
        _compare(cuda, graph, schema, _hop_plan("v", "e", [4, 3]), "e", seeds, walks, k,
                 ets={"e": "ts"} if temporal else None)


@pytest.mark.gpu
@pytest.mark.parametrize("gseed", [0, 1])
def test_gpu_matches_oracle_hetero(cuda, gseed):
    """Bipartite walks over a branching plan (several plan edges per node)."""
    from distributed_graph_flow_b200.sampling import config as cfg

    graph, schema = random_hetero_graph(gseed, temporal=False)
    leaf_b = cfg.PlanNode("b")
    a2 = cfg.PlanNode("a", [cfg.PlanEdge(edgeset="ab", reversed=False, hop_width=2, node=leaf_b),
                            cfg.PlanEdge(edgeset="aa", reversed=False, hop_width=2, node=cfg.PlanNode("a"))])
    b1 = cfg.PlanNode("b", [cfg.PlanEdge(edgeset="ab", reversed=True, hop_width=2, node=a2)])
    root = cfg.PlanNode("a", [cfg.PlanEdge(edgeset="ab", reversed=False, hop_width=3, node=b1),
                              cfg.PlanEdge(edgeset="aa", reversed=False, hop_width=3, node=cfg.PlanNode("a")),
                              cfg.PlanEdge(edgeset="ca", reversed=True, hop_width=3, node=cfg.PlanNode("c"))])
    plan = cfg.SamplingPlan(root=root)
    seeds = np.random.default_rng(gseed).integers(0, 40, 64)
    for target in ("ab", "aa"):
        for walks, k in ((20, 3), (200, 30)):
            _compare(cuda, graph, schema, plan, target, seeds, walks, k)


@pytest.mark.gpu
def test_gpu_matches_oracle_global_table(cuda):
    """Visit tables too large for shared memory (per-CTA workspace slices)."""
    graph, schema = _homogeneous(4, n=20000, m=200000)
    seeds = np.random.default_rng(0).integers(0, 20000, 40)
    got = _compare(cuda, graph, schema, _hop_plan("v", "e", [5]), "e", seeds, 6000, 50, calls=1)
    assert got.shape == (40, 50)


@pytest.mark.gpu
def test_gpu_fallback_chi_square(cuda):
    """num_walks = 0: every slot is a uniform draw over the target node set
    without the seed (homogeneous); chi-square over the 49 other nodes."""
    graph, schema = _homogeneous(5, n=50)
    s = _gpu(graph, schema, _hop_plan("v", "e", [2]))
    cc = s._cc_sampler
    seeds = cuda.zeros(20000, dtype=cuda.int64, device="cuda")
    rows = cc.random_walk_negatives(seeds, 0, 0, 5).cpu().numpy()
    assert not np.any(rows == 0)
    counts = np.bincount(rows.reshape(-1), minlength=50)[1:]
    exp = rows.size / 49
    chi2 = float(((counts - exp) ** 2 / exp).sum())
    # 48 degrees of freedom: the 0.999 quantile is about 84.0.
    assert chi2 < 84.0, chi2


@pytest.mark.gpu
def test_gpu_edge_cases_and_errors(cuda):
    graph, schema = _recommender()
    s = _gpu(graph, schema, _walk_plan("walk3"))
    cc = s._cc_sampler
    assert cc.RandomWalkNegativeSampling(np.zeros(0, np.int64), 0, 10, 3).shape == (0, 3)
    assert cc.RandomWalkNegativeSampling(np.array([0, 1]), 0, 10, 0).shape == (2, 0)
    with pytest.raises(ValueError, match="Invalid target_edgeset_idx"):
        cc.RandomWalkNegativeSampling(np.array([0]), 1, 10, 3)
    with pytest.raises(ValueError, match="not a node of the plan's root node set"):
        cc.RandomWalkNegativeSampling(np.array([0, 3]), 0, 10, 3)
    s2 = _gpu(graph, schema, _backward_only_plan())
    with pytest.raises(ValueError, match="Edgeset 'e2' does not have a forward index"):
        s2._cc_sampler.RandomWalkNegativeSampling(np.array([0]), 0, 10, 3)
    # The sampler keeps working after a failed call.
    rows = cc.RandomWalkNegativeSampling(np.array([0]), 0, 500, 3)
    assert rows[0, 0] == 2
