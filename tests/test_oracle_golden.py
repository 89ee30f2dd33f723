"""Pins the oracle against the reference's own known answers (CPU only).

Every expectation comes from the reference's tests (cited in
golden/reference_cases.py) or from the reference's compiled code in
oracle/_ref (bit-exact, random mode included), via fixtures committed under
tests/golden/.
"""

import numpy as np
import pytest

from golden import reference_cases as rc
from helpers import assert_sample_equal, random_hetero_graph, temporal_graph, toy_graph
from oracle import oracle as O

from distributed_graph_flow_b200.sampling import config as cfg

REFS = [False] + ([True] if O.available(ref=True) else [])


def _edges_arr(edges):
    if not edges:
        return np.zeros((2, 0), np.int64), None
    a = np.array([e[:2] for e in edges], np.int64).T
    ts = np.array([e[2] for e in edges], np.int64) if len(edges[0]) == 3 else None
    return a, ts


@pytest.mark.parametrize("ref", REFS)
@pytest.mark.parametrize("case", rc.CSR_CASES, ids=[c[0] for c in rc.CSR_CASES])
def test_csr_known_answers(case, ref):
    name, edges, n_src, n_dst, blocks, targets, ts = case
    adj, t = _edges_arr(edges)
    idx = O.Index(adj, t, False, n_src, n_dst, ref=ref)
    arr = idx.arrays()
    np.testing.assert_array_equal(arr["source_blocks"], blocks)
    np.testing.assert_array_equal(arr["target_node_idxs"], targets)
    if ts is not None:
        np.testing.assert_array_equal(arr["timestamps"], ts)


@pytest.mark.parametrize("ref", REFS)
@pytest.mark.parametrize("case", rc.INDEX_STRING_CASES)
def test_index_strings(case, ref):
    adj, rev, n_src, n_dst, expected = case
    idx = O.Index(np.array(adj, np.int64).reshape(2, -1), None, rev, n_src, n_dst, ref=ref)
    assert str(idx) == expected


def _test_index(ref):
    # CreateTestIndex: {0,3,3,5} / {10,11,12,20,21} as an edge list.
    adj = np.array([[0, 0, 0, 2, 2], [10, 11, 12, 20, 21]], np.int64)
    return O.Index(adj, None, False, 3, 22, ref=ref)


@pytest.mark.parametrize("ref", REFS)
def test_per_node_first(ref):
    idx = _test_index(ref)
    for name, src, k, expected in rc.PER_NODE_FIRST:
        np.testing.assert_array_equal(idx.sample(1, src, k), expected, err_msg=name)


@pytest.mark.parametrize("ref", REFS)
def test_per_node_random(ref):
    idx = _test_index(ref)
    for name, src, k, size, allowed in rc.PER_NODE_RANDOM:
        got = idx.sample(0, src, k)
        assert len(got) == size, name
        assert set(got.tolist()) <= set(allowed), name
        assert len(set(got.tolist())) == len(got), name


@pytest.mark.parametrize("ref", REFS)
def test_masking_known_answers(ref):
    name, k, masked, expected = rc.MASK_FIRST
    adj = np.array([[0, 0, 0], [1, 2, 3]], np.int64)
    idx = O.Index(adj, None, False, 1, 4, populate_edge_idxs=True, ref=ref)
    np.testing.assert_array_equal(idx.sample(1, 0, k, masked=masked), expected, err_msg=name)
    for name, targets, eidx, k, masked, size, allowed in rc.MASK_RANDOM:
        if len(set(eidx)) != len(eidx):
            # AllMasked gives every edge the same edge_idx, which an index
            # built from an edge list never has (edge_idx = list position).
            continue
        assert eidx == list(range(len(eidx)))
        adj = np.array([[0] * len(targets), targets], np.int64)
        idx = O.Index(adj, None, False, 1, max(targets) + 1, populate_edge_idxs=True, ref=ref)
        for seed in range(20):
            got = idx.sample(0, 0, k, masked=masked, rng_seed=seed)
            assert len(got) == size, name
            assert set(got.tolist()) <= set(allowed), name
    # A row whose every edge is masked yields nothing (the AllMasked intent).
    idx = O.Index(np.array([[0], [3]]), None, False, 1, 4, populate_edge_idxs=True, ref=ref)
    assert len(idx.sample(0, 0, 2, masked=0)) == 0


@pytest.mark.parametrize("ref", REFS)
def test_temporal_filter(ref):
    edges, n_src, n_dst, src, ts, k, expected = rc.TEMPORAL_FILTER
    adj, t = _edges_arr(edges)
    idx = O.Index(adj, t, False, n_src, n_dst, ref=ref)
    np.testing.assert_array_equal(idx.sample(2, src, k, seed_ts=ts), expected)
    np.testing.assert_array_equal(idx.sample(3, src, k, seed_ts=ts), expected)


def _oracle_sampler(graph, schema, conf, ref, **kw):
    plan = cfg.simple_sampling_config_to_sampling_plan(cfg.SimpleSamplingConfig(**conf), schema)
    return O.OracleSampler(graph, plan, schema, edgeset_timestamp_features=plan.edgeset_timestamp_features, ref=ref, **kw)


@pytest.mark.parametrize("ref", REFS)
@pytest.mark.parametrize("case", rc.TOY_SAMPLE_CASES, ids=[c[0] for c in rc.TOY_SAMPLE_CASES])
def test_toy_deterministic_goldens(case, ref):
    name, conf, seeds, masked, mask_es, expected = case
    graph, schema = toy_graph()
    s = _oracle_sampler(graph, schema, conf, ref, debug_sampling=True, seed=1)
    out = s.sample(seeds)
    for (nodes, edges), (en, ee) in zip(out, expected):
        assert_sample_equal(nodes, edges, en, ee, name)


@pytest.mark.parametrize("ref", REFS)
@pytest.mark.parametrize("case", rc.TOY_MASK_CASES, ids=[c[0] for c in rc.TOY_MASK_CASES])
def test_toy_masking_goldens(case, ref):
    name, conf, seed, masked, mask_es, expected = case
    graph, schema = toy_graph()
    s = _oracle_sampler(graph, schema, conf, ref, debug_sampling=True, seed=1, edgeset_to_mask=mask_es)
    nodes, _ = s.sample([seed], masks=[masked])[0]
    for k, v in expected.items():
        np.testing.assert_array_equal(nodes[k], v, err_msg=name)


@pytest.mark.parametrize("ref", REFS)
@pytest.mark.parametrize("ts", sorted(rc.TEMPORAL_CASES))
def test_temporal_goldens(ts, ref):
    graph, schema = temporal_graph()
    conf = dict(seed_nodeset="n1", num_hops=2, hop_width=2, reverse=False, temporal_sampling=True)
    s = _oracle_sampler(graph, schema, conf, ref, debug_sampling=True, seed=1)
    nodes, edges = s.sample([0], seed_ts=[ts])[0]
    en, ee, _, _ = rc.TEMPORAL_CASES[ts]
    assert_sample_equal(nodes, edges, en, ee, f"ts={ts}")


@pytest.mark.parametrize("ref", REFS)
def test_temporal_without_seed_ts_errors(ref):
    # in_memory_sampler_test.py:1088-1110.
    graph, schema = temporal_graph()
    conf = dict(seed_nodeset="n1", num_hops=2, hop_width=2, reverse=False, temporal_sampling=True)
    s = _oracle_sampler(graph, schema, conf, ref, seed=1)
    with pytest.raises(ValueError, match="Cannot use SampleRandomUniform when timestamps are available"):
        s.sample([0])


@pytest.mark.parametrize("ref", REFS)
def test_ego_sample_equals_wide_fanout(ref):
    # in_memory_sampler_test.py:832-881: with hop_width >= degree, sample()
    # returns the full 2-hop neighbourhood.
    adj = np.array(
        [[0, 0, 0, 1, 1, 1, 2, 2, 3, 4, 4, 4, 4, 5, 6, 6, 6, 7], [1, 4, 6, 0, 2, 3, 1, 4, 1, 0, 2, 5, 6, 4, 0, 4, 7, 6]]
    )
    from distributed_graph_flow_b200.data import in_memory_graph as img
    from distributed_graph_flow_b200.data import schema as sch

    graph = img.InMemoryGraph(
        node_sets={"n1": img.InMemoryNodeSet(num_nodes=8)}, edge_sets={"e11": img.InMemoryEdgeSet(adjacency=adj)}
    )
    schema = sch.GraphSchema(node_sets={"n1": sch.NodeSchema()}, edge_sets={"e11": sch.EdgeSchema("n1", "n1")})
    s = _oracle_sampler(graph, schema, dict(seed_nodeset="n1", num_hops=2, hop_width=20), ref, seed=3)
    nodes, edges = s.sample([0])[0]
    # Every node within 2 hops (either direction) of node 0.
    assert sorted(nodes["n1"].tolist()) == [0, 1, 2, 3, 4, 5, 6, 7]
    assert nodes["n1"][0] == 0


def test_restatement_matches_reference_code():
    """liboracle (restatement) == _ref (reference's compiled samplers) on
    random graphs in every mode, random mode bit for bit."""
    if not O.available(ref=True):
        pytest.skip("reference build not available")
    for seed in range(4):
        graph, schema = random_hetero_graph(seed, temporal=(seed % 2 == 0))
        for conf in (
            dict(seed_nodeset="a", num_hops=2, hop_width=3, temporal_sampling=seed % 2 == 0),
            dict(seed_nodeset="b", num_hops=3, hop_width=2, with_replacement=True, temporal_sampling=seed % 2 == 0),
        ):
            for debug in (False, True):
                outs = []
                for ref in (False, True):
                    s = _oracle_sampler(graph, schema, conf, ref, debug_sampling=debug, seed=7, num_threads=4)
                    seeds = np.arange(graph.node_sets[conf["seed_nodeset"]].num_nodes)
                    ts = np.full(len(seeds), 30) if conf.get("temporal_sampling") else None
                    outs.append([s.sample_raw(seeds, ts), s.sample_raw(seeds[::-1].copy(), ts)])
                for a, b in zip(outs[0], outs[1]):
                    for x, y in zip(a, b):
                        np.testing.assert_array_equal(x, y)


def test_committed_reference_vectors():
    """The restatement reproduces the vectors generated from the reference's
    compiled code (tests/golden/make_golden.py -> ref_vectors.npz)."""
    from golden import make_golden

    data = np.load(make_golden.OUT)
    for case in make_golden.cases():
        key = case["key"]
        s = make_golden.make_sampler(case, ref=False)
        got = s.sample_raw(case["seeds"], case.get("ts"), case.get("masks"))
        for i, arr in enumerate(got):
            np.testing.assert_array_equal(arr, data[f"{key}_{i}"], err_msg=key)
    for case in make_golden.index_cases():
        idx = make_golden.make_index(case, ref=False)
        arr = idx.arrays()
        for f in ("source_blocks", "target_node_idxs", "timestamps", "edge_idxs"):
            np.testing.assert_array_equal(arr[f], data[f"{case['key']}_{f}"], err_msg=case["key"])


def test_aggregation_oracle_small():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((7, 4))
    ids = np.array([0, 2, 2, 6, -1, 7, 2])
    out = O.segment_sum(x, ids, 7, mean=True)
    exp = np.zeros((7, 4))
    exp[0] = x[0]
    exp[2] = (x[1] + x[2] + x[6]) / 3
    exp[6] = x[3]
    np.testing.assert_allclose(out, exp)
    rowptr = np.array([0, 2, 2, 3])
    col = np.array([1, 3, 0])
    y = O.csr_spmm(rowptr, col, x, normalize=True)
    np.testing.assert_allclose(y[0], (x[1] + x[3]) / 2)
    np.testing.assert_allclose(y[1], 0)
    np.testing.assert_allclose(y[2], x[0])
