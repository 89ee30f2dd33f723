"""GPU sampler parity: the reference's deterministic goldens, bit-exact
agreement with the oracle in the deterministic modes (first-k / oldest-k,
newest-k, fanout >= degree), and membership + time-constraint + chi-square
checks in uniform random mode."""

import numpy as np
import pytest

from golden import reference_cases as rc
from helpers import assert_sample_equal, random_hetero_graph, temporal_graph, toy_graph
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def sampling(cuda):
    from distributed_graph_flow_b200 import sampling

    return sampling


def _graph_arrays(g):
    return {n: g.node_sets[n].features.get("#idx") for n in g.node_sets}, {n: g.edge_sets[n].adjacency for n in g.edge_sets}


@pytest.mark.parametrize("case", rc.TOY_SAMPLE_CASES, ids=[c[0] for c in rc.TOY_SAMPLE_CASES])
def test_toy_goldens(sampling, case):
    name, conf, seeds, masked, mask_es, expected = case
    graph, schema = toy_graph()
    s = sampling.create_sampler(graph, sampling.SimpleSamplingConfig(**conf), schema, debug_sampling=True,
                                return_features=False, return_node_idxs=True, batch_size=5)
    out = s.sample(seeds)
    assert len(out) == len(expected)
    for g, (en, ee) in zip(out, expected):
        assert set(g.node_sets) == {"n1", "n2"}
        assert set(g.edge_sets) == {"e11", "e12", "e22"}
        nodes, edges = _graph_arrays(g)
        assert_sample_equal(nodes, edges, en, ee, name)
        for n, ns in g.node_sets.items():
            assert ns.num_nodes == len(ns.features["#idx"])
            assert ns.features["#idx"].dtype == np.int64
        for e in g.edge_sets.values():
            assert e.adjacency.dtype == np.int64 and e.adjacency.shape[0] == 2


def test_single_int_seed_returns_one_graph(sampling):
    graph, schema = toy_graph()
    s = sampling.create_sampler(graph, sampling.SimpleSamplingConfig(seed_nodeset="n1", num_hops=1, hop_width=2),
                                schema, debug_sampling=True, return_features=False, return_node_idxs=True, batch_size=5)
    g = s.sample(0)
    np.testing.assert_array_equal(g.node_sets["n1"].features["#idx"], [0, 1])


@pytest.mark.parametrize("case", rc.TOY_MASK_CASES, ids=[c[0] for c in rc.TOY_MASK_CASES])
def test_toy_masking(sampling, case):
    name, conf, seed, masked, mask_es, expected = case
    graph, schema = toy_graph()
    s = sampling.create_sampler(graph, sampling.SimpleSamplingConfig(**conf), schema, debug_sampling=True,
                                return_features=False, return_node_idxs=True, batch_size=5, edgeset_to_mask=mask_es)
    g = s.sample(seed, masked_edge_idxs=masked)
    for k, v in expected.items():
        np.testing.assert_array_equal(g.node_sets[k].features["#idx"], np.asarray(v, np.int64), err_msg=name)


@pytest.mark.parametrize("ts", sorted(rc.TEMPORAL_CASES))
def test_temporal_goldens_with_features(sampling, ts):
    graph, schema = temporal_graph()
    s = sampling.create_sampler(
        graph,
        sampling.SimpleSamplingConfig(seed_nodeset="n1", num_hops=2, hop_width=2, reverse=False, temporal_sampling=True),
        schema, return_features=True, return_node_idxs=True, batch_size=5, debug_sampling=True,
    )
    g = s.sample([0], seed_timestamps=[ts])[0]
    en, ee, exp_ts, exp_feat = rc.TEMPORAL_CASES[ts]
    nodes, edges = _graph_arrays(g)
    assert_sample_equal(nodes, edges, en, ee, f"ts={ts}")
    np.testing.assert_array_equal(g.node_sets["n1"].features["timestamp"], exp_ts)
    np.testing.assert_array_equal(g.node_sets["n1"].features["feat"], np.asarray(exp_feat, np.float32))
    assert g.node_sets["n1"].features["feat"].dtype == np.float32


def test_sampler_string_golden(sampling):
    graph, schema = toy_graph()
    plan = sampling.simple_sampling_config_to_sampling_plan(
        sampling.SimpleSamplingConfig(seed_nodeset="n1", num_hops=2), schema
    )
    s = sampling.create_sampler(graph, plan, schema, batch_size=5)
    assert str(s) == rc.TOY_SAMPLER_STR


def test_select_output(sampling):
    # in_memory_sampler_test.py:542-576.
    graph, schema = toy_graph()
    for rf in (True, False):
        for ri in (True, False):
            s = sampling.create_sampler(graph, sampling.SimpleSamplingConfig(seed_nodeset="n1", num_hops=0, hop_width=2),
                                        schema, return_features=rf, return_node_idxs=ri, batch_size=5)
            f = s.sample(0).node_sets["n1"].features
            assert ("f1" in f) == rf and ("#idx" in f) == ri
            if rf:
                np.testing.assert_array_equal(f["f1"], [10])
            if ri:
                np.testing.assert_array_equal(f["#idx"], [0])


def test_errors_match_reference(sampling):
    graph, schema = toy_graph()
    s = sampling.create_sampler(graph, sampling.SimpleSamplingConfig(seed_nodeset="n1", num_hops=1, hop_width=2),
                                schema, return_features=False, batch_size=5)
    with pytest.raises(ValueError, match=r"The source node idx 7 is out of bounds. Should be lower than 2"):
        s.sample([0, 7])
    with pytest.raises(ValueError, match="masked_edge_idxs provided but no edgeset to mask configured"):
        s.sample([0], masked_edge_idxs=[1])
    with pytest.raises(ValueError, match="seed_timestamps must have the same length"):
        s.sample([0, 1], seed_timestamps=[1])
    # Recovery: the sampler still works after an error.
    assert s.sample([1])[0].node_sets["n1"].num_nodes >= 1
    tg, tschema = temporal_graph()
    t = sampling.create_sampler(
        tg, sampling.SimpleSamplingConfig(seed_nodeset="n1", num_hops=2, hop_width=2, reverse=False,
                                          temporal_sampling=True), tschema, batch_size=5)
    with pytest.raises(ValueError, match="Cannot use SampleRandomUniform when timestamps are available"):
        t.sample([0])
    with pytest.raises(ValueError, match="Temporal filtering and edge masking cannot be used at the same time"):
        sampling.create_sampler(tg, sampling.SimpleSamplingConfig(seed_nodeset="n1", num_hops=1, temporal_sampling=True),
                                tschema, edgeset_to_mask="e1", batch_size=5)


def test_empty_batch(sampling):
    graph, schema = toy_graph()
    s = sampling.create_sampler(graph, sampling.SimpleSamplingConfig(seed_nodeset="n1", num_hops=2, hop_width=2),
                                schema, batch_size=5)
    assert s.sample(np.zeros(0, np.int64)) == []


CONFS = [
    dict(seed_nodeset="a", num_hops=2, hop_width=3),
    dict(seed_nodeset="a", num_hops=3, hop_width=2, with_replacement=True),
    dict(seed_nodeset="b", num_hops=2, hop_width=4, reverse=False),
    dict(seed_nodeset="c", num_hops=3, hop_width=2),
]


def _compare(sampling, graph, schema, conf, mode, temporal, seeds, ts=None, masks=None, mask_es=None, oracle_mode=None):
    plan = sampling.simple_sampling_config_to_sampling_plan(sampling.SimpleSamplingConfig(**conf), schema)
    s = sampling.create_sampler(graph, plan, schema, return_features=False, return_node_idxs=True, batch_size=64,
                                sampling_mode=mode, seed=5, edgeset_to_mask=mask_es)
    o = O.OracleSampler(graph, plan, schema, seed=5, edgeset_to_mask=mask_es,
                        edgeset_timestamp_features=plan.edgeset_timestamp_features,
                        mode=mode if oracle_mode is None else oracle_mode)
    got = s.sample(seeds, seed_timestamps=ts, masked_edge_idxs=masks)
    exp = o.sample(seeds, ts, masks)
    for i, (g, (en, ee)) in enumerate(zip(got, exp)):
        nodes, edges = _graph_arrays(g)
        assert_sample_equal(nodes, edges, en, ee, f"seed #{i} ({seeds[i]}) conf={conf} mode={mode}")


@pytest.mark.parametrize("conf", CONFS)
@pytest.mark.parametrize("temporal", [False, True])
@pytest.mark.parametrize("gseed", [0, 1, 2])
def test_first_mode_bit_exact(sampling, conf, temporal, gseed):
    graph, schema = random_hetero_graph(gseed, temporal=temporal)
    conf = dict(conf, temporal_sampling=temporal)
    rng = np.random.default_rng(gseed)
    n = graph.node_sets[conf["seed_nodeset"]].num_nodes
    seeds = np.concatenate([np.arange(n), rng.integers(0, n, 100)])
    ts = rng.integers(0, 55, len(seeds)) if temporal else None
    _compare(sampling, graph, schema, conf, sampling.MODE_FIRST, temporal, seeds, ts)


@pytest.mark.parametrize("conf", CONFS[:2])
def test_most_recent_mode_bit_exact(sampling, conf):
    graph, schema = random_hetero_graph(4, temporal=True)
    conf = dict(conf, temporal_sampling=True)
    rng = np.random.default_rng(9)
    n = graph.node_sets[conf["seed_nodeset"]].num_nodes
    seeds = rng.integers(0, n, 200)
    ts = rng.integers(0, 55, len(seeds))
    _compare(sampling, graph, schema, conf, sampling.MODE_MOST_RECENT, True, seeds, ts)


@pytest.mark.parametrize("temporal", [False, True])
def test_random_mode_wide_fanout_bit_exact(sampling, temporal):
    # hop_width >= every degree: the random sampler takes whole rows in
    # adjacency order, exactly like the reference.
    graph, schema = random_hetero_graph(5, temporal=temporal)
    conf = dict(seed_nodeset="a", num_hops=2, hop_width=10000, temporal_sampling=temporal)
    rng = np.random.default_rng(1)
    seeds = rng.integers(0, 40, 50)
    ts = rng.integers(0, 55, 50) if temporal else None
    _compare(sampling, graph, schema, conf, sampling.MODE_RANDOM, temporal, seeds, ts)


@pytest.mark.parametrize("mode", ["first", "random"])
def test_masking_vs_oracle(sampling, mode):
    graph, schema = random_hetero_graph(6, temporal=False)
    rng = np.random.default_rng(2)
    m = graph.edge_sets["ab"].adjacency.shape[1]
    seeds = rng.integers(0, 40, 300)
    masks = rng.integers(-1, m, 300)
    # Mask edges that actually leave each seed, so masking takes effect.
    adj = graph.edge_sets["ab"].adjacency
    for i, sd in enumerate(seeds):
        out = np.nonzero(adj[0] == sd)[0]
        if len(out) and i % 2 == 0:
            masks[i] = out[rng.integers(0, len(out))]
    if mode == "first":
        _compare(sampling, graph, schema, dict(seed_nodeset="a", num_hops=2, hop_width=3), sampling.MODE_FIRST, False,
                 seeds, None, masks, "ab")
    else:
        _compare(sampling, graph, schema, dict(seed_nodeset="a", num_hops=2, hop_width=1000), sampling.MODE_RANDOM,
                 False, seeds, None, masks, "ab")


def test_random_mode_membership_and_time(sampling):
    """Uniform random mode: every sampled edge exists, respects the cutoff,
    and per-(instance, edge) counts are min(k, valid degree)."""
    graph, schema = random_hetero_graph(7, temporal=True)
    conf = dict(seed_nodeset="a", num_hops=2, hop_width=3, temporal_sampling=True, reverse=True)
    plan = sampling.simple_sampling_config_to_sampling_plan(sampling.SimpleSamplingConfig(**conf), schema)
    s = sampling.create_sampler(graph, plan, schema, return_features=False, return_node_idxs=True, batch_size=64)
    rng = np.random.default_rng(3)
    seeds = rng.integers(0, 40, 500)
    ts = rng.integers(0, 55, 500)
    got = s.sample(seeds, seed_timestamps=ts)
    es_def = {n: (schema.edge_sets[n].source, schema.edge_sets[n].target) for n in schema.edge_sets}
    valid = {}
    for n, es in graph.edge_sets.items():
        a = es.adjacency
        t = es.features["timestamp"]
        valid[n] = (a, t)
    for i, g in enumerate(got):
        for name, es in g.edge_sets.items():
            src_ns, dst_ns = es_def[name]
            a, t = valid[name]
            src_ids = g.node_sets[src_ns].features["#idx"][es.adjacency[0]]
            dst_ids = g.node_sets[dst_ns].features["#idx"][es.adjacency[1]]
            for u, v in zip(src_ids, dst_ids):
                ok = np.nonzero((a[0] == u) & (a[1] == v) & (t <= ts[i]))[0]
                assert len(ok) > 0, f"edge {name} {u}->{v} absent or later than {ts[i]}"
        # Seed first, no duplicate node ids per node set.
        assert g.node_sets["a"].features["#idx"][0] == seeds[i]
        for ns in g.node_sets.values():
            ids = ns.features["#idx"]
            assert len(np.unique(ids)) == len(ids)


def test_random_mode_chi_square(sampling):
    """Inclusion frequency of each neighbour = k / n (chi-square, 1-hop)."""
    from scipy import stats

    from distributed_graph_flow_b200.data import in_memory_graph as img
    from distributed_graph_flow_b200.data import schema as sch

    n_nb, k, trials = 23, 5, 4000
    # Node 0 has neighbours 1..23; node 24 has a temporal prefix test below.
    src = np.zeros(n_nb, np.int64)
    dst = np.arange(1, n_nb + 1)
    graph = img.InMemoryGraph(node_sets={"v": img.InMemoryNodeSet(num_nodes=n_nb + 1)},
                              edge_sets={"e": img.InMemoryEdgeSet(adjacency=np.stack([src, dst]))})
    schema = sch.GraphSchema(node_sets={"v": sch.NodeSchema()}, edge_sets={"e": sch.EdgeSchema("v", "v")})
    plan = sampling.explicit_plan("v", "e", [k])
    s = sampling.create_sampler(graph, plan, schema, return_features=False, return_node_idxs=True, batch_size=trials,
                                seed=11)
    counts = np.zeros(n_nb + 1)
    sizes = set()
    for _ in range(2):
        for g in s.sample(np.zeros(trials // 2, np.int64)):
            ids = g.node_sets["v"].features["#idx"][1:]
            sizes.add(len(ids))
            counts[ids] += 1
    assert sizes == {k}
    obs = counts[1:]
    expected = np.full(n_nb, trials * k / n_nb)
    chi2 = ((obs - expected) ** 2 / expected).sum()
    p = stats.chi2.sf(chi2, n_nb - 1)
    assert p > 1e-4, f"chi2={chi2:.1f} p={p:.2e} counts={obs}"
    # Pairwise independence sanity: distinct calls give different samples.
    a = s.sample([0])[0].node_sets["v"].features["#idx"]
    b = s.sample([0])[0].node_sets["v"].features["#idx"]
    c = s.sample([0])[0].node_sets["v"].features["#idx"]
    assert not (np.array_equal(a, b) and np.array_equal(b, c))


def test_temporal_random_prefix_chi_square(sampling):
    """Temporal random mode samples uniformly from the valid prefix only."""
    from scipy import stats

    from distributed_graph_flow_b200.data import in_memory_graph as img
    from distributed_graph_flow_b200.data import schema as sch

    n_nb, k, trials, cutoff = 30, 4, 4000, 17
    src = np.zeros(n_nb, np.int64)
    dst = np.arange(1, n_nb + 1)
    ts = np.arange(n_nb, dtype=np.int64)  # neighbour j+1 has ts j
    ts_feat = sch.FeatureSchema(format=sch.FeatureFormat.INTEGER_64, is_creation_time=True)
    graph = img.InMemoryGraph(node_sets={"v": img.InMemoryNodeSet(num_nodes=n_nb + 1)},
                              edge_sets={"e": img.InMemoryEdgeSet(adjacency=np.stack([src, dst]),
                                                                  features={"timestamp": ts})})
    schema = sch.GraphSchema(node_sets={"v": sch.NodeSchema()},
                             edge_sets={"e": sch.EdgeSchema("v", "v", features={"timestamp": ts_feat})})
    plan = sampling.explicit_plan("v", "e", [k])
    plan.edgeset_timestamp_features = {"e": "timestamp"}
    s = sampling.create_sampler(graph, plan, schema, return_features=False, return_node_idxs=True, batch_size=trials)
    counts = np.zeros(n_nb + 1)
    for g in s.sample(np.zeros(trials, np.int64), seed_timestamps=np.full(trials, cutoff)):
        ids = g.node_sets["v"].features["#idx"][1:]
        assert len(ids) == k
        counts[ids] += 1
    valid = cutoff + 1  # ts 0..cutoff inclusive
    assert counts[valid + 1:].sum() == 0
    obs = counts[1 : valid + 1]
    expected = np.full(valid, trials * k / valid)
    p = stats.chi2.sf(((obs - expected) ** 2 / expected).sum(), valid - 1)
    assert p > 1e-4


def test_large_tree_global_memory_path(sampling):
    """A plan whose padded tree exceeds the shared-memory limit runs from the
    workspace and still matches the oracle (first mode)."""
    graph, schema = random_hetero_graph(8, temporal=False, sizes={"a": 60, "b": 30, "c": 9})
    conf = dict(seed_nodeset="a", num_hops=3, hop_width=8)
    plan = sampling.simple_sampling_config_to_sampling_plan(sampling.SimpleSamplingConfig(**conf), schema)
    s = sampling.create_sampler(graph, plan, schema, return_features=False, return_node_idxs=True, batch_size=8,
                                debug_sampling=True)
    assert s._cc_sampler.tree_size > 8192
    _compare(sampling, graph, schema, conf, sampling.MODE_FIRST, False, np.arange(20))


def _chain_graph(n_hop2, masked_row=False):
    """Node 0 -> node 1 (its only neighbour), node 1 -> nodes 2 .. n_hop2 + 1:
    every sample of seed 0 expands node 1 at the second hop."""
    from distributed_graph_flow_b200.data import in_memory_graph as img
    from distributed_graph_flow_b200.data import schema as sch

    src = np.concatenate([[0], np.ones(n_hop2, np.int64)])
    dst = np.concatenate([[1], np.arange(2, n_hop2 + 2)])
    graph = img.InMemoryGraph(node_sets={"v": img.InMemoryNodeSet(num_nodes=n_hop2 + 2)},
                              edge_sets={"e": img.InMemoryEdgeSet(adjacency=np.stack([src, dst]).astype(np.int64))})
    schema = sch.GraphSchema(node_sets={"v": sch.NodeSchema()}, edge_sets={"e": sch.EdgeSchema("v", "v")})
    return graph, schema


def _chi2_p(obs, expected):
    from scipy import stats

    return stats.chi2.sf(((obs - expected) ** 2 / expected).sum(), len(obs) - 1)


@pytest.mark.parametrize("with_replacement", [False, True])
def test_random_mode_second_hop_chi_square(sampling, with_replacement):
    """Second-hop draws: node 1 (reached from every seed) picks k of its n
    neighbours uniformly; inclusion frequency k / n each. With replacement
    the picked nodes are new local nodes but the draws are the same."""
    n_nb, k, trials = 19, 4, 4000
    graph, schema = _chain_graph(n_nb)
    plan = sampling.explicit_plan("v", "e", [3, k])
    plan.with_replacement = with_replacement
    s = sampling.create_sampler(graph, plan, schema, return_features=False, return_node_idxs=True, batch_size=1000,
                                seed=21)
    counts = np.zeros(n_nb + 2)
    for _ in range(trials // 1000):
        for g in s.sample(np.zeros(1000, np.int64)):
            ids = g.node_sets["v"].features["#idx"]
            assert ids[0] == 0 and ids[1] == 1
            hop2 = ids[2:]
            assert len(hop2) == k and len(np.unique(hop2)) == k
            counts[hop2] += 1
    assert counts[:2].sum() == 0
    p = _chi2_p(counts[2:], np.full(n_nb, trials * k / n_nb))
    assert p > 1e-4, f"p={p:.2e} counts={counts[2:]}"


def test_random_mode_masked_chi_square(sampling):
    """A masked edge is never drawn; the other n - 1 neighbours are drawn
    with frequency k / (n - 1) each."""
    from distributed_graph_flow_b200.data import in_memory_graph as img
    from distributed_graph_flow_b200.data import schema as sch

    n_nb, k, trials, masked = 17, 5, 4000, 6
    src = np.zeros(n_nb, np.int64)
    dst = np.arange(1, n_nb + 1)
    graph = img.InMemoryGraph(node_sets={"v": img.InMemoryNodeSet(num_nodes=n_nb + 1)},
                              edge_sets={"e": img.InMemoryEdgeSet(adjacency=np.stack([src, dst]))})
    schema = sch.GraphSchema(node_sets={"v": sch.NodeSchema()}, edge_sets={"e": sch.EdgeSchema("v", "v")})
    plan = sampling.explicit_plan("v", "e", [k])
    s = sampling.create_sampler(graph, plan, schema, return_features=False, return_node_idxs=True, batch_size=trials,
                                seed=3, edgeset_to_mask="e")
    counts = np.zeros(n_nb + 1)
    for g in s.sample(np.zeros(trials, np.int64), masked_edge_idxs=np.full(trials, masked)):
        ids = g.node_sets["v"].features["#idx"][1:]
        assert len(ids) == k
        counts[ids] += 1
    assert counts[dst[masked]] == 0
    keep = np.ones(n_nb + 1, bool)
    keep[0] = keep[dst[masked]] = False
    p = _chi2_p(counts[keep], np.full(n_nb - 1, trials * k / (n_nb - 1)))
    assert p > 1e-4, f"p={p:.2e}"


def test_is_deterministic(sampling):
    """Fixed sampler seed: every new sampler draws the same random-mode
    samples (in_memory_sampler_test.py:578-612); another seed draws others."""
    graph, schema = toy_graph()
    for batch_size in [1, 2]:
        for seed_idxs in [[0, 1], [1]]:
            for num_hops in [0, 1, 2]:
                for hop_width in [1, 2]:
                    truth = None
                    for _ in range(20):
                        plan = sampling.simple_sampling_config_to_sampling_plan(
                            sampling.SimpleSamplingConfig(seed_nodeset="n1", num_hops=num_hops, hop_width=hop_width),
                            schema)
                        s = sampling.create_sampler(graph, plan, schema, return_node_idxs=True, batch_size=batch_size,
                                                    seed=1234)
                        got = _graph_arrays_list(s.sample(seed_idxs))
                        if truth is None:
                            truth = got
                        else:
                            assert _same(truth, got)
    # Larger graph, random mode with draws: same seed same stream; other seed differs.
    graph, schema = random_hetero_graph(11, temporal=False)
    plan = sampling.simple_sampling_config_to_sampling_plan(
        sampling.SimpleSamplingConfig(seed_nodeset="a", num_hops=2, hop_width=2), schema)
    seeds = np.arange(40)
    runs = [_graph_arrays_list(sampling.create_sampler(graph, plan, schema, return_node_idxs=True, batch_size=40,
                                                       seed=sd).sample(seeds)) for sd in (1234, 1234, 99)]
    assert _same(runs[0], runs[1])
    assert not _same(runs[0], runs[2])


def _graph_arrays_list(graphs):
    return [_graph_arrays(g) for g in graphs]


def _same(a, b):
    if len(a) != len(b):
        return False
    for (na, ea), (nb, eb) in zip(a, b):
        if na.keys() != nb.keys() or ea.keys() != eb.keys():
            return False
        if any(not np.array_equal(na[k], nb[k]) for k in na) or any(not np.array_equal(ea[k], eb[k]) for k in ea):
            return False
    return True
