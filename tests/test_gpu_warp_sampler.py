"""The warp sampler (one warp per seed over occupied positions) against the
padded sampler (one CTA per seed over every position) and the oracle.

Both kernels draw from the same Philox counters, so their batches must be
identical in every mode, random included: small heterogeneous graphs
(temporal, masking, with replacement, several plans), trees larger than the
warp's capacity (seeds handed to the padded sampler), and the power-law
generator with the [15, 10, 5] plan. FIRST mode is also compared with the
oracle where the warp path is taken."""

import numpy as np
import pytest
import torch

from helpers import random_hetero_graph

pytestmark = pytest.mark.gpu


def _pair(sampling, graph, schema, conf, mode, mask_es=None):
    plan = sampling.simple_sampling_config_to_sampling_plan(sampling.SimpleSamplingConfig(**conf), schema)
    a = sampling.create_sampler(graph, plan, schema, return_features=False, return_node_idxs=True, batch_size=64,
                                sampling_mode=mode, seed=5, edgeset_to_mask=mask_es)
    b = sampling.create_sampler(graph, plan, schema, return_features=False, return_node_idxs=True, batch_size=64,
                                sampling_mode=mode, seed=5, edgeset_to_mask=mask_es)
    b._cc_sampler.set_kernel(1)
    return a, b


def _same_batches(a, b, seeds, ts=None, masks=None, calls=2):
    from distributed_graph_flow_b200.sampling import _in_memory_sampler_ext as ext

    dev = torch.device("cuda", 0)
    sd = torch.as_tensor(np.asarray(seeds, np.int64), device=dev)
    st = None if ts is None else torch.as_tensor(np.asarray(ts, np.int64), device=dev)
    mk = None if masks is None else torch.as_tensor(np.asarray(masks, np.int64), device=dev)
    for c in range(calls):
        x = ext.batch_to_host(a._cc_sampler.sample_merged(sd, st, mk, call_index=c))
        y = ext.batch_to_host(b._cc_sampler.sample_merged(sd, st, mk, call_index=c))
        for u, v in zip(x, y):
            np.testing.assert_array_equal(u, v)
    a._cc_sampler.check()
    b._cc_sampler.check()


CONFS = [
    dict(seed_nodeset="a", num_hops=2, hop_width=3),
    dict(seed_nodeset="a", num_hops=3, hop_width=2, with_replacement=True),
    dict(seed_nodeset="b", num_hops=2, hop_width=4, reverse=False),
    dict(seed_nodeset="c", num_hops=3, hop_width=2),
    dict(seed_nodeset="a", num_hops=2, hop_width=7),
]


@pytest.fixture(scope="module")
def sampling(cuda):
    from distributed_graph_flow_b200 import sampling

    return sampling


@pytest.mark.parametrize("conf", CONFS)
@pytest.mark.parametrize("temporal", [False, True])
@pytest.mark.parametrize("mode_name", ["MODE_RANDOM", "MODE_FIRST", "MODE_MOST_RECENT"])
def test_warp_equals_padded(sampling, conf, temporal, mode_name):
    if mode_name == "MODE_MOST_RECENT" and not temporal:
        pytest.skip("newest-k needs timestamps")
    graph, schema = random_hetero_graph(3, temporal=temporal)
    conf = dict(conf, temporal_sampling=temporal)
    a, b = _pair(sampling, graph, schema, conf, getattr(sampling, mode_name))
    assert a._cc_sampler.warp_capacity > 0 and b._cc_sampler.warp_capacity == 0
    rng = np.random.default_rng(4)
    n = graph.node_sets[conf["seed_nodeset"]].num_nodes
    seeds = np.concatenate([np.arange(n), rng.integers(0, n, 200)])
    ts = rng.integers(-3, 55, len(seeds)) if temporal else None
    _same_batches(a, b, seeds, ts)


@pytest.mark.parametrize("mode_name", ["MODE_RANDOM", "MODE_FIRST"])
def test_warp_equals_padded_masking(sampling, mode_name):
    graph, schema = random_hetero_graph(6, temporal=False)
    a, b = _pair(sampling, graph, schema, dict(seed_nodeset="a", num_hops=2, hop_width=3),
                 getattr(sampling, mode_name), mask_es="ab")
    rng = np.random.default_rng(2)
    m = graph.edge_sets["ab"].adjacency.shape[1]
    seeds = rng.integers(0, 40, 300)
    masks = rng.integers(-1, m, 300)
    _same_batches(a, b, seeds, None, masks)


def _tiers(sampling, graph, schema, conf, mode):
    """Samplers of one plan under kernel kinds 0 (warp, large-tree tier,
    padded), 1 (padded only) and 2 (warp, padded)."""
    out = []
    for kind in (0, 1, 2):
        plan = sampling.simple_sampling_config_to_sampling_plan(sampling.SimpleSamplingConfig(**conf), schema)
        x = sampling.create_sampler(graph, plan, schema, return_features=False, return_node_idxs=True,
                                    batch_size=64, sampling_mode=mode, seed=5)
        x._cc_sampler.set_kernel(kind)
        out.append(x)
    return out


@pytest.mark.parametrize("mode_name", ["MODE_RANDOM", "MODE_FIRST"])
def test_overflow_to_large_tree_tier(sampling, mode_name):
    """A three-hop plan without reverse edges (313 tree positions) on a
    dense graph: trees beyond the warp capacity (128 entries; 30 of the 60
    seeds in FIRST mode) are redone by the large-tree tier (512 entries)
    under kind 0 and by the padded sampler under kind 2; the batches of
    kinds 0, 1 and 2 are identical."""
    graph, schema = random_hetero_graph(8, temporal=False, sizes={"a": 60, "b": 30, "c": 9},
                                        edges={"ab": ("a", "b", 3000), "aa": ("a", "a", 2000),
                                               "bc": ("b", "c", 600), "ca": ("c", "a", 300)})
    a, b, c = _tiers(sampling, graph, schema, dict(seed_nodeset="a", num_hops=3, hop_width=4, reverse=False),
                     getattr(sampling, mode_name))
    assert a._cc_sampler.tree_size == 313 and a._cc_sampler.warp_capacity == 128
    assert a._cc_sampler.large_tree_capacity == 512 and c._cc_sampler.large_tree_capacity == 0
    assert b._cc_sampler.warp_capacity == 0 and c._cc_sampler.warp_capacity == 128
    seeds = np.arange(60)
    _same_batches(a, b, seeds)
    warp, padded = a._cc_sampler.kernel_stats()
    assert padded == 0 and warp == len(seeds)
    _same_batches(c, b, seeds)
    warp, padded = c._cc_sampler.kernel_stats()
    assert warp > 0 and padded > 0 and warp + padded == len(seeds)


@pytest.mark.parametrize("mode_name", ["MODE_RANDOM", "MODE_FIRST"])
@pytest.mark.parametrize("replace", [False, True])
def test_beyond_large_tree_tier(sampling, mode_name, replace):
    """A three-hop plan with reverse edges (thousands of tree positions, far
    beyond the large-tree tier's 512 entries): in FIRST mode 3 of the 200
    seeds fill at most 128 entries, 49 at most 512 and 148 more, so every
    tier runs; the batch equals the padded sampler's."""
    graph, schema = random_hetero_graph(9, temporal=False, sizes={"a": 200, "b": 90, "c": 30},
                                        edges={"ab": ("a", "b", 800), "aa": ("a", "a", 600),
                                               "bc": ("b", "c", 300), "ca": ("c", "a", 200)})
    a, b, _ = _tiers(sampling, graph, schema, dict(seed_nodeset="a", num_hops=3, hop_width=6,
                                                    with_replacement=replace), getattr(sampling, mode_name))
    assert a._cc_sampler.tree_size > 512 and a._cc_sampler.large_tree_capacity == 512
    seeds = np.concatenate([np.arange(200), np.arange(200)[::-1]])
    _same_batches(a, b, seeds)
    warp, padded = a._cc_sampler.kernel_stats()
    assert warp > 0 and padded > 0 and warp + padded == len(seeds)


def test_large_generator_warp_equals_padded(cuda):
    """The power-law generator at 0.5 % with the [15, 10, 5] plan, random and
    FIRST modes, 4096 seeds: about a sixth outgrow the warp's 128 entries and
    finish in the large-tree tier (512 entries), or in the padded sampler
    with that tier off; all three kernel kinds give the same batches."""
    import dataclasses

    from distributed_graph_flow_b200 import _native, synth
    from distributed_graph_flow_b200.sampling import _in_memory_sampler_ext as ext
    from distributed_graph_flow_b200.sampling import config as cfg

    dev = torch.device("cuda", 0)
    s = synth.LARGE_SHARDED
    spec = dataclasses.replace(s, num_nodes=int(s.num_nodes * 0.005), num_edges=int(s.num_edges * 0.005))
    index, _, _ = synth.build_graph(spec, dev)
    plan = cfg.explicit_plan("paper", "cites", [15, 10, 5])
    seeds = synth.uniform_int(4096, 0, spec.num_nodes, 77, 5, dev)
    for mode in (_native.MODE_RANDOM, _native.MODE_FIRST):
        a, b, c = (ext.create_device_sampler(plan, ["paper"], [spec.num_nodes], ["cites"], [index], [None], mode,
                                             seed=9) for _ in range(3))
        b.set_kernel(1)
        c.set_kernel(2)
        assert a.large_tree_capacity == 512
        for call in range(2):
            x = ext.batch_to_host(a.sample_merged(seeds, call_index=call))
            warp_a, padded_a = a.kernel_stats()
            z = ext.batch_to_host(c.sample_merged(seeds, call_index=call))
            warp, padded = c.kernel_stats()
            assert warp > 0 and padded > 0 and warp + padded == 4096  # trees of 129..916 entries: padded sampler
            assert warp_a + padded_a == 4096 and padded_a * 20 < padded  # large trees: the large-tree tier
            y = ext.batch_to_host(b.sample_merged(seeds, call_index=call))
            for u, v, w in zip(x, y, z):
                np.testing.assert_array_equal(u, v)
                np.testing.assert_array_equal(w, v)
        a.check()
        b.check()
        c.check()


def test_split_call_alternating_handles(cuda):
    """dgfx_sampler_sample_split: two samplers alternated, each call's tail
    (large-tree tier or padded sampler, scans, compaction) on a second
    stream, give the same
    batches as one sampler's plain calls with the same call indices, with
    several batches in flight; the outputs stay allocated until their tail
    ends (record_stream)."""
    import dataclasses

    from distributed_graph_flow_b200 import _native, synth
    from distributed_graph_flow_b200.sampling import _in_memory_sampler_ext as ext
    from distributed_graph_flow_b200.sampling import config as cfg

    dev = torch.device("cuda", 0)
    s = synth.LARGE_SHARDED
    spec = dataclasses.replace(s, num_nodes=int(s.num_nodes * 0.005), num_edges=int(s.num_edges * 0.005))
    index, _, _ = synth.build_graph(spec, dev)
    plan = cfg.explicit_plan("paper", "cites", [15, 10, 5])
    seeds = synth.uniform_int(6 * 2048, 0, spec.num_nodes, 78, 5, dev).view(6, 2048)

    def make():
        return ext.create_device_sampler(plan, ["paper"], [spec.num_nodes], ["cites"], [index], [None],
                                         _native.MODE_RANDOM, seed=9)

    ref, a, b = make(), make(), make()
    b.set_kernel(2)  # b's tails run the padded sampler, a's the large-tree tier
    tail = torch.cuda.Stream(device=dev)
    main = torch.cuda.current_stream(dev)
    got = []
    for i in range(6):
        h = a if i % 2 == 0 else b
        got.append(h.sample_merged(seeds[i], call_index=i, check=False, tail_stream=tail))
    main.wait_stream(tail)
    a.check()
    b.check()
    warp, padded = b.kernel_stats()
    assert warp > 0 and padded > 0
    warp_a, padded_a = a.kernel_stats()
    assert warp_a + padded_a == 2048 and padded_a * 20 < padded
    for i in range(6):
        x = ext.batch_to_host(got[i])
        y = ext.batch_to_host(ref.sample_merged(seeds[i], call_index=i))
        for u, v in zip(x, y):
            np.testing.assert_array_equal(u, v)
    # A plain call after split calls on the same sampler waits for the tail.
    x = ext.batch_to_host(a.sample_merged(seeds[0], call_index=0))
    for u, v in zip(x, ext.batch_to_host(got[0])):
        np.testing.assert_array_equal(u, v)


def test_split_call_status_after_tail(cuda):
    """Status reads after a split call (check, kernel_stats) wait for the
    call's tail on the stream they are given, so the large-tree tier's counts
    are included without the caller joining the tail stream first."""
    import dataclasses

    from distributed_graph_flow_b200 import _native, synth
    from distributed_graph_flow_b200.sampling import _in_memory_sampler_ext as ext
    from distributed_graph_flow_b200.sampling import config as cfg

    dev = torch.device("cuda", 0)
    s = synth.LARGE_SHARDED
    spec = dataclasses.replace(s, num_nodes=int(s.num_nodes * 0.005), num_edges=int(s.num_edges * 0.005))
    index, _, _ = synth.build_graph(spec, dev)
    plan = cfg.explicit_plan("paper", "cites", [15, 10, 5])
    seeds = synth.uniform_int(4096, 0, spec.num_nodes, 79, 5, dev)
    a = ext.create_device_sampler(plan, ["paper"], [spec.num_nodes], ["cites"], [index], [None],
                                  _native.MODE_RANDOM, seed=4)
    tail = torch.cuda.Stream(device=dev)
    for call in range(3):
        a.sample_merged(seeds, call_index=call, check=False, tail_stream=tail)
        warp, padded = a.kernel_stats()  # the current stream, not joined to the tail
        assert warp + padded == 4096
    a.sample_merged(seeds, call_index=5, check=False, tail_stream=tail)
    a.check()
