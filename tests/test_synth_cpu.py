"""The host restatement of the synthetic generators (oracle/synth_cpu.h) and
the reference-indexed sampler built from it in source ranges: the index
equals one CreateFromEdgeList call over the whole edge list, rows follow the
generator's row pointers, and samples agree with a sampler built from the
plain edge list."""

import numpy as np
import pytest

from oracle import oracle as O


def _plan(widths):
    from distributed_graph_flow_b200.sampling import config as cfg

    return cfg.explicit_plan("v", "e", widths)


@pytest.mark.parametrize("has_ts", [False, True])
@pytest.mark.parametrize("threads", [1, 3, 8])
def test_chunked_index_equals_single_call(has_ts, threads):
    n, E, seed = 4000, 50_000, 9
    ref = O.available(ref=True)
    rp, src, dst = O.synth_graph(n, n, E, 2.0, 600, seed)
    assert rp[0] == 0 and rp[-1] == E and np.all(np.diff(rp) >= 0)
    np.testing.assert_array_equal(src, np.repeat(np.arange(n), np.diff(rp)))
    assert dst.min() >= 0 and dst.max() < n
    ts = O.synth_uniform_int(E, 0, 50, seed, 11) if has_ts else None
    single = O.Index(np.stack([src, dst]), ts, num_source_nodes=n, num_target_nodes=n, ref=ref).arrays()
    s = O.OracleSampler.from_synth(n, E, 2.0, 600, seed, _plan([4, 3]), ts_range=(0, 50) if has_ts else None,
                                   ts_seed=seed, ref=ref, build_threads=threads)
    rp2, col2, ts2 = s.forward_csr()
    np.testing.assert_array_equal(rp2, single["source_blocks"])
    np.testing.assert_array_equal(rp2, rp)
    np.testing.assert_array_equal(col2, single["target_node_idxs"])
    if has_ts:
        np.testing.assert_array_equal(ts2, single["timestamps"])


def test_synth_sampler_matches_edge_list_sampler():
    from types import SimpleNamespace

    n, E, seed = 3000, 30_000, 4
    ref = O.available(ref=True)
    plan = _plan([5, 3])
    _, src, dst = O.synth_graph(n, n, E, 2.0, 300, seed)
    graph = SimpleNamespace(node_sets={"v": SimpleNamespace(num_nodes=n)},
                            edge_sets={"e": SimpleNamespace(adjacency=np.stack([src, dst]), features={})})
    schema = SimpleNamespace(node_sets={"v": None}, edge_sets={"e": None})
    a = O.OracleSampler(graph, plan, schema, debug_sampling=True, ref=ref)
    b = O.OracleSampler.from_synth(n, E, 2.0, 300, seed, plan, mode=O.MODE_FIRST, ref=ref, build_threads=4)
    seeds = O.synth_uniform_int(500, 0, n, 77, 5)
    for x, y in zip(a.sample_raw(seeds), b.sample_raw(seeds)):
        np.testing.assert_array_equal(x, y)


def test_uniform_and_features_are_partition_independent():
    a = O.synth_uniform_int(1000, -5, 17, 3, 2)
    assert a.min() >= -5 and a.max() < 17
    np.testing.assert_array_equal(a[:10], O.synth_uniform_int(10, -5, 17, 3, 2))
    f = O.synth_normal_features(100, 50, 7, 12, bf16=False)
    np.testing.assert_array_equal(f[10:20], O.synth_normal_features(110, 10, 7, 12, bf16=False))
    assert abs(float(f.mean())) < 0.2 and 0.8 < float(f.std()) < 1.2
    h = O.synth_normal_features(100, 50, 7, 12, bf16=True)
    # bf16 bits are fp32 rounded to nearest even.
    as_f = (h.astype(np.uint32) << 16).view(np.float32)
    assert np.all(np.abs(as_f - f) <= np.abs(f) * 2.0 ** -8 + 1e-30)
