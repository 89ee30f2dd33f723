"""Parity on the benchmarked workloads, against an oracle that shares nothing
with the device path.

The oracle side generates each graph on the host (the generator's
restatement, oracle/synth_cpu.h) and indexes it with the reference's own
AdjacencyIndex::CreateFromEdgeList (oracle/_ref, when built); the device side
generates the same graph with the synth kernels and indexes it with the
device CSR build. Then:

* the device index equals the reference's index array for array;
* FIRST mode (the reference's debug_sampling: first-k / oldest-k under a
  cutoff) and the newest-k extension give the oracle's merged batch bit for
  bit: the 169,343-node temporal graph at full size (fanout [10, 5], 1024
  seeds, cutoff = seed timestamp), the 1.6B-edge generator at 1.5 % with
  the full [15, 10, 5] plan (916 padded positions, 8192 seeds), and the
  heterogeneous temporal graph at 5 % (fanout [15, 10] over every edge type
  in both directions, 4096 seeds, cutoff = seed year);
* random mode on the same graphs: every sampled edge exists (and respects
  the cutoff), node ids are unique per sample, the seed comes first, and a
  seed with a valid neighbour has an edge out of it (exact draw counts and
  their distribution are checked on constructed rows in
  test_gpu_sampler.py).
"""

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

REF = O.available(ref=True)


def _cores():
    import os

    try:
        return max(1, len(os.sched_getaffinity(0)))
    except Exception:  # noqa: BLE001
        return os.cpu_count() or 1


oracle_merged = O.merged_layout


def assert_batch_equal(batch, expected, what):
    from distributed_graph_flow_b200.sampling import _in_memory_sampler_ext as ext

    got = ext.batch_to_host(batch)
    for name, g, e in zip(("node offsets", "node ids", "edge offsets"), (got[1], got[0], got[3]),
                          (expected[1], expected[0], expected[3])):
        if not np.array_equal(g, e):
            bad = np.nonzero(g[: min(len(g), len(e))] != e[: min(len(g), len(e))])[0]
            raise AssertionError(f"{what}: {name} differ (len {len(g)} vs {len(e)}; first at {bad[:5]})")
    np.testing.assert_array_equal(got[2], expected[2], err_msg=f"{what}: edges differ")


def _device_homogeneous(spec, dev):
    from distributed_graph_flow_b200 import synth

    index, ts, _ = synth.build_graph(spec, dev)
    return index


def _check_index(index, oracle_sampler):
    rp, col, ts = oracle_sampler.forward_csr()
    np.testing.assert_array_equal(index.rowptr.cpu().numpy(), rp)
    np.testing.assert_array_equal(index.col.cpu().numpy().astype(np.int64), col)
    if ts is not None:
        np.testing.assert_array_equal(index.ts.cpu().numpy(), ts)


def _sampler(plan, n, index, mode, temporal):
    from distributed_graph_flow_b200.sampling import _in_memory_sampler_ext as ext

    return ext.create_device_sampler(plan, [plan.root.nodeset], [n], [plan.root.children[0].edgeset], [index], [None],
                                     mode, seed=5, has_temporal=temporal)


# ---------------------------------------------------------------------------
# Temporal 169,343-node graph at full size: fanout [10, 5], 1024 seeds.
# ---------------------------------------------------------------------------
@pytest.fixture(scope="module")
def temporal_full(cuda):
    from distributed_graph_flow_b200 import synth
    from distributed_graph_flow_b200.sampling import config as cfg

    dev = torch.device("cuda", 0)
    spec = synth.TEMPORAL_169K
    index = _device_homogeneous(spec, dev)
    node_ts = synth.uniform_int(spec.num_nodes, 0, 50, spec.seed, 12, dev)
    seeds = synth.uniform_int(1024, 0, spec.num_nodes, 21, 9, dev)
    plan = cfg.explicit_plan("v", "e", [10, 5])
    return dev, spec, index, node_ts, seeds, plan


@pytest.mark.parametrize("mode_name", ["MODE_FIRST", "MODE_MOST_RECENT"])
def test_temporal_169k_full_size_bit_exact(temporal_full, mode_name):
    from distributed_graph_flow_b200 import _native

    dev, spec, index, node_ts, seeds, plan = temporal_full
    o = O.OracleSampler.from_synth(spec.num_nodes, spec.num_edges, spec.alpha, spec.max_degree, spec.seed, plan,
                                   ts_range=spec.ts_range, ts_seed=spec.seed, ts_stream=11,
                                   mode=getattr(O, mode_name), ref=REF,
                                   build_threads=_cores())
    _check_index(index, o)
    sts = node_ts[seeds]
    s = _sampler(plan, spec.num_nodes, index, getattr(_native, mode_name), True)
    for call in range(2):  # two batches: the cutoff is each seed's own timestamp
        sd = seeds if call == 0 else seeds.flip(0)
        st = sts if call == 0 else sts.flip(0)
        batch = s.sample_merged(sd, st)
        exp = oracle_merged(*o.sample_raw(sd.cpu().numpy(), st.cpu().numpy(), threads=_cores()))
        assert_batch_equal(batch, exp, f"169K temporal {mode_name} batch {call}")
    s.check()


def test_temporal_169k_random_membership(temporal_full):
    from distributed_graph_flow_b200 import _native
    from distributed_graph_flow_b200.sampling import _in_memory_sampler_ext as ext

    dev, spec, index, node_ts, seeds, plan = temporal_full
    s = _sampler(plan, spec.num_nodes, index, _native.MODE_RANDOM, True)
    sts = node_ts[seeds]
    batch = s.sample_merged(seeds, sts)
    _check_random_batch(ext.batch_to_host(batch), index, seeds.cpu().numpy(), sts.cpu().numpy(), [10, 5])
    s.check()


def _check_random_batch(host, index, seeds, sts, widths):
    """Membership, cutoff, uniqueness and seed-first checks of a homogeneous
    random-mode batch."""
    nodes, off, edges, eoff = host
    rp = index.rowptr.cpu().numpy()
    col = index.col.cpu().numpy().astype(np.int64)
    ts = None if index.ts is None else index.ts.cpu().numpy()
    B = len(seeds)
    for i in range(B):
        ids = nodes[off[i]:off[i + 1]]
        assert ids[0] == seeds[i]
        assert len(np.unique(ids)) == len(ids)
        e = edges[:, eoff[i]:eoff[i + 1]]
        u, v = ids[e[0]], ids[e[1]]
        for a, b in zip(u, v):
            row = col[rp[a]:rp[a + 1]]
            hit = row == b
            if ts is not None:
                hit &= ts[rp[a]:rp[a + 1]] <= sts[i]
            assert hit.any(), f"seed #{i}: edge {a}->{b} absent or after the cutoff"
        deg = rp[seeds[i] + 1] - rp[seeds[i]]
        if ts is not None:
            deg = int(np.count_nonzero(ts[rp[seeds[i]]:rp[seeds[i] + 1]] <= sts[i]))
        # A seed with a valid neighbour has an edge out of it.
        if deg > 0:
            assert np.count_nonzero(e[0] == 0) >= 1


# ---------------------------------------------------------------------------
# The 1.6B-edge generator at 1.5 %, full [15, 10, 5] plan, 8192 seeds.
# ---------------------------------------------------------------------------
@pytest.fixture(scope="module")
def large_scaled(cuda):
    import dataclasses

    from distributed_graph_flow_b200 import synth
    from distributed_graph_flow_b200.sampling import config as cfg

    dev = torch.device("cuda", 0)
    s = synth.LARGE_SHARDED
    spec = dataclasses.replace(s, num_nodes=int(s.num_nodes * 0.015), num_edges=int(s.num_edges * 0.015))
    index = _device_homogeneous(spec, dev)
    plan = cfg.explicit_plan("paper", "cites", [15, 10, 5])
    seeds = synth.uniform_int(8192, 0, spec.num_nodes, 77, 5, dev)
    return dev, spec, index, plan, seeds


def test_large_scaled_first_mode_bit_exact(large_scaled):
    from distributed_graph_flow_b200 import _native

    dev, spec, index, plan, seeds = large_scaled
    o = O.OracleSampler.from_synth(spec.num_nodes, spec.num_edges, spec.alpha, spec.max_degree, spec.seed, plan,
                                   mode=O.MODE_FIRST, ref=REF, build_threads=_cores())
    _check_index(index, o)
    s = _sampler(plan, spec.num_nodes, index, _native.MODE_FIRST, False)
    assert s.tree_size == 916
    batch = s.sample_merged(seeds)
    exp = oracle_merged(*o.sample_raw(seeds.cpu().numpy(), threads=_cores()))
    assert_batch_equal(batch, exp, "large 1.5% [15,10,5] FIRST")
    s.check()


def test_large_scaled_random_membership(large_scaled):
    from distributed_graph_flow_b200 import _native
    from distributed_graph_flow_b200.sampling import _in_memory_sampler_ext as ext

    dev, spec, index, plan, seeds = large_scaled
    s = _sampler(plan, spec.num_nodes, index, _native.MODE_RANDOM, False)
    sd = seeds[:2048]
    batch = s.sample_merged(sd)
    _check_random_batch(ext.batch_to_host(batch), index, sd.cpu().numpy(), None, [15, 10, 5])
    s.check()


# ---------------------------------------------------------------------------
# Heterogeneous temporal graph at 5 %: both directions of every edge type,
# fanout [15, 10], 4096 A seeds, cutoff = seed year. The oracle indexes the
# device-generated edge lists with CreateFromEdgeList (not the device CSR).
# ---------------------------------------------------------------------------
def test_hetero_temporal_5pct_first_mode_bit_exact(cuda):
    from types import SimpleNamespace

    from distributed_graph_flow_b200 import _native, synth
    from distributed_graph_flow_b200.sampling import _in_memory_sampler_ext as ext

    dev = torch.device("cuda", 0)
    spec = synth.scaled_hetero(synth.HETERO_TEMPORAL, 0.05)
    g = synth.build_hetero_graph(spec, dev)
    plan = synth.hetero_plan(spec, "A", [15, 10])
    edge_sets, ets = {}, {}
    for name, (src, dst, ts) in g.edges.items():
        feats = {}
        if ts is not None:
            feats["ts"] = ts.cpu().numpy()
            ets[name] = "ts"
        edge_sets[name] = SimpleNamespace(adjacency=np.stack([src.cpu().numpy(), dst.cpu().numpy()]), features=feats)
    graph = SimpleNamespace(node_sets={n: SimpleNamespace(num_nodes=c) for n, c in zip(g.nodeset_names, g.num_nodes)},
                            edge_sets=edge_sets)
    schema = SimpleNamespace(node_sets={n: None for n in g.nodeset_names},
                             edge_sets={n: None for n in g.edgeset_names})
    o = O.OracleSampler(graph, plan, schema, edgeset_timestamp_features=ets, mode=O.MODE_FIRST, ref=REF)
    s = ext.create_device_sampler(plan, g.nodeset_names, g.num_nodes, g.edgeset_names, g.fwd, g.bwd,
                                  _native.MODE_FIRST, seed=5, has_temporal=True)
    a = g.nodeset_names.index("A")
    seeds = synth.uniform_int(4096, 0, g.num_nodes[a], 23, 9, dev)
    sts = g.node_ts["A"][seeds]
    batch = s.sample_merged(seeds, sts)
    exp = oracle_merged(*o.sample_raw(seeds.cpu().numpy(), sts.cpu().numpy(), threads=_cores()))
    assert_batch_equal(batch, exp, "hetero 5% [15,10] FIRST")
    s.check()
