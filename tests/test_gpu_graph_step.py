"""CUDA-graph-captured sampling steps and long time-sorted rows.

* CapturedSampleStep: replays equal eager calls in the deterministic mode
  (oldest-first), draw a fresh random stream on every replay in random mode
  (the device call index advances), and gather the right feature rows.
* Rows of hundreds to thousands of edges with many ties: the cooperative
  9-ary cutoff search gives the oracle's node and edge sets in FIRST and
  MOST_RECENT modes for cutoffs below, inside and above every row.
"""

import numpy as np
import pytest
import torch

from helpers import assert_sample_equal

pytestmark = pytest.mark.gpu


def _temporal_graph(dev, n=2000, e=60_000, seed=1, max_ts=50):
    from distributed_graph_flow_b200 import synth

    spec = synth.GraphSpec(n, e, 1.6, 4000, seed=seed, ts_range=(0, max_ts))
    index, ts, edges = synth.build_graph(spec, dev, keep_edges=True)
    return spec, index, ts, edges


def _sampler(index, n, mode, seed=7, fanout=(10, 5)):
    from distributed_graph_flow_b200.sampling import _in_memory_sampler_ext as ext
    from distributed_graph_flow_b200.sampling import config as cfg

    plan = cfg.explicit_plan("v", "e", list(fanout))
    return ext.create_device_sampler(plan, ["v"], [n], ["e"], [index], [None], mode, seed=seed,
                                     has_temporal=True), plan


def test_captured_step_matches_eager(cuda):
    from distributed_graph_flow_b200 import _native
    from distributed_graph_flow_b200.sampling import _in_memory_sampler_ext as ext

    dev = torch.device("cuda", 0)
    spec, index, _, _ = _temporal_graph(dev)
    table = torch.randn((spec.num_nodes, 64), device=dev)
    eager, _ = _sampler(index, spec.num_nodes, _native.MODE_FIRST)
    graph_s, _ = _sampler(index, spec.num_nodes, _native.MODE_FIRST)
    step = ext.CapturedSampleStep(graph_s, 256, True, table)
    rng = np.random.default_rng(0)
    for _ in range(3):
        seeds = torch.from_numpy(rng.integers(0, spec.num_nodes, 256)).to(dev)
        sts = torch.from_numpy(rng.integers(0, 55, 256)).to(dev)
        batch, rows = step.run(seeds, sts)
        step.wait()
        exp = eager.sample_merged(seeds, sts)
        g_nodes, g_off, g_edges, g_eoff = ext.batch_to_host(batch)
        e_nodes, e_off, e_edges, e_eoff = ext.batch_to_host(exp)
        np.testing.assert_array_equal(g_off, e_off)
        np.testing.assert_array_equal(g_nodes, e_nodes)
        np.testing.assert_array_equal(g_eoff, e_eoff)
        np.testing.assert_array_equal(g_edges, e_edges)
        n = int(g_off[-1])
        assert torch.equal(rows[:n], table[batch.node_ids[:n]])
    # Host inputs go through the same copies; bad inputs are refused.
    batch, _ = step.run(seeds.cpu(), sts.cpu())
    torch.cuda.current_stream().synchronize()
    np.testing.assert_array_equal(ext.batch_to_host(batch)[0], ext.batch_to_host(eager.sample_merged(seeds, sts))[0])
    with pytest.raises(ValueError, match="contiguous int64"):
        step.run(seeds.to(torch.int32), sts)
    with pytest.raises(ValueError, match="seed_ts is required"):
        step.run(seeds)
    graph_s.check()


@pytest.mark.parametrize("serial", [False, True])
def test_captured_step_aggregate_matches_separate_calls(cuda, serial):
    """CapturedSampleStep(aggregate=True) (gather + mean aggregation inside
    the graph, two samplers forked or serial) gives the rows and means of
    eager gather and mean calls on the eager FIRST-mode batches."""
    from distributed_graph_flow_b200 import _native, aggregation
    from distributed_graph_flow_b200.sampling import _in_memory_sampler_ext as ext

    dev = torch.device("cuda", 0)
    spec, index, _, _ = _temporal_graph(dev)
    table = torch.randn((spec.num_nodes, 128), device=dev)
    eager, _ = _sampler(index, spec.num_nodes, _native.MODE_FIRST)
    graph_s = [_sampler(index, spec.num_nodes, _native.MODE_FIRST)[0] for _ in range(2)]
    step = ext.CapturedSampleStep(graph_s, 256, True, table, aggregate=True, serial=serial)
    rng = np.random.default_rng(3)
    seeds = torch.from_numpy(rng.integers(0, spec.num_nodes, (2, 256))).to(dev)
    sts = torch.from_numpy(rng.integers(0, 55, (2, 256))).to(dev)
    for _ in range(2):
        outs = step.run(seeds, sts)
        torch.cuda.current_stream().synchronize()
        for k, (batch, rows, means) in enumerate(outs):
            exp = eager.sample_merged(seeds[k], sts[k])
            n = int(exp.node_offsets[-1])
            np.testing.assert_array_equal(ext.batch_to_host(batch)[0], ext.batch_to_host(exp)[0])
            exp_rows = aggregation.gather_rows(table, exp.node_ids)
            assert torch.equal(rows[:n], exp_rows[:n])
            assert torch.equal(means[:n], aggregation.batch_mean_aggregate(exp, exp_rows)[:n])
    for smp in graph_s:
        smp.check()


def test_captured_step_random_stream_advances(cuda):
    from distributed_graph_flow_b200 import _native
    from distributed_graph_flow_b200.sampling import _in_memory_sampler_ext as ext

    dev = torch.device("cuda", 0)
    spec, index, _, (src, dst) = _temporal_graph(dev)
    s, _ = _sampler(index, spec.num_nodes, _native.MODE_RANDOM)
    step = ext.CapturedSampleStep(s, 512, True)
    seeds = torch.arange(512, dtype=torch.int64, device=dev) % spec.num_nodes
    sts = torch.full((512,), 60, dtype=torch.int64, device=dev)  # no cutoff
    outs = []
    for _ in range(2):
        batch, _ = step.run(seeds, sts)
        step.wait()
        outs.append(ext.batch_to_host(batch))
    s.check()
    assert not (np.array_equal(outs[0][0], outs[1][0]) and np.array_equal(outs[0][2], outs[1][2])), \
        "two replays drew the same random stream"
    edge_set = set(zip(src.cpu().numpy().tolist(), dst.cpu().numpy().tolist()))
    for nodes, off, edges, eoff in outs:
        for i in range(512):
            ids = nodes[off[i]:off[i + 1]]
            for a, b in edges[:, eoff[i]:eoff[i + 1]].T:
                assert (int(ids[a]), int(ids[b])) in edge_set


@pytest.mark.parametrize("mode_name", ["MODE_FIRST", "MODE_MOST_RECENT"])
def test_long_rows_cutoff_matches_oracle(cuda, mode_name):
    from distributed_graph_flow_b200 import _native
    from distributed_graph_flow_b200.sampling import _in_memory_sampler_ext as ext
    from oracle import oracle as O

    dev = torch.device("cuda", 0)
    # 300 nodes, 150,000 edges: rows of up to 4000 edges, timestamps in [0, 20) (many ties).
    spec, index, _, _ = _temporal_graph(dev, n=300, e=150_000, seed=3, max_ts=20)
    mode = getattr(_native, mode_name)
    s, plan = _sampler(index, spec.num_nodes, mode, fanout=(6, 3))
    rng = np.random.default_rng(1)
    seeds = rng.integers(0, spec.num_nodes, 400)
    sts = rng.integers(-2, 23, 400)
    merged = s.sample_merged(torch.from_numpy(seeds).to(dev), torch.from_numpy(sts).to(dev))
    got = ext.export_graphs(merged)
    csr = {"e": (index.rowptr.cpu().numpy(), index.col.cpu().numpy(), index.ts.cpu().numpy())}
    o = O.OracleSampler.from_csr([spec.num_nodes], ["v"], ["e"], csr, plan, mode=getattr(O, mode_name), seed=5,
                                 temporal=True)
    exp = o.sample(seeds, sts)
    for i, (gr, (en, ee)) in enumerate(zip(got, exp)):
        nodes = {n: gr.node_sets[n].features["#idx"] for n in gr.node_sets}
        edges = {n: gr.edge_sets[n].adjacency for n in gr.edge_sets}
        assert_sample_equal(nodes, edges, en, ee, f"seed #{i} ({seeds[i]}, cutoff {sts[i]})")


def test_captured_multi_batch_step(cuda):
    """Three samplers forked inside one graph: each batch equals its eager
    counterpart (oldest-first mode), rows included."""
    from distributed_graph_flow_b200 import _native
    from distributed_graph_flow_b200.sampling import _in_memory_sampler_ext as ext

    dev = torch.device("cuda", 0)
    spec, index, _, _ = _temporal_graph(dev)
    table = torch.randn((spec.num_nodes, 32), device=dev)
    K, B = 3, 200
    samplers = [_sampler(index, spec.num_nodes, _native.MODE_FIRST, seed=k)[0] for k in range(K)]
    eager, _ = _sampler(index, spec.num_nodes, _native.MODE_FIRST)
    step = ext.CapturedSampleStep(samplers, B, True, table)
    rng = np.random.default_rng(2)
    for _ in range(2):
        seeds = torch.from_numpy(rng.integers(0, spec.num_nodes, (K, B))).to(dev)
        sts = torch.from_numpy(rng.integers(0, 55, (K, B))).to(dev)
        outs = step.run(seeds, sts)
        step.wait()
        assert len(outs) == K
        for k, (batch, rows) in enumerate(outs):
            exp = eager.sample_merged(seeds[k], sts[k])
            got_h, exp_h = ext.batch_to_host(batch), ext.batch_to_host(exp)
            for a, b in zip(got_h, exp_h):
                np.testing.assert_array_equal(a, b)
            n = int(got_h[1][-1])
            assert torch.equal(rows[:n], table[batch.node_ids[:n]])
    for smp in samplers:
        smp.check()
