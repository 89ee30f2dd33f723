"""Multi-GPU halo feature exchange with the real kernels and NCCL.

Runs only where at least two GPUs are visible: two spawned ranks each hold a
node-range partition of a feature table; rows gathered through
HaloFeatures (partition by owner, NCCL all-to-alls, local gather, scatter)
must equal the rows of the full table, and ShardedSampler steps on every rank
must produce features that match their sampled node ids.
"""

import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        from distributed_graph_flow_b200 import driver, synth
        from distributed_graph_flow_b200.sampling import _in_memory_sampler_ext as ext
        from distributed_graph_flow_b200.sampling import config as cfg

        spec = synth.GraphSpec(50_000, 600_000, 2.0, 2000, seed=3)
        F = 64
        full = synth.normal_features(0, spec.num_nodes, F, 9, torch.bfloat16, dev)
        rpr = -(-spec.num_nodes // world)
        lo, hi = rank * rpr, min(spec.num_nodes, (rank + 1) * rpr)
        hf = driver.HaloFeatures(full[lo:hi].contiguous(), rpr, rank, world)
        rng = np.random.default_rng(rank)
        for n in (0, 7, 10_000):
            ids = torch.from_numpy(rng.integers(0, spec.num_nodes, n)).to(dev)
            got = hf.gather(ids)
            assert torch.equal(got, full[ids]), f"halo gather rank {rank} n {n}"
        index, _, _ = synth.build_graph(spec, dev)
        plan = cfg.explicit_plan("v", "e", [5, 3])
        cc = ext.create_device_sampler(plan, ["v"], [spec.num_nodes], ["e"], [index], [None], 0, seed=5)
        ss = driver.ShardedSampler(cc, hf, rank, world)
        seeds = torch.from_numpy(rng.integers(0, spec.num_nodes, 512)).to(dev)
        for _ in range(2):
            merged, feats, total = ss.step(seeds)
            cc.check()
            assert total == int(merged.node_offsets[-1].item())
            assert torch.equal(feats[:total], full[merged.node_ids[:total]])
        # Peer-load gather over the same partition.
        pf = driver.PeerFeatures(hi - lo, F, torch.bfloat16, rpr, spec.num_nodes, rank, world, dev)
        pf.table.copy_(full[lo:hi])
        pf.connect()
        ids = torch.from_numpy(rng.integers(-3, spec.num_nodes + 3, 20_000)).to(dev)
        bounds = torch.tensor([5, 19_000], dtype=torch.int64, device=dev)
        out = torch.zeros((20_000, F), dtype=torch.bfloat16, device=dev)
        from distributed_graph_flow_b200 import _native

        pf.gather_range(ids, _native.elem_ptr(bounds, 0), _native.elem_ptr(bounds, 1), 20_000, out)
        sel = ids[5:19_000]
        ok = (sel >= 0) & (sel < spec.num_nodes)
        exp = torch.zeros((len(sel), F), dtype=torch.bfloat16, device=dev)
        exp[ok] = full[sel[ok]]
        assert torch.equal(out[: len(sel)], exp), f"p2p gather rank {rank}"
        ss2 = driver.ShardedSampler(cc, pf, rank, world)
        merged, feats, _ = ss2.step(seeds)
        cc.check()
        total = int(merged.node_offsets[-1].item())
        assert torch.equal(feats[:total], full[merged.node_ids[:total]])
        pf.close()
        q.put((rank, "ok"))
    except Exception as exc:  # noqa: BLE001
        q.put((rank, repr(exc)))
    finally:
        dist.destroy_process_group()


def test_peer_gather_single_rank(cuda):
    """The peer-load gather kernel with one partition (no IPC): rows in request
    order, zero rows for ids outside the graph, bounds read on the device."""
    from distributed_graph_flow_b200 import _native, driver, synth

    dev = torch.device("cuda", 0)
    n, F = 5000, 128
    pf = driver.PeerFeatures(n, F, torch.bfloat16, n, n, 0, 1, dev)
    synth.normal_features(0, n, F, 4, torch.bfloat16, dev, out=pf.table)
    pf.connect()
    full = pf.table.clone()
    ids = torch.tensor([7, -1, 4999, 5000, 0, 7], dtype=torch.int64, device=dev)
    bounds = torch.tensor([0, 6], dtype=torch.int64, device=dev)
    out = torch.full((8, F), 3.0, dtype=torch.bfloat16, device=dev)
    pf.gather_range(ids, _native.elem_ptr(bounds, 0), _native.elem_ptr(bounds, 1), 8, out)
    assert torch.equal(out[0], full[7]) and torch.equal(out[2], full[4999]) and torch.equal(out[4], full[0])
    assert torch.count_nonzero(out[1]) == 0 and torch.count_nonzero(out[3]) == 0
    assert torch.equal(out[6], torch.full((F,), 3.0, dtype=torch.bfloat16, device=dev))  # past *end: untouched
    pf.close()


def test_halo_exchange_two_gpus(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    assert res == {0: "ok", 1: "ok"}, res
