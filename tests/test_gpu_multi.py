"""Multi-GPU halo feature exchange with the real kernels and NCCL.

The two-rank test runs only where at least two GPUs are visible: two spawned
ranks each hold a node-range partition of a feature table; rows gathered
through HaloFeatures (NCCL all-to-alls), PeerFeatures peer loads and the
PeerFeatures bulk exchange must equal the rows of the full table, and
ShardedSampler steps on every rank must produce features that match their
sampled node ids. The exchange kernels are also run for several ranks
emulated on one GPU (no waits between them: stream order is the barrier),
and the device barrier's bounded wait is run out on one GPU with a flag that
nothing sets.
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
        # Bulk exchange over the same partition (IPC-shared exchange buffers),
        # with the device barrier and with NCCL all-reduce barriers, direct
        # and through pipelined steps.
        cap_nodes = int(merged.node_ids.numel())
        for barrier in ("device", "nccl"):
            pe = driver.PeerFeatures(hi - lo, F, torch.bfloat16, rpr, spec.num_nodes, rank, world, dev,
                                     exchange_rows=max(20_000, cap_nodes), barrier=barrier)
            pe.table.copy_(full[lo:hi])
            pe.connect()
            if barrier == "device":
                # A replica of the 5,000 nodes with most in-edges (served locally).
                nbytes = pe.replicate(driver.hot_rows(index, 5000))
                assert nbytes > 0
            out.fill_(0)
            pe.gather_range(ids, _native.elem_ptr(bounds, 0), _native.elem_ptr(bounds, 1), 20_000, out)
            torch.cuda.synchronize()
            assert torch.equal(out[: len(sel)], exp), f"exchange gather rank {rank} ({barrier})"
            # With the NCCL barrier: two sampler handles, split sampling
            # calls, three steps in flight before the drain.
            cc_alt = None
            if barrier == "nccl":
                cc_alt = ext.create_device_sampler(plan, ["v"], [spec.num_nodes], ["e"], [index], [None], 0, seed=5)
            ss3 = driver.ShardedSampler(cc, pe, rank, world, cc_alt=cc_alt)
            steps = []
            for _ in range(3):
                steps.append(ss3.step_overlapped(seeds))
                if cc_alt is None:
                    ss3.drain()
            ss3.drain()
            torch.cuda.synchronize()
            for merged, feats, _ in steps:
                total = int(merged.node_offsets[-1].item())
                assert torch.equal(feats[:total], full[merged.node_ids[:total]]), f"exchange step {rank} ({barrier})"
            cc.check()
            if cc_alt is not None:
                cc_alt.check()
            pe.check()
            pe.close()
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


def _run_exchange(lib, W, rpr, N, row_bytes, parts, ids, bounds, caps, outs, slot, sh, hot=None, replica=None):
    """The three exchange launches for W ranks whose buffers all live on one
    GPU; issuing every rank's step before the next step's launches (one
    stream) is the barrier. hot / replica: a shared node -> replica-row map
    and replica table used by every emulated rank."""
    import ctypes

    import torch

    from distributed_graph_flow_b200 import _native

    need = ctypes.c_size_t()
    _native.check(lib.dgfx_exchange_buffer_size(W, slot, row_bytes, ctypes.byref(need)))
    dev = outs[0].device
    bufs = [torch.zeros(need.value, dtype=torch.uint8, device=dev) for _ in range(W)]
    ptrs = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device=dev)
    pos = [torch.empty((W + 1) * slot, dtype=torch.int32, device=dev) for _ in range(W)]
    rep_rows = 0 if replica is None else int(replica.shape[0])
    for r in range(W):
        _native.check(lib.dgfx_exchange_partition(
            _native.ptr(bufs[r]), W, slot, rpr, N, row_bytes, _native.ptr(ids[r]), _native.elem_ptr(bounds[r], 0),
            _native.elem_ptr(bounds[r], 1), caps[r], _native.ptr(hot), _native.ptr(pos[r]), _native.ptr(outs[r]), sh))
    for r in range(W):
        _native.check(lib.dgfx_exchange_serve(
            _native.ptr(ptrs), W, r, slot, rpr, row_bytes, _native.ptr(parts[r]), int(parts[r].shape[0]),
            _native.ptr(replica), rep_rows, _native.ptr(pos[r]), _native.ptr(outs[r]), sh))
    for r in range(W):
        _native.check(lib.dgfx_exchange_scatter(_native.ptr(ptrs), W, r, slot, row_bytes, _native.ptr(pos[r]),
                                                _native.ptr(outs[r]), sh))
    return bufs


def test_exchange_emulated_ranks(cuda):
    """Bulk peer exchange (dgfx_exchange_partition / serve / scatter) for 1, 3
    and 8 ranks emulated on one GPU: every rank's rows equal the full table's
    rows in request order, ids outside the graph give zero rows, rows past
    min(*end - *begin, max_rows) stay untouched, buffers are reusable, and a
    slot smaller than a rank's requests to one owner is reported (and the
    flag cleared) by dgfx_exchange_check."""
    from distributed_graph_flow_b200 import _native, synth

    lib = _native.lib()
    dev = torch.device("cuda", 0)
    sh = _native.stream_handle()
    N, F = 20_011, 64
    row_bytes = F * 2
    full = synth.normal_features(0, N, F, 4, torch.bfloat16, dev)
    rng = np.random.default_rng(11)
    for W in (1, 3, 8):
        rpr = -(-N // W)
        parts = [full[r * rpr:min(N, (r + 1) * rpr)].contiguous() for r in range(W)]
        sizes = [int(x) for x in rng.choice([0, 1, 33, 4000, 9000], W)]
        sizes[0] = 9000
        ids, bounds, caps, outs = [], [], [], []
        for r in range(W):
            lo = int(rng.integers(0, 5))
            n = sizes[r]
            ids.append(torch.from_numpy(rng.integers(-3, N + 3, n + lo + 4)).to(dev))
            bounds.append(torch.tensor([lo, lo + n], dtype=torch.int64, device=dev))
            caps.append(n if r % 2 == 0 else max(0, n - 5))  # odd ranks: max_rows below the bound count
            outs.append(torch.full((n + 2, F), 3.0, dtype=torch.bfloat16, device=dev))
        slot = max(max(caps), 1)
        for _rep in range(2):
            for o in outs:
                o.fill_(3.0)
            bufs = _run_exchange(lib, W, rpr, N, row_bytes, parts, ids, bounds, caps, outs, slot, sh)
            torch.cuda.synchronize()
            for r in range(W):
                lo, n = int(bounds[r][0]), caps[r]
                sel = ids[r][lo:lo + n]
                ok = (sel >= 0) & (sel < N)
                exp = torch.zeros((n, F), dtype=torch.bfloat16, device=dev)
                exp[ok] = full[sel[ok]]
                assert torch.equal(outs[r][:n], exp), f"W={W} rank {r}"
                assert bool((outs[r][n:] == 3.0).all()), f"W={W} rank {r}: rows past the end written"
                _native.check(lib.dgfx_exchange_check(_native.ptr(bufs[r]), W, sh))
        # With a replica of 30 % of the nodes (hot rows served locally).
        hot_ids = torch.from_numpy(rng.choice(N, N * 3 // 10, replace=False)).to(dev)
        hot = torch.full((N,), -1, dtype=torch.int32, device=dev)
        hot[hot_ids] = torch.arange(len(hot_ids), dtype=torch.int32, device=dev)
        replica = full[hot_ids].contiguous()
        for o in outs:
            o.fill_(3.0)
        bufs = _run_exchange(lib, W, rpr, N, row_bytes, parts, ids, bounds, caps, outs, slot, sh, hot, replica)
        torch.cuda.synchronize()
        for r in range(W):
            lo, n = int(bounds[r][0]), caps[r]
            sel = ids[r][lo:lo + n]
            ok = (sel >= 0) & (sel < N)
            exp = torch.zeros((n, F), dtype=torch.bfloat16, device=dev)
            exp[ok] = full[sel[ok]]
            assert torch.equal(outs[r][:n], exp), f"W={W} rank {r} with replica"
            _native.check(lib.dgfx_exchange_check(_native.ptr(bufs[r]), W, sh))
        if W > 1:
            small = 16
            bufs = _run_exchange(lib, W, rpr, N, row_bytes, parts, ids, bounds, caps, outs, small, sh)
            with pytest.raises(RuntimeError, match="overflowed"):
                _native.check(lib.dgfx_exchange_check(_native.ptr(bufs[0]), W, sh))
            _native.check(lib.dgfx_exchange_check(_native.ptr(bufs[0]), W, sh))  # flag cleared


def test_exchange_gather_one_rank(cuda):
    """dgfx_exchange_gather (partition, barrier, serve, barrier, scatter in one
    call) with one rank, whose barrier passes at once: the rows equal the
    table's in request order, with and without a replica table, on repeated
    calls with advancing epochs."""
    import ctypes

    from distributed_graph_flow_b200 import _native, synth

    lib = _native.lib()
    dev = torch.device("cuda", 0)
    sh = _native.stream_handle()
    N, F = 9001, 64
    row_bytes = F * 2
    full = synth.normal_features(0, N, F, 6, torch.bfloat16, dev)
    rng = np.random.default_rng(12)
    n = 5000
    ids = torch.from_numpy(rng.integers(-3, N + 3, n + 7)).to(dev)
    bounds = torch.tensor([3, 3 + n], dtype=torch.int64, device=dev)
    slot = n
    need = ctypes.c_size_t()
    _native.check(lib.dgfx_exchange_buffer_size(1, slot, row_bytes, ctypes.byref(need)))
    buf = torch.zeros(need.value, dtype=torch.uint8, device=dev)
    ptrs = torch.tensor([buf.data_ptr()], dtype=torch.int64, device=dev)
    pos = torch.empty(2 * slot, dtype=torch.int32, device=dev)
    sel = ids[3:3 + n]
    ok = (sel >= 0) & (sel < N)
    exp = torch.zeros((n, F), dtype=torch.bfloat16, device=dev)
    exp[ok] = full[sel[ok]]
    hot_ids = torch.from_numpy(rng.choice(N, N // 4, replace=False)).to(dev)
    hot = torch.full((N,), -1, dtype=torch.int32, device=dev)
    hot[hot_ids] = torch.arange(len(hot_ids), dtype=torch.int32, device=dev)
    replica = full[hot_ids].contiguous()
    epoch = 1
    for with_replica in (False, True, False):
        out = torch.full((n + 2, F), 3.0, dtype=torch.bfloat16, device=dev)
        _native.check(lib.dgfx_exchange_gather(
            _native.ptr(ptrs), _native.ptr(buf), 1, 0, slot, N, N, row_bytes, _native.ptr(ids),
            _native.elem_ptr(bounds, 0), _native.elem_ptr(bounds, 1), n,
            _native.ptr(hot) if with_replica else None, _native.ptr(pos), _native.ptr(full), N,
            _native.ptr(replica) if with_replica else None, int(replica.shape[0]) if with_replica else 0,
            _native.ptr(out), epoch, 2_000_000_000, sh))
        epoch += 2
        torch.cuda.synchronize()
        assert torch.equal(out[:n], exp), f"replica={with_replica}"
        assert bool((out[n:] == 3.0).all())
        _native.check(lib.dgfx_exchange_check(_native.ptr(buf), 1, sh))


def test_exchange_barrier_single_gpu(cuda):
    """dgfx_exchange_barrier on one GPU: with one rank it passes at once; with
    two ranks whose peer flag already holds the epoch it passes; with a peer
    flag that nothing sets, the bounded wait runs out and dgfx_exchange_check
    reports the timeout (and clears it) while the context stays usable."""
    import ctypes
    import time

    from distributed_graph_flow_b200 import _native

    lib = _native.lib()
    dev = torch.device("cuda", 0)
    sh = _native.stream_handle()
    need = ctypes.c_size_t()
    _native.check(lib.dgfx_exchange_buffer_size(2, 64, 128, ctypes.byref(need)))
    buf = torch.zeros(need.value, dtype=torch.uint8, device=dev)
    ptrs = torch.tensor([buf.data_ptr(), buf.data_ptr()], dtype=torch.int64, device=dev)
    one = torch.tensor([buf.data_ptr()], dtype=torch.int64, device=dev)
    for epoch in (1, 2, 3):
        _native.check(lib.dgfx_exchange_barrier(_native.ptr(one), 1, 0, epoch, 10**9, sh))
    _native.check(lib.dgfx_exchange_check(buf.data_ptr(), 1, sh))
    flags = buf[320:384].view(torch.int32)  # arrival epochs, one uint32 per rank (exchange buffer byte 320)
    flags[1] = 7
    _native.check(lib.dgfx_exchange_barrier(_native.ptr(ptrs), 2, 0, 7, 10**9, sh))
    _native.check(lib.dgfx_exchange_check(buf.data_ptr(), 2, sh))
    flags[1] = 0
    t0 = time.time()
    _native.check(lib.dgfx_exchange_barrier(_native.ptr(ptrs), 2, 0, 8, 2 * 10**6, sh))  # 2 ms bound
    with pytest.raises(ValueError, match="timed out"):
        _native.check(lib.dgfx_exchange_check(buf.data_ptr(), 2, sh))
    assert time.time() - t0 < 5.0
    _native.check(lib.dgfx_exchange_check(buf.data_ptr(), 2, sh))  # cleared
    assert torch.cuda.is_available() and int(flags[0].item()) == 8


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


def test_step_to_host_single_rank(cuda):
    """ShardedSampler.step_to_host (totals published by the GPU into pinned
    memory and polled, copies of exactly the batch's sizes on a copy stream)
    fills its host buffers with what step() returns on the device, over
    alternating HostBatch objects and several steps in flight."""
    from distributed_graph_flow_b200 import driver, synth
    from distributed_graph_flow_b200.sampling import _in_memory_sampler_ext as ext
    from distributed_graph_flow_b200.sampling import config as cfg

    dev = torch.device("cuda", 0)
    spec = synth.GraphSpec(20_000, 200_000, 2.0, 1500, seed=5)
    index, _, _ = synth.build_graph(spec, dev)
    plan = cfg.explicit_plan("v", "e", [6, 4])
    cc = ext.create_device_sampler(plan, ["v"], [spec.num_nodes], ["e"], [index], [None], 0, seed=3)
    F = 64
    pf = driver.PeerFeatures(spec.num_nodes, F, torch.bfloat16, spec.num_nodes, spec.num_nodes, 0, 1, dev)
    synth.normal_features(0, spec.num_nodes, F, 4, torch.bfloat16, dev, out=pf.table)
    pf.connect()
    a = driver.ShardedSampler(cc, pf, 0, 1)
    b = driver.ShardedSampler(cc, pf, 0, 1)
    seeds = synth.uniform_int(4 * 512, 0, spec.num_nodes, 9, 5, dev).view(4, 512)
    host_seeds = seeds.cpu().pin_memory()
    hosts = [driver.HostBatch(512 * cc.tree_size, F, torch.bfloat16) for _ in range(2)]
    got = []
    for i in range(4):
        out = a.step_to_host(host_seeds[i], hosts[i % 2])
        if i >= 1:  # the previous batch of the other buffer set is complete once waited for
            prev = hosts[(i - 1) % 2]
            prev.wait()
            got.append((prev.n, prev.m, prev.node_ids[:prev.n].clone(), prev.edge_src[:prev.m].clone(),
                        prev.edge_dst[:prev.m].clone(), prev.features[:prev.n].clone()))
    last = hosts[3 % 2]
    last.wait()
    got.append((last.n, last.m, last.node_ids[:last.n].clone(), last.edge_src[:last.m].clone(),
                last.edge_dst[:last.m].clone(), last.features[:last.n].clone()))
    for i in range(4):
        merged, feats, _ = b.step(seeds[i])
        torch.cuda.synchronize()
        n = int(merged.node_offsets[-1].item())
        m = int(merged.edge_offsets[-1].item())
        gn, gm, nodes, src, dst, fh = got[i]
        assert (gn, gm) == (n, m)
        assert torch.equal(nodes, merged.node_ids[:n].cpu())
        assert torch.equal(src, merged.edge_src[:m].cpu()) and torch.equal(dst, merged.edge_dst[:m].cpu())
        assert torch.equal(fh, feats[:n].cpu())
    cc.check()
    pf.close()


@pytest.mark.parametrize("mode", [0, 1])
def test_captured_steps_single_rank(cuda, mode):
    """CapturedSteps (pipelined steps of two alternating samplers with split
    calls, captured in one CUDA graph): every replayed step's features are the
    table's rows of its sampled nodes; in FIRST mode (mode 1) each step's
    batch equals an eager step() on the same seeds; in random mode (mode 0)
    consecutive replays draw new random streams."""
    from distributed_graph_flow_b200 import driver, synth
    from distributed_graph_flow_b200.sampling import _in_memory_sampler_ext as ext
    from distributed_graph_flow_b200.sampling import config as cfg

    dev = torch.device("cuda", 0)
    spec = synth.GraphSpec(30_000, 400_000, 2.0, 3000, seed=6)
    index, _, _ = synth.build_graph(spec, dev)
    plan = cfg.explicit_plan("v", "e", [8, 4, 3])
    mk = lambda sd: ext.create_device_sampler(plan, ["v"], [spec.num_nodes], ["e"], [index], [None], mode, seed=sd)
    F = 64
    pf = driver.PeerFeatures(spec.num_nodes, F, torch.bfloat16, spec.num_nodes, spec.num_nodes, 0, 1, dev)
    synth.normal_features(0, spec.num_nodes, F, 4, torch.bfloat16, dev, out=pf.table)
    pf.connect()
    ss = driver.ShardedSampler(mk(3), pf, 0, 1, cc_alt=mk(4))
    cap = driver.CapturedSteps(ss, 1024, steps=4)
    blocks = synth.uniform_int(3 * 4 * 1024, 0, spec.num_nodes, 21, 5, dev).view(3, 4, 1024)
    ref = driver.ShardedSampler(mk(3), pf, 0, 1)
    prev = None
    for r in range(3):
        cap.replay(blocks[r])
        torch.cuda.synchronize()
        got = []
        for k, (merged, feats, _) in enumerate(cap.outputs):
            n = int(merged.node_offsets[-1].item())
            m = int(merged.edge_offsets[-1].item())
            nodes = merged.node_ids[:n]
            assert torch.equal(feats[:n], pf.table[nodes]), f"replay {r} step {k}"
            assert torch.equal(nodes[merged.node_offsets[:-1][merged.node_offsets[:-1] < n]],
                               blocks[r, k][merged.node_offsets[:-1] < n])  # every sample starts with its seed
            got.append((nodes.clone(), merged.edge_src[:m].clone(), merged.edge_dst[:m].clone()))
            if mode == 1:
                e_merged, _, _ = ref.step(blocks[r, k])
                torch.cuda.synchronize()
                en = int(e_merged.node_offsets[-1].item())
                em = int(e_merged.edge_offsets[-1].item())
                assert (en, em) == (n, m)
                assert torch.equal(e_merged.node_ids[:en], nodes)
                assert torch.equal(e_merged.edge_src[:em], merged.edge_src[:m])
                assert torch.equal(e_merged.edge_dst[:em], merged.edge_dst[:m])
        if mode == 0 and prev is not None:
            # Same seeds as the previous replay? No: new seeds and new streams; at least
            # one step's batch must differ from what the previous replay produced.
            assert any(not torch.equal(a[0], b[0]) for a, b in zip(got, prev))
        prev = got
    ss.cc.check()
    ss.cc_alt.check()
    pf.close()
