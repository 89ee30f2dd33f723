"""Single-box multi-GPU sampling driver.

Replaces the reference's Beam driver (dgf/src/sampling/
beam_semi_distributed_sampler_v2.py:51-158, 200-268): one process per GPU,
seed batches sharded across ranks, the graph topology replicated in every
GPU's HBM, node features node-range partitioned (rank r owns rows
[r * rows_per_rank, (r + 1) * rows_per_rank)). The only exchange is the halo
feature gather, replacing the Beam CoGroupByKey feature join
(beam_semi_distributed_sampler_v2.py:271-387). Three interchangeable paths:
  * HaloFeatures: requested ids are stably partitioned by owner
    (dgfx_halo_partition); counts, ids and rows move in NCCL all-to-alls;
    owners gather locally (dgfx_gather_rows_local) and received rows are
    scattered back to request order (dgfx_scatter_rows). Needs host-side
    counts (one device-to-host read per step).
  * PeerFeatures, peer loads: one kernel reads every row from its owner's
    partition through CUDA IPC mappings (dgfx_gather_rows_p2p).
  * PeerFeatures, bulk exchange: the same all-to-all done by three kernels
    over the IPC mappings (dgfx_exchange_*) with device-side counts and a
    device barrier; NVLink traffic moves in contiguous runs. The default at
    more than one rank.
With one rank every path degenerates to a local gather.
"""

from __future__ import annotations

import ctypes
from typing import Optional

from distributed_graph_flow_b200 import _native


class HaloFeatures:
    """Node features partitioned by node range across the process group."""

    def __init__(self, local_table, rows_per_rank: int, rank: int, world: int, group=None):
        self.table = local_table  # [local_rows, F] on this rank's GPU
        self.rows_per_rank = int(rows_per_rank)
        self.rank = int(rank)
        self.world = int(world)
        self.group = group
        self.row_bytes = local_table.element_size() * int(local_table.shape[1])
        if self.row_bytes % 16:
            raise ValueError("feature rows must be a multiple of 16 bytes")
        self._ws = None

    def _workspace(self, n: int):
        torch = _native.require_cuda()
        need = ctypes.c_size_t()
        _native.check(_native.lib().dgfx_halo_partition_workspace_size(n, self.world, ctypes.byref(need)))
        if self._ws is None or self._ws.numel() < need.value:
            self._ws = torch.empty(need.value, dtype=torch.uint8, device=self.table.device)
        return self._ws, need.value

    def gather(self, ids, out=None, stream=None):
        """Rows for int64 ids (global node ids) in request order."""
        torch = _native.require_cuda()
        import torch.distributed as dist

        n = int(ids.numel())
        dev = self.table.device
        F = int(self.table.shape[1])
        if out is None:
            out = torch.empty((max(n, 1), F), dtype=self.table.dtype, device=dev)[:n]
        sh = _native.stream_handle(stream)
        lib = _native.lib()
        if self.world == 1:
            _native.check(lib.dgfx_gather_rows_local(_native.ptr(self.table), int(self.table.shape[0]), self.row_bytes,
                                                     _native.ptr(ids), n, 0, _native.ptr(out), sh))
            return out
        sorted_ids = torch.empty(max(n, 1), dtype=torch.int64, device=dev)
        perm = torch.empty(max(n, 1), dtype=torch.int32, device=dev)
        send_counts = torch.empty(self.world, dtype=torch.int64, device=dev)
        ws, nbytes = self._workspace(n)
        _native.check(lib.dgfx_halo_partition(_native.ptr(ids), n, self.rows_per_rank, self.world,
                                              _native.ptr(sorted_ids), _native.ptr(perm), _native.ptr(send_counts),
                                              _native.ptr(ws), nbytes, sh))
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        sc = send_counts.tolist()
        rc = recv_counts.tolist()
        n_recv = int(sum(rc))
        recv_ids = torch.empty(max(n_recv, 1), dtype=torch.int64, device=dev)[:n_recv]
        dist.all_to_all_single(recv_ids, sorted_ids[:n], rc, sc, group=self.group)
        rows = torch.empty((max(n_recv, 1), F), dtype=self.table.dtype, device=dev)[:n_recv]
        _native.check(lib.dgfx_gather_rows_local(_native.ptr(self.table), int(self.table.shape[0]), self.row_bytes,
                                                 _native.ptr(recv_ids), n_recv, self.rank * self.rows_per_rank,
                                                 _native.ptr(rows), sh))
        back = torch.empty((max(n, 1), F), dtype=self.table.dtype, device=dev)[:n]
        dist.all_to_all_single(back, rows, sc, rc, group=self.group)
        _native.check(lib.dgfx_scatter_rows(_native.ptr(back), n, self.row_bytes, _native.ptr(perm), _native.ptr(out), sh))
        return out


class DeviceBuffer:
    """A cudaMalloc'd allocation (dgfx_device_alloc) seen by torch through
    __cuda_array_interface__. Needed for CUDA IPC, which shares whole
    allocations, not sub-blocks of torch's caching allocator."""

    def __init__(self, nbytes: int, device):
        self.device = device
        ptr = ctypes.c_void_p()
        _native.check(_native.lib().dgfx_device_alloc(int(nbytes), ctypes.byref(ptr)))
        self.ptr = int(ptr.value)
        self.nbytes = int(nbytes)
        self.__cuda_array_interface__ = {"shape": (max(1, self.nbytes),), "typestr": "|u1",
                                         "data": (self.ptr, False), "version": 3}

    def tensor(self, shape, dtype):
        torch = _native.require_cuda()
        raw = torch.as_tensor(self, device=self.device)
        n = 1
        for s in shape:
            n *= int(s)
        return raw[: n * torch.empty(0, dtype=dtype).element_size()].view(dtype).view(*shape)

    def free(self):
        if self.ptr:
            _native.check(_native.lib().dgfx_device_free(self.ptr))
            self.ptr = 0


class PeerFeatures:
    """Node-range-partitioned features gathered from peer memory.

    Each rank's partition lives in its own allocation whose CUDA IPC handle is
    shared with the other ranks once (all_gather of the 64-byte handles), so
    every rank holds pointers to all partitions. Two gather paths:

    * peer loads (``exchange_rows=0``): one kernel (dgfx_gather_rows_p2p)
      fetches any row from its owner over NVLink;
    * bulk exchange (``exchange_rows > 0``, more than one rank): requests are
      bucketed by owner; owners gather their rows locally and write them into
      each requester's inbox; requesters scatter the inbox into request order
      (dgfx_exchange_*), so every byte crossing NVLink moves in contiguous
      runs. Three stream-ordered launches separated by a device barrier over
      peer flags (``barrier="device"``, bounded wait, no host round trip) or
      a one-element NCCL all-reduce (``barrier="nccl"``). ``exchange_rows`` is
      the capacity of one (requester, owner) slot; the batch capacity never
      overflows it. ``check()`` reports overflow and barrier timeouts.

    Call ``close()`` on every rank before the process group is destroyed.
    """

    def __init__(self, local_rows: int, dim: int, dtype, rows_per_rank: int, num_nodes: int, rank: int,
                 world: int, device, group=None, exchange_rows: int = 0, barrier: str = "device",
                 barrier_timeout_s: float = 10.0):
        torch = _native.require_cuda()
        self.rank, self.world, self.group = int(rank), int(world), group
        self.rows_per_rank, self.num_nodes, self.dim = int(rows_per_rank), int(num_nodes), int(dim)
        self.local_rows = int(local_rows)
        self.dtype = dtype
        self.device = device
        self.row_bytes = torch.empty(0, dtype=dtype).element_size() * self.dim
        if self.row_bytes % 16:
            raise ValueError("feature rows must be a multiple of 16 bytes")
        self.exchange_rows = int(exchange_rows) if self.world > 1 else 0
        if barrier not in ("device", "nccl"):
            raise ValueError(f"barrier must be 'device' or 'nccl', got {barrier!r}")
        self.barrier = barrier
        self.barrier_timeout_ns = int(barrier_timeout_s * 1e9)
        self.buffer = DeviceBuffer(max(1, local_rows) * self.row_bytes, device)
        self.table = self.buffer.tensor((local_rows, self.dim), dtype)
        self._peers = []
        self._ptrs = None
        self._ex = None
        self._replica = None
        self._hot_slot = None

    def _share(self, local_ptr: int):
        """All ranks' pointers to the allocation each rank passes (collective)."""
        torch = _native.require_cuda()
        lib = _native.lib()
        ptrs = [0] * self.world
        ptrs[self.rank] = local_ptr
        if self.world > 1:
            import torch.distributed as dist

            h = (ctypes.c_uint8 * 64)()
            _native.check(lib.dgfx_ipc_get_handle(local_ptr, ctypes.cast(h, ctypes.c_void_p)))
            mine = torch.tensor(list(bytes(h)), dtype=torch.uint8, device=self.device)
            allh = torch.empty((self.world, 64), dtype=torch.uint8, device=self.device)
            dist.all_gather_into_tensor(allh, mine, group=self.group)
            allh = allh.cpu().numpy()
            for r in range(self.world):
                if r == self.rank:
                    continue
                buf = (ctypes.c_uint8 * 64)(*allh[r].tolist())
                p = ctypes.c_void_p()
                _native.check(lib.dgfx_ipc_open(ctypes.cast(buf, ctypes.c_void_p), ctypes.byref(p)))
                ptrs[r] = int(p.value)
                self._peers.append(int(p.value))
        return torch.tensor(ptrs, dtype=torch.int64, device=self.device)

    def connect(self):
        """Exchanges IPC handles (collective over the group). Call after the
        local partition is filled."""
        torch = _native.require_cuda()
        self._ptrs = self._share(self.buffer.ptr)
        if self.exchange_rows > 0:
            need = ctypes.c_size_t()
            _native.check(_native.lib().dgfx_exchange_buffer_size(self.world, self.exchange_rows, self.row_bytes,
                                                                  ctypes.byref(need)))
            self._ex = DeviceBuffer(need.value, self.device)
            self._ex.tensor((need.value,), torch.uint8).zero_()
            self._ex_ptrs = self._share(self._ex.ptr)
            self._req_pos = torch.empty((self.world + 1) * self.exchange_rows, dtype=torch.int32, device=self.device)
            self._bar = torch.zeros(1, dtype=torch.int32, device=self.device)
        torch.cuda.synchronize(self.device)
        return self

    def gather_range(self, ids, begin_ptr: int, end_ptr: int, max_rows: int, out, stream=None, stage_events=None):
        """out[i] = feature row of ids[*begin + i] for i < min(*end - *begin, max_rows).
        With a list ``stage_events`` (bulk exchange), CUDA events recorded on
        the stream after each stage (partition, barrier, serve, barrier,
        scatter) are appended to it."""
        if self._ex is None:
            _native.check(_native.lib().dgfx_gather_rows_p2p(
                _native.ptr(self._ptrs), self.world, self.rows_per_rank, self.num_nodes, self.row_bytes,
                _native.ptr(ids), begin_ptr, end_ptr, int(max_rows), _native.ptr(out), _native.stream_handle(stream)))
            return out
        torch = _native.require_cuda()

        s = torch.cuda.current_stream(self.device) if stream is None else stream
        sh = int(s.cuda_stream)
        lib = _native.lib()
        rep_rows = 0 if self._replica is None else int(self._replica.shape[0])
        if stage_events is None and self.barrier == "device":
            # One native call for the five launches (less host time per step);
            # barrier epochs from the device counter (epoch 0), as in
            # _group_barrier, so the launches can be captured in a CUDA graph.
            epoch = 0
            _native.check(lib.dgfx_exchange_gather(
                _native.ptr(self._ex_ptrs), self._ex.ptr, self.world, self.rank, self.exchange_rows,
                self.rows_per_rank, self.num_nodes, self.row_bytes, _native.ptr(ids), begin_ptr, end_ptr,
                int(max_rows), _native.ptr(self._hot_slot), _native.ptr(self._req_pos), self.buffer.ptr,
                self.local_rows, _native.ptr(self._replica), rep_rows, _native.ptr(out), epoch,
                self.barrier_timeout_ns, sh))
            return out

        def mark():
            if stage_events is not None:
                e = torch.cuda.Event(enable_timing=True)
                e.record(s)
                stage_events.append(e)

        mark()
        _native.check(lib.dgfx_exchange_partition(
            self._ex.ptr, self.world, self.exchange_rows, self.rows_per_rank, self.num_nodes, self.row_bytes,
            _native.ptr(ids), begin_ptr, end_ptr, int(max_rows), _native.ptr(self._hot_slot),
            _native.ptr(self._req_pos), _native.ptr(out), sh))
        mark()
        self._group_barrier(s)
        mark()
        _native.check(lib.dgfx_exchange_serve(
            _native.ptr(self._ex_ptrs), self.world, self.rank, self.exchange_rows, self.rows_per_rank, self.row_bytes,
            self.buffer.ptr, self.local_rows, _native.ptr(self._replica), rep_rows, _native.ptr(self._req_pos),
            _native.ptr(out), sh))
        mark()
        self._group_barrier(s)
        mark()
        _native.check(lib.dgfx_exchange_scatter(
            _native.ptr(self._ex_ptrs), self.world, self.rank, self.exchange_rows, self.row_bytes,
            _native.ptr(self._req_pos), _native.ptr(out), sh))
        mark()
        return out

    def replicate(self, hot_ids):
        """Keeps a read-only copy of the rows of ``hot_ids`` (int64 CUDA
        tensor, identical on every rank) in this GPU's HBM; requests for them
        are then served locally instead of crossing NVLink (bulk exchange
        only). Collective: every rank calls it with the same ids. Returns
        the bytes the copy takes on this GPU."""
        torch = _native.require_cuda()
        if self._ex is None:
            return 0  # one rank, or peer loads: nothing crosses an exchange
        n = int(hot_ids.numel())
        self._hot_slot = None
        self._replica = None
        replica = torch.empty((max(n, 1), self.dim), dtype=self.dtype, device=self.device)[:n]
        bounds = torch.zeros(2, dtype=torch.int64, device=self.device)
        for lo in range(0, n, self.exchange_rows):
            hi = min(n, lo + self.exchange_rows)
            bounds[0], bounds[1] = lo, hi
            self.gather_range(hot_ids, _native.elem_ptr(bounds, 0), _native.elem_ptr(bounds, 1), hi - lo,
                              replica[lo:hi])
        hot_slot = torch.full((self.num_nodes,), -1, dtype=torch.int32, device=self.device)
        hot_slot[hot_ids] = torch.arange(n, dtype=torch.int32, device=self.device)
        torch.cuda.synchronize(self.device)
        self.check()
        self._replica, self._hot_slot = replica, hot_slot
        return n * self.row_bytes + self.num_nodes * 4

    def _group_barrier(self, s):
        """Stream-ordered barrier over the group (every rank calls it in the same order)."""
        if self.barrier == "device":
            # Epoch 0: the kernel advances this rank's device-side epoch, so
            # a captured graph replays correctly (every barrier uses it).
            _native.check(_native.lib().dgfx_exchange_barrier(_native.ptr(self._ex_ptrs), self.world, self.rank,
                                                              0, self.barrier_timeout_ns, int(s.cuda_stream)))
        else:
            torch = _native.require_cuda()
            import torch.distributed as dist

            with torch.cuda.stream(s):
                dist.all_reduce(self._bar, op=dist.ReduceOp.MAX, group=self.group)

    def check(self, stream=None):
        """Raises if an exchange slot overflowed or a barrier wait timed out
        since the last check (synchronises)."""
        if self._ex is not None:
            _native.check(_native.lib().dgfx_exchange_check(self._ex.ptr, self.world, _native.stream_handle(stream)))

    def close(self):
        """Unmaps the peers' allocations and frees this rank's (collective)."""
        torch = _native.require_cuda()
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            import torch.distributed as dist

            dist.barrier(group=self.group)
            for p in self._peers:
                _native.check(_native.lib().dgfx_ipc_close(p))
            self._peers = []
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
        self.table = None
        self._replica = None
        self._hot_slot = None
        self.buffer.free()
        if self._ex is not None:
            self._ex.free()
            self._ex = None


def hot_rows(index, count: int):
    """The ``count`` nodes with the most in-edges of a forward adjacency
    index (int64 CUDA tensor, ties broken by node id): the rows a sampler
    walking that index requests most often. Deterministic, so every rank
    computes the same set."""
    torch = _native.require_cuda()
    num = int(index.num_dst)  # column ids of a forward index are target node ids
    deg = torch.bincount(index.col, minlength=num)
    order = torch.sort(deg, descending=True, stable=True).indices
    return order[: max(0, min(int(count), num))].to(torch.int64).contiguous()


class CapturedSteps:
    """`steps` pipelined steps of a ShardedSampler (``step_overlapped``)
    captured in one CUDA graph, for callers whose host would otherwise issue
    the launches slower than the GPU runs them. The seeds of the steps live
    in ``seeds`` ([steps, batch] int64 on the GPU; ``replay(block)`` copies a
    block in first); each replay overwrites ``outputs`` (a list of (merged
    batch, features, None) per step). Random streams come from the samplers'
    device counters (every replay draws new ones); exchange barriers take
    their epochs on the device, so at N > 1 every rank replays its own graph
    in step. Needs the peer-feature store (``PeerFeatures``)."""

    def __init__(self, sharded: "ShardedSampler", batch: int, steps: int = 4):
        torch = _native.require_cuda()
        if not isinstance(sharded.features, PeerFeatures):
            raise ValueError("CapturedSteps needs PeerFeatures")
        dev = sharded.features.device
        self.sharded = sharded
        self.steps = int(steps)
        self.seeds = torch.zeros((self.steps, int(batch)), dtype=torch.int64, device=dev)
        # Eager pass: streams, events, workspaces and size caches exist before capture.
        for k in range(self.steps):
            sharded.step_overlapped(self.seeds[k], call_index=_native.CALL_INDEX_DEVICE)
        sharded.drain()
        for h in (sharded.cc, sharded.cc_alt):
            if h is not None:
                h.check()  # synchronises and settles pending split tails
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        cs = torch.cuda.Stream(device=dev)
        cs.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.graph(self.graph, stream=cs):
            self.outputs = [sharded.step_overlapped(self.seeds[k], call_index=_native.CALL_INDEX_DEVICE)
                            for k in range(self.steps)]
            sharded.drain()
        torch.cuda.synchronize(dev)

    def replay(self, seeds_block=None):
        """Runs the captured steps (on the current stream) after copying
        `seeds_block` ([steps, batch]) into ``seeds`` if given."""
        if seeds_block is not None:
            self.seeds.copy_(seeds_block, non_blocking=True)
        self.graph.replay()


class HostBatch:
    """Pinned host buffers for one merged batch, filled by
    ``ShardedSampler.step_to_host``: node ids, edge endpoints (local ids)
    and the feature rows of every sampled node, sized for `node_capacity`
    nodes and edges (the sampler's batch capacity). ``n`` / ``m`` are the
    batch's node and edge counts; the arrays hold them once ``ready()``."""

    def __init__(self, node_capacity: int, feat_dim: int, feat_dtype):
        torch = _native.require_cuda()
        cap = int(node_capacity)
        self.node_ids = torch.empty(cap, dtype=torch.int64, pin_memory=True)
        self.edge_src = torch.empty(cap, dtype=torch.int64, pin_memory=True)
        self.edge_dst = torch.empty(cap, dtype=torch.int64, pin_memory=True)
        self.features = torch.empty((cap, int(feat_dim)), dtype=feat_dtype, pin_memory=True)
        self.totals = torch.full((2,), -1, dtype=torch.int64, pin_memory=True)  # written by the GPU
        self.n = self.m = 0
        self.done = None  # CUDA event recorded after the copies

    def ready(self) -> bool:
        return self.done is None or self.done.query()

    def wait(self):
        if self.done is not None:
            self.done.synchronize()


class ShardedSampler:
    """Per-rank sampler over the replicated topology plus halo features.

    ``step(seeds)`` samples this rank's seed shard (int64 device tensor) and
    returns (merged batch, features of every sampled node in merged order,
    number of sampled nodes)."""

    def __init__(self, cc_sampler, features: Optional[HaloFeatures], rank: int, world: int, cc_alt=None):
        self.cc = cc_sampler
        # A second sampler over the same index and plan (same seed): with it,
        # step_overlapped alternates the two so that one call's tail overlaps
        # the next call's first kernel (each sampler owns one workspace).
        self.cc_alt = cc_alt
        self.features = features
        self.rank = rank
        self.world = world
        self._calls = 0
        self.gather_stream = None
        self.tail_stream = None

    def step_overlapped(self, seeds, seed_ts=None, call_index=None):
        """Like step(), but the feature gather runs on a second stream so it
        overlaps the sampling of the next call (the sampler is latency-bound,
        the gather bandwidth-bound), and with ``cc_alt`` each sampling call
        is split (the large-tree kernel, scans and compaction on a tail
        stream) so that it overlaps the next call's first kernel. Results are
        valid once the caller's stream has waited on ``gather_stream``
        (``drain()``). Batches equal step()'s for the same call order.
        ``call_index=_native.CALL_INDEX_DEVICE`` draws the random stream
        index from each sampler's device counter (for CUDA-graph capture,
        ``CapturedSteps``)."""
        torch = _native.require_cuda()
        if not isinstance(self.features, PeerFeatures):
            return self.step(seeds, seed_ts)
        dev = self.features.device
        if self.gather_stream is None:
            # High priority: the gather's CTAs are scheduled ahead of the
            # queued sampler CTAs of the next call as SM slots free up.
            self.gather_stream = torch.cuda.Stream(device=dev, priority=-1)
            self.tail_stream = torch.cuda.Stream(device=dev) if self.cc_alt is not None else None
        main = torch.cuda.current_stream(dev)
        call = self._calls * self.world + self.rank if call_index is None else call_index
        cc = self.cc if self.cc_alt is None or self._calls % 2 == 0 else self.cc_alt
        self._calls += 1
        if self.tail_stream is None:
            merged = cc.sample_merged(seeds, seed_ts, None, call_index=call, check=False)
            self.gather_stream.wait_stream(main)
        else:
            merged = cc.sample_merged(seeds, seed_ts, None, call_index=call, check=False,
                                      tail_stream=self.tail_stream)
            self.gather_stream.wait_stream(self.tail_stream)
        cap = int(merged.node_ids.numel())
        with torch.cuda.stream(self.gather_stream):
            feats = torch.empty((cap, self.features.dim), dtype=self.features.dtype, device=dev)
            off = merged.node_offsets
            self.features.gather_range(merged.node_ids, _native.elem_ptr(off, 0), _native.elem_ptr(off, -1), cap,
                                       feats, stream=self.gather_stream)
        if not torch.cuda.is_current_stream_capturing():
            for t in (merged.node_ids, merged.node_offsets):
                t.record_stream(self.gather_stream)
        return merged, feats, None

    def drain(self):
        """Makes the current stream wait for every overlapped gather (and
        every split sampling tail)."""
        torch = _native.require_cuda()
        gs = self.gather_stream
        if gs is not None:
            torch.cuda.current_stream(gs.device).wait_stream(gs)
            if self.tail_stream is not None:
                torch.cuda.current_stream(gs.device).wait_stream(self.tail_stream)

    def step_to_host(self, host_seeds, out: HostBatch, timeout_s: float = 10.0) -> HostBatch:
        """One step from host seeds (a pinned int64 tensor) to host results
        in ``out``: seeds copied in, sampled and gathered as ``step``, then
        the batch's node / edge totals are written by the GPU into
        ``out.totals`` (pinned memory; ``dgfx_publish_totals``), which the
        host polls (bounded by ``timeout_s``), so the copies of exactly the
        batch's sizes are issued without a stream synchronisation and queue
        behind the previous step's copies on a copy stream instead of
        waiting for them. Returns ``out`` (its arrays valid once
        ``out.ready()`` / after ``out.wait()``). Reusing a HostBatch waits
        for its previous copies first; alternate two for overlap."""
        import time

        torch = _native.require_cuda()
        dev = self.cc._device if hasattr(self.cc, "_device") else torch.device("cuda", torch.cuda.current_device())
        if getattr(self, "_host_dev_seeds", None) is None or self._host_dev_seeds.numel() != host_seeds.numel():
            self._host_dev_seeds = torch.empty(host_seeds.numel(), dtype=torch.int64, device=dev)
            self._copy_stream = torch.cuda.Stream(device=dev)
        out.wait()
        tot = out.totals.numpy()
        tot[:] = -1
        seeds = self._host_dev_seeds
        seeds.copy_(host_seeds, non_blocking=True)
        merged, feats, _ = self.step(seeds)
        main = torch.cuda.current_stream(dev)
        _native.check(_native.lib().dgfx_publish_totals(
            _native.elem_ptr(merged.node_offsets, -1), _native.elem_ptr(merged.edge_offsets, -1),
            out.totals.data_ptr(), _native.stream_handle(main)))
        t0 = time.perf_counter()
        while tot[0] < 0 or tot[1] < 0:
            if time.perf_counter() - t0 > timeout_s:
                raise RuntimeError(f"step_to_host: the batch totals did not arrive within {timeout_s} s")
        out.n, out.m = int(tot[0]), int(tot[1])
        cs = self._copy_stream
        cs.wait_stream(main)
        if feats is not None and isinstance(self.features, PeerFeatures) and getattr(self, "gather_stream", None):
            cs.wait_stream(self.gather_stream)
        with torch.cuda.stream(cs):
            parts = [(out.node_ids, merged.node_ids, out.n), (out.edge_src, merged.edge_src, out.m),
                     (out.edge_dst, merged.edge_dst, out.m)]
            if feats is not None:
                parts.append((out.features, feats, out.n))
            for host, dev_t, rows in parts:
                host[:rows].copy_(dev_t[:rows], non_blocking=True)
                dev_t.record_stream(cs)
            out.done = torch.cuda.Event()
            out.done.record(cs)
        return out

    def drain_host(self):
        """Makes the current stream wait for every step_to_host copy."""
        torch = _native.require_cuda()
        cs = getattr(self, "_copy_stream", None)
        if cs is not None:
            torch.cuda.current_stream(cs.device).wait_stream(cs)

    def step(self, seeds, seed_ts=None, stream=None):
        call = self._calls * self.world + self.rank  # distinct random stream per rank and call
        self._calls += 1
        merged = self.cc.sample_merged(seeds, seed_ts, None, stream=stream, call_index=call, check=False)
        feats = None
        total = None
        if isinstance(self.features, PeerFeatures):
            # One kernel, bounds read on the device: local rows from HBM,
            # remote rows by peer loads. No host round trip at any world size.
            torch = _native.require_cuda()
            cap = int(merged.node_ids.numel())
            feats = torch.empty((cap, self.features.dim), dtype=self.features.dtype, device=self.features.device)
            off = merged.node_offsets
            self.features.gather_range(merged.node_ids, _native.elem_ptr(off, 0), _native.elem_ptr(off, -1), cap,
                                       feats, stream=stream)
        elif self.features is not None:
            if self.world == 1:
                # No host round trip: bounds of the gather are read on the device.
                torch = _native.require_cuda()
                cap = int(merged.node_ids.numel())
                F = int(self.features.table.shape[1])
                feats = torch.empty((cap, F), dtype=self.features.table.dtype, device=self.features.table.device)
                off = merged.node_offsets
                _native.check(_native.lib().dgfx_gather_rows_ranged(
                    _native.ptr(self.features.table), int(self.features.table.shape[0]), self.features.row_bytes,
                    _native.ptr(merged.node_ids), _native.elem_ptr(off, 0), _native.elem_ptr(off, -1), cap,
                    _native.ptr(feats), _native.stream_handle(stream)))
            else:
                total = int(merged.node_offsets[-1].item())
                feats = self.features.gather(merged.node_ids[:total], stream=stream)
        return merged, feats, total
