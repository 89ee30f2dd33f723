"""Halo-exchange orchestration of the multi-GPU driver, on CPU ranks.

Two gloo ranks run HaloFeatures.gather with the three device calls it makes
(partition by owner, local gather, scatter back) replaced by numpy fakes with
the C ABI's semantics, so the host logic (owner buckets, split sizes, the
three all-to-alls, request order) is tested without a GPU. The GPU kernels
themselves are covered by tests/test_gpu_multi.py.
"""

import ctypes
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _arr(ptr, n, dtype):
    ctype = {np.int64: ctypes.c_int64, np.int32: ctypes.c_int32, np.uint8: ctypes.c_uint8}[dtype]
    if n == 0:
        return np.zeros(0, dtype)
    return np.ctypeslib.as_array(ctypes.cast(ptr, ctypes.POINTER(ctype)), shape=(n,))


class FakeLib:
    """Host stand-ins for dgfx_halo_partition / dgfx_gather_rows_local /
    dgfx_scatter_rows (same arguments, same results)."""

    def dgfx_halo_partition_workspace_size(self, n, world, out):
        ctypes.cast(out, ctypes.POINTER(ctypes.c_size_t))[0] = 16
        return 0

    def dgfx_halo_partition(self, ids, n, rows_per_rank, world, sorted_ids, perm, counts, ws, nbytes, stream):
        a = _arr(ids, n, np.int64)
        owner = np.clip(a // rows_per_rank, 0, world - 1)
        order = np.argsort(owner, kind="stable")
        _arr(sorted_ids, n, np.int64)[:] = a[order]
        _arr(perm, n, np.int32)[:] = order.astype(np.int32)
        _arr(counts, world, np.int64)[:] = np.bincount(owner, minlength=world)
        return 0

    def dgfx_gather_rows_local(self, table, rows, row_bytes, ids, n, id_base, out, stream):
        t = _arr(table, rows * row_bytes, np.uint8).reshape(rows, row_bytes)
        o = _arr(out, n * row_bytes, np.uint8).reshape(n, row_bytes)
        r = _arr(ids, n, np.int64) - id_base
        ok = (r >= 0) & (r < rows)
        o[:] = 0
        o[ok] = t[r[ok]]
        return 0

    def dgfx_scatter_rows(self, rows, n, row_bytes, perm, out, stream):
        src = _arr(rows, n * row_bytes, np.uint8).reshape(n, row_bytes)
        o = _arr(out, n * row_bytes, np.uint8).reshape(n, row_bytes)
        o[_arr(perm, n, np.int32)] = src
        return 0


def _worker(rank, world, port, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from distributed_graph_flow_b200 import _native, driver

        _native.lib = lambda: FakeLib()
        _native.stream_handle = lambda stream=None: 0
        _native.require_cuda = lambda: torch
        n_nodes, F = 103, 8
        rpr = -(-n_nodes // world)
        full = torch.arange(n_nodes * F, dtype=torch.float32).reshape(n_nodes, F)
        lo, hi = rank * rpr, min(n_nodes, (rank + 1) * rpr)
        hf = driver.HaloFeatures(full[lo:hi].contiguous(), rpr, rank, world)
        rng = np.random.default_rng(rank)
        for n in (0, 1, 257):
            ids = torch.from_numpy(rng.integers(0, n_nodes, n))
            got = hf.gather(ids)
            assert torch.equal(got, full[ids]), (rank, n)
        result_q.put((rank, "ok"))
    except Exception as exc:  # noqa: BLE001
        result_q.put((rank, repr(exc)))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_halo_exchange_two_cpu_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: "ok", 1: "ok"}, res
