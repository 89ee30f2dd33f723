"""Seeded synthetic inputs generated on the device (dgfx_synth_* kernels).

Stand-ins for the benchmark datasets named by the workloads (none are
available offline): power-law graphs with the sizes of the named graphs,
N(0, 1) node features, uniform integer timestamps and seeds. Everything is a
pure function of (sizes, seed), so every rank of a multi-GPU run regenerates
the same graph and the partition of the features it owns.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional

from distributed_graph_flow_b200 import _native
from distributed_graph_flow_b200.sampling import _in_memory_sampler_ext as ext


@dataclass
class GraphSpec:
    num_nodes: int
    num_edges: int
    alpha: float
    max_degree: int
    seed: int = 0
    ts_range: Optional[tuple] = None  # (lo, hi) for uniform int edge timestamps


# Named workloads (sizes of the datasets they stand in for).
TEMPORAL_169K = GraphSpec(169_343, 1_166_243, 2.1, 20_000, seed=1, ts_range=(0, 50))
PRODUCTS_SPMM = GraphSpec(2_449_029, 61_859_140, 1.9, 17_000, seed=2)
LARGE_SHARDED = GraphSpec(111_059_956, 1_615_685_872, 2.0, 20_000, seed=4)


def _stream(stream=None) -> int:
    return _native.stream_handle(stream)


def rowptr_and_edges(spec: GraphSpec, device, with_edges: bool = True, stream=None):
    """Row pointers int64[N+1] and (optionally) the source-major edge list."""
    torch = _native.require_cuda()
    lib = _native.lib()
    need = ctypes.c_size_t()
    _native.check(lib.dgfx_synth_graph_workspace_size(spec.num_nodes, ctypes.byref(need)))
    ws = torch.empty(need.value, dtype=torch.uint8, device=device)
    rowptr = torch.empty(spec.num_nodes + 1, dtype=torch.int64, device=device)
    src = dst = None
    if with_edges:
        src = torch.empty(spec.num_edges, dtype=torch.int64, device=device)
        dst = torch.empty(spec.num_edges, dtype=torch.int64, device=device)
    _native.check(
        lib.dgfx_synth_graph(
            spec.num_nodes, spec.num_edges, float(spec.alpha), spec.max_degree, spec.seed, _native.ptr(rowptr),
            _native.ptr(src), _native.ptr(dst), _native.ptr(ws), need.value, _stream(stream),
        )
    )
    del ws
    return rowptr, src, dst


def uniform_int(n: int, lo: int, hi: int, seed: int, stream_id: int, device, stream=None):
    torch = _native.require_cuda()
    out = torch.empty(max(n, 1), dtype=torch.int64, device=device)[:n]
    _native.check(_native.lib().dgfx_synth_uniform_int(n, lo, hi, seed, stream_id, _native.ptr(out), _stream(stream)))
    return out


def normal_features(node_begin: int, count: int, dim: int, seed: int, dtype, device, stream=None, out=None):
    torch = _native.require_cuda()
    code = _native.BF16 if dtype == torch.bfloat16 else _native.F32
    if out is None:
        out = torch.empty((max(count, 1), dim), dtype=dtype, device=device)[:count]
    _native.check(
        _native.lib().dgfx_synth_normal_features(node_begin, count, dim, seed, code, _native.ptr(out), _stream(stream))
    )
    return out


def build_graph(spec: GraphSpec, device, keep_edges: bool = False):
    """Generates the graph and builds its forward index in HBM.

    Returns (index, edge_ts or None, (src, dst) or None). The edge list is
    freed unless keep_edges."""
    torch = _native.require_cuda()
    rowptr, src, dst = rowptr_and_edges(spec, device)
    del rowptr
    ts = None
    if spec.ts_range is not None:
        ts = uniform_int(spec.num_edges, spec.ts_range[0], spec.ts_range[1], spec.seed, 11, device)
    index = ext.build_adjacency_index_device(src, dst, ts, spec.num_nodes, spec.num_nodes, False, False)
    edges = (src, dst) if keep_edges else None
    if not keep_edges:
        del src, dst
    torch.cuda.synchronize(device)
    return index, ts, edges
