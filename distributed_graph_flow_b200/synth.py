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
    _native.check(lib.dgfx_synth_graph_workspace_size(spec.num_nodes, spec.max_degree, ctypes.byref(need)))
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


def normal_rows(ids, dim: int, seed: int, dtype, stream=None):
    """Rows ``ids`` (int64 device tensor) of the normal_features table."""
    torch = _native.require_cuda()
    code = _native.BF16 if dtype == torch.bfloat16 else _native.F32
    n = int(ids.numel())
    out = torch.empty((max(n, 1), dim), dtype=dtype, device=ids.device)[:n]
    _native.check(_native.lib().dgfx_synth_normal_rows(_native.ptr(ids.contiguous()), n, dim, seed, code,
                                                       _native.ptr(out), _stream(stream)))
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


# ---------------------------------------------------------------------------
# Heterogeneous temporal workload: four node sets, four edge types, creation
# times on node set A only (edge times propagated from it).
# ---------------------------------------------------------------------------
@dataclass
class HeteroSpec:
    node_sets: dict            # name -> node count
    edge_sets: dict            # name -> (source node set, target node set, edge count)
    alpha: float
    max_degree: int
    node_ts: dict              # name -> (lo, hi) uniform integer creation times
    feature_dims: dict         # name -> fp32 feature width
    seed: int = 0


HETERO_TEMPORAL = HeteroSpec(
    node_sets={"A": 736_389, "B": 1_134_649, "C": 8_740, "D": 59_965},
    edge_sets={"A_A": ("A", "A", 5_416_271), "A_D": ("A", "D", 7_505_078), "B_A": ("B", "A", 7_145_660),
               "B_C": ("B", "C", 1_043_998)},
    alpha=2.1, max_degree=5_000, node_ts={"A": (2010, 2020)}, feature_dims={"A": 128}, seed=3)


def scaled_hetero(spec: HeteroSpec, scale: float) -> HeteroSpec:
    import dataclasses

    if scale == 1.0:
        return spec
    return dataclasses.replace(
        spec, node_sets={k: max(16, int(v * scale)) for k, v in spec.node_sets.items()},
        edge_sets={k: (s, t, max(1, int(e * scale))) for k, (s, t, e) in spec.edge_sets.items()},
        max_degree=max(8, int(spec.max_degree * min(1.0, scale * 20))))


@dataclass
class HeteroGraph:
    nodeset_names: list        # sorted
    edgeset_names: list        # sorted
    num_nodes: list            # per node set, in nodeset_names order
    node_ts: dict              # name -> int64 device tensor
    edges: dict                # name -> (src, dst, ts or None) device tensors
    fwd: list                  # forward indices (AdjacencyIndex) per edge set
    bwd: list                  # backward indices per edge set
    features: dict             # name -> fp32 [n, dim] device tensor


def build_hetero_graph(spec: HeteroSpec, device) -> HeteroGraph:
    """Generates every edge type on the device, propagates node creation times
    to the edge types that touch a timestamped node set
    (transform.temporal.edge_timestamps), and builds forward and backward
    indices (temporal where the edge type has times)."""
    torch = _native.require_cuda()
    from distributed_graph_flow_b200.transform import temporal

    lib = _native.lib()
    ns_names = sorted(spec.node_sets)
    es_names = sorted(spec.edge_sets)
    node_ts = {n: uniform_int(spec.node_sets[n], lo, hi, spec.seed + 7 * i, 31, device)
               for i, (n, (lo, hi)) in enumerate(sorted(spec.node_ts.items()))}
    edges, fwd, bwd = {}, [], []
    for k, name in enumerate(es_names):
        s_ns, t_ns, ne = spec.edge_sets[name]
        n_s, n_t = spec.node_sets[s_ns], spec.node_sets[t_ns]
        need = ctypes.c_size_t()
        _native.check(lib.dgfx_synth_graph_workspace_size(n_s, spec.max_degree, ctypes.byref(need)))
        ws = torch.empty(need.value, dtype=torch.uint8, device=device)
        rowptr = torch.empty(n_s + 1, dtype=torch.int64, device=device)
        src = torch.empty(ne, dtype=torch.int64, device=device)
        dst = torch.empty(ne, dtype=torch.int64, device=device)
        _native.check(lib.dgfx_synth_bipartite(n_s, n_t, ne, float(spec.alpha), spec.max_degree,
                                               spec.seed * 1000 + 17 * k + 1, _native.ptr(rowptr), _native.ptr(src),
                                               _native.ptr(dst), _native.ptr(ws), need.value, _stream()))
        del ws, rowptr
        ts = None
        if s_ns in node_ts or t_ns in node_ts:
            ts = temporal.edge_timestamps(node_ts.get(s_ns), node_ts.get(t_ns), src, dst)
        edges[name] = (src, dst, ts)
        fwd.append(ext.build_adjacency_index_device(src, dst, ts, n_s, n_t, False, False))
        bwd.append(ext.build_adjacency_index_device(src, dst, ts, n_s, n_t, True, False))
    features = {n: normal_features(0, spec.node_sets[n], d, spec.seed + 50 + i, torch.float32, device)
                for i, (n, d) in enumerate(sorted(spec.feature_dims.items()))}
    torch.cuda.synchronize(device)
    return HeteroGraph(ns_names, es_names, [spec.node_sets[n] for n in ns_names], node_ts, edges, fwd, bwd, features)


def hetero_plan(spec: HeteroSpec, root: str, hop_widths):
    """Plan from `root` walking every edge type in both directions (sorted
    edge set names; forward from a source node set, reversed from a target
    node set), hop_widths[d] neighbours per plan edge at depth d."""
    from distributed_graph_flow_b200.sampling import config as cfg

    links = {}
    for name in sorted(spec.edge_sets):
        s_ns, t_ns, _ = spec.edge_sets[name]
        links.setdefault(s_ns, []).append((name, t_ns, False))
        links.setdefault(t_ns, []).append((name, s_ns, True))

    def build(ns, depth):
        children = []
        if depth < len(hop_widths):
            for name, other, rev in links.get(ns, []):
                children.append(cfg.PlanEdge(edgeset=name, reversed=rev, node=build(other, depth + 1),
                                             hop_width=int(hop_widths[depth])))
        return cfg.PlanNode(ns, children)

    return cfg.SamplingPlan(root=build(root, 0))
