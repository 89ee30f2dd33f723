"""Device implementation of DGF's native sampler module.

Mirrors the surface of the reference's nanobind module
``_in_memory_sampler_ext`` (dgf/src/sampling/in_memory_sampler_ext.cc:
1248-1276): ``CreateSampler``, ``Sampler.Sample`` / ``EdgesetNameToEdgesetIdx``
/ ``__str__`` and ``BuildAdjacencyIndex`` / ``AdjacencyIndex.__str__``, with
the same argument meaning and error messages. Adjacency indices live in HBM
(built by ``dgfx_csr_build``) and sampling runs in ``dgfx_sampler_sample``;
this module only marshals arrays and plans through the C ABI. Nothing here
computes on the host.
"""

from __future__ import annotations

import ctypes
import os
from typing import Dict, List, Optional, Tuple

import numpy as np

from distributed_graph_flow_b200 import _native
from distributed_graph_flow_b200.data import in_memory_graph as img
from distributed_graph_flow_b200.data import schema as schema_lib


def _torch():
    return _native.require_cuda()


def _cropped(values) -> str:
    vals = [int(v) for v in values[:10]]
    s = ", ".join(str(v) for v in vals)
    return s + (", ..." if len(values) > 10 else "")


class AdjacencyIndex:
    """CSR of one direction of one edge set, resident in HBM.

    rowptr int64[num_src + 1], col int32[E], optional ts int64[E] and
    edge_pos int64[E] (CSR position of each original edge; set when the edge
    set is masked). Same content as the reference's AdjacencyIndex
    (dgf/src/sampling/in_memory_sampler.h:60-163).
    """

    def __init__(self, rowptr, col, ts, edge_pos, num_src: int, num_dst: int):
        self.rowptr = rowptr
        self.col = col
        self.ts = ts
        self.edge_pos = edge_pos
        self.num_src = int(num_src)
        self.num_dst = int(num_dst)
        self.num_edges = int(col.numel())

    def view(self) -> _native.CsrView:
        return _native.CsrView(
            _native.ptr(self.rowptr),
            _native.ptr(self.col),
            _native.ptr(self.ts),
            _native.ptr(self.edge_pos),
            self.num_src,
            self.num_dst,
            self.num_edges,
        )

    def __str__(self) -> str:
        # AdjacencyIndex::to_string (in_memory_sampler.h:117-132): sizes and
        # at most the first ten entries.
        blocks = self.rowptr[:11].cpu().numpy()
        targets = self.col[:11].cpu().numpy()
        return (
            f"AdjacencyIndex(source_blocks=({self.num_src + 1})[{_cropped(blocks)}],"
            f" target_node_idxs=({self.num_edges})[{_cropped(targets)}])"
        )


def build_adjacency_index_device(
    src, dst, ts, num_source_nodes: int, num_target_nodes: int, reversed: bool, populate_edge_idxs: bool, stream=None
) -> AdjacencyIndex:
    """Builds an index from device int64 edge arrays (no host round trip)."""
    torch = _torch()
    lib = _native.lib()
    n = int(src.numel())
    num_src, num_dst = (num_target_nodes, num_source_nodes) if reversed else (num_source_nodes, num_target_nodes)
    dev = src.device
    rowptr = torch.empty(num_src + 1, dtype=torch.int64, device=dev)
    col = torch.empty(max(n, 1), dtype=torch.int32, device=dev)[:n]
    ts_out = torch.empty(max(n, 1), dtype=torch.int64, device=dev)[:n] if ts is not None else None
    edge_pos = torch.empty(max(n, 1), dtype=torch.int64, device=dev)[:n] if populate_edge_idxs else None
    need = ctypes.c_size_t()
    _native.check(lib.dgfx_csr_build_workspace_size(n, num_source_nodes, num_target_nodes, int(ts is not None), ctypes.byref(need)))
    ws = torch.empty(need.value, dtype=torch.uint8, device=dev)
    _native.check(
        lib.dgfx_csr_build(
            _native.ptr(src), _native.ptr(dst), _native.ptr(ts), n, num_source_nodes, num_target_nodes, int(bool(reversed)),
            _native.ptr(rowptr), _native.ptr(col), _native.ptr(ts_out), _native.ptr(edge_pos),
            _native.ptr(ws), need.value, _native.stream_handle(stream),
        )
    )
    return AdjacencyIndex(rowptr, col, ts_out, edge_pos, num_src, num_dst)


def BuildAdjacencyIndex(
    py_adjacency,
    py_timestamps=None,
    reversed: bool = False,
    num_source_nodes: int = 0,
    num_target_nodes: int = 0,
    populate_edge_idxs: bool = False,
) -> AdjacencyIndex:
    """Same contract as the reference's BuildAdjacencyIndex (ext.cc:1020-1093)."""
    torch = _torch()
    dev = torch.device("cuda", torch.cuda.current_device())
    if isinstance(py_adjacency, torch.Tensor) and py_adjacency.is_cuda:
        # Already in HBM (e.g. io.graph_in_memory.read_graph(device=...)).
        if py_adjacency.dim() != 2 or py_adjacency.shape[0] != 2:
            raise ValueError("adjacency must have shape [2, num_edges]")
        src = py_adjacency[0].to(device=dev, dtype=torch.int64).contiguous()
        dst = py_adjacency[1].to(device=dev, dtype=torch.int64).contiguous()
    else:
        adj = np.asarray(py_adjacency)
        if adj.ndim != 2 or adj.shape[0] != 2:
            raise ValueError("adjacency must have shape [2, num_edges]")
        adj = np.ascontiguousarray(adj.astype(np.int64, copy=False))
        src = torch.from_numpy(adj[0].copy()).to(dev, non_blocking=False)
        dst = torch.from_numpy(adj[1].copy()).to(dev, non_blocking=False)
    ts = None
    if py_timestamps is not None:
        if populate_edge_idxs:
            raise ValueError("Check failed !populate_edge_idxs")
        ts = torch.from_numpy(np.ascontiguousarray(np.asarray(py_timestamps, dtype=np.int64))).to(dev)
    return build_adjacency_index_device(src, dst, ts, int(num_source_nodes), int(num_target_nodes), reversed, populate_edge_idxs)


class _PlanArrays:
    """A SamplingPlan flattened for dgfx_sampler_create (node 0 = root)."""

    def __init__(self, plan, nodeset_index: Dict[str, int], edgeset_index: Dict[str, int]):
        self.node_nodeset: List[int] = []
        self.node_first_edge: List[int] = []
        self.node_num_edges: List[int] = []
        self.edge_edgeset: List[int] = []
        self.edge_reversed: List[int] = []
        self.edge_hop_width: List[int] = []
        self.edge_child: List[int] = []
        self.nodes = []  # python PlanNode per flattened node
        queue = [plan.root]
        self._add_node(plan.root, nodeset_index)
        head = 0
        while head < len(queue):
            pn = queue[head]
            i = head
            head += 1
            self.node_first_edge[i] = len(self.edge_edgeset)
            self.node_num_edges[i] = len(pn.children)
            for child in pn.children:
                if child.edgeset not in edgeset_index:
                    raise ValueError(f"Key not found in map: {child.edgeset}")
                self.edge_edgeset.append(edgeset_index[child.edgeset])
                self.edge_reversed.append(int(bool(child.reversed)))
                self.edge_hop_width.append(int(child.hop_width))
                self.edge_child.append(len(self.nodes))
                self._add_node(child.node, nodeset_index)
                queue.append(child.node)

    def _add_node(self, pn, nodeset_index):
        if pn.nodeset not in nodeset_index:
            raise ValueError(f"Key not found in map: {pn.nodeset}")
        self.nodes.append(pn)
        self.node_nodeset.append(nodeset_index[pn.nodeset])
        self.node_first_edge.append(0)
        self.node_num_edges.append(0)

    @staticmethod
    def arr32(v: List[int]):
        return (ctypes.c_int32 * max(1, len(v)))(*v)


def _plan_to_string(plan, nodeset_index, edgeset_index) -> str:
    """SamplingPlan::to_string (dgf/src/sampling/in_memory_sampler.h:184-238)."""

    def node_str(pn, indent: int) -> str:
        prefix = " " * (2 * indent)
        if not pn.children:
            kids = "[]"
        else:
            kids = "[\n" + ",\n".join(edge_str(c, indent + 1) for c in pn.children) + "\n" + prefix + "]"
        return f"{prefix}Node(nodeset_idx={nodeset_index[pn.nodeset]}, children={kids})"

    def edge_str(pe, indent: int) -> str:
        prefix = " " * (2 * indent)
        return (
            f"{prefix}Edge(edgeset_idx={edgeset_index[pe.edgeset]}, reversed={int(bool(pe.reversed))},"
            f" hop_width={pe.hop_width}, node=\n{node_str(pe.node, indent + 1)})"
        )

    return f"SamplingPlan(root=\n{node_str(plan.root, 0)},\n  with_replacement={int(bool(plan.with_replacement))}\n)"


class MergedBatch:
    """Device-resident sampler output for one call (see dgfx_sample_out).

    node_ids[node_offsets[s*B + i]:node_offsets[s*B + i + 1]] are the
    ``#idx`` of node set s in sample i; edge_src / edge_dst likewise per edge
    set e (local ids). Offsets carry one trailing total.
    """

    def __init__(self, B, nodeset_names, edgeset_names, node_ids, node_offsets, edge_src, edge_dst, edge_offsets):
        self.B = B
        self.nodeset_names = nodeset_names
        self.edgeset_names = edgeset_names
        self.node_ids = node_ids
        self.node_offsets = node_offsets
        self.edge_src = edge_src
        self.edge_dst = edge_dst
        self.edge_offsets = edge_offsets

    def nodeset_range(self, s: int, offsets_host: np.ndarray) -> Tuple[int, int]:
        return int(offsets_host[s * self.B]), int(offsets_host[(s + 1) * self.B])


class Sampler:
    """Device sampler created by CreateSampler."""

    def __init__(self):
        self._handle = None
        self._buffers = {}
        self._sizes = {}  # B -> (node capacity, edge capacity, workspace bytes)
        self._calls = 0

    def __del__(self):
        h = getattr(self, "_handle", None)
        if h:
            try:
                _native.lib().dgfx_sampler_destroy(h)
            except Exception:  # interpreter shutdown
                pass
            self._handle = None

    # -- introspection ---------------------------------------------------
    def __str__(self) -> str:
        ns = ", ".join(f"{n}: {i}" for n, i in sorted(self._nodeset_index.items()))
        es = ", ".join(f"{n}: {i}" for n, i in sorted(self._edgeset_index.items()))
        nodesets = ", ".join(f"{{idx={i}, num_nodes={n}}}" for i, n in enumerate(self._num_nodes))
        return (
            f"Sampler(\n  plan={_plan_to_string(self._plan, self._nodeset_index, self._edgeset_index)},\n"
            f"  nodeset_index={{{ns}}},\n  edgeset_index={{{es}}},\n  nodesets=[{nodesets}]\n)"
        )

    def EdgesetNameToEdgesetIdx(self, name: str) -> int:
        if name not in self._edgeset_index:
            raise ValueError(f"Key not found in map: {name}")
        return self._edgeset_index[name]

    @property
    def tree_size(self) -> int:
        v = ctypes.c_int64()
        _native.check(_native.lib().dgfx_sampler_tree_size(self._handle, ctypes.byref(v)))
        return v.value

    def set_kernel(self, kind: int) -> None:
        """0 (default): warp sampler, large-tree warp tier for seeds that
        outgrow it, padded sampler for trees beyond that; 1: padded sampler
        for every seed; 2: warp sampler with the padded sampler behind it.
        All give identical batches."""
        _native.check(_native.lib().dgfx_sampler_set_kernel(self._handle, int(kind)))
        self._sizes.clear()  # the workspace size depends on the kernel

    def _kernel_info(self):
        v, big = ctypes.c_int32(), ctypes.c_int32()
        _native.check(_native.lib().dgfx_sampler_kernel_info(self._handle, ctypes.byref(v), ctypes.byref(big)))
        return v.value, big.value

    @property
    def warp_capacity(self) -> int:
        """Per-seed entry capacity of the warp sampler (0: not used)."""
        return self._kernel_info()[0]

    @property
    def large_tree_capacity(self) -> int:
        """Per-seed entry capacity of the large-tree warp tier (0: not used)."""
        return self._kernel_info()[1]

    def kernel_stats(self, stream=None):
        """(seeds finished by a warp tier, seeds finished by the padded
        sampler) of the last call."""
        out = (ctypes.c_int64 * 2)()
        _native.check(_native.lib().dgfx_sampler_kernel_stats(self._handle, _native.stream_handle(stream), out))
        return int(out[0]), int(out[1])

    # -- sampling --------------------------------------------------------
    def _workspace(self, nbytes: int):
        """Scratch reused across calls (calls on one sampler are serialised
        on the stream they are issued on)."""
        torch = _torch()
        buf = self._buffers.get("ws")
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(max(1, nbytes), dtype=torch.uint8, device=self._device)
            self._buffers["ws"] = buf
        return buf

    def _validate_args(self, B, seed_ts, masks):
        if seed_ts is not None:
            if not self._has_temporal:
                raise ValueError(
                    "seed_timestamps provided but no temporal edgesets configured. Set "
                    "the 'edgeset_timestamp_features' field in the sampling plan."
                )
            if int(seed_ts.numel()) != B:
                raise ValueError("seed_node_idxs and seed_timestamps must have the same size")
        if masks is not None:
            if self._mask_edgeset < 0:
                raise ValueError("masked_edge_idxs provided but no edgeset to mask configured.")
            if int(masks.numel()) != B:
                raise ValueError("seed_node_idxs and masked_edge_idxs must have the same size")

    def sample_merged(self, seeds, seed_ts=None, masks=None, stream=None, call_index: Optional[int] = None,
                      check: bool = True, tail_stream=None) -> MergedBatch:
        """Samples one subgraph per seed into a device-resident merged batch.

        seeds / seed_ts / masks are int64 device tensors. With check=False the
        call stays asynchronous (errors are latched; call ``check()``).
        call_index=_native.CALL_INDEX_DEVICE takes the random-stream index from
        a device counter that every call advances (for CUDA-graph capture).
        With ``tail_stream`` (a torch stream other than ``stream``) the call
        runs split (dgfx_sampler_sample_split): the batch is complete in
        ``tail_stream`` order, and ``stream`` is free for the next batch once
        the first sampling kernel ends.
        """
        torch = _torch()
        lib = _native.lib()
        B = int(seeds.numel())
        self._validate_args(B, seed_ts, masks)
        sizes = self._sizes.get(B)
        if sizes is None:  # output capacity and workspace depend on B only
            max_nodes = ctypes.c_int64()
            max_edges = ctypes.c_int64()
            _native.check(lib.dgfx_sampler_output_capacity(self._handle, B, ctypes.byref(max_nodes),
                                                           ctypes.byref(max_edges)))
            need = ctypes.c_size_t()
            _native.check(lib.dgfx_sampler_workspace_size(self._handle, B, ctypes.byref(need)))
            sizes = self._sizes[B] = (max(1, max_nodes.value), max(1, max_edges.value), need.value)
        cap_nodes, cap_edges, need_bytes = sizes
        NS, ES = len(self._nodeset_names), len(self._edgeset_names)
        dev = self._device
        # One allocation for the five outputs (each starts on a 256-byte boundary).
        lens = (cap_nodes, NS * B + 1, cap_edges, cap_edges, ES * B + 1)
        starts, at = [], 0
        for n in lens:
            starts.append(at)
            at += (n + 31) // 32 * 32
        buf = torch.empty(at, dtype=torch.int64, device=dev)
        node_ids, node_off, edge_src, edge_dst, edge_off = (buf[a:a + n] for a, n in zip(starts, lens))
        ws = self._workspace(need_bytes)
        out = _native.SampleOut(
            _native.ptr(node_ids), _native.ptr(node_off), _native.ptr(edge_src), _native.ptr(edge_dst), _native.ptr(edge_off)
        )
        if call_index is None:
            call_index = self._calls
            self._calls += 1
        sh = _native.stream_handle(stream)
        if tail_stream is None:
            _native.check(
                lib.dgfx_sampler_sample(
                    self._handle, _native.ptr(seeds), _native.ptr(seed_ts), _native.ptr(masks), B, int(call_index),
                    ctypes.byref(out), _native.ptr(ws), need_bytes, sh,
                )
            )
        else:
            _native.check(
                lib.dgfx_sampler_sample_split(
                    self._handle, _native.ptr(seeds), _native.ptr(seed_ts), _native.ptr(masks), B, int(call_index),
                    ctypes.byref(out), _native.ptr(ws), need_bytes, sh, _native.stream_handle(tail_stream),
                )
            )
            # Tensors the tail reads or writes stay allocated until it ends
            # (a captured graph keeps its own allocations).
            if not torch.cuda.is_current_stream_capturing():
                for t in (seeds, seed_ts, masks, buf):
                    if t is not None:
                        t.record_stream(tail_stream)
        if check:
            self.check(stream if tail_stream is None else tail_stream)
        return MergedBatch(B, self._nodeset_names, self._edgeset_names, node_ids, node_off, edge_src, edge_dst,
                           edge_off)

    def check(self, stream=None) -> None:
        _native.check(_native.lib().dgfx_sampler_check(self._handle, _native.stream_handle(stream)))

    def _to_device(self, arr, name):
        torch = _torch()
        if arr is None:
            return None
        a = np.ascontiguousarray(np.asarray(arr, dtype=np.int64))
        return torch.from_numpy(a).to(self._device, non_blocking=False)

    def Sample(self, seed_node_idx, seed_timestamps=None, masked_edge_idxs=None) -> list:
        """Reference-compatible: a list of InMemoryGraph holding only "#idx"."""
        seeds = self._to_device(seed_node_idx, "seeds")
        ts = self._to_device(seed_timestamps, "ts")
        masks = self._to_device(masked_edge_idxs, "masks")
        batch = self.sample_merged(seeds, ts, masks)
        return export_graphs(batch)

    def _edgeset_endpoints(self):
        """(source, target) node set index of every edge set the plan walks
        (from the plan's edges: a reversed plan edge walks target -> source)."""
        src = [0] * len(self._edgeset_names)
        dst = [0] * len(self._edgeset_names)

        def walk(pn):
            for pe in pn.children:
                here, there = self._nodeset_index[pn.nodeset], self._nodeset_index[pe.node.nodeset]
                e = self._edgeset_index[pe.edgeset]
                src[e], dst[e] = (there, here) if pe.reversed else (here, there)
                walk(pe.node)

        walk(self._plan.root)
        return src, dst

    def SubGraph(self, seed_node_idx) -> img.InMemoryGraph:
        """One graph around all seeds (Sampler::SubGraph, ext.cc:959-972, with
        SubGraphExtractor :600-772): the seeds are the first nodes of the root
        node set in seed order, every other node is numbered in order of its
        first (seed, depth-first) discovery, edges deduplicated and sorted.
        Computed as the union of the seeds' samples on the device
        (dgfx_subgraph_union); exact in the deterministic modes (debug
        sampling, or hop_width >= degree)."""
        torch = _torch()
        lib = _native.lib()
        seeds = self._to_device(np.asarray(seed_node_idx, dtype=np.int64).reshape(-1), "seeds")
        batch = self.sample_merged(seeds)
        B = batch.B
        NS, ES = len(self._nodeset_names), len(self._edgeset_names)
        n = int(batch.node_offsets[-1].item())
        m = int(batch.edge_offsets[-1].item())
        dev = self._device
        out_nodes = torch.empty(max(n, 1), dtype=torch.int64, device=dev)
        out_src = torch.empty(max(m, 1), dtype=torch.int64, device=dev)
        out_dst = torch.empty(max(m, 1), dtype=torch.int64, device=dev)
        node_counts = (ctypes.c_int64 * NS)()
        edge_counts = (ctypes.c_int64 * max(ES, 1))()
        src_ns, dst_ns = self._edgeset_endpoints()
        need = ctypes.c_size_t()
        _native.check(lib.dgfx_subgraph_union_workspace_size(n, m, ctypes.byref(need)))
        ws = torch.empty(max(1, need.value), dtype=torch.uint8, device=dev)
        root = self._nodeset_index[self._root_nodeset]
        _native.check(lib.dgfx_subgraph_union(
            _native.ptr(batch.node_ids), _native.ptr(batch.node_offsets), _native.ptr(batch.edge_src),
            _native.ptr(batch.edge_dst), _native.ptr(batch.edge_offsets), B, NS, ES, root,
            (ctypes.c_int32 * max(ES, 1))(*src_ns), (ctypes.c_int32 * max(ES, 1))(*dst_ns), n, m,
            _native.ptr(out_nodes), node_counts, _native.ptr(out_src), _native.ptr(out_dst), edge_counts,
            _native.ptr(ws), need.value, _native.stream_handle()))
        nodes_h = out_nodes.cpu().numpy()
        src_h, dst_h = out_src.cpu().numpy(), out_dst.cpu().numpy()
        node_sets, edge_sets = {}, {}
        a = 0
        for s, name in enumerate(self._nodeset_names):
            c = int(node_counts[s])
            node_sets[name] = img.InMemoryNodeSet(num_nodes=c, features={"#idx": nodes_h[a:a + c].copy()})
            a += c
        a = 0
        for e, name in enumerate(self._edgeset_names):
            c = int(edge_counts[e]) if ES else 0
            edge_sets[name] = img.InMemoryEdgeSet(adjacency=np.stack([src_h[a:a + c], dst_h[a:a + c]]).astype(np.int64))
            a += c
        return img.InMemoryGraph(node_sets=node_sets, edge_sets=edge_sets)

    def MultiSubGraphs(self, seed_node_idx) -> list:
        """One independent subgraph per seed (Sampler::MultiSubGraphs,
        ext.cc:974-1017): the seed's sample, which equals its extracted
        subgraph in the deterministic modes (the reference documents
        multisubgraph as sample with an infinite width)."""
        seeds = self._to_device(np.asarray(seed_node_idx, dtype=np.int64).reshape(-1), "seeds")
        return export_graphs(self.sample_merged(seeds))

    def random_walk_negatives(self, seeds, target_edgeset_idx: int, num_walks: int, num_negatives_per_seed: int,
                              stream=None, call_index: Optional[int] = None, check: bool = True):
        """Random-walk negatives for device int64 seeds: an int64 CUDA tensor
        [num_seeds, num_negatives_per_seed] (dgfx_random_walk_negatives).
        With check=False the call stays asynchronous; call
        ``check_random_walk_negatives()`` before trusting the rows."""
        torch = _torch()
        lib = _native.lib()
        e = int(target_edgeset_idx)
        if e < 0 or e >= len(self._edgeset_names):
            raise ValueError("Invalid target_edgeset_idx")
        if self._fwd[e] is None:
            raise ValueError(f"Edgeset '{self._edgeset_names[e]}' does not have a forward index. "
                             "Ensure it is traversed forward in the SamplingPlan.")
        B, W, K = int(seeds.numel()), int(num_walks), int(num_negatives_per_seed)
        need = ctypes.c_size_t()
        _native.check(lib.dgfx_random_walk_negatives_workspace_size(self._handle, B, e, W, K, ctypes.byref(need)))
        ws = self._buffers.get("rw_ws")
        if ws is None or ws.numel() < need.value:
            ws = torch.empty(max(256, need.value), dtype=torch.uint8, device=self._device)
            self._buffers["rw_ws"] = ws
        out = torch.empty((B, K), dtype=torch.int64, device=self._device)
        if call_index is None:
            call_index = self._calls
            self._calls += 1
        _native.check(lib.dgfx_random_walk_negatives(self._handle, _native.ptr(seeds), B, e, W, K,
                                                     int(call_index) & ((1 << 64) - 1), _native.ptr(out),
                                                     _native.ptr(ws), ws.numel(), _native.stream_handle(stream)))
        if check:
            self.check_random_walk_negatives(stream)
        return out

    def check_random_walk_negatives(self, stream=None) -> None:
        ws = self._buffers.get("rw_ws")
        if ws is not None:
            _native.check(_native.lib().dgfx_random_walk_negatives_check(_native.ptr(ws), _native.stream_handle(stream)))

    def RandomWalkNegativeSampling(self, seed_node_idxs, target_edgeset_idx, num_walks, num_negatives_per_seed):
        """Sampler::RandomWalkNegativeSampling (ext.cc:875-948): int64 numpy
        [num_seeds, num_negatives_per_seed] of negative target nodes per seed
        (visit-ranked random-walk nodes the seed does not link to, then
        uniform fallback draws)."""
        seeds = self._to_device(np.asarray(seed_node_idxs, dtype=np.int64).reshape(-1), "seeds")
        return self.random_walk_negatives(seeds, target_edgeset_idx, num_walks, num_negatives_per_seed).cpu().numpy()


class CapturedSampleStep:
    """``sample_merged`` calls, plus optional gathers of the sampled nodes'
    feature rows, captured once in a CUDA graph over static buffers.

    With a list of K samplers the graph forks K independent batches of
    ``batch_size`` seeds onto K streams and joins them: one ``run`` samples K
    batches concurrently for the host cost of one graph launch. ``run(seeds,
    seed_ts)`` copies the inputs ([K, batch_size] or [batch_size] int64) into
    the static buffers and replays the graph; the random streams advance on
    every replay (device call index). Results are the static outputs, valid
    until the next ``run``: a list of K (MergedBatch, feature rows) pairs, or
    one pair for a single sampler. Each sampler handle belongs to this step
    (handles serialise their calls). ``table`` is a [num_rows, F] feature
    matrix of node set ``feature_nodeset``. With ``aggregate`` (one node set
    and edge set) every node's mean over the features of the neighbours it
    sampled follows the gather (aggregation.batch_mean_aggregate) and the
    results are (MergedBatch, feature rows, aggregates) triples. With
    ``serial`` the K batches run one after the other on one stream inside
    the graph (a training loop's sequence of batches, without the host's
    per-batch launch cost)."""

    def __init__(self, samplers, batch_size: int, with_timestamps: bool, table=None, feature_nodeset: int = 0,
                 stream=None, aggregate: bool = False, serial: bool = False):
        torch = _torch()
        from distributed_graph_flow_b200 import aggregation
        self.single = not isinstance(samplers, (list, tuple))
        self.samplers = [samplers] if self.single else list(samplers)
        K = len(self.samplers)
        dev = self.samplers[0]._device
        self.B = int(batch_size)
        self.stream = stream if stream is not None else torch.cuda.Stream(device=dev)
        if serial:  # the K batches one after the other on one stream
            self.branches = [self.stream] * K
        else:
            self.branches = [self.stream] + [torch.cuda.Stream(device=dev) for _ in range(K - 1)]
        self.seeds = torch.zeros((K, self.B), dtype=torch.int64, device=dev)
        self.seed_ts = torch.zeros((K, self.B), dtype=torch.int64, device=dev) if with_timestamps else None
        ns = int(feature_nodeset)
        self.features = [None] * K
        self.aggregates = [None] * K
        if aggregate and (table is None or any(len(smp._nodeset_index) != 1 or len(smp._edgeset_index) != 1
                                               for smp in self.samplers)):
            raise ValueError("aggregate needs a feature table and samplers over one node set and one edge set")
        if table is not None:
            for k, smp in enumerate(self.samplers):
                cap = self.B * smp.tree_size
                self.features[k] = torch.empty((cap, int(table.shape[1])), dtype=table.dtype, device=dev)
                if aggregate:
                    self.aggregates[k] = torch.empty((cap, int(table.shape[1])), dtype=table.dtype, device=dev)

        def body(k):
            smp = self.samplers[k]
            batch = smp.sample_merged(self.seeds[k], None if self.seed_ts is None else self.seed_ts[k], None,
                                      call_index=_native.CALL_INDEX_DEVICE, check=False)
            if table is not None:
                off = batch.node_offsets
                _native.check(_native.lib().dgfx_gather_rows_ranged(
                    _native.ptr(table), int(table.shape[0]), int(table.shape[1]) * table.element_size(),
                    _native.ptr(batch.node_ids), _native.elem_ptr(off, ns * self.B),
                    _native.elem_ptr(off, (ns + 1) * self.B), int(batch.node_ids.numel()),
                    _native.ptr(self.features[k]), _native.stream_handle()))
                if aggregate:  # mean over each node's sampled neighbours
                    aggregation.batch_mean_aggregate(batch, self.features[k], out=self.aggregates[k])
            return batch

        for k in range(K):  # allocates each sampler's workspace outside the capture
            with torch.cuda.stream(self.branches[k]):
                body(k)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        self.batches = [None] * K
        with torch.cuda.graph(self.graph, stream=self.stream):
            if not serial:
                for k in range(1, K):  # fork
                    self.branches[k].wait_stream(self.stream)
            for k in range(K):
                with torch.cuda.stream(self.branches[k]):
                    self.batches[k] = body(k)
            if not serial:
                for k in range(1, K):  # join
                    self.stream.wait_stream(self.branches[k])
        torch.cuda.synchronize(dev)
        # One foreign call per run: input copies + launch of the graph exec.
        self._exec = int(self.graph.raw_cuda_graph_exec())
        self._launch = _native.lib().dgfx_graph_launch_with_inputs
        self._seed_bytes = self.seeds.numel() * 8
        self._ts_ptr = None if self.seed_ts is None else int(self.seed_ts.data_ptr())
        self._seeds_ptr = int(self.seeds.data_ptr())
        if self.aggregates[0] is not None:
            out = list(zip(self.batches, self.features, self.aggregates))
        else:
            out = list(zip(self.batches, self.features))
        self._out = out[0] if self.single else out

    def _input_ptr(self, t, name):
        torch = _torch()
        if t.dtype != torch.int64 or t.numel() != self.seeds.numel() or not t.is_contiguous():
            raise ValueError(f"CapturedSampleStep.run: {name} must be a contiguous int64 tensor of "
                             f"{self.seeds.numel()} elements")
        return t.data_ptr()

    def run(self, seeds, seed_ts=None):
        """Samples ``seeds`` in the caller's current stream order: one native
        call copies the inputs into the static buffers and launches the
        captured graph on that stream. The inputs must stay alive until the
        copies have run (stream order of their own allocation suffices), and
        consecutive runs must come from one stream, since each run rewrites
        the static inputs and outputs."""
        src_ts, ts_bytes = None, 0
        if self.seed_ts is not None:
            if seed_ts is None:
                raise ValueError("CapturedSampleStep.run: seed_ts is required (captured with timestamps)")
            src_ts, ts_bytes = self._input_ptr(seed_ts, "seed_ts"), self._seed_bytes
        _native.check(self._launch(self._exec, self._seeds_ptr, self._input_ptr(seeds, "seeds"), self._seed_bytes,
                                   self._ts_ptr, src_ts, ts_bytes, _native.stream_handle()))
        return self._out

    def wait(self):
        """Kept for callers of the earlier two-stream form: run() now works in
        the caller's stream order, so there is nothing to join."""

    @property
    def sampler(self):
        return self.samplers[0]


def batch_to_host(batch: MergedBatch):
    """Copies a merged batch's exact-size arrays to host numpy arrays."""
    node_off = batch.node_offsets.cpu().numpy()
    edge_off = batch.edge_offsets.cpu().numpy()
    n_nodes = int(node_off[-1])
    n_edges = int(edge_off[-1])
    node_ids = batch.node_ids[:n_nodes].cpu().numpy()
    edges = np.empty((2, n_edges), dtype=np.int64)
    if n_edges:
        edges[0] = batch.edge_src[:n_edges].cpu().numpy()
        edges[1] = batch.edge_dst[:n_edges].cpu().numpy()
    return node_ids, node_off, edges, edge_off


def export_graphs(batch: MergedBatch, host=None) -> List[img.InMemoryGraph]:
    """One InMemoryGraph per seed with "#idx" and [2, E] adjacency
    (ExportToInMemoryGraph, in_memory_sampler_ext.cc:372-397): every node set
    and edge set is present, in index (sorted-name) order."""
    node_ids, node_off, edges, edge_off = host if host is not None else batch_to_host(batch)
    B = batch.B
    graphs = []
    for i in range(B):
        nodesets = {}
        for s, name in enumerate(batch.nodeset_names):
            a, b = int(node_off[s * B + i]), int(node_off[s * B + i + 1])
            nodesets[name] = img.InMemoryNodeSet(num_nodes=b - a, features={"#idx": node_ids[a:b]})
        edgesets = {}
        for e, name in enumerate(batch.edgeset_names):
            a, b = int(edge_off[e * B + i]), int(edge_off[e * B + i + 1])
            edgesets[name] = img.InMemoryEdgeSet(adjacency=edges[:, a:b])
        graphs.append(img.InMemoryGraph(node_sets=nodesets, edge_sets=edgesets))
    return graphs


def CreateSampler(
    graph: img.InMemoryGraph,
    plan,
    debug_sampling: bool,
    num_threads: int,
    seed: int,
    py_schema: schema_lib.GraphSchema,
    edgeset_to_mask: Optional[str] = None,
    edgeset_timestamp_features: Optional[Dict[str, str]] = None,
    sampling_mode: Optional[int] = None,
    device=None,
) -> Sampler:
    """Same contract as the reference's CreateSampler (ext.cc:1216-1246).

    num_threads is accepted for compatibility; the GPU grid replaces the
    reference's thread pool. sampling_mode (an extension) overrides the mode
    chosen by debug_sampling, e.g. MODE_MOST_RECENT.
    """
    torch = _torch()
    edgeset_timestamp_features = dict(edgeset_timestamp_features or {})
    nodeset_index = py_schema.nodeset_index()
    edgeset_index = py_schema.edgeset_index()
    nodeset_names = sorted(py_schema.node_sets)
    edgeset_names = sorted(py_schema.edge_sets)
    plan_arrays = _PlanArrays(plan, nodeset_index, edgeset_index)

    mask_idx = -1
    if edgeset_to_mask is not None:
        if edgeset_to_mask not in edgeset_index:
            raise ValueError(f"Edgeset '{edgeset_to_mask}' does not exist in schema")
        mask_idx = edgeset_index[edgeset_to_mask]
    for name in edgeset_timestamp_features:
        if name not in edgeset_index:
            raise ValueError(f"Edgeset '{name}' does not exist in schema")

    num_nodes = []
    for name in nodeset_names:
        if name not in graph.node_sets:
            raise ValueError(f"Key not found in dict: {name}")
        n = graph.node_sets[name].num_nodes
        if n is None:
            raise ValueError(f"num_nodes of nodeset '{name}' is not set")
        num_nodes.append(int(n))

    # Which directions of which edge sets the plan walks, with endpoint
    # consistency checks (Sampler::IndexEdgeSets, ext.cc:1124-1163).
    src_ns = [-1] * len(edgeset_names)
    dst_ns = [-1] * len(edgeset_names)
    need_fwd = [False] * len(edgeset_names)
    need_bwd = [False] * len(edgeset_names)
    for i, _ in enumerate(plan_arrays.nodes):
        for c in range(plan_arrays.node_num_edges[i]):
            j = plan_arrays.node_first_edge[i] + c
            e = plan_arrays.edge_edgeset[j]
            here = plan_arrays.node_nodeset[i]
            there = plan_arrays.node_nodeset[plan_arrays.edge_child[j]]
            s, t = (there, here) if plan_arrays.edge_reversed[j] else (here, there)
            if not (src_ns[e] in (-1, s)):
                raise ValueError("Check failed edgeset.source_nodeset == -1 || edgeset.source_nodeset == node.nodeset_idx")
            if not (dst_ns[e] in (-1, t)):
                raise ValueError("Check failed edgeset.target_nodeset == -1 || edgeset.target_nodeset == child.node->nodeset_idx")
            src_ns[e], dst_ns[e] = s, t
            if plan_arrays.edge_reversed[j]:
                need_bwd[e] = True
            else:
                need_fwd[e] = True

    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    fwd: List[Optional[AdjacencyIndex]] = [None] * len(edgeset_names)
    bwd: List[Optional[AdjacencyIndex]] = [None] * len(edgeset_names)
    with torch.cuda.device(dev):
        for e, name in enumerate(edgeset_names):
            if not (need_fwd[e] or need_bwd[e]):
                continue
            if name not in graph.edge_sets:
                raise ValueError(f"Key not found in dict: {name}")
            es = graph.edge_sets[name]
            ts = None
            if name in edgeset_timestamp_features:
                feat = edgeset_timestamp_features[name]
                if feat not in es.features:
                    raise ValueError(f"Key not found in dict: {feat}")
                ts = es.features[feat]
            ns_src, ns_dst = num_nodes[src_ns[e]], num_nodes[dst_ns[e]]
            if need_fwd[e]:
                fwd[e] = BuildAdjacencyIndex(es.adjacency, ts, False, ns_src, ns_dst, e == mask_idx)
            if need_bwd[e]:
                bwd[e] = BuildAdjacencyIndex(es.adjacency, ts, True, ns_src, ns_dst, e == mask_idx)
    mode = _native.MODE_FIRST if debug_sampling else _native.MODE_RANDOM
    if sampling_mode is not None:
        mode = int(sampling_mode)
    return create_device_sampler(
        plan, nodeset_names, num_nodes, edgeset_names, fwd, bwd, mode, seed, mask_idx,
        has_temporal=bool(edgeset_timestamp_features), device=dev, plan_arrays=plan_arrays,
    )


def create_device_sampler(
    plan,
    nodeset_names: List[str],
    num_nodes: List[int],
    edgeset_names: List[str],
    fwd: List[Optional[AdjacencyIndex]],
    bwd: List[Optional[AdjacencyIndex]],
    mode: int,
    seed: Optional[int],
    mask_idx: int = -1,
    has_temporal: bool = False,
    device=None,
    plan_arrays: Optional[_PlanArrays] = None,
) -> Sampler:
    """Sampler over indices already resident in HBM (e.g. built on the device
    from a generated edge list). Node/edge set lists are in index order."""
    torch = _torch()
    nodeset_index = {n: i for i, n in enumerate(nodeset_names)}
    edgeset_index = {n: i for i, n in enumerate(edgeset_names)}
    if plan_arrays is None:
        plan_arrays = _PlanArrays(plan, nodeset_index, edgeset_index)
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(dev):
        if seed is None or seed < 0:
            seed = int.from_bytes(os.urandom(8), "little") >> 1
        empty = _native.CsrView()
        fwd_views = (_native.CsrView * max(1, len(edgeset_names)))(*[x.view() if x else empty for x in fwd])
        bwd_views = (_native.CsrView * max(1, len(edgeset_names)))(*[x.view() if x else empty for x in bwd])
        pa = plan_arrays
        handle = ctypes.c_void_p()
        _native.check(
            _native.lib().dgfx_sampler_create(
                len(pa.node_nodeset), pa.arr32(pa.node_nodeset), pa.arr32(pa.node_first_edge), pa.arr32(pa.node_num_edges),
                len(pa.edge_edgeset), pa.arr32(pa.edge_edgeset), pa.arr32(pa.edge_reversed), pa.arr32(pa.edge_hop_width),
                pa.arr32(pa.edge_child), int(bool(plan.with_replacement)), len(nodeset_names),
                (ctypes.c_int64 * len(num_nodes))(*num_nodes), len(edgeset_names), fwd_views, bwd_views, mode, mask_idx,
                int(seed) & ((1 << 64) - 1), ctypes.byref(handle),
            )
        )
    s = Sampler()
    s._handle = handle.value
    s._device = dev
    s._plan = plan
    s._nodeset_index = nodeset_index
    s._edgeset_index = edgeset_index
    s._nodeset_names = nodeset_names
    s._edgeset_names = edgeset_names
    s._num_nodes = num_nodes
    s._fwd = fwd
    s._bwd = bwd
    s._mask_edgeset = mask_idx
    s._has_temporal = bool(has_temporal)
    s._mode = mode
    s._seed = seed
    s._root_nodeset = plan.root.nodeset
    return s
