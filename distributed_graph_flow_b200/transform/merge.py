"""Batching of sampled graphs.

``merge_graphs`` keeps the contract of dgf/src/transform/merge.py:33-232
(same arguments, returned graph and offsets, padding rules and
``InsufficientPaddingError`` messages): per-node-set offsets are the cumsum of
the graphs' node counts, every adjacency is shifted by its graph's offsets,
and with ``padding`` each set is filled up to its fixed size (zero / empty
feature rows, padding edges between the sets' last nodes, the sentinels).
The adjacency arithmetic runs on the GPU (``dgfx_merge_edgeset``); feature
columns are concatenated as they come (they may be byte strings).

``merge_batch`` does the same for a device-resident ``MergedBatch`` straight
from the sampler, without leaving the GPU.
"""

from __future__ import annotations

from typing import Dict, List, Optional, Tuple

import numpy as np

from distributed_graph_flow_b200 import _native
from distributed_graph_flow_b200.data import in_memory_graph
from distributed_graph_flow_b200.data import padding as padding_lib
from distributed_graph_flow_b200.data import schema as schema_lib


class InsufficientPaddingError(ValueError):
    pass


def _check_node_padding(node_set_name: str, num_real: int, padding) -> int:
    num_nodes = padding.node_sets[node_set_name].num_nodes
    if num_nodes - num_real < 1:
        raise InsufficientPaddingError(
            f"Padding for node set '{node_set_name}' is insufficient. Required"
            f" at least {num_real + 1} nodes (including the sentinel"
            f" node), but the padder only defines {num_nodes}."
        )
    return num_nodes


def _check_edge_padding(edge_set_name: str, num_real: int, padding) -> int:
    num_edges = padding.edge_sets[edge_set_name].num_edges
    if num_edges - num_real < 0:
        raise InsufficientPaddingError(
            f"Padding for edge set '{edge_set_name}' is insufficient. "
            f"Required at least {num_real} edges, but the padder only "
            f"defines {num_edges}."
        )
    return num_edges


def _merged_adjacency(node_offsets, edge_offsets, edge_src, edge_dst, batch: int, e: int, s_src: int, s_dst: int,
                      num_out: int, sentinel_src: int, sentinel_dst: int):
    """[2, num_out] int64 CUDA tensor (dgfx_merge_edgeset)."""
    torch = _native.require_cuda()
    dev = node_offsets.device
    out = torch.empty((2, max(num_out, 1)), dtype=torch.int64, device=dev)[:, :num_out]
    _native.check(_native.lib().dgfx_merge_edgeset(
        _native.ptr(node_offsets), _native.ptr(edge_offsets), _native.ptr(edge_src), _native.ptr(edge_dst), batch, e,
        s_src, s_dst, num_out, sentinel_src, sentinel_dst, _native.elem_ptr(out.reshape(-1), 0),
        _native.elem_ptr(out.reshape(-1), num_out) if num_out > 0 else None, _native.stream_handle()))
    return out


def _pad_rows(values: List[np.ndarray], count: int) -> np.ndarray:
    first = values[0]
    shape = list(first.shape)
    shape[0] = count
    if first.dtype.type is np.bytes_:
        return np.full(shape, b"", dtype=first.dtype)
    return np.zeros(shape=shape, dtype=first.dtype)


def merge_graphs(
    graphs: List[in_memory_graph.InMemoryGraph],
    schema: schema_lib.GraphSchema,
    padding: Optional[padding_lib.Padding],
    sentinel_offset: bool = True,
) -> Tuple[in_memory_graph.InMemoryGraph, Dict[str, np.ndarray]]:
    """Concatenates ``graphs`` (node indices offset per graph), optionally
    padded; returns the merged graph and, per node set, the first node of
    each graph (plus the sentinel offset when ``sentinel_offset``)."""
    if not graphs:
        return in_memory_graph.InMemoryGraph({}, {}), {}
    B = len(graphs)
    ns_names = list(schema.node_sets)
    es_names = list(schema.edge_sets)
    node_set_offsets: Dict[str, np.ndarray] = {}
    for name in ns_names:
        counts = np.array([g.node_sets[name].num_nodes for g in graphs], dtype=np.int32)
        node_set_offsets[name] = np.insert(np.cumsum(counts), 0, 0)

    merged_node_sets = {}
    for name, ns_schema in schema.node_sets.items():
        num_real = int(node_set_offsets[name][-1])
        num_nodes = num_real
        if padding:
            num_nodes = _check_node_padding(name, num_real, padding)
        feats = {}
        for feature_name in ns_schema.features:
            values = [g.node_sets[name].features[feature_name] for g in graphs]
            if padding:
                values.append(_pad_rows(values, num_nodes - num_real))
            feats[feature_name] = np.concatenate(values, axis=0)
        merged_node_sets[name] = in_memory_graph.InMemoryNodeSet(features=feats, num_nodes=num_nodes)

    # Edge counts and padding checks (host metadata), then the device layout
    # of the batch: offsets set-major then graph (trailing total), adjacencies
    # concatenated in the same order.
    edge_plan = {}
    for name, es_schema in schema.edge_sets.items():
        num_real = sum(int(np.asarray(g.edge_sets[name].adjacency).reshape(2, -1).shape[1]) for g in graphs)
        if padding:
            edge_plan[name] = (num_real, _check_edge_padding(name, num_real, padding),
                               padding.node_sets[es_schema.source].num_nodes - 1,
                               padding.node_sets[es_schema.target].num_nodes - 1)
        else:
            edge_plan[name] = (num_real, num_real, 0, 0)
    torch = _native.require_cuda()
    dev = torch.device("cuda", torch.cuda.current_device())
    ns_index = {n: i for i, n in enumerate(ns_names)}
    node_off = np.zeros(len(ns_names) * B + 1, dtype=np.int64)
    acc = 0
    for s, name in enumerate(ns_names):
        for i, g in enumerate(graphs):
            node_off[s * B + i] = acc
            acc += int(g.node_sets[name].num_nodes)
    node_off[-1] = acc
    edge_off = np.zeros(len(es_names) * B + 1, dtype=np.int64)
    srcs, dsts = [], []
    acc = 0
    for e, name in enumerate(es_names):
        for i, g in enumerate(graphs):
            adj = np.asarray(g.edge_sets[name].adjacency, dtype=np.int64).reshape(2, -1)
            edge_off[e * B + i] = acc
            acc += adj.shape[1]
            srcs.append(adj[0])
            dsts.append(adj[1])
    edge_off[-1] = acc
    d_node_off = torch.from_numpy(node_off).to(dev)
    d_edge_off = torch.from_numpy(edge_off).to(dev)
    d_src = torch.from_numpy(np.concatenate(srcs) if srcs else np.zeros(0, np.int64)).to(dev)
    d_dst = torch.from_numpy(np.concatenate(dsts) if dsts else np.zeros(0, np.int64)).to(dev)

    merged_edge_sets = {}
    for e, (name, es_schema) in enumerate(schema.edge_sets.items()):
        num_real, num_edges, sentinel_src, sentinel_dst = edge_plan[name]
        adjacency = _merged_adjacency(d_node_off, d_edge_off, d_src, d_dst, B, e, ns_index[es_schema.source],
                                      ns_index[es_schema.target], num_edges, sentinel_src, sentinel_dst)
        feats = {}
        for feature_name in es_schema.features:
            if graphs and feature_name not in graphs[0].edge_sets[name].features:
                continue
            values = [g.edge_sets[name].features[feature_name] for g in graphs]
            if padding:
                values.append(_pad_rows(values, num_edges - num_real))
            feats[feature_name] = np.concatenate(values, axis=0)
        merged_edge_sets[name] = in_memory_graph.InMemoryEdgeSet(adjacency=adjacency.cpu().numpy(), features=feats)

    if not sentinel_offset:
        node_set_offsets = {k: v[:-1] for k, v in node_set_offsets.items()}
    return in_memory_graph.InMemoryGraph(merged_node_sets, merged_edge_sets), node_set_offsets


def merge_batch(batch, schema: schema_lib.GraphSchema, padding: Optional[padding_lib.Padding] = None,
                sentinel_offset: bool = True):
    """``merge_graphs`` for a sampler's device-resident ``MergedBatch``.

    Returns (node_ids, adjacency, node_set_offsets), dicts of CUDA tensors:
    node_ids[ns] the merged "#idx" column (padding rows 0), adjacency[es]
    [2, E] int64 in merged ids (padding edges between the sentinels),
    node_set_offsets[ns] the first node of each sample (+ sentinel offset).
    One device-to-host read of the offsets checks the padding."""
    torch = _native.require_cuda()
    B = batch.B
    node_off_h = batch.node_offsets.cpu().numpy()
    edge_off_h = batch.edge_offsets.cpu().numpy()
    ns_index = {n: i for i, n in enumerate(batch.nodeset_names)}
    node_ids, offsets = {}, {}
    for s, name in enumerate(batch.nodeset_names):
        lo, hi = int(node_off_h[s * B]), int(node_off_h[(s + 1) * B])
        num_real = hi - lo
        num_nodes = _check_node_padding(name, num_real, padding) if padding else num_real
        col = torch.zeros(num_nodes, dtype=torch.int64, device=batch.node_ids.device)
        col[:num_real] = batch.node_ids[lo:hi]
        node_ids[name] = col
        off = batch.node_offsets[s * B:(s + 1) * B + 1] - lo
        offsets[name] = off if sentinel_offset else off[:-1]
    adjacency = {}
    for e, name in enumerate(batch.edgeset_names):
        es_schema = schema.edge_sets[name]
        num_real = int(edge_off_h[(e + 1) * B] - edge_off_h[e * B])
        num_edges, sentinel_src, sentinel_dst = num_real, 0, 0
        if padding:
            num_edges = _check_edge_padding(name, num_real, padding)
            sentinel_src = padding.node_sets[es_schema.source].num_nodes - 1
            sentinel_dst = padding.node_sets[es_schema.target].num_nodes - 1
        adjacency[name] = _merged_adjacency(batch.node_offsets, batch.edge_offsets, batch.edge_src, batch.edge_dst, B,
                                            e, ns_index[es_schema.source], ns_index[es_schema.target], num_edges,
                                            sentinel_src, sentinel_dst)
    return node_ids, adjacency, offsets
