"""Temporal graph transforms.

``propagate_timestamp_to_edges`` mirrors dgf/src/transform/temporal.py:24-131
(same signature, same checks and messages, same returned graph and schema);
the per-edge max of the endpoint creation times runs on the GPU
(dgfx_edge_timestamps). ``edge_timestamps`` is the device-level entry point
for callers that hold the adjacency and node times as CUDA tensors.
"""

from __future__ import annotations

import ctypes
from typing import List, Optional

import numpy as np

from distributed_graph_flow_b200 import _native
from distributed_graph_flow_b200.data import in_memory_graph
from distributed_graph_flow_b200.data import schema as schema_lib
from distributed_graph_flow_b200.util import temporal as temporal_util


def edge_timestamps(src_ts, dst_ts, src, dst, stream=None):
    """int64 CUDA tensor of edge times: max(src_ts[src], dst_ts[dst]), or the
    endpoint time that is given when the other is None. All inputs are CUDA
    tensors (int64 ids; times of any integer type, widened to int64)."""
    torch = _native.require_cuda()
    ref = src if src is not None else dst
    n = int(ref.numel())
    dev = ref.device
    out = torch.empty(max(n, 1), dtype=torch.int64, device=dev)[:n]
    ws = torch.empty(1, dtype=torch.int64, device=dev)

    def prep(t):
        return None if t is None else t.to(device=dev, dtype=torch.int64).contiguous()

    s_ts, d_ts = prep(src_ts), prep(dst_ts)
    s_id = prep(src) if s_ts is not None else None
    d_id = prep(dst) if d_ts is not None else None
    status = _native.lib().dgfx_edge_timestamps(
        _native.ptr(s_ts), 0 if s_ts is None else int(s_ts.numel()), _native.ptr(d_ts),
        0 if d_ts is None else int(d_ts.numel()), _native.ptr(s_id), _native.ptr(d_id), n, _native.ptr(out),
        _native.ptr(ws), _native.stream_handle(stream))
    if status == _native.ERR_INVALID_ARGUMENT and "out of bounds" in _native.last_error():
        raise IndexError(_native.last_error())
    _native.check(status)
    return out


def _edge_timestamps_host(src_ts, tgt_ts, adjacency) -> np.ndarray:
    """numpy in, numpy out (device compute); output dtype as numpy's own
    ``np.maximum`` / fancy indexing would give."""
    torch = _native.require_cuda()
    dev = torch.device("cuda", torch.cuda.current_device())
    src_idx = np.asarray(adjacency[0])
    tgt_idx = np.asarray(adjacency[1])
    if src_ts is not None and tgt_ts is not None:
        out_dtype = np.result_type(np.asarray(src_ts).dtype, np.asarray(tgt_ts).dtype)
    else:
        out_dtype = np.asarray(src_ts if src_ts is not None else tgt_ts).dtype

    def dev_t(a):
        return None if a is None else torch.from_numpy(np.ascontiguousarray(a, dtype=np.int64)).to(dev)

    out = edge_timestamps(dev_t(src_ts), dev_t(tgt_ts), dev_t(src_idx), dev_t(tgt_idx))
    return out.cpu().numpy().astype(out_dtype, copy=False)


def propagate_timestamp_to_edges(
    graph: in_memory_graph.InMemoryGraph,
    schema: schema_lib.GraphSchema,
    target_edgesets: Optional[List[str]] = None,
    target_feature: str = "timestamps",
) -> tuple[in_memory_graph.InMemoryGraph, schema_lib.GraphSchema]:
    """Adds the edge feature ``target_feature`` = max of the endpoint node
    creation times (or the one endpoint that has one) to every edge set of
    ``target_edgesets`` (all edge sets if None), marked as the edge set's
    creation time in the returned schema."""
    new_edge_sets = dict(graph.edge_sets)
    new_edge_set_schemas = dict(schema.edge_sets)

    def get_node_ts(nodeset_name: str):
        feat_name = temporal_util.creation_time_feature_name(schema.node_sets[nodeset_name].features)
        if feat_name and feat_name in graph.node_sets[nodeset_name].features:
            return (graph.node_sets[nodeset_name].features[feat_name],
                    schema.node_sets[nodeset_name].features[feat_name].format)
        return None, None

    for edgeset_name, edgeset_schema in schema.edge_sets.items():
        if target_edgesets is not None and edgeset_name not in target_edgesets:
            continue
        if target_feature in edgeset_schema.features:
            raise ValueError(f"Target feature '{target_feature}' already exists in edgeset '{edgeset_name}'.")
        src_ts, src_format = get_node_ts(edgeset_schema.source)
        tgt_ts, tgt_format = get_node_ts(edgeset_schema.target)
        if src_ts is None and tgt_ts is None:
            raise ValueError(
                f"Neither source nodeset '{edgeset_schema.source}' nor target nodeset"
                f" '{edgeset_schema.target}' has timestamps for edgeset '{edgeset_name}'."
            )
        edgeset_value = graph.edge_sets[edgeset_name]
        edge_ts = _edge_timestamps_host(src_ts, tgt_ts, edgeset_value.adjacency)
        ts_format = src_format if src_ts is not None else tgt_format
        new_edge_sets[edgeset_name] = in_memory_graph.InMemoryEdgeSet(
            adjacency=edgeset_value.adjacency,
            features={**edgeset_value.features, target_feature: edge_ts},
        )
        new_edge_set_schemas[edgeset_name] = schema_lib.EdgeSchema(
            source=edgeset_schema.source,
            target=edgeset_schema.target,
            features={
                **edgeset_schema.features,
                target_feature: schema_lib.FeatureSchema(
                    format=ts_format,
                    semantic=schema_lib.FeatureSemantic.TIMESTAMP,
                    is_creation_time=True,
                ),
            },
        )
    return (
        in_memory_graph.InMemoryGraph(node_sets=graph.node_sets, edge_sets=new_edge_sets),
        schema_lib.GraphSchema(node_sets=schema.node_sets, edge_sets=new_edge_set_schemas),
    )
