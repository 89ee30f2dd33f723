"""Causal slicing of timeseries features on the GPU.

``filter_timeseries_by_timestamp`` keeps the contract of
dgf/src/sampling/temporal.py:66-130: in every node set and edge set of a
graph, each group of ``is_timeseries`` features that has a timestamp series
is cut, per entity, to the entries with timestamp <= ``target_timestamp``
(``np.searchsorted(times, target, side="right")``), keeping the most recent
``max_timeseries_len`` of them; features are replaced by object arrays of
per-entity arrays; groups without a timestamp series are left alone.

``TimeseriesSlicer`` holds a feature set's series in HBM as ragged arrays
(row offsets + packed values, uploaded once) and slices any list of entities,
each with its own cutoff: one ``dgfx_timeseries_windows`` launch finds every
window by binary search over the timestamp rows, one
``dgfx_gather_segments`` launch per feature copies the windows. The sampler
uses it with each sampled node's seed timestamp.
"""

from __future__ import annotations

import ctypes
from typing import Dict, List, Optional, Union

import numpy as np

from distributed_graph_flow_b200 import _native
from distributed_graph_flow_b200.data import in_memory_graph
from distributed_graph_flow_b200.util import temporal as temporal_util


class _Ragged:
    """One feature's per-entity series: values packed in HBM (bytes), row
    offsets in elements on the device and on the host."""

    def __init__(self, column, device, dtype=None):
        torch = _native.require_cuda()
        col = np.asarray(column)
        if col.dtype != object and col.ndim >= 2:
            rows = [col[i] for i in range(col.shape[0])]
        else:
            rows = [np.asarray(x) for x in col]
        n = len(rows)
        first = next((r for r in rows if r.size), rows[0] if rows else np.zeros(0, np.int64))
        self.dtype = np.dtype(dtype) if dtype is not None else np.asarray(first).dtype
        self.inner = tuple(np.asarray(first).shape[1:])
        lengths = np.array([r.shape[0] if r.ndim else 0 for r in rows], np.int64)
        self.offsets_host = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
        total = int(self.offsets_host[-1])
        if total:
            values = np.concatenate([np.asarray(r, dtype=self.dtype).reshape((-1,) + self.inner) for r in rows if r.size])
        else:
            values = np.zeros((0,) + self.inner, self.dtype)
        self.elem_bytes = max(1, self.dtype.itemsize * int(np.prod(self.inner, dtype=np.int64)))
        raw = np.ascontiguousarray(values).view(np.uint8).reshape(-1)
        self.values = torch.from_numpy(raw.copy() if raw.size else np.zeros(16, np.uint8)).to(device)
        self.offsets = torch.from_numpy(self.offsets_host).to(device)
        self.n = n


def _require_integer_times(name: str, column) -> None:
    """Timestamp series are searched as int64: a float series would be
    truncated (an entry at t = 1.5 would pass a cutoff of 1), so it is
    rejected instead."""
    col = np.asarray(column)
    kinds = {col.dtype.kind} if col.dtype != object else {np.asarray(r).dtype.kind for r in col if np.size(r)}
    if kinds - set("iub"):
        raise ValueError(f"Timestamp feature `{name}` must hold integer timestamps, got dtype kinds {sorted(kinds)}.")


class TimeseriesSlicer:
    """The timestamped timeseries groups of one feature set, in HBM."""

    def __init__(self, features: Dict[str, np.ndarray], specs: List[temporal_util.TimeseriesGroupSpec], device=None):
        for g in specs:
            if g.timestamp_feature_name is not None:
                _require_integer_times(g.timestamp_feature_name, features[g.timestamp_feature_name])
        torch = _native.require_cuda()
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.groups = []
        for g in specs:
            if g.timestamp_feature_name is None:
                continue
            # Timestamp rows must be sorted (np.searchsorted's contract).
            times = _Ragged(np.asarray(features[g.timestamp_feature_name]), self.device, dtype=np.int64)
            series = {f: _Ragged(np.asarray(features[f]), self.device) for f in g.feature_names}
            self.groups.append((g.timestamp_feature_name, times, series))
        self._ws = torch.empty(64, dtype=torch.uint8, device=self.device)

    @property
    def feature_names(self) -> List[str]:
        return [f for _, _, series in self.groups for f in series]

    def slice(self, rows: np.ndarray, cutoffs: np.ndarray, max_len: Optional[int]) -> Dict[str, np.ndarray]:
        """{feature: object array [len(rows)] of each row's causal window}."""
        torch = _native.require_cuda()
        lib = _native.lib()
        if max_len is not None and max_len < 0:
            # numpy's times[max(0, end - max_len):end] is empty for a negative
            # length, exactly as a cap of 0 is.
            max_len = 0
        rows = np.ascontiguousarray(np.asarray(rows, np.int64))
        cutoffs = np.ascontiguousarray(np.asarray(cutoffs, np.int64))
        n = len(rows)
        out = {}
        sh = _native.stream_handle()
        with torch.cuda.device(self.device):
            d_rows = torch.from_numpy(rows).to(self.device)
            d_cut = torch.from_numpy(cutoffs).to(self.device)
            for _, times, series in self.groups:
                rel = torch.empty(max(1, n), dtype=torch.int64, device=self.device)
                ln = torch.empty(max(1, n), dtype=torch.int64, device=self.device)
                _native.check(lib.dgfx_timeseries_windows(
                    _native.ptr(times.offsets), _native.ptr(times.values), times.n, _native.ptr(d_rows),
                    _native.ptr(d_cut), n, -1 if max_len is None else int(max_len), _native.ptr(rel), _native.ptr(ln),
                    _native.ptr(self._ws), sh))
                rel_h = rel[:n].cpu().numpy()
                end_h = rel_h + ln[:n].cpu().numpy()
                for fname, r in series.items():
                    # numpy slicing of each feature's own row: clip to its length.
                    rowlen = r.offsets_host[rows + 1] - r.offsets_host[rows]
                    start = np.minimum(rel_h, rowlen)
                    length = np.maximum(0, np.minimum(end_h, rowlen) - start)
                    out_off = np.concatenate([[0], np.cumsum(length)]).astype(np.int64)
                    total = int(out_off[-1])
                    dst = torch.empty(max(16, total * r.elem_bytes), dtype=torch.uint8, device=self.device)
                    src = torch.from_numpy(np.ascontiguousarray(r.offsets_host[rows] + start)).to(self.device)
                    d_len = torch.from_numpy(np.ascontiguousarray(length)).to(self.device)
                    d_off = torch.from_numpy(out_off[:-1].copy()).to(self.device)
                    _native.check(lib.dgfx_gather_segments(
                        _native.ptr(r.values), r.elem_bytes, _native.ptr(src), _native.ptr(d_len), _native.ptr(d_off),
                        n, _native.ptr(dst), sh))
                    packed = dst[:total * r.elem_bytes].cpu().numpy().view(r.dtype).reshape((total,) + r.inner)
                    col = np.empty(n, dtype=object)
                    for i in range(n):
                        col[i] = packed[out_off[i]:out_off[i + 1]]
                    out[fname] = col
        return out


def _filter_entity_set(entity, specs, num_entities: int, target_timestamp: int,
                       max_timeseries_len: Optional[int]) -> None:
    slicer = TimeseriesSlicer(entity.features, specs)
    if not slicer.groups:
        return
    rows = np.arange(num_entities, dtype=np.int64)
    sliced = slicer.slice(rows, np.full(num_entities, int(target_timestamp), np.int64), max_timeseries_len)
    entity.features.update(sliced)


def filter_timeseries_by_timestamp(
    graph: in_memory_graph.InMemoryGraph,
    schema_cache: temporal_util.TimeseriesSchemaCache,
    target_timestamp: Union[int, np.integer],
    max_timeseries_len: Optional[int] = None,
) -> None:
    """Causally slices the graph's timestamped timeseries features in place
    (see the module docstring)."""
    for name, specs in schema_cache.node_sets.items():
        ns = graph.node_sets.get(name)
        if ns and ns.num_nodes:
            _filter_entity_set(ns, specs, ns.num_nodes, target_timestamp, max_timeseries_len)
    for name, specs in schema_cache.edge_sets.items():
        es = graph.edge_sets.get(name)
        if es and es.num_edges():
            _filter_entity_set(es, specs, es.num_edges(), target_timestamp, max_timeseries_len)
