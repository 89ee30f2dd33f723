"""In-memory sampler: DGF's Python sampling API on B200 kernels.

``create_sampler`` / ``Sampler.sample`` keep the reference's names, arguments,
defaults, outputs and error messages (dgf/src/sampling/in_memory_sampler.py:
28-445): ``sample(seed_node_idxs, seed_timestamps=None,
masked_edge_idxs=None)`` returns one ``InMemoryGraph`` per seed (or a single
graph for an int seed) holding the sampled node features, optionally the
"#idx" node ids, and [2, E] int64 local-id adjacencies.

Underneath, sampling runs in ``dgfx_sampler_sample`` (one CTA per seed) and
the feature gather of ``add_features_to_samples`` runs as one
``dgfx_gather_rows`` launch per (node set, feature) over the merged batch,
from feature tables uploaded to HBM once. ``sample_batch`` is the zero-copy
path for a GNN on the same device: the merged batch and its features stay in
HBM.

With ``slice_timeseries_by_seed`` and seed timestamps, every sampled node's
``is_timeseries`` features are cut to its seed's past on the device
(``sampling.temporal``).

Extension beyond the reference: ``sampling_mode=MODE_MOST_RECENT`` (newest-k
temporal neighbours).
"""

from __future__ import annotations

import os
from typing import Dict, List, Optional, Union

import numpy as np

from distributed_graph_flow_b200 import _native
from distributed_graph_flow_b200.data import in_memory_graph as in_memory_graph_lib
from distributed_graph_flow_b200.data import schema as schema_lib
from distributed_graph_flow_b200.sampling import _in_memory_sampler_ext
from distributed_graph_flow_b200.sampling import config as config_lib
from distributed_graph_flow_b200.sampling import temporal as sampling_temporal
from distributed_graph_flow_b200.util import temporal as temporal_util

MODE_RANDOM = _native.MODE_RANDOM
MODE_FIRST = _native.MODE_FIRST
MODE_MOST_RECENT = _native.MODE_MOST_RECENT


def _is_device_type(arr: np.ndarray) -> bool:
    return arr.dtype.kind in "biuf" and arr.ndim >= 1


class DeviceFeatureStore:
    """Node features resident in HBM as rows padded to 16 bytes.

    Any numeric dtype and per-node shape is stored as raw bytes so a single
    vectorised gather kernel serves all of them. Non-numeric (object, string)
    features have no device representation and stay in host memory.
    """

    def __init__(self, graph: in_memory_graph_lib.InMemoryGraph, device):
        torch = _native.require_cuda()
        self.device = device
        self.tables: Dict[str, Dict[str, tuple]] = {}
        self.host_only: Dict[str, Dict[str, np.ndarray]] = {}
        for ns_name, ns in graph.node_sets.items():
            self.tables[ns_name] = {}
            self.host_only[ns_name] = {}
            for fname, full in ns.features.items():
                arr = np.asarray(full)
                if not _is_device_type(arr):
                    self.host_only[ns_name][fname] = arr
                    continue
                arr = np.ascontiguousarray(arr)
                n = arr.shape[0]
                row_bytes = arr.dtype.itemsize * int(np.prod(arr.shape[1:], dtype=np.int64))
                padded = (row_bytes + 15) // 16 * 16
                raw = np.zeros((n, padded), dtype=np.uint8)
                if n and row_bytes:
                    raw[:, :row_bytes] = arr.reshape(n, -1).view(np.uint8).reshape(n, row_bytes)
                table = torch.from_numpy(raw).to(device)
                self.tables[ns_name][fname] = (table, row_bytes, padded, arr.dtype, arr.shape[1:])

    def gather(self, ns_name: str, node_ids, stream=None) -> Dict[str, tuple]:
        """Gathers every device feature of a node set for int64 node_ids
        (device). Returns {name: (padded_rows_device, row_bytes, dtype, shape)}."""
        torch = _native.require_cuda()
        out = {}
        n = int(node_ids.numel())
        for fname, (table, row_bytes, padded, dtype, shape) in self.tables.get(ns_name, {}).items():
            rows = torch.empty((max(n, 1), padded), dtype=torch.uint8, device=self.device)
            _native.check(
                _native.lib().dgfx_gather_rows(
                    _native.ptr(table), int(table.shape[0]), padded, _native.ptr(node_ids), n, _native.ptr(rows),
                    _native.stream_handle(stream),
                )
            )
            out[fname] = (rows[:n], row_bytes, dtype, shape)
        return out

    @staticmethod
    def to_numpy(rows_host: np.ndarray, row_bytes: int, dtype, shape) -> np.ndarray:
        n = rows_host.shape[0]
        raw = np.ascontiguousarray(rows_host[:, :row_bytes])
        return raw.view(dtype).reshape((n,) + tuple(shape))


class SampledBatch:
    """Merged batch of one ``sample_batch`` call, resident in HBM.

    ``merged`` is the sampler output (node ids / local-id edges with per-seed
    offsets, see ``_in_memory_sampler_ext.MergedBatch``); ``features[ns][f]``
    holds the gathered rows of node set ns as a [num_nodes, ...] tensor of the
    feature's dtype (numeric features only).
    """

    def __init__(self, merged, features):
        self.merged = merged
        self.features = features


class Sampler:
    """Sampler for generating subgraphs from an in-memory graph."""

    def __init__(
        self,
        cc_sampler,
        full_graph: in_memory_graph_lib.InMemoryGraph,
        return_features: bool,
        return_node_idxs: bool,
        schema: Optional[schema_lib.GraphSchema] = None,
        slice_timeseries_by_seed: bool = True,
        max_timeseries_len: Optional[int] = None,
        has_temporal_edgesets: bool = False,
    ):
        self._cc_sampler = cc_sampler
        self._full_graph = full_graph
        self._return_features = return_features
        self._return_node_idxs = return_node_idxs
        self._schema = schema
        self._slice_timeseries_by_seed = slice_timeseries_by_seed
        self._max_timeseries_len = max_timeseries_len
        self._has_temporal_edgesets = has_temporal_edgesets
        self._store: Optional[DeviceFeatureStore] = None
        self._ts_cache = None
        self._slicers: Dict[str, "sampling_temporal.TimeseriesSlicer"] = {}

    def set_return_options(self, return_features: bool, return_node_idxs: bool):
        self._return_features = return_features
        self._return_node_idxs = return_node_idxs

    def _feature_store(self) -> DeviceFeatureStore:
        if self._store is None:
            self._store = DeviceFeatureStore(self._full_graph, self._cc_sampler._device)
        return self._store

    @staticmethod
    def _as_int64(value, name: str):
        if isinstance(value, (int, np.integer)) and not isinstance(value, bool):
            return np.array([value], dtype=np.int64), True
        if isinstance(value, list):
            return np.array(value, dtype=np.int64), False
        if isinstance(value, np.ndarray):
            return value.astype(np.int64, copy=False), False
        raise ValueError(f"{name} must be an int, a list of ints, or a numpy array, but got {type(value)!r}.")

    def _normalise(self, seed_node_idxs, seed_timestamps, masked_edge_idxs):
        seeds, single = self._as_int64(seed_node_idxs, "seed_node_idxs")
        ts = masks = None
        if seed_timestamps is not None:
            ts, _ = self._as_int64(seed_timestamps, "seed_timestamps")
            if len(ts) != len(seeds):
                raise ValueError("seed_timestamps must have the same length as seed_node_idxs")
        if masked_edge_idxs is not None:
            masks, _ = self._as_int64(masked_edge_idxs, "masked_edge_idxs")
            if len(masks) != len(seeds):
                raise ValueError("masked_edge_idxs must have the same length as seed_node_idxs")
        return seeds, ts, masks, single

    def sample(
        self,
        seed_node_idxs: Union[int, List[int], np.ndarray],
        seed_timestamps: Optional[Union[int, List[int], np.ndarray]] = None,
        masked_edge_idxs: Optional[Union[int, List[int], np.ndarray]] = None,
    ):
        """Samples one subgraph per seed (see module docstring)."""
        seeds, ts, masks, single = self._normalise(seed_node_idxs, seed_timestamps, masked_edge_idxs)
        cc = self._cc_sampler
        d_seeds = cc._to_device(seeds, "seeds")
        d_ts = cc._to_device(ts, "ts") if (ts is not None and self._has_temporal_edgesets) else None
        d_masks = cc._to_device(masks, "masks")
        merged = cc.sample_merged(d_seeds, d_ts, d_masks)
        host = _in_memory_sampler_ext.batch_to_host(merged)
        graphs = _in_memory_sampler_ext.export_graphs(merged, host)
        self._finalize(merged, host, graphs)
        if self._slice_timeseries_by_seed and self._return_features:
            self._slice_timeseries(merged, host, graphs, ts)
        return graphs[0] if single else graphs

    def _timeseries_cache(self):
        if self._ts_cache is None and self._schema is not None:
            self._ts_cache = temporal_util.extract_timeseries_schema_cache(self._schema)
        return self._ts_cache

    def _slice_timeseries(self, merged, host, graphs, ts):
        """Causal slicing of every sampled node's timeseries features by its
        seed's timestamp (in_memory_sampler.py:270-310), on the device
        (sampling.temporal.TimeseriesSlicer over the whole merged batch)."""
        cache = self._timeseries_cache()
        if ts is None:
            if cache is not None and cache.has_timeseries:
                raise ValueError(
                    "`seed_timestamps` must be provided when `slice_timeseries_by_seed=True` and the schema contains"
                    " `is_timeseries=True` features."
                )
            return
        if self._schema is None:
            raise ValueError(
                "schema must be provided when `slice_timeseries_by_seed=True` and `seed_timestamps` are passed."
            )
        node_ids_host, node_off = host[0], host[1]
        B = merged.B
        for s, ns_name in enumerate(merged.nodeset_names):
            specs = cache.node_sets.get(ns_name)
            if not specs or ns_name not in self._full_graph.node_sets:
                continue
            slicer = self._slicers.get(ns_name)
            if slicer is None:
                slicer = sampling_temporal.TimeseriesSlicer(self._full_graph.node_sets[ns_name].features, specs,
                                                            self._cc_sampler._device)
                self._slicers[ns_name] = slicer
            if not slicer.groups:
                continue
            a = int(node_off[s * B])
            counts = np.diff(node_off[s * B:(s + 1) * B + 1])
            cutoffs = np.repeat(np.asarray(ts, np.int64), counts)
            sliced = slicer.slice(node_ids_host[a:int(node_off[(s + 1) * B])], cutoffs, self._max_timeseries_len)
            for i, g in enumerate(graphs):
                lo, hi = int(node_off[s * B + i]) - a, int(node_off[s * B + i + 1]) - a
                for fname, col in sliced.items():
                    g.node_sets[ns_name].features[fname] = col[lo:hi]

    def _finalize(self, merged, host, graphs):
        """Adds features (gathered on device over the merged batch) and drops
        "#idx" unless requested (add_features_to_samples semantics)."""
        if not (self._return_features or not self._return_node_idxs):
            return
        node_ids_host, node_off, _, _ = host
        B = merged.B
        per_ns = {}
        if self._return_features:
            store = self._feature_store()
            for s, ns_name in enumerate(merged.nodeset_names):
                a, b = int(node_off[s * B]), int(node_off[(s + 1) * B])
                gathered = store.gather(ns_name, merged.node_ids[a:b])
                feats = {}
                for fname, (rows, row_bytes, dtype, shape) in gathered.items():
                    feats[fname] = DeviceFeatureStore.to_numpy(rows.cpu().numpy(), row_bytes, dtype, shape)
                for fname, arr in store.host_only.get(ns_name, {}).items():
                    feats[fname] = arr[node_ids_host[a:b]]
                per_ns[ns_name] = (a, feats)
        for i, g in enumerate(graphs):
            for s, ns_name in enumerate(merged.nodeset_names):
                ns = g.node_sets[ns_name]
                if not self._return_node_idxs:
                    del ns.features["#idx"]
                if self._return_features and ns_name in per_ns:
                    base, feats = per_ns[ns_name]
                    a, b = int(node_off[s * B + i]) - base, int(node_off[s * B + i + 1]) - base
                    for fname, arr in feats.items():
                        ns.features[fname] = arr[a:b]

    def sample_batch(self, seeds, seed_timestamps=None, masked_edge_idxs=None, features: bool = True, stream=None,
                     check: bool = True) -> SampledBatch:
        """Device path: int64 CUDA tensors in, a SampledBatch in HBM out.

        No host synchronisation when check=False: each node set's features
        are gathered with bounds read from the device offsets into a
        capacity-sized buffer (B * tree positions rows); the valid rows are
        [0, node_offsets[(s+1)B] - node_offsets[sB]).
        """
        torch = _native.require_cuda()
        cc = self._cc_sampler
        merged = cc.sample_merged(seeds, seed_timestamps, masked_edge_idxs, stream=stream, check=check)
        feats = {}
        if features:
            store = self._feature_store()
            B = merged.B
            cap = B * cc.tree_size
            sh = _native.stream_handle(stream)
            for s, ns_name in enumerate(merged.nodeset_names):
                tables = store.tables.get(ns_name, {})
                if not tables:
                    continue
                off = merged.node_offsets
                feats[ns_name] = {}
                for fname, (table, row_bytes, padded, dtype, shape) in tables.items():
                    rows = torch.empty((max(cap, 1), padded), dtype=torch.uint8, device=store.device)
                    _native.check(
                        _native.lib().dgfx_gather_rows_ranged(
                            _native.ptr(table), int(table.shape[0]), padded, _native.ptr(merged.node_ids),
                            _native.elem_ptr(off, s * B), _native.elem_ptr(off, (s + 1) * B), cap,
                            _native.ptr(rows), sh,
                        )
                    )
                    feats[ns_name][fname] = (rows, row_bytes, dtype, shape)
        return SampledBatch(merged, feats)

    def subgraph(self, seed_node_idxs: List[int]):
        graph = self._cc_sampler.SubGraph(seed_node_idxs)
        self._finalize_simple([graph])
        return graph

    def multisubgraph(self, seed_node_idxs: List[int]):
        graphs = self._cc_sampler.MultiSubGraphs(seed_node_idxs)
        self._finalize_simple(graphs)
        return graphs

    def _finalize_simple(self, graphs):
        add_features_to_samples(self._full_graph, graphs, self._return_features, self._return_node_idxs)

    def __str__(self) -> str:
        return str(self._cc_sampler)


def add_features_to_samples(
    full_graph: in_memory_graph_lib.InMemoryGraph,
    samples: List[in_memory_graph_lib.InMemoryGraph],
    return_features: bool,
    return_node_idxs: bool,
):
    """Adds full-graph features to sampled graphs in place and drops "#idx"
    unless requested (in_memory_sampler.py:313-346). Numeric features are
    gathered on the device, one launch per (node set, feature) over all
    samples."""
    if not (return_features or not return_node_idxs):
        return
    store = DeviceFeatureStore(full_graph, _native.require_cuda().device("cuda")) if return_features else None
    torch = _native.require_cuda()
    names = list(full_graph.node_sets)
    for ns_name in names:
        idx_lists = [g.node_sets[ns_name].features["#idx"] for g in samples if ns_name in g.node_sets]
        if return_features:
            cat = np.concatenate(idx_lists) if idx_lists else np.zeros(0, np.int64)
            d_ids = torch.from_numpy(np.ascontiguousarray(cat.astype(np.int64))).to(store.device)
            gathered = store.gather(ns_name, d_ids)
            feats = {f: DeviceFeatureStore.to_numpy(r.cpu().numpy(), rb, dt, sh) for f, (r, rb, dt, sh) in gathered.items()}
            for f, arr in store.host_only.get(ns_name, {}).items():
                feats[f] = arr[cat]
        off = 0
        for g in samples:
            if ns_name not in g.node_sets:
                continue
            ns = g.node_sets[ns_name]
            idx = ns.features["#idx"]
            if not return_node_idxs:
                del ns.features["#idx"]
            if return_features:
                for f, arr in feats.items():
                    ns.features[f] = arr[off : off + len(idx)]
            off += len(idx)


def create_sampler(
    graph: in_memory_graph_lib.InMemoryGraph,
    plan: Union[config_lib.SimpleSamplingConfig, config_lib.SamplingPlan],
    schema: schema_lib.GraphSchema,
    *,
    batch_size: Optional[int] = None,
    return_features: bool = True,
    return_node_idxs: bool = False,
    debug_sampling: bool = False,
    num_threads: Optional[int] = None,
    seed: Optional[int] = None,
    edgeset_to_mask: Optional[str] = None,
    slice_timeseries_by_seed: Optional[bool] = None,
    max_timeseries_len: Optional[int] = None,
    sampling_mode: Optional[int] = None,
) -> Sampler:
    """Creates a sampler (same arguments as the reference's create_sampler,
    in_memory_sampler.py:349-445, plus the ``sampling_mode`` extension)."""
    if isinstance(plan, config_lib.SimpleSamplingConfig):
        plan = config_lib.simple_sampling_config_to_sampling_plan(plan, schema)
    if slice_timeseries_by_seed is None:
        slice_timeseries_by_seed = plan.temporal_sampling
    edgeset_timestamp_features = plan.edgeset_timestamp_features
    if edgeset_timestamp_features and edgeset_to_mask is not None:
        raise ValueError("Temporal filtering and edge masking cannot be used at the same time (yet).")
    if seed is None:
        seed = -1
    if batch_size is None and num_threads is None:
        raise ValueError("At least one of 'batch_size' or 'num_threads' must be specified.")
    if num_threads is None:
        num_threads = min(batch_size, os.cpu_count() or 1)
    cc = _in_memory_sampler_ext.CreateSampler(
        graph,
        plan,
        debug_sampling,
        num_threads,
        seed,
        schema,
        edgeset_to_mask,
        edgeset_timestamp_features,
        sampling_mode=sampling_mode,
    )
    return Sampler(
        cc,
        full_graph=graph,
        return_features=return_features,
        return_node_idxs=return_node_idxs,
        schema=schema,
        slice_timeseries_by_seed=slice_timeseries_by_seed,
        max_timeseries_len=max_timeseries_len,
        has_temporal_edgesets=bool(edgeset_timestamp_features),
    )
