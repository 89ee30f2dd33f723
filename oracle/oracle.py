"""ORACLE — test infrastructure only.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
import this module, and only as the checker or as the timed CPU baseline.
The product (distributed_graph_flow_b200/) never imports it.

Two CPU implementations of DGF's sampling path behind one wrapper:
  * ``liboracle.so`` — the C++ restatement (grow.h + dgf_oracle.cc), which
    follows dgf/src/sampling/in_memory_sampler.{h,cc} and
    in_memory_sampler_ext.cc:231-533, 1020-1246;
  * ``_ref/libdgf_ref.so`` — the same driver over the reference's own
    AdjacencyIndex, compiled from its unmodified in_memory_sampler.cc.
And a float64 numpy restatement of the aggregation math:
  * segment_sum / mean pooling, dgf/src/learning/jax/layers/hetero_gnn.py:
    283-295 (jax.ops.segment_sum(data, ids, n) / max(count, 1));
  * CSR SpMM (sparse_deferred SparseMatrix @ dense,
    homo_gnn_sparse_deferred.py:138-161) as the same segment sum with
    row = target, col = source.
And a numpy restatement of the edge-time propagation,
dgf/src/transform/temporal.py:95-103, and a pure-Python restatement of
SubGraphExtractor (in_memory_sampler_ext.cc:600-772) for small graphs in the
deterministic modes; the C++ libraries also restate the random-walk negative
sampler (in_memory_sampler_ext.cc:774-948) and the raw-id mapping of GF
graph loading (dgf/src/io/io_ext.cc:26-170), and a numpy restatement of the
causal timeseries slicing (dgf/src/sampling/temporal.py:24-63).
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path
from typing import Dict, List, Optional

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_ORACLE = HERE / "liboracle.so"
LIB_REF = HERE / "_ref" / "libdgf_ref.so"

MODE_RANDOM, MODE_FIRST, MODE_MOST_RECENT = 0, 1, 2

_libs: Dict[str, ctypes.CDLL] = {}

_p64 = ctypes.POINTER(ctypes.c_int64)
_pi = ctypes.POINTER(ctypes.c_int)


def build(ref: bool = True) -> None:
    """Builds liboracle.so (and _ref/ when the reference sources exist)."""
    import subprocess

    target = "ref" if ref else "all"
    subprocess.run(["make", "-s", "-C", str(HERE), target], check=True)


def available(ref: bool = False) -> bool:
    return (LIB_REF if ref else LIB_ORACLE).exists()


def _lib(ref: bool) -> ctypes.CDLL:
    key = "ref" if ref else "oracle"
    if key not in _libs:
        path = LIB_REF if ref else LIB_ORACLE
        if not path.exists():
            raise RuntimeError(f"{path} not built (make -C oracle{' ref' if ref else ''})")
        lib = ctypes.CDLL(str(path), mode=os.RTLD_NOW | os.RTLD_LOCAL)
        lib.oracle_last_error.restype = ctypes.c_char_p
        lib.oracle_sampler_create.restype = ctypes.c_void_p
        lib.oracle_sampler_create.argtypes = [
            ctypes.c_int, _p64, ctypes.c_int, ctypes.POINTER(_p64), ctypes.POINTER(_p64), ctypes.POINTER(_p64), _p64,
            ctypes.c_int, _pi, _pi, _pi, ctypes.c_int, _pi, _pi, _pi, _pi, ctypes.c_int, ctypes.c_int, ctypes.c_int,
            ctypes.c_int64, ctypes.c_int, ctypes.c_int,
        ]
        lib.oracle_sampler_free.argtypes = [ctypes.c_void_p]
        _p32 = ctypes.POINTER(ctypes.c_int32)
        lib.oracle_sampler_create_csr.restype = ctypes.c_void_p
        lib.oracle_sampler_create_csr.argtypes = [
            ctypes.c_int, _p64, ctypes.c_int, ctypes.POINTER(_p64), ctypes.POINTER(_p32), ctypes.POINTER(_p64),
            ctypes.POINTER(_p64), ctypes.POINTER(_p32), ctypes.POINTER(_p64), _p64, ctypes.c_int, _pi, _pi, _pi,
            ctypes.c_int, _pi, _pi, _pi, _pi, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int64, ctypes.c_int,
            ctypes.c_int,
        ]
        lib.oracle_sample.restype = ctypes.c_int
        lib.oracle_sample.argtypes = [ctypes.c_void_p, _p64, _p64, _p64, ctypes.c_int64, ctypes.c_int]
        lib.oracle_random_walk_negatives.restype = ctypes.c_int
        lib.oracle_random_walk_negatives.argtypes = [ctypes.c_void_p, _p64, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                                     ctypes.c_int, ctypes.c_int, ctypes.c_uint64, ctypes.c_uint64,
                                                     ctypes.c_int, _p64]
        lib.oracle_bytes_map.argtypes = [ctypes.c_char_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_char_p,
                                          ctypes.c_int64, ctypes.c_int64, ctypes.c_int, _p64, _p64]
        lib.oracle_result_counts.argtypes = [ctypes.c_void_p, _p64, _p64]
        lib.oracle_result_copy.argtypes = [ctypes.c_void_p, _p64, _p64, _p64]
        lib.oracle_index_build.restype = ctypes.c_void_p
        lib.oracle_index_build.argtypes = [_p64, _p64, _p64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                           ctypes.c_int, ctypes.c_int]
        lib.oracle_index_free.argtypes = [ctypes.c_void_p]
        lib.oracle_index_sizes.argtypes = [ctypes.c_void_p, _p64]
        lib.oracle_index_copy.argtypes = [ctypes.c_void_p, _p64, _p64, _p64, _p64]
        lib.oracle_index_string.restype = ctypes.c_int64
        lib.oracle_index_string.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int64]
        lib.oracle_index_sample.restype = ctypes.c_int64
        lib.oracle_index_sample.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_int64,
                                            ctypes.c_int64, ctypes.c_int64, ctypes.c_uint64, _p64, ctypes.c_int64]
        _i64, _u64, _u32, _dbl = ctypes.c_int64, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_double
        lib.oracle_synth_rowptr.argtypes = [_i64, _i64, _dbl, _i64, _u64, _p64, ctypes.c_int]
        lib.oracle_synth_edges.argtypes = [_p64, _i64, _i64, _u64, _p64, _p64, ctypes.c_int]
        lib.oracle_synth_uniform_int.argtypes = [_i64, _i64, _i64, _u64, _u32, _p64, ctypes.c_int]
        lib.oracle_synth_normal_features.argtypes = [_i64, _i64, _i64, _u64, ctypes.c_int, ctypes.c_void_p,
                                                     ctypes.c_int]
        lib.oracle_sampler_create_synth.restype = ctypes.c_void_p
        lib.oracle_sampler_create_synth.argtypes = [
            _i64, _i64, _dbl, _i64, _u64, ctypes.c_int, _i64, _i64, _u64, _u32, ctypes.c_int, _pi, _pi, ctypes.c_int,
            _pi, _pi, ctypes.c_int, ctypes.c_int, ctypes.c_int, _i64, ctypes.c_int]
        lib.oracle_sampler_set_mode.argtypes = [ctypes.c_void_p, ctypes.c_int]
        lib.oracle_sampler_fwd_csr.restype = ctypes.c_int
        lib.oracle_sampler_fwd_csr.argtypes = [ctypes.c_void_p, ctypes.c_int, _p64, _p64, _p64]
        _libs[key] = lib
    return _libs[key]


def _p(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data_as(_p64)


def _err(lib) -> str:
    m = lib.oracle_last_error()
    return m.decode() if m else ""


class OracleError(ValueError):
    pass


class Index:
    """One adjacency index built by the oracle (or by the reference code)."""

    def __init__(self, adjacency, timestamps=None, reversed=False, num_source_nodes=0, num_target_nodes=0,
                 populate_edge_idxs=False, ref=False):
        self.lib = _lib(ref)
        adj = np.ascontiguousarray(np.asarray(adjacency).astype(np.int64))
        self._src = np.ascontiguousarray(adj[0])
        self._dst = np.ascontiguousarray(adj[1])
        self._ts = None if timestamps is None else np.ascontiguousarray(np.asarray(timestamps, dtype=np.int64))
        self.h = self.lib.oracle_index_build(_p(self._src), _p(self._dst), _p(self._ts), len(self._src),
                                             int(num_source_nodes), int(num_target_nodes), int(reversed),
                                             int(populate_edge_idxs))
        if not self.h:
            raise OracleError(_err(self.lib))

    def __del__(self):
        if getattr(self, "h", None):
            self.lib.oracle_index_free(self.h)

    def arrays(self):
        sizes = np.zeros(4, np.int64)
        self.lib.oracle_index_sizes(self.h, _p(sizes))
        out = [np.zeros(int(n), np.int64) for n in sizes]
        self.lib.oracle_index_copy(self.h, *[_p(a) for a in out])
        return {"source_blocks": out[0], "target_node_idxs": out[1], "timestamps": out[2], "edge_idxs": out[3]}

    def __str__(self):
        n = self.lib.oracle_index_string(self.h, None, 0)
        buf = ctypes.create_string_buffer(int(n) + 1)
        self.lib.oracle_index_string(self.h, buf, n + 1)
        return buf.value.decode()

    def sample(self, kind: int, source: int, k: int, seed_ts: int = 0, masked: int = -1, rng_seed: int = 42):
        cap = 1 << 16
        out = np.zeros(cap, np.int64)
        n = self.lib.oracle_index_sample(self.h, kind, source, k, seed_ts, masked, rng_seed, _p(out), cap)
        if n < 0:
            raise OracleError(_err(self.lib))
        return out[: min(n, cap)]


def _flatten_plan(plan, nodeset_index, edgeset_index):
    nodes = [plan.root]
    node_ns, first, num, e_es, e_rev, e_hw, e_child = [], [], [], [], [], [], []
    head = 0
    node_ns.append(nodeset_index[plan.root.nodeset])
    first.append(0)
    num.append(0)
    while head < len(nodes):
        pn = nodes[head]
        i = head
        head += 1
        first[i] = len(e_es)
        num[i] = len(pn.children)
        for c in pn.children:
            e_es.append(edgeset_index[c.edgeset])
            e_rev.append(int(bool(c.reversed)))
            e_hw.append(int(c.hop_width))
            e_child.append(len(nodes))
            nodes.append(c.node)
            node_ns.append(nodeset_index[c.node.nodeset])
            first.append(0)
            num.append(0)
    return node_ns, first, num, e_es, e_rev, e_hw, e_child


def _ints(v):
    return (ctypes.c_int * max(1, len(v)))(*v)


class OracleSampler:
    """CPU sampler with the reference's semantics (see module docstring).

    ``graph`` is any object with ``node_sets[name].num_nodes`` and
    ``edge_sets[name].adjacency`` / ``.features``; ``plan`` any object with
    the SamplingPlan fields. Node/edge sets are indexed in sorted-name order.
    """

    def __init__(self, graph, plan, schema, debug_sampling=False, num_threads=0, seed=0, edgeset_to_mask=None,
                 edgeset_timestamp_features=None, mode=None, ref=False):
        self.lib = _lib(ref)
        ets = dict(edgeset_timestamp_features or {})
        self.nodesets = sorted(schema.node_sets)
        self.edgesets = sorted(schema.edge_sets)
        ns_idx = {n: i for i, n in enumerate(self.nodesets)}
        es_idx = {n: i for i, n in enumerate(self.edgesets)}
        node_ns, first, num, e_es, e_rev, e_hw, e_child = _flatten_plan(plan, ns_idx, es_idx)
        num_nodes = np.array([int(graph.node_sets[n].num_nodes) for n in self.nodesets], np.int64)
        self._keep = []
        srcs, dsts, tss, counts = [], [], [], []
        for name in self.edgesets:
            adj = np.ascontiguousarray(np.asarray(graph.edge_sets[name].adjacency).astype(np.int64))
            s, d = np.ascontiguousarray(adj[0]), np.ascontiguousarray(adj[1])
            t = None
            if name in ets:
                t = np.ascontiguousarray(np.asarray(graph.edge_sets[name].features[ets[name]], np.int64))
            self._keep += [s, d, t]
            srcs.append(_p(s))
            dsts.append(_p(d))
            tss.append(_p(t) if t is not None else None)
            counts.append(len(s))
        n_es = len(self.edgesets)
        src_arr = (_p64 * max(1, n_es))(*srcs)
        dst_arr = (_p64 * max(1, n_es))(*dsts)
        ts_arr = (_p64 * max(1, n_es))(*tss)
        cnt = np.array(counts + [0], np.int64)
        if mode is None:
            mode = MODE_FIRST if debug_sampling else MODE_RANDOM
        mask_idx = es_idx[edgeset_to_mask] if edgeset_to_mask is not None else -1
        self.h = self.lib.oracle_sampler_create(
            len(self.nodesets), _p(num_nodes), n_es, src_arr, dst_arr, ts_arr, _p(cnt), len(node_ns), _ints(node_ns),
            _ints(first), _ints(num), len(e_es), _ints(e_es), _ints(e_rev), _ints(e_hw), _ints(e_child),
            int(bool(plan.with_replacement)), int(mode), int(num_threads), int(seed), mask_idx, int(bool(ets)),
        )
        if not self.h:
            raise OracleError(_err(self.lib))

    @classmethod
    def from_synth(cls, num_nodes, num_edges, alpha, max_degree, graph_seed, plan, ts_range=None, ts_seed=0,
                   ts_stream=11, mode=MODE_RANDOM, num_threads=0, seed=0, ref=False, build_threads=8):
        """Sampler over the library's synthetic power-law graph (one node set,
        one edge set, optional uniform integer edge times drawn from stream
        `ts_stream` of `ts_seed`), generated on the host by the generator's
        restatement and indexed by CreateFromEdgeList (the reference's own
        with ref=True) in source ranges on build_threads threads."""
        self = cls.__new__(cls)
        self.lib = _lib(ref)
        self.nodesets = [plan.root.nodeset]
        self.edgesets = [plan.root.children[0].edgeset]
        node_ns, first, num, e_es, e_rev, e_hw, e_child = _flatten_plan(plan, {self.nodesets[0]: 0},
                                                                        {self.edgesets[0]: 0})
        if any(e_rev) or any(e != 0 for e in e_es):
            raise OracleError("from_synth: plans over one forward edge set only")
        lo, hi = ts_range if ts_range is not None else (0, 1)
        self._keep = []
        self.h = self.lib.oracle_sampler_create_synth(
            int(num_nodes), int(num_edges), float(alpha), int(max_degree), int(graph_seed), int(ts_range is not None),
            int(lo), int(hi), int(ts_seed), int(ts_stream), len(node_ns), _ints(first), _ints(num), len(e_es),
            _ints(e_hw), _ints(e_child), int(bool(plan.with_replacement)), int(mode), int(num_threads), int(seed),
            int(build_threads))
        if not self.h:
            raise OracleError(_err(self.lib))
        self._synth = (int(num_nodes), int(num_edges), ts_range is not None)
        return self

    def set_mode(self, mode: int) -> None:
        self.lib.oracle_sampler_set_mode(self.h, int(mode))

    def forward_csr(self):
        """(rowptr, col, ts or None) of the forward index of a from_synth
        sampler, as int64 arrays."""
        n, e, has_ts = self._synth
        rp = np.empty(n + 1, np.int64)
        col = np.empty(e, np.int64)
        ts = np.empty(e, np.int64) if has_ts else None
        if self.lib.oracle_sampler_fwd_csr(self.h, 0, _p(rp), _p(col), _p(ts)) != 0:
            raise OracleError("no forward index")
        return rp, col, ts

    @classmethod
    def from_csr(cls, num_nodes, nodesets, edgesets, csr_fwd, plan, mode=MODE_RANDOM, num_threads=0, seed=0,
                 temporal=False, ref=False, fill_threads=8, csr_bwd=None):
        """Sampler over prebuilt CSR arrays {edgeset: (rowptr int64, col
        int32, ts int64 | None)} already in CreateFromEdgeList order: forward
        indices in csr_fwd, backward (reversed) ones in csr_bwd, each only for
        the edge sets the plan walks in that direction."""
        self = cls.__new__(cls)
        self.lib = _lib(ref)
        self.nodesets = list(nodesets)
        self.edgesets = list(edgesets)
        ns_idx = {n: i for i, n in enumerate(self.nodesets)}
        es_idx = {n: i for i, n in enumerate(self.edgesets)}
        node_ns, first, num, e_es, e_rev, e_hw, e_child = _flatten_plan(plan, ns_idx, es_idx)
        nn = np.asarray(num_nodes, np.int64)
        self._keep = []
        _p32 = ctypes.POINTER(ctypes.c_int32)
        csr_bwd = csr_bwd or {}

        def arrays(table):
            rps, cols, tss, counts = [], [], [], []
            for name in self.edgesets:
                if name not in table:
                    rps.append(None)
                    cols.append(None)
                    tss.append(None)
                    counts.append(None)
                    continue
                rp, col, ts = table[name]
                rp = np.ascontiguousarray(rp, np.int64)
                col = np.ascontiguousarray(col, np.int32)
                ts = None if ts is None else np.ascontiguousarray(ts, np.int64)
                self._keep += [rp, col, ts]
                rps.append(rp.ctypes.data_as(_p64))
                cols.append(col.ctypes.data_as(_p32))
                tss.append(None if ts is None else ts.ctypes.data_as(_p64))
                counts.append(len(col))
            return rps, cols, tss, counts

        f_rp, f_col, f_ts, f_cnt = arrays(csr_fwd)
        b_rp, b_col, b_ts, b_cnt = arrays(csr_bwd)
        n_es = len(self.edgesets)
        counts = [f if f is not None else (b if b is not None else 0) for f, b in zip(f_cnt, b_cnt)]
        cnt = np.array(counts + [0], np.int64)
        self.h = self.lib.oracle_sampler_create_csr(
            len(self.nodesets), _p(nn), n_es, (_p64 * n_es)(*f_rp), (_p32 * n_es)(*f_col), (_p64 * n_es)(*f_ts),
            (_p64 * n_es)(*b_rp), (_p32 * n_es)(*b_col), (_p64 * n_es)(*b_ts), _p(cnt), len(node_ns), _ints(node_ns),
            _ints(first), _ints(num), len(e_es), _ints(e_es),
            _ints(e_rev), _ints(e_hw), _ints(e_child), int(bool(plan.with_replacement)), int(mode), int(num_threads),
            int(seed), int(bool(temporal)), int(fill_threads),
        )
        if not self.h:
            raise OracleError(_err(self.lib))
        return self

    def __del__(self):
        if getattr(self, "h", None):
            self.lib.oracle_sampler_free(self.h)

    def sample_raw(self, seeds, seed_ts=None, masks=None, threads: int = 1):
        """Samples and returns the merged (sample-major) flat arrays:
        (node_counts[B, NS], edge_counts[B, ES], nodes, esrc, edst)."""
        seeds = np.ascontiguousarray(np.asarray(seeds, np.int64))
        ts = None if seed_ts is None else np.ascontiguousarray(np.asarray(seed_ts, np.int64))
        mk = None if masks is None else np.ascontiguousarray(np.asarray(masks, np.int64))
        st = self.lib.oracle_sample(self.h, _p(seeds), _p(ts), _p(mk), len(seeds), int(threads))
        if st != 0:
            raise OracleError(_err(self.lib))
        B = len(seeds)
        nc = np.zeros((B, len(self.nodesets)), np.int64)
        ec = np.zeros((B, len(self.edgesets)), np.int64)
        self.lib.oracle_result_counts(self.h, _p(nc), _p(ec))
        nodes = np.zeros(int(nc.sum()), np.int64)
        esrc = np.zeros(int(ec.sum()), np.int64)
        edst = np.zeros(int(ec.sum()), np.int64)
        self.lib.oracle_result_copy(self.h, _p(nodes), _p(esrc), _p(edst))
        return nc, ec, nodes, esrc, edst

    def sample_merged(self, seeds, seed_ts=None, masks=None, threads: int = 1):
        """The batch in the device's merged layout: (node_ids, node_offsets,
        edges [2, E] of local ids, edge_offsets), node-set major then sample,
        offsets with a trailing total."""
        return merged_layout(*self.sample_raw(seeds, seed_ts, masks, threads))

    def sample(self, seeds, seed_ts=None, masks=None, threads: int = 1):
        """Per seed: ({nodeset: ids}, {edgeset: [2, E] adjacency})."""
        nc, ec, nodes, esrc, edst = self.sample_raw(seeds, seed_ts, masks, threads)
        out = []
        a = b = 0
        for i in range(nc.shape[0]):
            ns = {}
            for s, name in enumerate(self.nodesets):
                ns[name] = nodes[a : a + nc[i, s]]
                a += nc[i, s]
            es = {}
            for e, name in enumerate(self.edgesets):
                es[name] = np.stack([esrc[b : b + ec[i, e]], edst[b : b + ec[i, e]]])
                b += ec[i, e]
            out.append((ns, es))
        return out


    def random_walk_negatives(self, seeds, target_edgeset: int, num_walks: int, k: int, kind: int = 0,
                              sampler_seed: int = 0, call_index: int = 0, threads: int = 1) -> np.ndarray:
        """RandomWalkNegativeSampling (in_memory_sampler_ext.cc:774-948) as
        int64 [len(seeds), k]. kind 0 draws from the reference's generator
        (this sampler's std::mt19937_64, one per seed); kind 1 replays the
        device's Philox stream for (sampler_seed, call_index)."""
        seeds = np.ascontiguousarray(np.asarray(seeds, np.int64).reshape(-1))
        out = np.zeros((len(seeds), max(int(k), 0)), np.int64)
        st = self.lib.oracle_random_walk_negatives(self.h, _p(seeds), len(seeds), int(target_edgeset), int(num_walks),
                                                   int(k), int(kind), int(sampler_seed) & ((1 << 64) - 1),
                                                   int(call_index) & ((1 << 64) - 1), int(threads), _p(out))
        if st != 0:
            raise OracleError(_err(self.lib))
        return out


# ---------------------------------------------------------------------------
# Raw id -> index (dgf/src/io/io_ext.cc:26-170; integer ids:
# dgf/src/io/graph_in_memory.py:111-125).
# ---------------------------------------------------------------------------
def merged_layout(nc, ec, nodes, esrc, edst):
    """sample_raw's output (sample-major; node sets / edge sets in order
    within a sample) rearranged node-set (edge-set) major, then by sample."""
    B, NS = nc.shape
    ES = ec.shape[1]
    n_start = np.concatenate([[0], np.cumsum(nc.sum(1))])
    e_start = np.concatenate([[0], np.cumsum(ec.sum(1))])
    n_in = np.concatenate([np.zeros((B, 1), np.int64), np.cumsum(nc, 1)], 1)
    e_in = np.concatenate([np.zeros((B, 1), np.int64), np.cumsum(ec, 1)], 1)
    node_off = np.concatenate([[0], np.cumsum(nc.T.ravel())]).astype(np.int64)
    edge_off = np.concatenate([[0], np.cumsum(ec.T.ravel())]).astype(np.int64)
    if NS == 1 and ES <= 1:
        return nodes, node_off, np.stack([esrc, edst]), edge_off
    node_parts, src_parts, dst_parts = [], [], []
    for s in range(NS):
        for i in range(B):
            a = n_start[i] + n_in[i, s]
            node_parts.append(nodes[a:a + nc[i, s]])
    for e in range(ES):
        for i in range(B):
            a = e_start[i] + e_in[i, e]
            src_parts.append(esrc[a:a + ec[i, e]])
            dst_parts.append(edst[a:a + ec[i, e]])

    def cat(parts):
        return np.concatenate(parts) if parts else np.zeros(0, np.int64)

    return cat(node_parts), node_off, np.stack([cat(src_parts), cat(dst_parts)]), edge_off


def _id_key(v):
    if isinstance(v, (bytes, np.bytes_)):
        return bytes(v).rstrip(b"\0")
    return int(v)


def id_map(index_ids, query_ids):
    """(int64 indices, -1 for unknown ids; last unknown position or -1): a
    dict from id to its last position, byte ids without trailing zeros."""
    table = {}
    for i, v in enumerate(np.asarray(index_ids).tolist()):
        table[_id_key(v)] = i
    q = np.asarray(query_ids).tolist()
    out = np.empty(len(q), np.int64)
    mismatch = -1
    for i, v in enumerate(q):
        r = table.get(_id_key(v))
        if r is None:
            out[i] = -1
            mismatch = i
        else:
            out[i] = r
    return out, mismatch


def synth_graph(num_src: int, num_dst: int, num_edges: int, alpha: float, max_degree: int, seed: int,
                with_edges: bool = True, threads: int = 8):
    """Host restatement of the library's power-law graph generator
    (synth_cpu.h): rowptr int64[num_src + 1] and the source-major edge list
    (src, dst) int64[num_edges] (None unless with_edges)."""
    lib = _lib(False)
    rp = np.empty(num_src + 1, np.int64)
    lib.oracle_synth_rowptr(num_src, num_edges, float(alpha), max_degree, seed, _p(rp), threads)
    if not with_edges:
        return rp, None, None
    src = np.empty(num_edges, np.int64)
    dst = np.empty(num_edges, np.int64)
    lib.oracle_synth_edges(_p(rp), num_src, num_dst, seed, _p(src), _p(dst), threads)
    return rp, src, dst


def synth_uniform_int(n: int, lo: int, hi: int, seed: int, stream_id: int, threads: int = 8) -> np.ndarray:
    out = np.empty(n, np.int64)
    _lib(False).oracle_synth_uniform_int(n, lo, hi, seed, stream_id, _p(out), threads)
    return out


def synth_normal_features(node_begin: int, count: int, dim: int, seed: int, bf16: bool, threads: int = 8,
                          out: Optional[np.ndarray] = None) -> np.ndarray:
    """N(0, 1) rows; bf16=True returns the bf16 bit patterns as uint16."""
    if out is None:
        out = np.empty((count, dim), np.uint16 if bf16 else np.float32)
    _lib(False).oracle_synth_normal_features(node_begin, count, dim, seed, int(bool(bf16)),
                                             out.ctypes.data_as(ctypes.c_void_p), threads)
    return out


def bytes_map(index_ids: np.ndarray, query_ids: np.ndarray, threads: int = 1):
    """id_map for numpy byte arrays in C++ (unordered_map over string views,
    the query loop split over `threads`, like PairMapping)."""
    lib = _lib(False)
    a = np.ascontiguousarray(index_ids)
    b = np.ascontiguousarray(query_ids)
    out = np.empty(len(b), np.int64)
    mm = np.full(1, -1, np.int64)
    lib.oracle_bytes_map(a.tobytes() if a.size else b"", len(a), max(1, a.dtype.itemsize),
                         b.tobytes() if b.size else b"", len(b), max(1, b.dtype.itemsize), int(threads), _p(out),
                         _p(mm))
    return out, int(mm[0])


# ---------------------------------------------------------------------------
# Causal timeseries slicing (dgf/src/sampling/temporal.py:24-63).
# ---------------------------------------------------------------------------
def timeseries_window(times, values, cutoff: int, max_len: Optional[int]):
    """One entity's window of one feature: entries with time <= cutoff
    (np.searchsorted side="right"), the last max_len of them."""
    end = int(np.searchsorted(np.asarray(times), cutoff, side="right"))
    start = max(0, end - max_len) if max_len is not None else 0
    return np.asarray(values)[slice(start, end)]


def filter_timeseries(features: dict, groups, cutoffs, max_len: Optional[int]) -> dict:
    """{feature: object array} for entities 0..n-1 with per-entity cutoffs;
    groups = [(timestamp feature or None, [feature names])]."""
    out = {}
    for ts_name, names in groups:
        if ts_name is None:
            continue
        times = features[ts_name]
        for f in names:
            col = np.empty(len(cutoffs), dtype=object)
            for i, c in enumerate(cutoffs):
                col[i] = timeseries_window(times[i], features[f][i], int(c), max_len)
            out[f] = col
    return out


# ---------------------------------------------------------------------------
# Aggregation (float64).
# ---------------------------------------------------------------------------
def segment_sum(data: np.ndarray, segment_ids: np.ndarray, num_segments: int, mean: bool = False) -> np.ndarray:
    """jax.ops.segment_sum semantics in float64 (out-of-range ids dropped);
    mean divides by max(count, 1) (hetero_gnn.py:288-295)."""
    data = np.asarray(data, np.float64)
    ids = np.asarray(segment_ids, np.int64)
    keep = (ids >= 0) & (ids < num_segments)
    out = np.zeros((num_segments,) + data.shape[1:], np.float64)
    np.add.at(out, ids[keep], data[keep])
    if mean:
        cnt = np.bincount(ids[keep], minlength=num_segments).astype(np.float64)
        out /= np.maximum(cnt, 1.0).reshape((-1,) + (1,) * (data.ndim - 1))
    return out


def csr_spmm(rowptr: np.ndarray, col: np.ndarray, x: np.ndarray, val: Optional[np.ndarray] = None,
             normalize: bool = False) -> np.ndarray:
    """Y[r] = scale_r * sum_j val_j * X[col_j] in float64 (scipy CSR)."""
    import scipy.sparse as sp

    rowptr = np.asarray(rowptr, np.int64)
    n_rows = len(rowptr) - 1
    v = np.ones(len(col), np.float64) if val is None else np.asarray(val, np.float64)
    a = sp.csr_matrix((v, np.asarray(col, np.int64), rowptr), shape=(n_rows, x.shape[0]))
    y = a @ np.asarray(x, np.float64)
    if normalize:
        deg = np.diff(rowptr).astype(np.float64)
        y /= np.maximum(deg, 1.0)[:, None]
    return y


def csr_spmm_grad_x(rowptr: np.ndarray, col: np.ndarray, dy: np.ndarray, num_x_rows: int,
                    val: Optional[np.ndarray] = None, normalize: bool = False) -> np.ndarray:
    """d loss / d X of Y = S A X for an upstream gradient dY: A^T S dY in
    float64 (S = diag(1 / max(deg, 1)) when normalize)."""
    import scipy.sparse as sp

    rowptr = np.asarray(rowptr, np.int64)
    n_rows = len(rowptr) - 1
    v = np.ones(len(col), np.float64) if val is None else np.asarray(val, np.float64)
    a = sp.csr_matrix((v, np.asarray(col, np.int64), rowptr), shape=(n_rows, num_x_rows))
    g = np.asarray(dy, np.float64)
    if normalize:
        g = g / np.maximum(np.diff(rowptr).astype(np.float64), 1.0)[:, None]
    return a.T @ g


def segment_sum_grad(dy: np.ndarray, segment_ids: np.ndarray, num_segments: int, mean: bool = False) -> np.ndarray:
    """d loss / d data of jax.ops.segment_sum(data, ids, n) [/ max(count, 1)]
    (hetero_gnn.py:283-295): each item gets its segment's upstream gradient
    (scaled by 1 / max(count, 1) for the mean), zero for ids out of range."""
    ids = np.asarray(segment_ids, np.int64)
    g = np.asarray(dy, np.float64)
    ok = (ids >= 0) & (ids < num_segments)
    out = np.zeros((len(ids),) + g.shape[1:], np.float64)
    out[ok] = g[ids[ok]]
    if mean:
        cnt = np.bincount(ids[ok], minlength=num_segments).astype(np.float64)
        out[ok] /= np.maximum(cnt[ids[ok]], 1.0).reshape((-1,) + (1,) * (g.ndim - 1))
    return out


def propagation_matrix(src: np.ndarray, dst: np.ndarray, num_nodes: int, diag: float,
                       normalize_symmetric: bool) -> np.ndarray:
    """Dense float64 (A + A^T + diag * I), optionally D^-1/2 (.) D^-1/2 with
    D the row sums, for an edge list on one node set: the propagation
    matrices of dgf/src/learning/jax/layers/homo_gnn_sparse_deferred.py:293
    (GCN: ``(adj + adj.transpose()).add_eye().normalize_symmetric()``) and
    :526 (GIN: ``(adj + adj.transpose()).add_eye(1 + epsilon)``). Their
    arithmetic is the third-party sparse-deferred package (requirements.txt:
    13, unpinned, not in the reference tree), restated from its published
    semantics: a SparseMatrix is a COO sum (duplicate entries add),
    transpose swaps the indices, add_eye(v) adds v on the diagonal, and
    normalize_symmetric divides entry (i, j) by sqrt(rowsum_i) *
    sqrt(colsum_j)."""
    m = np.zeros((num_nodes, num_nodes), np.float64)
    s = np.asarray(src, np.int64)
    d = np.asarray(dst, np.int64)
    np.add.at(m, (d, s), 1.0)
    np.add.at(m, (s, d), 1.0)
    m[np.arange(num_nodes), np.arange(num_nodes)] += diag
    if normalize_symmetric:
        r = np.sqrt(m.sum(1))
        c = np.sqrt(m.sum(0))
        m = m / r[:, None] / c[None, :]
    return m


def batch_mean_aggregate(node_offsets: np.ndarray, edge_offsets: np.ndarray, edges: np.ndarray,
                         features: np.ndarray) -> np.ndarray:
    """Mean aggregation over a merged sampled batch (one node set and edge
    set), float64: out[v] = mean of features[u] over the batch edges v -> u
    (jax.ops.segment_sum of the neighbours' features over the edge sources,
    divided by max(count, 1); hetero_gnn.py:282-294 with the edge direction
    reversed), zero for nodes without edges."""
    n = int(node_offsets[-1])
    B = len(node_offsets) - 1
    samp = np.repeat(np.arange(B), np.diff(edge_offsets))
    gsrc = node_offsets[:-1][samp] + edges[0]
    gdst = node_offsets[:-1][samp] + edges[1]
    out = np.zeros((n, features.shape[1]), np.float64)
    np.add.at(out, gsrc, np.asarray(features[gdst], np.float64))
    cnt = np.bincount(gsrc, minlength=n).astype(np.float64)
    return out / np.maximum(cnt, 1.0)[:, None]


# ---------------------------------------------------------------------------
# Edge creation times (dgf/src/transform/temporal.py:95-103).
# ---------------------------------------------------------------------------
def edge_timestamps(src_ts: Optional[np.ndarray], tgt_ts: Optional[np.ndarray], adjacency: np.ndarray) -> np.ndarray:
    """max(src_ts[src], tgt_ts[tgt]); the one side given when the other is
    None (temporal.py:95-103)."""
    src, tgt = adjacency
    if src_ts is not None and tgt_ts is not None:
        return np.maximum(src_ts[src], tgt_ts[tgt])
    if src_ts is not None:
        return src_ts[src]
    return tgt_ts[tgt]


# ---------------------------------------------------------------------------
# SubGraphExtractor (in_memory_sampler_ext.cc:600-772), deterministic modes:
# every plan edge takes the first min(hop_width, degree) neighbours in index
# order (SampleFirst, :250-279; with hop_width >= degree SampleRandomUniform
# returns the whole row in the same order, in_memory_sampler.cc:130-132).
# ---------------------------------------------------------------------------
def subgraph(graph, plan, seeds, nodeset_names: List[str], edgeset_names: List[str], schema) -> tuple:
    """Returns ({nodeset: node idxs}, {edgeset: [2, E] adjacency})."""
    adj = {}
    for name in edgeset_names:
        es = schema.edge_sets[name]
        a = np.asarray(graph.edge_sets[name].adjacency, dtype=np.int64).reshape(2, -1)
        for rev in (False, True):
            src, dst = (a[1], a[0]) if rev else (a[0], a[1])
            order = np.lexsort((dst, src))  # CreateFromEdgeList: sorted by (source, target)
            rows = {}
            for s_, d_ in zip(src[order].tolist(), dst[order].tolist()):
                rows.setdefault(s_, []).append(d_)
            adj[(name, rev)] = rows
    # Plan nodes numbered depth-first (the step index of a plan node).
    steps = {}

    def number(pn):
        steps[id(pn)] = len(steps)
        for c in pn.children:
            number(c.node)

    number(plan.root)
    node_idxs = {n: [] for n in nodeset_names}
    visited = {n: {} for n in nodeset_names}       # node -> sample idx
    visited_step = {n: set() for n in nodeset_names}
    edges = {e: set() for e in edgeset_names}

    def grow(pn, source, source_sampled):
        for pe in pn.children:
            targets = adj[(pe.edgeset, bool(pe.reversed))].get(source, [])[: pe.hop_width]
            tns = pe.node.nodeset
            step = steps[id(pe.node)]
            for t in targets:
                cont = True
                if t in visited[tns]:
                    eff = visited[tns][t]
                    if (t, step) in visited_step[tns]:
                        cont = False
                    else:
                        visited_step[tns].add((t, step))
                else:
                    eff = len(node_idxs[tns])
                    visited[tns][t] = eff
                    node_idxs[tns].append(t)
                    visited_step[tns].add((t, step))
                edges[pe.edgeset].add((eff, source_sampled) if pe.reversed else (source_sampled, eff))
                if cont:
                    grow(pe.node, t, eff)

    root = plan.root.nodeset
    for sd in seeds:
        visited[root][sd] = len(node_idxs[root])
        node_idxs[root].append(sd)
        visited_step[root].add((sd, steps[id(plan.root)]))
    for sd in seeds:
        grow(plan.root, sd, visited[root][sd])
    out_edges = {}
    for e in edgeset_names:
        pairs = sorted(edges[e])
        out_edges[e] = np.array([[p[0] for p in pairs], [p[1] for p in pairs]], dtype=np.int64).reshape(2, -1)
    return {n: np.array(v, dtype=np.int64) for n, v in node_idxs.items()}, out_edges
