"""Reads and writes graphs in the GF on-disk format, mapping ids on the GPU.

Same functions, arguments, results and error messages as
dgf/src/io/graph_in_memory.py:56-470: a GF graph is a directory with
``schema.json`` (the GraphSchema as JSON), ``metadata.json`` (format version
and optional timestamp), ``nodesets/<name>-*.parquet`` (node features,
including the primary-id column) and ``edgesets/<name>-*.parquet`` (``#source``
and ``#target`` raw ids plus edge features). Loading turns every edge's raw
endpoint ids into node indices; here that join runs on the GPU
(``io.ids.IdIndex``: one device hash index per node set, probed by all edge
endpoints), dangling-edge removal is a device compaction, and with
``device=...`` the adjacencies stay in HBM as int64 CUDA tensors that
``create_sampler`` indexes without a host round trip. Parquet decoding is
host IO (pyarrow).
"""

from __future__ import annotations

import ctypes
import json
import logging
import os
import time
from typing import Dict, Optional, Tuple

import numpy as np

from distributed_graph_flow_b200 import _native
from distributed_graph_flow_b200.data import in_memory_graph as in_memory_graph_lib
from distributed_graph_flow_b200.data import schema as schema_lib
from distributed_graph_flow_b200.io import ids as ids_lib
from distributed_graph_flow_b200.io import parquet as parquet_lib

FILENAME_SCHEMA = "schema.json"
FILENAME_METADATA = "metadata.json"
FILENAME_NODE_FEATURE = "nodesets"
FILENAME_EDGES_ADJACENCIES = "edgesets"
KEY_SOURCE = "#source"
KEY_TARGET = "#target"
MAX_SUPPORTED_GF_VERSION = 0
_PRIMARY_CANDIDATES = ["#id", "#ID", "id", "ID"]

log = logging.getLogger(__name__)


# ---------------------------------------------------------------------------
# Schema helpers (dgf/src/io/schema.py, dgf/src/analyse/schema.py:20-290,
# dgf/src/transform/schema.py:20-80).
# ---------------------------------------------------------------------------
def read_schema(path: str) -> schema_lib.GraphSchema:
    with open(path, "r") as f:
        return schema_lib.GraphSchema.from_json(f.read())


def write_schema(schema: schema_lib.GraphSchema, path: str) -> None:
    with open(path, "w") as f:
        f.write(schema.to_json(indent=2))


def primary_feature_or_none(name: str, schema) -> Optional[str]:
    found = [k for k, f in schema.features.items() if f.semantic == schema_lib.FeatureSemantic.PRIMARY_ID]
    if not found:
        return None
    if len(found) > 1:
        raise ValueError(f"Multiple primary features found in the schema of {name!r}: {found}. Currently, DGF does "
                         "not support multi-primary keys.")
    return found[0]


def primary_feature(name: str, schema) -> str:
    feature = primary_feature_or_none(name, schema)
    if feature is None:
        raise ValueError(f"No primary feature found in the schema of {name!r}. This operation requires for the schema "
                         "to define a primary key i.e. a feature with semantic=PRIMARY_ID. The available features "
                         f"are: {schema.features.keys()!r}.")
    return feature


def _infer_primary_key_or_none(name: str, schema) -> Optional[str]:
    matching = [c for c in _PRIMARY_CANDIDATES if c in schema.features]
    if len(matching) > 1:
        raise ValueError(f"No primary feature found in the schema of {name!r} (i.e. semantic=PRIMARY_ID), but "
                         f"multiple feature that look like primary key found ({matching!r}). The available features "
                         f"are: {schema.features.keys()!r}. Solution: Specify the primary key in the schema.")
    return matching[0] if matching else None


_TF_EXAMPLE_FORMATS = {schema_lib.FeatureFormat.INTEGER_32: schema_lib.FeatureFormat.INTEGER_64,
                       schema_lib.FeatureFormat.BOOL: schema_lib.FeatureFormat.INTEGER_64,
                       schema_lib.FeatureFormat.FLOAT_64: schema_lib.FeatureFormat.FLOAT_32}


def fix_schema(schema: schema_lib.GraphSchema, create_pound_id_as_fall_back: bool = False, fix_shape: bool = True,
               tf_example: bool = False) -> None:
    """Repairs a schema in place (dgf/src/analyse/schema.py:168-265).

    Sets missing primary keys (``#id``-like names) and drops the extra leading
    None of [None, k] shapes when every feature of a set has one. With
    ``create_pound_id_as_fall_back`` a node set with no key-like feature gets
    a BYTES feature ``#id`` as its key (whether the data holds it is not
    checked). With ``tf_example`` formats a TF Example cannot hold are
    widened or narrowed to the ones it can: int32 and bool to int64, float64
    to float32."""

    def suspicious(shape):
        return shape is not None and len(shape) == 2 and shape[0] is None and shape[1] is not None

    def fix_shapes(features):
        if fix_shape and all(suspicious(f.shape) for f in features.values()):
            for f in features.values():
                f.shape = tuple() if f.shape[1] == 1 else tuple(f.shape[1:])

    def fix_formats(features):
        if tf_example:
            for f in features.values():
                f.format = _TF_EXAMPLE_FORMATS.get(f.format, f.format)

    for name, ns in schema.node_sets.items():
        fix_formats(ns.features)
        fix_shapes(ns.features)
        if primary_feature_or_none(name, ns) is not None:
            continue
        pk = _infer_primary_key_or_none(name, ns)
        if pk is None and create_pound_id_as_fall_back:
            pk = "#id"
            ns.features[pk] = schema_lib.FeatureSchema(format=schema_lib.FeatureFormat.BYTES)
        if pk is None:
            raise ValueError(f"No primary feature found in the schema of {name!r} (i.e. semantic=PRIMARY_ID) and no "
                             f"feature look like a primary key ({_PRIMARY_CANDIDATES!r}). The available features are: "
                             f"{ns.features.keys()!r}. Solution: Specify the primary key in the schema.")
        ns.features[pk].semantic = schema_lib.FeatureSemantic.PRIMARY_ID
    for name, es in schema.edge_sets.items():
        fix_formats(es.features)
        fix_shapes(es.features)
        if primary_feature_or_none(name, es) is not None:
            continue
        pk = _infer_primary_key_or_none(name, es)
        if pk is not None:
            es.features[pk].semantic = schema_lib.FeatureSemantic.PRIMARY_ID


def filter_schema(schema: schema_lib.GraphSchema, flt: schema_lib.GraphSchemaFilter) -> schema_lib.GraphSchema:
    node_sets = {}
    for name, ns in schema.node_sets.items():
        if flt.nodeset_fn(name, ns):
            node_sets[name] = schema_lib.NodeSchema(features={
                k: f for k, f in ns.features.items() if flt.feature_fn(k, f) and flt.node_feature_fn(k, f)})
    edge_sets = {}
    for name, es in schema.edge_sets.items():
        if not flt.edgeset_fn(name, es):
            continue
        if es.source not in node_sets or es.target not in node_sets:
            continue  # an edge set whose endpoints were filtered out
        edge_sets[name] = schema_lib.EdgeSchema(source=es.source, target=es.target, features={
            k: f for k, f in es.features.items() if flt.feature_fn(k, f) and flt.edge_feature_fn(k, f)})
    return schema_lib.GraphSchema(node_sets=node_sets, edge_sets=edge_sets)


# ---------------------------------------------------------------------------
# Reading.
# ---------------------------------------------------------------------------
def _read_sharded(base_path: str, name: str, columns):
    paths = parquet_lib.list_shards(base_path)
    if not paths:
        raise ValueError(f"No files found matching pattern {base_path}-*{parquet_lib.PARQUET_EXTENSION} or "
                         f"{base_path}-*{parquet_lib.PARQUET_EXTENSION}")
    try:
        return parquet_lib.read_tables(paths, columns)
    except Exception as e:
        raise ValueError(f"Failed to read sharded Parquet file at {base_path} for '{name}'") from e


def _bad_id(ids: np.ndarray, pos: int):
    v = ids[pos]
    v = v.item() if hasattr(v, "item") else v
    return v.decode() if isinstance(v, bytes) else v


def read_graph(
    path: str,
    *,
    override_schema: Optional[schema_lib.GraphSchema] = None,
    verbose: bool = False,
    remove_dangling_edges: bool = False,
    schema_filter: Optional[schema_lib.GraphSchemaFilter] = None,
    device=None,
) -> Tuple[in_memory_graph_lib.InMemoryGraph, schema_lib.GraphSchema]:
    """Reads a GF graph directory into an InMemoryGraph (and its schema).

    With ``device`` (e.g. "cuda"), every edge set's adjacency is returned as
    an int64 CUDA tensor [2, E] instead of a numpy array (features stay
    numpy)."""
    torch = _native.require_cuda()
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    start = time.monotonic()
    schema = read_schema(os.path.join(path, FILENAME_SCHEMA)) if override_schema is None else override_schema
    if schema_filter:
        schema = filter_schema(schema, schema_filter)
    fix_schema(schema)
    with open(os.path.join(path, FILENAME_METADATA), "r") as f:
        metadata = json.loads(f.read())
    version = int(metadata.get("version", 0))
    if version > MAX_SUPPORTED_GF_VERSION:
        raise NotImplementedError(f"Unsupported metadata version: {version}. Only versions <= "
                                  f"{MAX_SUPPORTED_GF_VERSION} are supported.")

    node_sets, indexes = {}, {}
    with torch.cuda.device(dev):
        for name, ns in schema.node_sets.items():
            if verbose:
                log.info("Reading nodeset %s from %s", name, path)
            base = os.path.join(path, FILENAME_NODE_FEATURE, name)
            pk = primary_feature(name, ns)
            try:
                table = _read_sharded(base, name, list(ns.features.keys()))
            except ValueError as e:
                raise ValueError(f"Failed to read nodeset {name} from {base}") from e
            features, count = parquet_lib.table_to_numpy_dict(table)
            raw = features[pk]
            if raw.ndim != 1:
                raise ValueError(f"Expected node raw IDs for nodeset '{name}' to be a 1D array but got shape: "
                                 f"{raw.shape}")
            indexes[name] = ids_lib.IdIndex(raw, dev)
            node_sets[name] = in_memory_graph_lib.InMemoryNodeSet(features=features, num_nodes=count)

        edge_sets = {}
        for name, es in schema.edge_sets.items():
            if verbose:
                log.info("Reading edgeset %s from %s", name, path)
            base = os.path.join(path, FILENAME_EDGES_ADJACENCIES, name)
            columns = [KEY_SOURCE, KEY_TARGET, *[k for k in es.features if k not in (KEY_SOURCE, KEY_TARGET)]]
            try:
                table = _read_sharded(base, name, columns)
            except ValueError as e:
                raise ValueError(f"Failed to read edgeset {name} from {base}") from e
            features, count = parquet_lib.table_to_numpy_dict(table)
            src_ids, dst_ids = features[KEY_SOURCE], features[KEY_TARGET]
            adj = torch.empty((2, max(1, count)), dtype=torch.int64, device=dev)
            _, m_src = indexes[es.source].lookup(src_ids, out=adj[0, :count])
            _, m_dst = indexes[es.target].lookup(dst_ids, out=adj[1, :count])
            adj = adj[:, :count]
            if remove_dangling_edges:
                if m_src != -1 or m_dst != -1:
                    adj, kept = _drop_dangling(adj)
                    dropped = count - adj.shape[1]
                    if dropped > 0:
                        log.warning("Removed %d dangling edges in edgeset %r.", dropped, name)
                    keep = kept.cpu().numpy()
                    features = {k: v[keep] for k, v in features.items()}
            else:
                if m_src != -1:
                    raise ValueError(f"Node ID {_bad_id(src_ids, m_src)!r} not found in nodeset {es.source!r}.")
                if m_dst != -1:
                    raise ValueError(f"Node ID {_bad_id(dst_ids, m_dst)!r} not found in nodeset {es.target!r}.")
            if KEY_SOURCE not in es.features:
                features.pop(KEY_SOURCE, None)
            if KEY_TARGET not in es.features:
                features.pop(KEY_TARGET, None)
            adjacency = adj if device is not None else adj.cpu().numpy()
            edge_sets[name] = in_memory_graph_lib.InMemoryEdgeSet(adjacency=adjacency, features=features)
    log.info("Graph read in memory in %.3f s", time.monotonic() - start)
    graph = in_memory_graph_lib.InMemoryGraph(node_sets=node_sets, edge_sets=edge_sets,
                                              timestamp=metadata.get("timestamp"))
    return graph, schema


def _drop_dangling(adj):
    """Edges whose two endpoints are known, in order (dgfx_compact_pairs), and
    their positions."""
    torch = _native.require_cuda()
    n = int(adj.shape[1])
    dev = adj.device
    out = torch.empty((2, max(1, n)), dtype=torch.int64, device=dev)
    pos = torch.empty(max(1, n), dtype=torch.int64, device=dev)
    need = ctypes.c_size_t()
    _native.check(_native.lib().dgfx_compact_pairs_workspace_size(n, ctypes.byref(need)))
    ws = torch.empty(max(1, need.value), dtype=torch.uint8, device=dev)
    kept = ctypes.c_int64()
    src, dst = adj[0].contiguous(), adj[1].contiguous()
    _native.check(_native.lib().dgfx_compact_pairs(
        _native.ptr(src), _native.ptr(dst), n, _native.ptr(out[0]), _native.ptr(out[1]), _native.ptr(pos),
        ctypes.byref(kept), _native.ptr(ws), ws.numel(), _native.stream_handle()))
    k = kept.value
    return out[:, :k], pos[:k]


# ---------------------------------------------------------------------------
# Writing.
# ---------------------------------------------------------------------------
def write_graph(graph: in_memory_graph_lib.InMemoryGraph, schema: schema_lib.GraphSchema, path: str,
                verbose: bool = False, max_num_shards: Optional[int] = None, compression: str = "snappy") -> None:
    """Writes an InMemoryGraph and its schema as a GF graph directory (edge
    endpoints written as the nodes' raw primary ids)."""
    os.makedirs(path, exist_ok=True)
    write_schema(schema, os.path.join(path, FILENAME_SCHEMA))
    with open(os.path.join(path, FILENAME_METADATA), "w") as f:
        f.write(json.dumps({"version": MAX_SUPPORTED_GF_VERSION, "timestamp": graph.timestamp}, indent=2))
    node_dir = os.path.join(path, FILENAME_NODE_FEATURE)
    os.makedirs(node_dir, exist_ok=True)
    for name, ns_schema in schema.node_sets.items():
        ns = graph.node_sets[name]
        primary_feature(name, ns_schema)
        shards = parquet_lib.estimate_num_shards(int(ns.num_nodes))
        if max_num_shards is not None:
            shards = min(shards, max_num_shards)
        if ns.features is None:
            raise ValueError(f"Node set {name} has no features to write.")
        parquet_lib.write_numpy_dict(ns.features, name, node_dir, ns_schema.features, shards, compression)
    edge_dir = os.path.join(path, FILENAME_EDGES_ADJACENCIES)
    os.makedirs(edge_dir, exist_ok=True)
    for name, es_schema in schema.edge_sets.items():
        es = graph.edge_sets[name]
        src_pk = primary_feature(es_schema.source, schema.node_sets[es_schema.source])
        dst_pk = primary_feature(es_schema.target, schema.node_sets[es_schema.target])
        adjacency = es.adjacency
        if hasattr(adjacency, "cpu"):
            adjacency = adjacency.cpu().numpy()
        adjacency = np.asarray(adjacency)
        feats = dict(es.features) if es.features else {}
        feats[KEY_SOURCE] = graph.node_sets[es_schema.source].features[src_pk][adjacency[0]]
        feats[KEY_TARGET] = graph.node_sets[es_schema.target].features[dst_pk][adjacency[1]]
        fschema = dict(es_schema.features)
        fschema[KEY_SOURCE] = schema.node_sets[es_schema.source].features[src_pk]
        fschema[KEY_TARGET] = schema.node_sets[es_schema.target].features[dst_pk]
        shards = parquet_lib.estimate_num_shards(int(adjacency.shape[1]))
        if max_num_shards is not None:
            shards = min(shards, max_num_shards)
        parquet_lib.write_numpy_dict(feats, name, edge_dir, fschema, shards, compression)
