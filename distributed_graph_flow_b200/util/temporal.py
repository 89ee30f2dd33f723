"""Creation-time timestamp inference from the schema.

Follows dgf/src/util/temporal.py:48-206: a feature with is_creation_time
(not a timeseries, no group) is the entity's timestamp and must be
INTEGER_64; an edge set uses its own creation-time feature, else a source or
target node set's creation-time feature name if the edge set also carries a
feature of that name. Timeseries features (is_timeseries) are grouped by
their ``group`` (a creation-time series without a group forms its own group);
a group's timestamp series is its is_creation_time timeseries member.
"""

from __future__ import annotations

import collections
import dataclasses
from typing import Dict, List, Optional

from distributed_graph_flow_b200.data import schema as schema_lib


def creation_time_feature_name(schemas: schema_lib.FeatureSetSchema) -> Optional[str]:
    found = []
    for name, feat in schemas.items():
        if feat.is_creation_time and not feat.is_timeseries and feat.group is None:
            if feat.format != schema_lib.FeatureFormat.INTEGER_64:
                raise ValueError(
                    f"Creation time feature '{name}' must have format INTEGER_64. Got {feat.format}."
                )
            found.append(name)
    if len(found) > 1:
        raise ValueError(f"Multiple creation time features found: {found}. Please only provide one.")
    return found[0] if found else None


def edgeset_creation_time_feature_name(
    es_schema: schema_lib.EdgeSchema, schema: schema_lib.GraphSchema
) -> Optional[str]:
    name = creation_time_feature_name(es_schema.features)
    if name is not None:
        return name
    for end in (es_schema.source, es_schema.target):
        if end in schema.node_sets:
            ts = creation_time_feature_name(schema.node_sets[end].features)
            if ts in es_schema.features:
                return ts
    return None


def nodeset_timestamp_features(schema: schema_lib.GraphSchema) -> Dict[str, str]:
    out = {}
    for name, ns in schema.node_sets.items():
        ts = creation_time_feature_name(ns.features)
        if ts is not None:
            out[name] = ts
    return out


def edgeset_timestamp_features(schema: schema_lib.GraphSchema) -> Dict[str, str]:
    out = {}
    for name, es in schema.edge_sets.items():
        ts = edgeset_creation_time_feature_name(es, schema)
        if ts is not None:
            out[name] = ts
    return out


@dataclasses.dataclass(frozen=True)
class TimeseriesGroupSpec:
    """Features sharing one timestamp series (None: the series has none)."""

    timestamp_feature_name: Optional[str]
    feature_names: List[str]


@dataclasses.dataclass(frozen=True)
class TimeseriesSchemaCache:
    """Timeseries groups per node set and edge set."""

    node_sets: Dict[str, List[TimeseriesGroupSpec]]
    edge_sets: Dict[str, List[TimeseriesGroupSpec]]
    has_timeseries: bool


def group_creation_time_feature_name(group_name: str, schemas: schema_lib.FeatureSetSchema) -> Optional[str]:
    for name, sch in schemas.items():
        if sch.is_creation_time and sch.is_timeseries and (sch.group or name) == group_name:
            return name
    return None


def _timeseries_specs(features: schema_lib.FeatureSetSchema) -> List[TimeseriesGroupSpec]:
    groups: Dict[Optional[str], List[str]] = collections.defaultdict(list)
    for fname, fs in features.items():
        if not fs.is_timeseries:
            continue
        groups[fs.group or (fname if fs.is_creation_time else None)].append(fname)
    return [TimeseriesGroupSpec(None if g is None else group_creation_time_feature_name(g, features), names)
            for g, names in groups.items()]


def extract_timeseries_schema_cache(schema: schema_lib.GraphSchema) -> TimeseriesSchemaCache:
    nodes = {n: _timeseries_specs(ns.features) for n, ns in schema.node_sets.items()}
    edges = {n: _timeseries_specs(es.features) for n, es in schema.edge_sets.items()}
    return TimeseriesSchemaCache(nodes, edges, any(nodes.values()) or any(edges.values()))
