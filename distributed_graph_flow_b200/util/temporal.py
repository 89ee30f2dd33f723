"""Creation-time timestamp inference from the schema.

Follows dgf/src/util/temporal.py:48-128: a feature with is_creation_time
(not a timeseries, no group) is the entity's timestamp and must be
INTEGER_64; an edge set uses its own creation-time feature, else a source or
target node set's creation-time feature name if the edge set also carries a
feature of that name.
"""

from __future__ import annotations

from typing import Dict, Optional

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
