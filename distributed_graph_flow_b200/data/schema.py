"""Graph schema: the subset of DGF's schema the sampler reads.

Field names follow dgf/src/data/schema.py:25-160 (FeatureFormat,
FeatureSemantic, FeatureSchema, NodeSchema, EdgeSchema, GraphSchema) so that
schemas written for the reference load unchanged. The sampler uses the
node/edge set names (indexed in sorted-name order, like the reference's
native schema, dgf/src/data/schema_nb.cc:125-150), the edge set endpoints and
the creation-time flags of timestamp features.
"""

from __future__ import annotations

import dataclasses
import enum
import json
from typing import Callable, Dict, Optional, Tuple


class FeatureFormat(enum.Enum):
    """How a value is stored (dgf/src/data/schema.py:25-43)."""

    INTEGER_32 = "INTEGER_32"
    INTEGER_64 = "INTEGER_64"
    FLOAT_32 = "FLOAT_32"
    FLOAT_64 = "FLOAT_64"
    BYTES = "BYTES"
    BOOL = "BOOL"

    def is_integer(self) -> bool:
        return self in (FeatureFormat.INTEGER_32, FeatureFormat.INTEGER_64)

    def is_float(self) -> bool:
        return self in (FeatureFormat.FLOAT_32, FeatureFormat.FLOAT_64)

    def is_numerical(self) -> bool:
        return self.is_integer() or self.is_float()


class FeatureSemantic(enum.Enum):
    """How a value is interpreted (dgf/src/data/schema.py:46-74)."""

    UNKNOWN = "UNKNOWN"
    NUMERICAL = "NUMERICAL"
    CATEGORICAL = "CATEGORICAL"
    EMBEDDING = "EMBEDDING"
    TIMESTAMP = "TIMESTAMP"
    TIMEDELTA = "TIMEDELTA"
    TIMESERIES = "TIMESERIES"
    PRIMARY_ID = "PRIMARY_ID"
    MASK = "MASK"


Shape = Optional[Tuple[Optional[int], ...]]


@dataclasses.dataclass
class FeatureSchema:
    format: FeatureFormat
    semantic: FeatureSemantic = FeatureSemantic.UNKNOWN
    shape: Shape = None
    num_categorical_values: Optional[int] = None
    is_utf8_string: Optional[bool] = False
    is_timeseries: bool = False
    is_creation_time: bool = False
    group: Optional[str] = None


FeatureSetSchema = Dict[str, FeatureSchema]


@dataclasses.dataclass
class NodeSchema:
    features: FeatureSetSchema = dataclasses.field(default_factory=dict)


@dataclasses.dataclass
class EdgeSchema:
    source: str
    target: str
    features: FeatureSetSchema = dataclasses.field(default_factory=dict)


@dataclasses.dataclass
class GraphSchema:
    node_sets: Dict[str, NodeSchema]
    edge_sets: Dict[str, EdgeSchema]

    def nodeset_index(self) -> Dict[str, int]:
        """Name -> index in sorted-name order (the reference's numbering)."""
        return {n: i for i, n in enumerate(sorted(self.node_sets))}

    def edgeset_index(self) -> Dict[str, int]:
        return {n: i for i, n in enumerate(sorted(self.edge_sets))}

    # JSON in the layout the reference's dataclasses_json encoding gives
    # (field names as keys, enums by value, shapes as lists), the content of
    # a GF graph's schema.json.
    def to_dict(self) -> dict:
        def feats(fs):
            return {name: {"format": f.format.value, "semantic": f.semantic.value,
                           "shape": None if f.shape is None else list(f.shape),
                           "num_categorical_values": f.num_categorical_values, "is_utf8_string": f.is_utf8_string,
                           "is_timeseries": f.is_timeseries, "is_creation_time": f.is_creation_time,
                           "group": f.group} for name, f in fs.items()}

        return {"node_sets": {n: {"features": feats(ns.features)} for n, ns in self.node_sets.items()},
                "edge_sets": {n: {"source": es.source, "target": es.target, "features": feats(es.features)}
                              for n, es in self.edge_sets.items()}}

    def to_json(self, indent: Optional[int] = None) -> str:
        return json.dumps(self.to_dict(), indent=indent)

    @classmethod
    def from_dict(cls, d: dict) -> "GraphSchema":
        def feats(fs):
            out = {}
            for name, f in (fs or {}).items():
                shape = f.get("shape")
                out[name] = FeatureSchema(
                    format=FeatureFormat(f["format"]),
                    semantic=FeatureSemantic(f.get("semantic", "UNKNOWN")),
                    shape=None if shape is None else tuple(shape),
                    num_categorical_values=f.get("num_categorical_values"),
                    is_utf8_string=f.get("is_utf8_string", False),
                    is_timeseries=bool(f.get("is_timeseries", False)),
                    is_creation_time=bool(f.get("is_creation_time", False)),
                    group=f.get("group"))
            return out

        return cls(node_sets={n: NodeSchema(features=feats(v.get("features"))) for n, v in d["node_sets"].items()},
                   edge_sets={n: EdgeSchema(source=v["source"], target=v["target"], features=feats(v.get("features")))
                              for n, v in d["edge_sets"].items()})

    @classmethod
    def from_json(cls, text: str) -> "GraphSchema":
        return cls.from_dict(json.loads(text))


@dataclasses.dataclass
class GraphSchemaFilter:
    """Sub-selects node sets, edge sets and features
    (dgf/src/data/schema.py:163-190); see ``filter_schema``."""

    nodeset_fn: Callable[[str, NodeSchema], bool] = lambda key, sch: True
    edgeset_fn: Callable[[str, EdgeSchema], bool] = lambda key, sch: True
    feature_fn: Callable[[str, FeatureSchema], bool] = lambda key, sch: True
    node_feature_fn: Callable[[str, FeatureSchema], bool] = lambda key, sch: True
    edge_feature_fn: Callable[[str, FeatureSchema], bool] = lambda key, sch: True
