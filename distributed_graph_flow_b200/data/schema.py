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
from typing import Dict, Optional, Tuple


class FeatureFormat(enum.Enum):
    UNKNOWN = "UNKNOWN"
    FLOAT_32 = "FLOAT_32"
    FLOAT_64 = "FLOAT_64"
    INTEGER_32 = "INTEGER_32"
    INTEGER_64 = "INTEGER_64"
    BOOLEAN = "BOOLEAN"
    BYTES = "BYTES"


class FeatureSemantic(enum.Enum):
    UNKNOWN = "UNKNOWN"
    NUMERICAL = "NUMERICAL"
    CATEGORICAL = "CATEGORICAL"
    EMBEDDING = "EMBEDDING"
    TIMESTAMP = "TIMESTAMP"
    PRIMARY_ID = "PRIMARY_ID"
    TEXT = "TEXT"


Shape = Optional[Tuple[int, ...]]


@dataclasses.dataclass
class FeatureSchema:
    format: FeatureFormat
    semantic: FeatureSemantic = FeatureSemantic.UNKNOWN
    shape: Shape = None
    num_categorical_values: Optional[int] = None
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
