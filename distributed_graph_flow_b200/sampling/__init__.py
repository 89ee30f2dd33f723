"""Sampling API (names of dgf/src/api/sampling.py:20-30)."""

from distributed_graph_flow_b200.sampling.config import (
    PlanEdge,
    PlanNode,
    SamplingPlan,
    SimpleSamplingConfig,
    explicit_plan,
    simple_sampling_config_to_sampling_plan,
)
from distributed_graph_flow_b200.sampling.in_memory_sampler import (
    MODE_FIRST,
    MODE_MOST_RECENT,
    MODE_RANDOM,
    Sampler,
    add_features_to_samples,
    create_sampler,
)
