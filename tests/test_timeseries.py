"""Causal slicing of timeseries features (dgf/src/sampling/temporal.py,
in_memory_sampler.py:270-310).

CPU: the oracle restatement against the reference tests' vectors and the
schema grouping (extract_timeseries_schema_cache). GPU: the device slicer
through filter_timeseries_by_timestamp on the same vectors, through the
sampler on the reference's causal sampling test (per-seed cutoffs, the
slice_timeseries_by_seed switch, the missing-timestamps error), and against
the oracle on random ragged series (dtypes, inner shapes, per-node cutoffs,
caps, rows of different lengths in one group).
"""

import numpy as np
import pytest

from golden import reference_cases as rc


def _obj(rows, dtype=None):
    col = np.empty(len(rows), dtype=object)
    for i, r in enumerate(rows):
        col[i] = np.asarray(r, dtype=dtype)
    return col


def _assert_cols(got, exp, msg=""):
    assert len(got) == len(exp), msg
    for g, e in zip(got, exp):
        g = np.asarray(g)
        np.testing.assert_array_equal(g, np.asarray(e, dtype=g.dtype), err_msg=msg)


@pytest.mark.parametrize("case", rc.TS_FILTER_CASES, ids=[c[0] for c in rc.TS_FILTER_CASES])
def test_oracle_timeseries_goldens(case):
    from oracle import oracle as O

    _, feats, groups, target, max_len, expected = case
    features = {k: _obj(v) for k, v in feats.items()}
    n = len(next(iter(feats.values())))
    out = O.filter_timeseries(features, groups, [target] * n, max_len)
    for k, v in expected.items():
        _assert_cols(out.get(k, features[k]), v, k)


def test_timeseries_schema_cache():
    from distributed_graph_flow_b200.data import schema as S
    from distributed_graph_flow_b200.util import temporal as T

    F, Fm, Sm = S.FeatureSchema, S.FeatureFormat, S.FeatureSemantic
    feats = {"time": F(Fm.INTEGER_64, Sm.TIMESTAMP, is_timeseries=True, is_creation_time=True, group="time"),
             "signal": F(Fm.FLOAT_32, Sm.NUMERICAL, is_timeseries=True, group="time"),
             "waveform": F(Fm.FLOAT_32, Sm.NUMERICAL, is_timeseries=True),
             "solo": F(Fm.INTEGER_64, Sm.TIMESTAMP, is_timeseries=True, is_creation_time=True),
             "static": F(Fm.INTEGER_64)}
    cache = T.extract_timeseries_schema_cache(S.GraphSchema({"hw": S.NodeSchema(feats)}, {}))
    specs = {(g.timestamp_feature_name, tuple(g.feature_names)) for g in cache.node_sets["hw"]}
    assert specs == {("time", ("time", "signal")), (None, ("waveform",)), ("solo", ("solo",))}
    assert cache.has_timeseries
    empty = T.extract_timeseries_schema_cache(S.GraphSchema({"hw": S.NodeSchema({"static": feats["static"]})}, {}))
    assert not empty.has_timeseries


@pytest.mark.gpu
@pytest.mark.parametrize("case", rc.TS_FILTER_CASES, ids=[c[0] for c in rc.TS_FILTER_CASES])
def test_gpu_filter_timeseries_goldens(cuda, case):
    from distributed_graph_flow_b200.data import in_memory_graph as img
    from distributed_graph_flow_b200.sampling import temporal
    from distributed_graph_flow_b200.util import temporal as T

    _, feats, groups, target, max_len, expected = case
    n = len(next(iter(feats.values())))
    features = {k: _obj(v, np.int64 if k in ("time", "timestamps") else np.float32) for k, v in feats.items()}
    specs = [T.TimeseriesGroupSpec(ts, names) for ts, names in groups]
    edge = "edge" in case[0]
    if edge:
        graph = img.InMemoryGraph(node_sets={"a": img.InMemoryNodeSet(num_nodes=1)},
                                  edge_sets={"e": img.InMemoryEdgeSet(np.zeros((2, n), np.int64), features)})
        cache = T.TimeseriesSchemaCache({}, {"e": specs}, True)
    else:
        graph = img.InMemoryGraph(node_sets={"hw": img.InMemoryNodeSet(num_nodes=n, features=features)}, edge_sets={})
        cache = T.TimeseriesSchemaCache({"hw": specs, "missing": specs}, {}, True)
    temporal.filter_timeseries_by_timestamp(graph, cache, target, max_len)
    got = graph.edge_sets["e"].features if edge else graph.node_sets["hw"].features
    for k, v in expected.items():
        _assert_cols(got[k], v, k)


def _causal_graph():
    from distributed_graph_flow_b200.data import in_memory_graph as img
    from distributed_graph_flow_b200.data import schema as S
    from distributed_graph_flow_b200.transform import temporal as tt

    F, Fm, Sm = S.FeatureSchema, S.FeatureFormat, S.FeatureSemantic
    graph = img.InMemoryGraph(
        node_sets={"alerts": img.InMemoryNodeSet(num_nodes=2, features={"#creation_time": np.array([30, 60])}),
                   "hardware": img.InMemoryNodeSet(num_nodes=1, features={
                       "time": _obj([rc.TS_SAMPLER_TIME], np.int64),
                       "signal": _obj([np.arange(1, 8, dtype=np.float32)])})},
        edge_sets={"hardware_to_alert": img.InMemoryEdgeSet(np.array([[0, 0], [0, 1]], np.int64))})
    schema = S.GraphSchema(
        node_sets={"alerts": S.NodeSchema({"#creation_time": F(Fm.INTEGER_64, Sm.TIMESTAMP, is_creation_time=True)}),
                   "hardware": S.NodeSchema({
                       "time": F(Fm.INTEGER_64, Sm.TIMESTAMP, is_timeseries=True, is_creation_time=True, group="time"),
                       "signal": F(Fm.FLOAT_32, Sm.NUMERICAL, is_timeseries=True, group="time")})},
        edge_sets={"hardware_to_alert": S.EdgeSchema(source="hardware", target="alerts")})
    return tt.propagate_timestamp_to_edges(graph, schema)


@pytest.mark.gpu
def test_gpu_sampler_causal_slicing(cuda):
    from distributed_graph_flow_b200 import sampling

    graph, schema = _causal_graph()
    conf = sampling.SimpleSamplingConfig(seed_nodeset="alerts", num_hops=1, hop_width=10, reverse=True,
                                         temporal_sampling=True)
    s = sampling.create_sampler(graph, conf, schema, batch_size=2, return_features=True, max_timeseries_len=3)
    assert s._slice_timeseries_by_seed
    samples = s.sample([0, 1], seed_timestamps=np.array([30, 60], np.int64))
    assert samples[0].node_sets["alerts"].features["#creation_time"][0] == 30
    assert samples[1].node_sets["alerts"].features["#creation_time"][0] == 60
    for smp, (t, sig) in zip(samples, rc.TS_SAMPLER_EXPECTED):
        np.testing.assert_array_equal(smp.node_sets["hardware"].features["time"][0], t)
        np.testing.assert_array_equal(smp.node_sets["hardware"].features["signal"][0], sig)
    off = sampling.create_sampler(graph, conf, schema, batch_size=2, return_features=True, max_timeseries_len=3,
                                  slice_timeseries_by_seed=False)
    full = off.sample([0], seed_timestamps=np.array([30], np.int64))
    np.testing.assert_array_equal(full[0].node_sets["hardware"].features["time"][0], rc.TS_SAMPLER_TIME)
    # Slicing requested on a non-temporal plan: seed timestamps are required.
    conf2 = sampling.SimpleSamplingConfig(seed_nodeset="alerts", num_hops=1, hop_width=10, reverse=True)
    s2 = sampling.create_sampler(graph, conf2, schema, batch_size=2, return_features=True,
                                 slice_timeseries_by_seed=True)
    with pytest.raises(ValueError, match="`seed_timestamps` must be provided"):
        s2.sample([0])


@pytest.mark.gpu
@pytest.mark.parametrize("max_len", [None, -1, 0, 2, 1000])
def test_gpu_slicer_matches_oracle(cuda, max_len):
    from distributed_graph_flow_b200.sampling import temporal
    from distributed_graph_flow_b200.util import temporal as T
    from oracle import oracle as O

    rng = np.random.default_rng(0 if max_len is None else abs(max_len))
    n = 300
    lens = rng.integers(0, 40, n)
    times = [np.sort(rng.integers(0, 100, k)) for k in lens]
    feats = {"t": _obj(times, np.int64),
             "f32": _obj([rng.standard_normal(k).astype(np.float32) for k in lens]),
             "i32x3": _obj([rng.integers(-5, 5, (k, 3)).astype(np.int32) for k in lens]),
             # one feature with rows a little shorter than the timestamps: numpy clips the slice
             "short": _obj([rng.standard_normal(max(0, k - 2)) for k in lens])}
    groups = [("t", ["t", "f32", "i32x3", "short"])]
    slicer = temporal.TimeseriesSlicer(feats, [T.TimeseriesGroupSpec("t", groups[0][1])])
    rows = rng.integers(0, n, 500)
    cutoffs = rng.integers(-5, 110, 500)
    got = slicer.slice(rows, cutoffs, max_len)
    sub = {k: v[rows] for k, v in feats.items()}
    exp = O.filter_timeseries(sub, groups, cutoffs, max_len)
    for k in groups[0][1]:
        _assert_cols(got[k], exp[k], k)
        assert all(np.asarray(g).dtype == np.asarray(e).dtype for g, e in zip(got[k], exp[k])), k


def test_float_timestamps_rejected():
    """A fractional timestamp series is refused before any device work (an
    int64 search would let t = 1.5 pass a cutoff of 1)."""
    from distributed_graph_flow_b200.sampling import temporal
    from distributed_graph_flow_b200.util import temporal as T

    feats = {"t": _obj([np.array([0.5, 1.5]), np.array([2.0])]), "v": _obj([np.ones(2), np.ones(1)])}
    with pytest.raises(ValueError, match="integer timestamps"):
        temporal.TimeseriesSlicer(feats, [T.TimeseriesGroupSpec("t", ["t", "v"])])
