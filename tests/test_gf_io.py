"""GF graph loading (dgf/src/io/graph_in_memory.py, io_ext.cc).

CPU: the oracle's id mapping against io_cc_test.py's vectors, the schema JSON
round trip, primary-key fixing and filtering, and write_graph's files read
back with pyarrow. GPU: the device id index against the same vectors and
against the oracle on random ids (integers with repeats, fixed-width bytes of
different widths and trailing zeros, Arrow binary columns, unknown ids), and
read_graph on the reference's GF fixture (schema, features, adjacency,
filter, dangling-edge error and removal, write/read round trip, timestamp)
plus the device-resident path into create_sampler.
"""

import json
import os

import numpy as np
import pytest

from golden import reference_cases as rc


def _schema():
    from distributed_graph_flow_b200.data import schema as S

    F, M, FS = S.FeatureFormat, S.FeatureSemantic, S.FeatureSchema
    n1 = {"f2": FS(F.FLOAT_32, M.EMBEDDING, shape=(2,)), "f1": FS(F.BYTES, M.CATEGORICAL, shape=(1,)),
          "#id": FS(F.BYTES, M.PRIMARY_ID)}
    n2 = {"f3": FS(F.INTEGER_64, M.NUMERICAL, shape=None), "f4": FS(F.INTEGER_64, M.NUMERICAL, shape=()),
          "f5": FS(F.INTEGER_64, M.NUMERICAL, shape=(None,)), "f6": FS(F.INTEGER_64, M.NUMERICAL, shape=(None, 2)),
          "#id": FS(F.INTEGER_64, M.PRIMARY_ID)}
    eid = lambda: {"#id": FS(F.BYTES, M.PRIMARY_ID)}  # noqa: E731
    return S.GraphSchema(node_sets={"n1": S.NodeSchema(n1), "n2": S.NodeSchema(n2)},
                         edge_sets={"e1": S.EdgeSchema("n1", "n1", eid()), "e2": S.EdgeSchema("n1", "n2", eid())})


def _expected_graph(timestamp=None):
    from distributed_graph_flow_b200.data import in_memory_graph as img

    obj = lambda xs: np.array([np.array(x, np.int64) for x in xs] + [None], dtype=object)[:-1]  # noqa: E731
    n1 = {"f2": np.array(rc.GF_N1["f2"], np.float32), "f1": np.array(rc.GF_N1["f1"]), "#id": np.array(rc.GF_N1["#id"])}
    sh = rc.GF_N2_SHARDS
    n2 = {"f3": np.array(sh[0]["f3"] + sh[1]["f3"]), "f4": np.array(sh[0]["f4"] + sh[1]["f4"]),
          "f5": obj(sh[0]["f5"] + sh[1]["f5"]), "f6": obj(sh[0]["f6"] + sh[1]["f6"]),
          "#id": np.array(sh[0]["#id"] + sh[1]["#id"])}
    return img.InMemoryGraph(
        node_sets={"n1": img.InMemoryNodeSet(num_nodes=2, features=n1), "n2": img.InMemoryNodeSet(num_nodes=2, features=n2)},
        edge_sets={"e1": img.InMemoryEdgeSet(np.array(rc.GF_ADJACENCY["e1"]), {"#id": np.array(rc.GF_E1["#id"])}),
                   "e2": img.InMemoryEdgeSet(np.array(rc.GF_ADJACENCY["e2"]), {"#id": np.array(rc.GF_E2["#id"])})},
        timestamp=timestamp)


def _write_fixture(path, dangling=False):
    """The reference's generate_gf_graph(path, edge_ids=True) layout."""
    import pyarrow as pa
    import pyarrow.parquet as pq

    from distributed_graph_flow_b200.io import graph_in_memory as gim

    os.makedirs(os.path.join(path, "nodesets"))
    os.makedirs(os.path.join(path, "edgesets"))
    gim.write_schema(_schema(), os.path.join(path, "schema.json"))
    with open(os.path.join(path, "metadata.json"), "w") as f:
        f.write(json.dumps({"version": 0, "timestamp": None}))
    pq.write_table(pa.Table.from_arrays(
        [pa.array(rc.GF_N1["#id"]), pa.array(rc.GF_N1["f1"], type=pa.list_(pa.binary(), 1)),
         pa.array(rc.GF_N1["f2"], type=pa.list_(pa.float32(), 2))], names=["#id", "f1", "f2"]),
        os.path.join(path, "nodesets", "n1-00000-of-00001.parquet"))
    for i, sh in enumerate(rc.GF_N2_SHARDS):
        pq.write_table(pa.Table.from_arrays(
            [pa.array(sh["#id"]), pa.array(sh["f3"]), pa.array(sh["f4"]), pa.array(sh["f5"]),
             pa.array(sh["f6"], type=pa.list_(pa.list_(pa.int64(), 2)))], names=["#id", "f3", "f4", "f5", "f6"]),
            os.path.join(path, "nodesets", f"n2-0000{i}-of-00002.parquet"))
    pq.write_table(pa.Table.from_arrays([pa.array(rc.GF_E1[k]) for k in ("#source", "#target", "#id")],
                                        names=["#source", "#target", "#id"]),
                   os.path.join(path, "edgesets", "e1-00000-of-00001.parquet"))
    src = [rc.GF_E2["#source"][0], b"missing" if dangling else rc.GF_E2["#source"][1]]
    pq.write_table(pa.Table.from_arrays([pa.array(src), pa.array(rc.GF_E2["#target"]), pa.array(rc.GF_E2["#id"])],
                                        names=["#source", "#target", "#id"]),
                   os.path.join(path, "edgesets", "e2-00000-of-00001.parquet"))


def _assert_values(a, b, msg):
    a, b = np.asarray(a), np.asarray(b)
    if b.dtype == object:
        assert a.dtype == object and len(a) == len(b), msg
        for x, y in zip(a, b):
            np.testing.assert_array_equal(np.asarray(x), np.asarray(y), err_msg=msg)
    else:
        assert a.dtype.kind == b.dtype.kind, f"{msg}: {a.dtype} vs {b.dtype}"
        np.testing.assert_array_equal(a, b, err_msg=msg)


def _assert_graph(got, exp):
    assert set(got.node_sets) == set(exp.node_sets) and set(got.edge_sets) == set(exp.edge_sets)
    for n, ns in exp.node_sets.items():
        assert got.node_sets[n].num_nodes == ns.num_nodes
        assert set(got.node_sets[n].features) == set(ns.features), n
        for k, v in ns.features.items():
            _assert_values(got.node_sets[n].features[k], v, f"{n}.{k}")
    for n, es in exp.edge_sets.items():
        adj = got.edge_sets[n].adjacency
        adj = adj.cpu().numpy() if hasattr(adj, "cpu") else adj
        np.testing.assert_array_equal(adj, es.adjacency, err_msg=n)
        assert set(got.edge_sets[n].features) == set(es.features), n
        for k, v in es.features.items():
            _assert_values(got.edge_sets[n].features[k], v, f"{n}.{k}")
    assert got.timestamp == exp.timestamp


# ---------------------------------------------------------------------------
# CPU
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("case", rc.ID_MAP_CASES, ids=[c[0] for c in rc.ID_MAP_CASES])
def test_oracle_id_map_goldens(case):
    from oracle import oracle as O

    _, index, query, exp, mm = case
    a, b = np.array(index, dtype=np.bytes_), np.array(query, dtype=np.bytes_)
    for fn in (O.id_map, lambda x, y: O.bytes_map(x, y, threads=3)):
        out, m = fn(a, b)
        np.testing.assert_array_equal(out, exp)
        assert m == mm


def test_schema_json_fix_filter():
    from distributed_graph_flow_b200.data import schema as S
    from distributed_graph_flow_b200.io import graph_in_memory as gim

    s = _schema()
    assert S.GraphSchema.from_json(s.to_json(indent=2)) == s
    d = json.loads(s.to_json())
    assert d["node_sets"]["n2"]["features"]["f6"]["shape"] == [None, 2]
    assert d["node_sets"]["n1"]["features"]["#id"]["semantic"] == "PRIMARY_ID"
    # Primary keys are inferred from #id-like names.
    t = _schema()
    t.node_sets["n1"].features["#id"].semantic = S.FeatureSemantic.UNKNOWN
    t.edge_sets["e1"].features["#id"].semantic = S.FeatureSemantic.UNKNOWN
    gim.fix_schema(t)
    assert t == s
    t.node_sets["n1"].features["id"] = S.FeatureSchema(S.FeatureFormat.BYTES)
    t.node_sets["n1"].features["#id"].semantic = S.FeatureSemantic.UNKNOWN
    with pytest.raises(ValueError, match="multiple feature that look like primary key"):
        gim.fix_schema(t)
    f = gim.filter_schema(s, S.GraphSchemaFilter(edgeset_fn=lambda k, sch: False))
    assert f.edge_sets == {} and f.node_sets == s.node_sets
    f = gim.filter_schema(s, S.GraphSchemaFilter(nodeset_fn=lambda k, sch: k == "n1"))
    assert list(f.edge_sets) == ["e1"]


def test_write_graph_files(tmp_path):
    import pyarrow.parquet as pq

    from distributed_graph_flow_b200.io import graph_in_memory as gim

    out = str(tmp_path / "g")
    gim.write_graph(_expected_graph(), _schema(), out)
    files = sorted(os.path.relpath(os.path.join(d, f), out) for d, _, fs in os.walk(out) for f in fs)
    assert files == ["edgesets/e1-00000-of-00001.parquet", "edgesets/e2-00000-of-00001.parquet", "metadata.json",
                     "nodesets/n1-00000-of-00001.parquet", "nodesets/n2-00000-of-00001.parquet", "schema.json"]
    e2 = pq.read_table(os.path.join(out, "edgesets/e2-00000-of-00001.parquet")).to_pydict()
    assert e2["#source"] == [b"1", b"1"] and e2["#target"] == [1, 2] and e2["#id"] == [b"A", b"B"]
    assert json.load(open(os.path.join(out, "metadata.json"))) == {"version": 0, "timestamp": None}


# ---------------------------------------------------------------------------
# GPU
# ---------------------------------------------------------------------------
@pytest.mark.gpu
def test_gpu_id_mapper_goldens(cuda):
    from distributed_graph_flow_b200.io import ids

    for _, index, query, exp, mm in rc.ID_MAP_CASES:
        out, m = ids.ByteIdToIdxMapper(np.array(index, dtype=np.bytes_))(np.array(query, dtype=np.bytes_))
        np.testing.assert_array_equal(out, exp)
        assert m == mm
    i1, i2, q1, q2, exp, m1, m2 = rc.PAIR_MAP_CASE
    res, a, b = ids.PairMapping(ids.ByteIdToIdxMapper(np.array(i1)), ids.ByteIdToIdxMapper(np.array(i2)),
                                np.array(q1), np.array(q2), 3)
    np.testing.assert_array_equal(res, exp)
    assert (a, b) == (m1, m2)


@pytest.mark.gpu
@pytest.mark.parametrize("seed", [0, 1])
def test_gpu_id_index_matches_oracle(cuda, seed):
    import pyarrow as pa

    from distributed_graph_flow_b200.io import ids
    from oracle import oracle as O

    rng = np.random.default_rng(seed)
    # Integer ids with repeats (the last position wins) and unknown queries.
    index = rng.integers(-(1 << 40), 1 << 40, 50_000)
    index[rng.integers(0, 50_000, 3000)] = index[rng.integers(0, 50_000, 3000)]
    query = np.concatenate([index[rng.integers(0, 50_000, 70_000)], rng.integers(0, 1 << 40, 5000)])
    rng.shuffle(query)
    got, m = ids.IdIndex(index).lookup(query)
    exp, me = O.id_map(index, query)
    np.testing.assert_array_equal(got.cpu().numpy(), exp)
    assert m == me
    # Byte ids: index width 12, queries width 16 (extra zero padding), some
    # ids ending in zero bytes, repeats, unknown ids.
    words = [b"n%d" % v for v in rng.integers(0, 10**9, 40_000)] + [b"z\0", b"", b"q\0\0"]
    index_b = np.array(words, dtype="S12")
    qb = index_b[rng.integers(0, len(index_b), 60_000)].astype("S16")
    qb = np.concatenate([qb, np.array([b"nope%d" % i for i in range(500)], dtype="S16")])
    rng.shuffle(qb)
    exp, me = O.id_map(index_b, qb)
    got, m = ids.IdIndex(index_b).lookup(qb)
    np.testing.assert_array_equal(got.cpu().numpy(), exp)
    assert m == me
    # The same width on both sides (row-compare build and lookup kernels, 1, 3
    # and 5 words per id), with explicit repeats: the last position wins.
    index_r = index_b.copy()
    index_r[rng.integers(0, len(index_r), 2000)] = index_r[rng.integers(0, len(index_r), 2000)]
    for width in ("S12", "S20", "S4"):
        ix = index_r.astype(width)  # S4 truncates the ids: more repeats
        qq = np.concatenate([ix[rng.integers(0, len(ix), 30_000)],
                             np.array([b"nope%d" % i for i in range(300)], dtype=width)])
        rng.shuffle(qq)
        exp, me = O.id_map(ix, qq)
        got, m = ids.IdIndex(ix).lookup(qq)
        np.testing.assert_array_equal(got.cpu().numpy(), exp, err_msg=width)
        assert m == me, width
    # Arrow binary columns (variable length, two chunks, sliced) on both sides.
    arrow_index = pa.chunked_array([pa.array([bytes(x) for x in index_b[:20_000]]),
                                    pa.array([bytes(x) for x in index_b[20_000:]])])
    arrow_q = pa.array([bytes(x) for x in qb]).slice(7)
    got, m = ids.IdIndex(arrow_index).lookup(arrow_q)
    exp, me = O.id_map(index_b, qb[7:])
    np.testing.assert_array_equal(got.cpu().numpy(), exp)
    assert m == me
    with pytest.raises(ValueError, match="integer ids against byte ids"):
        ids.IdIndex(index).lookup(qb[:3])


@pytest.mark.gpu
def test_gpu_read_graph_fixture(cuda, tmp_path):
    from distributed_graph_flow_b200.data import schema as S
    from distributed_graph_flow_b200.io import graph_in_memory as gim

    path = str(tmp_path / "gf")
    _write_fixture(path)
    graph, schema = gim.read_graph(path)
    assert schema == _schema()
    _assert_graph(graph, _expected_graph())
    graph, schema = gim.read_graph(path, schema_filter=S.GraphSchemaFilter(edgeset_fn=lambda k, sch: False))
    assert schema.edge_sets == {} and graph.edge_sets == {}
    bad = str(tmp_path / "bad")
    _write_fixture(bad, dangling=True)
    with pytest.raises(ValueError, match="Node ID 'missing' not found in nodeset 'n1'"):
        gim.read_graph(bad)
    graph, _ = gim.read_graph(bad, remove_dangling_edges=True)
    assert graph.edge_sets["e2"].num_edges() == 1
    np.testing.assert_array_equal(graph.edge_sets["e2"].adjacency, [[0], [0]])
    np.testing.assert_array_equal(graph.edge_sets["e2"].features["#id"], [b"A"])
    # Round trip through write_graph, with and without a timestamp.
    for ts in (123456, None):
        out = str(tmp_path / f"rt{ts}")
        gim.write_graph(_expected_graph(ts), _schema(), out)
        g2, s2 = gim.read_graph(out)
        assert s2 == _schema()
        _assert_graph(g2, _expected_graph(ts))


@pytest.mark.gpu
def test_gpu_read_graph_device_into_sampler(cuda, tmp_path):
    """read_graph(device=...) keeps adjacencies in HBM; the sampler built on
    them samples exactly what the host-array path samples."""
    from distributed_graph_flow_b200 import sampling
    from distributed_graph_flow_b200.data import in_memory_graph as img
    from distributed_graph_flow_b200.data import schema as S
    from distributed_graph_flow_b200.io import graph_in_memory as gim

    rng = np.random.default_rng(3)
    n, m = 3000, 40_000
    ids_ = np.array([b"user/%07d" % v for v in rng.permutation(10**6)[:n]])
    adj = np.stack([rng.integers(0, n, m), rng.integers(0, n, m)])
    g = img.InMemoryGraph(node_sets={"u": img.InMemoryNodeSet(num_nodes=n, features={"#id": ids_})},
                          edge_sets={"f": img.InMemoryEdgeSet(adjacency=adj)})
    sch = S.GraphSchema(node_sets={"u": S.NodeSchema({"#id": S.FeatureSchema(S.FeatureFormat.BYTES,
                                                                              S.FeatureSemantic.PRIMARY_ID)})},
                        edge_sets={"f": S.EdgeSchema("u", "u")})
    path = str(tmp_path / "g")
    gim.write_graph(g, sch, path)
    host, _ = gim.read_graph(path)
    dev, _ = gim.read_graph(path, device="cuda")
    assert dev.edge_sets["f"].adjacency.is_cuda
    np.testing.assert_array_equal(host.edge_sets["f"].adjacency, adj)
    plan = sampling.explicit_plan("u", "f", [8, 4])
    seeds = rng.integers(0, n, 64)
    a = sampling.create_sampler(host, plan, sch, debug_sampling=True, return_node_idxs=True, return_features=False,
                                batch_size=64).sample(seeds)
    b = sampling.create_sampler(dev, plan, sch, debug_sampling=True, return_node_idxs=True, return_features=False,
                                batch_size=64).sample(seeds)
    for x, y in zip(a, b):
        np.testing.assert_array_equal(x.node_sets["u"].features["#idx"], y.node_sets["u"].features["#idx"])
        np.testing.assert_array_equal(x.edge_sets["f"].adjacency, y.edge_sets["f"].adjacency)


def test_parquet_columns_to_numpy():
    """Column conversions of dgf/src/io/parquet.py:63-135: binary -> 'S<max>'
    (zero padded, chunked and sliced), string -> bytes, fixed-size lists ->
    [n, k] (nested), variable lists -> object arrays, numbers as they are."""
    import pyarrow as pa

    from distributed_graph_flow_b200.io import parquet as P

    col = pa.chunked_array([pa.array([b"1", b"22", b""]), pa.array([b"abc", b"z"]).slice(1)])
    out = P.column_to_numpy(col)
    assert out.dtype == np.dtype("S2") and out.tolist() == [b"1", b"22", b"", b"z"]  # the slice drops "abc"
    assert P.column_to_numpy(pa.chunked_array([pa.array([b""])])).dtype == np.dtype("S1")
    assert P.column_to_numpy(pa.chunked_array([pa.array(["ab", "c"])])).tolist() == [b"ab", b"c"]
    fixed = P.column_to_numpy(pa.chunked_array([pa.array([[[1, 2], [3, 4]]], type=pa.list_(pa.list_(pa.int64(), 2), 2))]))
    assert fixed.shape == (1, 2, 2) and fixed.tolist() == [[[1, 2], [3, 4]]]
    var = P.column_to_numpy(pa.chunked_array([pa.array([[1], [2, 3]]), pa.array([[4, 5, 6]])]))
    assert var.dtype == object and [v.tolist() for v in var] == [[1], [2, 3], [4, 5, 6]]
    f = P.column_to_numpy(pa.chunked_array([pa.array([1.5, 2.5], type=pa.float32())]))
    assert f.dtype == np.float32 and f.tolist() == [1.5, 2.5]
    assert P.sharded_filename("e1", 3, 12) == "e1-00003-of-00012.parquet"
    assert [P.estimate_num_shards(n) for n in (0, 1, 1000, 1001, 10**9)] == [0, 1, 1, 2, 100]


def test_oracle_id_maps_agree():
    """The Python and C++ restatements of the id map agree on random ids with
    repeats, trailing zeros, different widths and unknown ids."""
    from oracle import oracle as O

    rng = np.random.default_rng(4)
    index = np.array([b"k%d" % v for v in rng.integers(0, 5000, 4000)] + [b"t\0", b""], dtype="S10")
    query = np.concatenate([index[rng.integers(0, len(index), 9000)].astype("S14"),
                            np.array([b"miss%d" % i for i in range(50)], dtype="S14")])
    rng.shuffle(query)
    a, ma = O.id_map(index, query)
    for th in (1, 4):
        b, mb = O.bytes_map(index, query, threads=th)
        np.testing.assert_array_equal(a, b)
        assert ma == mb


def test_parquet_write_read_round_trip(tmp_path):
    """write_numpy_dict then the reader's column conversion give back every
    feature kind of the GF fixture (scalars, fixed and variable lists, bytes),
    split over several shards."""
    from distributed_graph_flow_b200.io import parquet as P

    exp = _expected_graph()
    for name, ns in exp.node_sets.items():
        P.write_numpy_dict(ns.features, name, str(tmp_path), _schema().node_sets[name].features, num_shards=2)
        table = P.read_tables(P.list_shards(str(tmp_path / name)))
        got, count = P.table_to_numpy_dict(table)
        assert count == ns.num_nodes
        for k, v in ns.features.items():
            _assert_values(got[k], v, f"{name}.{k}")


def test_fix_schema_suspicious_shapes():
    from distributed_graph_flow_b200.data import schema as S
    from distributed_graph_flow_b200.io import graph_in_memory as gim

    F = S.FeatureSchema
    s = S.GraphSchema(node_sets={"n": S.NodeSchema({"#id": F(S.FeatureFormat.BYTES, shape=(None, 1)),
                                                   "x": F(S.FeatureFormat.FLOAT_32, shape=(None, 4))})},
                      edge_sets={})
    gim.fix_schema(s)
    f = s.node_sets["n"].features
    assert f["#id"].shape == () and f["x"].shape == (4,)
    assert f["#id"].semantic == S.FeatureSemantic.PRIMARY_ID
    with pytest.raises(ValueError, match="no feature look like a primary key"):
        gim.fix_schema(S.GraphSchema(node_sets={"m": S.NodeSchema({"y": F(S.FeatureFormat.INTEGER_64)})},
                                     edge_sets={}))


def test_fix_schema_pound_id_fallback_and_tf_example():
    """dgf/src/analyse/schema.py:168-265: the '#id' fallback key and the TF
    Example format fix (int32 / bool -> int64, float64 -> float32)."""
    from distributed_graph_flow_b200.data import schema as S
    from distributed_graph_flow_b200.io import graph_in_memory as gim

    F = S.FeatureSchema
    s = S.GraphSchema(node_sets={"m": S.NodeSchema({"y": F(S.FeatureFormat.INTEGER_32),
                                                   "b": F(S.FeatureFormat.BOOL)})},
                      edge_sets={"e": S.EdgeSchema(source="m", target="m",
                                                   features={"w": F(S.FeatureFormat.FLOAT_64),
                                                             "z": F(S.FeatureFormat.BYTES)})})
    gim.fix_schema(s, create_pound_id_as_fall_back=True, tf_example=True)
    nf = s.node_sets["m"].features
    assert nf["#id"].format == S.FeatureFormat.BYTES and nf["#id"].semantic == S.FeatureSemantic.PRIMARY_ID
    assert nf["y"].format == S.FeatureFormat.INTEGER_64 and nf["b"].format == S.FeatureFormat.INTEGER_64
    ef = s.edge_sets["e"].features
    assert ef["w"].format == S.FeatureFormat.FLOAT_32 and ef["z"].format == S.FeatureFormat.BYTES
    # Without tf_example the formats stay; a key-like feature wins over the fallback.
    s2 = S.GraphSchema(node_sets={"m": S.NodeSchema({"#id": F(S.FeatureFormat.BYTES),
                                                    "y": F(S.FeatureFormat.INTEGER_32)})}, edge_sets={})
    gim.fix_schema(s2, create_pound_id_as_fall_back=True)
    assert s2.node_sets["m"].features["y"].format == S.FeatureFormat.INTEGER_32
    assert s2.node_sets["m"].features["#id"].semantic == S.FeatureSemantic.PRIMARY_ID
