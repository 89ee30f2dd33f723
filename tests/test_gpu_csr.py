"""Device CSR builder vs the oracle and the reference's known answers."""

import numpy as np
import pytest

from golden import reference_cases as rc
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ext(cuda):
    from distributed_graph_flow_b200.sampling import _in_memory_sampler_ext

    return _in_memory_sampler_ext


def _edges(edges):
    if not edges:
        return np.zeros((2, 0), np.int64), None
    a = np.array([e[:2] for e in edges], np.int64).T
    ts = np.array([e[2] for e in edges], np.int64) if len(edges[0]) == 3 else None
    return a, ts


@pytest.mark.parametrize("case", rc.CSR_CASES, ids=[c[0] for c in rc.CSR_CASES])
def test_known_answers(ext, case):
    name, edges, n_src, n_dst, blocks, targets, ts = case
    adj, t = _edges(edges)
    idx = ext.BuildAdjacencyIndex(adj, t, False, n_src, n_dst)
    np.testing.assert_array_equal(idx.rowptr.cpu().numpy(), blocks)
    np.testing.assert_array_equal(idx.col.cpu().numpy(), targets)
    if ts is not None:
        np.testing.assert_array_equal(idx.ts.cpu().numpy(), ts)


@pytest.mark.parametrize("case", rc.INDEX_STRING_CASES)
def test_index_strings(ext, case):
    adj, rev, n_src, n_dst, expected = case
    idx = ext.BuildAdjacencyIndex(np.array(adj, np.int64).reshape(2, -1), None, rev, n_src, n_dst)
    assert str(idx) == expected


def _random_edges(rng, n_src, n_dst, m, ts_range=None):
    src = np.minimum((rng.pareto(1.1, m) * 3).astype(np.int64), n_src - 1)
    dst = rng.integers(0, n_dst, m)
    # Duplicated edges on purpose.
    dup = rng.integers(0, m, m // 10)
    src = np.concatenate([src, src[dup]])
    dst = np.concatenate([dst, dst[dup]])
    ts = None
    if ts_range is not None:
        lo, hi = ts_range
        ts = rng.integers(lo, hi, len(src), dtype=np.int64)
    return np.stack([src, dst]), ts


@pytest.mark.parametrize("reversed_", [False, True])
@pytest.mark.parametrize(
    "ts_range", [None, (0, 50), (-(1 << 62), 1 << 62)], ids=["plain", "ts-narrow", "ts-wide-multipass"]
)
@pytest.mark.parametrize("m", [1, 1000, 70000])
def test_matches_oracle(ext, reversed_, ts_range, m):
    rng = np.random.default_rng(m + (7 if reversed_ else 0))
    n_src, n_dst = 300, 5000
    adj, ts = _random_edges(rng, n_src, n_dst, m, ts_range)
    mine = ext.BuildAdjacencyIndex(adj, ts, reversed_, n_src, n_dst)
    ref = O.Index(adj, ts, reversed_, n_src, n_dst).arrays()
    np.testing.assert_array_equal(mine.rowptr.cpu().numpy(), ref["source_blocks"])
    np.testing.assert_array_equal(mine.col.cpu().numpy(), ref["target_node_idxs"])
    if ts is not None:
        np.testing.assert_array_equal(mine.ts.cpu().numpy(), ref["timestamps"])


def test_edge_positions_invert_the_sort(ext):
    rng = np.random.default_rng(3)
    adj, _ = _random_edges(rng, 50, 80, 3000)
    for rev in (False, True):
        idx = ext.BuildAdjacencyIndex(adj, None, rev, 50, 80, populate_edge_idxs=True)
        pos = idx.edge_pos.cpu().numpy()
        col = idx.col.cpu().numpy()
        rowptr = idx.rowptr.cpu().numpy()
        assert sorted(pos.tolist()) == list(range(adj.shape[1]))
        row_of = np.repeat(np.arange(len(rowptr) - 1), np.diff(rowptr))
        s, d = (adj[1], adj[0]) if rev else (adj[0], adj[1])
        np.testing.assert_array_equal(row_of[pos], s)
        np.testing.assert_array_equal(col[pos], d)


def test_invalid_ids_report_reference_message(ext):
    adj = np.array([[0, 1, 5, 9], [0, 1, 2, 3]])
    with pytest.raises(ValueError, match=r"Invalid source node index 5. The node index should be between 0 and 4."):
        ext.BuildAdjacencyIndex(adj, None, False, 4, 4)
    adj = np.array([[0, 1, 2], [0, -1, 2]])
    with pytest.raises(ValueError, match=r"Invalid target node index -1. The node index should be between 0 and 4."):
        ext.BuildAdjacencyIndex(adj, None, False, 4, 4)
    # Reversed: the roles swap, as in the reference.
    adj = np.array([[0, 1], [0, 7]])
    with pytest.raises(ValueError, match=r"Invalid source node index 7. The node index should be between 0 and 5."):
        ext.BuildAdjacencyIndex(adj, None, True, 3, 5)
