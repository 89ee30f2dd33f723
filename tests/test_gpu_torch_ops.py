"""The aggregation boundary as torch operators (dgfx::csr_spmm,
dgfx::segment_sum, dgfx::segment_softmax, dgfx::sage_mean_linear_relu):
forward and gradients against the float64 oracle, torch.library's own op
checks (schema, fake tensors, autograd registration), the GCN / GIN
propagation matrices of the reference's sparse layers, and the mean
aggregation over a merged sampled batch.

Tolerances: fp32 1e-5 and bf16 1e-2 relative to the magnitude of the
summed terms (sum |a| |x| per output element), as for the forward SpMM."""

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops(cuda):
    from distributed_graph_flow_b200 import torch_ops

    return torch_ops


def _csr(rng, rows, cols, max_deg=40):
    deg = np.minimum((rng.pareto(1.3, rows) * 3).astype(np.int64), max_deg)
    rowptr = np.concatenate([[0], np.cumsum(deg)]).astype(np.int64)
    col = rng.integers(0, cols, rowptr[-1]).astype(np.int32)
    return rowptr, col


def _close(got, exp, mag, rel):
    got = np.asarray(got, np.float64)
    bad = np.abs(got - exp) > rel * np.maximum(mag, 1e-30) + 1e-30
    assert not bad.any(), f"{bad.sum()} elements off; worst {np.abs(got - exp).max():.3e}"


@pytest.mark.parametrize("normalize", [False, True])
@pytest.mark.parametrize("with_val", [False, True])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_csr_spmm_forward_backward(ops, normalize, with_val, dtype):
    rng = np.random.default_rng(3)
    R, C, F = 500, 300, 64
    rowptr, col = _csr(rng, R, C)
    val = rng.standard_normal(len(col)).astype(np.float32) if with_val else None
    x = rng.standard_normal((C, F)).astype(np.float32)
    dy = rng.standard_normal((R, F)).astype(np.float32)
    d = "cuda"
    xt = torch.from_numpy(x).to(d, dtype).requires_grad_(True)
    y = torch.ops.dgfx.csr_spmm(torch.from_numpy(rowptr).to(d), torch.from_numpy(col).to(d),
                                None if val is None else torch.from_numpy(val).to(d), xt, normalize, -1)
    y.backward(torch.from_numpy(dy).to(d, dtype))
    xq = xt.detach().float().cpu().numpy()  # the rounded inputs the kernel saw
    rel = 1e-5 if dtype == torch.float32 else 1e-2
    exp = O.csr_spmm(rowptr, col, xq, val, normalize)
    mag = O.csr_spmm(rowptr, col, np.abs(xq), None if val is None else np.abs(val), normalize)
    _close(y.detach().float().cpu().numpy(), exp, mag, rel)
    dyq = torch.from_numpy(dy).to(dtype).float().numpy()
    gexp = O.csr_spmm_grad_x(rowptr, col, dyq, C, val, normalize)
    gmag = O.csr_spmm_grad_x(rowptr, col, np.abs(dyq), C, None if val is None else np.abs(val), normalize)
    _close(xt.grad.float().cpu().numpy(), gexp, gmag, rel)


@pytest.mark.parametrize("mean", [False, True])
def test_segment_sum_forward_backward(ops, mean):
    rng = np.random.default_rng(5)
    n, S, F = 3000, 200, 32
    ids = rng.integers(-3, S + 3, n)  # some ids out of range: dropped
    data = rng.standard_normal((n, F)).astype(np.float32)
    dy = rng.standard_normal((S, F)).astype(np.float32)
    dt = torch.from_numpy(data).cuda().requires_grad_(True)
    y = torch.ops.dgfx.segment_sum(dt, torch.from_numpy(ids).cuda(), S, mean)
    y.backward(torch.from_numpy(dy).cuda())
    keep = (ids >= 0) & (ids < S)
    exp = O.segment_sum(data[keep], ids[keep], S, mean=mean)
    mag = O.segment_sum(np.abs(data[keep]), ids[keep], S, mean=mean)
    _close(y.detach().cpu().numpy(), exp, mag, 1e-5)
    _close(dt.grad.cpu().numpy(), O.segment_sum_grad(dy, ids, S, mean), np.abs(O.segment_sum_grad(dy, ids, S, mean)),
           1e-6)


def test_opcheck(ops):
    rng = np.random.default_rng(7)
    rowptr, col = _csr(rng, 64, 40)
    rp, cl = torch.from_numpy(rowptr).cuda(), torch.from_numpy(col).cuda()
    x = torch.randn((40, 16), device="cuda", requires_grad=True)
    torch.library.opcheck(torch.ops.dgfx.csr_spmm.default, (rp, cl, None, x, True, -1))
    ids = torch.from_numpy(rng.integers(0, 10, 50)).cuda()
    d = torch.randn((50, 8), device="cuda", requires_grad=True)
    torch.library.opcheck(torch.ops.dgfx.segment_sum.default, (d, ids, 10, True))
    lg = torch.randn((50, 2), device="cuda")
    ms = torch.randn((50, 2, 8), device="cuda")
    torch.library.opcheck(torch.ops.dgfx.segment_softmax.default, (lg, ms, ids, 10),
                          test_utils=("test_schema", "test_faketensor"))


@pytest.mark.parametrize("kind", ["gcn", "gin"])
def test_propagation_matrices(ops, kind):
    from distributed_graph_flow_b200 import aggregation

    rng = np.random.default_rng(11)
    n, m = 120, 700
    src = rng.integers(0, n, m)
    dst = rng.integers(0, n, m)
    src[:5] = dst[:5]  # self loops
    src[5:10], dst[5:10] = src[10:15], dst[10:15]  # duplicates
    eps = 0.25
    s_t, d_t = torch.from_numpy(src).cuda(), torch.from_numpy(dst).cuda()
    if kind == "gcn":
        rp, cl, vl = aggregation.gcn_matrix(s_t, d_t, n)
        dense = O.propagation_matrix(src, dst, n, 1.0, True)
    else:
        rp, cl, vl = aggregation.gin_matrix(s_t, d_t, n, eps)
        dense = O.propagation_matrix(src, dst, n, 1.0 + eps, False)
    rp_h, cl_h, vl_h = rp.cpu().numpy(), cl.cpu().numpy(), vl.cpu().numpy().astype(np.float64)
    assert rp_h[-1] == 2 * m + n
    got = np.zeros((n, n))
    rows = np.repeat(np.arange(n), np.diff(rp_h))
    np.add.at(got, (rows, cl_h), vl_h)
    np.testing.assert_allclose(got, dense, rtol=1e-6, atol=1e-7)
    x = torch.randn((n, 32), device="cuda", requires_grad=True)
    prop = ops.gcn_propagate if kind == "gcn" else ops.gin_propagate
    y = prop(x, (rp, cl, vl))
    g = torch.randn_like(y)
    y.backward(g)
    xh = x.detach().cpu().numpy().astype(np.float64)
    _close(y.detach().cpu().numpy(), dense @ xh, np.abs(dense) @ np.abs(xh), 1e-5)
    gh = g.cpu().numpy().astype(np.float64)
    _close(x.grad.cpu().numpy(), dense.T @ gh, np.abs(dense.T) @ np.abs(gh), 1e-5)


def test_batch_mean_aggregate(cuda):
    """Mean aggregation over a FIRST-mode merged batch of the temporal graph
    (fp32 features) against the float64 restatement over the oracle's
    batch."""
    from distributed_graph_flow_b200 import _native, aggregation, synth
    from distributed_graph_flow_b200.sampling import _in_memory_sampler_ext as ext
    from distributed_graph_flow_b200.sampling import config as cfg

    dev = torch.device("cuda", 0)
    spec = synth.GraphSpec(5000, 60_000, 2.1, 2000, seed=1, ts_range=(0, 50))
    index, _, _ = synth.build_graph(spec, dev)
    plan = cfg.explicit_plan("v", "e", [10, 5])
    s = ext.create_device_sampler(plan, ["v"], [spec.num_nodes], ["e"], [index], [None], _native.MODE_FIRST, seed=3,
                                  has_temporal=True)
    seeds = synth.uniform_int(256, 0, spec.num_nodes, 21, 9, dev)
    sts = synth.uniform_int(256, 0, 55, 22, 9, dev)
    batch = s.sample_merged(seeds, sts)
    table = synth.normal_features(0, spec.num_nodes, 64, 9, torch.float32, dev)
    feats = aggregation.gather_rows(table, batch.node_ids)
    agg = aggregation.batch_mean_aggregate(batch, feats)
    nodes, off, edges, eoff = ext.batch_to_host(batch)
    n = int(off[-1])
    fh = table.cpu().numpy()[nodes]
    exp = O.batch_mean_aggregate(off, eoff, edges, fh)
    samp = np.repeat(np.arange(256), np.diff(eoff))
    mag = O.batch_mean_aggregate(off, eoff, edges, np.abs(fh))
    _close(agg[:n].cpu().numpy(), exp, mag, 1e-5)
    assert samp.size == edges.shape[1]
    # The batch CSR + general SpMM route gives the same values.
    rp, cl = aggregation.batch_csr(batch)
    agg2 = aggregation.csr_spmm(rp, cl, feats, normalize=True)
    _close(agg2[:n].cpu().numpy(), exp, mag, 1e-5)
    assert torch.count_nonzero(agg2[n:]) == 0
    # Rows of several 32-chunk groups (200 fp32 = 50 chunks) and bf16 rows.
    for dim, dt, tol in ((200, torch.float32, 1e-5), (256, torch.bfloat16, 1e-2)):
        tab = synth.normal_features(0, spec.num_nodes, dim, 10, dt, dev)
        got = aggregation.batch_mean_aggregate(batch, aggregation.gather_rows(tab, batch.node_ids))
        th = tab.float().cpu().numpy().astype(np.float64)[nodes]
        _close(got[:n].float().cpu().numpy(), O.batch_mean_aggregate(off, eoff, edges, th),
               O.batch_mean_aggregate(off, eoff, edges, np.abs(th)), tol)
