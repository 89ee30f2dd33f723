"""Aggregation kernels vs the float64 oracle.

Tolerances (the stated bar): fp32 results within 1e-5 relative, bf16 within
1e-2 relative, both measured against the row's magnitude
sum_j |val_j * x_j| so that cancellation does not inflate the error."""

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

FP32_RTOL = 1e-5
BF16_RTOL = 1e-2


@pytest.fixture(scope="module")
def agg(cuda):
    from distributed_graph_flow_b200 import aggregation

    return aggregation


def _powerlaw_csr(rng, rows, cols, mean_deg, max_deg):
    deg = np.minimum((rng.pareto(1.0, rows) * mean_deg / 3).astype(np.int64), max_deg)
    deg[rng.integers(0, rows, max(1, rows // 50))] = 0  # some empty rows
    deg[0] = max_deg  # at least one split row
    rowptr = np.concatenate([[0], np.cumsum(deg)])
    col = rng.integers(0, cols, rowptr[-1]).astype(np.int32)
    return rowptr.astype(np.int64), col


def _check(y, ref, bound, rtol):
    err = np.abs(y.astype(np.float64) - ref)
    lim = rtol * (bound + 1e-30)
    bad = err > lim
    assert not bad.any(), f"max err {err.max():.3e} at {np.argwhere(bad)[:3]}, lim {lim[bad][:3]}"


@pytest.mark.parametrize("feat", [8, 64, 128, 256, 520])
@pytest.mark.parametrize("normalize", [False, True])
@pytest.mark.parametrize("with_val", [False, True])
def test_spmm_fp32(agg, cuda, feat, normalize, with_val):
    torch = cuda
    rng = np.random.default_rng(feat)
    rowptr, col = _powerlaw_csr(rng, 3000, 2000, 12, 1500)
    x = rng.standard_normal((2000, feat)).astype(np.float32)
    val = rng.standard_normal(len(col)).astype(np.float32) if with_val else None
    d = lambda a: None if a is None else torch.from_numpy(a).cuda()
    y = agg.csr_spmm(d(rowptr), d(col), d(x), val=d(val), normalize=normalize).cpu().numpy()
    ref = O.csr_spmm(rowptr, col, x, val, normalize)
    bound = O.csr_spmm(rowptr, col, np.abs(x), None if val is None else np.abs(val), normalize)
    _check(y, ref, bound, FP32_RTOL)


@pytest.mark.parametrize("out_bf16", [False, True])
def test_spmm_bf16(agg, cuda, out_bf16):
    torch = cuda
    rng = np.random.default_rng(1)
    rowptr, col = _powerlaw_csr(rng, 5000, 4000, 20, 3000)
    x = torch.randn(4000, 256, generator=torch.Generator().manual_seed(0)).to(torch.bfloat16)
    y = agg.csr_spmm(torch.from_numpy(rowptr).cuda(), torch.from_numpy(col).cuda(), x.cuda(), normalize=True,
                     out_dtype=torch.bfloat16 if out_bf16 else torch.float32)
    xf = x.float().numpy()
    ref = O.csr_spmm(rowptr, col, xf, None, True)
    bound = O.csr_spmm(rowptr, col, np.abs(xf), None, True)
    _check(y.float().cpu().numpy(), ref, bound, BF16_RTOL if out_bf16 else FP32_RTOL)


def test_spmm_deterministic(agg, cuda):
    torch = cuda
    rng = np.random.default_rng(2)
    rowptr, col = _powerlaw_csr(rng, 2000, 2000, 30, 5000)
    x = torch.from_numpy(rng.standard_normal((2000, 256)).astype(np.float32)).cuda()
    r, c = torch.from_numpy(rowptr).cuda(), torch.from_numpy(col).cuda()
    a = agg.csr_spmm(r, c, x)
    b = agg.csr_spmm(r, c, x)
    assert torch.equal(a, b)


@pytest.mark.parametrize("sorted_ids", [False, True])
@pytest.mark.parametrize("mean", [False, True])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_segment_sum(agg, cuda, sorted_ids, mean, dtype):
    torch = cuda
    rng = np.random.default_rng(3)
    n, F, nseg = 20000, 64, 777
    ids = rng.integers(-5, nseg + 5, n)  # out-of-range ids are dropped
    if sorted_ids:
        ids = np.sort(ids)
    data = rng.standard_normal((n, F)).astype(np.float32)
    td = torch.from_numpy(data).cuda()
    if dtype == "bf16":
        td = td.to(torch.bfloat16)
        data = td.float().cpu().numpy()
    out = agg.segment_sum(td, torch.from_numpy(ids).cuda(), nseg, mean=mean, indices_are_sorted=sorted_ids,
                          out_dtype=torch.float32)
    ref = O.segment_sum(data, ids, nseg, mean)
    bound = O.segment_sum(np.abs(data), ids, nseg, mean)
    _check(out.cpu().numpy(), ref, bound, FP32_RTOL)


def test_gather_rows(agg, cuda):
    torch = cuda
    table = torch.randn(1000, 128, device="cuda")
    ids = torch.tensor([5, 0, 999, 5, -1, 1000], device="cuda")
    out = agg.gather_rows(table, ids)
    assert torch.equal(out[:4], table[torch.tensor([5, 0, 999, 5], device="cuda")])
    assert torch.count_nonzero(out[4:]) == 0
    tb = torch.randn(50, 128, device="cuda").to(torch.bfloat16)
    assert torch.equal(agg.gather_rows(tb, torch.arange(49, -1, -1, device="cuda")), tb.flip(0))


# ---------------------------------------------------------------------------
# Segment softmax (graph attention), hetero_graph_attention_network.py:242-263
# ---------------------------------------------------------------------------
def _softmax_reference(logits, messages, ids, nseg):
    """The reference's sequence in torch fp32: segment_max, exp, segment_sum,
    divide (+1e-9), weighted segment_sum. Items outside [0, nseg) dropped."""
    keep = (ids >= 0) & (ids < nseg)
    l, m, t = logits[keep].double(), messages[keep].double(), ids[keep]
    H = logits.shape[1]
    mx = torch.full((nseg, H), -float("inf"), dtype=torch.float64, device=l.device)
    mx = mx.scatter_reduce(0, t[:, None].expand(-1, H), l, reduce="amax")
    ex = torch.exp(l - mx[t])
    den = torch.zeros((nseg, H), dtype=torch.float64, device=l.device).index_add_(0, t, ex)
    w = ex / (den[t] + 1e-9)
    out = torch.zeros((nseg,) + tuple(messages.shape[1:]), dtype=torch.float64, device=l.device)
    return out.index_add_(0, t, w[..., None] * m)


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
@pytest.mark.parametrize("sorted_ids", [False, True])
@pytest.mark.parametrize("H,D", [(1, 8), (4, 32), (8, 32), (2, 64)])
def test_segment_softmax(cuda, dtype, sorted_ids, H, D):
    from distributed_graph_flow_b200 import aggregation

    dev = torch.device("cuda", 0)
    g = torch.Generator(device="cuda").manual_seed(H * 100 + D)
    E, nseg = 50_000, 3_001
    dt = getattr(torch, dtype)
    # Skewed segment sizes, some empty segments, a few ids out of range.
    ids = (torch.rand(E, generator=g, device=dev) ** 3 * (nseg + 20)).long() - 10
    if sorted_ids:
        ids = torch.sort(ids).values
    logits = torch.randn((E, H), generator=g, device=dev) * 4
    msgs = torch.randn((E, H, D), generator=g, device=dev).to(dt)
    got = aggregation.segment_softmax(logits, msgs, ids, nseg, indices_are_sorted=sorted_ids, out_dtype=torch.float32)
    ref = _softmax_reference(logits, msgs.float(), ids, nseg)
    # fp32 output: 1e-5 of the row scale (the bf16 messages are exact in the
    # reference, which reads the same rounded values); bf16 output: 1e-2.
    err = (got.double() - ref).abs()
    scale = ref.abs().amax(dim=-1, keepdim=True).clamp(min=1e-3)
    assert float((err / scale).max()) <= 1e-5, float((err / scale).max())
    got16 = aggregation.segment_softmax(logits, msgs, ids, nseg, indices_are_sorted=sorted_ids)
    assert got16.dtype == dt
    assert float(((got16.double() - ref).abs() / scale).max()) <= (1e-5 if dtype == "float32" else 1e-2)


@pytest.mark.parametrize("sorted_ids", [False, True])
@pytest.mark.parametrize("H,D", [(8, 32), (32, 8), (3, 8)])
def test_segment_softmax_masked_logits(cuda, sorted_ids, H, D):
    """Masked attention: about a third of the logits are -inf. Segment heads
    with a finite logit match the reference sequence; a segment head whose
    logits are all -inf (NaN in the reference's exp(-inf - -inf)) gives 0."""
    from distributed_graph_flow_b200 import aggregation

    dev = torch.device("cuda", 0)
    g = torch.Generator(device="cuda").manual_seed(77 + H)
    E, nseg = 40_000, 2_000
    ids = (torch.rand(E, generator=g, device=dev) ** 3 * nseg).long()
    if sorted_ids:
        ids = torch.sort(ids).values
    logits = torch.randn((E, H), generator=g, device=dev) * 3
    logits[torch.rand((E, H), generator=g, device=dev) < 0.35] = -float("inf")
    msgs = torch.randn((E, H, D), generator=g, device=dev).to(torch.bfloat16)
    got = aggregation.segment_softmax(logits, msgs, ids, nseg, indices_are_sorted=sorted_ids, out_dtype=torch.float32)
    ref = _softmax_reference(logits, msgs.float(), ids, nseg)
    assert bool(torch.isfinite(got).all())
    finite = torch.isfinite(ref).all(dim=-1)
    assert int((~finite).sum()) > 0  # some segment heads are fully masked
    assert torch.count_nonzero(got[~finite]) == 0
    err = (got.double() - ref).abs()[finite]
    scale = ref.abs().amax(dim=-1)[finite].clamp(min=1e-3)
    assert float((err.amax(dim=-1) / scale).max()) <= 1e-5


def test_segment_softmax_deterministic_and_empty(cuda):
    from distributed_graph_flow_b200 import aggregation

    dev = torch.device("cuda", 0)
    ids = torch.tensor([5, 2, 5, 2, 5], device=dev)
    logits = torch.tensor([[1.0], [2.0], [3.0], [-1.0], [0.5]], device=dev)
    msgs = torch.arange(5 * 8, dtype=torch.float32, device=dev).view(5, 1, 8)
    a = aggregation.segment_softmax(logits, msgs, ids, 7)
    b = aggregation.segment_softmax(logits, msgs, ids, 7)
    assert torch.equal(a, b)
    assert torch.count_nonzero(a[[0, 1, 3, 4, 6]]) == 0
    ref = _softmax_reference(logits, msgs, ids, 7)
    assert torch.allclose(a.double(), ref, rtol=1e-6, atol=1e-6)
    empty = aggregation.segment_softmax(logits[:0], msgs[:0], ids[:0], 3)
    assert torch.count_nonzero(empty) == 0
