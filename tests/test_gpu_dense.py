"""Tensor-core dense layer after aggregation (dgfx_dense_concat_bf16).

Numerics against a plain PyTorch fp32 reference of the same op:
relu(concat[x1, x2] @ w.T + b). Inputs are bf16, the kernel accumulates in
fp32 and rounds the output to bf16, so the tolerance is bf16's: 1e-2
relative to the output scale.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _case(m, k1, k2, n, bias=True, relu=True, seed=0):
    from distributed_graph_flow_b200 import aggregation

    g = torch.Generator(device="cuda").manual_seed(seed)
    dev = torch.device("cuda", 0)
    x1 = torch.randn((m, k1), generator=g, device=dev).to(torch.bfloat16)
    x2 = torch.randn((m, k2), generator=g, device=dev).to(torch.bfloat16) if k2 else None
    lim = (6.0 / (k1 + k2 + n)) ** 0.5
    w = ((torch.rand((n, k1 + k2), generator=g, device=dev) * 2 - 1) * lim).to(torch.bfloat16)
    b = torch.randn(n, generator=g, device=dev) * 0.1 if bias else None
    y = aggregation.dense_concat(x1, x2, w, b, relu=relu)
    aggregation.dense_check()
    xcat = x1.float() if x2 is None else torch.cat([x1.float(), x2.float()], dim=1)
    ref = xcat @ w.float().t()
    if b is not None:
        ref = ref + b
    if relu:
        ref = torch.relu(ref)
    scale = max(float(ref.abs().max()), 1e-3)
    err = float((y.float() - ref).abs().max())
    assert err <= 1e-2 * scale, f"m={m} k1={k1} k2={k2} n={n}: max abs err {err} vs scale {scale}"
    return y, ref


def test_small_single_tile(cuda):
    _case(128, 64, 0, 64)


@pytest.mark.parametrize("m,k1,k2,n", [
    (1, 64, 64, 64),
    (129, 128, 64, 128),
    (1000, 256, 256, 256),
    (4097, 256, 256, 256),
    (515, 64, 192, 512),
    (777, 320, 0, 192),
])
def test_shapes(cuda, m, k1, k2, n):
    _case(m, k1, k2, n, seed=m)


@pytest.mark.parametrize("bias,relu", [(False, False), (False, True), (True, False)])
def test_bias_relu_variants(cuda, bias, relu):
    _case(640, 128, 128, 256, bias=bias, relu=relu, seed=7)


def test_rejects_bad_shapes(cuda):
    from distributed_graph_flow_b200 import aggregation

    dev = torch.device("cuda", 0)
    x = torch.zeros((8, 96), dtype=torch.bfloat16, device=dev)
    w = torch.zeros((64, 96), dtype=torch.bfloat16, device=dev)
    with pytest.raises(ValueError, match="multiples of 64"):
        aggregation.dense_concat(x, None, w)
    with pytest.raises(ValueError, match="bfloat16"):
        aggregation.dense_concat(x.float(), None, w)


def test_sage_mean_layer(cuda):
    """GraphSAGE-mean: mean SpMM over in-neighbours, then the dense layer
    (the two launches of sage_mean_linear_relu) against fp32 torch."""
    from distributed_graph_flow_b200 import aggregation

    dev = torch.device("cuda", 0)
    g = torch.Generator(device="cuda").manual_seed(3)
    n_nodes, f, n_out, e = 3000, 128, 256, 40_000
    dst = torch.randint(0, n_nodes, (e,), generator=g, device=dev)
    src = torch.randint(0, n_nodes, (e,), generator=g, device=dev)
    order = torch.argsort(dst, stable=True)
    dst, src = dst[order], src[order]
    rowptr = torch.zeros(n_nodes + 1, dtype=torch.int64, device=dev)
    rowptr[1:] = torch.cumsum(torch.bincount(dst, minlength=n_nodes), 0)
    col = src.to(torch.int32)
    x = torch.randn((n_nodes, f), generator=g, device=dev).to(torch.bfloat16)
    lim = (6.0 / (2 * f + n_out)) ** 0.5
    w = ((torch.rand((n_out, 2 * f), generator=g, device=dev) * 2 - 1) * lim).to(torch.bfloat16)
    b = torch.zeros(n_out, device=dev)
    y = aggregation.sage_mean_linear_relu(rowptr, col, x, w, b)
    aggregation.dense_check()
    deg = torch.bincount(dst, minlength=n_nodes).clamp(min=1).float()
    agg = torch.zeros((n_nodes, f), device=dev).index_add_(0, dst, x.float()[src]) / deg[:, None]
    ref = torch.relu(torch.cat([x.float(), agg.to(torch.bfloat16).float()], 1) @ w.float().t() + b)
    scale = float(ref.abs().max())
    assert float((y.float() - ref).abs().max()) <= 1e-2 * scale
