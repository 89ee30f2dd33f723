"""The device generators (csrc/synth.cu) against their host restatement
(oracle/synth_cpu.h): graphs and uniform integers bit for bit, N(0, 1)
features to the last bit of fp32 / bf16 up to the rounding of the
transcendental functions."""

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

SPECS = [(5000, 5000, 60_000, 2.0, 700, 4), (30_000, 30_000, 400_000, 2.1, 20_000, 1),
         (2000, 777, 25_000, 1.9, 5000, 11), (1, 1, 0, 2.0, 1, 3)]


@pytest.mark.parametrize("spec", SPECS, ids=[f"{s[0]}x{s[1]}_{s[2]}" for s in SPECS])
def test_graph_bit_equal(cuda, spec):
    from distributed_graph_flow_b200 import synth

    n_src, n_dst, E, alpha, max_deg, seed = spec
    torch = cuda
    import ctypes

    from distributed_graph_flow_b200 import _native

    lib = _native.lib()
    need = ctypes.c_size_t()
    _native.check(lib.dgfx_synth_graph_workspace_size(n_src, max_deg, ctypes.byref(need)))
    ws = torch.empty(need.value, dtype=torch.uint8, device="cuda")
    rp = torch.empty(n_src + 1, dtype=torch.int64, device="cuda")
    src = torch.empty(max(E, 1), dtype=torch.int64, device="cuda")
    dst = torch.empty(max(E, 1), dtype=torch.int64, device="cuda")
    _native.check(lib.dgfx_synth_bipartite(n_src, n_dst, E, alpha, max_deg, seed, _native.ptr(rp), _native.ptr(src),
                                           _native.ptr(dst), _native.ptr(ws), need.value, _native.stream_handle()))
    torch.cuda.synchronize()
    h_rp, h_src, h_dst = O.synth_graph(n_src, n_dst, E, alpha, max_deg, seed)
    np.testing.assert_array_equal(rp.cpu().numpy(), h_rp)
    np.testing.assert_array_equal(src[:E].cpu().numpy(), h_src)
    np.testing.assert_array_equal(dst[:E].cpu().numpy(), h_dst)
    if n_src == n_dst and E > 0:
        spec_obj = synth.GraphSpec(n_src, E, alpha, max_deg, seed=seed)
        rp2, s2, d2 = synth.rowptr_and_edges(spec_obj, "cuda")
        np.testing.assert_array_equal(rp2.cpu().numpy(), h_rp)
        np.testing.assert_array_equal(d2.cpu().numpy(), h_dst)


def test_uniform_int_bit_equal(cuda):
    from distributed_graph_flow_b200 import synth

    for n, lo, hi, seed, stream in [(100_000, 0, 111_059_956, 77, 5), (5000, 2010, 2020, 3, 31), (7, -4, 9, 0, 0)]:
        d = synth.uniform_int(n, lo, hi, seed, stream, "cuda").cpu().numpy()
        np.testing.assert_array_equal(d, O.synth_uniform_int(n, lo, hi, seed, stream))


@pytest.mark.parametrize("bf16", [False, True])
def test_normal_features_match(cuda, bf16):
    from distributed_graph_flow_b200 import synth

    torch = cuda
    begin, count, dim, seed = 12_345, 4000, 129, 104
    d = synth.normal_features(begin, count, dim, seed, torch.bfloat16 if bf16 else torch.float32, "cuda")
    h = O.synth_normal_features(begin, count, dim, seed, bf16=bf16)
    if bf16:
        dv = d.cpu().view(torch.int16).numpy().view(np.uint16)
        assert np.mean(dv == h) > 0.9999
        df = (dv.astype(np.uint32) << 16).view(np.float32)
        hf = (h.astype(np.uint32) << 16).view(np.float32)
        np.testing.assert_allclose(df, hf, rtol=2.0 ** -7, atol=0)
    else:
        dv = d.cpu().numpy()
        assert np.mean(dv == h) > 0.999
        np.testing.assert_allclose(dv, h, rtol=1e-6, atol=1e-7)
