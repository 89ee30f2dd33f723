"""The allocation-free sampling entry point, called through the C ABI.

Some callers cannot allocate device memory when they sample (their framework
owns the whole memory pool, or they run where allocation is not allowed), so
dgfx_sampler_sample_noalloc takes its scratch from a fixed device array
inside the library instead of a caller workspace. Its output must equal the
workspace entry point's output for the same call index, exactly (the output
is integer ids), on two calls in a row (the second call reuses the scratch
the first one left behind). This file sorts last so that a failure here
cannot hide other tests' results.
"""

import ctypes

import numpy as np
import pytest

from helpers import random_hetero_graph

pytestmark = pytest.mark.gpu


def _alloc_out(torch, lib, handle, B, NS, ES):
    from distributed_graph_flow_b200 import _native

    mn, me = ctypes.c_int64(), ctypes.c_int64()
    _native.check(lib.dgfx_sampler_output_capacity(handle, B, ctypes.byref(mn), ctypes.byref(me)))
    bufs = {
        "node_ids": torch.full((max(1, mn.value),), -7, dtype=torch.int64, device="cuda"),
        "node_offsets": torch.full((NS * B + 1,), -7, dtype=torch.int64, device="cuda"),
        "edge_src": torch.full((max(1, me.value),), -7, dtype=torch.int64, device="cuda"),
        "edge_dst": torch.full((max(1, me.value),), -7, dtype=torch.int64, device="cuda"),
        "edge_offsets": torch.full((ES * B + 1,), -7, dtype=torch.int64, device="cuda"),
    }
    out = _native.SampleOut(*[_native.ptr(bufs[k]) for k in ("node_ids", "node_offsets", "edge_src", "edge_dst",
                                                               "edge_offsets")])
    return bufs, out


def _host(bufs):
    n = int(bufs["node_offsets"][-1].item())
    m = int(bufs["edge_offsets"][-1].item())
    return (bufs["node_offsets"].cpu().numpy(), bufs["node_ids"][:n].cpu().numpy(),
            bufs["edge_offsets"].cpu().numpy(), bufs["edge_src"][:m].cpu().numpy(),
            bufs["edge_dst"][:m].cpu().numpy())


def test_noalloc_matches_workspace_entry_point(cuda):
    torch = cuda
    from distributed_graph_flow_b200 import _native
    from distributed_graph_flow_b200 import sampling

    graph, schema = random_hetero_graph(11, temporal=True)
    plan = sampling.simple_sampling_config_to_sampling_plan(
        sampling.SimpleSamplingConfig(seed_nodeset="a", num_hops=2, hop_width=3, temporal_sampling=True), schema
    )
    s = sampling.create_sampler(graph, plan, schema, batch_size=256, seed=17)
    cc = s._cc_sampler
    lib = _native.lib()
    rng = np.random.default_rng(5)
    B = 256
    seeds = torch.from_numpy(rng.integers(0, 40, B)).cuda()
    ts = torch.from_numpy(rng.integers(0, 55, B)).cuda()
    NS, ES = len(cc._nodeset_names), len(cc._edgeset_names)
    stream = _native.stream_handle()

    need = ctypes.c_size_t()
    _native.check(lib.dgfx_sampler_workspace_size(cc._handle, B, ctypes.byref(need)))
    ws = torch.empty(need.value, dtype=torch.uint8, device="cuda")
    ref_bufs, ref_out = _alloc_out(torch, lib, cc._handle, B, NS, ES)
    _native.check(lib.dgfx_sampler_sample(cc._handle, _native.ptr(seeds), _native.ptr(ts), None, B, 3,
                                          ctypes.byref(ref_out), _native.ptr(ws), need.value, stream))
    _native.check(lib.dgfx_sampler_check(cc._handle, stream))
    expected = _host(ref_bufs)
    assert len(expected[1]) > B  # the samples are not trivial

    for _ in range(2):
        bufs, out = _alloc_out(torch, lib, cc._handle, B, NS, ES)
        _native.check(lib.dgfx_sampler_sample_noalloc(cc._handle, _native.ptr(seeds), _native.ptr(ts), None, B, 3,
                                                      ctypes.byref(out), stream))
        _native.check(lib.dgfx_sampler_check(cc._handle, stream))
        got = _host(bufs)
        for a, b in zip(got, expected):
            np.testing.assert_array_equal(a, b)


def test_noalloc_rejects_oversized_batches(cuda):
    from distributed_graph_flow_b200 import _native
    from distributed_graph_flow_b200 import sampling

    graph, schema = random_hetero_graph(12, temporal=False)
    plan = sampling.simple_sampling_config_to_sampling_plan(
        sampling.SimpleSamplingConfig(seed_nodeset="a", num_hops=2, hop_width=3), schema
    )
    s = sampling.create_sampler(graph, plan, schema, batch_size=8, seed=1)
    cc = s._cc_sampler
    lib = _native.lib()
    B = (64 << 20) // (12 * cc.tree_size) + 1  # scratch need grows ~12 bytes per tree position per seed
    out = _native.SampleOut()
    status = lib.dgfx_sampler_sample_noalloc(cc._handle, None, None, None, B, 0, ctypes.byref(out),
                                             _native.stream_handle())
    assert status == _native.ERR_INVALID_ARGUMENT
    assert "more than the fixed" in _native.last_error()
