"""Heterogeneous temporal sampling on a device-built graph (the
four-node-set / four-edge-type workload at reduced size).

Edge times come from propagate_timestamp_to_edges' kernel (node set A's
creation times; the B->C edge type has none and samples without a cutoff).
The plan walks every edge type in both directions from A seeds with per-hop
widths [15, 10]. FIRST mode (the reference's debug_sampling, oldest-first
under a cutoff) must equal the oracle bit for bit; random mode must respect
the cutoff, draw only existing edges and take min(k, valid) neighbours.
"""

import numpy as np
import pytest
import torch

from helpers import assert_sample_equal

pytestmark = pytest.mark.gpu


def _setup(scale=0.002):
    from distributed_graph_flow_b200 import synth

    dev = torch.device("cuda", 0)
    spec = synth.scaled_hetero(synth.HETERO_TEMPORAL, scale)
    g = synth.build_hetero_graph(spec, dev)
    plan = synth.hetero_plan(spec, "A", [15, 10])
    return dev, spec, g, plan


def _oracle(g, plan, mode, seed=5):
    from oracle import oracle as O

    fwd, bwd = {}, {}
    for name, f, b in zip(g.edgeset_names, g.fwd, g.bwd):
        fwd[name] = (f.rowptr.cpu().numpy(), f.col.cpu().numpy(), None if f.ts is None else f.ts.cpu().numpy())
        bwd[name] = (b.rowptr.cpu().numpy(), b.col.cpu().numpy(), None if b.ts is None else b.ts.cpu().numpy())
    return O.OracleSampler.from_csr(g.num_nodes, g.nodeset_names, g.edgeset_names, fwd, plan, mode=mode, seed=seed,
                                    temporal=True, csr_bwd=bwd)


def _device(g, plan, mode):
    from distributed_graph_flow_b200.sampling import _in_memory_sampler_ext as ext

    return ext.create_device_sampler(plan, g.nodeset_names, g.num_nodes, g.edgeset_names, g.fwd, g.bwd, mode, seed=5,
                                     has_temporal=True)


def test_edge_times_propagated(cuda):
    """Edge types touching A carry max(endpoint creation time) = A's time;
    B->C has none."""
    dev, spec, g, plan = _setup()
    a_ts = g.node_ts["A"]
    for name, (src, dst, ts) in g.edges.items():
        s_ns, t_ns, _ = spec.edge_sets[name]
        if "A" not in (s_ns, t_ns):
            assert ts is None
            continue
        if s_ns == "A" and t_ns == "A":
            exp = torch.maximum(a_ts[src], a_ts[dst])
        else:
            exp = a_ts[src] if s_ns == "A" else a_ts[dst]
        assert torch.equal(ts, exp), name


def test_first_mode_matches_oracle(cuda):
    from distributed_graph_flow_b200 import _native
    from distributed_graph_flow_b200.sampling import _in_memory_sampler_ext as ext
    from oracle import oracle as O

    dev, spec, g, plan = _setup()
    rng = np.random.default_rng(3)
    n_a = g.num_nodes[g.nodeset_names.index("A")]
    seeds = rng.integers(0, n_a, 300)
    a_ts = g.node_ts["A"].cpu().numpy()
    sts = a_ts[seeds] - rng.integers(0, 3, len(seeds))  # cutoffs at and below the seed's own year
    cc = _device(g, plan, _native.MODE_FIRST)
    merged = cc.sample_merged(torch.from_numpy(seeds).to(dev), torch.from_numpy(sts).to(dev))
    cc.check()
    got = ext.export_graphs(merged)
    exp = _oracle(g, plan, O.MODE_FIRST).sample(seeds, sts)
    for i, (gr, (en, ee)) in enumerate(zip(got, exp)):
        nodes = {n: gr.node_sets[n].features["#idx"] for n in gr.node_sets}
        edges = {n: gr.edge_sets[n].adjacency for n in gr.edge_sets}
        assert_sample_equal(nodes, edges, en, ee, f"seed #{i} ({seeds[i]})")


def test_random_mode_properties(cuda):
    """Every sampled edge exists in the graph, respects the seed's cutoff on
    temporal edge types, and each expanded node takes min(k, valid) picks."""
    from distributed_graph_flow_b200 import _native
    from distributed_graph_flow_b200.sampling import _in_memory_sampler_ext as ext

    dev, spec, g, plan = _setup()
    rng = np.random.default_rng(4)
    n_a = g.num_nodes[g.nodeset_names.index("A")]
    seeds = rng.integers(0, n_a, 400)
    sts = g.node_ts["A"].cpu().numpy()[seeds]
    cc = _device(g, plan, _native.MODE_RANDOM)
    merged = cc.sample_merged(torch.from_numpy(seeds).to(dev), torch.from_numpy(sts).to(dev))
    cc.check()
    graphs = ext.export_graphs(merged)
    edge_ts = {}
    for name, (src, dst, ts) in g.edges.items():
        s, d = src.cpu().numpy(), dst.cpu().numpy()
        t = None if ts is None else ts.cpu().numpy()
        edge_ts[name] = {}
        for j in range(len(s)):
            key = (int(s[j]), int(d[j]))
            tj = -1 if t is None else int(t[j])
            edge_ts[name][key] = min(edge_ts[name].get(key, tj), tj)
    for i, gr in enumerate(graphs):
        for name in g.edgeset_names:
            s_ns, t_ns, _ = spec.edge_sets[name]
            adj = gr.edge_sets[name].adjacency
            src_ids = gr.node_sets[s_ns].features["#idx"]
            dst_ids = gr.node_sets[t_ns].features["#idx"]
            for a, b in adj.T:
                key = (int(src_ids[a]), int(dst_ids[b]))
                assert key in edge_ts[name], f"seed #{i}: {name} edge {key} does not exist"
                if g.edges[name][2] is not None:
                    assert edge_ts[name][key] <= sts[i], f"seed #{i}: {name} edge {key} after the cutoff"
