"""Generates tests/golden/ref_vectors.npz from the reference's own compiled
sampler code (oracle/_ref/libdgf_ref.so: dgf/src/sampling/in_memory_sampler.cc
built unmodified, driven by the restated per-seed driver).

Run from the repository root after ``make -C oracle ref``:
    python tests/golden/make_golden.py
The vectors pin the oracle's restatement where the reference sources are not
available (e.g. on a GPU box).
"""

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

from oracle import oracle as O  # noqa: E402

OUT = HERE / "ref_vectors.npz"


def _graph(seed, temporal):
    from helpers import random_hetero_graph

    return random_hetero_graph(seed, temporal=temporal)


def cases():
    out = []
    for seed in range(3):
        for temporal in (False, True):
            for debug in (False, True):
                for wr in (False, True):
                    key = f"s{seed}_t{int(temporal)}_d{int(debug)}_w{int(wr)}"
                    g, schema = _graph(seed, temporal)
                    seeds = np.random.default_rng(100 + seed).integers(0, 40, 64)
                    c = dict(key=key, seed=seed, temporal=temporal, debug=debug, wr=wr, seeds=seeds,
                             conf=dict(seed_nodeset="a", num_hops=2, hop_width=3, with_replacement=wr,
                                       temporal_sampling=temporal))
                    if temporal:
                        c["ts"] = np.random.default_rng(200 + seed).integers(0, 50, 64)
                    out.append(c)
    # Masking (non-temporal).
    for seed in range(2):
        g, _ = _graph(seed, False)
        m = g.edge_sets["ab"].adjacency.shape[1]
        masks = np.random.default_rng(300 + seed).integers(-1, m, 64)
        out.append(dict(key=f"mask{seed}", seed=seed, temporal=False, debug=seed == 1, wr=False,
                        seeds=np.random.default_rng(400 + seed).integers(0, 40, 64), masks=masks, mask_es="ab",
                        conf=dict(seed_nodeset="a", num_hops=2, hop_width=2)))
    return out


def make_sampler(case, ref):
    from distributed_graph_flow_b200.sampling import config as cfg

    g, schema = _graph(case["seed"], case["temporal"])
    plan = cfg.simple_sampling_config_to_sampling_plan(cfg.SimpleSamplingConfig(**case["conf"]), schema)
    return O.OracleSampler(g, plan, schema, debug_sampling=case["debug"], num_threads=3, seed=1234 + case["seed"],
                           edgeset_to_mask=case.get("mask_es"),
                           edgeset_timestamp_features=plan.edgeset_timestamp_features, ref=ref)


def index_cases():
    out = []
    for seed in range(3):
        for temporal in (False, True):
            for rev in (False, True):
                out.append(dict(key=f"idx{seed}_t{int(temporal)}_r{int(rev)}", seed=seed, temporal=temporal, rev=rev,
                                populate=not temporal))
    return out


def make_index(case, ref):
    g, _ = _graph(case["seed"], case["temporal"])
    es = g.edge_sets["ab"]
    ts = es.features.get("timestamp") if case["temporal"] else None
    return O.Index(es.adjacency, ts, case["rev"], 40, 25, populate_edge_idxs=case["populate"], ref=ref)


def main():
    if not O.available(ref=True):
        raise SystemExit("build oracle/_ref first: make -C oracle ref")
    data = {}
    for case in cases():
        s = make_sampler(case, ref=True)
        res = s.sample_raw(case["seeds"], case.get("ts"), case.get("masks"))
        for i, arr in enumerate(res):
            data[f"{case['key']}_{i}"] = arr
    for case in index_cases():
        arr = make_index(case, ref=True).arrays()
        for f, a in arr.items():
            data[f"{case['key']}_{f}"] = a
    np.savez_compressed(OUT, **data)
    print(f"wrote {OUT} ({len(data)} arrays)")


if __name__ == "__main__":
    main()
