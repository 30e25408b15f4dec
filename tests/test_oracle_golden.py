"""Pin the CPU oracle and the input generators against vectors produced by the reference's own code
(tests/golden/make_golden.py imports moelab.problem / torch_backend / torch_loop from the reference)."""
import hashlib
import json
import os

import numpy as np
import pytest
import torch

import oracle
from moelab_b200.problem import make_problem, make_routing
from moelab_b200.shapes import MoEShape

GOLD = os.path.join(os.path.dirname(__file__), "golden")
META = json.load(open(os.path.join(GOLD, "reference_vectors.json")))
VEC = np.load(os.path.join(GOLD, "reference_vectors.npz"))


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.mark.parametrize("case", META["routing"], ids=lambda c: f"{c['mode']}-T{c['T']}-E{c['E']}")
def test_make_routing_bit_exact(case):
    idx, w = make_routing(case["T"], case["E"], case["k"], case["mode"], np.random.default_rng(case["seed"]))
    np.testing.assert_array_equal(idx, VEC[f"routing{case['id']}_idx"])
    np.testing.assert_array_equal(w, VEC[f"routing{case['id']}_wts"])


def _problem(c):
    return make_problem(MoEShape("g", c["d"], c["f"], c["E"], c["k"]), c["T"], c["mode"], c["seed"])


@pytest.mark.parametrize("case", META["problems"], ids=lambda c: f"p{c['id']}-{c['mode']}-T{c['T']}")
def test_make_problem_bit_exact(case):
    p = _problem(case)
    for n, h in case["sha256"].items():
        assert sha(p[n]) == h, n
    np.testing.assert_array_equal(p["idx"], VEC[f"prob{case['id']}_idx"])
    np.testing.assert_array_equal(p["wts"], VEC[f"prob{case['id']}_wts"])


@pytest.mark.parametrize("case", META["problems"], ids=lambda c: f"p{c['id']}-{c['mode']}-T{c['T']}")
def test_oracle_references_match_reference_outputs(case):
    p = _problem(case)
    y64, y32 = VEC[f"prob{case['id']}_y64"], VEC[f"prob{case['id']}_y32"]
    # fp64 restatement (problem.py:67-85)
    assert oracle.error_metrics(oracle.reference_fp64(p), y64)["rel_fro"] < 1e-6
    # fp32 torch restatement (torch_backend.py:57-67)
    t = {n: torch.from_numpy(p[n]) for n in ("x", "w_gate", "w_up", "w_down", "wts")}
    yr = oracle.reference_fp32(t["w_gate"], t["w_up"], t["w_down"], t["x"], torch.from_numpy(p["idx"]), t["wts"])
    assert oracle.error_metrics(yr.numpy(), y32)["rel_fro"] < 1e-5
    # the C oracle (fp64 accumulation) against the reference's fp64 truth
    yc = oracle.moe_forward(p["x"], p["w_gate"], p["w_up"], p["w_down"], p["idx"], p["wts"])
    assert oracle.error_metrics(yc, y64)["rel_fro"] < 1e-6


@pytest.mark.parametrize("case", META["problems"], ids=lambda c: f"p{c['id']}-{c['mode']}-T{c['T']}")
def test_torch_loop_port_matches_reference_torch_loop(case):
    p = _problem(case)
    s = {k: torch.from_numpy(p[n]).to(torch.bfloat16) for k, n in (("wg", "w_gate"), ("wu", "w_up"), ("wd", "w_down"))}
    y = oracle.torch_loop_run(s, torch.from_numpy(p["x"]).to(torch.bfloat16), torch.from_numpy(p["idx"]),
                              torch.from_numpy(p["wts"]))
    np.testing.assert_array_equal(y.float().numpy(), VEC[f"prob{case['id']}_yloop"])


def test_trace_windows_reproduce_reference_draws():
    """Trace routing (moelab/problem.py:38-50): the windows and weights the reference's own make_inputs drew for
    every stored (seed, T) are reproduced bit for bit from the committed fixture."""
    import os
    from moelab_b200.problem import TRACE_FIXTURE, make_inputs
    z = np.load(TRACE_FIXTURE)
    n = 0
    for name in z.files:
        if not name.startswith("idx_"):
            continue
        _, seed, T = name.split("_")
        x, idx, wts = make_inputs(2048, 128, 8, int(T), "trace", int(seed))
        np.testing.assert_array_equal(idx, z[name])
        np.testing.assert_array_equal(wts, z[f"wts_{seed}_{T}"])
        n += 1
    assert n == 64 and os.path.getsize(TRACE_FIXTURE) < 200_000
