"""Seeded synthetic MoE problems: the input generator side of moelab/problem.py.

Kernel contract (moelab/problem.py:3-10): y = moe(x, w_gate, w_up, w_down, idx, wts) with
x [T, d], w_gate/w_up [E, f, d], w_down [E, d, f] (out, in), idx [T, k] int32, wts [T, k] float,
y[t] = sum_j wts[t,j] * down_e(silu(gate_e x_t) * up_e x_t), e = idx[t,j].

make_routing / make_problem restate moelab/problem.py:15-64 call for call (same numpy Generator draws), so a
seed gives the reference's own inputs; tests/golden pins that. The "trace" mode (recorded Qwen3-30B-A3B routing,
moelab/problem.py:38-50) makes the reference's draws - a domain, a layer and a start token of the recorded traces,
then random combine weights - and takes the window from TraceWindows, the windows the reference drew for a set of
seeds (tests/golden/trace_qwen3.npz, written by tests/golden/make_trace.py from the reference's own code); a draw
outside that set raises KeyError.
"""
import os

import numpy as np

_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TRACE_FIXTURE = os.path.join(_ROOT, "tests", "golden", "trace_qwen3.npz")


class TraceWindows:
    """Recorded-routing windows by (domain, layer, start, T), and the domains' (layers, tokens) shapes."""

    def __init__(self, path=TRACE_FIXTURE):
        z = np.load(path)
        self.shapes = [tuple(int(v) for v in s) for s in z["shapes"]]
        self.win = {tuple(int(v) for v in key): z["windows"][i] for i, key in enumerate(z["keys"])}
        self.E, self.k = 128, int(z["windows"].shape[2])

    def draw(self, T, E, k, rng):
        """moelab/problem.py:38-50: domain, layer, start, then weights = rng.random((T, k)) normalised."""
        assert E == self.E and k == self.k, "trace recorded for E=128, k=8 (Qwen3) only"
        dom = int(rng.integers(len(self.shapes)))
        layer, start = int(rng.integers(self.shapes[dom][0])), int(rng.integers(self.shapes[dom][1] - T))
        key = (dom, layer, start, T)
        if key not in self.win:
            raise KeyError(f"trace window {key} is not in the fixture (seeds 0..15, T in 1/8/16/32 are)")
        idx = self.win[key][:T].astype(np.int32)
        w = rng.random((T, k)).astype(np.float32)
        return idx, w / w.sum(1, keepdims=True)


_TRACE = None


def make_routing(T, E, k, mode="uniform", rng=None, zipf_a=1.2, trace=None):
    global _TRACE
    rng = rng or np.random.default_rng(0)
    if mode == "trace":
        if trace is None:
            if _TRACE is None:
                _TRACE = TraceWindows()
            trace = _TRACE
        return trace.draw(T, E, k, rng)
    if mode == "uniform":
        logits = rng.standard_normal((T, E))
    elif mode == "zipf":  # skewed popularity over a seeded expert permutation
        pop = 1.0 / np.arange(1, E + 1) ** zipf_a
        logits = rng.standard_normal((T, E)) + np.log(pop)[rng.permutation(E)] * 2.0
    elif mode == "one_hot":  # every token to the same k experts (worst imbalance)
        logits = np.tile(np.arange(E, 0, -1, dtype=np.float64), (T, 1))
    elif mode == "round_robin":  # balanced: token t takes experts (t*k + j) % E
        idx = ((np.arange(T)[:, None] * k + np.arange(k)[None, :]) % E).astype(np.int32)
        w = rng.random((T, k)).astype(np.float32)
        return idx, (w / w.sum(1, keepdims=True)).astype(np.float32)
    else:
        raise ValueError(mode)
    idx = np.argsort(-logits, axis=1)[:, :k].astype(np.int32)
    top = np.take_along_axis(logits, idx, axis=1)
    w = np.exp(top - top.max(1, keepdims=True))
    w = (w / w.sum(1, keepdims=True)).astype(np.float32)
    return idx, w


def zipf_bias(E, s=1.1, seed=0, gain=2.0):
    """Per-expert router bias for the skewed DeepSeek-V2-Lite config: gain * log(Zipf(s) popularity), the
    popularity ranks assigned over a seeded expert permutation (the "zipf" routing mode above with s = 1.1), so
    a few experts are hot. float32 [E]."""
    rng = np.random.default_rng(seed)
    pop = 1.0 / np.arange(1, E + 1) ** s
    return (np.log(pop)[rng.permutation(E)] * gain).astype(np.float32)


def make_problem(shape, T, routing="uniform", seed=0):
    rng = np.random.default_rng(seed)
    d, f, E, k = shape.d, shape.f, shape.E, shape.k
    s_in, s_hid = 1.0 / np.sqrt(d), 1.0 / np.sqrt(f)
    p = {
        "x": rng.standard_normal((T, d)).astype(np.float32),
        "w_gate": (rng.standard_normal((E, f, d)) * s_in).astype(np.float32),
        "w_up": (rng.standard_normal((E, f, d)) * s_in).astype(np.float32),
        "w_down": (rng.standard_normal((E, d, f)) * s_hid).astype(np.float32),
    }
    p["idx"], p["wts"] = make_routing(T, E, k, routing, rng)
    return p


def error_metrics(y, y_ref):
    """moelab/problem.py:88-98, plus max_rowrel = max |err| / row max |ref|."""
    y = np.asarray(y, dtype=np.float64)
    r = np.asarray(y_ref, dtype=np.float64)
    diff = y - r
    nr = np.linalg.norm(r) + 1e-30
    rowmax = np.abs(r).max(axis=-1, keepdims=True) + 1e-30
    return {
        "rel_fro": float(np.linalg.norm(diff) / nr),
        "max_abs": float(np.abs(diff).max()) if diff.size else 0.0,
        "max_rowrel": float((np.abs(diff) / rowmax).max()) if diff.size else 0.0,
        "cos": float((y * r).sum() / (np.linalg.norm(y) * nr + 1e-30)),
        "finite": bool(np.isfinite(y).all()),
    }


TOLERANCE = {"float32": 1e-4, "float16": 3e-3, "bfloat16": 2e-2, "q8": 2e-2, "q4": 2e-2}
ROWREL_TOL = 1e-2  # north star: max |err| <= 1e-2 * row max |ref| for bf16 activations


def make_inputs(d, E, k, T, routing, seed):
    """The reference's benchmark inputs (moelab/torch_backend.py:50-54): rng = default_rng(seed),
    x = rng.standard_normal((T, d)) then make_routing(T, E, k, routing, rng). -> (x fp32, idx, wts)."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((T, d)).astype(np.float32)
    idx, wts = make_routing(T, E, k, routing, rng)
    return x, idx, wts
