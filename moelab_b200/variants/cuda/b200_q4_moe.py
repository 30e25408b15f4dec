"""B200-native int4 affine g64 MoE variant (moe-lab variant contract).

Drop-in for moelab/variants/mlx/metal_q4_moe.py (the production int4 dispatcher, :54-64) on NVIDIA B200:
  META, MODE/GS/BITS, W_BITS               (metal_q4_moe.py:26-29)
  prepare(w_gate, w_up, w_down) -> state   quantise on the GPU into the B200 layout (metal_q4_moe.py:32-35)
  dequant(state) -> (wg, wu, wd)           fp32 weights the kernels multiply (metal_q4_moe.py:38-39)
  run(state, x, idx, wts, act=0) -> y      grouped expert kernels (metal_q4_moe.py:54-64)
  run_slots(state, x, idx, act=0)          per-slot unweighted outputs [T*k, d] (metal_q4_moe.py:49-51)
  layer(state, x, gate_w, k, ...)          router + run in one stream-ordered sequence (e2e.py:51-65)
  custom_wins / POLICY                     dispatcher hook the tests can pin (metal_q4_moe.py:42-46)
All tensors are CUDA tensors; there is no CPU fallback.
"""
import os
import sys

import torch

_ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
if _ROOT not in sys.path:
    sys.path.insert(0, _ROOT)

from moelab_b200 import ops  # noqa: E402

META = {"name": "b200_q4_moe", "description": "B200 sm_100a int4-g64: fused router, grouped tensor-core experts, "
                                               "deterministic fused combine"}
MODE, GS, BITS = "affine", 64, 4
W_BITS = BITS + 32 / GS
POLICY = None  # None = the library's load-based dispatcher; tests pin ops.POLICY_* here


def _policy():
    return ops.POLICY_AUTO if POLICY is None else POLICY


def prepare(w_gate, w_up, w_down):
    E, f, d = w_gate.shape
    assert d % 64 == 0 and f % 64 == 0, "d, f must be multiples of 64"
    assert w_gate.is_cuda, "moelab_b200 runs on CUDA devices only"
    wb = [w.to(torch.bfloat16).contiguous() for w in (w_gate, w_up, w_down)]
    return {"g": ops.quantize_q4(wb[0]), "u": ops.quantize_q4(wb[1]), "d": ops.quantize_q4(wb[2]),
            "E": E, "f": f, "dm": d, "ws": ops.Workspace(d, f, E, 0, w_gate.device)}


def state_from_mlx(g, u, d_, E, f, dm, bg=None, bu=None, bd=None, act=0):
    """State from mlx-layout triplets (wq int32, scales bf16, biases bf16) per projection."""
    st = {"g": ops.q4_from_mlx(*g), "u": ops.q4_from_mlx(*u), "d": ops.q4_from_mlx(*d_), "E": E, "f": f, "dm": dm,
          "ws": ops.Workspace(dm, f, E, 0, g[0].device)}
    if bg is not None:
        st.update(bg=bg.float().contiguous(), bu=bu.float().contiguous(), bd=bd.float().contiguous())
    st["act"] = act
    return st


def dequant(s):
    return tuple(ops.dequant_q4(*s[n]) for n in ("g", "u", "d"))


def _ws(s, k):
    ws = s["ws"]
    if ws.k != k:
        s["ws"] = ws = ops.Workspace(s["dm"], s["f"], s["E"], k, ws.device)
    return ws


def run(s, x, idx, wts, act=None):
    T, k = idx.shape
    act = s.get("act", 0) if act is None else act
    _ws(s, k)
    xb = x if x.dtype == torch.bfloat16 else x.to(torch.bfloat16)
    y = ops.experts_q4(s, xb.contiguous(), idx.to(torch.int32).contiguous(), wts.to(torch.float32).contiguous(),
                       act=act, policy=_policy())
    return y if x.dtype == torch.bfloat16 else y.to(x.dtype)


def run_slots(s, x, idx, act=None):
    """Unweighted per-slot expert outputs [T*k, d] (each slot run as its own token with weight 1)."""
    T, k = idx.shape
    xs = x.to(torch.bfloat16).repeat_interleave(k, dim=0).contiguous()
    ones = torch.ones(T * k, 1, dtype=torch.float32, device=x.device)
    act = s.get("act", 0) if act is None else act
    _ws(s, 1)
    y = ops.experts_q4(s, xs, idx.reshape(T * k, 1).to(torch.int32).contiguous(), ones, act=act, policy=_policy())
    return y if x.dtype == torch.bfloat16 else y.to(x.dtype)


def prepare_shared(w_gate, w_up, w_down, sw_gate, sw_up, sw_down):
    """DeepSeek layer: routed experts [E, f, d], [E, f, d], [E, d, f] plus the always-on shared MLP
    (gate/up [fs, d], down [d, fs]; moelab/e2e.py:146-147). The shared MLP is split along its width into
    fs / f experts of width f appended after the routed ones: SwiGLU acts per row of h and down sums over the
    width, so the split changes nothing but the fp32 summation grouping."""
    E, f, d = w_gate.shape
    fs = sw_gate.shape[0]
    assert fs % f == 0, "shared width must be a multiple of the expert width"
    n = fs // f
    sg = sw_gate.reshape(n, f, d)
    su = sw_up.reshape(n, f, d)
    sd = sw_down.reshape(d, n, f).permute(1, 0, 2)
    s = prepare(torch.cat([w_gate, sg]), torch.cat([w_up, su]), torch.cat([w_down, sd]))
    s["n_shared"] = n
    return s


def layer(s, x, gate_w, k, gate_b=None, norm=True, rscale=1.0, act=None, residual=None, return_routing=False,
          stage_events=None):
    """Router + experts (+ the state's shared experts, if any) -> y; routing has k + n_shared slots per token."""
    act = s.get("act", 0) if act is None else act
    ns = s.get("n_shared", 0)
    _ws(s, k + ns)
    return ops.layer_q4(s, x, gate_w, k, gate_b=gate_b, norm=norm, rscale=rscale, act=act, policy=_policy(),
                        residual=residual, return_routing=return_routing, stage_events=stage_events, n_shared=ns)


def custom_wins(T, k, E, D, F):
    """The dispatcher's choice for these dims (True = grouped expert tiles, False = per-slot tiles)."""
    return ops.policy(T, E, k) not in (ops.POLICY_SLOTS, ops.POLICY_DECODE)
