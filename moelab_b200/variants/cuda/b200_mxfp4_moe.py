"""B200-native MXFP4 MoE variant (moe-lab variant contract).

Drop-in for moelab/variants/mlx/metal_mxfp4_moe.py (:474-512 run, :448-455 prepare/dequant) on NVIDIA B200:
E2M1 codes with one E8M0 scale per 32 inputs (mx.quantize(w, mode="mxfp4"), W_BITS 4.25). The kernels fold the
E8M0 scale into exact bf16 MMA operands (e2m1 * 2^(s-127) is representable in bf16), so no accuracy is lost
to the format conversion. POLICY pins one kernel path; LOAD_MAX moves the decode -> tile switch like the
reference's LOAD_MAX / load_max (:465-471).
"""
import os
import sys

import torch

_ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
if _ROOT not in sys.path:
    sys.path.insert(0, _ROOT)

from moelab_b200 import ops  # noqa: E402

META = {"name": "b200_mxfp4_moe", "description": "B200 sm_100a MXFP4: fused router, grouped tensor-core experts "
                                                 "with exact E2M1/E8M0 decode, deterministic fused combine"}
MODE, GS, BITS = "mxfp4", 32, 4
W_BITS = 4 + 8 / 32
POLICY = None  # None = the library's load-based dispatcher; tests pin ops.POLICY_* here
LOAD_MAX = None  # a number: the decode path up to this load (T*k/E), the grouped tile kernels above it


def load_max(E, k):
    """Largest load T*k/E the dispatcher serves with the decode kernels (LOAD_MAX when set)."""
    if LOAD_MAX is not None:
        return LOAD_MAX
    T = 1
    while ops.policy(T + 1, E, k) in (ops.POLICY_SLOTS, ops.POLICY_DECODE):
        T += 1
    return T * k / E


def _policy(T=None, E=None, k=None):
    if POLICY is not None:
        return POLICY
    if LOAD_MAX is not None and T is not None:
        return ops.POLICY_DECODE if T * k / E <= LOAD_MAX else ops.POLICY_TILES16_RING
    return ops.POLICY_AUTO


def prepare(w_gate, w_up, w_down):
    E, f, d = w_gate.shape
    assert d % 64 == 0 and f % 64 == 0, "d, f must be multiples of 64"
    assert w_gate.is_cuda, "moelab_b200 runs on CUDA devices only"
    wb = [w.to(torch.bfloat16).contiguous() for w in (w_gate, w_up, w_down)]
    return {"g": ops.quantize_mxfp4(wb[0]), "u": ops.quantize_mxfp4(wb[1]), "d": ops.quantize_mxfp4(wb[2]),
            "E": E, "f": f, "dm": d, "fmt": "mxfp4", "ws": ops.Workspace(d, f, E, 0, w_gate.device)}


def state_from_mlx(g, u, d_, E, f, dm, bg=None, bu=None, bd=None, act=0):
    """State from mlx-layout pairs (wq int32, scales uint8) per projection (metal_mxfp4_gptoss.py:100-107)."""
    st = {"g": ops.mxfp4_from_mlx(*g), "u": ops.mxfp4_from_mlx(*u), "d": ops.mxfp4_from_mlx(*d_), "E": E, "f": f,
          "dm": dm, "fmt": "mxfp4", "ws": ops.Workspace(dm, f, E, 0, g[0].device), "act": act}
    if bg is not None:
        st.update(bg=bg.float().contiguous(), bu=bu.float().contiguous(), bd=bd.float().contiguous())
    return st


def dequant(s):
    return tuple(ops.dequant_mxfp4(*s[n]) for n in ("g", "u", "d"))


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
    y = ops.experts(s, xb.contiguous(), idx.to(torch.int32).contiguous(), wts.to(torch.float32).contiguous(),
                    act=act, policy=_policy(T, s["E"], k))
    return y if x.dtype == torch.bfloat16 else y.to(x.dtype)


def layer(s, x, gate_w, k, gate_b=None, norm=True, rscale=1.0, act=None, residual=None, return_routing=False,
          stage_events=None):
    act = s.get("act", 0) if act is None else act
    _ws(s, k)
    return ops.layer(s, x, gate_w, k, gate_b=gate_b, norm=norm, rscale=rscale, act=act,
                     policy=_policy(x.shape[0], s["E"], k),
                     residual=residual, return_routing=return_routing, stage_events=stage_events)
