"""B200-native MXFP4 MoE variant for gpt-oss (mlx-lm SwitchGLU with bias=True).

Mirrors moelab/variants/mlx/metal_mxfp4_gptoss.py: the same kernels as b200_mxfp4_moe with
  * per-expert biases: gate/up bias added before the activation, down bias before the routing weight
    (y = sum_k w_k * (W_down h + b_down), metal_mxfp4_gptoss.py:35-43, :110-126);
  * act = 1 (gpt-oss clamped SwiGLU: g = min(g, 7), u = clip(u, -7, 7), h = g * sigmoid(1.702 g) * (u + 1))
    for states built by state(); prepare() keeps the lab contract (plain SwiGLU, zero biases) like the
    reference (:88-97).
The C ABI numbers the activations 0 SwiGLU, 1 tanh-GELU, 2 clamped SwiGLU; this module maps its act = 1 to 2.
"""
import os
import sys

import torch

_ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
if _ROOT not in sys.path:
    sys.path.insert(0, _ROOT)

from moelab_b200.variants.cuda import b200_mxfp4_moe as _b  # noqa: E402

META = {"name": "b200_mxfp4_gptoss", "description": "b200_mxfp4_moe kernels + per-expert biases + gpt-oss clamped "
                                                    "SwiGLU (alpha 1.702, limit 7, up + 1)"}
MODE, GS, BITS, W_BITS = _b.MODE, _b.GS, _b.BITS, _b.W_BITS
ALPHA, LIMIT = 1.702, 7.0
_ABI_ACT = {0: 0, 1: 2}


def prepare(w_gate, w_up, w_down):
    """Lab contract (standard SwiGLU, zero biases): exercises the same kernels with act 0."""
    s = _b.prepare(w_gate, w_up, w_down)
    E, f, d = w_gate.shape
    dev = w_gate.device
    s.update(bg=torch.zeros(E, f, device=dev), bu=torch.zeros(E, f, device=dev), bd=torch.zeros(E, d, device=dev),
             act=0)
    return s


def state(w_gate, w_up, w_down, b_gate, b_up, b_down):
    """gpt-oss experts: bf16 weights [E,f,d],[E,f,d],[E,d,f] quantised to MXFP4 + fp32 biases, act 1."""
    s = _b.prepare(w_gate, w_up, w_down)
    s.update(bg=b_gate.float().contiguous(), bu=b_up.float().contiguous(), bd=b_down.float().contiguous(), act=1)
    return s


def dequant(s):
    return _b.dequant(s)


def run(s, x, idx, wts):
    return _b.run(s, x, idx, wts, act=_ABI_ACT[s.get("act", 0)])


def layer(s, x, gate_w, k, gate_b=None, residual=None, return_routing=False):
    """gpt-oss MLPBlock: router = Linear with bias, softmax over the top-k (e2e.py:171-176)."""
    return _b.layer(s, x, gate_w, k, gate_b=gate_b, norm=True, act=_ABI_ACT[s.get("act", 0)], residual=residual,
                    return_routing=return_routing)


@torch.no_grad()
def reference(s, x, idx, wts):
    """fp32 truth for quality checks (metal_mxfp4_gptoss.py:110-126): dequantise the selected experts and compute
    in fp32 with torch (slow; not the kernel path)."""
    wg, wu, wd = dequant(s)
    x32 = x.float()
    y = torch.zeros_like(x32)
    for e in idx.unique().tolist():
        t, j = (idx == e).nonzero(as_tuple=True)
        g = x32[t] @ wg[e].T + s["bg"][e]
        u = x32[t] @ wu[e].T + s["bu"][e]
        if s.get("act", 0):
            g, u = g.clamp(max=LIMIT), u.clamp(-LIMIT, LIMIT)
            h = g * torch.sigmoid(ALPHA * g) * (u + 1)
        else:
            h = torch.nn.functional.silu(g) * u
        o = h @ wd[e].T + s["bd"][e]
        y.index_add_(0, t, o * wts[t, j, None].float())
    return y.to(x.dtype)
