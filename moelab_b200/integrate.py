"""Model integration: run the sparse-MoE blocks of a Hugging Face transformers model (Qwen3-MoE, Mixtral) through
this library's layer call.

This is the torch counterpart of the reference's mlx-lm patch (moelab/e2e.py:29-72). That patch swaps the expert
compute of every Qwen3MoeSparseMoeBlock for a variant's `run` at decode-sized calls (<= MAX_T tokens, e2e.py:26)
and keeps the stock path above. Here each block's expert weights (`experts.gate_up_proj` [E, 2f, d],
`experts.down_proj` [E, d, f]) are quantized once into the variant state, int4 affine g64 or MXFP4. The block's
forward then runs router + experts + combine as one `layer` call for up to `max_tokens` tokens.

The router semantics match the blocks' own routers:
- softmax over all experts, top-k, renormalised when `norm_topk_prob` (Qwen3-MoE) or always (Mixtral);
- the library computes the logits in fp32 from the bf16 inputs, where the stock block computes them in the model
  dtype. Near-ties can therefore pick a different expert.

`dequantize_into_stock` writes the variant's dequantized weights back into the stock parameters. A stock model
then runs on exactly the weights the kernels see, and the tests compare the two on that basis (the quality check
of e2e.py:210-241 compares against fp32 truth the same way).
"""
import types

import torch

from . import ops
from .variants.cuda import b200_mxfp4_moe, b200_q4_moe

# sparse-MoE block classes whose structure this patch knows: .gate (router with .weight [E, d], .top_k) and
# .experts (.gate_up_proj [E, 2f, d], .down_proj [E, d, f]) with SiLU-gated experts
KNOWN_BLOCKS = ("Qwen3MoeSparseMoeBlock", "MixtralSparseMoeBlock")
MAX_TOKENS = 256  # decode-sized calls use the library; larger ones keep the stock block (e2e.py:26)


def moe_blocks(model):
    """The model's sparse-MoE blocks this patch can take over, in module order."""
    return [m for m in model.modules() if type(m).__name__ in KNOWN_BLOCKS]


def _variant(fmt):
    if fmt == "q4":
        return b200_q4_moe
    if fmt == "mxfp4":
        return b200_mxfp4_moe
    raise ValueError(f"unknown format {fmt!r} (q4 or mxfp4)")


def _block_weights(block):
    ex = block.experts
    E, f2, d = ex.gate_up_proj.shape
    f = f2 // 2
    assert ex.down_proj.shape == (E, d, f), "unexpected expert layout"
    act = getattr(ex, "act_fn", None)
    assert act is None or isinstance(act, torch.nn.SiLU) or type(act).__name__ in ("SiLU", "SiLUActivation"), \
        "only SiLU-gated experts are supported"
    w = ex.gate_up_proj.detach()
    return w[:, :f], w[:, f:], ex.down_proj.detach()


def patch_hf_moe(model, fmt="q4", max_tokens=MAX_TOKENS):
    """Quantize every known sparse-MoE block's experts and route its forward through the library for calls of up to
    `max_tokens` tokens. Returns the number of blocks patched. Idempotent (a patched block is re-quantized)."""
    mod = _variant(fmt)
    blocks = moe_blocks(model)
    for b in blocks:
        wg, wu, wd = _block_weights(b)
        assert wg.is_cuda, "moelab_b200 runs on CUDA devices only"
        gate = b.gate
        st = mod.prepare(wg.to(torch.bfloat16), wu.to(torch.bfloat16), wd.to(torch.bfloat16))
        if "_moeb_stock" not in b.__dict__:
            b._moeb_stock = b.forward
        b._moeb = {"mod": mod, "state": st, "k": int(gate.top_k),
                   "norm": bool(getattr(gate, "norm_topk_prob", True)), "max_tokens": int(max_tokens)}
        b.forward = types.MethodType(_forward, b)
    return len(blocks)


def unpatch_hf_moe(model):
    """Restore the stock forward of every patched block."""
    n = 0
    for b in moe_blocks(model):
        if "_moeb_stock" in b.__dict__:
            b.forward = b._moeb_stock
            del b._moeb_stock
            del b._moeb
            n += 1
    return n


def dequantize_into_stock(model):
    """Write each patched block's dequantized expert weights into its stock parameters (in their dtype), so the
    stock forward runs on the weights the kernels use."""
    for b in moe_blocks(model):
        cfg = b.__dict__.get("_moeb")
        if cfg is None:
            continue
        wg, wu, wd = cfg["mod"].dequant(cfg["state"])
        ex = b.experts
        with torch.no_grad():
            ex.gate_up_proj.copy_(torch.cat([wg, wu], dim=1).to(ex.gate_up_proj.dtype))
            ex.down_proj.copy_(wd.to(ex.down_proj.dtype))


def _forward(self, hidden_states):
    cfg = self._moeb
    shape = hidden_states.shape
    T = hidden_states.numel() // shape[-1]
    if T > cfg["max_tokens"] or self.training:
        return self._moeb_stock(hidden_states)
    x = hidden_states.reshape(T, shape[-1]).to(torch.bfloat16).contiguous()
    gw = self.gate.weight.detach().to(torch.bfloat16).contiguous()
    y = cfg["mod"].layer(cfg["state"], x, gw, cfg["k"], norm=cfg["norm"])
    return y.to(hidden_states.dtype).reshape(shape)


def policy_for(T, block):
    """The expert kernel family the library picks for a T-token call of this block (for reports)."""
    st = block._moeb["state"]
    return ops.policy(T, st["E"], block._moeb["k"])
