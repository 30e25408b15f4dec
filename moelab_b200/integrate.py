"""Model integration: run the sparse-MoE blocks of a Hugging Face transformers model through this library's layer
call.

This is the torch counterpart of the reference's mlx-lm patch (moelab/e2e.py:29-72 and its _patch_gptoss /
_patch_deepseek variants). That patch swaps the expert compute of every MoE block for a variant's `run` at
decode-sized calls (<= MAX_T tokens, e2e.py:26) and keeps the stock path above. Here each block's expert
weights are quantized once into the variant state, and the block's forward runs router + experts + combine as
one `layer` call for up to `max_tokens` tokens. Supported blocks:

- Qwen3MoeSparseMoeBlock, MixtralSparseMoeBlock. `experts.gate_up_proj` [E, 2f, d] and `experts.down_proj`
  [E, d, f], SiLU-gated. Router: softmax over all experts, top-k, renormalised when `norm_topk_prob`
  (Qwen3-MoE) or always (Mixtral). int4 affine g64 or MXFP4.
- GptOssMLP. `experts.gate_up_proj` [E, d, 2f] with gate and up columns interleaved, `down_proj` [E, f, d],
  per-expert biases, clamped SwiGLU (alpha 1.702, limit 7, (u + 1)). Router: linear with bias, softmax over
  the top-k logits (e2e.py:171-176). MXFP4, the format gpt-oss ships in. Returns (y, routing weights) like the
  stock block.
- DeepseekV2Moe with `topk_method == "greedy"`. The routed experts are laid out as in Qwen3-MoE. The
  `shared_experts` MLP (width n * f) runs as n always-on experts of weight 1 (e2e.py:146-147). Router: fp32
  softmax over all experts, top-k without renormalisation, times `routed_scaling_factor` (e2e.py:136-140).
  int4.

The library computes router logits in fp32 from bf16 inputs. Where a stock block computes them in the model
dtype, near-ties can pick a different expert. `dequantize_into_stock` writes the variant's dequantized weights
back into the stock parameters, so a stock model runs on exactly the weights the kernels see; the tests compare
the two on that basis.
"""
import types

import torch

from . import ops
from .variants.cuda import b200_mxfp4_gptoss, b200_mxfp4_moe, b200_q4_moe

FAMILIES = {"Qwen3MoeSparseMoeBlock": "switch", "MixtralSparseMoeBlock": "switch", "GptOssMLP": "gptoss",
            "DeepseekV2Moe": "deepseek"}
KNOWN_BLOCKS = tuple(FAMILIES)
MAX_TOKENS = 256  # decode-sized calls use the library; larger ones keep the stock block (e2e.py:26)


def moe_blocks(model):
    """The model's sparse-MoE blocks this patch can take over, in module order."""
    return [m for m in model.modules() if type(m).__name__ in FAMILIES]


def _variant(fmt):
    if fmt == "q4":
        return b200_q4_moe
    if fmt == "mxfp4":
        return b200_mxfp4_moe
    raise ValueError(f"unknown format {fmt!r} (q4 or mxfp4)")


def _is_silu(act):
    return act is None or isinstance(act, torch.nn.SiLU) or type(act).__name__ in ("SiLU", "SiLUActivation")


def _bf16(t):
    return t.detach().to(torch.bfloat16).contiguous()


def _switch_weights(ex):
    E, f2, d = ex.gate_up_proj.shape
    f = f2 // 2
    assert ex.down_proj.shape == (E, d, f), "unexpected expert layout"
    assert _is_silu(getattr(ex, "act_fn", None)), "only SiLU-gated experts are supported"
    w = ex.gate_up_proj.detach()
    return w[:, :f], w[:, f:], ex.down_proj.detach()


def _prepare(b, fmt):
    """(variant module, state, forward kind, static call arguments) for one block."""
    fam = FAMILIES[type(b).__name__]
    if fam == "switch":
        mod = _variant(fmt)
        wg, wu, wd = _switch_weights(b.experts)
        assert wg.is_cuda, "moelab_b200 runs on CUDA devices only"
        st = mod.prepare(_bf16(wg), _bf16(wu), _bf16(wd))
        return mod, st, {"k": int(b.gate.top_k), "norm": bool(getattr(b.gate, "norm_topk_prob", True))}
    if fam == "gptoss":
        ex = b.experts
        assert ex.gate_up_proj.is_cuda, "moelab_b200 runs on CUDA devices only"
        assert float(ex.alpha) == 1.702 and float(ex.limit) == 7.0, "clamped SwiGLU constants differ"
        gu, bgu = ex.gate_up_proj.detach(), ex.gate_up_proj_bias.detach()
        wg, wu = gu[..., ::2].transpose(1, 2), gu[..., 1::2].transpose(1, 2)  # [E, f, d]
        wd = ex.down_proj.detach().transpose(1, 2)                               # [E, d, f]
        st = b200_mxfp4_gptoss.state(_bf16(wg), _bf16(wu), _bf16(wd), bgu[:, ::2], bgu[:, 1::2],
                                     ex.down_proj_bias.detach())
        return b200_mxfp4_gptoss, st, {"k": int(b.router.top_k)}
    # deepseek
    if fmt != "q4":
        raise ValueError("DeepSeek shared experts run on the int4 path")
    assert b.topk_method == "greedy", "only greedy top-k routing is supported"
    wg, wu, wd = _switch_weights(b.experts)
    assert wg.is_cuda, "moelab_b200 runs on CUDA devices only"
    sh = b.shared_experts
    assert sh.gate_proj.bias is None and _is_silu(getattr(sh, "act_fn", None)), "unsupported shared MLP"
    st = b200_q4_moe.prepare_shared(_bf16(wg), _bf16(wu), _bf16(wd), _bf16(sh.gate_proj.weight),
                                    _bf16(sh.up_proj.weight), _bf16(sh.down_proj.weight))
    return b200_q4_moe, st, {"k": int(b.top_k), "norm": False, "rscale": float(b.routed_scaling_factor)}


def patch_hf_moe(model, fmt="q4", max_tokens=MAX_TOKENS):
    """Quantize every known sparse-MoE block's experts and route its forward through the library for calls of up to
    `max_tokens` tokens. Returns the number of blocks patched. Idempotent (a patched block is re-quantized).
    gpt-oss blocks always use MXFP4."""
    if fmt not in ("q4", "mxfp4"):
        raise ValueError(f"unknown format {fmt!r} (q4 or mxfp4)")
    blocks = moe_blocks(model)
    for b in blocks:
        mod, st, kw = _prepare(b, fmt)
        if "_moeb_stock" not in b.__dict__:
            b._moeb_stock = b.forward
        b._moeb = {"family": FAMILIES[type(b).__name__], "mod": mod, "state": st, "kw": kw,
                   "max_tokens": int(max_tokens)}
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
            if cfg["family"] == "gptoss":
                gu = ex.gate_up_proj
                gu[..., ::2].copy_(wg.transpose(1, 2).to(gu.dtype))
                gu[..., 1::2].copy_(wu.transpose(1, 2).to(gu.dtype))
                ex.down_proj.copy_(wd.transpose(1, 2).to(ex.down_proj.dtype))
                continue
            E = ex.gate_up_proj.shape[0]
            ex.gate_up_proj.copy_(torch.cat([wg[:E], wu[:E]], dim=1).to(ex.gate_up_proj.dtype))
            ex.down_proj.copy_(wd[:E].to(ex.down_proj.dtype))
            if cfg["family"] == "deepseek":  # the shared MLP: experts E .. E + n - 1 of the state
                sh = b.shared_experts
                sh.gate_proj.weight.copy_(wg[E:].reshape(-1, wg.shape[-1]).to(sh.gate_proj.weight.dtype))
                sh.up_proj.weight.copy_(wu[E:].reshape(-1, wu.shape[-1]).to(sh.up_proj.weight.dtype))
                sh.down_proj.weight.copy_(torch.cat(list(wd[E:]), dim=1).to(sh.down_proj.weight.dtype))


def _forward(self, hidden_states):
    cfg = self._moeb
    shape = hidden_states.shape
    T = hidden_states.numel() // shape[-1]
    if T > cfg["max_tokens"] or self.training:
        return self._moeb_stock(hidden_states)
    x = hidden_states.reshape(T, shape[-1]).to(torch.bfloat16).contiguous()
    kw = cfg["kw"]
    if cfg["family"] == "gptoss":
        y, _, wts = cfg["mod"].layer(cfg["state"], x, _bf16(self.router.weight), kw["k"],
                                     gate_b=_bf16(self.router.bias), return_routing=True)
        return y.to(hidden_states.dtype).reshape(shape), wts.to(hidden_states.dtype)
    gate = self.gate.weight
    y = cfg["mod"].layer(cfg["state"], x, _bf16(gate), kw["k"], norm=kw["norm"], rscale=kw.get("rscale", 1.0))
    return y.to(hidden_states.dtype).reshape(shape)


def policy_for(T, block):
    """The expert kernel family the library picks for a T-token call of this block (for reports)."""
    st = block._moeb["state"]
    return ops.policy(T, st["E"], block._moeb["kw"]["k"])
