"""Model integration (moelab_b200/integrate.py): Hugging Face sparse-MoE blocks through the library.

Torch counterpart of the reference's mlx-lm patch and its quality check (moelab/e2e.py:29-72, :210-241). The
models are tiny Qwen3-MoE / Mixtral configurations with seeded random weights (no checkpoints offline)."""
import numpy as np
import pytest
import torch

from moelab_b200 import integrate

transformers = pytest.importorskip("transformers")


def _qwen3(dtype=torch.bfloat16, norm=True):
    cfg = transformers.Qwen3MoeConfig(vocab_size=512, hidden_size=256, intermediate_size=512,
                                      moe_intermediate_size=128, num_hidden_layers=2, num_attention_heads=4,
                                      num_key_value_heads=2, head_dim=64, num_experts=16, num_experts_per_tok=4,
                                      norm_topk_prob=norm, max_position_embeddings=128)
    torch.manual_seed(0)
    return transformers.AutoModelForCausalLM.from_config(cfg, dtype=dtype)


def _mixtral(dtype=torch.bfloat16):
    cfg = transformers.MixtralConfig(vocab_size=512, hidden_size=256, intermediate_size=128, num_hidden_layers=2,
                                     num_attention_heads=4, num_key_value_heads=2, head_dim=64,
                                     num_local_experts=8, num_experts_per_tok=2, max_position_embeddings=128)
    torch.manual_seed(1)
    return transformers.AutoModelForCausalLM.from_config(cfg, dtype=dtype)


def _gptoss(dtype=torch.bfloat16):
    cfg = transformers.GptOssConfig(vocab_size=512, hidden_size=256, intermediate_size=256, num_hidden_layers=2,
                                    num_attention_heads=4, num_key_value_heads=2, head_dim=64, num_local_experts=8,
                                    num_experts_per_tok=2, max_position_embeddings=128, sliding_window=64)
    torch.manual_seed(2)
    m = transformers.AutoModelForCausalLM.from_config(cfg, dtype=dtype)
    g = torch.Generator().manual_seed(7)
    with torch.no_grad():  # the stock init leaves the expert biases at zero; give them N(0, 0.01)
        for b in integrate.moe_blocks(m):
            for t in (b.experts.gate_up_proj_bias, b.experts.down_proj_bias):
                t.copy_((torch.randn(t.shape, generator=g) * 0.01).to(t.dtype))
    return m


def _deepseek(dtype=torch.bfloat16):
    cfg = transformers.DeepseekV2Config(vocab_size=512, hidden_size=256, intermediate_size=512, moe_intermediate_size=128,
                                        num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=4,
                                        n_routed_experts=16, num_experts_per_tok=4, n_shared_experts=2,
                                        topk_method="greedy", routed_scaling_factor=1.5, first_k_dense_replace=0,
                                        kv_lora_rank=64, q_lora_rank=None, qk_rope_head_dim=32, qk_nope_head_dim=32,
                                        v_head_dim=32, max_position_embeddings=128, rope_scaling=None)
    torch.manual_seed(3)
    return transformers.AutoModelForCausalLM.from_config(cfg, dtype=dtype)


def test_finds_blocks_and_refuses_cpu_weights():
    m = _qwen3()
    assert len(integrate.moe_blocks(m)) == 2
    assert len(integrate.moe_blocks(_mixtral())) == 2
    assert len(integrate.moe_blocks(_gptoss())) == 2
    ds = _deepseek()
    assert len(integrate.moe_blocks(ds)) == 2
    with pytest.raises(ValueError, match="int4"):
        integrate.patch_hf_moe(ds, fmt="mxfp4")
    with pytest.raises(AssertionError, match="CUDA"):
        integrate.patch_hf_moe(m)
    with pytest.raises(ValueError):
        integrate.patch_hf_moe(m, fmt="int8")


class _TorchVariant:
    """Stand-in for a variant module (CPU, plain torch): prepare keeps the weights, layer runs the block's math
    (softmax, top-k, renormalise or not, SiLU-gated experts) and counts its calls."""
    calls = 0

    @staticmethod
    def prepare(wg, wu, wd):
        return {"g": wg.float(), "u": wu.float(), "d": wd.float(), "E": wg.shape[0]}

    @staticmethod
    def dequant(st):
        return st["g"], st["u"], st["d"]

    @classmethod
    def layer(cls, st, x, gate_w, k, norm=True, rscale=1.0):
        cls.calls += 1
        p = torch.softmax(x.float() @ gate_w.float().T, dim=-1)
        w, i = torch.topk(p, k, dim=-1)
        if norm:
            w = w / w.sum(-1, keepdim=True)
        w = w * rscale
        y = torch.zeros(x.shape, dtype=torch.float32)
        for t in range(x.shape[0]):
            for j in range(k):
                e = int(i[t, j])
                h = torch.nn.functional.silu(st["g"][e] @ x[t].float()) * (st["u"][e] @ x[t].float())
                y[t] += w[t, j] * (st["d"][e] @ h)
        return y.to(x.dtype)


def test_patch_routes_decode_calls_and_unpatches(monkeypatch):
    """Host logic of the patch with a CPU stand-in for the variant: calls of up to max_tokens tokens go through
    `layer` (same result as the stock block on the same weights), larger ones through the stock forward, and
    unpatching restores the stock forward."""
    m = _qwen3(dtype=torch.float32).eval()
    monkeypatch.setattr(integrate, "_variant", lambda fmt: _TorchVariant)
    monkeypatch.setattr(torch.Tensor, "is_cuda", property(lambda self: True))  # the CUDA-only guard
    ids = torch.arange(6).view(1, 6)
    ref = _logits(m, ids)
    assert integrate.patch_hf_moe(m, max_tokens=6) == 2
    monkeypatch.undo()
    monkeypatch.setattr(integrate, "_variant", lambda fmt: _TorchVariant)
    _TorchVariant.calls = 0
    out = _logits(m, ids)
    assert _TorchVariant.calls == 2  # one call per block
    assert torch.allclose(out, ref, rtol=1e-2, atol=5e-3)  # the layer call takes bf16 activations and gate
    _TorchVariant.calls = 0
    _logits(m, torch.arange(7).view(1, 7))  # 7 > 6 tokens: stock blocks
    assert _TorchVariant.calls == 0
    assert integrate.unpatch_hf_moe(m) == 2
    assert "_moeb" not in integrate.moe_blocks(m)[0].__dict__


def _logits(model, ids):
    with torch.no_grad():
        return model(ids).logits.float()


@pytest.mark.gpu
@pytest.mark.parametrize("family,fmt", [("qwen3", "q4"), ("qwen3_nonorm", "q4"), ("mixtral", "q4"),
                                        ("mixtral", "mxfp4"), ("gptoss", "mxfp4"), ("deepseek", "q4")])
def test_patched_matches_stock_on_the_same_weights(family, fmt):
    """Patched model vs the stock model on the dequantized weights: the same network, so logits agree to the
    kernels' bf16 / fp32 arithmetic (and the top-1 tokens almost everywhere). gpt-oss: biases and the clamped
    SwiGLU; DeepSeek: greedy routing with a scaling factor and two shared experts."""
    make = {"qwen3": _qwen3, "qwen3_nonorm": lambda: _qwen3(norm=False), "mixtral": _mixtral, "gptoss": _gptoss,
            "deepseek": _deepseek}[family]
    patched, stock = make().cuda().eval(), make().cuda().eval()
    assert integrate.patch_hf_moe(patched, fmt=fmt) == 2
    integrate.dequantize_into_stock(patched)  # the stock parameters of `patched` now hold the dequantized weights
    stock.load_state_dict(patched.state_dict())
    ids = torch.randint(0, 512, (2, 24), generator=torch.Generator().manual_seed(5)).cuda()
    a, b = _logits(patched, ids), _logits(stock, ids)
    rel = (a - b).norm() / b.norm()
    assert rel < 2e-2, rel.item()
    agree = (a.argmax(-1) == b.argmax(-1)).float().mean().item()
    assert agree >= 0.9, agree


@pytest.mark.gpu
def test_stock_path_above_max_tokens_and_unpatch():
    m = _qwen3().cuda().eval()
    ref = _logits(m, torch.arange(16).view(1, 16).cuda())
    integrate.patch_hf_moe(m, max_tokens=8)
    assert torch.equal(_logits(m, torch.arange(16).view(1, 16).cuda()), ref)  # 16 > 8 tokens: stock blocks
    assert integrate.unpatch_hf_moe(m) == 2
    assert torch.equal(_logits(m, torch.arange(16).view(1, 16).cuda()), ref)


@pytest.mark.gpu
def test_decode_with_kv_cache():
    """Greedy decode with the KV cache: every step is a T = 1 call of the library (slot kernels); the tokens of
    the patched model follow those of the stock model on the same dequantized weights."""
    patched, stock = _qwen3().cuda().eval(), _qwen3().cuda().eval()
    integrate.patch_hf_moe(patched)
    integrate.dequantize_into_stock(patched)
    stock.load_state_dict(patched.state_dict())
    ids = torch.randint(0, 512, (1, 6), generator=torch.Generator().manual_seed(9)).cuda()
    kw = dict(max_new_tokens=12, do_sample=False, pad_token_id=0)
    with torch.no_grad():
        ga, gb = patched.generate(ids, **kw), stock.generate(ids, **kw)
    same = (ga == gb).float().mean().item()
    assert same >= 0.9, (ga.tolist(), gb.tolist())


@pytest.mark.gpu
def test_perplexity_against_fp32_truth():
    """Quality check in the manner of e2e.py:210-241: cross-entropy on a token sequence of the int4 model, of the
    stock bf16 model (original weights) and of the fp32 truth. On random weights the NLL is ~6.3 nats; a wrong
    kernel moves it by far more than quantization and bf16 do (both stay within 0.1 nats of the truth here)."""
    truth = _qwen3(dtype=torch.float32).cuda().eval()
    stock = _qwen3().cuda().eval()
    patched = _qwen3().cuda().eval()
    integrate.patch_hf_moe(patched)
    ids = torch.randint(0, 512, (4, 32), generator=torch.Generator().manual_seed(3)).cuda()

    def nll(model):
        lg = _logits(model, ids)[:, :-1]
        return torch.nn.functional.cross_entropy(lg.reshape(-1, lg.shape[-1]), ids[:, 1:].reshape(-1)).item()

    n_truth, n_stock, n_patched = nll(truth), nll(stock), nll(patched)
    assert np.isfinite(n_patched)
    assert abs(n_patched - n_truth) < 0.1, (n_truth, n_stock, n_patched)
    assert abs(n_patched - n_stock) < 0.1, (n_truth, n_stock, n_patched)
