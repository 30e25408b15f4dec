"""Checkpoint loader (moelab_b200/checkpoint.py): safetensors files with the reference's real-checkpoint tensor
names (moelab/e2e.py:48-49, :163; tests/test_real_checkpoints.py:36-66), written here as small synthetic
checkpoints from the oracle's quantizers (no downloads). CPU: the container reader, the host dequant of a
quantized router gate, the OCP -> mlx word conversion. GPU: the loaded state equals the quantize path's state bit
for bit (int4 mlx triplets, MXFP4 mlx and OCP layouts with E8M0 bytes >= 129), and runs the layer."""
import os

import numpy as np
import pytest
import torch

import oracle
from moelab_b200 import checkpoint as ck

E, F, D = 4, 128, 256


def _bf16_bits(a):
    return oracle.bf16_bits(torch.from_numpy(np.asarray(a, np.float32)))


def _q4_checkpoint(path, layer, seed=0):
    """mlx-community style int4 triplets (switch_mlp) + an 8-bit-quantized router gate; returns the bf16 weights."""
    g = torch.Generator().manual_seed(seed)
    ws = [(torch.randn(E, F, D, generator=g) * 0.02).bfloat16(), (torch.randn(E, F, D, generator=g) * 0.02).bfloat16(),
          (torch.randn(E, D, F, generator=g) * 0.02).bfloat16()]
    t = {}
    P = f"model.layers.{layer}.mlp.switch_mlp."
    for w, pr in zip(ws, ("gate_proj", "up_proj", "down_proj")):
        qw, s, b = oracle.q4_quantize(w)
        t[P + pr + ".weight"] = (qw.reshape(w.shape[0], w.shape[1], -1), "U32")
        t[P + pr + ".scales"] = (s.reshape(w.shape[0], w.shape[1], -1), "BF16")
        t[P + pr + ".biases"] = (b.reshape(w.shape[0], w.shape[1], -1), "BF16")
    # router gate quantized at 8 bits, group 64 (as mlx-lm quantizes the MoE gate of some checkpoints)
    rng = np.random.default_rng(seed)
    codes = rng.integers(0, 256, size=(E, D), dtype=np.uint32)
    words = np.zeros((E, D // 4), np.uint32)
    for i in range(4):
        words |= codes[:, i::4] << (8 * i)
    sc = _bf16_bits(rng.random((E, D // 64)) * 1e-3)
    bi = _bf16_bits(-rng.random((E, D // 64)) * 0.1)
    t[f"model.layers.{layer}.mlp.gate.weight"] = (words, "U32")
    t[f"model.layers.{layer}.mlp.gate.scales"] = (sc, "BF16")
    t[f"model.layers.{layer}.mlp.gate.biases"] = (bi, "BF16")
    ck.write_safetensors(path, t)
    return ws, (codes, sc, bi)


def test_reader_and_gate_dequant(tmp_path):
    p = str(tmp_path / "model.safetensors")
    ws, (codes, sc, bi) = _q4_checkpoint(p, 3)
    c = ck.Checkpoint(str(tmp_path))  # a directory without an index: model.safetensors
    qw, s, b = oracle.q4_quantize(ws[0])
    np.testing.assert_array_equal(c.get("model.layers.3.mlp.switch_mlp.gate_proj.weight").reshape(-1), qw.reshape(-1))
    np.testing.assert_array_equal(c.get("model.layers.3.mlp.switch_mlp.gate_proj.scales").reshape(-1), s.reshape(-1))
    deq = ck.dequant_affine(np.asarray(c.get("model.layers.3.mlp.gate.weight")),
                            np.asarray(c.get("model.layers.3.mlp.gate.scales")),
                            np.asarray(c.get("model.layers.3.mlp.gate.biases")))
    s32 = (sc.astype(np.uint32) << 16).view(np.float32)
    b32 = (bi.astype(np.uint32) << 16).view(np.float32)
    ref = codes.reshape(E, D // 64, 64) * s32[:, :, None] + b32[:, :, None]
    np.testing.assert_array_equal(deq, ref.reshape(E, D).astype(np.float32))


def test_sharded_index(tmp_path):
    a = np.arange(12, dtype=np.uint32).reshape(3, 4)
    b = np.arange(6, dtype=np.uint16).reshape(2, 3)
    ck.write_safetensors(str(tmp_path / "s1.safetensors"), {"x": (a, "U32")})
    ck.write_safetensors(str(tmp_path / "s2.safetensors"), {"y": (b, "BF16")})
    import json
    json.dump({"weight_map": {"x": "s1.safetensors", "y": "s2.safetensors"}},
              open(tmp_path / "model.safetensors.index.json", "w"))
    c = ck.Checkpoint(str(tmp_path))
    np.testing.assert_array_equal(c.get("x"), a)
    np.testing.assert_array_equal(c.get("y"), b)
    with pytest.raises(KeyError):
        c.get("z")


def test_ocp_blocks_are_mlx_words():
    rng = np.random.default_rng(0)
    nib = rng.integers(0, 16, size=(2, 3, 64), dtype=np.uint32)  # natural element order
    blocks = (nib[..., 0::2] | (nib[..., 1::2] << 4)).astype(np.uint8).reshape(2, 3, 2, 16)
    words = np.zeros((2, 3, 8), np.uint32)
    for i in range(8):
        words |= nib[..., i::8] << (4 * i)
    np.testing.assert_array_equal(ck.ocp_blocks_to_words(blocks), words)


# ------------------------------------------------------------------ GPU: parity with the quantize path
@pytest.mark.gpu
def test_q4_state_from_checkpoint_equals_quantize_path(tmp_path):
    from helpers import assert_close, ref_from_state
    from moelab_b200.variants.cuda import b200_q4_moe as v
    p = str(tmp_path / "model.safetensors")
    ws, _ = _q4_checkpoint(p, 0, seed=1)
    st = ck.q4_layer_state(p, 0)
    ref = v.prepare(*(w.cuda() for w in ws))
    for n in ("g", "u", "d"):
        assert torch.equal(st[n][0], ref[n][0]) and torch.equal(st[n][1], ref[n][1]), n
    gate = ck.gate_weight(p, 0)
    assert gate.shape == (E, D) and gate.dtype == torch.bfloat16
    x = torch.randn(5, D, device="cuda").to(torch.bfloat16)
    y, idx, wts = v.layer(st, x, gate, 2, return_routing=True)
    assert_close(y, ref_from_state(v, st, x, idx, wts))


def _fp4_weights(seed):
    g = torch.Generator().manual_seed(seed)
    ws = [torch.randn(E, F, D, generator=g), torch.randn(E, F, D, generator=g), torch.randn(E, D, F, generator=g)]
    ws[0][:, :, :32] *= 2.0 ** 10  # E8M0 bytes >= 129 (scales above 1), the real-checkpoint regression
    return [(w * 0.02).bfloat16() for w in ws]


@pytest.mark.gpu
@pytest.mark.parametrize("layout", ["mlx", "ocp"])
def test_mxfp4_state_from_checkpoint_equals_quantize_path(tmp_path, layout):
    from helpers import assert_close
    from moelab_b200.variants.cuda import b200_mxfp4_gptoss as vg
    ws = _fp4_weights(2)
    g = torch.Generator().manual_seed(3)
    bs = [(torch.randn(E, F, generator=g) * 0.01).bfloat16(), (torch.randn(E, F, generator=g) * 0.01).bfloat16(),
          (torch.randn(E, D, generator=g) * 0.01).bfloat16()]
    P = "model.layers.7.mlp.experts."
    q = [oracle.mxfp4_quantize(w) for w in ws]
    t = {}
    if layout == "mlx":
        for (qw, sc), b, pr, w in zip(q, bs, ("gate_proj", "up_proj", "down_proj"), ws):
            t[P + pr + ".weight"] = (qw.reshape(w.shape[0], w.shape[1], -1), "U32")
            t[P + pr + ".scales"] = (sc.reshape(w.shape[0], w.shape[1], -1), "U8")
            t[P + pr + ".bias"] = (oracle.bf16_bits(b), "BF16")
    else:  # OCP blocks: gate and up interleaved along the rows, two codes per byte
        def blocks(qw, N, K):
            wd = qw.reshape(E, N, K // 8)
            nib = np.stack([(wd >> (4 * i)) & 0xF for i in range(8)], -1).reshape(E, N, K)
            return (nib[..., 0::2] | (nib[..., 1::2] << 4)).astype(np.uint8).reshape(E, N, K // 32, 16)
        gb, ub = blocks(q[0][0], F, D), blocks(q[1][0], F, D)
        gu = np.empty((E, 2 * F, D // 32, 16), np.uint8)
        gu[:, 0::2], gu[:, 1::2] = gb, ub
        gs = np.empty((E, 2 * F, D // 32), np.uint8)
        gs[:, 0::2], gs[:, 1::2] = q[0][1].reshape(E, F, -1), q[1][1].reshape(E, F, -1)
        gbias = np.empty((E, 2 * F), np.uint16)
        gbias[:, 0::2], gbias[:, 1::2] = oracle.bf16_bits(bs[0]), oracle.bf16_bits(bs[1])
        t[P + "gate_up_proj_blocks"] = (gu, "U8")
        t[P + "gate_up_proj_scales"] = (gs, "U8")
        t[P + "gate_up_proj_bias"] = (gbias, "BF16")
        t[P + "down_proj_blocks"] = (blocks(q[2][0], D, F), "U8")
        t[P + "down_proj_scales"] = (q[2][1].reshape(E, D, -1), "U8")
        t[P + "down_proj_bias"] = (oracle.bf16_bits(bs[2]), "BF16")
    p = str(tmp_path / "model.safetensors")
    ck.write_safetensors(p, t)
    st = ck.mxfp4_layer_state(p, 7)
    ref = vg.state(*(w.cuda() for w in ws), *(b.cuda() for b in bs))
    for n in ("g", "u", "d"):
        assert torch.equal(st[n][0], ref[n][0]), ("codes", n)
        assert torch.equal(st[n][1], ref[n][1]), ("scales", n)
    for n in ("bg", "bu", "bd"):
        assert torch.equal(st[n], ref[n]), n
    assert int(st["g"][1].max().item()) >= 129, int(st["g"][1].max().item())  # E8M0 >= 129 carried through
    x = torch.randn(3, D, device="cuda").to(torch.bfloat16)
    idx = torch.tensor([[0, 1], [2, 3], [1, 2]], dtype=torch.int32, device="cuda")
    wts = torch.full((3, 2), 0.5, device="cuda")
    assert_close(vg.run(st, x, idx, wts), vg.reference(st, x, idx, wts).float().cpu().numpy())
