"""GPU parity of the MXFP4 path (b200_mxfp4_moe) and the gpt-oss epilogue (b200_mxfp4_gptoss) against the fp64
oracle on the kernels' own dequantised weights. Ports the reference's MXFP4 properties: every dispatch path,
odd shapes, large E8M0 scales (tests/test_mxfp4_large_scales.py), fp32 activations, zero weights, and the gpt-oss
biases + clamped SwiGLU with the clamps reachable (tests/test_gptoss_patch.py:17-84)."""
import numpy as np
import pytest
import torch

import oracle
from helpers import guard_tc_shapes, ROOT, assert_close, load_variant, problem_tensors, ref_from_state
from moelab_b200 import ops
from moelab_b200.shapes import MoEShape

pytestmark = pytest.mark.gpu
FP4 = ROOT + "/moelab_b200/variants/cuda/b200_mxfp4_moe.py"
GPTOSS = ROOT + "/moelab_b200/variants/cuda/b200_mxfp4_gptoss.py"
POLICIES = {"auto": None, "slots": ops.POLICY_SLOTS, "tiles8": ops.POLICY_TILES8, "tiles16": ops.POLICY_TILES16,
            "tiles8ring": ops.POLICY_TILES8_RING, "tiles16ring": ops.POLICY_TILES16_RING,
            "tiles24ring": ops.POLICY_TILES24_RING, "decode": ops.POLICY_DECODE,
            "tc": ops.POLICY_TC}


@pytest.fixture(scope="module")
def mod():
    return load_variant(FP4)


@pytest.fixture(params=list(POLICIES))
def policy(request, mod, monkeypatch):
    monkeypatch.setattr(mod, "POLICY", POLICIES[request.param])
    if request.param == "tc":
        guard_tc_shapes(mod, monkeypatch)
    return request.param


@pytest.mark.parametrize("T", [1, 2, 3, 4, 5, 7, 8, 9, 17, 33, 65, 129])
def test_dispatch_boundaries(mod, policy, T):
    sh = MoEShape("q", d=256, f=384, E=16, k=4)
    p, w, x, idx, wts = problem_tensors(sh, T, "zipf", seed=T)
    st = mod.prepare(*w)
    assert_close(mod.run(st, x, idx, wts), ref_from_state(mod, st, x, idx, wts), what=T)


SHAPES = [MoEShape("d192", d=192, f=256, E=8, k=2), MoEShape("f320", d=256, f=320, E=8, k=2),
          MoEShape("gptoss-like", d=576, f=576, E=8, k=4), MoEShape("k1", d=128, f=256, E=8, k=1),
          MoEShape("E1", d=128, f=256, E=1, k=1)]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: s.name)
@pytest.mark.parametrize("T", [1, 6, 33])
def test_shapes(mod, policy, shape, T):
    p, w, x, idx, wts = problem_tensors(shape, T)
    st = mod.prepare(*w)
    assert_close(mod.run(st, x, idx, wts), ref_from_state(mod, st, x, idx, wts), what=(shape.name, T))


@pytest.mark.parametrize("T,routing", [(1, "uniform"), (3, "uniform"), (16, "one_hot"), (32, "uniform")])
def test_large_e8m0_scales(mod, policy, T, routing):
    """weights * 256 so E8M0 bytes reach >= 129; x / 256 (tests/test_mxfp4_large_scales.py:20-34)."""
    sh = MoEShape("big-scales", d=256, f=256, E=8, k=2)
    p, w, x, idx, wts = problem_tensors(sh, T, routing, seed=T)
    w = [(t.float() * 256).to(torch.bfloat16) for t in w]
    x = (x.float() / 256).to(torch.bfloat16)
    st = mod.prepare(*w)
    assert int(max(st[n][1].max().item() for n in ("g", "u", "d"))) >= 129
    assert_close(mod.run(st, x, idx, wts), ref_from_state(mod, st, x, idx, wts))


def test_zero_weights_give_exact_zero(mod, policy):
    sh = MoEShape("w", d=256, f=256, E=8, k=4)
    p, w, x, idx, wts = problem_tensors(sh, 4)
    wts = wts.clone()
    wts[0] = 0
    st = mod.prepare(*w)
    y = mod.run(st, x, idx, wts)
    assert float(y[0].float().abs().max()) == 0.0


def test_fp32_activations(mod, policy):
    sh = MoEShape("b", d=2048, f=1408, E=16, k=6)
    p, w, x, idx, wts = problem_tensors(sh, 32)
    x32 = torch.from_numpy(p["x"]).cuda()
    st = mod.prepare(*w)
    y = mod.run(st, x32, idx, wts)
    assert oracle.error_metrics(y.cpu().numpy(), ref_from_state(mod, st, x32, idx, wts))["rel_fro"] < 1e-2


# ------------------------------------------------------------------ gpt-oss epilogue
@pytest.fixture(scope="module")
def gmod():
    return load_variant(GPTOSS)


@pytest.mark.parametrize("T", [1, 2, 3, 8, 32, 128])
@pytest.mark.parametrize("pol", [None, ops.POLICY_SLOTS, ops.POLICY_TILES8])
def test_gptoss_biases_and_clamped_swiglu(gmod, T, pol):
    """Biases large enough that the +-7 clamps are hit (tests/test_gptoss_patch.py:24-29), vs the fp64 oracle."""
    sh = MoEShape("gptoss-like", d=576, f=576, E=16, k=4)
    g = torch.Generator(device="cuda").manual_seed(T)
    mk = lambda *s, sc=0.02: (torch.randn(*s, generator=g, device="cuda") * sc).to(torch.bfloat16)  # noqa: E731
    w = [mk(sh.E, sh.f, sh.d), mk(sh.E, sh.f, sh.d), mk(sh.E, sh.d, sh.f)]
    bg, bu, bd = (4 * torch.randn(sh.E, sh.f, generator=g, device="cuda"),
                  4 * torch.randn(sh.E, sh.f, generator=g, device="cuda"),
                  0.1 * torch.randn(sh.E, sh.d, generator=g, device="cuda"))
    assert (bg > 7).any() and (bu.abs() > 7).any()  # clamps reachable
    st = gmod.state(*w, bg, bu, bd)
    x = torch.randn(T, sh.d, generator=g, device="cuda").to(torch.bfloat16)
    gate = mk(sh.E, sh.d, sc=0.05)
    gb = mk(sh.E, sc=1.0)
    mod_b = gmod._b
    old = mod_b.POLICY
    mod_b.POLICY = pol
    try:
        y, idx, wts = gmod.layer(st, x, gate, sh.k, gate_b=gb, return_routing=True)
    finally:
        mod_b.POLICY = old
    ri, rw = oracle.router(x, gate, sh.k, bias=gb)
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    ref = ref_from_state(gmod, st, x, idx, wts, act=2, bg=bg, bu=bu, bd=bd)
    assert_close(y, ref, what=T)
    # the clamped activation reached the kernel (plain SwiGLU would be far off)
    other = ref_from_state(gmod, st, x, idx, wts, act=0, bg=bg, bu=bu, bd=bd)
    assert oracle.error_metrics(y.float().cpu().numpy(), other)["rel_fro"] > 0.05
    # the variant's own fp32 reference agrees as well
    assert_close(gmod.reference(st, x, idx, wts), ref, tol=2e-2, rowrel=2e-2)


@pytest.mark.parametrize("T", [1, 8, 32, 128])
def test_gptoss20b_shape_layer(gmod, T):
    """gpt-oss-20b-shaped MXFP4 layer (d=f=2880, E=32, k=4), biases N(0, 0.01), gate with bias."""
    sh = MoEShape("gpt-oss-20b", d=2880, f=2880, E=32, k=4)
    g = torch.Generator(device="cuda").manual_seed(100 + T)
    mk = lambda *s, sc=0.02: (torch.randn(*s, generator=g, device="cuda") * sc).to(torch.bfloat16)  # noqa: E731
    w = [mk(sh.E, sh.f, sh.d), mk(sh.E, sh.f, sh.d), mk(sh.E, sh.d, sh.f)]
    b = [mk(sh.E, sh.f, sc=0.01).float(), mk(sh.E, sh.f, sc=0.01).float(), mk(sh.E, sh.d, sc=0.01).float()]
    st = gmod.state(*w, *b)
    x = torch.randn(T, sh.d, generator=g, device="cuda").to(torch.bfloat16)
    gate, gb = mk(sh.E, sh.d), mk(sh.E, sc=0.01)
    y, idx, wts = gmod.layer(st, x, gate, sh.k, gate_b=gb, return_routing=True)
    ri, _ = oracle.router(x, gate, sh.k, bias=gb)
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    assert_close(y, ref_from_state(gmod, st, x, idx, wts, act=2, bg=b[0], bu=b[1], bd=b[2]), what=T)


# ------------------------------------------------------------------ tensor-core policy (tcgen05), MXFP4
@pytest.mark.parametrize("T,routing", [(1, "uniform"), (9, "uniform"), (200, "uniform"), (300, "one_hot"),
                                       (513, "zipf")])
def test_tc_mxfp4_vs_oracle(mod, T, routing):
    """E2M1 * E8M0 decoded exactly into the swizzled UMMA tiles; tiles of up to 128 slots."""
    sh = MoEShape("tc", d=256, f=384, E=8, k=2)
    p, w, x, idx, wts = problem_tensors(sh, T, routing, seed=T)
    st = mod.prepare(*w)
    mod._ws(st, sh.k)
    y = ops.experts(st, x, idx, wts, policy=ops.POLICY_TC)
    assert_close(y, ref_from_state(mod, st, x, idx, wts), what=(T, routing))


@pytest.mark.parametrize("T", [64, 300])
def test_tc_mxfp4_large_scales(mod, T):
    sh = MoEShape("big-scales", d=256, f=256, E=8, k=2)
    p, w, x, idx, wts = problem_tensors(sh, T, seed=T)
    w = [(t.float() * 256).to(torch.bfloat16) for t in w]
    x = (x.float() / 256).to(torch.bfloat16)
    st = mod.prepare(*w)
    mod._ws(st, sh.k)
    y = ops.experts(st, x, idx, wts, policy=ops.POLICY_TC)
    assert_close(y, ref_from_state(mod, st, x, idx, wts))


def test_tc_gptoss_epilogue():
    """Biases + clamped SwiGLU in the tensor-core epilogue (d = f = 1152, multiples of 128)."""
    g = load_variant(GPTOSS)
    E, d, f, k, T = 8, 1152, 1152, 4, 256
    gen = torch.Generator(device="cuda").manual_seed(5)
    mk = lambda *s, sc=0.02: (torch.randn(*s, generator=gen, device="cuda") * sc).to(torch.bfloat16)  # noqa: E731
    w = [mk(E, f, d), mk(E, f, d), mk(E, d, f)]
    b = (4 * torch.randn(E, f, generator=gen, device="cuda"), 4 * torch.randn(E, f, generator=gen, device="cuda"),
         0.1 * torch.randn(E, d, generator=gen, device="cuda"))
    st = g.state(*w, *b)
    g._b._ws(st, k)
    x = torch.randn(T, d, generator=gen, device="cuda").to(torch.bfloat16)
    idx = torch.stack([torch.randperm(E, generator=gen, device="cuda")[:k] for _ in range(T)]).to(torch.int32)
    wts = torch.rand(T, k, generator=gen, device="cuda")
    y = ops.experts(st, x, idx, wts, act=2, policy=ops.POLICY_TC)
    assert_close(y, ref_from_state(g, st, x, idx, wts, act=2, bg=b[0], bu=b[1], bd=b[2]))
