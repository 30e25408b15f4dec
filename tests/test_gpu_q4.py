"""GPU parity of the int4 path against the CPU oracle (pytest -m gpu).

Bit-exact: the quantizer's packed codes / scales / biases, fp32 dequantisation, router logits and top-k ids.
Within tolerance (rel_fro < 1e-2 and max|err| <= 1e-2 * row max|ref|): layer outputs against the fp64 oracle on
the kernels' own dequantised weights. The cases port the reference's property tests
(tests/test_mlx_variants.py, test_edge_cases.py, test_int4_small_scales.py, test_geglu.py) to this path.
"""
import numpy as np
import pytest
import torch

import oracle
from helpers import (guard_tc_shapes, Q4_VARIANT, assert_close, load_variant, problem_tensors, ref_from_state, to_b200_fp4,
                     to_b200_q4, u32)
from moelab_b200 import ops
from moelab_b200.shapes import MoEShape

pytestmark = pytest.mark.gpu

POLICIES = {"auto": None, "slots": ops.POLICY_SLOTS, "tiles8": ops.POLICY_TILES8, "tiles16": ops.POLICY_TILES16,
            "tiles8ring": ops.POLICY_TILES8_RING, "tiles16ring": ops.POLICY_TILES16_RING,
            "tiles24ring": ops.POLICY_TILES24_RING, "decode": ops.POLICY_DECODE,
            "tc": ops.POLICY_TC}


@pytest.fixture(scope="module")
def mod():
    return load_variant(Q4_VARIANT)


@pytest.fixture(params=list(POLICIES))
def policy(request, mod, monkeypatch):
    """Every expert case runs under the shipped dispatcher and under each forced kernel path
    (the reference's 'forced-custom' fixture, tests/test_edge_cases.py:26-37)."""
    monkeypatch.setattr(mod, "POLICY", POLICIES[request.param])
    if request.param == "tc":
        guard_tc_shapes(mod, monkeypatch)
    return request.param


# ------------------------------------------------------------------ formats
@pytest.mark.parametrize("rows,K", [(16, 64), (96, 256), (144, 2048), (16, 1408)])
def test_quantize_q4_bit_exact(rows, K):
    g = torch.Generator(device="cuda").manual_seed(rows + K)
    w = (torch.randn(rows, K, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    w[0, :64] = 0  # an all-zero group (q0 = 0 branch)
    w[1, :64] = torch.linspace(-1, 1, 64, device="cuda").to(torch.bfloat16)
    q, sb = ops.quantize_q4(w)
    qw, s, b = oracle.q4_quantize(w)
    ref_q, ref_sb = to_b200_q4(qw, s, b)
    np.testing.assert_array_equal(u32(q).reshape(-1), ref_q)
    np.testing.assert_array_equal(u32(sb).reshape(-1), ref_sb)
    np.testing.assert_array_equal(ops.dequant_q4(q, sb).cpu().numpy(), oracle.q4_dequant(qw, s, b))


def test_q4_from_mlx_layout():
    g = torch.Generator(device="cuda").manual_seed(3)
    w = (torch.randn(32, 512, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    qw, s, b = oracle.q4_quantize(w)
    dev = lambda a, dt: torch.from_numpy(a.view(dt)).cuda()  # noqa: E731
    q, sb = ops.q4_from_mlx(dev(qw, np.int32), dev(s, np.int16).view(torch.bfloat16), dev(b, np.int16).view(torch.bfloat16))
    q2, sb2 = ops.quantize_q4(w)
    assert torch.equal(q, q2) and torch.equal(sb, sb2)
    np.testing.assert_array_equal(u32(q).reshape(-1), to_b200_q4(qw, s, b)[0])


@pytest.mark.parametrize("rows,K", [(16, 64), (64, 2880), (48, 256)])
@pytest.mark.parametrize("mult", [1.0, 256.0])
def test_quantize_mxfp4_bit_exact(rows, K, mult):
    g = torch.Generator(device="cuda").manual_seed(rows * 7 + K)
    w = (torch.randn(rows, K, generator=g, device="cuda") * 0.02 * mult).to(torch.bfloat16)
    w[0, :32] = 0
    q, sc = ops.quantize_mxfp4(w)
    qw, s = oracle.mxfp4_quantize(w)
    ref_q, ref_sc = to_b200_fp4(qw, s)
    np.testing.assert_array_equal(u32(q).reshape(-1), ref_q)
    np.testing.assert_array_equal(sc.cpu().numpy().reshape(-1), ref_sc)
    np.testing.assert_array_equal(ops.dequant_mxfp4(q, sc).cpu().numpy(), oracle.mxfp4_dequant(qw, s))
    if mult > 1:
        assert int(s.max()) >= 129  # the large-E8M0 regime of tests/test_mxfp4_large_scales.py


# ------------------------------------------------------------------ router
@pytest.mark.parametrize("E,k", [(8, 2), (16, 6), (32, 4), (60, 4), (64, 6), (128, 8), (256, 8), (128, 1), (512, 32),
                                 (1000, 8)])
@pytest.mark.parametrize("T", [1, 7, 18, 64, 300])
def test_router_bit_exact(E, k, T):
    g = torch.Generator(device="cuda").manual_seed(E * 131 + T + k)
    d = 256 if E >= 512 else 2048
    x = torch.randn(T, d, generator=g, device="cuda").to(torch.bfloat16)
    wg = (torch.randn(E, d, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    idx, wts, lg = ops.router(x, wg, k, return_logits=True)
    ref_lg = oracle.router_logits(x, wg)
    np.testing.assert_array_equal(lg.cpu().numpy(), ref_lg)           # bit-exact logits
    ref_i, ref_w = oracle.topk(ref_lg, k)
    np.testing.assert_array_equal(idx.cpu().numpy(), ref_i)           # bit-exact ids
    np.testing.assert_allclose(wts.cpu().numpy(), ref_w, rtol=2e-6, atol=1e-7)
    np.testing.assert_allclose(wts.sum(-1).cpu().numpy(), 1.0, atol=1e-5)
    # against the fp64 stock sequence: ids may differ only where fp32 rounding reorders a near-tie
    st_i, _, lg64 = oracle.router_stock(x, wg, k)
    for t in range(T):
        a, b = set(idx[t].tolist()), set(st_i[t].tolist())
        if a != b:
            gap = np.sort(lg64[t])[::-1]
            assert abs(gap[k - 1] - gap[k]) < 1e-4, (t, a ^ b)


_TILED_ROUTER_CHECK = """
import sys, numpy as np, torch
sys.path.insert(0, {root!r})
import oracle
from moelab_b200 import ops
for E, k, d in [(8, 2, 4096), (16, 6, 2048), (32, 4, 2880), (128, 8, 2048)]:
    for T in [1, 5, 18, 64]:
        g = torch.Generator(device="cuda").manual_seed(E + T)
        x = torch.randn(T, d, generator=g, device="cuda").to(torch.bfloat16)
        wg = (torch.randn(E, d, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
        b = torch.randn(E, generator=g, device="cuda").to(torch.bfloat16)
        idx, wts, lg = ops.router(x, wg, k, gate_b=b, return_logits=True)
        ref_lg = oracle.router_logits(x, wg, b)
        assert np.array_equal(lg.cpu().numpy(), ref_lg), (E, T)
        assert np.array_equal(idx.cpu().numpy(), oracle.topk(ref_lg, k)[0]), (E, T)
print("ok")
"""


@pytest.mark.parametrize("tw8_from", ["1000000", "1"])
def test_router_tiled_kernel_every_variant(tw8_from):
    """The register-tiled router (normally from T * E >= 16384) forced on for every T: 1, 2 and 4 experts per
    warp, 4 or 8 tokens per warp (8 is normally used from T = 512), partial token blocks, bias; bit-exact logits
    and ids."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, MOEB_ROUTER_TILED_T="1", MOEB_ROUTER_TW8_T=tw8_from)
    r = subprocess.run([sys.executable, "-c", _TILED_ROUTER_CHECK.format(root=root)], env=env, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stderr[-2000:]


@pytest.mark.parametrize("E,k", [(32, 4), (128, 8), (256, 8)])
@pytest.mark.parametrize("T", [517, 1029])
def test_router_bit_exact_large_T(E, k, T):
    """Large T (the register-tiled router with 8 tokens per warp, partial last token block): bit-exact logits and
    ids against the oracle."""
    g = torch.Generator(device="cuda").manual_seed(E * 7 + T)
    x = torch.randn(T, 2048, generator=g, device="cuda").to(torch.bfloat16)
    wg = (torch.randn(E, 2048, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    idx, wts, lg = ops.router(x, wg, k, return_logits=True)
    ref_lg = oracle.router_logits(x, wg)
    np.testing.assert_array_equal(lg.cpu().numpy(), ref_lg)
    ref_i, ref_w = oracle.topk(ref_lg, k)
    np.testing.assert_array_equal(idx.cpu().numpy(), ref_i)
    np.testing.assert_allclose(wts.cpu().numpy(), ref_w, rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("E,k", [(16, 6), (60, 4), (64, 6), (128, 8)])
@pytest.mark.parametrize("T", [1, 33])
def test_router_full_softmax_and_bias(E, k, T):
    g = torch.Generator(device="cuda").manual_seed(T + E)
    d = 512
    x = torch.randn(T, d, generator=g, device="cuda").to(torch.bfloat16)
    wg = (torch.randn(E, d, generator=g, device="cuda") * 0.05).to(torch.bfloat16)
    b = torch.randn(E, generator=g, device="cuda").to(torch.bfloat16)
    idx, wts, lg = ops.router(x, wg, k, gate_b=b, norm=False, scale=2.5, return_logits=True)
    ref_lg = oracle.router_logits(x, wg, b)
    np.testing.assert_array_equal(lg.cpu().numpy(), ref_lg)
    ref_i, ref_w = oracle.topk(ref_lg, k, norm=False, scale=2.5)
    np.testing.assert_array_equal(idx.cpu().numpy(), ref_i)
    np.testing.assert_allclose(wts.cpu().numpy(), ref_w, rtol=1e-5, atol=1e-7)


def test_router_ties_and_nonfinite():
    """All-tied logits -> k distinct ids, equal weights (reference tests/test_router.py:36-41); NaN / -inf
    rows -> k distinct in-range ids, finite ones first, zero weight on the rest (:73-86)."""
    d, E, k = 64, 64, 6
    x = torch.zeros(3, d, dtype=torch.bfloat16, device="cuda")
    wg = torch.zeros(E, d, dtype=torch.bfloat16, device="cuda")
    idx, wts = ops.router(x, wg, k)
    assert idx.tolist() == [list(range(k))] * 3
    np.testing.assert_allclose(wts.cpu().numpy(), 1 / k, atol=1e-6)
    # non-finite logits through the bias: row 1 keeps only experts 0..2 finite
    for bad in (float("nan"), float("-inf")):
        x = torch.zeros(2, d, dtype=torch.bfloat16, device="cuda")
        x[1, 0] = 1.0
        wg = torch.zeros(E, d, dtype=torch.bfloat16, device="cuda")
        wg[:3, 0] = torch.tensor([0.5, 0.25, 0.125])
        bias = torch.full((E,), bad, dtype=torch.bfloat16, device="cuda")
        bias[:3] = 0
        idx, wts = ops.router(x, wg, k, gate_b=bias)
        i = idx.cpu().numpy()
        assert ((i >= 0) & (i < E)).all()
        for t in range(2):
            assert len(set(i[t].tolist())) == k
        assert set(i[1, :3].tolist()) == {0, 1, 2}
        np.testing.assert_allclose(wts[1].sum().item(), 1.0, atol=1e-5)
        assert np.allclose(wts[1, 3:].cpu().numpy(), 0)
        ri, rw = oracle.topk(oracle.router_logits(x, wg, bias), k)
        np.testing.assert_array_equal(i, ri)


# ------------------------------------------------------------------ experts
SMALL = MoEShape("t", d=128, f=256, E=8, k=2)
CASES = [(1, "uniform"), (7, "uniform"), (33, "zipf"), (100, "uniform"), (64, "one_hot")]


@pytest.mark.parametrize("T,routing", CASES)
def test_variant_small(mod, policy, T, routing):
    p, w, x, idx, wts = problem_tensors(SMALL, T, routing)
    st = mod.prepare(*w)
    y = mod.run(st, x, idx, wts)
    assert y.shape == x.shape and y.dtype == x.dtype
    assert_close(y, ref_from_state(mod, st, x, idx, wts), what=(T, routing))


@pytest.mark.parametrize("T", [1, 2, 3, 4, 5, 7, 8, 9, 15, 17, 31, 63, 65, 127, 129, 257])
def test_dispatch_boundaries(mod, policy, T):
    sh = MoEShape("q", d=256, f=384, E=16, k=4)
    p, w, x, idx, wts = problem_tensors(sh, T, "zipf", seed=T)
    st = mod.prepare(*w)
    assert_close(mod.run(st, x, idx, wts), ref_from_state(mod, st, x, idx, wts), what=T)


SHAPES = [MoEShape("d192", d=192, f=256, E=8, k=2), MoEShape("f320", d=256, f=320, E=8, k=2),
          MoEShape("odd", d=320, f=448, E=8, k=3), MoEShape("k1", d=128, f=256, E=8, k=1),
          MoEShape("kE", d=128, f=256, E=4, k=4), MoEShape("E1", d=128, f=256, E=1, k=1)]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: s.name)
@pytest.mark.parametrize("T", [1, 2, 6, 33])
def test_shapes(mod, policy, shape, T):
    p, w, x, idx, wts = problem_tensors(shape, T)
    st = mod.prepare(*w)
    assert_close(mod.run(st, x, idx, wts), ref_from_state(mod, st, x, idx, wts), what=(shape.name, T))


@pytest.mark.parametrize("T", [1, 4, 16])
def test_zero_and_unnormalized_weights(mod, policy, T):
    sh = MoEShape("w", d=256, f=256, E=8, k=4)
    rng = np.random.default_rng(T)
    wts = rng.random((T, 4)).astype(np.float32) * 3
    wts[:, 1] = 0
    wts[0] = 0
    p, w, x, idx, _ = problem_tensors(sh, T)
    wt = torch.from_numpy(wts).cuda()
    st = mod.prepare(*w)
    y = mod.run(st, x, idx, wt)
    assert_close(y, ref_from_state(mod, st, x, idx, wt))
    assert float(y[0].float().abs().max()) == 0.0  # all-zero weights -> exactly zero output


@pytest.mark.parametrize("T", [2, 8, 32])
def test_all_tokens_one_expert_set(mod, policy, T):
    sh = MoEShape("o", d=256, f=256, E=16, k=4)
    p, w, x, _, wts = problem_tensors(sh, T)
    idx = torch.tensor([[3, 7, 0, 15]] * T, dtype=torch.int32, device="cuda")
    st = mod.prepare(*w)
    assert_close(mod.run(st, x, idx, wts), ref_from_state(mod, st, x, idx, wts))


@pytest.mark.parametrize("T", [1, 8])
def test_permutation_invariance(mod, policy, T):
    sh = MoEShape("p", d=256, f=256, E=16, k=4)
    p, w, x, idx, wts = problem_tensors(sh, T, seed=1)
    st = mod.prepare(*w)
    perm = torch.tensor([2, 0, 3, 1], device="cuda")
    y1 = mod.run(st, x, idx, wts).float()
    y2 = mod.run(st, x, idx[:, perm].contiguous(), wts[:, perm].contiguous()).float()
    assert ((y1 - y2).norm() / y1.norm()).item() < 1e-2


def test_batch_consistency(mod, policy):
    sh = MoEShape("b", d=256, f=256, E=16, k=4)
    p, w, x, idx, wts = problem_tensors(sh, 16, seed=2)
    st = mod.prepare(*w)
    full = mod.run(st, x, idx, wts).float()
    for t in (0, 5, 15):
        one = mod.run(st, x[t:t + 1].contiguous(), idx[t:t + 1].contiguous(), wts[t:t + 1].contiguous()).float()
        assert ((one - full[t:t + 1]).norm() / full[t:t + 1].norm()).item() < 1e-2


def test_large_activations(mod, policy):
    sh = MoEShape("big", d=256, f=256, E=8, k=2)
    p, w, x, idx, wts = problem_tensors(sh, 8, seed=3)
    x = (x.float() * 100).to(torch.bfloat16)
    st = mod.prepare(*w)
    assert_close(mod.run(st, x, idx, wts), ref_from_state(mod, st, x, idx, wts))


@pytest.mark.parametrize("T,routing", [(1, "uniform"), (3, "uniform"), (16, "one_hot"), (32, "uniform")])
def test_tiny_affine_scales(mod, policy, T, routing):
    sh = MoEShape("tiny-scales", d=256, f=256, E=8, k=2)
    p, w, x, idx, wts = problem_tensors(sh, T, routing, seed=T)
    w = [(t.float() * 1e-6).to(torch.bfloat16) for t in w]
    x = (x.float() * 1e6).to(torch.bfloat16)
    st = mod.prepare(*w)
    assert_close(mod.run(st, x, idx, wts), ref_from_state(mod, st, x, idx, wts))


@pytest.mark.parametrize("act", [0, 1])
@pytest.mark.parametrize("T", [1, 3, 17, 64])
def test_activations(mod, policy, act, T):
    sh = MoEShape("mma", d=256, f=384, E=16, k=4)
    p, w, x, idx, wts = problem_tensors(sh, T, "zipf", seed=T)
    st = mod.prepare(*w)
    y = mod.run(st, x, idx, wts, act)
    e = assert_close(y, ref_from_state(mod, st, x, idx, wts, act=act))
    other = oracle.error_metrics(y.float().cpu().numpy(), ref_from_state(mod, st, x, idx, wts, act=1 - act))
    assert other["rel_fro"] > 3 * e["rel_fro"], "activation did not reach the kernel"


def test_fp32_activations(mod, policy):
    sh = MoEShape("b", d=2048, f=1408, E=16, k=6)
    p, w, x, idx, wts = problem_tensors(sh, 32)
    x32 = torch.from_numpy(p["x"]).cuda()
    st = mod.prepare(*w)
    y = mod.run(st, x32, idx, wts)
    assert y.dtype == torch.float32
    ref = ref_from_state(mod, st, x32, idx, wts)
    assert oracle.error_metrics(y.cpu().numpy(), ref)["rel_fro"] < 1e-2


def test_run_slots(mod, policy):
    sh = MoEShape("small", d=256, f=320, E=8, k=2)
    p, w, x, idx, wts = problem_tensors(sh, 1, seed=7)
    st = mod.prepare(*w)
    ys = mod.run_slots(st, x, idx)
    assert ys.shape == (sh.k, sh.d)
    for j in range(sh.k):
        ref = ref_from_state(mod, st, x, idx[:, j:j + 1].contiguous(), torch.ones(1, 1, device="cuda"))
        assert_close(ys[j:j + 1], ref, what=j)


def test_deterministic(mod, policy):
    sh = MoEShape("q", d=512, f=384, E=16, k=4)
    p, w, x, idx, wts = problem_tensors(sh, 77, "zipf", seed=5)
    st = mod.prepare(*w)
    y1, y2 = mod.run(st, x, idx, wts), mod.run(st, x, idx, wts)
    assert torch.equal(y1, y2)


# ------------------------------------------------------------------ the layer call (router + experts)
@pytest.mark.parametrize("T", [1, 4, 32])
def test_layer_qwen3_shape(mod, policy, T):
    """Qwen3-30B-A3B-shaped layer, N(0, 0.02) weights, gate N(0, 0.02), x ~ N(0, 1)."""
    sh = MoEShape("qwen3-30b-a3b", d=2048, f=768, E=128, k=8)
    g = torch.Generator(device="cuda").manual_seed(1234 + T)
    mk = lambda *s: (torch.randn(*s, generator=g, device="cuda") * 0.02).to(torch.bfloat16)  # noqa: E731
    w = [mk(sh.E, sh.f, sh.d), mk(sh.E, sh.f, sh.d), mk(sh.E, sh.d, sh.f)]
    gate = mk(sh.E, sh.d)
    x = torch.randn(T, sh.d, generator=g, device="cuda").to(torch.bfloat16)
    st = mod.prepare(*w)
    y, idx, wts = mod.layer(st, x, gate, sh.k, return_routing=True)
    ri, rw = oracle.router(x, gate, sh.k)
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    np.testing.assert_allclose(wts.cpu().numpy(), rw, rtol=2e-6, atol=1e-7)
    assert_close(y, ref_from_state(mod, st, x, idx, wts), what=T)
    # residual fused into the combine: y2 = bf16(x + moe(x))
    y2 = mod.layer(st, x, gate, sh.k, residual=x)
    assert_close(y2, ref_from_state(mod, st, x, idx, wts) + x.float().cpu().numpy())


def test_rows_not_multiple_of_16_rejected():
    w = torch.zeros(8, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ops._lib.MoebError, match="multiple of 16"):
        ops.quantize_q4(w)


def test_invalid_expert_ids_flagged(mod):
    sh = MoEShape("t", d=128, f=256, E=8, k=2)
    for pol in (ops.POLICY_SLOTS, ops.POLICY_TILES8):
        mod.POLICY = pol
        try:
            p, w, x, idx, wts = problem_tensors(sh, 5)
            st = mod.prepare(*w)
            bad = idx.clone()
            bad[2, 1] = 99
            bad[4, 0] = -3
            y = mod.run(st, x, bad, wts)
            assert st["ws"].read_error() & ops._lib.DEVERR_EXPERT_ID
            assert st["ws"].read_error() == 0  # cleared
            w2 = wts.clone()
            w2[2, 1] = 0
            w2[4, 0] = 0
            ok = torch.where(bad < 0, 0, torch.where(bad >= sh.E, 0, bad)).to(torch.int32)
            assert_close(y, ref_from_state(mod, st, x, ok, w2))
        finally:
            mod.POLICY = None
