"""Layer parity on the BASELINE configurations not covered elsewhere (Qwen3-30B int4 is in test_gpu_q4, the
gpt-oss-20b MXFP4 layer in test_gpu_mxfp4):
  - DeepSeek-V2-Lite int4: Zipf(1.1)-biased greedy router (full-softmax weights), 2 always-on shared experts;
  - Qwen3-235B-A22B int4 layer, T up to 2048 (the compute-bound end);
  - Mixtral-8x7B in int4 and MXFP4 under uniform, one-hot and round-robin routing, T from 1 to 4096.
Router ids are bit-exact against the oracle; outputs are checked against the fp64 oracle where it finishes in
seconds, and against a plain PyTorch fp32 reference on the GPU (dequantised weights) at the large sizes."""
import numpy as np
import pytest
import torch

import oracle
from helpers import assert_close, ref_from_state
from moelab_b200 import ops
from moelab_b200.problem import make_routing, zipf_bias
from moelab_b200.variants.cuda import b200_mxfp4_moe, b200_q4_moe

pytestmark = pytest.mark.gpu


def _w(E, f, d, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    mk = lambda *s: (torch.randn(*s, generator=g, device="cuda") * 0.02).to(torch.bfloat16)  # noqa: E731
    return [mk(E, f, d), mk(E, f, d), mk(E, d, f)], mk


@torch.no_grad()
def torch_ref(v, st, x, idx, wts, deq=None):
    """fp32 PyTorch reference on the GPU: loop over the used experts of the variant's dequantised weights."""
    torch.backends.cuda.matmul.allow_tf32 = False
    wg, wu, wd = deq if deq is not None else v.dequant(st)
    x32 = x.float()
    y = torch.zeros_like(x32)
    for e in idx.unique().tolist():
        t, j = (idx == e).nonzero(as_tuple=True)
        g, u = x32[t] @ wg[e].T, x32[t] @ wu[e].T
        h = torch.nn.functional.silu(g) * u
        y.index_add_(0, t, (h @ wd[e].T) * wts[t, j, None])
    return y.cpu().numpy()


# ------------------------------------------------------------------ DeepSeek-V2-Lite
@pytest.mark.parametrize("T", [1, 16, 64, 256])
def test_deepseek_v2_lite_layer(T):
    d, f, E, k, ns = 2048, 1408, 64, 6, 2
    w, mk = _w(E, f, d, seed=T)
    sw = [mk(ns * f, d), mk(ns * f, d), mk(d, ns * f)]
    st = b200_q4_moe.prepare_shared(*w, *sw)
    gate = mk(E, d)
    gb = torch.from_numpy(zipf_bias(E, 1.1, seed=7)).to("cuda", torch.bfloat16)
    x = torch.randn(T, d, generator=torch.Generator(device="cuda").manual_seed(T), device="cuda").to(torch.bfloat16)
    y, idx, wts = b200_q4_moe.layer(st, x, gate, k, gate_b=gb, norm=False, rscale=1.0, residual=x,
                                    return_routing=True)
    ri, rw = oracle.router(x, gate, k, bias=gb, norm=False, scale=1.0)
    np.testing.assert_array_equal(idx[:, :k].cpu().numpy(), ri)
    np.testing.assert_allclose(wts[:, :k].cpu().numpy(), rw, rtol=2e-6, atol=1e-7)
    assert (idx[:, k:].cpu().numpy() == np.arange(E, E + ns)).all() and (wts[:, k:] == 1).all()
    if T >= 16:  # the Zipf bias makes a few experts hot
        counts = np.bincount(ri.reshape(-1), minlength=E)
        assert counts.max() >= 3 * counts.mean()
    ref = ref_from_state(b200_q4_moe, st, x, idx, wts)
    assert_close(y, ref + x.float().cpu().numpy(), what=T)


def test_shared_split_equals_dense_shared_mlp():
    """The shared MLP split into n experts of width f equals the dense MLP of width n*f (one token, fp64)."""
    d, f, E, k, ns = 256, 128, 8, 2, 2
    w, mk = _w(E, f, d, seed=1)
    sw = [mk(ns * f, d), mk(ns * f, d), mk(d, ns * f)]
    st = b200_q4_moe.prepare_shared(*w, *sw)
    wg, wu, wd = (t.cpu().numpy().astype(np.float64) for t in b200_q4_moe.dequant(st))
    x = torch.randn(3, d).to(torch.bfloat16)
    xs = x.float().numpy().astype(np.float64)
    # dense shared MLP rebuilt from the split experts E, E+1 (the quantizer works per 64-group along K, so the
    # split weights are the dense MLP's rows / columns)
    g = xs @ np.concatenate([wg[E], wg[E + 1]]).T
    u = xs @ np.concatenate([wu[E], wu[E + 1]]).T
    h = g / (1 + np.exp(-g)) * u
    dense = h @ np.concatenate([wd[E], wd[E + 1]], axis=1).T
    idx = np.tile(np.array([[E, E + 1]], np.int32), (3, 1))
    split = oracle.moe_forward(xs.astype(np.float32), wg, wu, wd, idx, np.ones((3, 2), np.float32))
    np.testing.assert_allclose(split, dense, rtol=1e-5, atol=1e-6)


# ------------------------------------------------------------------ Qwen3-235B-A22B
@pytest.mark.parametrize("T", [1, 32, 256, 2048])
def test_qwen3_235b_layer(T):
    d, f, E, k = 4096, 1536, 128, 8
    w, mk = _w(E, f, d, seed=235 + T)
    st = b200_q4_moe.prepare(*w)
    del w
    gate = mk(E, d)
    x = torch.randn(T, d, generator=torch.Generator(device="cuda").manual_seed(T), device="cuda").to(torch.bfloat16)
    y, idx, wts = b200_q4_moe.layer(st, x, gate, k, return_routing=True)
    ri, _ = oracle.router(x, gate, k)
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    ref = ref_from_state(b200_q4_moe, st, x, idx, wts) if T == 1 else torch_ref(b200_q4_moe, st, x, idx, wts)
    assert_close(y, ref, what=T)


# ------------------------------------------------------------------ Mixtral-8x7B
MIXTRAL_T = [1, 2, 4, 8, 16, 32, 64, 128, 256, 512, 1024, 2048, 4096]  # every power of two (BASELINE)


@pytest.fixture(scope="module")
def mixtral():
    d, f, E = 4096, 14336, 8
    w, _ = _w(E, f, d, seed=87)
    states = {"q4": b200_q4_moe.prepare(*w), "mxfp4": b200_mxfp4_moe.prepare(*w)}
    del w
    deq = {"q4": b200_q4_moe.dequant(states["q4"]), "mxfp4": b200_mxfp4_moe.dequant(states["mxfp4"])}
    torch.cuda.empty_cache()
    return states, deq


@pytest.mark.parametrize("fmt", ["q4", "mxfp4"])
@pytest.mark.parametrize("routing", ["uniform", "one_hot", "round_robin"])
@pytest.mark.parametrize("T", MIXTRAL_T)
def test_mixtral(mixtral, fmt, routing, T):
    v = b200_mxfp4_moe if fmt == "mxfp4" else b200_q4_moe
    st, deq = mixtral[0][fmt], mixtral[1][fmt]
    idx, wts = make_routing(T, 8, 2, routing, np.random.default_rng(T))
    if routing == "one_hot":
        assert (idx == [0, 1]).all()
    x = torch.randn(T, 4096, generator=torch.Generator(device="cuda").manual_seed(T), device="cuda").to(torch.bfloat16)
    it, wt = torch.from_numpy(idx).cuda(), torch.from_numpy(wts).cuda()
    y = v.run(st, x, it, wt)
    if T == 1 and routing == "uniform":  # the fp64 oracle once per format
        ref = oracle.moe_forward(x.float().cpu().numpy(), *(t.cpu().numpy() for t in deq), idx, wts)
    else:
        ref = torch_ref(v, st, x, it, wt, deq)
    assert_close(y, ref, what=(fmt, routing, T))


# ------------------------------------------------------------------ tensor-core policy (tcgen05, tiles of 32..256)
# E = 8, k = 2: T = 1, 3, 64 -> tiles of 32 slots, 200 -> 64, 300 -> 128, 480 / 513 -> 192, 600 -> 256
@pytest.mark.parametrize("T,routing", [(1, "uniform"), (3, "uniform"), (64, "uniform"), (200, "uniform"),
                                       (200, "one_hot"), (300, "uniform"), (300, "one_hot"), (480, "uniform"),
                                       (480, "one_hot"), (513, "zipf"), (600, "uniform"), (600, "one_hot")])
def test_tc_small_vs_oracle(T, routing):
    """tcgen05 tiles of every size: partial tiles, several tiles per expert, empty experts."""
    from helpers import problem_tensors
    from moelab_b200.shapes import MoEShape
    sh = MoEShape("tc", d=256, f=384, E=8, k=2)
    p, w, x, idx, wts = problem_tensors(sh, T, routing, seed=T)
    st = b200_q4_moe.prepare(*w)
    b200_q4_moe._ws(st, sh.k)
    y = ops.experts(st, x, idx, wts, policy=ops.POLICY_TC)
    assert_close(y, ref_from_state(b200_q4_moe, st, x, idx, wts), what=(T, routing))
    assert st["ws"].read_error() == 0
    # the same through the layer call with a fused residual
    gate = (torch.randn(sh.E, sh.d, device="cuda") * 0.02).to(torch.bfloat16)
    b200_q4_moe.POLICY = ops.POLICY_TC
    try:
        y2, i2, w2 = b200_q4_moe.layer(st, x, gate, sh.k, residual=x, return_routing=True)
    finally:
        b200_q4_moe.POLICY = None
    assert_close(y2, ref_from_state(b200_q4_moe, st, x, i2, w2) + x.float().cpu().numpy())


@pytest.mark.parametrize("T", [256, 2048])
def test_tc_qwen3_235b(T):
    d, f, E, k = 4096, 1536, 128, 8
    w, mk = _w(E, f, d, seed=900 + T)
    st = b200_q4_moe.prepare(*w)
    del w
    b200_q4_moe._ws(st, k)
    x = torch.randn(T, d, generator=torch.Generator(device="cuda").manual_seed(T), device="cuda").to(torch.bfloat16)
    idx, wts = make_routing(T, E, k, "uniform", np.random.default_rng(T))
    it, wt = torch.from_numpy(idx).cuda(), torch.from_numpy(wts).cuda()
    y = ops.experts(st, x, it, wt, policy=ops.POLICY_TC)
    assert_close(y, torch_ref(b200_q4_moe, st, x, it, wt), what=T)


@pytest.mark.parametrize("routing", ["uniform", "one_hot", "round_robin"])
@pytest.mark.parametrize("T", [256, 1024, 4096])
def test_tc_mixtral(mixtral, routing, T):
    st, deq = mixtral[0]["q4"], mixtral[1]["q4"]
    idx, wts = make_routing(T, 8, 2, routing, np.random.default_rng(T))
    x = torch.randn(T, 4096, generator=torch.Generator(device="cuda").manual_seed(T), device="cuda").to(torch.bfloat16)
    it, wt = torch.from_numpy(idx).cuda(), torch.from_numpy(wts).cuda()
    b200_q4_moe._ws(st, 2)
    y = ops.experts(st, x, it, wt, policy=ops.POLICY_TC)
    assert_close(y, torch_ref(b200_q4_moe, st, x, it, wt, deq), what=(routing, T))


@pytest.mark.parametrize("T", [256, 1024])
def test_tc_mixtral_mxfp4(mixtral, T):
    st, deq = mixtral[0]["mxfp4"], mixtral[1]["mxfp4"]
    idx, wts = make_routing(T, 8, 2, "uniform", np.random.default_rng(T))
    x = torch.randn(T, 4096, generator=torch.Generator(device="cuda").manual_seed(T), device="cuda").to(torch.bfloat16)
    it, wt = torch.from_numpy(idx).cuda(), torch.from_numpy(wts).cuda()
    b200_mxfp4_moe._ws(st, 2)
    y = ops.experts(st, x, it, wt, policy=ops.POLICY_TC)
    assert_close(y, torch_ref(b200_mxfp4_moe, st, x, it, wt, deq), what=T)


@pytest.mark.parametrize("T", [3, 200, 300, 480, 600])
def test_tc_small_mxfp4(T):
    """MXFP4 on the tensor cores (E2M1 x 2^(S-127) dequantized exactly to bf16) for each tile size."""
    from helpers import problem_tensors
    from moelab_b200.shapes import MoEShape
    sh = MoEShape("tc", d=256, f=384, E=8, k=2)
    p, w, x, idx, wts = problem_tensors(sh, T, "uniform", seed=T)
    st = b200_mxfp4_moe.prepare(*w)
    b200_mxfp4_moe._ws(st, sh.k)
    y = ops.experts(st, x, idx, wts, policy=ops.POLICY_TC)
    assert_close(y, ref_from_state(b200_mxfp4_moe, st, x, idx, wts), what=T)
    assert st["ws"].read_error() == 0


def test_tc_rejects_unsupported_shapes():
    from moelab_b200.shapes import MoEShape
    from helpers import problem_tensors
    sh = MoEShape("odd", d=192, f=256, E=4, k=2)
    p, w, x, idx, wts = problem_tensors(sh, 8)
    st = b200_q4_moe.prepare(*w)
    b200_q4_moe._ws(st, 2)
    with pytest.raises(ops._lib.MoebError, match="multiples of 128"):
        ops.experts(st, x, idx, wts, policy=ops.POLICY_TC)


# ------------------------------------------------------------------ Qwen3-30B-A3B on recorded routing traces
@pytest.fixture(scope="module")
def qwen3_trace_layer():
    from moelab_b200.shapes import MoEShape
    sh = MoEShape("qwen3-30b-a3b", d=2048, f=768, E=128, k=8)
    w, _ = _w(sh.E, sh.f, sh.d, seed=301)
    st = b200_q4_moe.prepare(*w)
    del w
    deq = b200_q4_moe.dequant(st)
    return sh, st, deq


@pytest.mark.parametrize("T", [1, 8, 16, 32])
@pytest.mark.parametrize("seed", [0, 5, 11])
@pytest.mark.parametrize("policy", [None, ops.POLICY_DECODE, ops.POLICY_TILES8_RING])
def test_qwen3_trace_routing(qwen3_trace_layer, T, seed, policy, monkeypatch):
    """The reference's trace inputs (moelab/problem.py:38-50 via moelab/torch_backend.py:50-54: recorded
    Qwen3-30B-A3B routing windows, skewed and repeated experts) through the harness contract run(); the ids are
    the reference's own draws (tests/golden/trace_qwen3.npz)."""
    from moelab_b200.problem import make_inputs
    sh, st, deq = qwen3_trace_layer
    monkeypatch.setattr(b200_q4_moe, "POLICY", policy)
    x, idx, wts = make_inputs(sh.d, sh.E, sh.k, T, "trace", seed)
    xt = torch.from_numpy(x).to("cuda", torch.bfloat16)
    it, wt = torch.from_numpy(idx).cuda(), torch.from_numpy(wts).cuda()
    b200_q4_moe._ws(st, sh.k)
    y = b200_q4_moe.run(st, xt, it, wt)
    assert_close(y, torch_ref(b200_q4_moe, st, xt, it, wt, deq), what=(T, seed, policy))
    assert st["ws"].read_error() == 0
