"""moeb_experts_q4_static: the expert forward for callers that cannot allocate device memory (a host runtime that
owns the device heap, or a path with a fixed memory plan). Its scratch is a static device array inside the
library, so the call takes only inputs and the output. This file sorts last so a stop-at-first-failure run has
already run every other test; it must pass both on its own in a fresh process and after the rest.

Checked through the C ABI against moeb_experts_q4 (which uses a caller-provided workspace) and against the fp64
oracle on the layer's own dequantised weights: calls in a row with different inputs, a large call followed by a
small one (the array keeps the last call's contents), the tcgen05 and decode paths, a residual, and a size beyond
the static scratch, which is rejected with a clear error.
"""
import pytest
import torch

import oracle
from helpers import Q4_VARIANT, assert_close, load_variant, problem_tensors
from moelab_b200 import _lib, ops
from moelab_b200.shapes import MoEShape

pytestmark = pytest.mark.gpu

SHAPE = MoEShape("qwen3-like", d=2048, f=768, E=128, k=8)


def _call_static(st, x, idx, wts, act=0, policy=0, residual=None):
    T, d = x.shape
    k = idx.shape[1]
    y = torch.empty_like(x)
    p = ops._p
    _lib.call("moeb_experts_q4_static", p(x), *ops._expert_ptrs(st), p(idx), p(wts), T, d, st["f"], st["E"], k,
              act, policy, p(residual), p(y), ops._stream())
    return y


@pytest.fixture(scope="module")
def layer():
    mod = load_variant(Q4_VARIANT)
    _, w, _, _, _ = problem_tensors(SHAPE, 1, seed=11)
    st = mod.prepare(*w)
    mod._ws(st, SHAPE.k)
    deq = [t.cpu().numpy() for t in mod.dequant(st)]  # the layer's own dequantised weights, once
    return st, deq


def _oracle(deq, x, idx, wts):
    return oracle.moe_forward(x.float().cpu().numpy(), *deq, idx.cpu().numpy(), wts.cpu().numpy())


# (T, seed) sequences: the second call of each pair reuses the array the first one left behind; 32 -> 4 is the
# large-then-small order (a smaller layout over stale contents of a larger one)
@pytest.mark.parametrize("policy,calls", [
    (ops.POLICY_AUTO, [(4, 1), (32, 2), (4, 3)]),
    (ops.POLICY_AUTO, [(32, 4), (1, 5), (2, 6)]),
    (ops.POLICY_SLOTS, [(2, 7), (1, 8)]),
    (ops.POLICY_TILES8, [(32, 9), (4, 10)]),
    (ops.POLICY_TILES16_RING, [(64, 11), (8, 12)]),
    (ops.POLICY_TC, [(64, 13), (16, 14)]),
    (ops.POLICY_DECODE, [(1, 15), (2, 16)]),
])
def test_static_scratch_matches_workspace_path_and_oracle(layer, policy, calls):
    st, deq = layer
    for call, (T, seed) in enumerate(calls):
        _, _, x, idx, wts = problem_tensors(SHAPE, T, "uniform", seed=seed)
        ref = ops.experts_q4(st, x, idx, wts, policy=policy)
        y = _call_static(st, x, idx, wts, policy=policy)
        torch.cuda.synchronize()
        # against the workspace path (same kernels, same inputs): within the tests' bf16 tolerance
        assert_close(y, ref.float().cpu().numpy(), what=("vs workspace path", policy, call, T))
        # against the oracle on the layer's dequantised weights
        assert_close(y, _oracle(deq, x, idx, wts), what=("vs oracle", policy, call, T))
    assert st["ws"].read_error() == 0


def test_static_scratch_residual(layer):
    st, deq = layer
    for T, seed in [(32, 21), (1, 22)]:
        _, _, x, idx, wts = problem_tensors(SHAPE, T, "uniform", seed=seed)
        r = torch.randn(T, SHAPE.d, generator=torch.Generator(device="cuda").manual_seed(seed),
                        device="cuda").to(torch.bfloat16)
        y = _call_static(st, x, idx, wts, residual=r)
        torch.cuda.synchronize()
        ref = _oracle(deq, x, idx, wts) + r.float().cpu().numpy()
        assert_close(y, ref, what=("residual", T))


def test_static_scratch_rejects_oversize(layer):
    st, _ = layer
    T = 4096
    assert _lib.load().moeb_workspace_bytes(T, SHAPE.d, SHAPE.f, SHAPE.E, SHAPE.k) > (16 << 20)
    x = torch.zeros(T, SHAPE.d, dtype=torch.bfloat16, device="cuda")
    idx = torch.zeros(T, SHAPE.k, dtype=torch.int32, device="cuda")
    wts = torch.zeros(T, SHAPE.k, dtype=torch.float32, device="cuda")
    with pytest.raises(_lib.MoebError, match="static scratch holds"):
        _call_static(st, x, idx, wts)


def test_static_scratch_error_bits(layer):
    """An expert id outside [0, E) is computed on expert 0 with weight 0 and recorded as MOEB_DEVERR_EXPERT_ID in the
    static array's error word; the read returns it once and clears it, and the next clean call reads 0."""
    import ctypes
    st, deq = layer
    _, _, x, idx, wts = problem_tensors(SHAPE, 4, "uniform", seed=31)

    def read():
        v = ctypes.c_uint(0)
        _lib.call("moeb_experts_q4_static_read_error", ctypes.byref(v), ops._stream())
        return v.value

    bad = idx.clone()
    bad[1, 2] = SHAPE.E
    y = _call_static(st, x, bad, wts)
    assert read() == _lib.DEVERR_EXPERT_ID
    assert read() == 0
    ok_w = wts.clone()
    ok_w[1, 2] = 0.0
    ok_i = idx.clone()
    ok_i[1, 2] = 0
    assert_close(y, _oracle(deq, x, ok_i, ok_w), what="invalid id weighted 0")
    _call_static(st, x, idx, wts)
    assert read() == 0
