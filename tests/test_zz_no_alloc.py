"""moeb_experts_q4_static: the expert forward for callers that cannot allocate device memory (a host runtime that
owns the device heap, or a path with a fixed memory plan). Its scratch is a static device array inside the
library, so the call takes only inputs and the output. This file sorts last so a stop-at-first-failure run has
already run every other test; it must pass both on its own in a fresh process and after the rest.

Checked through the C ABI against moeb_experts_q4 (which uses a caller-provided workspace): two calls in a row
with different inputs, and a size beyond the static scratch is rejected with a clear error.
"""
import ctypes

import pytest
import torch

from helpers import Q4_VARIANT, load_variant, problem_tensors
from moelab_b200 import _lib, ops
from moelab_b200.shapes import MoEShape

pytestmark = pytest.mark.gpu


def _call_static(st, x, idx, wts, act=0, policy=0):
    T, d = x.shape
    k = idx.shape[1]
    y = torch.empty_like(x)
    p = ops._p
    _lib.call("moeb_experts_q4_static", p(x), *ops._expert_ptrs(st), p(idx), p(wts), T, d, st["f"], st["E"], k,
              act, policy, None, p(y), ops._stream())
    return y


@pytest.mark.parametrize("policy", [ops.POLICY_AUTO, ops.POLICY_SLOTS, ops.POLICY_TILES8])
def test_static_scratch_matches_workspace_path(policy):
    mod = load_variant(Q4_VARIANT)
    sh = MoEShape("qwen3-like", d=2048, f=768, E=128, k=8)
    _, w, _, _, _ = problem_tensors(MoEShape("w", d=sh.d, f=sh.f, E=sh.E, k=sh.k), 1, seed=11)
    st = mod.prepare(*w)
    mod._ws(st, sh.k)
    for call, (T, seed) in enumerate([(4, 1), (32, 2)]):  # two calls in a row share the static array
        _, _, x, idx, wts = problem_tensors(sh, T, "uniform", seed=seed)
        ref = ops.experts_q4(st, x, idx, wts, policy=policy)
        y = _call_static(st, x, idx, wts, policy=policy)
        torch.cuda.synchronize()
        rel = ((y.float() - ref.float()).norm() / ref.float().norm()).item()
        assert rel < 1e-2, (call, rel)
        rowmax = ref.float().abs().amax(dim=1, keepdim=True)
        assert bool(((y.float() - ref.float()).abs() <= 1e-2 * rowmax + 1e-6).all()), call


def test_static_scratch_rejects_oversize():
    mod = load_variant(Q4_VARIANT)
    sh = MoEShape("big", d=2048, f=768, E=128, k=8)
    _, w, _, _, _ = problem_tensors(MoEShape("w", d=sh.d, f=sh.f, E=sh.E, k=sh.k), 1, seed=12)
    st = mod.prepare(*w)
    T = 4096
    assert _lib.load().moeb_workspace_bytes(T, sh.d, sh.f, sh.E, sh.k) > (16 << 20)
    x = torch.zeros(T, sh.d, dtype=torch.bfloat16, device="cuda")
    idx = torch.zeros(T, sh.k, dtype=torch.int32, device="cuda")
    wts = torch.zeros(T, sh.k, dtype=torch.float32, device="cuda")
    with pytest.raises(_lib.MoebError, match="static scratch holds"):
        _call_static(st, x, idx, wts)
