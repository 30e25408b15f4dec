"""Shared test helpers: layout conversion for bit-exact checks, oracle references, error bounds."""
import os

import numpy as np
import torch

import oracle
from moelab_b200.problem import ROWREL_TOL, make_problem

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
Q4_VARIANT = os.path.join(ROOT, "moelab_b200", "variants", "cuda", "b200_q4_moe.py")
TOL_BF16 = 1e-2  # rel_fro bound used by the reference's bf16 tests (mlx_backend.py:163); outputs also <= ROWREL_TOL


def interleave_words(nat):
    """natural nibble order (element i at nibble i) -> B200 order (pairs (2p, 2p+1) at nibbles p, p+4)."""
    nat = np.asarray(nat, np.uint32)
    out = np.zeros_like(nat)
    for p in range(4):
        out |= ((nat >> (8 * p)) & 0xF) << (4 * p)
        out |= ((nat >> (8 * p + 4)) & 0xF) << (4 * (p + 4))
    return out


def deinterleave_words(w):
    w = np.asarray(w, np.uint32)
    out = np.zeros_like(w)
    for p in range(4):
        out |= ((w >> (4 * p)) & 0xF) << (8 * p)
        out |= ((w >> (4 * (p + 4))) & 0xF) << (8 * p + 4)
    return out


def fm_q_index(rows, K):
    """Flat word index in the fragment-major layout of every (row, k-word j) of a natural [rows, K/8] array."""
    r = np.arange(rows)[:, None]
    j = np.arange(K // 8)[None, :]
    rb, rr, g, jj = r // 16, r % 16, j // 8, j % 8
    lane = (rr % 8) * 4 + jj // 2
    return ((rb * (K // 64) + g) * 32 + lane) * 4 + (rr // 8) * 2 + (jj % 2)


def to_b200_q4(qw, s, b):
    """oracle (natural mlx) int4 state -> flat B200 arrays (q words, sb words)."""
    rows, K = qw.shape[0], qw.shape[1] * 8
    q = np.zeros(rows * K // 8, np.uint32)
    q[fm_q_index(rows, K)] = interleave_words(qw)
    r = np.arange(rows)[:, None]
    g = np.arange(K // 64)[None, :]
    sbi = ((r // 16 * (K // 64) + g) * 8 + (r % 16) % 8) * 2 + (r % 16) // 8
    sb = np.zeros(rows * K // 64, np.uint32)
    sb[sbi] = s.astype(np.uint32) | (b.astype(np.uint32) << 16)
    return q, sb


def to_b200_fp4(qw, sc):
    rows, K = qw.shape[0], qw.shape[1] * 8
    q = np.zeros(rows * K // 8, np.uint32)
    q[fm_q_index(rows, K)] = interleave_words(qw)
    r = np.arange(rows)[:, None]
    h = np.arange(K // 32)[None, :]
    sci = (((r // 16 * (K // 64) + h // 2) * 8 + (r % 16) % 8) * 2 + (r % 16) // 8) * 2 + h % 2
    out = np.zeros(rows * K // 32, np.uint8)
    out[sci] = sc
    return q, out


def u32(t):
    return t.detach().cpu().numpy().view(np.uint32)


def load_variant(path):
    import importlib.util
    spec = importlib.util.spec_from_file_location(f"variant_{abs(hash(path))}", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def guard_tc_shapes(mod, monkeypatch):
    """Under the forced tcgen05 policy, skip (instead of failing) the cases whose d or f is not a multiple of 128:
    the library rejects those shapes for that path (tested separately)."""
    import pytest

    for name in ("run", "run_slots", "layer"):
        f = getattr(mod, name, None)
        if f is None:
            continue

        def guarded(s, *a, _f=f, **kw):
            if s["dm"] % 128 or s["f"] % 128:
                pytest.skip("tcgen05 tiles need d and f multiples of 128")
            return _f(s, *a, **kw)

        monkeypatch.setattr(mod, name, guarded)


def problem_tensors(shape, T, routing="uniform", seed=0, dtype=torch.bfloat16, device="cuda"):
    p = make_problem(shape, T, routing, seed)
    w = [torch.from_numpy(p[n]).to(device, dtype) for n in ("w_gate", "w_up", "w_down")]
    x = torch.from_numpy(p["x"]).to(device, dtype)
    return p, w, x, torch.from_numpy(p["idx"]).to(device), torch.from_numpy(p["wts"]).to(device)


def ref_from_state(mod, st, x, idx, wts, act=0, bg=None, bu=None, bd=None):
    """fp64-accumulated oracle output on the variant's own dequantised weights (fp32)."""
    wg, wu, wd = (t.cpu().numpy() for t in mod.dequant(st))
    xx = x.float().cpu().numpy()
    f = lambda t: None if t is None else t.float().cpu().numpy()  # noqa: E731
    return oracle.moe_forward(xx, wg, wu, wd, idx.cpu().numpy(), wts.float().cpu().numpy(), act=act, bg=f(bg),
                              bu=f(bu), bd=f(bd))


def assert_close(y, ref, tol=TOL_BF16, rowrel=ROWREL_TOL, what=""):
    e = oracle.error_metrics(y.float().cpu().numpy(), ref)
    assert e["finite"], (what, e)
    assert e["rel_fro"] < tol, (what, e)
    assert e["max_rowrel"] <= rowrel, (what, e)
    return e
