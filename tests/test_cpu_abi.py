"""The C-ABI library loads and exports every symbol include/*.h declares; host-only entry points work without
a GPU (no compute calls here)."""
import glob
import os
import re

import pytest

from moelab_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = re.sub(r"/\*.*?\*/", "", open(h).read(), flags=re.S)
        names |= set(re.findall(r"\b(moeb_\w+)\s*\(", src))
    return names


def declared_arity():
    """Parameter count of every declared function (comments stripped; `void` alone counts as none)."""
    out = {}
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = re.sub(r"/\*.*?\*/", "", open(h).read(), flags=re.S)
        for name, params in re.findall(r"\b(moeb_\w+)\s*\(([^)]*)\)\s*;", src):
            params = params.strip()
            out[name] = 0 if params in ("", "void") else params.count(",") + 1
    return out


def test_header_matches_binding_table():
    assert declared_functions() == set(_lib.SIGNATURES), declared_functions() ^ set(_lib.SIGNATURES)


def test_binding_arity_matches_header():
    ar = declared_arity()
    assert set(ar) == set(_lib.SIGNATURES)
    bad = {n: (ar[n], len(_lib.SIGNATURES[n][1])) for n in ar if ar[n] != len(_lib.SIGNATURES[n][1])}
    assert not bad, bad


def test_library_exports_every_symbol():
    lib = _lib.load()
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_host_only_calls():
    lib = _lib.load()
    assert lib.moeb_version() == 1
    # workspace size grows with T and covers h / per-slot partials
    a = lib.moeb_workspace_bytes(1, 2048, 768, 128, 8)
    b = lib.moeb_workspace_bytes(256, 2048, 768, 128, 8)
    assert 0 < a < b
    assert b >= 256 * 8 * (768 * 2 + 2048 * 4)
    # dispatcher: decode -> per-slot tiles; high load -> grouped tiles
    assert lib.moeb_policy(1, 128, 8) == _lib.POLICY_SLOTS
    assert lib.moeb_policy(2, 128, 8) == _lib.POLICY_SLOTS
    assert lib.moeb_policy(4, 128, 8) == _lib.POLICY_TILES8_RING
    assert lib.moeb_policy(128, 128, 8) == _lib.POLICY_TILES16_RING  # 8 slots per expert
    assert lib.moeb_policy(192, 128, 8) == _lib.POLICY_TILES16_RING  # 12 slots per expert
    assert lib.moeb_policy(224, 128, 8) == _lib.POLICY_TC  # 14 slots per expert: tcgen05 tiles
    assert lib.moeb_policy(384, 128, 8) == _lib.POLICY_TC


def test_bad_shape_is_rejected_before_any_device_work():
    # idx / wts are non-null dummies: the shape check runs before anything is dereferenced
    with pytest.raises(_lib.MoebError, match="multiples of 64"):
        _lib.call("moeb_experts_q4", *([None] * 10), 8, 8, 4, 100, 256, 8, 2, 0, 0, None, None, None, 0, None)
    with pytest.raises(_lib.MoebError, match="k must be"):
        _lib.call("moeb_experts_q4", *([None] * 10), 8, 8, 4, 128, 256, 8, 9, 0, 0, None, None, None, 0, None)


def test_fragment_major_layout_is_a_permutation():
    """The numpy model of the B200 weight layout (used by the bit-exact GPU tests) is a bijection."""
    import numpy as np

    from helpers import fm_q_index, to_b200_q4
    for rows, K in [(16, 64), (48, 256), (32, 2880 // 64 * 64)]:
        idx = fm_q_index(rows, K).ravel()
        assert np.array_equal(np.sort(idx), np.arange(rows * K // 8))
    rng = np.random.default_rng(0)
    qw = rng.integers(0, 2**32, (32, 64), dtype=np.uint32)
    s = rng.integers(0, 2**16, (32, 8), dtype=np.uint16)
    q, sb = to_b200_q4(qw, s, s)
    assert q.shape == (32 * 64,) and sb.shape == (32 * 8,)


def test_header_layout_formulas_match_the_packing():
    """The weight layout spelled out in include/moelab_b200.h, implemented element by element, gives the same words
    as the packing the GPU tests check bit-exact against the kernels (helpers.to_b200_q4 / to_b200_fp4)."""
    import numpy as np
    from helpers import to_b200_fp4, to_b200_q4
    rng = np.random.default_rng(0)
    rows, K = 32, 128
    codes = rng.integers(0, 16, size=(rows, K), dtype=np.uint32)
    nat = np.zeros((rows, K // 8), np.uint32)
    for i in range(8):
        nat |= codes[:, i::8] << (4 * i)
    s = rng.integers(0, 1 << 16, size=(rows, K // 64), dtype=np.uint32)
    b = rng.integers(0, 1 << 16, size=(rows, K // 64), dtype=np.uint32)
    q_ref, sb_ref = to_b200_q4(nat, s, b)
    q = np.zeros(rows * K // 8, np.uint32)
    sb = np.zeros(rows * K // 64, np.uint32)
    for r in range(rows):
        rb, rr = r // 16, r % 16
        for k in range(K):
            g, j, e = k // 64, (k % 64) // 8, k % 8
            lane = (rr % 8) * 4 + j // 2
            w = ((rb * (K // 64) + g) * 32 + lane) * 4 + (rr // 8) * 2 + j % 2
            nib = e // 2 if e % 2 == 0 else 4 + e // 2
            q[w] |= codes[r, k] << (4 * nib)
        for g in range(K // 64):
            sb[((rb * (K // 64) + g) * 8 + rr % 8) * 2 + rr // 8] = s[r, g] | (b[r, g] << 16)
    np.testing.assert_array_equal(q, q_ref)
    np.testing.assert_array_equal(sb, sb_ref)
    sc = rng.integers(0, 256, size=(rows, K // 32), dtype=np.uint8)
    _, sc_ref = to_b200_fp4(nat, sc)
    sc_h = np.zeros(rows * K // 32, np.uint8)
    for r in range(rows):
        rb, rr = r // 16, r % 16
        for h in range(K // 32):
            sc_h[(((rb * (K // 64) + h // 2) * 8 + rr % 8) * 2 + rr // 8) * 2 + h % 2] = sc[r, h]
    np.testing.assert_array_equal(sc_h, sc_ref)
