"""The routing step's integer work, bit-exact: per-expert counts, prefix offsets, the slot permutation grouped by
expert and the tile list, from the CUDA tile builder (moeb_route_tables, the same code every tiled layer call
runs) against the oracle's stable counting sort, whose tile grouping is checked against a restatement of the
reference's map kernel (moelab/variants/mlx/metal_q4_tiles_v2.py:362-373) on the CPU.
"""
import numpy as np
import pytest
import torch

import oracle
from moelab_b200 import ops
from moelab_b200.problem import make_routing

T_VALUES = [1, 7, 33, 257, 2048]
E_VALUES = [8, 64, 128]
ROUTINGS = ["uniform", "one_hot", "zipf", "round_robin"]


def _ids(T, E, k, routing, seed):
    idx, _ = make_routing(T, E, k, routing, np.random.default_rng(seed))
    return idx


def _check(idx_np, E, nt, expect_bad=False):
    idx = torch.from_numpy(np.ascontiguousarray(idx_np, np.int32)).cuda()
    counts, offsets, sorted_, tiles, err = ops.route_tables(idx, E, nt)
    rc, ro, rs, rt, bad = oracle.route_tables(idx_np, E, nt)
    np.testing.assert_array_equal(counts.cpu().numpy(), rc)
    np.testing.assert_array_equal(offsets.cpu().numpy(), ro)
    np.testing.assert_array_equal(sorted_.cpu().numpy(), rs)
    np.testing.assert_array_equal(tiles.cpu().numpy(), rt)
    assert bool(err & 1) == bad == expect_bad
    return tiles.cpu().numpy(), sorted_.cpu().numpy()


def test_oracle_tiles_follow_reference_map_contract():
    """CPU: the oracle's tiles, as (expert, member slots), are exactly the reference map kernel's tiles."""
    for T, E, k, routing, VT in [(33, 8, 2, "uniform", 8), (64, 16, 4, "zipf", 8), (40, 8, 2, "one_hot", 8),
                                 (25, 12, 3, "round_robin", 4), (1, 8, 2, "uniform", 8)]:
        idx = _ids(T, E, k, routing, seed=T + E)
        _, _, s, tiles, bad = oracle.route_tables(idx, E, VT)
        assert not bad
        got = {(int(t[0]), tuple(int(v) for v in s[t[1]:t[1] + t[2]])) for t in tiles}
        assert got == oracle.reference_map_tiles(idx, VT)


@pytest.mark.gpu
@pytest.mark.parametrize("routing", ROUTINGS)
@pytest.mark.parametrize("E", E_VALUES)
@pytest.mark.parametrize("T", T_VALUES)
def test_route_tables_bit_exact(T, E, routing):
    k = 2 if E == 8 else 8
    idx = _ids(T, E, k, routing, seed=17 * T + E)
    for nt in (8, 16, 128):
        _check(idx, E, nt)


@pytest.mark.gpu
@pytest.mark.parametrize("T", [1, 33, 2048])
def test_route_tables_invalid_ids(T):
    """Ids outside [0, E) are grouped under expert 0 and flagged, never written out of bounds."""
    E, k = 64, 6
    idx = _ids(T, E, k, "uniform", seed=T)
    rng = np.random.default_rng(T)
    bad = rng.random(idx.shape) < 0.1
    bad.flat[0] = True
    idx = np.where(bad, rng.choice([-1, E, E + 7, -(2 ** 30)], size=idx.shape), idx).astype(np.int32)
    _check(idx, E, 16, expect_bad=True)


@pytest.mark.gpu
def test_route_tables_large_and_repeatable():
    """T*k = 65536 slots (ids not cached in shared memory): bit-exact and identical across runs."""
    T, E, k = 8192, 128, 8
    idx = _ids(T, E, k, "zipf", seed=3)
    t1, s1 = _check(idx, E, 256)
    t2, s2 = _check(idx, E, 256)
    np.testing.assert_array_equal(t1, t2)
    np.testing.assert_array_equal(s1, s2)
