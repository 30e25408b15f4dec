"""Expert parallelism on the CPU: the oracle's restatement of the dispatch / combine steps, and the collective
choreography of moelab_b200.ep.layer run as gloo ranks (world size 2 and 4) with host kernels, checked against
the single-process oracle layer. No GPU."""
import multiprocessing as mp

import numpy as np
import pytest
import torch

from ep_workers import free_port, host_rank
from oracle import ep as oep


def test_plan_is_a_stable_sort_by_owner():
    rng = np.random.default_rng(0)
    E, P, T, k = 16, 4, 37, 3
    idx = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    counts, pos = oep.ep_plan(idx, E, P)
    owner = idx.reshape(-1) // (E // P)
    assert counts.tolist() == [int((owner == p).sum()) for p in range(P)]
    assert sorted(pos.tolist()) == list(range(T * k))  # a permutation of the send rows
    for p in range(P):
        s = np.nonzero(owner == p)[0]
        assert (np.diff(pos[s]) == 1).all()  # slot order kept inside an owner
        assert pos[s][0] == counts[:p].sum() if len(s) else True


def test_plan_drops_invalid_ids():
    idx = np.array([[0, 9], [-1, 3]], np.int32)
    counts, pos = oep.ep_plan(idx, 8, 2)
    assert pos.tolist() == [0, -1, -1, 1] and counts.tolist() == [2, 0]


def test_pack_and_unpack_round_trip():
    rng = np.random.default_rng(1)
    T, d, E, P, k = 5, 64, 8, 2, 2
    x = torch.randn(T, d).to(torch.bfloat16)
    idx = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    wts = rng.random((T, k)).astype(np.float32)
    counts, pos = oep.ep_plan(idx, E, P)
    rows = oep.ep_pack(x, idx, wts, pos, E, P)
    xr, e, w = oep.unpack_rows(rows)
    for s in range(T * k):
        assert np.array_equal(xr[pos[s]], x[s // k].float().numpy())
        assert e[pos[s]] == idx.reshape(-1)[s] % (E // P) and w[pos[s]] == wts.reshape(-1)[s]
    assert (rows[:, d + 4:] == 0).all()


def test_combine_fixed_order():
    back = np.array([[1.0, 2.0], [3.0, 1e-8], [-4.0, 5.0]], np.float32).repeat(32, axis=1)
    pos = np.array([2, 0, 1, -1], np.int32)  # token 0: rows 2 then 0; token 1: row 1, dropped slot
    from oracle import bits_to_f32
    y = bits_to_f32(oep.ep_combine(back, pos, 2, 2))
    assert y[0, 0] == -3.0 and y[1, 0] == 3.0


def _run_ranks(P, tokens, d=128, f=128, E=8, k=2, seed=3):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=host_rank, args=(r, P, port, tokens, d, f, E, k, seed, q)) for r in range(P)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(P):
            rank, status, payload = q.get(timeout=240)
            assert status == "ok", payload
            out[rank] = payload
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    return out


@pytest.mark.parametrize("P,tokens", [(2, [9, 6]), (2, [5, 0]), (4, [7, 3, 1, 16])])
def test_gloo_ranks_match_the_single_process_layer(P, tokens):
    out = _run_ranks(P, tokens)
    k = 2
    for r in range(P):
        m = out[r]["metrics"]
        assert m["finite"] and m["rel_fro"] < 3e-3 and m["max_rowrel"] < 1e-2, (r, m)
        assert out[r]["tot"] == [sum(tokens) * k, sum(tokens) * k]  # every slot sent and received once
        assert out[r]["sent"] == tokens[r] * k
