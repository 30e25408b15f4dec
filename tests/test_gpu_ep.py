"""Expert parallelism on one B200: the dispatch / combine kernels bit-exact against the oracle's restatement, the
expert kernels on received rows against the fp64 oracle, and the whole expert-parallel layer (P ranks emulated
by threads sharing the GPU, exchanging through ThreadGroup) bit-exact against the single-GPU layer when both
run the same expert kernels."""
import numpy as np
import pytest
import torch

import oracle
from ep_workers import ThreadGroup
from helpers import assert_close, load_variant, ref_from_state
from moelab_b200 import ep, ops
from moelab_b200.variants.cuda import b200_mxfp4_moe, b200_q4_moe
from oracle import ep as oep

pytestmark = pytest.mark.gpu


def _ids(T, E, k, seed, invalid=False):
    rng = np.random.default_rng(seed)
    idx = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    if invalid and T:
        idx[0, 0] = E + 3
        idx[T - 1, k - 1] = -1
    w = rng.random((T, k)).astype(np.float32)
    return idx, w


@pytest.mark.parametrize("P", [1, 2, 4, 8])
@pytest.mark.parametrize("T", [1, 5, 64, 300])
@pytest.mark.parametrize("invalid", [False, True])
def test_dispatch_bit_exact(P, T, invalid):
    E, k, d = 64, 8, 256
    idx, w = _ids(T, E, k, seed=T + P, invalid=invalid)
    x = torch.randn(T, d, device="cuda").to(torch.bfloat16)
    ws = ops.Workspace(d, 64, E, k, "cuda")
    rows, counts, pos = ops.ep_dispatch(x, torch.from_numpy(idx).cuda(), torch.from_numpy(w).cuda(), E, P, ws)
    rc, rp = oep.ep_plan(idx, E, P)
    np.testing.assert_array_equal(counts.cpu().numpy(), rc)
    np.testing.assert_array_equal(pos.cpu().numpy(), rp)
    ref_rows = oep.ep_pack(x, idx, w, rp, E, P)
    got = rows[:ref_rows.shape[0]].view(torch.int16).cpu().numpy().view(np.uint16)
    np.testing.assert_array_equal(got, ref_rows)
    assert (ws.read_error() == ops._lib.DEVERR_EXPERT_ID) == invalid


@pytest.mark.parametrize("T,k", [(1, 1), (3, 8), (40, 4), (257, 6)])
@pytest.mark.parametrize("residual", [False, True])
def test_combine_bit_exact(T, k, residual):
    d = 192
    n = T * k
    rng = np.random.default_rng(T * k)
    perm = rng.permutation(n + 5)[:n].astype(np.int32)  # rows of back in any order, some unused
    perm[rng.random(n) < 0.1] = -1  # dropped slots
    back = rng.standard_normal((n + 5, d)).astype(np.float32)
    res = torch.randn(T, d).to(torch.bfloat16) if residual else None
    y = ops.ep_combine(torch.from_numpy(back).cuda(), torch.from_numpy(perm).cuda(), T, k,
                       None if res is None else res.cuda())
    ref = oep.ep_combine(back, perm, T, k, res)
    np.testing.assert_array_equal(oracle.bf16_bits(y), ref)


def _layer(E, d, f, seed, fmt="q4"):
    g = torch.Generator(device="cuda").manual_seed(seed)
    mk = lambda *s: (torch.randn(*s, generator=g, device="cuda") * 0.02).to(torch.bfloat16)  # noqa: E731
    return [mk(E, f, d), mk(E, f, d), mk(E, d, f)], mk(E, d)


@pytest.mark.parametrize("fmt", ["q4", "mxfp4"])
@pytest.mark.parametrize("R", [1, 9, 100])
def test_expert_rows_vs_oracle(fmt, R):
    E, d, f, P = 16, 256, 320, 4
    v = b200_mxfp4_moe if fmt == "mxfp4" else b200_q4_moe
    w, _ = _layer(E, d, f, seed=R)
    st = ep.shard(v, *w, rank=1, world=P)
    El = E // P
    rng = np.random.default_rng(R)
    x = torch.randn(R, d).to(torch.bfloat16)
    e = rng.integers(0, El, R).astype(np.int32)
    wt = rng.random(R).astype(np.float32)
    rows = np.zeros((R, d + 8), np.uint16)
    rows[:, :d] = oracle.bf16_bits(x)
    rows[:, d:d + 2] = e[:, None].view(np.uint16).reshape(R, 2)
    rows[:, d + 2:d + 4] = wt[:, None].view(np.uint16).reshape(R, 2)
    rt = torch.from_numpy(rows.view(np.int16)).view(torch.bfloat16).cuda()
    yp = ops.ep_experts(st, rt)
    wg, wu, wd = (t.cpu().numpy() for t in v.dequant(st))
    ref = oep.ep_expert_rows(rows, wg, wu, wd)
    assert_close(yp, ref, what=(fmt, R))


def _emulated(P, v, w, gate, tokens, k, policy, seed, act=0, biases=None, gate_b=None):
    """P threads run ep.layer on their own tokens; returns per-rank (y, idx, wts, x)."""
    grp = ThreadGroup(P)
    states = [ep.shard(v, *w, r, P, *(biases or (None, None, None)), act=act) for r in range(P)]
    xs = [torch.randn(T, w[0].shape[2], generator=torch.Generator(device="cuda").manual_seed(seed + r),
                      device="cuda").to(torch.bfloat16) for r, T in enumerate(tokens)]
    torch.cuda.synchronize()

    def body(r, comm):
        return ep.layer(states[r], xs[r], gate, k, gate_b=gate_b, residual=xs[r], policy=policy, comm=comm,
                        return_routing=True)

    out = grp.run(body)
    torch.cuda.synchronize()
    return [(y, i, wt, x) for (y, i, wt), x in zip(out, xs)]


POL = {"slots": ops.POLICY_SLOTS, "tiles8": ops.POLICY_TILES8, "tiles16": ops.POLICY_TILES16}


@pytest.mark.parametrize("P,tokens", [(2, [4, 7]), (4, [1, 0, 33, 16]), (8, [2, 9, 1, 1, 40, 0, 3, 17])])
@pytest.mark.parametrize("pol", list(POL))
def test_emulated_ep_bit_exact_vs_single_gpu(P, tokens, pol):
    E, d, f, k = 32, 256, 384, 4
    w, gate = _layer(E, d, f, seed=P)
    full = b200_q4_moe.prepare(*w)
    b200_q4_moe._ws(full, k)
    for y, idx, wts, x in _emulated(P, b200_q4_moe, w, gate, tokens, k, POL[pol], seed=10 * P):
        if x.shape[0] == 0:
            assert y.shape == (0, d)
            continue
        ri, _ = oracle.router(x, gate, k)
        np.testing.assert_array_equal(idx.cpu().numpy(), ri)
        ys = ops.experts(full, x, idx, wts, policy=POL[pol], residual=x)
        assert torch.equal(y, ys), (pol, (y.float() - ys.float()).abs().max())


@pytest.mark.parametrize("P", [2, 4])
def test_emulated_ep_auto_policy_vs_oracle(P):
    E, d, f, k = 64, 512, 256, 8
    w, gate = _layer(E, d, f, seed=7)
    full = b200_q4_moe.prepare(*w)
    wg, wu, wd = (t.cpu().numpy() for t in b200_q4_moe.dequant(full))
    for y, idx, wts, x in _emulated(P, b200_q4_moe, w, gate, [1, 64, 2, 3][:P], k, None, seed=3):
        ref = oracle.moe_forward(x.float().cpu().numpy(), wg, wu, wd, idx.cpu().numpy(), wts.cpu().numpy())
        assert_close(y, ref + x.float().cpu().numpy())


@pytest.mark.parametrize("pol", ["slots", "tiles8"])
def test_emulated_ep_gptoss_mxfp4_bit_exact(pol):
    """gpt-oss: MXFP4 experts, biases, clamped SwiGLU, router bias, over 4 ranks."""
    E, d, f, k, P = 16, 576, 576, 4, 4
    w, gate = _layer(E, d, f, seed=11)
    g = torch.Generator(device="cuda").manual_seed(12)
    b = (4 * torch.randn(E, f, generator=g, device="cuda"), 4 * torch.randn(E, f, generator=g, device="cuda"),
         0.1 * torch.randn(E, d, generator=g, device="cuda"))
    gb = (torch.randn(E, generator=g, device="cuda")).to(torch.bfloat16)
    full = b200_mxfp4_moe.prepare(*w)
    full.update(bg=b[0], bu=b[1], bd=b[2])
    b200_mxfp4_moe._ws(full, k)
    for y, idx, wts, x in _emulated(P, b200_mxfp4_moe, w, gate, [3, 8, 0, 21], k, POL[pol], seed=5, act=2,
                                    biases=b, gate_b=gb):
        if x.shape[0] == 0:
            continue
        ys = ops.experts(full, x, idx, wts, act=2, policy=POL[pol], residual=x)
        assert torch.equal(y, ys)


def _back_region(xch):
    """(device address, rows) of an exchange buffer's return rows [P][C][d] fp32 (the layout of
    moeb_ep_p2p_bytes: 256 bytes of flags and counters, per-source flags / counts / return flags padded to 256,
    the dispatched rows [P][C][d + 8] bf16, then the return rows)."""
    up = lambda v: (v + 255) & ~255  # noqa: E731
    P, C, d = xch.P, xch.C, xch.d
    rows_off = 256 + 3 * up(4 * P)
    back_off = rows_off + up(P * C * (d + 8) * 2)
    return xch.base + back_off, P * C


def _fill_back(xch, byte):
    from cuda.bindings import runtime as rt
    ptr, n = _back_region(xch)
    assert rt.cudaMemset(ptr, byte, n * xch.d * 4)[0] == rt.cudaError_t.cudaSuccess


def _read_back(xch):
    from cuda.bindings import runtime as rt
    ptr, n = _back_region(xch)
    out = np.empty((n, xch.d), np.float32)
    err = rt.cudaMemcpy(out.ctypes.data, ptr, out.nbytes, rt.cudaMemcpyKind.cudaMemcpyDeviceToHost)[0]
    assert err == rt.cudaError_t.cudaSuccess
    return out


# ------------------------------------------------------------------ tensor-core expert kernels, explicitly requested
@pytest.mark.parametrize("P,tokens", [(2, [40, 33]), (4, [17, 0, 64, 9])])
def test_ep_tc_policy_vs_oracle(P, tokens):
    """The tcgen05 kernels serving expert-parallel rows (explicit policy here; the dispatcher picks them from 14
    rows per local expert): rows with their 16-byte tails gathered in expert order, slot outputs stored into the
    owners' return blocks (peer memory, emulated phase by phase) or the caller's rows (NCCL path, emulated by
    threads). Against the fp64 oracle on the dequantized weights. Peer memory: blocks are only partly filled
    (C above every rank's rows) and one rank sends nothing; every return row that no slot maps to keeps the
    sentinel written before the experts ran."""
    E, d, f, k = 32, 256, 384, 4
    w, gate = _layer(E, d, f, seed=300 + P)
    full = b200_q4_moe.prepare(*w)
    b200_q4_moe._ws(full, k)
    # NCCL path
    for y, idx, wts, x in _emulated(P, b200_q4_moe, w, gate, tokens, k, ops.POLICY_TC, seed=40 * P):
        if x.shape[0]:
            assert_close(y, ref_from_state(b200_q4_moe, full, x, idx, wts) + x.float().cpu().numpy(), what=("nccl", P))
    # peer-memory path
    C = max(tokens) * k + 4
    xchs = ep.PeerExchange.local_group(P, C, d, "cuda")
    states = [ep.shard(b200_q4_moe, *w, r, P) for r in range(P)]
    try:
        for call in range(2):
            xs = [torch.randn(T, d, generator=torch.Generator(device="cuda").manual_seed(call * 50 + r),
                              device="cuda").to(torch.bfloat16) for r, T in enumerate(tokens)]
            routing = []
            for r in range(P):
                idx, wts = ops.router(xs[r], gate, k)
                routing.append((idx, wts, ops.ep_p2p_dispatch(xs[r], idx, wts, E, xchs[r])))
            torch.cuda.synchronize()
            for r in range(P):
                _fill_back(xchs[r], 0xFF)  # NaN sentinel in every return row
            for r in range(P):
                ops.ep_p2p_experts(states[r], xchs[r], policy=ops.POLICY_TC)
            torch.cuda.synchronize()
            for r in range(P):  # only the rows this rank's slots map to were written
                back = _read_back(xchs[r])
                sp = routing[r][2].cpu().numpy().reshape(-1)
                written = np.zeros(back.shape[0], bool)
                written[sp[sp >= 0]] = True
                assert np.isfinite(back[written]).all(), (call, r)
                assert (back[~written].view(np.uint32) == 0xFFFFFFFF).all(), (call, r)
            for r in range(P):
                idx, wts, sp = routing[r]
                y = ops.ep_p2p_combine(xchs[r], sp, tokens[r], k, d, residual=xs[r], device="cuda")
                if tokens[r]:
                    ref = ref_from_state(b200_q4_moe, full, xs[r], idx, wts) + xs[r].float().cpu().numpy()
                    assert_close(y, ref, what=("p2p", call, r))
        torch.cuda.synchronize()
        assert all(x.read_error() == 0 for x in xchs)
        assert all(s["ep_ws"].read_error() == 0 for s in states)
    finally:
        for x in xchs:
            x.close()


# ------------------------------------------------------------------ exchange over peer memory, emulated
P2P_POL = {"tiles8ring": ops.POLICY_TILES8_RING, "tiles16ring": ops.POLICY_TILES16_RING, "slots": ops.POLICY_SLOTS}


@pytest.mark.parametrize("P,tokens", [(2, [4, 7]), (4, [1, 0, 33, 16]), (8, [2, 9, 1, 1, 40, 0, 3, 17])])
@pytest.mark.parametrize("pol", list(P2P_POL))
@pytest.mark.parametrize("blocks", ["capacity", "tight"])
def test_p2p_emulated_bit_exact_vs_single_gpu(P, tokens, pol, blocks):
    """P ranks emulated phase by phase on one GPU (all dispatches, then all experts, then all combines), so
    every flag a kernel waits for was released by an earlier kernel on the stream. Three calls in a row reuse
    the buffers with advancing epochs; every output must equal the single-GPU layer bit for bit. Blocks of the
    whole capacity, or of the call's own bound (Cs = max T * k < C)."""
    E, d, f, k = 32, 256, 384, 4
    w, gate = _layer(E, d, f, seed=100 + P)
    full = b200_q4_moe.prepare(*w)
    b200_q4_moe._ws(full, k)
    C = 2 * max(tokens) * k + 4
    Cs = 0 if blocks == "capacity" else max(tokens) * k
    xchs = ep.PeerExchange.local_group(P, C, d, "cuda")
    states = [ep.shard(b200_q4_moe, *w, r, P) for r in range(P)]
    try:
        for call in range(3):
            xs = [torch.randn(T, d, generator=torch.Generator(device="cuda").manual_seed(call * 100 + r),
                              device="cuda").to(torch.bfloat16) for r, T in enumerate(tokens)]
            routing = []
            for r in range(P):
                idx, wts = ops.router(xs[r], gate, k)
                routing.append((idx, wts, ops.ep_p2p_dispatch(xs[r], idx, wts, E, xchs[r], Cs=Cs)))
            for r in range(P):
                ops.ep_p2p_experts(states[r], xchs[r], policy=P2P_POL[pol], Cs=Cs)
            for r in range(P):
                idx, wts, sp = routing[r]
                y = ops.ep_p2p_combine(xchs[r], sp, tokens[r], k, d, residual=xs[r], device="cuda")
                if tokens[r] == 0:
                    continue
                ys = ops.experts(full, xs[r], idx, wts, policy=P2P_POL[pol], residual=xs[r])
                assert torch.equal(y, ys), (call, r, (y.float() - ys.float()).abs().max())
        torch.cuda.synchronize()
        assert all(x.read_error() == 0 for x in xchs)
        assert all(s["ep_ws"].read_error() == 0 for s in states)
    finally:
        for x in xchs:
            x.close()


# ------------------------------------------------------------------ failure detection: a peer that never signals
@pytest.mark.parametrize("pol", ["slots", "tiles8ring"])
def test_p2p_peer_never_signals_times_out(pol):
    """Two ranks emulated on one GPU; rank 1 never dispatches nor returns rows (a dead peer, made on the host by
    not calling it). Rank 0's bounded waits - for rank 1's dispatch flag in the expert call, for its return flag
    in the combine - run out after the short limit set here, record DEVERR_TIMEOUT, and the calls return; the
    GPU stays usable (a later call on a healthy pair is checked)."""
    E, d, f, k, T = 16, 256, 384, 2, 3
    w, gate = _layer(E, d, f, seed=5)
    C = T * k
    xchs = ep.PeerExchange.local_group(2, C, d, "cuda")
    states = [ep.shard(b200_q4_moe, *w, r, 2) for r in range(2)]
    try:
        xchs[0].set_wait_limit(0.05)
        x = torch.randn(T, d, generator=torch.Generator(device="cuda").manual_seed(1), device="cuda").to(torch.bfloat16)
        idx, wts = ops.router(x, gate, k)
        sp = ops.ep_p2p_dispatch(x, idx, wts, E, xchs[0])
        ops.ep_p2p_experts(states[0], xchs[0], policy=P2P_POL[pol])
        y = ops.ep_p2p_combine(xchs[0], sp, T, k, d, residual=x, device="cuda")
        torch.cuda.synchronize()
        assert states[0]["ep_ws"].read_error() & ops._lib.DEVERR_TIMEOUT
        assert xchs[0].read_error() & ops._lib.DEVERR_TIMEOUT
        assert bool(torch.isfinite(y.float()).all())
    finally:
        for x_ in xchs:
            x_.close()
    # the context is still usable
    full = b200_q4_moe.prepare(*w)
    b200_q4_moe._ws(full, k)
    y2 = ops.experts(full, x, idx, wts)
    assert_close(y2, ref_from_state(b200_q4_moe, full, x, idx, wts))
