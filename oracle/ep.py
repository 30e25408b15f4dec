"""CPU restatement of the expert-parallel device steps (moelab_b200/csrc/ep.cu) and a host implementation of the
`kernels` object that moelab_b200.ep.layer drives.

TEST INFRASTRUCTURE ONLY (imported by tests/). moe-lab runs one device, so these steps have no reference
counterpart; their definition is the single-GPU layer: the expert-parallel result must equal it. ep_plan /
ep_pack / ep_combine are bit-exact targets for the CUDA kernels; ep_expert_rows is the fp64-accumulated
expert math (oracle.moe_forward) on one slot per row.
"""
import numpy as np
import torch

from . import bf16_bits, moe_forward, router


def ep_plan(idx, E, P):
    """Stable counting sort of the T*k slots by owning rank (owner = id // (E/P)).
    Returns send_counts int32 [P] and slot_pos int32 [T*k] (-1 for an id outside [0, E))."""
    ids = np.asarray(idx, np.int64).reshape(-1)
    El = E // P
    valid = (ids >= 0) & (ids < E)
    owner = np.where(valid, ids // El, -1)
    counts = np.array([(owner == p).sum() for p in range(P)], np.int32)
    off = np.concatenate([[0], np.cumsum(counts)[:-1]]).astype(np.int64)
    pos = np.full(ids.shape, -1, np.int32)
    seen = np.zeros(P, np.int64)
    for s, o in enumerate(owner):  # slot order kept inside an owner
        if o >= 0:
            pos[s] = off[o] + seen[o]
            seen[o] += 1
    return counts, pos


def ep_pack(x, idx, wts, slot_pos, E, P):
    """Send rows as uint16 [n_valid, d + 8]: the slot's token row (bf16 bits), then {int32 local expert,
    fp32 weight, 0, 0} as little-endian 16-bit halves."""
    xb = bf16_bits(x)
    T, d = xb.shape
    ids = np.asarray(idx, np.int64).reshape(-1)
    w = np.asarray(wts, np.float32).reshape(-1)
    k = ids.size // max(T, 1)
    El = E // P
    n = int((np.asarray(slot_pos) >= 0).sum())
    rows = np.zeros((n, d + 8), np.uint16)
    for s, p in enumerate(np.asarray(slot_pos)):
        if p < 0:
            continue
        rows[p, :d] = xb[s // k]
        tail = np.array([ids[s] % El], np.int32).view(np.uint16)
        rows[p, d:d + 2] = tail
        rows[p, d + 2:d + 4] = w[s:s + 1].view(np.uint16)
    return rows


def unpack_rows(rows_u16):
    """(x fp32 [R, d], local expert int32 [R], weight fp32 [R]) from send rows."""
    r = np.ascontiguousarray(rows_u16, np.uint16)
    d = r.shape[1] - 8
    x = (r[:, :d].astype(np.uint32) << 16).view(np.float32)
    e = np.ascontiguousarray(r[:, d:d + 2]).view(np.int32).reshape(-1)
    w = np.ascontiguousarray(r[:, d + 2:d + 4]).view(np.float32).reshape(-1)
    return x, e, w


def ep_expert_rows(rows_u16, wg, wu, wd, act=0, bg=None, bu=None, bd=None):
    """yp fp32 [R, d] = w * (W_down h + b_down) for each received row, fp64-accumulated."""
    x, e, w = unpack_rows(rows_u16)
    if x.shape[0] == 0:
        return np.zeros((0, x.shape[1]), np.float32)
    return moe_forward(x, wg, wu, wd, e[:, None], w[:, None], act=act, bg=bg, bu=bu, bd=bd)


def ep_combine(back, slot_pos, T, k, residual=None):
    """bf16 bits [T, d]: fp32 sum over j of back[slot_pos[t*k + j]] in j order, + residual, rounded once."""
    back = np.asarray(back, np.float32)
    d = back.shape[1]
    pos = np.asarray(slot_pos).reshape(T, k)
    acc = np.zeros((T, d), np.float32)
    for j in range(k):
        p = pos[:, j]
        m = p >= 0
        acc[m] = acc[m] + back[p[m]]
    if residual is not None:
        acc = acc + (bf16_bits(residual).astype(np.uint32) << 16).view(np.float32)
    return bf16_bits(torch.from_numpy(acc).to(torch.bfloat16))


# ------------------------------------------------------------------ host `kernels` for moelab_b200.ep.layer
def _bf16_tensor(u16):
    return torch.from_numpy(np.ascontiguousarray(u16).view(np.int16)).view(torch.bfloat16)


def host_shard(wg, wu, wd, rank, world, act=0, bg=None, bu=None, bd=None):
    """State of rank `rank` for HostKernels: fp32 numpy weights of its E/world experts."""
    E = wg.shape[0]
    El = E // world
    sl = slice(rank * El, (rank + 1) * El)
    cut = lambda a: None if a is None else np.ascontiguousarray(np.asarray(a, np.float32)[sl])  # noqa: E731
    return {"wg": cut(wg), "wu": cut(wu), "wd": cut(wd), "bg": cut(bg), "bu": cut(bu), "bd": cut(bd), "act": act,
            "E": El, "E_global": E, "ep_rank": rank, "ep_world": world}


class HostKernels:
    """The expert-parallel device steps restated on the CPU (torch CPU tensors in and out)."""

    @staticmethod
    def router(x, gate_w, k, gate_b, norm, rscale):
        idx, wts = router(x, gate_w, k, bias=gate_b, norm=norm, scale=rscale)
        return torch.from_numpy(idx), torch.from_numpy(wts)

    @staticmethod
    def dispatch(state, x, idx, wts):
        E, P = state["E_global"], state["ep_world"]
        counts, pos = ep_plan(idx.numpy(), E, P)
        rows = ep_pack(x, idx.numpy(), wts.numpy(), pos, E, P)
        full = np.zeros((pos.size, rows.shape[1] if rows.size else x.shape[1] + 8), np.uint16)
        full[:rows.shape[0]] = rows
        return _bf16_tensor(full), torch.from_numpy(counts), torch.from_numpy(pos)

    @staticmethod
    def experts(state, rows, act, policy):
        u16 = rows.view(torch.int16).numpy().view(np.uint16)
        yp = ep_expert_rows(u16, state["wg"], state["wu"], state["wd"], act=act, bg=state["bg"], bu=state["bu"],
                            bd=state["bd"])
        return torch.from_numpy(np.ascontiguousarray(yp, np.float32))

    @staticmethod
    def combine(back, slot_pos, T, k, residual):
        y = ep_combine(back.numpy(), slot_pos.numpy(), T, k, residual)
        return _bf16_tensor(y)
