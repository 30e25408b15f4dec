"""Expert-parallel MoE layer: P ranks (one process per GPU), rank r owns experts [r*E/P, (r+1)*E/P).

moe-lab runs one device and has no counterpart; the layer call keeps its contract
(x, gate weights, packed experts, k) -> y (moelab/e2e.py:51-65) with the experts spread over the ranks:

  1. router on every rank for its own tokens (the gate is replicated)           -> idx, wts (global ids)
  2. dispatch kernels: slots sorted by owning rank, send rows = x row + {local expert, weight} tail
  3. all-to-all of the P send counts, read once on the host (the split sizes of the next two exchanges)
  4. all-to-all-v of the send rows                                              -> rows for my experts
  5. grouped expert kernels on the received rows (k = 1 per row)                -> fp32 w * (W_d h + b_d)
  6. all-to-all-v of those outputs back to the owners of the tokens
  7. combine kernel: y[t] = sum_j (fixed j order) + residual, rounded once to bf16

Steps 4 and 6 move bytes only (rows travel as uint8 so any backend carries them). The device steps come from a
`kernels` object: CudaKernels (the product) or a host implementation the CPU tests supply, so the collective
choreography is the same code in both. Every rank takes the same collective steps in the same order, including
for T = 0 tokens.
"""
import ctypes

import torch
import torch.distributed as dist

from . import _lib, ops


class CudaKernels:
    """The device steps as CUDA kernels of libmoelab_b200 (no host fallback)."""

    @staticmethod
    def router(x, gate_w, k, gate_b, norm, rscale):
        return ops.router(x, gate_w, k, gate_b=gate_b, norm=norm, scale=rscale)

    @staticmethod
    def dispatch(state, x, idx, wts):
        return ops.ep_dispatch(x, idx, wts, state["E_global"], state["ep_world"], state["ep_ws"])

    @staticmethod
    def experts(state, rows, act, policy):
        return ops.ep_experts(state, rows, act=act, policy=policy)

    @staticmethod
    def combine(back, slot_pos, T, k, residual):
        return ops.ep_combine(back, slot_pos, T, k, residual)


def shard(variant, w_gate, w_up, w_down, rank, world, b_gate=None, b_up=None, b_down=None, act=0):
    """This rank's experts of a layer given as full [E, ...] weights: the variant's prepare() on the slice, plus
    the expert-parallel bookkeeping. variant: b200_q4_moe or b200_mxfp4_moe (any module with prepare())."""
    E, f, d = w_gate.shape
    if E % world:
        raise ValueError(f"E={E} experts do not split over {world} ranks")
    El = E // world
    sl = slice(rank * El, (rank + 1) * El)
    st = variant.prepare(w_gate[sl].contiguous(), w_up[sl].contiguous(), w_down[sl].contiguous())
    if b_gate is not None:
        st.update(bg=b_gate[sl].float().contiguous(), bu=b_up[sl].float().contiguous(),
                  bd=b_down[sl].float().contiguous())
    st.update(act=act)
    return attach(st, rank, world, E)


def attach(state, rank, world, E):
    """Mark a prepared local-expert state (E/world experts) as rank `rank` of an expert-parallel layer."""
    state.update(ep_rank=rank, ep_world=world, E_global=E)
    if "ws" in state:
        state["ep_ws"] = ops.Workspace(state["dm"], state["f"], state["E"], 1, state["ws"].device, ep=True)
    return state


class TorchComm:
    """all-to-all over a torch.distributed process group (NCCL on GPUs, gloo on CPU)."""

    def __init__(self, group=None):
        self.group = group

    def all_to_all_single(self, out, inp, out_splits=None, in_splits=None):
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)


def _as_bytes(t):
    if t.numel() == 0:  # an empty block may carry any strides; send a plain empty byte tensor
        return torch.empty(0, t.shape[1] * t.element_size(), dtype=torch.uint8, device=t.device)
    return t.view(torch.uint8)


def _a2a_rows(comm, out, inp, out_splits, in_splits):
    """all-to-all-v of row blocks, carried as bytes."""
    comm.all_to_all_single(_as_bytes(out), _as_bytes(inp), out_splits, in_splits)


def layer(state, x, gate_w, k, gate_b=None, norm=True, rscale=1.0, act=None, residual=None, policy=None,
          group=None, comm=None, kernels=CudaKernels, return_routing=False, timings=None):
    """y [T, d] for this rank's T tokens. state: from shard()/attach(). comm: object with
    all_to_all_single(out, inp, out_splits, in_splits) (default TorchComm(group)). timings: optional dict that
    receives the rows sent / received (and the received rows); if it holds "events" (two CUDA events) they are
    recorded around the expert kernels."""
    P = state["ep_world"]
    comm = comm or TorchComm(group)
    act = state.get("act", 0) if act is None else act
    policy = ops.POLICY_AUTO if policy is None else policy
    T, d = x.shape
    idx, wts = kernels.router(x, gate_w, k, gate_b, norm, rscale)
    rows, send_counts, slot_pos = kernels.dispatch(state, x, idx, wts)
    recv_counts = torch.empty_like(send_counts)
    comm.all_to_all_single(recv_counts, send_counts)
    both = torch.cat([send_counts, recv_counts]).tolist()  # the layer's one host synchronisation
    send, recv = both[:P], both[P:]
    ns, nr = sum(send), sum(recv)
    recv_rows = rows.new_empty(nr, d + 8)
    _a2a_rows(comm, recv_rows, rows[:ns], recv, send)
    ev = timings.get("events") if timings is not None else None
    if ev:
        ev[0].record()
    yp = kernels.experts(state, recv_rows, act, policy)
    if ev:
        ev[1].record()
    back = yp.new_empty(ns, d)
    _a2a_rows(comm, back, yp, send, recv)
    y = kernels.combine(back, slot_pos, T, k, residual)
    if timings is not None:
        timings.update(rows_sent=ns, rows_received=nr, recv_rows=recv_rows)
    return (y, idx, wts) if return_routing else y


# ------------------------------------------------------------------ exchange over NVLink peer memory
class PeerExchange:
    """The exchange buffers of an expert-parallel group: one device allocation per rank (rows in, weighted
    rows back, flags), mapped into every rank of the group with CUDA IPC (plain peer mappings, no multicast).
    C = rows per (source, owner) block: at least the largest T*k of any call. `peers` is a device array of the
    P buffer addresses as this rank sees them."""

    def __init__(self, P, me, C, d, device, base, ptrs, opened=(), owns=True):
        self.P, self.me, self.C, self.d, self.device = P, me, C, d, device
        self.base = base
        self.ptrs = list(ptrs)
        self.peers = torch.tensor(self.ptrs, dtype=torch.int64, device=device)
        self._opened = list(opened)
        self._owns = owns

    @staticmethod
    def nbytes(P, C, d):
        return _lib.load().moeb_ep_p2p_bytes(P, C, d)

    @staticmethod
    def _alloc(nbytes):
        p = ctypes.c_void_p()
        _lib.call("moeb_ep_ipc_alloc", nbytes, ctypes.byref(p))
        return p.value

    @classmethod
    def create(cls, C, d, group=None, device=None):
        """Collective over `group` (every rank calls it): allocate, exchange IPC handles, map the peers."""
        P, me = dist.get_world_size(group), dist.get_rank(group)
        device = device or torch.device("cuda", torch.cuda.current_device())
        base = cls._alloc(cls.nbytes(P, C, d))
        h = (ctypes.c_ubyte * 64)()
        _lib.call("moeb_ep_ipc_handle", ctypes.c_void_p(base), h)
        mine = torch.tensor(list(bytes(h)), dtype=torch.uint8, device=device)
        allh = [torch.empty_like(mine) for _ in range(P)]
        dist.all_gather(allh, mine, group=group)
        ptrs, opened = [], []
        for r in range(P):
            if r == me:
                ptrs.append(base)
                continue
            hr = (ctypes.c_ubyte * 64)(*allh[r].cpu().tolist())
            p = ctypes.c_void_p()
            _lib.call("moeb_ep_ipc_open", hr, ctypes.byref(p))
            ptrs.append(p.value)
            opened.append(p.value)
        dist.barrier(group=group)
        return cls(P, me, C, d, device, base, ptrs, opened)

    @classmethod
    def local_group(cls, P, C, d, device):
        """P exchanges for P ranks emulated in one process on one device (tests): plain buffers, no IPC."""
        bases = [cls._alloc(cls.nbytes(P, C, d)) for _ in range(P)]
        return [cls(P, r, C, d, device, bases[r], bases, owns=True) for r in range(P)]

    def set_wait_limit(self, seconds):
        """Limit of this rank's bounded waits for peers (seconds; 0 = the 2 s default). A wait that runs out
        records DEVERR_TIMEOUT (see read_error) and the call carries on without that peer."""
        _lib.call("moeb_ep_p2p_set_wait_limit", ctypes.c_void_p(self.base), self.P, self.C, self.d, float(seconds),
                  ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))

    def read_error(self):
        out = ctypes.c_uint(0)
        _lib.call("moeb_ep_p2p_read_error", ctypes.c_void_p(self.base), self.P, self.C, self.d, ctypes.byref(out),
                  ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        return out.value

    def close(self):
        for p in self._opened:
            _lib.call("moeb_ep_ipc_close", ctypes.c_void_p(p))
        self._opened = []
        if self._owns and self.base:
            _lib.call("moeb_ep_ipc_free", ctypes.c_void_p(self.base))
        self.base = 0


def layer_p2p(state, x, gate_w, k, xch, gate_b=None, norm=True, rscale=1.0, act=None, residual=None, policy=None,
              return_routing=False, max_tokens=None):
    """The expert-parallel layer call over peer memory: router, dispatch (rows stored into the owners'
    buffers), this rank's experts on what it received (rows stored back), combine. No host synchronisation:
    the sequence can be captured in a CUDA graph. Every rank of the group must make the same calls.
    max_tokens: a bound on every rank's T for this call, the same on all ranks (default: the exchange's
    capacity); a small bound keeps the owners' scan of the source blocks short."""
    act = state.get("act", 0) if act is None else act
    policy = ops.POLICY_AUTO if policy is None else policy  # the library picks by the call's block size
    T, d = x.shape
    Cs = xch.C if max_tokens is None else min(xch.C, max(1, int(max_tokens) * k))
    idx, wts = ops.router(x, gate_w, k, gate_b=gate_b, norm=norm, scale=rscale)
    slot_pos = ops.ep_p2p_dispatch(x, idx, wts, state["E_global"], xch, Cs=Cs)
    ops.ep_p2p_experts(state, xch, act=act, policy=policy, Cs=Cs)
    y = ops.ep_p2p_combine(xch, slot_pos, T, k, d, residual=residual, device=x.device)
    return (y, idx, wts) if return_routing else y
