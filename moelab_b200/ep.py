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
import torch
import torch.distributed as dist

from . import ops


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
