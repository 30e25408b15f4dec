"""torch-level wrappers over the C ABI (device tensors in, device tensors out, current stream).

Every function here launches CUDA kernels from libmoelab_b200.so; there is no CPU path. Tensors must be
CUDA, contiguous, with the dtypes documented in include/moelab_b200.h (packed codes are carried in int32 /
uint8 tensors).
"""
import ctypes
import threading

import torch

from . import _lib

POLICY_AUTO, POLICY_SLOTS, POLICY_TILES8, POLICY_TILES16 = (_lib.POLICY_AUTO, _lib.POLICY_SLOTS,
                                                            _lib.POLICY_TILES8, _lib.POLICY_TILES16)
POLICY_TILES8_RING, POLICY_TILES16_RING = _lib.POLICY_TILES8_RING, _lib.POLICY_TILES16_RING
POLICY_TC = _lib.POLICY_TC
POLICY_DECODE = _lib.POLICY_DECODE
POLICY_TILES24_RING = _lib.POLICY_TILES24_RING


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _need(t, dtype, name):
    if t is None:
        return
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (moelab_b200 has no CPU path)")
    if dtype is not None and t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


class Workspace:
    """Caller-owned scratch for the layer kernels, grown on demand (allocation happens here, in Python,
    never inside the library). Zeroed once at allocation; the kernels keep its counters zero."""

    def __init__(self, d, f, E, k, device=None, ep=False):
        self.d, self.f, self.E, self.k = d, f, E, k
        self.device = device
        self.ep = ep  # expert-parallel rows (k = 1, no per-slot output region): sized by moeb_ep_workspace_bytes
        self.T = 0
        self.buf = None
        self._lock = threading.Lock()  # callers on several threads must not see a buffer before it is zeroed

    def get(self, T):
        with self._lock:
            if T > self.T:
                Tn = max(T, 2 * self.T, 16)
                if self.ep:
                    nbytes = _lib.load().moeb_ep_workspace_bytes(Tn, self.d, self.f, self.E)
                else:
                    nbytes = _lib.load().moeb_workspace_bytes(Tn, self.d, self.f, self.E, self.k)
                buf = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
                _lib.call("moeb_workspace_init", _p(buf), nbytes, _stream())
                self.buf, self.T = buf, Tn
            return self.buf

    def for_k(self, k):
        """This workspace if it was sized for k slots per token, else a new one for k (the layout depends on k)."""
        return self if self.k == k else Workspace(self.d, self.f, self.E, k, self.device, self.ep)

    def read_error(self):
        """Sticky device error bits (MOEB_DEVERR_*); synchronises the current stream and clears them."""
        if self.buf is None:
            return 0
        out = ctypes.c_uint(0)
        _lib.call("moeb_read_error", _p(self.buf), ctypes.byref(out), _stream())
        return out.value


# ------------------------------------------------------------------ quantizers
def quantize_q4(w):
    """bf16 [..., N, K] -> (q int32 [..., N, K/8], sb int32 [..., N, K/64]) in the B200 layout."""
    _need(w, torch.bfloat16, "w")
    K = w.shape[-1]
    rows = w.numel() // K
    q = torch.empty(*w.shape[:-1], K // 8, dtype=torch.int32, device=w.device)
    sb = torch.empty(*w.shape[:-1], K // 64, dtype=torch.int32, device=w.device)
    _lib.call("moeb_quantize_q4", _p(w), rows, K, _p(q), _p(sb), _stream())
    return q, sb


def dequant_q4(q, sb):
    _need(q, torch.int32, "q")
    _need(sb, torch.int32, "sb")
    K = q.shape[-1] * 8
    rows = q.numel() // q.shape[-1]
    out = torch.empty(*q.shape[:-1], K, dtype=torch.float32, device=q.device)
    _lib.call("moeb_dequant_q4", _p(q), _p(sb), rows, K, _p(out), _stream())
    return out


def q4_from_mlx(wq, scales, biases):
    """mlx affine state (uint32 natural nibble order as int32, bf16 scales, bf16 biases) -> (q, sb)."""
    _need(wq, torch.int32, "wq")
    _need(scales, torch.bfloat16, "scales")
    _need(biases, torch.bfloat16, "biases")
    K = wq.shape[-1] * 8
    rows = wq.numel() // wq.shape[-1]
    q = torch.empty_like(wq)
    sb = torch.empty(*wq.shape[:-1], K // 64, dtype=torch.int32, device=wq.device)
    _lib.call("moeb_q4_from_mlx", _p(wq), _p(scales), _p(biases), rows, K, _p(q), _p(sb), _stream())
    return q, sb


def quantize_mxfp4(w):
    """bf16 [..., N, K] -> (q int32 [..., N, K/8], sc uint8 [..., N, K/32]) in the B200 layout."""
    _need(w, torch.bfloat16, "w")
    K = w.shape[-1]
    rows = w.numel() // K
    q = torch.empty(*w.shape[:-1], K // 8, dtype=torch.int32, device=w.device)
    sc = torch.empty(*w.shape[:-1], K // 32, dtype=torch.uint8, device=w.device)
    _lib.call("moeb_quantize_mxfp4", _p(w), rows, K, _p(q), _p(sc), _stream())
    return q, sc


def dequant_mxfp4(q, sc):
    _need(q, torch.int32, "q")
    _need(sc, torch.uint8, "sc")
    K = q.shape[-1] * 8
    rows = q.numel() // q.shape[-1]
    out = torch.empty(*q.shape[:-1], K, dtype=torch.float32, device=q.device)
    _lib.call("moeb_dequant_mxfp4", _p(q), _p(sc), rows, K, _p(out), _stream())
    return out


def mxfp4_from_mlx(wq, scales):
    _need(wq, torch.int32, "wq")
    _need(scales, torch.uint8, "scales")
    K = wq.shape[-1] * 8
    rows = wq.numel() // wq.shape[-1]
    q = torch.empty_like(wq)
    sc = torch.empty_like(scales)
    _lib.call("moeb_mxfp4_from_mlx", _p(wq), _p(scales), rows, K, _p(q), _p(sc), _stream())
    return q, sc


# ------------------------------------------------------------------ router
_ROUTER_WS = {}
_ROUTER_LOCK = threading.Lock()


def router(x, gate_w, k, gate_b=None, norm=True, scale=1.0, return_logits=False):
    """x bf16 [T, d], gate_w bf16 [E, d], gate_b bf16 [E] -> idx int32 [T, k], wts fp32 [T, k] (+ logits)."""
    _need(x, torch.bfloat16, "x")
    _need(gate_w, torch.bfloat16, "gate_w")
    _need(gate_b, torch.bfloat16, "gate_b")
    T, d = x.shape
    E = gate_w.shape[0]
    idx = torch.empty(T, k, dtype=torch.int32, device=x.device)
    wts = torch.empty(T, k, dtype=torch.float32, device=x.device)
    logits = torch.empty(T, E, dtype=torch.float32, device=x.device) if return_logits else None
    key = (x.device, d, E, k)
    with _ROUTER_LOCK:
        ws = _ROUTER_WS.get(key)
        if ws is None:
            ws = _ROUTER_WS[key] = Workspace(d, 64, E, k, x.device)
    buf = ws.get(max(T, 1))
    _lib.call("moeb_router", _p(x), _p(gate_w), _p(gate_b), T, d, E, k, int(bool(norm)), float(scale), _p(idx),
              _p(wts), _p(logits), _p(buf), buf.numel(), _stream())
    return (idx, wts, logits) if return_logits else (idx, wts)


def route_tables(idx, E, nt):
    """The routing step alone (moeb_route_tables): idx int32 [T, k] -> (counts [E], offsets [E], sorted [T*k],
    tiles [ntiles, 4]) int32, plus the device error bits (MOEB_DEVERR_*). For bit-exact checks of the tile builder."""
    _need(idx, torch.int32, "idx")
    T, k = idx.shape
    dev = idx.device
    counts = torch.empty(E, dtype=torch.int32, device=dev)
    offsets = torch.empty(E, dtype=torch.int32, device=dev)
    sorted_ = torch.empty(max(T * k, 1), dtype=torch.int32, device=dev)
    tiles = torch.empty(T * k + E, 4, dtype=torch.int32, device=dev)
    ntiles = torch.empty(1, dtype=torch.int32, device=dev)
    ws = Workspace(64, 64, E, k, dev)
    buf = ws.get(max(T, 1))
    _lib.call("moeb_route_tables", _p(idx), T, k, E, int(nt), _p(counts), _p(offsets), _p(sorted_), _p(tiles),
              _p(ntiles), _p(buf), buf.numel(), _stream())
    n = int(ntiles.item())
    return counts, offsets, sorted_[:T * k], tiles[:n], ws.read_error()


# ------------------------------------------------------------------ experts / layer (int4)
def _expert_ptrs(state):
    (qg, sg), (qu, su), (qd, sd) = state["g"], state["u"], state["d"]
    return [_p(qg), _p(sg), _p(qu), _p(su), _p(qd), _p(sd), _p(state.get("bg")), _p(state.get("bu")),
            _p(state.get("bd"))]


def _fmt(state):
    return state.get("fmt", "q4")


def experts_q4(state, x, idx, wts, act=0, policy=POLICY_AUTO, residual=None):
    """y = sum_j wts * expert(x) (+ residual), bf16 [T, d]. The state's format picks the int4 or MXFP4 entry."""
    _need(x, torch.bfloat16, "x")
    _need(idx, torch.int32, "idx")
    _need(wts, torch.float32, "wts")
    _need(residual, torch.bfloat16, "residual")
    T, d = x.shape
    k = idx.shape[1]
    E, f = state["E"], state["f"]
    ws = state["ws"] = state["ws"].for_k(k)
    buf = ws.get(max(T, 1))
    y = torch.empty_like(x)
    fn = "moeb_experts_mxfp4" if _fmt(state) == "mxfp4" else "moeb_experts_q4"
    _lib.call(fn, _p(x), *_expert_ptrs(state), _p(idx), _p(wts), T, d, f, E, k, int(act),
              int(policy), _p(residual), _p(y), _p(buf), buf.numel(), _stream())
    return y


experts = experts_q4


def layer_q4(state, x, gate_w, k, gate_b=None, norm=True, rscale=1.0, act=0, policy=POLICY_AUTO, residual=None,
             return_routing=False, stage_events=None, n_shared=0):
    """The layer call (x, gate weights, packed experts, k) -> y: router + routing + experts + combine.
    stage_events: optional 4 torch.cuda.Event (before router, after router, after gate/up, after down).
    n_shared: the state's last n_shared experts are always-on shared experts (int4 only); the routing returned
    then has k + n_shared slots per token."""
    _need(x, torch.bfloat16, "x")
    _need(gate_w, torch.bfloat16, "gate_w")
    _need(gate_b, torch.bfloat16, "gate_b")
    _need(residual, torch.bfloat16, "residual")
    T, d = x.shape
    E, f = state["E"], state["f"]
    ks = k + n_shared
    state["ws"] = state["ws"].for_k(ks)
    buf = state["ws"].get(max(T, 1))
    y = torch.empty_like(x)
    idx = torch.empty(T, ks, dtype=torch.int32, device=x.device) if return_routing else None
    wts = torch.empty(T, ks, dtype=torch.float32, device=x.device) if return_routing else None
    evp = None
    if stage_events is not None:
        for ev in stage_events:
            if ev.cuda_event == 0:
                ev.record()  # creates the underlying cudaEvent_t
        evp = (ctypes.c_void_p * 4)(*[ctypes.c_void_p(ev.cuda_event) for ev in stage_events])
    if n_shared:
        if _fmt(state) != "q4":
            raise ValueError("shared experts are supported for int4 states")
        _lib.call("moeb_layer_q4_shared", _p(x), _p(gate_w), _p(gate_b), int(bool(norm)), float(rscale),
                  int(n_shared), *_expert_ptrs(state), T, d, f, E - n_shared, k, int(act), int(policy),
                  _p(residual), _p(y), _p(idx), _p(wts), evp, _p(buf), buf.numel(), _stream())
    else:
        fn = "moeb_layer_mxfp4" if _fmt(state) == "mxfp4" else "moeb_layer_q4"
        _lib.call(fn, _p(x), _p(gate_w), _p(gate_b), int(bool(norm)), float(rscale), *_expert_ptrs(state),
                  T, d, f, E, k, int(act), int(policy), _p(residual), _p(y), _p(idx), _p(wts), evp, _p(buf),
                  buf.numel(), _stream())
    return (y, idx, wts) if return_routing else y


layer = layer_q4


def policy(T, E, k):
    return _lib.load().moeb_policy(T, E, k)


# ------------------------------------------------------------------ expert parallelism (device steps)
def ep_dispatch(x, idx, wts, E, P, ws):
    """Sort the T*k slots by owning rank and pack their send rows (x row + {local expert, weight} tail).
    Returns rows bf16 [T*k, d + 8] (the first sum(send_counts) are valid), send_counts int32 [P] and
    slot_pos int32 [T*k]. ws: any Workspace (its error word records invalid ids)."""
    _need(x, torch.bfloat16, "x")
    _need(idx, torch.int32, "idx")
    _need(wts, torch.float32, "wts")
    T, d = x.shape
    k = idx.shape[1]
    rows = torch.empty(T * k, d + 8, dtype=torch.bfloat16, device=x.device)
    send_counts = torch.empty(P, dtype=torch.int32, device=x.device)
    slot_pos = torch.empty(T * k, dtype=torch.int32, device=x.device)
    buf = ws.get(1)
    _lib.call("moeb_ep_dispatch", _p(x), _p(idx), _p(wts), T, d, k, E, P, _p(rows), _p(send_counts),
              _p(slot_pos), _p(buf), buf.numel(), _stream())
    return rows, send_counts, slot_pos


def ep_experts(state, rows, act=0, policy=POLICY_AUTO):
    """The local experts on received rows (bf16 [R, d + 8]) -> yp fp32 [R, d], weight * (W_down h + b_down)."""
    _need(rows, torch.bfloat16, "rows")
    R, d = rows.shape[0], rows.shape[1] - 8
    yp = torch.empty(R, d, dtype=torch.float32, device=rows.device)
    if R == 0:
        return yp
    buf = state["ep_ws"].get(R)
    fn = "moeb_ep_experts_mxfp4" if _fmt(state) == "mxfp4" else "moeb_ep_experts_q4"
    _lib.call(fn, _p(rows), R, d, state["f"], state["E"], *_expert_ptrs(state), int(act), int(policy), _p(yp),
              _p(buf), buf.numel(), _stream())
    return yp


def ep_combine(back, slot_pos, T, k, residual=None):
    """y bf16 [T, d] = sum_j back[slot_pos[t*k + j]] (fixed j order) + residual."""
    _need(back, torch.float32, "back")
    _need(slot_pos, torch.int32, "slot_pos")
    _need(residual, torch.bfloat16, "residual")
    d = back.shape[1]
    y = torch.empty(T, d, dtype=torch.bfloat16, device=back.device)
    _lib.call("moeb_ep_combine", _p(back), _p(slot_pos), T, d, k, _p(residual), _p(y), _stream())
    return y


# ------------------------------------------------------------------ expert parallelism over peer memory
def ep_p2p_dispatch(x, idx, wts, E, xch, Cs=0):
    """Route this rank's slots straight into the owners' exchange buffers. Returns slot_pos int32 [T*k] in
    block layout (owner * Cs + row) for the combine. Cs: this call's rows per source block (0 = capacity)."""
    _need(x, torch.bfloat16, "x")
    _need(idx, torch.int32, "idx")
    _need(wts, torch.float32, "wts")
    T, d = x.shape
    k = idx.shape[1]
    send_counts = torch.empty(xch.P, dtype=torch.int32, device=x.device)
    slot_pos = torch.empty(T * k, dtype=torch.int32, device=x.device)
    _lib.call("moeb_ep_p2p_dispatch", _p(x), _p(idx), _p(wts), T, d, k, E, xch.P, xch.me, xch.C, int(Cs),
              _p(xch.peers), ctypes.c_void_p(xch.base), _p(send_counts), _p(slot_pos), _stream())
    return slot_pos


def ep_p2p_experts(state, xch, act=0, policy=POLICY_AUTO, Cs=0):
    """This rank's experts on the rows every source sent it; outputs go straight back to the owners."""
    if _fmt(state) != "q4":
        raise ValueError("the peer-memory exchange runs int4 states")
    Cs = Cs or xch.C
    buf = state["ep_ws"].get(xch.P * Cs)
    _lib.call("moeb_ep_p2p_experts_q4", _p(xch.peers), ctypes.c_void_p(xch.base), xch.P, xch.me, xch.C, int(Cs),
              state["dm"], state["f"], state["E"], *_expert_ptrs(state), int(act), int(policy), _p(buf),
              buf.numel(), _stream())


def ep_p2p_combine(xch, slot_pos, T, k, d, residual=None, device=None):
    _need(residual, torch.bfloat16, "residual")
    y = torch.empty(T, d, dtype=torch.bfloat16, device=device or slot_pos.device)
    _lib.call("moeb_ep_p2p_combine", ctypes.c_void_p(xch.base), _p(slot_pos), xch.P, xch.C, T, d, k,
              _p(residual), _p(y), _stream())
    return y
