"""CPU oracle for moe-lab's quantized MoE-layer forward.

TEST INFRASTRUCTURE ONLY: imported by tests/, by __graft_entry__.smoke() (as the checker) and by bench.py's
CPU-baseline / reference arm. The product path (moelab_b200) never imports it.

numpy/ctypes wrappers around moe_oracle.c plus torch restatements of the reference's CPU paths:
  reference_fp32   moelab/torch_backend.py:57-67  (fp32 loop over unique experts)
  reference_fp64   moelab/problem.py:67-85        (fp64 loop over experts)
  torch_loop_run   moelab/variants/cuda/torch_loop.py:11-18 (HF-style eager loop; the CPU baseline)
  router_stock     moelab/e2e.py:58-63 (softmax precise -> top-k -> renormalise) and :171-176 (gpt-oss)
Parity: the MoE math is pinned by tests/golden (vectors produced by the reference's own Python code);
the int4/MXFP4 quantizers restate mlx's published algorithm and are unpinned against MLX itself.
"""
import ctypes
import os
import subprocess

import numpy as np
import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libmoe_oracle.so")
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_u32p = ctypes.POINTER(ctypes.c_uint32)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_i32p = ctypes.POINTER(ctypes.c_int32)
_i64 = ctypes.c_int64


def build():
    """Compile moe_oracle.c (make). Idempotent."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(
                os.path.join(_HERE, "moe_oracle.c")):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.orc_q4_quantize.argtypes = [_u16p, _i64, _i64, _u32p, _u16p, _u16p]
        L.orc_q4_dequant.argtypes = [_u32p, _u16p, _u16p, _i64, _i64, _f32p]
        L.orc_mxfp4_quantize.argtypes = [_u16p, _i64, _i64, _u32p, _u8p]
        L.orc_mxfp4_dequant.argtypes = [_u32p, _u8p, _i64, _i64, _f32p]
        L.orc_router_logits.argtypes = [_u16p, _u16p, _u16p, _i64, _i64, _i64, _f32p]
        L.orc_topk.argtypes = [_f32p, _i64, _i64, ctypes.c_int, ctypes.c_int, ctypes.c_float, _i32p, _f32p]
        L.orc_moe_forward.argtypes = [_f32p] * 7 + [_i32p, _f32p, _i64, _i64, _i64, _i64, ctypes.c_int,
                                                    ctypes.c_int, ctypes.c_int, _f32p]
        L.orc_f32_to_bf16.argtypes = [ctypes.c_float]
        L.orc_f32_to_bf16.restype = ctypes.c_uint16
        _lib = L
    return _lib


def _p(a, t):
    return a.ctypes.data_as(t) if a is not None else None


def bf16_bits(t):
    """torch bf16 tensor (any device) or uint16 array -> contiguous numpy uint16 of the bf16 bit patterns."""
    if isinstance(t, np.ndarray):
        assert t.dtype == np.uint16
        return np.ascontiguousarray(t)
    return np.ascontiguousarray(t.detach().to("cpu", torch.bfloat16).contiguous().view(torch.int16).numpy()
                                .view(np.uint16))


def bits_to_f32(u16):
    return (np.asarray(u16, np.uint16).astype(np.uint32) << 16).view(np.float32)


# ------------------------------------------------------------------ quantizers (natural mlx layout)
def q4_quantize(w):
    """w: bf16 [..., K] -> (qw uint32 [..., K/8], scales uint16 [..., K/64], biases uint16 [..., K/64])."""
    wb = bf16_bits(w)
    shp, K = wb.shape[:-1], wb.shape[-1]
    rows = int(np.prod(shp)) if shp else 1
    assert K % 64 == 0
    qw = np.zeros(shp + (K // 8,), np.uint32)
    s = np.zeros(shp + (K // 64,), np.uint16)
    b = np.zeros(shp + (K // 64,), np.uint16)
    lib().orc_q4_quantize(_p(wb, _u16p), rows, K, _p(qw, _u32p), _p(s, _u16p), _p(b, _u16p))
    return qw, s, b


def q4_dequant(qw, s, b):
    qw, s, b = (np.ascontiguousarray(a) for a in (qw, s, b))
    shp, K = qw.shape[:-1], qw.shape[-1] * 8
    rows = int(np.prod(shp)) if shp else 1
    out = np.zeros(shp + (K,), np.float32)
    lib().orc_q4_dequant(_p(qw, _u32p), _p(s, _u16p), _p(b, _u16p), rows, K, _p(out, _f32p))
    return out


def mxfp4_quantize(w):
    """w: bf16 [..., K] -> (qw uint32 [..., K/8], scales uint8 [..., K/32])."""
    wb = bf16_bits(w)
    shp, K = wb.shape[:-1], wb.shape[-1]
    rows = int(np.prod(shp)) if shp else 1
    assert K % 32 == 0
    qw = np.zeros(shp + (K // 8,), np.uint32)
    s = np.zeros(shp + (K // 32,), np.uint8)
    lib().orc_mxfp4_quantize(_p(wb, _u16p), rows, K, _p(qw, _u32p), _p(s, _u8p))
    return qw, s


def mxfp4_dequant(qw, s):
    qw, s = np.ascontiguousarray(qw), np.ascontiguousarray(s)
    shp, K = qw.shape[:-1], qw.shape[-1] * 8
    rows = int(np.prod(shp)) if shp else 1
    out = np.zeros(shp + (K,), np.float32)
    lib().orc_mxfp4_dequant(_p(qw, _u32p), _p(s, _u8p), rows, K, _p(out, _f32p))
    return out


# ------------------------------------------------------------------ router
def router_logits(x, wg, bias=None):
    """fp32 logits in the CUDA router's summation order (bit-exact target). x [T,d], wg [E,d] bf16."""
    xb, wb = bf16_bits(x), bf16_bits(wg)
    bb = bf16_bits(bias) if bias is not None else None
    T, d = xb.shape
    E = wb.shape[0]
    out = np.zeros((T, E), np.float32)
    lib().orc_router_logits(_p(xb, _u16p), _p(wb, _u16p), _p(bb, _u16p), T, E, d, _p(out, _f32p))
    return out


def topk(logits, k, norm=True, scale=1.0):
    lg = np.ascontiguousarray(logits, np.float32)
    T, E = lg.shape
    idx = np.zeros((T, k), np.int32)
    w = np.zeros((T, k), np.float32)
    lib().orc_topk(_p(lg, _f32p), T, E, k, int(bool(norm)), float(scale), _p(idx, _i32p), _p(w, _f32p))
    return idx, w


def router(x, wg, k, bias=None, norm=True, scale=1.0):
    return topk(router_logits(x, wg, bias), k, norm, scale)


def router_stock(x, wg, k, bias=None, norm=True):
    """The stock routing sequence in fp64: softmax over all E -> k largest -> renormalise (norm) or keep the
    full-softmax probabilities (e2e.py:58-63, :136-140, :171-176). Returns (idx, wts, logits64)."""
    x64 = bits_to_f32(bf16_bits(x)).astype(np.float64)
    w64 = bits_to_f32(bf16_bits(wg)).astype(np.float64)
    lg = x64 @ w64.T
    if bias is not None:
        lg = lg + bits_to_f32(bf16_bits(bias)).astype(np.float64)
    idx = np.argsort(-lg, axis=1, kind="stable")[:, :k].astype(np.int32)
    p = np.exp(lg - lg.max(1, keepdims=True))
    p /= p.sum(1, keepdims=True)
    w = np.take_along_axis(p, idx, 1)
    if norm:
        w = w / w.sum(1, keepdims=True)
    return idx, w.astype(np.float32), lg


# ------------------------------------------------------------------ MoE references
def moe_forward(x, wg, wu, wd, idx, wts, act=0, bg=None, bu=None, bd=None, h_round=False):
    """fp64-accumulated MoE forward on fp32 weights (C). Arrays are numpy; x fp32 [T,d]."""
    f32 = lambda a: None if a is None else np.ascontiguousarray(np.asarray(a, np.float32))  # noqa: E731
    x, wg, wu, wd, bg, bu, bd, wts = map(f32, (x, wg, wu, wd, bg, bu, bd, wts))
    idx = np.ascontiguousarray(np.asarray(idx, np.int32))
    T, d = x.shape
    E, f, _ = wg.shape
    k = idx.shape[1]
    y = np.zeros((T, d), np.float32)
    lib().orc_moe_forward(_p(x, _f32p), _p(wg, _f32p), _p(wu, _f32p), _p(wd, _f32p), _p(bg, _f32p),
                          _p(bu, _f32p), _p(bd, _f32p), _p(idx, _i32p), _p(wts, _f32p), T, d, f, E, k, act,
                          int(bool(h_round)), _p(y, _f32p))
    return y


@torch.no_grad()
def reference_fp32(wg, wu, wd, x, idx, wts, act=0, bg=None, bu=None, bd=None):
    """Restates moelab/torch_backend.py:57-67 (fp32 loop over unique experts, index_add_), extended with the
    gpt-oss biases/clamp of metal_mxfp4_gptoss.py:110-126 (act=2) and tanh-GELU (act=1). CPU torch."""
    x32 = x.detach().float().cpu()
    idx, wts = idx.cpu(), wts.float().cpu()
    y = torch.zeros_like(x32)
    for e in idx.unique().tolist():
        t, j = (idx == e).nonzero(as_tuple=True)
        xe = x32[t]
        g, u = xe @ wg[e].float().cpu().T, xe @ wu[e].float().cpu().T
        if bg is not None:
            g, u = g + bg[e].float().cpu(), u + bu[e].float().cpu()
        if act == 2:
            g, u = g.clamp(max=7.0), u.clamp(-7.0, 7.0)
            h = g * torch.sigmoid(1.702 * g) * (u + 1)
        elif act == 1:
            h = torch.nn.functional.gelu(g, approximate="tanh") * u
        else:
            h = torch.nn.functional.silu(g) * u
        o = h @ wd[e].float().cpu().T
        if bd is not None:
            o = o + bd[e].float().cpu()
        y.index_add_(0, t, o * wts[t, j, None])
    return y


def reference_fp64(p):
    """Restates moelab/problem.py:67-85: fp64 loop over experts on a numpy problem dict."""
    x = p["x"].astype(np.float64)
    T, d = x.shape
    y = np.zeros((T, d))
    for e in np.unique(p["idx"]):
        t, j = np.nonzero(p["idx"] == e)
        xe = x[t]
        g = xe @ p["w_gate"][e].T.astype(np.float64)
        u = xe @ p["w_up"][e].T.astype(np.float64)
        h = g / (1.0 + np.exp(-g)) * u
        o = h @ p["w_down"][e].T.astype(np.float64)
        np.add.at(y, t, o * p["wts"][t, j][:, None])
    return y.astype(np.float32)


@torch.no_grad()
def torch_loop_run(s, x, idx, wts):
    """Port of moelab/variants/cuda/torch_loop.py:11-18 (the reference's CPU torch path): eager loop over the
    active experts, x.dtype math, routing weights cast to x.dtype. s = {"wg","wu","wd"} dense weights."""
    y = torch.zeros_like(x)
    for e in idx.unique().tolist():
        t, j = (idx == e).nonzero(as_tuple=True)
        xe = x[t]
        h = torch.nn.functional.silu(xe @ s["wg"][e].T) * (xe @ s["wu"][e].T)
        y.index_add_(0, t, (h @ s["wd"][e].T) * wts[t, j, None].to(x.dtype))
    return y


@torch.no_grad()
def torch_router_stock(x, wg, k, bias=None, norm=True):
    """Torch restatement of the stock routing (e2e.py:58-63): softmax in fp32 over bf16 logits, top-k,
    renormalise. Used by the CPU baseline arm together with torch_loop_run."""
    lg = x @ wg.T
    if bias is not None:
        lg = lg + bias
    g = torch.softmax(lg.float(), dim=-1)
    w, i = torch.topk(g, k, dim=-1)
    if norm:
        w = w / w.sum(-1, keepdim=True)
    return i.to(torch.int32), w


def error_metrics(y, y_ref):
    """Restates moelab/problem.py:88-98 plus the north-star bound max|err| / row max|ref|."""
    y = np.asarray(y, dtype=np.float64)
    r = np.asarray(y_ref, dtype=np.float64)
    diff = y - r
    nr = np.linalg.norm(r) + 1e-30
    rowmax = np.abs(r).max(axis=-1, keepdims=True) + 1e-30
    return {
        "rel_fro": float(np.linalg.norm(diff) / nr),
        "max_abs": float(np.abs(diff).max()) if diff.size else 0.0,
        "max_rowrel": float((np.abs(diff) / rowmax).max()) if diff.size else 0.0,
        "cos": float((y * r).sum() / (np.linalg.norm(y) * nr + 1e-30)),
        "finite": bool(np.isfinite(y).all()),
    }


# ------------------------------------------------------------------ routing step (integer work)
SLOT_SKIP = -(2 ** 31)


def route_tables(idx, E, nt):
    """Restatement of the routing step (moelab_b200's tile builder) on the CPU: the T*k slots grouped by expert
    with a stable sort, each expert's run cut every nt slots. Ids outside [0, E) are grouped under expert 0 (and
    reported as `bad`); SLOT_SKIP entries are left out.
    Returns counts [E], offsets [E], sorted slot ids, tiles [n, 4] {expert, start, n, 0} (experts in increasing
    order) and bad (any invalid id) - all int32 / bool.
    The grouping contract is that of the reference's map kernel (moelab/variants/mlx/metal_q4_tiles_v2.py:362-373):
    slot p starts a tile iff its rank among the earlier slots of the same expert is a multiple of VT, and the tile
    holds the next <= VT slots of that expert in slot order."""
    ids = np.asarray(idx, np.int64).reshape(-1)
    keep = ids != SLOT_SKIP
    bad = bool(((ids < 0) | (ids >= E))[keep].any())
    e = np.where((ids < 0) | (ids >= E), 0, ids)
    slots = np.nonzero(keep)[0]
    ek = e[keep]
    order = np.argsort(ek, kind="stable")
    sorted_ = slots[order].astype(np.int32)
    counts = np.bincount(ek, minlength=E).astype(np.int32)
    offsets = (np.cumsum(counts) - counts).astype(np.int32)
    tiles = []
    for x in range(E):
        for i in range(0, int(counts[x]), nt):
            tiles.append((x, int(offsets[x]) + i, min(nt, int(counts[x]) - i), 0))
    return counts, offsets, sorted_, np.asarray(tiles, np.int32).reshape(-1, 4), bad


def reference_map_tiles(idx, VT):
    """The reference's map kernel as a set of tiles (metal_q4_tiles_v2.py:362-373): for every slot p whose rank
    among the earlier same-expert slots is a multiple of VT, the tuple (expert, next <= VT same-expert slots from p
    in slot order). Valid ids only (the reference has no invalid-id path)."""
    ids = np.asarray(idx, np.int64).reshape(-1)
    seen = {}
    out = set()
    for p, e in enumerate(ids):
        r = seen.get(int(e), 0)
        seen[int(e)] = r + 1
        if r % VT == 0:
            mem = [q for q in range(p, len(ids)) if ids[q] == e][:VT]
            out.add((int(e), tuple(mem)))
    return out
