"""Checkpoint loader: MoE expert weights from safetensors files into the B200 state.

Two on-disk formats of the reference's real-checkpoint path (moelab/e2e.py:48-49, :163;
tests/test_real_checkpoints.py:36-66):
  - mlx-community affine int4 triplets, per projection `{prefix}{gate,up,down}_proj.{weight,scales,biases}`:
    weight uint32 [E, N, K/8] (element 8j+i at nibble i of word j), scales / biases bf16 [E, N, K/64];
    prefix `model.layers.{L}.mlp.switch_mlp.` (Qwen3-MoE, Mixtral, DeepSeek routed experts);
  - MXFP4 (gpt-oss): mlx-community `{prefix}{gate,up,down}_proj.{weight,scales,bias}` (weight uint32 [E, N, K/8]
    E2M1 codes, scales uint8 [E, N, K/32] E8M0) with prefix `model.layers.{L}.mlp.experts.`, or the OCP / Hugging
    Face layout `gate_up_proj_blocks` uint8 [E, 2f, K/32, 16] (two E2M1 codes per byte, low nibble first; gate and up
    rows interleaved, gate at even rows), `gate_up_proj_scales` uint8 [E, 2f, K/32], `gate_up_proj_bias`, and
    `down_proj_{blocks,scales,bias}`.
The safetensors container (an 8-byte little-endian header size, a JSON header of name -> dtype / shape / byte range,
then the raw data) is read here with numpy memory maps; sharded checkpoints are followed through
`model.safetensors.index.json`. The converted tensors go through the library's own layout converters
(moeb_q4_from_mlx / moeb_mxfp4_from_mlx), so the state equals what prepare() builds from the dequantised weights.
"""
import json
import os
import struct

import numpy as np
import torch

from . import ops

_DT = {"U8": np.uint8, "I8": np.int8, "U16": np.uint16, "I16": np.int16, "U32": np.uint32, "I32": np.int32,
       "U64": np.uint64, "I64": np.int64, "F16": np.float16, "F32": np.float32, "F64": np.float64,
       "BF16": np.uint16}  # bf16 carried as its bit pattern


def read_header(path):
    """{name: (dtype string, shape, (begin, end) byte range in the data section)} and the data section's offset."""
    with open(path, "rb") as fh:
        n = struct.unpack("<Q", fh.read(8))[0]
        hdr = json.loads(fh.read(n))
    hdr.pop("__metadata__", None)
    return {k: (v["dtype"], tuple(v["shape"]), tuple(v["data_offsets"])) for k, v in hdr.items()}, 8 + n


def load_tensor(path, name, header=None):
    """One tensor as a numpy array (bf16 as uint16 bits); memory-mapped, copied on conversion."""
    header = header or read_header(path)
    meta, base = header
    if name not in meta:
        raise KeyError(f"{name} not in {path}")
    dt, shape, (b, e) = meta[name]
    if dt not in _DT:
        raise ValueError(f"{name}: unsupported safetensors dtype {dt}")
    arr = np.memmap(path, dtype=np.uint8, mode="r", offset=base + b, shape=(e - b,))
    return arr.view(_DT[dt]).reshape(shape)


def write_safetensors(path, tensors):
    """Write {name: numpy array} (uint16 arrays named in `bf16` are stored as BF16) - used by the tests' synthetic
    checkpoints. tensors: {name: (array, dtype string)}."""
    meta, blobs, off = {}, [], 0
    for name, (arr, dt) in tensors.items():
        raw = np.ascontiguousarray(arr).tobytes()
        meta[name] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    h = json.dumps(meta).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as fh:
        fh.write(struct.pack("<Q", len(h)))
        fh.write(h)
        for b in blobs:
            fh.write(b)


class Checkpoint:
    """A safetensors checkpoint: one file, or a directory with model.safetensors.index.json (shards)."""

    def __init__(self, path):
        self.files = {}
        if os.path.isdir(path):
            idx = os.path.join(path, "model.safetensors.index.json")
            if os.path.exists(idx):
                wm = json.load(open(idx))["weight_map"]
                self.where = {k: os.path.join(path, v) for k, v in wm.items()}
            else:
                single = os.path.join(path, "model.safetensors")
                self.where = {k: single for k in read_header(single)[0]}
        else:
            self.where = {k: path for k in read_header(path)[0]}

    def __contains__(self, name):
        return name in self.where

    def get(self, name):
        f = self.where.get(name)
        if f is None:
            raise KeyError(name)
        if f not in self.files:
            self.files[f] = read_header(f)
        return load_tensor(f, name, self.files[f])


def _cuda(a, dtype):
    """numpy array -> CUDA tensor of `dtype` with the same bits (unsigned integers go through their signed view)."""
    a = np.ascontiguousarray(a)
    signed = {np.dtype(np.uint32): np.int32, np.dtype(np.uint16): np.int16, np.dtype(np.uint64): np.int64}
    if a.dtype in signed:
        a = a.view(signed[a.dtype])
    return torch.from_numpy(a).to("cuda").view(dtype)


def q4_layer_state(ckpt, layer, prefix="model.layers.{L}.mlp.switch_mlp."):
    """b200_q4_moe state of one layer's routed experts from mlx affine int4 (group size 64) triplets."""
    ck = ckpt if isinstance(ckpt, Checkpoint) else Checkpoint(ckpt)
    p = prefix.format(L=layer)
    st = {}
    for n, pr in (("g", "gate_proj"), ("u", "up_proj"), ("d", "down_proj")):
        w, s, b = (ck.get(f"{p}{pr}.{x}") for x in ("weight", "scales", "biases"))
        if w.shape[-1] * 8 != s.shape[-1] * 64:
            raise ValueError(f"{p}{pr}: not 4-bit with group size 64 (weight {w.shape}, scales {s.shape})")
        st[n] = ops.q4_from_mlx(_cuda(w, torch.int32), _cuda(s, torch.bfloat16), _cuda(b, torch.bfloat16))
    E, f, d = st["g"][0].shape[0], st["g"][0].shape[1], st["g"][0].shape[2] * 8
    st.update(E=E, f=f, dm=d, ws=ops.Workspace(d, f, E, 0, torch.device("cuda")))
    return st


def gate_weight(ckpt, layer, name="model.layers.{L}.mlp.gate"):
    """The router gate of one layer as bf16 [E, d]: a plain weight, or mlx affine-quantized (weight / scales /
    biases, bits from the packed width) dequantised on the host in fp32 and rounded once to bf16."""
    ck = ckpt if isinstance(ckpt, Checkpoint) else Checkpoint(ckpt)
    n = name.format(L=layer)
    w = ck.get(f"{n}.weight")
    if f"{n}.scales" not in ck:
        return _cuda(w, torch.bfloat16) if w.dtype == np.uint16 else torch.from_numpy(np.asarray(w)).cuda().bfloat16()
    deq = dequant_affine(np.asarray(w), np.asarray(ck.get(f"{n}.scales")), np.asarray(ck.get(f"{n}.biases")))
    return torch.from_numpy(deq).cuda().bfloat16()


def dequant_affine(w, scales, biases, group=64):
    """mlx affine dequantisation on the host (fp32): w uint32 [N, K*bits/32] (element i of a word at bits
    i*bits), scales / biases bf16 bits [N, K/group]; bits from the packed width."""
    N, G = scales.shape
    bits = w.shape[1] * 32 // (G * group)
    per = 32 // bits
    codes = (w.astype(np.uint32)[:, :, None] >> (np.arange(per, dtype=np.uint32) * bits)) & ((1 << bits) - 1)
    s = (scales.astype(np.uint32) << 16).view(np.float32)
    b = (biases.astype(np.uint32) << 16).view(np.float32)
    q = codes.reshape(N, G, group).astype(np.float32)
    return (q * s[:, :, None] + b[:, :, None]).reshape(N, G * group)


def ocp_blocks_to_words(blocks):
    """OCP MXFP4 blocks uint8 [..., K/32, 16] (two E2M1 codes per byte, low nibble = even element) -> mlx packed
    words uint32 [..., K/8] (element 8j+i at nibble i): the same bytes read as little-endian words."""
    b = np.ascontiguousarray(blocks)
    return b.reshape(*b.shape[:-2], b.shape[-2] * 16).view(np.uint32)


def mxfp4_layer_state(ckpt, layer, prefix="model.layers.{L}.mlp.experts.", act=1):
    """b200_mxfp4_gptoss state (fp32 biases; act 1 = the gpt-oss variant's clamped SwiGLU) of one gpt-oss layer,
    from mlx-community tensors or the OCP / Hugging Face blocks layout."""
    ck = ckpt if isinstance(ckpt, Checkpoint) else Checkpoint(ckpt)
    p = prefix.format(L=layer)
    st = {}
    if f"{p}gate_up_proj_blocks" in ck:  # OCP / HF: gate and up interleaved along the output rows
        gu_w = ocp_blocks_to_words(ck.get(f"{p}gate_up_proj_blocks"))
        gu_s = np.asarray(ck.get(f"{p}gate_up_proj_scales"))
        gu_b = np.asarray(ck.get(f"{p}gate_up_proj_bias"))
        dn_w = ocp_blocks_to_words(ck.get(f"{p}down_proj_blocks"))
        trip = {"g": (gu_w[:, 0::2], gu_s[:, 0::2], gu_b[:, 0::2]), "u": (gu_w[:, 1::2], gu_s[:, 1::2], gu_b[:, 1::2]),
                "d": (dn_w, np.asarray(ck.get(f"{p}down_proj_scales")), np.asarray(ck.get(f"{p}down_proj_bias")))}
    else:
        trip = {n: (np.asarray(ck.get(f"{p}{pr}.weight")), np.asarray(ck.get(f"{p}{pr}.scales")),
                    np.asarray(ck.get(f"{p}{pr}.bias")))
                for n, pr in (("g", "gate_proj"), ("u", "up_proj"), ("d", "down_proj"))}
    for n, (w, s, b) in trip.items():
        if w.shape[-1] * 8 != s.shape[-1] * 32:
            raise ValueError(f"{p}{n}: not MXFP4 (weight {w.shape}, scales {s.shape})")
        st[n] = ops.mxfp4_from_mlx(_cuda(w, torch.int32), _cuda(s, torch.uint8))
        bt = (_cuda(b, torch.bfloat16).float() if b.dtype == np.uint16  # bf16 bits, or plain fp16 / fp32
              else torch.from_numpy(np.asarray(b, np.float32)).cuda())
        st["b" + n] = bt.contiguous()
    E, f, d = st["g"][0].shape[0], st["g"][0].shape[1], st["g"][0].shape[2] * 8
    st.update(E=E, f=f, dm=d, fmt="mxfp4", act=act, ws=ops.Workspace(d, f, E, 0, torch.device("cuda")))
    return st
