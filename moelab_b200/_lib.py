"""ctypes binding of libmoelab_b200.so (the C ABI declared in include/moelab_b200.h).

The library is built in-tree by `python -m moelab_b200.build` (or __graft_entry__.build()). There is no
fallback: if the library is missing or a call fails, an exception is raised.
"""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libmoelab_b200.so")

MOEB_OK, MOEB_EINVAL, MOEB_ELAUNCH, MOEB_ETIMEOUT, MOEB_EUNSUP = 0, 1, 2, 3, 4
POLICY_AUTO, POLICY_SLOTS, POLICY_TILES8, POLICY_TILES16, POLICY_TILES8_RING, POLICY_TILES16_RING = 0, 1, 2, 3, 4, 5
POLICY_TC = 6
POLICY_DECODE = 7
POLICY_TILES24_RING = 8
DEVERR_EXPERT_ID, DEVERR_TIMEOUT = 1, 2

_P = ctypes.c_void_p
_I = ctypes.c_int
_L = ctypes.c_long
_F = ctypes.c_float
_S = ctypes.c_size_t

# name -> (restype, argtypes); every symbol the header declares
SIGNATURES = {
    "moeb_version": (_I, []),
    "moeb_last_error": (ctypes.c_char_p, []),
    "moeb_workspace_bytes": (_S, [_I, _I, _I, _I, _I]),
    "moeb_workspace_init": (_I, [_P, _S, _P]),
    "moeb_read_error": (_I, [_P, ctypes.POINTER(ctypes.c_uint), _P]),
    "moeb_policy": (_I, [_I, _I, _I]),
    "moeb_quantize_q4": (_I, [_P, _L, _L, _P, _P, _P]),
    "moeb_quantize_mxfp4": (_I, [_P, _L, _L, _P, _P, _P]),
    "moeb_dequant_q4": (_I, [_P, _P, _L, _L, _P, _P]),
    "moeb_dequant_mxfp4": (_I, [_P, _P, _L, _L, _P, _P]),
    "moeb_q4_from_mlx": (_I, [_P, _P, _P, _L, _L, _P, _P, _P]),
    "moeb_mxfp4_from_mlx": (_I, [_P, _P, _L, _L, _P, _P, _P]),
    "moeb_router": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, _F, _P, _P, _P, _P, _S, _P]),
    "moeb_route_tables": (_I, [_P, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _S, _P]),
    "moeb_experts_q4": (_I, [_P] * 12 + [_I] * 7 + [_P, _P, _P, _S, _P]),
    "moeb_experts_q4_static": (_I, [_P] * 12 + [_I] * 7 + [_P, _P, _P]),
    "moeb_experts_q4_static_read_error": (_I, [ctypes.POINTER(ctypes.c_uint), _P]),
    "moeb_layer_q4": (_I, [_P, _P, _P, _I, _F] + [_P] * 9 + [_I] * 7 + [_P, _P, _P, _P, _P, _P, _S, _P]),
    "moeb_experts_mxfp4": (_I, [_P] * 12 + [_I] * 7 + [_P, _P, _P, _S, _P]),
    "moeb_layer_mxfp4": (_I, [_P, _P, _P, _I, _F] + [_P] * 9 + [_I] * 7 + [_P, _P, _P, _P, _P, _P, _S, _P]),
    "moeb_layer_q4_shared": (_I, [_P, _P, _P, _I, _F, _I] + [_P] * 9 + [_I] * 7 + [_P] * 6 + [_S, _P]),
    "moeb_ep_dispatch": (_I, [_P, _P, _P] + [_I] * 5 + [_P, _P, _P, _P, _S, _P]),
    "moeb_ep_workspace_bytes": (_S, [_I, _I, _I, _I]),
    "moeb_ep_experts_q4": (_I, [_P] + [_I] * 4 + [_P] * 9 + [_I, _I, _P, _P, _S, _P]),
    "moeb_ep_experts_mxfp4": (_I, [_P] + [_I] * 4 + [_P] * 9 + [_I, _I, _P, _P, _S, _P]),
    "moeb_ep_combine": (_I, [_P, _P, _I, _I, _I, _P, _P, _P]),
    "moeb_ep_p2p_bytes": (_S, [_I, _I, _I]),
    "moeb_ep_ipc_alloc": (_I, [_S, ctypes.POINTER(ctypes.c_void_p)]),
    "moeb_ep_ipc_free": (_I, [_P]),
    "moeb_ep_ipc_handle": (_I, [_P, _P]),
    "moeb_ep_ipc_open": (_I, [_P, ctypes.POINTER(ctypes.c_void_p)]),
    "moeb_ep_ipc_close": (_I, [_P]),
    "moeb_ep_p2p_dispatch": (_I, [_P, _P, _P] + [_I] * 8 + [_P, _P, _P, _P, _P]),
    "moeb_ep_p2p_experts_q4": (_I, [_P, _P] + [_I] * 7 + [_P] * 9 + [_I, _I, _P, _S, _P]),
    "moeb_ep_p2p_combine": (_I, [_P, _P] + [_I] * 5 + [_P, _P, _P]),
    "moeb_ep_p2p_set_wait_limit": (_I, [_P, _I, _I, _I, ctypes.c_double, _P]),
    "moeb_ep_p2p_read_error": (_I, [_P, _I, _I, _I, ctypes.POINTER(ctypes.c_uint), _P]),
    "moeb_probe_tc_issue": (_I, [_I] * 7 + [ctypes.POINTER(ctypes.c_double)] * 3),
    "moeb_probe_mma_sync": (_I, [_I, _I, ctypes.POINTER(ctypes.c_double)]),
}

_lib = None


class MoebError(RuntimeError):
    pass


def load():
    """Load the library (once). Raises if it is missing: the CUDA path is the product, not optional."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise MoebError(f"{LIB_PATH} is missing: build it with `python -m moelab_b200.build`")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def call(name, *args):
    rc = getattr(load(), name)(*args)
    if rc != MOEB_OK:
        msg = load().moeb_last_error().decode(errors="replace")
        raise MoebError(f"{name} failed with status {rc}: {msg}")
    return rc
