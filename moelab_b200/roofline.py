"""Analytic cost model of a quantized SwiGLU MoE layer (restates moelab/roofline.py:21-41) with B200 peaks.

FLOPs = 6 * d * f * T * k                         (gate + up + down, 2 FLOP/MAC)
Bytes = U * 3 * d * f * w_bits / 8 + activations   (U = unique experts touched)
E[U]  = E * (1 - (1 - k/E)^T)                      (uniform routing)
The B200 peaks are the pool's measured copy bandwidth and cuBLAS bf16 rate (MEASURED_PEAKS.json at the repo
root, written by the driver); the fallbacks are the profiling recipe's earlier measurement.
"""
import json
import os

FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def b200_peaks():
    p = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")
    try:
        with open(p) as fh:
            m = json.load(fh)
        return {"hbm_gbs": float(m["hbm_gbs"]), "bf16_tflops": float(m["bf16_tflops"]),
                "bf16_tflops_sustained": float(m.get("bf16_tflops_sustained", m["bf16_tflops"])),
                "source": "measured"}
    except (OSError, KeyError, ValueError):
        return dict(FALLBACK)


BITS = {"bfloat16": 16, "float16": 16, "float32": 32, "q4": 4.5, "mxfp4": 4.25}


def expected_unique_experts(T, E, k):
    return E * (1.0 - (1.0 - k / E) ** T)


def flops(T, d, f, k):
    return 6.0 * d * f * T * k


def bytes_moved(T, d, f, E, k, w_bits=4.5, a_bytes=2, unique=None):
    U = expected_unique_experts(T, E, k) if unique is None else unique
    return U * 3.0 * d * f * w_bits / 8.0 + 2.0 * T * d * a_bytes + 2.0 * T * k * f * a_bytes


def router_bytes(T, d, E, a_bytes=2):
    return E * d * 2.0 + T * d * a_bytes + T * E * 4.0


def floor_time_s(nbytes, nflops, peaks=None):
    p = peaks or b200_peaks()
    return max(nbytes / (p["hbm_gbs"] * 1e9), nflops / (p["bf16_tflops"] * 1e12))
