"""Generate tests/golden/trace_qwen3.npz: recorded-trace routing windows drawn by the reference's OWN code.

    MOELAB_REF=<path to the moe-lab checkout> python tests/golden/make_trace.py

The reference's benchmark inputs for `routing="trace"` (moelab/torch_backend.py:50-54, moelab/mlx_backend.py:39-45)
are rng = default_rng(seed); x = rng.standard_normal((T, d)); make_routing(T, E, k, "trace", rng), where trace
routing (moelab/problem.py:38-50) draws a domain, a layer and a start token of the recorded Qwen3-30B-A3B routing
(runs/routing_qwen3.npz: three domains of [48 layers, tokens, top-8] expert ids) and random combine weights.
This script runs exactly that for seeds 0..NSEED-1 and T in TS with d = 2048, E = 128, k = 8, and stores
  keys     int32 [N, 4]   (domain, layer, start, T) of every window drawn
  windows  int16 [N, 32, 8]  the window's ids (first T rows valid)
  shapes   int32 [3, 2]   (layers, tokens) of each domain, in file order
  idx / wts per (seed, T): the reference's own make_inputs outputs, for the bit-exact test
so that moelab_b200.problem can redraw the same windows without the 4 MB trace file.
"""
import importlib.util
import os
import sys

import numpy as np

REF = os.environ.get("MOELAB_REF")
if not REF:
    sys.exit("set MOELAB_REF to the root of the moe-lab reference checkout")
OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "trace_qwen3.npz")
NSEED, TS, D, E, K = 16, (1, 8, 16, 32), 2048, 128, 8


def main():
    spec = importlib.util.spec_from_file_location("ref_problem", os.path.join(REF, "moelab", "problem.py"))
    rp = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(rp)
    z = np.load(os.path.join(REF, "runs", "routing_qwen3.npz"))
    doms = [n for n in z.files if n != "E"]
    shapes = np.array([z[n].shape[:2] for n in doms], np.int32)
    keys, wins, out = [], [], {}
    for seed in range(NSEED):
        for T in TS:
            rng = np.random.default_rng(seed)
            rng.standard_normal((T, D))
            probe = np.random.default_rng(seed)  # the same draws, to record which window was taken
            probe.standard_normal((T, D))
            dom = int(probe.integers(len(doms)))
            layer, start = int(probe.integers(shapes[dom][0])), int(probe.integers(shapes[dom][1] - T))
            idx, wts = rp.make_routing(T, E, K, "trace", rng)  # the reference's own draw
            assert np.array_equal(idx, z[doms[dom]][layer, start:start + T].astype(np.int32))
            key = (dom, layer, start, T)
            if key not in keys:
                keys.append(key)
                w = np.zeros((32, K), np.int16)
                w[:T] = idx
                wins.append(w)
            out[f"idx_{seed}_{T}"] = idx.astype(np.int32)
            out[f"wts_{seed}_{T}"] = wts.astype(np.float32)
    np.savez_compressed(OUT, keys=np.array(keys, np.int32), windows=np.stack(wins), shapes=shapes,
                        domains=np.array(doms), **out)
    print(OUT, len(keys), "windows")


if __name__ == "__main__":
    main()
