"""Generate the golden fixtures in tests/golden from the reference's OWN Python code.

Run where the reference checkout (read-only) is available, naming its root in MOELAB_REF:

    MOELAB_REF=<path to the moe-lab checkout> python tests/golden/make_golden.py

It imports moelab.problem (make_routing, make_problem, reference, error_metrics), moelab.torch_backend
(reference, fp32) and moelab/variants/cuda/torch_loop.py (the CPU torch path) from the reference tree and
records their outputs. Large arrays (weights) are recorded as sha256 digests of their bytes; outputs are
stored in full. The tests regenerate the inputs with moelab_b200.problem and the oracle, and must match these
vectors: bit for bit for the generators, within 1e-5 relative for the float references.
"""
import hashlib
import importlib.util
import json
import os
import sys

import numpy as np
import torch

REF = os.environ.get("MOELAB_REF")
if not REF:
    sys.exit("set MOELAB_REF to the root of the moe-lab reference checkout")
OUT = os.path.dirname(os.path.abspath(__file__))


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main():
    sys.path.insert(0, REF)
    from moelab import problem, torch_backend  # noqa: E402  (reference code)
    from moelab.shapes import MoEShape  # noqa: E402
    spec = importlib.util.spec_from_file_location("ref_torch_loop", os.path.join(REF, "moelab/variants/cuda/torch_loop.py"))
    torch_loop = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(torch_loop)

    meta = {"source": "Tigerly1/moe-lab reference python (moelab/problem.py, moelab/torch_backend.py, "
                      "moelab/variants/cuda/torch_loop.py)", "routing": [], "problems": []}
    arrays = {}

    # 1. routing generator (problem.py:15-32): bit-exact ids and weights
    rid = 0
    for (T, E, k, mode, seed) in [(1, 128, 8, "uniform", 0), (7, 8, 2, "uniform", 1), (33, 16, 4, "zipf", 2),
                                  (64, 8, 2, "one_hot", 3), (100, 64, 6, "zipf", 4), (16, 32, 4, "uniform", 5)]:
        idx, w = problem.make_routing(T, E, k, mode, np.random.default_rng(seed))
        arrays[f"routing{rid}_idx"], arrays[f"routing{rid}_wts"] = idx, w
        meta["routing"].append({"id": rid, "T": T, "E": E, "k": k, "mode": mode, "seed": seed})
        rid += 1

    # 2. problems (problem.py:53-64) + fp64 reference + fp32 torch reference + torch_loop on bf16 weights
    pid = 0
    for (d, f, E, k, T, mode, seed) in [(128, 256, 8, 2, 7, "uniform", 0), (128, 256, 8, 2, 33, "zipf", 1),
                                        (256, 384, 16, 4, 5, "uniform", 2), (128, 256, 8, 2, 64, "one_hot", 3),
                                        (192, 256, 8, 2, 6, "uniform", 4), (128, 256, 4, 4, 9, "uniform", 5)]:
        sh = MoEShape("g", d=d, f=f, E=E, k=k)
        p = problem.make_problem(sh, T, mode, seed)
        y64 = problem.reference(p)
        t = {n: torch.from_numpy(p[n]) for n in ("x", "w_gate", "w_up", "w_down", "wts")}
        idx_t = torch.from_numpy(p["idx"])
        y32 = torch_backend.reference(t["w_gate"], t["w_up"], t["w_down"], t["x"], idx_t, t["wts"]).numpy()
        s = torch_loop.prepare(*(t[n].to(torch.bfloat16) for n in ("w_gate", "w_up", "w_down")))
        yl = torch_loop.run(s, t["x"].to(torch.bfloat16), idx_t, t["wts"]).float().numpy()
        em = problem.error_metrics(yl, y64)
        arrays[f"prob{pid}_idx"], arrays[f"prob{pid}_wts"] = p["idx"], p["wts"]
        arrays[f"prob{pid}_y64"], arrays[f"prob{pid}_y32"], arrays[f"prob{pid}_yloop"] = y64, y32, yl
        meta["problems"].append({"id": pid, "d": d, "f": f, "E": E, "k": k, "T": T, "mode": mode, "seed": seed,
                                 "sha256": {n: sha(p[n]) for n in ("x", "w_gate", "w_up", "w_down")},
                                 "loop_vs_fp64": em})
        pid += 1

    np.savez_compressed(os.path.join(OUT, "reference_vectors.npz"), **arrays)
    with open(os.path.join(OUT, "reference_vectors.json"), "w") as fh:
        json.dump(meta, fh, indent=1)
    print("wrote", len(arrays), "arrays")


if __name__ == "__main__":
    main()
