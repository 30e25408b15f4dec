"""The reference's correctness gate for a variant, restated for the GPU box (TEST INFRASTRUCTURE ONLY).

moelab/torch_backend.py:103-126 (bench_variant, check=True) on DEVICE = "cuda":
  weights  make_weights (:43-47): torch.Generator(device="cuda").manual_seed(seed), N(0, 1) * d^-1/2 (gate, up)
           and * f^-1/2 (down), cast to the activation dtype;
  state    mod.prepare(wg, wu, wd); reference weights mod.dequant(state) when the variant has it;
  inputs   make_inputs (:50-54) for seed 0: x = rng.standard_normal((T, d)), then make_routing(T, E, k, routing, rng);
  check    errors(mod.run(state, x, idx, wts), reference(rw..., x, idx, wts)) (:57-74, the fp32 loop over the used
           experts) and ok = finite and rel_fro < TOL[dtype] (:19, bfloat16 3e-2).
The reference module itself cannot travel to the GPU box; its pieces are restated here line for line, and the
CPU-side ones are pinned by tests/golden (make_routing, the fp32 reference).
"""
import numpy as np
import torch

from moelab_b200.problem import make_routing

DTYPES = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}
TOL = {"float32": 1e-4, "float16": 5e-3, "bfloat16": 3e-2}


def make_weights(shape, dtype, seed=0, device="cuda"):
    g = torch.Generator(device=device).manual_seed(seed)
    d, f, E = shape.d, shape.f, shape.E
    mk = lambda *s, sc: (torch.randn(*s, generator=g, device=device) * sc).to(DTYPES[dtype])  # noqa: E731
    return mk(E, f, d, sc=d ** -0.5), mk(E, f, d, sc=d ** -0.5), mk(E, d, f, sc=f ** -0.5)


def make_inputs(shape, T, dtype, routing, seed, device="cuda"):
    rng = np.random.default_rng(seed)
    x = torch.from_numpy(rng.standard_normal((T, shape.d)).astype(np.float32)).to(device, DTYPES[dtype])
    idx, wts = make_routing(T, shape.E, shape.k, routing, rng)
    return x, torch.from_numpy(idx).to(device), torch.from_numpy(wts).to(device)


@torch.no_grad()
def reference(wg, wu, wd, x, idx, wts):
    x32 = x.float()
    y = torch.zeros_like(x32)
    for e in idx.unique().tolist():
        t, j = (idx == e).nonzero(as_tuple=True)
        xe = x32[t]
        g, u = xe @ wg[e].float().T, xe @ wu[e].float().T
        o = (torch.nn.functional.silu(g) * u) @ wd[e].float().T
        y.index_add_(0, t, o * wts[t, j, None])
    return y


def errors(y, y_ref):
    diff = y.float() - y_ref
    return {"rel_fro": (diff.norm() / (y_ref.norm() + 1e-30)).item(), "max_abs": diff.abs().max().item(),
            "finite": bool(torch.isfinite(y).all().item())}


@torch.no_grad()
def check_variant(mod, shape, tokens, dtype="bfloat16", routing="uniform"):
    """bench_variant's correctness records (type, variant, T, rel_fro, max_abs, finite, ok) for every T."""
    torch.backends.cuda.matmul.allow_tf32 = False
    wg, wu, wd = make_weights(shape, dtype)
    state = mod.prepare(wg, wu, wd)
    rw = mod.dequant(state) if hasattr(mod, "dequant") else (wg, wu, wd)
    out = []
    for T in tokens:
        x, idx, wts = make_inputs(shape, T, dtype, routing, seed=0)
        res = {"type": "result", "variant": mod.META["name"], "T": T}
        res.update(errors(mod.run(state, x, idx, wts), reference(*rw, x, idx, wts)))
        res["ok"] = res["finite"] and res["rel_fro"] < TOL[dtype]
        out.append(res)
    return out
