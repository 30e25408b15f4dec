"""The variants through the reference's own correctness gate (moelab/torch_backend.py:103-126 bench_variant with
check=True: its weights, inputs, fp32 reference, error metrics and ok = rel_fro < TOL["bfloat16"]), restated in
oracle/harness.py because the reference cannot travel to the GPU box; and, where the reference checkout is present
(MOELAB_REF) together with a GPU, through the reference's bench_variant itself."""
import os

import pytest

from helpers import Q4_VARIANT, load_variant
from moelab_b200.shapes import MoEShape

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
VARIANTS = {"b200_q4_moe": Q4_VARIANT,
            "b200_mxfp4_moe": os.path.join(ROOT, "moelab_b200", "variants", "cuda", "b200_mxfp4_moe.py")}
SHAPES = [MoEShape("qwen3-30b-a3b", d=2048, f=768, E=128, k=8), MoEShape("tiny", d=256, f=128, E=8, k=2)]


@pytest.mark.parametrize("name", list(VARIANTS))
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: s.name)
@pytest.mark.parametrize("routing", ["uniform", "zipf"])
def test_reference_gate_restated(name, shape, routing):
    from oracle.harness import check_variant
    mod = load_variant(VARIANTS[name])
    res = check_variant(mod, shape, [1, 4, 32, 300], "bfloat16", routing)
    assert all(r["ok"] for r in res), res
    # the library's own bound is tighter than the gate's 3e-2
    assert all(r["rel_fro"] < 1e-2 for r in res), res


@pytest.mark.skipif(not os.environ.get("MOELAB_REF"), reason="MOELAB_REF (the reference checkout) is not set")
@pytest.mark.parametrize("name", list(VARIANTS))
def test_reference_bench_variant_itself(name):
    import sys
    sys.path.insert(0, os.environ["MOELAB_REF"])
    from moelab import torch_backend as tb  # the reference's own harness
    from moelab.shapes import SHAPES as REF_SHAPES
    mod = tb.load_variant(VARIANTS[name])
    recs = []
    tb.bench_variant(mod, REF_SHAPES["qwen3-30b-a3b"], [1, 8, 32], dtype="bfloat16", iters=3, n_rot=2,
                     emit=recs.append)
    assert recs and all(r["ok"] for r in recs), recs
