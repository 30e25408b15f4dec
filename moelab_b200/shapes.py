"""MoE layer shapes (per layer, routed experts): d = hidden, f = expert FFN width, E = experts, k = top-k.

Mirrors moelab/shapes.py:9-39 (MoEShape and the real-model table). The per-family router rules (Qwen3 renormalised
top-k, DeepSeek-V2 greedy + shared experts, gpt-oss biased gate) are arguments of the layer call (norm, rscale,
gate_b, shared experts in the state), not part of the shape.
"""
from dataclasses import asdict, dataclass


@dataclass(frozen=True)
class MoEShape:
    name: str
    d: int
    f: int
    E: int
    k: int
    shared: int = 0  # number of always-on shared experts (DeepSeek), each of width f

    def to_dict(self):
        return asdict(self)


SHAPES = {s.name: s for s in [
    MoEShape("tiny", d=256, f=512, E=8, k=2),
    MoEShape("olmoe-1b-7b", d=2048, f=1024, E=64, k=8),
    MoEShape("qwen3-30b-a3b", d=2048, f=768, E=128, k=8),
    MoEShape("gpt-oss-20b", d=2880, f=2880, E=32, k=4),
    MoEShape("deepseek-v2-lite", d=2048, f=1408, E=64, k=6, shared=2),
    MoEShape("mixtral-8x7b", d=4096, f=14336, E=8, k=2),
    MoEShape("qwen3-235b-a22b", d=4096, f=1536, E=128, k=8),
    MoEShape("gpt-oss-120b", d=2880, f=2880, E=128, k=4),
    MoEShape("deepseek-v3", d=7168, f=2048, E=256, k=8, shared=1),
    MoEShape("kimi-k2", d=7168, f=2048, E=384, k=8, shared=1),
]}

TOKEN_SWEEP = [1, 2, 4, 8, 16, 32, 64, 128, 256, 512, 1024]
