#!/usr/bin/env python
"""Benchmark of the quantized MoE-layer forward (moe-lab's hot path) on B200.

Workload: Qwen3-30B-A3B-shaped int4-g64 MoE layer, d=2048, f=768, E=128, k=8,
weights N(0, 0.02) bf16 quantised to int4 affine g64 (bf16 scale/bias), gate N(0, 0.02), x ~ N(0, 1) bf16,
routing from the gate (softmax, top-8, renormalised). One step = one layer call (router + routing + grouped
experts + weighted combine, residual fused) on T tokens per GPU. 16 independent seeded layers are cycled so
the weights streamed between steps (16 x 340 MB) are far larger than the 126 MB L2.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--tokens T] [--impl reference]

Prints one JSON line (rank 0). value = whole-job tokens/s; the T sweep, per-kernel times and the roofline
fraction explain it. --impl reference times the reference's CPU torch path (the oracle's port of
moelab/variants/cuda/torch_loop.py plus the stock torch router) on the same config with all host threads.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402

D, F, E, K_TOP = 2048, 768, 128, 8
W_BITS = 4.5
WORKLOAD = "qwen3-30b-a3b int4-g64 MoE layer: router + routing + grouped experts + combine (residual fused)"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2048)
    ap.add_argument("--warmup", type=int, default=32)
    ap.add_argument("--tokens", type=int, default=32)
    ap.add_argument("--layers", type=int, default=16)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--sweep", default="1,4,32,256", help="extra T values measured after the headline ('' = none)")
    ap.add_argument("--e2e-steps", type=int, default=256)
    ap.add_argument("--cpu-seconds", type=float, default=15.0, help="bound on the CPU baseline sample")
    ap.add_argument("--soak-seconds", type=float, default=1.5, help="replays before the timed region (clocks)")
    ap.add_argument("--configs", type=int, default=1, help="1: also time the other BASELINE configurations (1 GPU)")
    ap.add_argument("--trace", type=int, default=1, help="1: also time Qwen3-30B on the reference's recorded routing "
                    "traces (T = 1, 8, 16, 32)")
    ap.add_argument("--ep-stack", default="1,32,256,2048", help="also time BASELINE's expert-parallel stack (8 "
                    "Qwen3-235B-shaped layers, experts split over the N GPUs; N = 1 runs the same code on one GPU) at "
                    "these tokens per GPU ('' = none)")
    ap.add_argument("--profile-config", default="", help="run 3 eager layer calls of the CONFIGS entry whose name "
                    "starts with this, or of the headline layer ('qwen3-30b'), for ncu captures of one kernel, and exit")
    ap.add_argument("--profile-tokens", type=int, default=1024)
    ap.add_argument("--probe-tc", action="store_true", help="print the tcgen05 issue-rate table (MMA shapes of the "
                    "expert kernels: N, issuing threads, MMAs between barrier waits) and mma.sync for comparison, "
                    "then exit")
    ap.add_argument("--profile-policy", default="", help="pin the expert kernels for --profile-config (slots, "
                    "tiles8, tiles16, ring8, ring16, ring24, tc, decode; default: the load-based dispatcher)")
    return ap.parse_args()


# ------------------------------------------------------------------ distributed plumbing
def dist_init(a):
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return ws, rank, local


def barrier(ws):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(ws, v):
    if ws == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------------ clocks
CLOCK_Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
           "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
           "clocks_event_reasons.sw_power_cap")


class ClockSampler:
    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.path = os.path.join(tempfile.gettempdir(), f"moelab_b200_clocks_gpu{gpu_index}_{os.getpid()}.csv")

    def start(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={CLOCK_Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.fh, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.fh.close()
        rows = []
        for line in open(self.path):
            p = [x.strip() for x in line.split(",")]
            if len(p) >= 9:
                rows.append(p)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = max(float(r[2]) for r in rows if r[2].replace(".", "").isdigit())
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": reasons,
                "samples": len(rows), "power_w_max": max(float(r[3]) for r in rows)}


# ------------------------------------------------------------------ workload
def make_layers(n_layers, seed, device):
    from moelab_b200.variants.cuda import b200_q4_moe as v
    g = torch.Generator(device=device).manual_seed(seed)
    layers = []
    for _ in range(n_layers):
        mk = lambda *s: (torch.randn(*s, generator=g, device=device) * 0.02).to(torch.bfloat16)  # noqa: E731
        w = [mk(E, F, D), mk(E, F, D), mk(E, D, F)]
        st = v.prepare(*w)
        del w
        layers.append((st, mk(E, D)))
    torch.cuda.synchronize()
    return v, layers


def layer_bytes(idx_list, T):
    """Algorithmic bytes of one layer call (moelab/roofline.py:29-33 with the actual unique experts U, plus the
    router's gate read): U*3*d*f*w_bits/8 + 2*T*d*2 + 2*T*k*f*2 + E*d*2."""
    out = []
    for idx in idx_list:
        U = int(torch.unique(idx).numel())
        out.append(U * 3 * D * F * W_BITS / 8 + 2 * T * D * 2 + 2 * T * K_TOP * F * 2 + E * D * 2)
    return out


def gate_up_bytes(idx, T):
    U = int(torch.unique(idx).numel())
    return U * 2 * D * F * W_BITS / 8 + T * D * 2 + T * K_TOP * F * 2


def down_bytes(idx, T):
    U = int(torch.unique(idx).numel())
    return U * D * F * W_BITS / 8 + T * K_TOP * F * 2 + T * D * 2 * 2


def make_inputs(T, L, seed):
    """One seeded token batch x_l ~ N(0, 1) per layer. Steps are independent layer calls y = x_l + moe_l(x_l)
    (no chaining: without the model's norms a chained residual stream grows without bound and would degrade the
    routing; stream order still serialises the calls)."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    return [torch.randn(T, D, generator=g, device="cuda").to(torch.bfloat16) for _ in range(L)]


def capture(v, layers, xs, n_steps, k0=0):
    """CUDA graph of n_steps layer calls cycling through the layers (step i uses layer and input i mod L)."""
    L = len(layers)

    def chain():
        y = None
        for i in range(n_steps):
            st, gate = layers[(k0 + i) % L]
            x = xs[(k0 + i) % L]
            y = v.layer(st, x, gate, K_TOP, residual=x)
        return y

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        chain()
    torch.cuda.current_stream().wait_stream(s)
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        out = chain()
    return gr, out


def e2e_loop(call, xh_list, yh_list, steps, ws):
    """End-to-end timing through the public API with host buffers: every step copies its input from pinned host
    memory to the device and its result back to pinned host memory. The copies run on a side stream, double
    buffered, so step i + 1's input and step i's result move while step i computes (stream-ordered: compute i + 1
    waits for its input copy, the copy of result i waits for compute i). call(i, x_device) -> y_device.
    Returns seconds for `steps` steps (CUDA events on the compute stream around the whole loop, both streams
    drained inside it)."""
    comp, cp = torch.cuda.current_stream(), torch.cuda.Stream()
    nb = len(xh_list)
    xd = [torch.empty_like(xh_list[0], device="cuda") for _ in range(2)]
    ready = [torch.cuda.Event() for _ in range(2)]
    done = [torch.cuda.Event() for _ in range(2)]

    def run(n):
        with torch.cuda.stream(cp):
            xd[0].copy_(xh_list[0], non_blocking=True)
            ready[0].record(cp)
        for i in range(n):
            b = i & 1
            if i + 1 < n:  # next input into the other buffer once the step that used it has finished
                with torch.cuda.stream(cp):
                    if i >= 1:
                        cp.wait_event(done[1 - b])
                    xd[1 - b].copy_(xh_list[(i + 1) % nb], non_blocking=True)
                    ready[1 - b].record(cp)
            comp.wait_event(ready[b])
            y = call(i, xd[b])
            done[b].record(comp)
            y.record_stream(cp)  # the allocator keeps y until the copy stream has read it
            with torch.cuda.stream(cp):
                cp.wait_event(done[b])
                yh_list[i % nb].copy_(y, non_blocking=True)
        comp.wait_stream(cp)

    run(4)
    torch.cuda.synchronize()
    barrier(ws)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(comp)
    run(steps)
    e1.record(comp)
    e1.synchronize()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / 1e3


def time_graph(gr, ws, reps=1):
    barrier(ws)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        gr.replay()
    b.record()
    b.synchronize()
    torch.cuda.synchronize()
    barrier(ws)
    return a.elapsed_time(b) / 1e3


def routing_of_chain(v, layers, xs, n_steps, k0=0):
    idxs = []
    for i in range(n_steps):
        st, gate = layers[(k0 + i) % len(layers)]
        x = xs[(k0 + i) % len(layers)]
        _, idx, _ = v.layer(st, x, gate, K_TOP, residual=x, return_routing=True)
        idxs.append(idx)
    return idxs


def stage_times(v, layers, xs, n_steps):
    """Per-kernel durations from CUDA events recorded between the stages (router, gate/up, down)."""
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(n_steps)]
    idxs = []
    for i in range(n_steps):
        st, gate = layers[i % len(layers)]
        x = xs[i % len(layers)]
        _, idx, _ = v.layer(st, x, gate, K_TOP, residual=x, return_routing=True, stage_events=ev[i])
        idxs.append(idx)
    torch.cuda.synchronize()
    r = [ev[i][0].elapsed_time(ev[i][1]) * 1e3 for i in range(n_steps)]
    gu = [ev[i][1].elapsed_time(ev[i][2]) * 1e3 for i in range(n_steps)]
    dn = [ev[i][2].elapsed_time(ev[i][3]) * 1e3 for i in range(n_steps)]
    return r, gu, dn, idxs


def measure_T(v, layers, T, ws, rank, n_steps, seed, peaks):
    xs = make_inputs(T, len(layers), seed)
    gr, _ = capture(v, layers, xs, n_steps)
    gr.replay()
    torch.cuda.synchronize()
    t = max_over_ranks(ws, time_graph(gr, ws))
    idxs = routing_of_chain(v, layers, xs, n_steps)
    nb = layer_bytes(idxs, T)
    us = t / n_steps * 1e6
    return {"T": T, "us": round(us, 2), "gbs": round(sum(nb) / t / 1e9, 1),
            "frac": round(layer_frac(sum(nb) / len(nb), 6.0 * D * F * T * K_TOP, us * 1e-6, peaks), 3)}


def layer_frac(byts, flops, t, peaks):
    """Fraction of the layer roofline (north star: the slower of the bytes at the HBM peak and the FLOPs at the bf16
    tensor peak; moelab/roofline.py:36-41) that a call of t seconds reaches."""
    return max(byts / (peaks["hbm_gbs"] * 1e9), flops / (peaks["bf16_tflops"] * 1e12)) / t


# reference's published M4 Pro numbers for the trace rows (runs/repro/q4_qwen3_trace.txt:2-5, custom kernel B)
TRACE_M4PRO_US = {1: 110.9, 8: 367.7, 16: 576.1, 32: 923.6}


def measure_trace(v, layers, peaks, Ts=(1, 8, 16, 32), n_calls=64):
    """Qwen3-30B on recorded routing traces: the reference's own trace inputs (moelab/problem.py:38-50 drawn by
    moelab/torch_backend.py:50-54's make_inputs, tests/golden/trace_qwen3.npz) through the harness contract
    run(state, x, idx, wts) - the call the reference's trace numbers time. 16 seeds cycled over the 16 layers."""
    from moelab_b200.problem import make_inputs
    out = []
    for T in Ts:
        ins = []
        for s in range(16):
            x, idx, wts = make_inputs(D, E, K_TOP, T, "trace", s)
            ins.append((torch.from_numpy(x).to("cuda", torch.bfloat16), torch.from_numpy(idx).cuda(),
                        torch.from_numpy(wts).cuda()))
        for i in range(16):
            v.run(layers[i][0], *ins[i])
        torch.cuda.synchronize()
        s_ = torch.cuda.Stream()
        s_.wait_stream(torch.cuda.current_stream())
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s_):
            with torch.cuda.graph(gr, stream=s_):
                for i in range(n_calls):
                    v.run(layers[i % 16][0], *ins[i % 16])
        torch.cuda.current_stream().wait_stream(s_)
        gr.replay()
        torch.cuda.synchronize()
        t = min(time_graph(gr, 1) for _ in range(3)) / n_calls
        del gr
        U = float(np.mean([torch.unique(i[1]).numel() for i in ins]))
        byts = U * 3 * D * F * W_BITS / 8 + 2 * T * D * 2 + 2 * T * K_TOP * F * 2
        out.append([T, round(t * 1e6, 2), round(layer_frac(byts, 6.0 * D * F * T * K_TOP, t, peaks), 3),
                    TRACE_M4PRO_US[T]])
    return out


# ------------------------------------------------------------------ the other BASELINE configurations (1 GPU)
CONFIGS = [
    # name, shape, format/options, T values
    ("gpt-oss-20b mxfp4 (biases, clamped SwiGLU, gate bias)", dict(d=2880, f=2880, E=32, k=4), "gptoss", [1, 8, 32, 128]),
    ("deepseek-v2-lite int4 + 2 shared experts (Zipf-biased greedy router)", dict(d=2048, f=1408, E=64, k=6),
     "deepseek", [1, 16, 64, 256]),
    ("qwen3-235b-a22b int4", dict(d=4096, f=1536, E=128, k=8), "q4", [1, 32, 256, 2048]),
    ("mixtral-8x7b int4", dict(d=4096, f=14336, E=8, k=2), "q4", [1, 16, 256, 1024, 4096]),
    ("mixtral-8x7b mxfp4", dict(d=4096, f=14336, E=8, k=2), "mxfp4", [1, 16, 256, 1024]),
]


def config_layers(d, f, E, k, kind, n_layers=2, seed=11):
    """n_layers seeded layers of one configuration and a layer-call closure (router included)."""
    from moelab_b200.problem import zipf_bias
    from moelab_b200.variants.cuda import b200_mxfp4_gptoss as vg, b200_mxfp4_moe as vm, b200_q4_moe as vq
    g = torch.Generator(device="cuda").manual_seed(seed)
    mk = lambda *s_, sc=0.02: (torch.randn(*s_, generator=g, device="cuda") * sc).to(torch.bfloat16)  # noqa: E731
    layers = []
    for _ in range(n_layers):
        w = [mk(E, f, d), mk(E, f, d), mk(E, d, f)]
        gate = mk(E, d)
        if kind == "gptoss":
            b = [mk(E, f, sc=0.01).float(), mk(E, f, sc=0.01).float(), mk(E, d, sc=0.01).float()]
            st = vg.state(*w, *b)
            gb = mk(E, sc=0.01)
            call = (lambda st, x, gate, gb=gb: vg.layer(st, x, gate, k, gate_b=gb, residual=x))
            bits = 4.25
        elif kind == "deepseek":
            sw = [mk(2 * f, d), mk(2 * f, d), mk(d, 2 * f)]
            st = vq.prepare_shared(*w, *sw)
            gb = torch.from_numpy(zipf_bias(E, 1.1, seed=7)).to("cuda", torch.bfloat16)
            call = (lambda st, x, gate, gb=gb: vq.layer(st, x, gate, k, gate_b=gb, norm=False, residual=x))
            bits = 4.5
        elif kind == "mxfp4":
            st = vm.prepare(*w)
            call = (lambda st, x, gate: vm.layer(st, x, gate, k, residual=x))
            bits = 4.25
        else:
            st = vq.prepare(*w)
            call = (lambda st, x, gate: vq.layer(st, x, gate, k, residual=x))
            bits = 4.5
        del w
        layers.append((st, gate, call))
    torch.cuda.synchronize()
    return layers, bits


def measure_config(name, shp, kind, Ts, peaks, n_calls=8):
    d, f, E, k = shp["d"], shp["f"], shp["E"], shp["k"]
    layers, bits = config_layers(d, f, E, k, kind)
    ns = 2 if kind == "deepseek" else 0
    out = []
    for T in Ts:
        g = torch.Generator(device="cuda").manual_seed(1000 + T)
        xs = [torch.randn(T, d, generator=g, device="cuda").to(torch.bfloat16) for _ in layers]
        for i, (st, gate, call) in enumerate(layers):  # warm-up (sizes the workspaces)
            call(st, xs[i], gate)
        torch.cuda.synchronize()
        s_ = torch.cuda.Stream()
        s_.wait_stream(torch.cuda.current_stream())
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s_):
            with torch.cuda.graph(gr, stream=s_):
                for i in range(n_calls):
                    st, gate, call = layers[i % len(layers)]
                    call(st, xs[i % len(layers)], gate)
        torch.cuda.current_stream().wait_stream(s_)
        gr.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(3):
            gr.replay()
        e1.record()
        e1.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (3 * n_calls)
        del gr
        # algorithmic bytes / flops of one call (unique routed experts of layer 0's routing, + shared experts)
        from moelab_b200 import ops
        idx, _ = ops.router(xs[0], layers[0][1], k)
        U = int(torch.unique(idx).numel()) + ns
        ks = k + ns
        byts = U * 3 * d * f * bits / 8 + 2 * T * d * 2 + 2 * T * ks * f * 2 + E * d * 2
        flops = 6.0 * d * f * T * ks
        t_roof = max(byts / (peaks["hbm_gbs"] * 1e9), flops / (peaks["bf16_tflops"] * 1e12))
        out.append({"config": name, "T": T, "us_per_call": round(us, 2), "tokens_per_s": round(T / us * 1e6, 1),
                    "gbs": round(byts / us / 1e3, 1), "tflops": round(flops / us / 1e6, 1),
                    "roofline_frac": round(t_roof / (us * 1e-6), 3),
                    "bound": "hbm" if byts / (peaks["hbm_gbs"] * 1e9) >= flops / (peaks["bf16_tflops"] * 1e12)
                    else "tensor"})
    del layers
    torch.cuda.empty_cache()
    return out


# ------------------------------------------------------------------ CPU baseline (reference's CPU torch path)
def cpu_layer(seed=0):
    """One Qwen3-30B-shaped layer on the CPU: int4-g64 quantised by the oracle, dequantised to bf16 (the weights
    the reference's torch path multiplies)."""
    import oracle
    g = torch.Generator().manual_seed(seed)
    mk = lambda *s: (torch.randn(*s, generator=g) * 0.02).to(torch.bfloat16)  # noqa: E731
    dq = []
    for shape in ((E, F, D), (E, F, D), (E, D, F)):
        q, s, b = oracle.q4_quantize(mk(*shape))
        dq.append(torch.from_numpy(oracle.q4_dequant(q, s, b)).to(torch.bfloat16))
    return {"wg": dq[0], "wu": dq[1], "wd": dq[2]}, mk(E, D)


def cpu_step(s, gate, x):
    import oracle
    idx, wts = oracle.torch_router_stock(x, gate, K_TOP)
    return oracle.torch_loop_run(s, x, idx, wts) + x  # same layer call as the GPU arm: y = x + moe(x)


def cpu_baseline(T, seconds, warmup=1, steps=None):
    torch.set_num_threads(os.cpu_count() or 1)
    s, gate = cpu_layer()
    x = torch.randn(T, D, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    for _ in range(warmup):
        cpu_step(s, gate, x)
    n, t0 = 0, time.perf_counter()
    while True:
        cpu_step(s, gate, x)
        n += 1
        el = time.perf_counter() - t0
        if (steps is not None and (n >= steps or el >= 120.0)) or (steps is None and (el >= seconds or n >= 10000)):
            break  # the reference arm stops at K steps or 120 s of timed work, whichever comes first
    return T * n / el, n, el


# ------------------------------------------------------------------ expert parallel (N > 1)
def make_ep_layers(n_layers, rank, world, d=D, f=F, e=E):
    """This rank's E/world experts of n_layers layers (seeded per layer and rank) and each layer's gate (seeded
    per layer, the same on every rank)."""
    from moelab_b200 import ep
    from moelab_b200.variants.cuda import b200_q4_moe as v
    El = e // world
    layers = []
    for li in range(n_layers):
        g = torch.Generator(device="cuda").manual_seed(1000 + 7919 * li + 104729 * rank)
        mk = lambda *s_: (torch.randn(*s_, generator=g, device="cuda") * 0.02).to(torch.bfloat16)  # noqa: E731
        st = v.prepare(mk(El, f, d), mk(El, f, d), mk(El, d, f))
        ep.attach(st, rank, world, e)
        gg = torch.Generator(device="cuda").manual_seed(555 + li)
        layers.append((st, (torch.randn(e, d, generator=gg, device="cuda") * 0.02).to(torch.bfloat16)))
    torch.cuda.synchronize()
    return layers


def ep_steps(layers, xs, n, xch, k=K_TOP, k0=0):
    """n expert-parallel layer calls over the peer-memory exchange (layer and input i mod L)."""
    from moelab_b200 import ep
    y = None
    for i in range(n):
        st, gate = layers[(k0 + i) % len(layers)]
        x = xs[(k0 + i) % len(xs)]
        y = ep.layer_p2p(st, x, gate, k, xch, residual=x, max_tokens=x.shape[0])  # every rank has T tokens
    return y


def ep_graph(layers, xs, n, xch, ws):
    """CUDA graph of n expert-parallel layer calls (every rank captures and replays the same sequence)."""
    barrier(ws)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(gr, stream=s):
            ep_steps(layers, xs, n, xch)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    barrier(ws)
    gr.replay()  # warm replay (every rank)
    torch.cuda.synchronize()
    return gr


def ep_layer_bytes(layers, xs, n, xch, ws, d=D, f=F, k=K_TOP):
    """Algorithmic bytes one GPU moves per layer call: the weights of its experts that received rows, the rows
    in, h out and back in, and the weighted rows out (measured on n eager calls)."""
    from moelab_b200 import ep, ops
    total = 0.0
    for i in range(n):
        st, gate = layers[i % len(layers)]
        x = xs[i % len(xs)]
        idx, _ = ops.router(x, gate, k)
        allidx = [torch.empty_like(idx) for _ in range(ws)]
        import torch.distributed as dist
        dist.all_gather(allidx, idx)
        ids = torch.cat(allidx).reshape(-1)
        El = E // ws
        mine = ids[(ids // El) == xch.me]
        U = int(torch.unique(mine).numel())
        R = int(mine.numel())
        total += U * 3 * d * f * W_BITS / 8 + R * (d + 8) * 2 + 2 * R * f * 2 + R * d * 4
        ep.layer_p2p(st, x, gate, k, xch, residual=x, max_tokens=x.shape[0])
    return total / n


def ep_stack(a, ws, rank):
    """BASELINE's expert-parallel configuration: a stack of 8 Qwen3-235B-shaped int4 layers (d 4096, f 1536, 128
    experts, top-8; independent seeded weights per layer) with the experts split over the ws GPUs. One step is one
    pass of T tokens per GPU through the 8 layers, in a CUDA graph, timed on the device (max over ranks)."""
    from moelab_b200 import ep
    d, f, e, k, L = 4096, 1536, 128, 8, 8
    Ts = [int(s_) for s_ in a.ep_stack.split(",") if s_.strip()]
    layers = make_ep_layers(L, rank, ws, d=d, f=f, e=e)
    xch = ep.PeerExchange.create(max(Ts) * k, d) if ws > 1 else ep.PeerExchange.local_group(1, max(Ts) * k, d,
                                                                                                "cuda")[0]
    rows = []
    try:
        for T in Ts:
            g = torch.Generator(device="cuda").manual_seed(31 + T + rank)
            xs = [torch.randn(T, d, generator=g, device="cuda").to(torch.bfloat16) for _ in range(L)]
            ep_steps(layers, xs, L, xch, k=k)  # eager pass (sizes the workspaces)
            torch.cuda.synchronize()
            gr = ep_graph(layers, xs, L, xch, ws)
            t = max_over_ranks(ws, time_graph(gr, ws))  # one replay = one pass through the stack
            del gr
            row = [T, round(t / L * 1e6, 2), round(ws * T / t, 1)]
            if ws > 1:  # the NCCL all-to-all-v exchange on the same stack (eager: one host read per layer)
                from moelab_b200 import ep as ep_
                for i in range(L):
                    ep_.layer(layers[i][0], xs[i], layers[i][1], k, residual=xs[i])
                barrier(ws)
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for i in range(L):
                    ep_.layer(layers[i][0], xs[i], layers[i][1], k, residual=xs[i])
                e1.record()
                e1.synchronize()
                tn = max_over_ranks(ws, e0.elapsed_time(e1) / 1e3)
                row += [round(tn / L * 1e6, 2), round(ws * T / tn, 1)]
            rows.append(row)
        errs = xch.read_error()
        torch.cuda.synchronize()
        barrier(ws)
    finally:
        torch.cuda.synchronize()
        barrier(ws)
        xch.close()
    del layers
    torch.cuda.empty_cache()
    fields = ["T_per_gpu", "us_per_layer", "tokens_per_s"] + (
        ["nccl_us_per_layer", "nccl_tokens_per_s"] if ws > 1 else [])
    return {"config": "qwen3-235b-a22b int4-g64, 8 layers, experts split over the GPUs (peer-memory exchange, "
                      "CUDA graph; NCCL all-to-all-v eager beside it)",
            "experts_per_gpu": e // ws, "fields": fields, "rows": rows, "device_errors": errs}


def run_ep(a, ws, rank, local, peaks):
    from moelab_b200 import ep
    T = a.tokens
    sweep_T = [int(s_) for s_ in a.sweep.split(",") if s_.strip()]
    layers = make_ep_layers(a.layers, rank, ws)
    xch = ep.PeerExchange.create(max([T] + sweep_T) * K_TOP, D)
    try:
        xs = make_inputs(T, a.layers, seed=5 + rank)
        ep_steps(layers, xs, max(a.warmup, 3), xch)  # eager warm-up (also sizes the workspaces)
        torch.cuda.synchronize()
        gr = ep_graph(layers, xs, a.steps, xch, ws)
        clocks = ClockSampler(local)
        clocks.start()
        t_soak = time.perf_counter()
        while time.perf_counter() - t_soak < a.soak_seconds:
            barrier(ws)
            gr.replay()
            torch.cuda.synchronize()
        t = max_over_ranks(ws, time_graph(gr, ws))
        ck = clocks.stop()
        value = ws * T * a.steps / t
        lay_b = ep_layer_bytes(layers, xs, len(layers), xch, ws)
        lay_ach = lay_b / (t / a.steps) / 1e9
        del gr
        sweep = []
        for Ts in sweep_T:
            xs_s = make_inputs(Ts, a.layers, seed=77 + Ts + rank)
            ep_steps(layers, xs_s, 3, xch)
            n_s = 2 * a.layers
            gs = ep_graph(layers, xs_s, n_s, xch, ws)
            ts = max_over_ranks(ws, time_graph(gs, ws))
            del gs
            sweep.append({"T": Ts, "us_per_call": round(ts / n_s * 1e6, 3), "tokens_per_s": round(ws * Ts * n_s / ts, 1)})
        # end to end through the public API with host buffers (eager, copies double-buffered on a side stream)
        gh = torch.Generator().manual_seed(9 + rank)
        xh = [torch.randn(T, D, generator=gh).to(torch.bfloat16).pin_memory() for _ in range(8)]
        yh = [torch.empty_like(xh[0]).pin_memory() for _ in range(8)]

        def call(i, xd):
            st, gate = layers[i % len(layers)]
            return ep.layer_p2p(st, xd, gate, K_TOP, xch, residual=xd, max_tokens=T)

        te = max_over_ranks(ws, e2e_loop(call, xh, yh, a.e2e_steps, ws))
        errs = xch.read_error()
        torch.cuda.synchronize()
        barrier(ws)
    finally:
        torch.cuda.synchronize()
        barrier(ws)
        xch.close()
    stack = ep_stack(a, ws, rank) if a.ep_stack else None  # every rank takes part
    if rank != 0:
        return
    line = {
        "metric": "MoE-layer tokens/s", "value": round(value, 1), "unit": "tokens/s", "n_gpus": ws,
        "steps": a.steps, "warmup": max(a.warmup, 3), "ms_per_step": round(t / a.steps * 1e3, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,0.02) weights, N(0,1) tokens)",
        "config": {"workload": WORKLOAD + ", experts split over the GPUs", "tokens_per_gpu": T, "d": D, "f": F,
                   "E": E, "k": K_TOP, "layers": a.layers, "experts_per_gpu": E // ws,
                   "weights_gb_per_gpu": round(a.layers * 3 * (E // ws) * D * F * W_BITS / 8 / 1e9, 2),
                   "l2": "inputs larger than L2: 16 independent layers cycled",
                   "parallelism": f"ep{ws}",
                   "exchange": "NVLink peer memory (CUDA IPC buffers): dispatch and return stored by the kernels, "
                               "epoch flags, no host synchronisation",
                   "graph": "one CUDA graph of K steps per rank"},
        "us_per_call": round(t / a.steps * 1e6, 3),
        "layer_gbs_per_gpu": round(lay_ach, 1), "layer_frac_of_hbm_peak": round(lay_ach / peaks["hbm_gbs"], 3),
        "sweep": sweep,
        "roofline": {"bound": "hbm", "kernel": "whole expert-parallel layer per GPU (router, dispatch, experts, "
                                               "return, combine)",
                     "achieved": round(lay_ach, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(lay_ach / peaks["hbm_gbs"], 3), "traffic": None,
                     "peak_source": f"{peaks['source']} (MEASURED_PEAKS.json hbm_gbs)",
                     "algorithmic_bytes_per_launch": round(lay_b)},
        "cpu_baseline": None,
        "e2e": {"value": round(ws * T * a.e2e_steps / te, 1), "unit": "tokens/s", "h2d_bytes_per_step": T * D * 2,
                "d2h_bytes_per_step": T * D * 2, "us_per_call": round(te / a.e2e_steps * 1e6, 3),
                "note": "public API ep.layer_p2p() eager; every step's x in from / y out to pinned host memory, on a "
                        "side stream double-buffered against the compute"},
        "device_errors": errs,
        "clocks": ck,
        "gpu_launches": 8 * a.steps,  # router, plan, send, prep, gate/up, down, signal, combine
    }
    if stack is not None:
        line["ep_stack"] = stack
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ main
def run_reference(a, ws, rank):
    if rank != 0:
        return
    val, n, el = cpu_baseline(a.tokens, a.cpu_seconds, warmup=a.warmup, steps=a.steps)
    cores = torch.get_num_threads()
    line = {"metric": "MoE-layer tokens/s", "value": round(val, 2), "unit": "tokens/s", "n_gpus": a.gpus,
            "steps": n, "warmup": a.warmup, "ms_per_step": round(el / n * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": WORKLOAD, "tokens_per_step": a.tokens, "d": D, "f": F, "E": E, "k": K_TOP,
                       "layers": 1, "parallelism": "cpu"},
            "cpu_baseline": {"value": round(val, 2), "unit": "tokens/s", "cores": cores, "kind": "port",
                             "sample": f"{n} layer calls of T={a.tokens} tokens (router + torch_loop) on one "
                                       f"dequantised layer, {el:.1f} s"},
            "e2e": {"value": round(val, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def probe_tc():
    """One JSON line per case of moeb_probe_tc_issue (cycles per M=128, K=16 MMA per SM; TFLOP/s over the GPU),
    then mma.sync m16n8k16 rates. 200k MMAs per issuer per case."""
    import ctypes
    from moelab_b200 import _lib
    cyc, tf, sc = ctypes.c_double(), ctypes.c_double(), ctypes.c_double()
    for n in (16, 32, 64, 128):  # MMAs beside TMEM stores (dequant warps) / loads (epilogue warps), random operands
        for iss in (1, 2, 4):
            if iss * (64 if n <= 64 else 128) > 384:
                continue
            for side in (1, 2, 3):
                _lib.call("moeb_probe_tc_issue", n, iss, 16, 1, 1, side, 200000, ctypes.byref(cyc), ctypes.byref(tf),
                          ctypes.byref(sc))
                print(json.dumps({"probe": "tcgen05.mma M128 K16 beside " + ("TMEM stores", "TMEM loads", "ALU work")[side - 1],
                                  "N": n, "issuers": iss, "cycles_per_mma_per_sm": round(cyc.value, 1),
                                  "side_cycles_per_op_per_warp": round(sc.value, 1)}), flush=True)
    for data in (0, 1):
        for n in (16, 32, 64, 128, 256):
            for iss in (1, 2, 3, 4):
                if iss * (64 if n <= 64 else 128 if n <= 128 else 256) > 384:
                    continue
                for per, wait in ((16, 0), (4, 1), (16, 1)):
                    _lib.call("moeb_probe_tc_issue", n, iss, per, wait, data, 0, 200000, ctypes.byref(cyc),
                              ctypes.byref(tf), None)
                    print(json.dumps({"probe": "tcgen05.mma M128 K16", "operands": "random" if data else "zero",
                                      "N": n, "issuers": iss, "mmas_per_wait": per, "wait": bool(wait),
                                      "cycles_per_mma_per_sm": round(cyc.value, 1), "tflops": round(tf.value, 1)}),
                          flush=True)
    for w in (4, 8, 16):
        _lib.call("moeb_probe_mma_sync", w, 20000, ctypes.byref(tf))
        print(json.dumps({"probe": "mma.sync m16n8k16 bf16", "warps_per_sm": w, "tflops": round(tf.value, 1)}),
              flush=True)


def profile_config(a):
    """A few eager layer calls of one configuration: the small, self-ending workload ncu captures are taken on."""
    headline = ("qwen3-30b-a3b int4 (headline layer)", dict(d=D, f=F, E=E, k=K_TOP), "q4", [])
    name, shp, kind, _ = next(c for c in [headline] + CONFIGS if c[0].startswith(a.profile_config))
    if a.profile_policy:
        from moelab_b200 import ops
        from moelab_b200.variants.cuda import b200_mxfp4_moe as vm, b200_q4_moe as vq
        pol = {"slots": ops.POLICY_SLOTS, "tiles8": ops.POLICY_TILES8, "tiles16": ops.POLICY_TILES16,
               "ring8": ops.POLICY_TILES8_RING, "ring16": ops.POLICY_TILES16_RING,
               "ring24": ops.POLICY_TILES24_RING, "tc": ops.POLICY_TC,
               "decode": ops.POLICY_DECODE}[a.profile_policy]
        vq.POLICY = vm.POLICY = pol  # the gpt-oss variant runs through vm
    layers, _ = config_layers(shp["d"], shp["f"], shp["E"], shp["k"], kind, n_layers=1)
    st, gate, call = layers[0]
    x = torch.randn(a.profile_tokens, shp["d"], generator=torch.Generator(device="cuda").manual_seed(3),
                    device="cuda").to(torch.bfloat16)
    for _ in range(3):
        call(st, x, gate)
    torch.cuda.synchronize()
    print(json.dumps({"profile_config": name, "T": a.profile_tokens, "ok": True}))


def main():
    a = parse()
    if a.probe_tc:
        probe_tc()
        return
    if a.profile_config:
        profile_config(a)
        return
    ws, rank, local = dist_init(a)
    if a.impl == "reference":
        run_reference(a, ws, rank)
        return
    from moelab_b200 import roofline
    peaks = roofline.b200_peaks()
    if ws > 1:
        run_ep(a, ws, rank, local, peaks)
        return
    T = a.tokens
    v, layers = make_layers(a.layers, seed=1000 + 7919 * rank, device="cuda")
    xs = make_inputs(T, a.layers, seed=5 + rank)
    # warm-up: W untimed eager steps
    for i in range(a.warmup):
        st, gate = layers[i % len(layers)]
        v.layer(st, xs[i % len(layers)], gate, K_TOP, residual=xs[i % len(layers)])
    torch.cuda.synchronize()
    # headline: one CUDA graph of exactly K steps
    gr, _ = capture(v, layers, xs, a.steps)
    gr.replay()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    t_soak = time.perf_counter()
    while time.perf_counter() - t_soak < a.soak_seconds:
        gr.replay()
        torch.cuda.synchronize()
    t = time_graph(gr, ws)
    ck = clocks.stop()
    t = max_over_ranks(ws, t)
    value = ws * T * a.steps / t
    # per-kernel times and roofline of the dominant kernel (gate/up)
    n_stage = min(4 * a.layers, a.steps)
    r_us, gu_us, dn_us, idxs = stage_times(v, layers, xs, n_stage)
    gu_b = [gate_up_bytes(i, T) for i in idxs]
    dn_b = [down_bytes(i, T) for i in idxs]
    gu_ach = sum(gu_b) / (sum(gu_us) * 1e-6) / 1e9
    dn_ach = sum(dn_b) / (sum(dn_us) * 1e-6) / 1e9
    lay_b = layer_bytes(idxs[:len(layers)], T)  # the graph cycles the same L (layer, input) pairs
    lay_ach = sum(lay_b) / len(lay_b) / (t / a.steps) / 1e9
    traffic = None
    tp = os.path.join(ROOT, "profiles", "traffic_gate_up.json")
    if os.path.exists(tp):
        try:
            traffic = json.load(open(tp)).get(str(T))  # ncu dram bytes of one launch, committed summary
        except (OSError, ValueError):
            traffic = None
    sweep = []
    for Ts in [int(s) for s in a.sweep.split(",") if s.strip()]:
        sweep.append(measure_T(v, layers, Ts, ws, rank, 2 * a.layers if Ts >= 256 else 4 * a.layers, 77 + Ts, peaks))
    trace = measure_trace(v, layers, peaks) if a.trace else []
    # end to end through the public API with host buffers (8 distinct pinned inputs cycled)
    gh = torch.Generator().manual_seed(9)
    xh = [torch.randn(T, D, generator=gh).to(torch.bfloat16).pin_memory() for _ in range(8)]
    yh = [torch.empty_like(xh[0]).pin_memory() for _ in range(8)]

    def call(i, xd):
        st, gate = layers[i % len(layers)]
        return v.layer(st, xd, gate, K_TOP, residual=xd)

    te = max_over_ranks(ws, e2e_loop(call, xh, yh, a.e2e_steps, ws))
    e2e = {"value": round(ws * T * a.e2e_steps / te, 1), "unit": "tokens/s", "h2d_bytes_per_step": T * D * 2,
           "d2h_bytes_per_step": T * D * 2, "us_per_call": round(te / a.e2e_steps * 1e6, 3),
           "note": "public API v.layer() eager, no graph; every step's x copied in from pinned host memory and y "
                   "copied out to it, on a side stream double-buffered against the compute"}
    configs = []
    if a.configs:
        for name, shp, kind, Ts in CONFIGS:
            configs += measure_config(name, shp, kind, Ts, peaks)
    del layers
    torch.cuda.empty_cache()
    stack = ep_stack(a, ws, rank) if a.ep_stack else None  # the expert-parallel stack's N = 1 row
    cpu = None
    if rank == 0 and ws == 1:
        val, n, el = cpu_baseline(T, a.cpu_seconds)
        cpu = {"value": round(val, 2), "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
               "sample": f"{n} layer calls of T={T} tokens (torch router + port of torch_loop.run) on one "
                         f"dequantised layer, {el:.1f} s"}
    if rank != 0:
        return
    lay_t = t / a.steps
    lay_flops = 6.0 * D * F * T * K_TOP
    cfg = {"fields": ["T", "us_per_call", "layer_roofline_frac"]}
    for c in configs:
        cfg.setdefault(c["config"].split(" (")[0], []).append([c["T"], c["us_per_call"], c["roofline_frac"]])
    # key figures last, so a truncated record still ends with them: sweep, layer fraction, roofline, CPU baseline
    line = {
        "metric": "MoE-layer tokens/s", "value": round(value, 1), "unit": "tokens/s", "n_gpus": ws,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(t / a.steps * 1e3, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,0.02) weights, N(0,1) tokens)",
        "config": {"workload": WORKLOAD, "tokens_per_gpu": T, "d": D, "f": F, "E": E, "k": K_TOP,
                   "layers": a.layers, "weights_gb_per_gpu": round(a.layers * 3 * E * D * F * W_BITS / 8 / 1e9, 2),
                   "l2": "inputs larger than L2: 16 independent layers cycled (5.4 GB of expert weights)",
                   "parallelism": "single" if ws == 1 else f"replicas{ws}", "graph": "one CUDA graph of K steps"},
        "us_per_call": round(t / a.steps * 1e6, 3),
        "e2e": e2e, "clocks": ck,
        "gpu_launches": (3 if T * K_TOP <= 16 else 4) * a.steps,  # router, gate/up, down (+ combine in tile mode)
        "kernels_us": {"router": round(statistics.mean(r_us), 2), "gate_up": round(statistics.mean(gu_us), 2),
                       "down": round(statistics.mean(dn_us), 2), "note": "CUDA events between stages (eager)"},
        "configs": cfg,
        "trace": {"workload": "qwen3-30b int4 on the reference's recorded routing traces, harness run()",
                  "fields": ["T", "us_per_call", "layer_roofline_frac", "reference_m4pro_us"], "rows": trace},
        "ep_stack": stack,
        "sweep": {"fields": ["T", "us_per_call", "layer_roofline_frac", "layer_gbs"],
                  "rows": [[s_["T"], s_["us"], s_["frac"], s_["gbs"]] for s_ in sweep]},
        "layer_frac_of_hbm_peak": round(lay_ach / peaks["hbm_gbs"], 3),
        "roofline": {"bound": "hbm", "kernel": "k_gate_up_slots" if T * K_TOP <= 16 else "k_experts_ws (gate/up)",
                     "achieved": round(gu_ach, 1), "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": round(gu_ach / peaks["hbm_gbs"], 3), "traffic": traffic,
                     "peak_source": "MEASURED_PEAKS.json hbm_gbs" if peaks["source"] == "measured"
                     else "fallback 6650 GB/s",
                     "algorithmic_bytes_per_launch": round(statistics.mean(gu_b)),
                     "down_achieved_gbs": round(dn_ach, 1),
                     "layer": {"frac": round(layer_frac(statistics.mean(lay_b), lay_flops, lay_t, peaks), 3),
                               "us": round(lay_t * 1e6, 2), "bytes": round(statistics.mean(lay_b)),
                               "flops": lay_flops, "def": "max(bytes / HBM peak, FLOPs / bf16 peak) / measured"}},
        "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    try:
        main()
    finally:
        if int(os.environ.get("WORLD_SIZE", "1")) > 1:
            import torch.distributed as dist
            if dist.is_initialized():
                dist.destroy_process_group()
