"""Rank bodies for the expert-parallel tests (run in spawned processes: gloo on CPU, NCCL on GPUs)."""
import datetime
import os
import traceback

import numpy as np
import torch
import torch.distributed as dist


def free_port():
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _init(rank, P, port, backend):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group(backend, rank=rank, world_size=P, timeout=datetime.timedelta(seconds=60))


def full_layer_cpu(d, f, E, seed):
    """int4-g64 layer quantised by the oracle, dequantised to fp32 (the weights every rank agrees on)."""
    import oracle
    g = torch.Generator().manual_seed(seed)
    mk = lambda *s: (torch.randn(*s, generator=g) * 0.02).to(torch.bfloat16)  # noqa: E731
    w = []
    for shape in ((E, f, d), (E, f, d), (E, d, f)):
        w.append(oracle.q4_dequant(*oracle.q4_quantize(mk(*shape))))
    return w, mk(E, d)


def host_rank(rank, P, port, tokens, d, f, E, k, seed, q):
    """gloo rank: moelab_b200.ep.layer driven by the host kernels; checked against the single-process oracle."""
    try:
        _init(rank, P, port, "gloo")
        import oracle
        from oracle.ep import HostKernels, host_shard
        from moelab_b200 import ep
        (wg, wu, wd), gate = full_layer_cpu(d, f, E, seed)
        T = tokens[rank]
        x = torch.randn(T, d, generator=torch.Generator().manual_seed(seed + 1 + rank)).to(torch.bfloat16)
        st = host_shard(wg, wu, wd, rank, P)
        tm = {}
        y, idx, wts = ep.layer(st, x, gate, k, residual=x, kernels=HostKernels, return_routing=True, timings=tm)
        ri, rw = oracle.router(x, gate, k)
        assert np.array_equal(idx.numpy(), ri) and np.array_equal(wts.numpy(), rw)
        ref = oracle.moe_forward(x.float().numpy(), wg, wu, wd, ri, rw) + x.float().numpy()
        e = oracle.error_metrics(y.float().numpy(), ref) if T else {"rel_fro": 0.0, "max_rowrel": 0.0,
                                                                    "finite": True}
        # conservation: every slot is sent once and comes back once
        tot = torch.tensor([tm["rows_sent"], tm["rows_received"]], dtype=torch.int64)
        dist.all_reduce(tot)
        q.put((rank, "ok", {"metrics": e, "sent": tm["rows_sent"], "recv": tm["rows_received"],
                            "tot": tot.tolist(), "T": T}))
    except Exception:  # reported to the parent, which fails the test
        q.put((rank, "error", traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def nccl_rank(rank, P, port, tokens, d, f, E, k, seed, policy, fmt, q):
    """NCCL rank on GPU `rank`: the CUDA expert-parallel layer against the single-GPU layer on the full weights
    (computed on every rank) - bit-exact under a pinned policy."""
    try:
        torch.cuda.set_device(rank)
        _init(rank, P, port, "nccl")
        import importlib
        from moelab_b200 import ep, ops
        v = importlib.import_module("moelab_b200.variants.cuda." + ("b200_mxfp4_moe" if fmt == "mxfp4"
                                                                    else "b200_q4_moe"))
        v.POLICY = policy
        g = torch.Generator(device="cuda").manual_seed(seed)
        mk = lambda *s: (torch.randn(*s, generator=g, device="cuda") * 0.02).to(torch.bfloat16)  # noqa: E731
        w = [mk(E, f, d), mk(E, f, d), mk(E, d, f)]
        gate = mk(E, d)
        full = v.prepare(*w)
        st = ep.shard(v, *w, rank, P)
        T = tokens[rank]
        x = torch.randn(T, d, generator=torch.Generator(device="cuda").manual_seed(seed + 1 + rank),
                        device="cuda").to(torch.bfloat16)
        y, idx, wts = ep.layer(st, x, gate, k, residual=x, policy=policy, return_routing=True)
        v._ws(full, k)
        ysingle = ops.experts(full, x, idx, wts, policy=policy, residual=x) if T else y
        torch.cuda.synchronize()
        q.put((rank, "ok", {"y": y.float().cpu(), "x": x.float().cpu(), "idx": idx.cpu(), "wts": wts.cpu(),
                            "ysingle": ysingle.float().cpu()}))
    except Exception:
        q.put((rank, "error", traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


class ThreadGroup:
    """P ranks emulated by P threads of one process on one device: all_to_all_single over shared memory.
    The threads share the device's default stream, so a receiver's copy is ordered after the sender's kernels."""

    def __init__(self, P):
        import threading
        self.P = P
        self.barrier = threading.Barrier(P, timeout=120)
        self.box = [None] * P

    def comm(self, rank):
        group = self

        class _Comm:
            def all_to_all_single(self, out, inp, out_splits=None, in_splits=None):
                P = group.P
                ins = in_splits or [inp.shape[0] // P] * P
                outs = out_splits or [out.shape[0] // P] * P
                group.box[rank] = list(torch.split(inp, ins))
                group.barrier.wait()
                parts = [group.box[src][rank] for src in range(P)]
                assert [p.shape[0] for p in parts] == list(outs), "split sizes disagree between ranks"
                if out.numel():
                    torch.cat(parts, out=out)
                group.barrier.wait()

        return _Comm()

    def run(self, body):
        """body(rank, comm) on P threads; returns the P results (re-raises the first failure)."""
        import threading
        res, err = [None] * self.P, []

        def wrap(r):
            try:
                res[r] = body(r, self.comm(r))
            except Exception as e:  # noqa: BLE001
                err.append(e)
                self.barrier.abort()

        th = [threading.Thread(target=wrap, args=(r,)) for r in range(self.P)]
        for t in th:
            t.start()
        for t in th:
            t.join()
        if err:
            raise err[0]
        return res


def p2p_rank(rank, P, port, tokens, d, f, E, k, seed, policy, calls, q):
    """Rank on GPU `rank`: the peer-memory expert-parallel layer (CUDA IPC buffers, eager and in a CUDA graph)
    against the single-GPU layer on the full weights, bit-exact."""
    xch = None
    try:
        torch.cuda.set_device(rank)
        _init(rank, P, port, "nccl")
        from moelab_b200 import ep, ops
        from moelab_b200.variants.cuda import b200_q4_moe as v
        g = torch.Generator(device="cuda").manual_seed(seed)
        mk = lambda *s: (torch.randn(*s, generator=g, device="cuda") * 0.02).to(torch.bfloat16)  # noqa: E731
        w = [mk(E, f, d), mk(E, f, d), mk(E, d, f)]
        gate = mk(E, d)
        full = v.prepare(*w)
        v._ws(full, k)
        st = ep.shard(v, *w, rank, P)
        xch = ep.PeerExchange.create(max(tokens) * k, d)
        T = tokens[rank]
        bad = []
        xs = []
        for c in range(calls):
            x = torch.randn(T, d, generator=torch.Generator(device="cuda").manual_seed(seed + 10 * c + rank),
                            device="cuda").to(torch.bfloat16)
            xs.append(x)
            y, idx, wts = ep.layer_p2p(st, x, gate, k, xch, residual=x, policy=policy, return_routing=True)
            if T:
                ys = ops.experts(full, x, idx, wts, policy=policy, residual=x)
                if not torch.equal(y, ys):
                    bad.append(("eager", c, float((y.float() - ys.float()).abs().max())))
        # the same sequence captured in a CUDA graph and replayed (every rank replays it)
        torch.cuda.synchronize()
        dist.barrier()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(gr, stream=s):
                ys_g = [ep.layer_p2p(st, x, gate, k, xch, residual=x, policy=policy, max_tokens=max(tokens))
                        for x in xs]
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        dist.barrier()
        gr.replay()
        torch.cuda.synchronize()
        for c, x in enumerate(xs):
            if T:
                idx, wts = ops.router(x, gate, k)
                ys = ops.experts(full, x, idx, wts, policy=policy, residual=x)
                if not torch.equal(ys_g[c], ys):
                    bad.append(("graph", c, float((ys_g[c].float() - ys.float()).abs().max())))
        dist.barrier()
        err = xch.read_error() | st["ep_ws"].read_error()
        del gr
        q.put((rank, "ok", {"bad": bad, "err": err}))
    except Exception:
        q.put((rank, "error", traceback.format_exc()))
    finally:
        if xch is not None:
            try:
                torch.cuda.synchronize()
                if dist.is_initialized():
                    dist.barrier()
                xch.close()
            except Exception:  # noqa: BLE001
                pass
        if dist.is_initialized():
            dist.destroy_process_group()
