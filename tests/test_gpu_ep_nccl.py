"""Expert parallelism over real GPUs: P processes, one per GPU, NCCL all-to-all over NVLink. Each rank's output
must equal, bit for bit, the single-GPU layer on the full weights (same expert kernels, pinned policy).
Needs >= 2 GPUs (skipped otherwise)."""
import multiprocessing as mp

import pytest
import torch

from ep_workers import free_port, nccl_rank
from moelab_b200 import ops

pytestmark = pytest.mark.gpu


def _ngpu():
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.mark.skipif(_ngpu() < 2, reason="needs 2 or more GPUs")
@pytest.mark.parametrize("fmt,policy", [("q4", ops.POLICY_TILES8), ("q4", ops.POLICY_SLOTS),
                                        ("mxfp4", ops.POLICY_TILES8)])
def test_nccl_ep_bit_exact_vs_single_gpu(fmt, policy):
    P = min(_ngpu(), 8)
    tokens = [5, 0, 17, 1, 64, 3, 2, 9][:P]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    args = lambda r: (r, P, port, tokens, 512, 256, 32, 4, 21, policy, fmt, q)  # noqa: E731
    procs = [ctx.Process(target=nccl_rank, args=args(r)) for r in range(P)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(P):
            rank, status, payload = q.get(timeout=300)
            assert status == "ok", payload
            out[rank] = payload
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for r in range(P):
        assert torch.equal(out[r]["y"], out[r]["ysingle"]), r


@pytest.mark.skipif(_ngpu() < 2, reason="needs 2 or more GPUs")
@pytest.mark.parametrize("policy", [ops.POLICY_TILES8_RING, ops.POLICY_TILES16_RING, ops.POLICY_SLOTS])
def test_p2p_ep_bit_exact_vs_single_gpu(policy):
    """The peer-memory exchange over real GPUs (CUDA IPC mappings over NVLink), eager and as a CUDA graph."""
    from ep_workers import p2p_rank
    P = min(_ngpu(), 8)
    tokens = [5, 0, 17, 1, 64, 3, 2, 9][:P]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=p2p_rank, args=(r, P, port, tokens, 512, 256, 32, 4, 31, policy, 3, q))
             for r in range(P)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(P):
            rank, status, payload = q.get(timeout=300)
            assert status == "ok", payload
            out[rank] = payload
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for r in range(P):
        assert out[r]["bad"] == [] and out[r]["err"] == 0, (r, out[r])
