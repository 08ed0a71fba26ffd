"""Ulysses layout on GPUs (NCCL, two ranks): sequence-sharded q/k/v go through the
all-to-all to head shards, the local sm_100a Sol-Attn runs on whole sequences, and the
inverse all-to-all returns sequence shards. The result must equal the single-GPU call
on the full tensors bit for bit (heads are independent). Skipped with fewer than two
GPUs; NVLS is switched off and the process group has a short timeout."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, int8, q_ref):
    import sys
    from datetime import timedelta
    from pathlib import Path
    repo = Path(__file__).resolve().parent.parent
    sys.path[:0] = [str(repo), str(repo / "comfyui-solattn_triton_b200")]
    import torch.distributed as dist
    import solb200
    from solb200.parallel import ulysses_attention
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        q, k, v = (t.cuda() for t in q_ref)
        T = q.shape[1]
        tl = T // world
        ql, kl, vl = (t[:, rank * tl:(rank + 1) * tl].contiguous() for t in (q, k, v))
        fn = solb200.sol_attn_int8 if int8 else solb200.sol_attn
        out = ulysses_attention(ql, kl, vl, fn, tau=0.9, block=128)
        want = fn(q, k, v, tau=0.9, block=128)[:, rank * tl:(rank + 1) * tl]
        torch.cuda.synchronize()
        ok = torch.equal(out, want)
        dist.barrier()
    finally:
        dist.destroy_process_group()
    if not ok:
        raise AssertionError(f"rank {rank}: Ulysses output differs from the single-GPU call")


@pytest.mark.parametrize("int8", [False, True])
def test_ulysses_two_gpus(cuda_device, int8):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    g = torch.Generator().manual_seed(5)
    B, T, H, D = 1, 4096, 8, 128
    qkv = tuple(torch.randn(B, T, H, D, generator=g).to(torch.bfloat16) for _ in range(3))
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, int8, qkv)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0, 0], f"rank exit codes {codes}"
