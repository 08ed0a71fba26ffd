"""Multi-rank layout logic on CPU ranks (gloo, world size 2): the Ulysses re-sharding
is an exact permutation, and attention computed through it equals attention on the
full tensors (heads are independent). The attention here is the CPU oracle, standing
in for the GPU kernel, so the test needs no GPU."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from solb200.parallel import head_shard, head_to_seq, seq_to_head, ulysses_attention


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_q):
    import sys
    from pathlib import Path
    repo = Path(__file__).resolve().parent.parent
    sys.path[:0] = [str(repo), str(repo / "comfyui-solattn_triton_b200")]
    from oracle import solattn_oracle as O
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(7)
        B, T, H, D = 1, 256, 4, 64
        q, k, v = (torch.randn(B, T, H, D, generator=g).to(torch.bfloat16) for _ in range(3))
        Tl = T // world
        ql, kl, vl = (t[:, rank * Tl:(rank + 1) * Tl] for t in (q, k, v))
        # round trip is the identity
        back = head_to_seq(seq_to_head(ql))
        ok_rt = torch.equal(back, ql)
        # rank r receives the full sequence of heads r*H/W ..
        full = seq_to_head(ql)
        ok_heads = torch.equal(full, q[:, :, head_shard(rank, world, H)])

        def attn(a, b, c, **kw):
            o = O.sol_attn(O.to_np(a), O.to_np(b), O.to_np(c), tau=0.9, block=64)
            return torch.from_numpy(o).to(torch.bfloat16)

        out = ulysses_attention(ql, kl, vl, attn)
        want = O.sol_attn(O.to_np(q), O.to_np(k), O.to_np(v), tau=0.9, block=64)
        want_local = torch.from_numpy(want[:, rank * Tl:(rank + 1) * Tl]).to(torch.bfloat16)
        ok_attn = torch.equal(out, want_local)
        out_q.put((rank, ok_rt, ok_heads, ok_attn))
    finally:
        dist.destroy_process_group()


def test_ulysses_resharding_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert [r[0] for r in res] == [0, 1]
    for rank, ok_rt, ok_heads, ok_attn in res:
        assert ok_rt, f"rank {rank}: round trip"
        assert ok_heads, f"rank {rank}: head slice"
        assert ok_attn, f"rank {rank}: attention through the all-to-all"


def test_head_shard():
    assert head_shard(1, 4, 40) == slice(10, 20)
    with pytest.raises(ValueError):
        head_shard(0, 3, 40)
