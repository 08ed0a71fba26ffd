"""Host-memory Sol-Attn streamed by head chunks (solb200.sol_attn_host): the chunk plan
and argument checks on CPU; on the GPU, every head's output must equal the one-shot
device call's bit for bit (heads are independent and run the same kernels)."""

import pytest
import torch

import solb200
from solb200.streamed import plan_chunks


def test_plan_chunks():
    assert plan_chunks(40) == [(h, 2) for h in range(0, 40, 2)]
    assert plan_chunks(64) == [(h, 2) for h in range(0, 64, 2)]
    assert plan_chunks(5) == [(h, 1) for h in range(5)]     # a rank of eight at 40 heads
    assert plan_chunks(6, 4) == [(0, 4), (4, 2)]
    assert plan_chunks(3) == [(0, 1), (1, 1), (2, 1)]
    assert plan_chunks(1) == [(0, 1)]
    assert plan_chunks(1, 8) == [(0, 1)]
    with pytest.raises(ValueError):
        plan_chunks(0)


def test_host_arguments_rejected():
    q = torch.zeros(1, 64, 2, 64, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="bfloat16"):
        solb200.sol_attn_host(q, q, q)
    q = torch.zeros(1, 64, 2, 64, dtype=torch.bfloat16).transpose(1, 2)
    with pytest.raises(RuntimeError, match="contiguous"):
        solb200.sol_attn_host(q, q, q)


@pytest.mark.gpu
@pytest.mark.parametrize("shape,block,hpc", [((1, 4096, 6, 128), 128, 4), ((2, 1000, 3, 64), 64, 2)])
@pytest.mark.parametrize("int8", [False, True])
def test_streamed_equals_device_call(cuda_device, shape, block, hpc, int8):
    g = torch.Generator().manual_seed(3)
    q, k, v = (torch.randn(*shape, generator=g).to(torch.bfloat16).pin_memory() for _ in range(3))
    got = solb200.sol_attn_host(q, k, v, tau=0.9, block=block, int8=int8, heads_per_chunk=hpc)
    fn = solb200.sol_attn_int8 if int8 else solb200.sol_attn
    want = fn(q.cuda(), k.cuda(), v.cuda(), tau=0.9, block=block).cpu()
    assert got.shape == want.shape and got.dtype == torch.bfloat16
    assert torch.equal(got, want)


@pytest.mark.gpu
def test_streamed_buffers_kept_across_calls(cuda_device):
    """Back-to-back calls (no synchronisation in between) reuse the kept chunk slots and
    streams; each call's output is its own device call's."""
    g = torch.Generator().manual_seed(4)
    shape = (1, 4096, 5, 128)
    inputs = [tuple(torch.randn(*shape, generator=g).to(torch.bfloat16).pin_memory() for _ in range(3))
              for _ in range(3)]
    outs = [solb200.sol_attn_host(*x, tau=0.9, block=128, synchronize=False) for x in inputs]
    torch.cuda.synchronize()
    for x, got in zip(inputs, outs):
        want = solb200.sol_attn(*(t.cuda() for t in x), tau=0.9, block=128).cpu()
        assert torch.equal(got, want)
    solb200.release_host_buffers()
