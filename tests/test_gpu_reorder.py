"""The reordered call (``token_order=``, C ABI ``solb200_sol_attn_reordered``): attention over
the tokens in a given order with the output returned in input order, the Morton hooks'
gathers of the reference (``_morton.py:115-148``, ``_morton_h3.py:161-218``) fused into the
pooling pass and the forward's epilogue. It must equal, bit for bit, gathering q/k/v by
the order, the plain call, and gathering the output by the inverse order."""

import ctypes

import pytest
import torch

from conftest import golden_meta, load_golden

import solb200
from solb200.workloads import CONFIGS, make_qkv

pytestmark = pytest.mark.gpu


def _unfused(fn, q, k, v, perm, inv, **kw):
    qp, kp, vp = solb200.permute_tokens_many([t.contiguous() for t in (q, k, v)], perm)
    return solb200.permute_tokens(fn(qp, kp, vp, **kw), inv)


def _paths():
    return [("bf16", solb200.sol_attn, {}), ("int8", solb200.sol_attn_int8, {"int8_pv": True}),
            ("int8-bf16pv", solb200.sol_attn_int8, {"int8_pv": False})]


@pytest.mark.parametrize("name,curve", [("c1", "3d"), ("d128", "2d_frame"), ("ragged", "3d")])
@pytest.mark.parametrize("path,fn,extra", _paths())
def test_reordered_equals_gather_call_gather(cuda_device, name, curve, path, fn, extra):
    g = load_golden(name)
    B, T, H, D, blk = golden_meta(g)
    q, k, v = (torch.from_numpy(g[x]).to(torch.bfloat16).cuda() for x in ("q", "k", "v"))
    # a permutation of the T tokens: the Morton order of a grid holding them, or a seeded shuffle
    grid = {512: (2, 16, 16)}.get(T)
    if grid is not None:
        perm, inv = solb200.morton_perm(grid, cuda_device, curve)
    else:
        gen = torch.Generator(device="cpu").manual_seed(T)
        perm = torch.randperm(T, generator=gen).to(cuda_device)
        inv = torch.argsort(perm)
    kw = dict(tau=float(g["tau"]), block=blk, **extra)
    got = fn(q, k, v, token_order=perm, **kw)
    want = _unfused(fn, q, k, v, perm, inv, **kw)
    assert torch.equal(got, want), f"{name} {path}: {(got != want).sum().item()} elements differ"


@pytest.mark.parametrize("path,fn,extra", _paths())
def test_reordered_config3_slice_morton(cuda_device, path, fn, extra):
    """The headline grid (21, 30, 52), two heads, both curves, with q/k/v as BHND views."""
    cfg = CONFIGS["c3"]
    q, k, v = make_qkv(cfg, device=cuda_device, heads=slice(0, 2))
    q, k, v = (t.transpose(1, 2).contiguous().transpose(1, 2) for t in (q, k, v))   # strided views
    for curve in ("3d", "2d_frame"):
        perm, inv = solb200.morton_perm(cfg.grid, cuda_device, curve)
        kw = dict(tau=cfg.tau, block=cfg.block, **extra)
        got = fn(q, k, v, token_order=perm, **kw)
        want = _unfused(fn, q, k, v, perm, inv, **kw)
        assert torch.equal(got, want), f"{curve} {path}"


def test_reordered_rejects_bad_index_without_fault(cuda_device):
    """An index outside [0, T) is recorded in the device error word and never dereferenced:
    the call reports an invalid-argument error, the context stays usable."""
    g = torch.Generator(device="cpu").manual_seed(2)
    q, k, v = (torch.randn(1, 1024, 2, 128, generator=g).to(torch.bfloat16).cuda() for _ in range(3))
    perm = torch.arange(1024, device=cuda_device)
    perm[17] = 5000
    with pytest.raises(RuntimeError, match="outside"):
        solb200.sol_attn(q, k, v, tau=0.9, block=128, token_order=perm)
    perm[17] = 17
    assert torch.equal(solb200.sol_attn(q, k, v, tau=0.9, block=128, token_order=perm),
                       solb200.sol_attn(q, k, v, tau=0.9, block=128))


def test_reordered_workspace_extends_the_plain_one(cuda_device):
    n = ctypes.c_int64(0)
    plain = solb200.workspace_bytes(1, 32760, 40, 128, 128, False)
    from solb200._lib import lib
    assert lib().solb200_workspace_bytes_reordered(1, 32760, 40, 128, 128, 0, 0, ctypes.byref(n)) == 0
    assert n.value >= plain + 3 * 32760 * 40 * 128 * 2
    assert lib().solb200_workspace_bytes_reordered(1, 32760, 40, 128, 128, 1, 1, ctypes.byref(n)) == 0
    int8 = solb200.workspace_bytes(1, 32760, 40, 128, 128, True)
    assert int8 + 32760 * 40 * 128 * 2 <= n.value < int8 + 2 * 32760 * 40 * 128 * 2   # q only
