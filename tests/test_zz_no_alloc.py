"""The allocation-free entry point, ``solb200_sol_attn_bf16_noalloc``, called through the C ABI.

It serves callers that cannot allocate device memory when they call attention: hosts
that plan every device allocation up front and forbid allocating afterwards, plugins
whose host owns the allocator, and paths that cannot take cudaMalloc's implicit
device synchronisation. Its scratch is a fixed 16 MiB array inside the library, shared
by every call on a device, so these tests check that two calls in a row (different
shapes, so the second starts from the first call's leftovers) each give the same
result as ``solb200_sol_attn_bf16`` with a caller workspace, within the parity
tolerance of the other GPU tests, with no bounded-wait timeout recorded in the scratch's
device error word (read after every call), and that a call whose scratch would not fit
is refused with a workspace error.

The file sorts last so that it also runs after every other GPU test in one process;
it must pass alone in a fresh process too, where its first call does the per-device
set-up.
"""

import ctypes
from ctypes import c_int64

import numpy as np
import pytest
import torch

import solb200
from solb200._lib import check, last_error, lib
from solb200.workloads import custom_config, make_qkv

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MIN_COS = 0.999
STATIC_SCRATCH_BYTES = 16 << 20
ERR_WORKSPACE = 3


def _strides(t):
    return (c_int64 * 3)(*t.stride()[:3])


def _noalloc(q, k, v, *, tau, block, scale=None, sink_blocks=(0, 0), sink_q=(0, 0)):
    B, T, H, D = q.shape
    out = torch.empty_like(q)
    scale = D ** -0.5 if scale is None else scale
    rc = lib().solb200_sol_attn_bf16_noalloc(
        q.data_ptr(), _strides(q), k.data_ptr(), _strides(k), v.data_ptr(), _strides(v),
        out.data_ptr(), B, T, H, D, block, scale, tau, (c_int64 * 2)(*sink_blocks),
        (c_int64 * 2)(*sink_q), torch.cuda.current_stream().cuda_stream)
    check(rc, "sol_attn_bf16_noalloc")
    _assert_no_device_error()
    return out


def _assert_no_device_error():
    """The call's device error word (in the static scratch) records no bounded-wait
    timeout; reading it synchronises the stream and clears it."""
    code = ctypes.c_int32(-1)
    rc = lib().solb200_noalloc_read_device_error(ctypes.byref(code),
                                                 torch.cuda.current_stream().cuda_stream)
    check(rc, "noalloc_read_device_error")
    assert code.value == 0


def _assert_close(got, want, label):
    torch.cuda.synchronize()
    a = got.float().cpu().numpy().astype(np.float64).ravel()
    b = want.float().cpu().numpy().astype(np.float64).ravel()
    assert np.isfinite(a).all(), f"{label}: non-finite output"
    d = np.abs(a - b).max()
    cos = float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-30))
    assert d <= MAX_ABS and cos >= MIN_COS, f"{label}: max|d|={d:.3e} cos={cos:.6f}"


def _workspace_bytes(B, T, H, D, block):
    n = c_int64(0)
    check(lib().solb200_workspace_bytes(B, T, H, D, block, 0, ctypes.byref(n)), "workspace_bytes")
    return n.value


def test_noalloc_matches_workspace_entry_two_calls(cuda_device):
    # Two calls in a row on different shapes: the second one's scratch layout differs
    # from the first's, so it runs over whatever the first call left in the array.
    cases = [
        dict(shape=(1, 4096, 4, 128), tau=0.9, block=64, sink_blocks=(0, 0), sink_q=(0, 0), seed=11),
        dict(shape=(2, 3000, 3, 64), tau=0.5, block=128, sink_blocks=(1, 2), sink_q=(0, 1), seed=12),
    ]
    inputs = []
    for c in cases:
        B, T, H, D = c["shape"]
        assert _workspace_bytes(B, T, H, D, c["block"]) <= STATIC_SCRATCH_BYTES
        g = torch.Generator(device="cpu").manual_seed(c["seed"])
        q, k, v = (torch.randn(B, T, H, D, generator=g).to(torch.bfloat16).cuda() for _ in range(3))
        inputs.append((q, k, v))
    got = []
    for (q, k, v), c in zip(inputs, cases):
        got.append(_noalloc(q, k, v, tau=c["tau"], block=c["block"], sink_blocks=c["sink_blocks"],
                            sink_q=c["sink_q"]))
    for i, ((q, k, v), c) in enumerate(zip(inputs, cases)):
        want = solb200.sol_attn(q, k, v, tau=c["tau"], block=c["block"], sink_blocks=c["sink_blocks"],
                                sink_q=c["sink_q"])
        _assert_close(got[i], want, f"call {i + 1} {c['shape']}")


def test_noalloc_repeat_same_inputs(cuda_device):
    # The same call twice: the second call starts from the first call's scratch contents.
    cfg = custom_config("noalloc", 1, 2, 128, (2, 32, 32), 64, 0.9, (1.0, 3.0, 3.0), 5)
    q, k, v = make_qkv(cfg, device=cuda_device)
    a = _noalloc(q, k, v, tau=0.9, block=64)
    b = _noalloc(q, k, v, tau=0.9, block=64)
    want = solb200.sol_attn(q, k, v, tau=0.9, block=64)
    _assert_close(a, want, "first call")
    _assert_close(b, want, "second call")


def test_noalloc_rejects_oversize(cuda_device):
    # 40 heads at 64k tokens need more scratch than the static array holds: refused
    # before anything is launched, so small placeholder tensors serve as q/k/v/out.
    B, T, H, D, block = 1, 65536, 40, 128, 64
    assert _workspace_bytes(B, T, H, D, block) > STATIC_SCRATCH_BYTES
    x = torch.zeros(8, dtype=torch.bfloat16, device=cuda_device)
    st = (c_int64 * 3)(T * H * D, H * D, D)
    rc = lib().solb200_sol_attn_bf16_noalloc(
        x.data_ptr(), st, x.data_ptr(), st, x.data_ptr(), st, x.data_ptr(), B, T, H, D, block,
        D ** -0.5, 0.9, (c_int64 * 2)(0, 0), (c_int64 * 2)(0, 0),
        torch.cuda.current_stream().cuda_stream)
    assert rc == ERR_WORKSPACE
    assert "static scratch" in last_error()
    torch.cuda.synchronize()
