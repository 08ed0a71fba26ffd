"""Kernel-level Python API, mirroring the reference's host wrappers.

    sol_attn(q, k, v, *, scale=None, tau=1.0, sink_blocks=(0, 0), sink_q=(0, 0),
             use_tma=False, block=64)                       _tri_fwd.py:354-434
    sol_attn_int8(..., int8_pv=True)                        _int8_fwd.py:379-458
    prepare(q, k, v, *, tau, scale, tokens=None, block=64)  _preprocess.py:268-280
    fused_preprocess(q, k, v, *, tau, scale, tokens=None, int8_pv=True, block=64)
                                                            _fused_prep.py:62-98
    routing(...)                                            the exact-block mask /
                                                            index lists of _tri_fwd.py:279-286

q/k/v are BTHD bf16 CUDA tensors with any strides whose last dim is contiguous; an
input whose other strides are not multiples of 8 elements (16 bytes) is copied to a
packed tensor first, as the reference copies non-contiguous last dims. The result is
a fresh BTHD bf16 tensor with exactly T rows. Everything runs through libsolb200.so
on the current CUDA stream; there is no CPU path.

``block`` is the routing block size: 64 is the reference's (hard-coded) value and the
default; 128 is the block of the benchmark configurations.
"""

from __future__ import annotations

import ctypes
import os
from ctypes import c_int32, c_int64, c_void_p

import torch

from . import _lib
from ._lib import BUF, I64x2, I64x3, STAGES_ALL, STAGES_PREPARE, check, lib

BLOCK = 64
_SYNC_CHECK = os.environ.get("SOLB200_SYNC_CHECK", "0") not in ("0", "", "false")


def _stream_ptr(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ready(t: torch.Tensor, name: str) -> torch.Tensor:
    if not t.is_cuda:
        raise RuntimeError(f"solb200: {name} must be a CUDA tensor")
    if t.dtype != torch.bfloat16:
        raise RuntimeError(f"solb200: {name} must be bfloat16 (got {t.dtype})")
    if t.dim() != 4:
        raise RuntimeError(f"solb200: {name} must be BTHD (4-D), got shape {tuple(t.shape)}")
    s = t.stride()
    aligned = (t.stride(-1) == 1 and t.data_ptr() % 16 == 0
               and all(x % 8 == 0 and x > 0 for x in s[1:3])
               and (t.shape[0] == 1 or (s[0] % 8 == 0 and s[0] > 0)))
    return t if aligned else t.contiguous()


def _strides(t):
    return I64x3(t.stride(0), t.stride(1), t.stride(2))


def workspace_bytes(B, T, H, D, block=BLOCK, int8=False) -> int:
    n = c_int64(0)
    check(lib().solb200_workspace_bytes(B, T, H, D, block, int(int8), ctypes.byref(n)),
          "workspace_bytes")
    return n.value


def _offset(geom, which) -> int:
    n = c_int64(0)
    check(lib().solb200_workspace_offset(*geom, BUF[which], ctypes.byref(n)), "workspace_offset")
    return n.value


def workspace_bytes_reordered(B, T, H, D, block=BLOCK, int8=False, int8_pv=True) -> int:
    n = c_int64(0)
    check(lib().solb200_workspace_bytes_reordered(B, T, H, D, block, int(int8), int(bool(int8_pv)),
                                                  ctypes.byref(n)), "workspace_bytes_reordered")
    return n.value


class Workspace:
    """A workspace allocation plus typed views of its intermediates (``reordered``: sized
    for solb200_sol_attn_reordered, the same offsets plus the reordered copies)."""

    def __init__(self, B, T, H, D, block, int8, device, reordered=False, int8_pv=True):
        self.geom = (B, T, H, D, block, int(int8))
        self.B, self.T, self.H, self.D, self.block = B, T, H, D, block
        self.N = -(-T // block)
        self.npad = -(-self.N // 64) * 64
        self.nw = -(-self.N // 32)
        self.nbytes = (workspace_bytes_reordered(B, T, H, D, block, int8, int8_pv) if reordered
                       else workspace_bytes(B, T, H, D, block, int8))
        self.buf = torch.empty(self.nbytes, dtype=torch.uint8, device=device)

    def ptr(self) -> int:
        return self.buf.data_ptr()

    def view(self, which, dtype, shape):
        off = _offset(self.geom, which)
        count = 1
        for s in shape:
            count *= s
        nbytes = count * torch.empty((), dtype=dtype).element_size()
        return self.buf[off:off + nbytes].view(dtype).view(shape)

    def check_device_error(self):
        code = c_int32(0)
        stream = _stream_ptr(self.buf.device)
        check(lib().solb200_read_device_error(self.ptr(), ctypes.byref(code), stream),
              "device error check")


def _attn_reordered(q, k, v, order, *, scale, tau, sink_blocks, sink_q, block, int8, int8_pv):
    """solb200_sol_attn_reordered: the call on tokens taken in `order`, output in input order."""
    q, k, v = _ready(q, "q"), _ready(k, "k"), _ready(v, "v")
    if q.shape != k.shape or q.shape != v.shape:
        raise RuntimeError(f"solb200: q/k/v shapes differ: {tuple(q.shape)}, {tuple(k.shape)}, "
                           f"{tuple(v.shape)}")
    B, T, H, D = q.shape
    if not torch.is_tensor(order) or order.dtype != torch.int64 or order.dim() != 1 or order.numel() != T:
        raise RuntimeError("solb200: token_order must be an int64 tensor of one index per token")
    if order.device != q.device:
        raise RuntimeError("solb200: token_order must be on the tensors' device")
    order = order.contiguous()
    scale = D ** -0.5 if scale is None else float(scale)
    with torch.cuda.device(q.device):
        ws = Workspace(B, T, H, D, block, int8, q.device, reordered=True, int8_pv=int8_pv)
        out = torch.empty((B, T, H, D), dtype=torch.bfloat16, device=q.device)
        rc = lib().solb200_sol_attn_reordered(
            q.data_ptr(), _strides(q), k.data_ptr(), _strides(k), v.data_ptr(), _strides(v), out.data_ptr(),
            B, T, H, D, block, scale, float(tau), I64x2(int(sink_blocks[0]), int(sink_blocks[1])),
            I64x2(int(sink_q[0]), int(sink_q[1])), order.data_ptr(), int(bool(int8)), int(bool(int8_pv)),
            ws.ptr(), ws.nbytes, _stream_ptr(q.device))
        check(rc, "sol_attn (token order)")
        if _SYNC_CHECK:
            ws.check_device_error()
    return out


def _attn(q, k, v, *, scale, tau, sink_blocks, sink_q, block, int8, int8_pv, stages,
          want_lists=False, want_stat=False):
    q, k, v = _ready(q, "q"), _ready(k, "k"), _ready(v, "v")
    if q.shape != k.shape or q.shape != v.shape:
        raise RuntimeError(f"solb200: q/k/v shapes differ: {tuple(q.shape)}, {tuple(k.shape)}, "
                           f"{tuple(v.shape)}")
    if not (q.device == k.device == v.device):
        raise RuntimeError("solb200: q/k/v on different devices")
    B, T, H, D = q.shape
    scale = D ** -0.5 if scale is None else float(scale)
    with torch.cuda.device(q.device):
        ws = Workspace(B, T, H, D, block, int8, q.device)
        out = torch.empty((B, T, H, D), dtype=torch.bfloat16, device=q.device) \
            if stages == STAGES_ALL else None
        N = ws.N
        lists = torch.empty((B, H, N, N), dtype=torch.int32, device=q.device) if want_lists else None
        stat = torch.empty((B, H, N, N), dtype=torch.float32, device=q.device) if want_stat else None
        sk = I64x2(int(sink_blocks[0]), int(sink_blocks[1]))
        sq = I64x2(int(sink_q[0]), int(sink_q[1]))
        args = [q.data_ptr(), _strides(q), k.data_ptr(), _strides(k), v.data_ptr(), _strides(v),
                out.data_ptr() if out is not None else None, B, T, H, D, block, scale, float(tau),
                sk, sq]
        tail = [stages, ws.ptr(), ws.nbytes, lists.data_ptr() if lists is not None else None,
                stat.data_ptr() if stat is not None else None, _stream_ptr(q.device)]
        if int8:
            rc = lib().solb200_sol_attn_int8(*args, int(bool(int8_pv)), *tail)
        else:
            rc = lib().solb200_sol_attn_bf16(*args, *tail)
        check(rc, "sol_attn_int8" if int8 else "sol_attn")
        if _SYNC_CHECK:
            ws.check_device_error()
    return out, ws, lists, stat


def sol_attn(q, k, v, *, scale=None, tau=1.0, sink_blocks=(0, 0), sink_q=(0, 0), use_tma=False,
             block=BLOCK, token_order=None):
    """BF16 Sol-Attn on BTHD inputs. ``use_tma`` is accepted for signature parity and
    ignored: the sm_100a kernel always stages tiles with TMA. ``token_order`` (this build's
    addition; int64 [T] on the device, e.g. a Morton permutation): attend over the tokens
    in that order and return the output in input order, equal to
    ``sol_attn(q[:, order], ...)[:, inverse]`` without the two gather passes."""
    if token_order is not None:
        return _attn_reordered(q, k, v, token_order, scale=scale, tau=tau, sink_blocks=sink_blocks,
                               sink_q=sink_q, block=block, int8=False, int8_pv=False)
    out, _, _, _ = _attn(q, k, v, scale=scale, tau=tau, sink_blocks=sink_blocks, sink_q=sink_q,
                         block=block, int8=False, int8_pv=False, stages=STAGES_ALL)
    return out


def sol_attn_int8(q, k, v, *, scale=None, tau=1.0, sink_blocks=(0, 0), sink_q=(0, 0),
                  use_tma=False, int8_pv=True, block=BLOCK, token_order=None):
    """Sol-Attn with an INT8 exact branch. Same contract as ``sol_attn``."""
    if token_order is not None:
        return _attn_reordered(q, k, v, token_order, scale=scale, tau=tau, sink_blocks=sink_blocks,
                               sink_q=sink_q, block=block, int8=True, int8_pv=int8_pv)
    out, _, _, _ = _attn(q, k, v, scale=scale, tau=tau, sink_blocks=sink_blocks, sink_q=sink_q,
                         block=block, int8=True, int8_pv=int8_pv, stages=STAGES_ALL)
    return out


# element types of an attention mask, as the C ABI numbers them (SOLB200_MASK_*)
MASK_KINDS = {torch.bool: 1, torch.float32: 2, torch.bfloat16: 3, torch.float16: 4}


def mask_layout(mask, B, H, Tq, Tk):
    """(mask, kind, [4 element strides]) of an attention mask for queries [B, Tq, H, D] and
    keys [B, Tk, H, D], read the way the host's attention reads one: a 2-D mask is
    [Tq, Tk], a 3-D mask [B, Tq, Tk] (every head alike), a 4-D mask [B, H, Tq, Tk]; a
    dimension of size 1 broadcasts (stride 0). bool masks attend where true; float masks
    are added to the scaled scores. Raises ValueError for any other shape or dtype."""
    if mask.dtype not in MASK_KINDS:
        raise ValueError(f"solb200: mask dtype {mask.dtype} is not bool, float32, bfloat16 or float16")
    m = mask
    if m.dim() == 2:
        m = m.unsqueeze(0)
    if m.dim() == 3:
        m = m.unsqueeze(1)
    if m.dim() != 4:
        raise ValueError(f"solb200: mask of shape {tuple(mask.shape)} is not 2-, 3- or 4-D")
    strides = []
    for size, want, st in zip(m.shape, (B, H, Tq, Tk), m.stride()):
        if size == 1:
            strides.append(0)
        elif size == want:
            strides.append(st)
        else:
            raise ValueError(f"solb200: mask of shape {tuple(mask.shape)} does not broadcast to "
                             f"{(B, H, Tq, Tk)}")
    return m, MASK_KINDS[m.dtype], strides


def dense_attn(q, k, v, *, scale=None, mask=None):
    """Dense BF16 attention softmax(q k^T * scale + mask) v on the sm_100a tensor cores (C
    ABI ``solb200_attn_dense`` / ``solb200_attn_dense_masked``): q [B, Tq, H, D], k / v
    [B, Tk, H, D] (BTHD, any strides with a contiguous head dim; Tq may differ from Tk), D
    64 or 128; ``mask`` as ``mask_layout`` reads it (None: no mask); returns a fresh
    [B, Tq, H, D] bf16 tensor. For the calls the Sol-Attn path declines (cross-attention,
    head_dim != 128, short sequences, masks), which the reference hands back to the host's
    attention."""
    q, k, v = _ready(q, "q"), _ready(k, "k"), _ready(v, "v")
    if k.shape != v.shape or q.shape[0] != k.shape[0] or q.shape[2:] != k.shape[2:]:
        raise RuntimeError(f"solb200: dense_attn shapes q {tuple(q.shape)}, k {tuple(k.shape)}, "
                           f"v {tuple(v.shape)}")
    if not (q.device == k.device == v.device):
        raise RuntimeError("solb200: q/k/v on different devices")
    B, Tq, H, D = q.shape
    Tk = k.shape[1]
    scale = D ** -0.5 if scale is None else float(scale)
    if mask is not None:
        if mask.device != q.device:
            raise RuntimeError("solb200: mask on a different device from q")
        m, kind, ms = mask_layout(mask, B, H, Tq, Tk)
    with torch.cuda.device(q.device):
        ws = torch.empty(256, dtype=torch.uint8, device=q.device)
        out = torch.empty((B, Tq, H, D), dtype=torch.bfloat16, device=q.device)
        if mask is None:
            rc = lib().solb200_attn_dense(q.data_ptr(), _strides(q), k.data_ptr(), _strides(k), v.data_ptr(),
                                          _strides(v), out.data_ptr(), B, Tq, Tk, H, D, scale, ws.data_ptr(), 256,
                                          _stream_ptr(q.device))
        else:
            rc = lib().solb200_attn_dense_masked(q.data_ptr(), _strides(q), k.data_ptr(), _strides(k),
                                                 v.data_ptr(), _strides(v), m.data_ptr(), kind,
                                                 (c_int64 * 4)(*ms), out.data_ptr(), B, Tq, Tk, H, D, scale,
                                                 ws.data_ptr(), 256, _stream_ptr(q.device))
        check(rc, "dense_attn")
        if _SYNC_CHECK:
            code = c_int32(0)
            check(lib().solb200_read_device_error(ws.data_ptr(), ctypes.byref(code), _stream_ptr(q.device)),
                  "device error check")
    return out


def _tokens_check(q, tokens):
    if tokens is not None and int(tokens) != q.shape[1]:
        raise RuntimeError("solb200: tokens must equal q.shape[1] (inputs are never padded here)")


def prepare(q, k, v, *, tau, scale, tokens=None, block=BLOCK):
    """(kc, vc, threshold): kc/vc bf16 [B, Npad, H, D], threshold fp32 [B, N, H]."""
    _tokens_check(q, tokens)
    _, ws, _, _ = _attn(q, k, v, scale=scale, tau=tau, sink_blocks=(0, 0), sink_q=(0, 0),
                        block=block, int8=False, int8_pv=False, stages=STAGES_PREPARE)
    B, H, D, N, npad = ws.B, ws.H, ws.D, ws.N, ws.npad
    kc = ws.view("kc", torch.bfloat16, (B, npad, H, D)).clone()
    vc = ws.view("vc", torch.bfloat16, (B, npad, H, D)).clone()
    thr = ws.view("thr", torch.float32, (B, N, H)).clone()
    return kc, vc, thr


def fused_preprocess(q, k, v, *, tau, scale, tokens=None, int8_pv=True, block=BLOCK):
    """(kc, vc, threshold, qi, qs, ki, ks, vi, vsc) in the reference's shapes: kc
    centred; qi/ki/vi int8 [B, T, H, D]; qs/ks fp32 [B, T, H]; vsc fp32 [B*H, D]
    (vi / vsc are None without int8_pv)."""
    _tokens_check(q, tokens)
    _, ws, _, _ = _attn(q, k, v, scale=scale, tau=tau, sink_blocks=(0, 0), sink_q=(0, 0),
                        block=block, int8=True, int8_pv=int8_pv, stages=STAGES_PREPARE)
    B, T, H, D, N, npad = ws.B, ws.T, ws.H, ws.D, ws.N, ws.npad
    tp = N * block
    kc = ws.view("kc", torch.bfloat16, (B, npad, H, D)).clone()
    vc = ws.view("vc", torch.bfloat16, (B, npad, H, D)).clone()
    thr = ws.view("thr", torch.float32, (B, N, H)).clone()
    qi = ws.view("qi", torch.int8, (B, T, H, D)).clone()
    ki = ws.view("ki", torch.int8, (B, T, H, D)).clone()
    qs = ws.view("qs", torch.float32, (B, H, tp))[:, :, :T].transpose(1, 2).contiguous()
    ks = ws.view("ks", torch.float32, (B, H, tp))[:, :, :T].transpose(1, 2).contiguous()
    if int8_pv:
        vi = ws.view("vi", torch.int8, (B, T, H, D)).clone()
        vsc = ws.view("vscale", torch.float32, (B * H, D)).clone()
    else:
        vi = vsc = None
    return kc, vc, thr, qi, qs, ki, ks, vi, vsc


def routing(q, k, v, *, tau=1.0, scale=None, sink_blocks=(0, 0), sink_q=(0, 0), block=BLOCK,
            int8=False, int8_pv=True):
    """The exact-block routing of one call: dict with ``mask`` bool [B, H, N, N],
    ``lists`` int32 [B, H, N, N] (ascending, -1 padded), ``counts`` int32 [B, H, N],
    ``stat`` fp32 [B, H, N, N] (the routing score of each block) and ``thr`` [B, N, H]."""
    _, ws, lists, stat = _attn(q, k, v, scale=scale, tau=tau, sink_blocks=sink_blocks,
                               sink_q=sink_q, block=block, int8=int8, int8_pv=int8_pv,
                               stages=STAGES_PREPARE, want_lists=True, want_stat=True)
    B, H, N, nw = ws.B, ws.H, ws.N, ws.nw
    words = ws.view("mask", torch.int32, (B, H, N, nw))
    bits = torch.arange(32, device=words.device, dtype=torch.int32)
    mask = ((words.unsqueeze(-1) >> bits) & 1).bool().reshape(B, H, N, nw * 32)[..., :N]
    return dict(mask=mask, lists=lists, counts=ws.view("count", torch.int32, (B, H, N)).clone(),
                stat=stat, thr=ws.view("thr", torch.float32, (B, ws.N, H)).clone())
