"""Morton (Z-order) token reordering on the device.

    morton_perm(grid, device, curve="3d") -> (perm, inverse)     _morton.py:35-73
    perm_for_span(grid, curve, device, start, block=64)          _morton_h3.py:42-61
    permute_tokens(x, index) / permute_tokens_many(xs, index)    x.index_select(1, index)
                                                                 of the model hooks

The permutation is computed by a kernel that ranks every token's Morton code
directly (no sort) and is bit-identical to the reference's argsort. Results are
cached per (grid, curve, roll, device), like the reference's perm cache.
"""

from __future__ import annotations

from ctypes import c_void_p

import torch

from ._lib import check, lib
from .ops import _stream_ptr

_CACHE = {}
CURVES = {"3d": 0, "2d_frame": 1}


def _compute(grid, curve, roll, device):
    frames, height, width = (int(g) for g in grid)
    T = frames * height * width
    perm = torch.empty(T, dtype=torch.int64, device=device)
    inverse = torch.empty(T, dtype=torch.int64, device=device)
    with torch.cuda.device(device):
        check(lib().solb200_morton_perm(frames, height, width, CURVES[curve], int(roll),
                                        perm.data_ptr(), inverse.data_ptr(), _stream_ptr(device)),
              "morton_perm")
    return perm, inverse


def _get(grid, curve, roll, device):
    if curve not in CURVES:
        raise ValueError(f"unknown Morton curve {curve!r}; use '3d' or '2d_frame'")
    device = torch.device(device)
    cuda_dev = device if device.type == "cuda" else torch.device("cuda", torch.cuda.current_device())
    key = (tuple(int(g) for g in grid), curve, int(roll), str(cuda_dev))
    hit = _CACHE.get(key)
    if hit is None:
        hit = _compute(grid, curve, roll, cuda_dev)
        _CACHE[key] = hit
    if device.type != "cuda":
        return hit[0].to(device), hit[1].to(device)
    return hit


def morton_perm(grid, device, curve="3d"):
    """Z-order permutation of a (frames, height, width) grid and its inverse, int64."""
    return _get(grid, curve, 0, device)


def perm_for_span(grid, curve, device, start, block=64):
    """Permutation for a video span starting at absolute row ``start``, rotated by
    (-start) % block so that Z-order cells stay aligned to the kernel's blocks."""
    pad = (-int(start)) % int(block)
    return _get(grid, curve, pad, device)


def _rows_geometry(x: torch.Tensor):
    if x.dim() < 2:
        raise RuntimeError("solb200: permute_tokens needs [B, T, ...]")
    inner = x[0, 0]
    if not inner.is_contiguous():
        raise RuntimeError("solb200: per-token rows must be contiguous")
    row_bytes = inner.numel() * x.element_size()
    return row_bytes, x.stride(0) * x.element_size(), x.stride(1) * x.element_size()


def permute_tokens_many(xs, index: torch.Tensor):
    """[x[:, index] for x in xs] for up to 4 same-shaped [B, T, ...] CUDA tensors, in one
    launch (one warp per destination row, 16-byte vectors)."""
    xs = [x if x.data_ptr() % 16 == 0 and _rows_geometry(x)[0] % 16 == 0 else x.contiguous()
          for x in xs]
    if not 1 <= len(xs) <= 4:
        raise RuntimeError("solb200: 1..4 tensors per permute call")
    x0 = xs[0]
    for x in xs:
        if x.shape != x0.shape or x.dtype != x0.dtype or x.stride() != x0.stride():
            raise RuntimeError("solb200: tensors permuted together must share shape and strides")
    if index.device != x0.device or index.dtype != torch.int64 or index.numel() != x0.shape[1]:
        raise RuntimeError("solb200: index must be int64 on the tensors' device, one per token")
    index = index.contiguous()
    row_bytes, sb, sr = _rows_geometry(x0)
    outs = [torch.empty_like(x0, memory_format=torch.contiguous_format) for _ in xs]
    o_row_bytes, ob, orow = _rows_geometry(outs[0])
    src = (c_void_p * 4)(*[x.data_ptr() for x in xs], *([None] * (4 - len(xs))))
    dst = (c_void_p * 4)(*[o.data_ptr() for o in outs], *([None] * (4 - len(xs))))
    with torch.cuda.device(x0.device):
        check(lib().solb200_gather_rows(src, dst, len(xs), index.data_ptr(), x0.shape[0],
                                        x0.shape[1], row_bytes, sb, sr, ob, orow,
                                        _stream_ptr(x0.device)), "gather_rows")
    return outs


def permute_tokens(x, index):
    return permute_tokens_many([x], index)[0]
