"""CPU oracle for the Sol-Attn hot path: TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
(``cpu_baseline`` / ``--impl reference``) may import this module, and only as the
checker or as the timed CPU arm. The product path (``solb200``) never imports it:
it runs the sm_100a kernels or raises.

What it is: a numpy restatement of the reference's Triton kernels and torch glue
(kijai/ComfyUI-SolAttn_triton), step for step, with the reference's arithmetic:

* bf16 values are carried as float32 arrays holding bf16-representable numbers;
  every fp32->bf16 cast rounds to nearest even (``bf16``), which is what the
  reference's ``.to(tl.bfloat16)`` / bf16 stores compile to on a GPU.
* ``tl.dot`` of bf16 operands is an fp32 ``np.matmul`` of the exact bf16 values;
  ``tl.sum`` of bf16 accumulates in fp32 and rounds once to bf16.
* fp32 reductions use the same numpy calls the Triton interpreter uses
  (``np.sum`` along the same axis of the same tile shape), so that an interpreter
  run of the reference (``tests/golden/make_golden.py``) and this module agree
  bit for bit on the committed fixtures.
* torch glue of the reference (kc moments, k centring, V scales) is restated with
  the same torch calls.

Pinning: ``tests/test_oracle.py`` checks every function here against fixtures made
by running the reference's own kernels on CPU (``tests/golden/*.npz``).
"""

from __future__ import annotations

import numpy as np
import torch

LOG2E = 1.4426950408889634
F32 = np.float32


# --------------------------------------------------------------------------- bf16

def bf16(x) -> np.ndarray:
    """Round float32 values to the nearest bf16 (ties to even); returns float32."""
    a = np.ascontiguousarray(np.asarray(x, dtype=F32))
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    nan = np.isnan(a)
    out = r.astype(np.uint32).view(F32).reshape(a.shape)
    if nan.any():
        out = out.copy()
        out[nan] = np.nan
    return out


def to_np(t: torch.Tensor) -> np.ndarray:
    """torch tensor (bf16/fp32/int) -> numpy (bf16 becomes exact float32)."""
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        t = t.float()
    return t.numpy()


# ------------------------------------------------------------------------- Morton

def _part1by2(value: np.ndarray) -> np.ndarray:
    """21-bit spread, bit i -> bit 3i (_morton.py:56-63)."""
    value = value & 0x1FFFFF
    value = (value | (value << 32)) & 0x1F00000000FFFF
    value = (value | (value << 16)) & 0x1F0000FF0000FF
    value = (value | (value << 8)) & 0x100F00F00F00F00F
    value = (value | (value << 4)) & 0x10C30C30C30C30C3
    value = (value | (value << 2)) & 0x1249249249249249
    return value


def morton_perm(grid, curve: str = "3d"):
    """(perm, inverse) int64 as in ``morton_perm`` (_morton.py:35-73).

    code = p(x) | p(y)<<1 | p(z)<<2 for "3d", (z<<42) | p(x) | p(y)<<1 for
    "2d_frame", with (z, y, x) = (frame, row, column) of the row-major token index;
    perm = argsort(code), inverse = argsort(perm).
    """
    frames, height, width = (int(g) for g in grid)
    linear = np.arange(frames * height * width, dtype=np.int64)
    area = height * width
    z = linear // area
    rem = linear - z * area
    y = rem // width
    x = rem - y * width
    if curve == "2d_frame":
        code = (z << 42) | _part1by2(x) | (_part1by2(y) << 1)
    else:
        code = _part1by2(x) | (_part1by2(y) << 1) | (_part1by2(z) << 2)
    perm = linear[np.argsort(code, kind="stable")]
    inverse = np.argsort(perm, kind="stable")
    return perm, inverse


def morton_perm_for_span(grid, curve: str, start: int, block: int = 64):
    """Block-aligned perm of a video span starting at absolute row ``start``
    (_morton_h3.py:42-61): roll by (-start) % block, inverse recomputed."""
    perm, inverse = morton_perm(grid, curve)
    pad = (-int(start)) % block
    if pad:
        perm = np.roll(perm, pad)
        inverse = np.argsort(perm, kind="stable")
    return perm, inverse


# ------------------------------------------------------------------ pooling (a3/a4)

def pool_kv(k: np.ndarray, v: np.ndarray, tokens: int, block: int,
            group_pad: int = 64, v_absmax: bool = False,
            reference_batch_stride: bool = False):
    """kc = bf16(bf16(sum K) / len), vc = bf16(sum V), optional per-block |V| max.

    _reduce_kc_kernel (_preprocess.py:23-62), _reduce_vc_kernel (:65-113) and
    _reduce_kv (:172-224). Layout [B, Npad, H, D] with Npad a multiple of
    ``group_pad`` and zero padding. Rows are summed in order (row 0 first), in fp32.

    ``reference_batch_stride`` reproduces the reference's write index for B > 1:
    its pooling kernels address kc/vc as ((batch * N + block) * H + head) * D with
    the UNPADDED block count N (_preprocess.py:59,102; N = blocks at :192-203) while
    the buffers are [B, Npad, H, D] and every reader uses Npad (_preprocess.py:241,
    _tri_fwd.py:272-277), so batch b >= 1 lands in rows b*N.. of the flat buffer.
    Off (the default) pools every batch into its own rows, which is what the
    readers expect; for B = 1 the two are identical.
    """
    B, _, H, D = k.shape
    T = int(tokens)
    N = -(-T // block)
    npad = -(-N // group_pad) * group_pad
    kc = np.zeros((B, npad, H, D), F32)
    vc = np.zeros((B, npad, H, D), F32)
    vamax = np.zeros((B, N, H, D), F32) if v_absmax else None
    for n in range(N):
        r0, r1 = n * block, min(T, (n + 1) * block)
        ks = np.zeros((B, H, D), F32)
        vs = np.zeros((B, H, D), F32)
        for r in range(r0, r1):
            ks = ks + k[:, r]
            vs = vs + v[:, r]
        length = F32(r1 - r0)
        kc[:, n] = bf16(bf16(ks) / length)
        vc[:, n] = bf16(vs)
        if v_absmax:
            vamax[:, n] = np.abs(v[:, r0:r1]).max(axis=1)
    if reference_batch_stride and B > 1:
        flat_k = np.zeros((B * npad, H, D), F32)
        flat_v = np.zeros((B * npad, H, D), F32)
        for b in range(B):
            flat_k[b * N:b * N + N] = kc[b, :N]
            flat_v[b * N:b * N + N] = vc[b, :N]
        kc, vc = flat_k.reshape(kc.shape), flat_v.reshape(vc.shape)
    return (kc, vc, vamax) if v_absmax else (kc, vc)


# --------------------------------------------------------------- threshold (a5)

def kc_moments(kc: np.ndarray, blocks: int):
    """Per-(b,h) mean and diagonal variance of kc over valid blocks, fp32 [B,H,D]
    (_preprocess.py:240-243, the same torch calls)."""
    kcb = torch.from_numpy(np.ascontiguousarray(kc, F32)).to(torch.bfloat16)
    kv = kcb[:, :blocks].float().permute(0, 2, 1, 3)
    kc_mean = kv.mean(dim=2).contiguous()
    kc_var = (kv - kc_mean.unsqueeze(2)).pow(2).mean(dim=2).contiguous()
    return kc_mean.numpy(), kc_var.numpy()


def q_centroids(q: np.ndarray, tokens: int, block: int) -> np.ndarray:
    """fp32 sum of each q block's rows (in order) / q_len -> [B, N, H, D]
    (_preprocess.py:149, _fused_prep.py:51)."""
    B, _, H, D = q.shape
    T = int(tokens)
    N = -(-T // block)
    out = np.zeros((B, N, H, D), F32)
    for n in range(N):
        r0, r1 = n * block, min(T, (n + 1) * block)
        acc = np.zeros((B, H, D), F32)
        for r in range(r0, r1):
            acc = acc + q[:, r]
        out[:, n] = acc / F32(r1 - r0)
    return out


def _log2_scale(scale: float):
    return F32(scale) * F32(LOG2E)


def diag_threshold(q, kc_mean, kc_var, tau, scale, tokens, block):
    """thr[b,n,h] = (c.mean_kc)*s2 + tau*sqrt(max((c^2.var)*s2^2, 0) + 1e-6)
    (_diag_threshold_kernel, _preprocess.py:116-164). tau scalar or per head."""
    c = q_centroids(q, tokens, block)                            # [B,N,H,D]
    s2 = _log2_scale(scale)
    H = q.shape[2]
    taus = np.broadcast_to(np.asarray(tau, F32), (H,)).astype(F32)
    mean = np.sum(c * kc_mean[:, None], axis=-1) * s2            # [B,N,H]
    variance = np.sum(c * c * kc_var[:, None], axis=-1) * (s2 * s2)
    std = np.sqrt(np.maximum(variance, F32(0.0)) + F32(1.0e-6))
    return (mean + taus[None, None, :] * std).astype(F32)


def prepare(q, k, v, tau, scale, tokens, block, group_pad=64, reference_batch_stride=False):
    """(kc, vc, thr) as in ``prepare`` (_preprocess.py:268-280)."""
    N = -(-int(tokens) // block)
    kc, vc = pool_kv(k, v, tokens, block, group_pad,
                     reference_batch_stride=reference_batch_stride)
    kcm, kcv = kc_moments(kc, N)
    thr = diag_threshold(q, kcm, kcv, tau, scale, tokens, block)
    return kc, vc, thr


# --------------------------------------------------------------- routing (a6)

def route_unit(q_tile, kc_bh, thr_val, q_block, q_len, N, s2, sink_blocks, sink_q,
               group=64):
    """Exact-block mask for one (b, h, q-block) and the routing statistic.

    Inline routing of _forward_ptr (_tri_fwd.py:279-286): scores = q . kc^T * s2 per
    row (fp32 matmul of bf16 values), column mean over the q_len rows, compared with
    the threshold; neighbours |qb - j| <= 1 and sink KV blocks are always exact; a
    query block inside sink_q attends every valid block exactly.
    Returns (exact [N] bool, stat [N] fp32) with stat = colsum / q_len.
    """
    exact = np.zeros(N, bool)
    stat = np.zeros(N, F32)
    q_in_sink = sink_q[0] <= q_block < sink_q[1]
    for g0 in range(0, N, group):
        idx = g0 + np.arange(group)
        valid = idx < N
        kc_g = kc_bh[g0:g0 + group]
        scores = _dot(q_tile, kc_g.T) * s2
        colmean = np.sum(scores, axis=0) / F32(q_len)
        routed = ((colmean > thr_val) | (np.abs(q_block - idx) <= 1)
                  | ((idx >= sink_blocks[0]) & (idx < sink_blocks[1]))) & valid
        ex = valid if q_in_sink else routed
        exact[idx[valid]] = ex[valid]
        stat[idx[valid]] = colmean[valid]
    return exact, stat


def route_mask(q, kc, thr, scale, tokens, block, sink_blocks=(0, 0), sink_q=(0, 0),
               group=64):
    """mask [B,H,N,N] bool and stat [B,H,N,N] (colsum/q_len) for every unit."""
    B, _, H, D = q.shape
    T = int(tokens)
    N = -(-T // block)
    s2 = _log2_scale(scale)
    mask = np.zeros((B, H, N, N), bool)
    stat = np.zeros((B, H, N, N), F32)
    kcp = _pad_rows(kc, group)
    for b in range(B):
        for h in range(H):
            for qb in range(N):
                q_tile = _tile(q[b, :, h], qb * block, block)
                q_len = min(block, T - qb * block)
                ex, st = route_unit(q_tile, kcp[b, :, h], thr[b, qb, h], qb, q_len, N,
                                    s2, sink_blocks, sink_q, group)
                mask[b, h, qb] = ex
                stat[b, h, qb] = st
    return mask, stat


def _dot(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """fp32 matmul of two tiles, each first made C-contiguous as the interpreter's
    converted operands are (it materialises transposes before ``np.matmul``)."""
    return np.matmul(np.ascontiguousarray(a, F32), np.ascontiguousarray(b, F32), dtype=F32)


def _tile(x2d: np.ndarray, start: int, rows: int) -> np.ndarray:
    """rows [start, start+rows) of a [T, D] array; rows past T read 0.0."""
    out = np.zeros((rows,) + x2d.shape[1:], x2d.dtype)
    stop = min(x2d.shape[0], start + rows)
    if stop > start:
        out[: stop - start] = x2d[start:stop]
    return out


def _pad_rows(kc: np.ndarray, group: int) -> np.ndarray:
    """Pad the block axis of [B, Npad, H, D] to a multiple of ``group`` with zeros."""
    npad = kc.shape[1]
    need = -(-npad // group) * group
    if need == npad:
        return kc
    out = np.zeros((kc.shape[0], need) + kc.shape[2:], kc.dtype)
    out[:, :npad] = kc
    return out


# ------------------------------------------------------------ BF16 forward (a7/a8)

def _fwd_unit_bf16(q_tile, k_bh, v_bh, kc_bh, vc_bh, thr_val, q_block, T, N, block,
                   s2, sink_blocks, sink_q, group):
    """One (b, h, q-block) of _forward_ptr (_tri_fwd.py:238-347), BV = D."""
    q_len = F32(min(block, T - q_block * block))
    D = q_tile.shape[1]
    out = np.zeros((block, D), F32)
    row_sum = np.zeros(block, F32)
    row_max = np.full(block, -np.inf, F32)
    tail = F32(T - (N - 1) * block)
    q_in_sink = sink_q[0] <= q_block < sink_q[1]
    tok = np.arange(block)
    for g0 in range(0, N, group):
        idx = g0 + np.arange(group)
        valid = idx < N
        kc = kc_bh[g0:g0 + group]
        vc = vc_bh[g0:g0 + group]
        scores = _dot(q_tile, kc.T) * s2
        routed = ((np.sum(scores, axis=0) / q_len > thr_val)
                  | (np.abs(q_block - idx) <= 1)
                  | ((idx >= sink_blocks[0]) & (idx < sink_blocks[1]))) & valid
        exact = valid if q_in_sink else routed
        approx = valid & ~exact
        a_scores = np.where(approx[None, :], scores, F32(-np.inf))
        new_max = np.maximum(row_max, np.max(a_scores, axis=1))
        alpha = np.exp2(np.where(row_max == new_max, F32(0.0), row_max - new_max))
        a_prob = np.where(approx[None, :], np.exp2(a_scores - new_max[:, None]), F32(0.0))
        out = out * alpha[:, None] + _dot(bf16(a_prob), vc)
        lengths = np.where(idx == N - 1, tail, F32(block)).astype(F32)
        row_sum = row_sum * alpha + np.sum(a_prob * lengths[None, :], axis=1)
        row_max = new_max
        for off in np.nonzero(exact)[0]:
            kv0 = (g0 + int(off)) * block
            kv_ok = kv0 + tok < T
            k = _tile(k_bh, kv0, block)
            e_scores = _dot(q_tile, k.T) * s2
            e_scores = e_scores + np.where(kv_ok[None, :], F32(0.0), F32(-np.inf))
            new_max = np.maximum(row_max, np.max(e_scores, axis=1))
            alpha = np.exp2(row_max - new_max)
            p = np.exp2(e_scores - new_max[:, None])
            row_sum = row_sum * alpha + np.sum(p, axis=1)
            v = _tile(v_bh, kv0, block)
            out = out * alpha[:, None] + _dot(bf16(p), v)
            row_max = new_max
    return bf16(out / row_sum[:, None])


def sol_attn(q, k, v, scale=None, tau=1.0, sink_blocks=(0, 0), sink_q=(0, 0),
             block=64, group=64, units=None, return_parts=False,
             reference_batch_stride=False):
    """BF16 Sol-Attn: ``sol_attn`` (_tri_fwd.py:354-434) with _forward_ptr, BV = D.

    q/k/v: float32 arrays [B, T, H, D] of bf16 values. ``units`` optionally limits
    the computation to an iterable of (b, h, q_block) (rows of other units stay 0);
    used for bounded CPU timing samples.
    """
    B, T, H, D = q.shape
    scale = D ** -0.5 if scale is None else float(scale)
    N = -(-T // block)
    kc, vc, thr = prepare(q, k, v, tau, scale, T, block,
                          reference_batch_stride=reference_batch_stride)
    kcp, vcp = _pad_rows(kc, group), _pad_rows(vc, group)
    s2 = _log2_scale(scale)
    out = np.zeros((B, T, H, D), F32)
    todo = units if units is not None else (
        (b, h, n) for b in range(B) for h in range(H) for n in range(N))
    with np.errstate(invalid="ignore", over="ignore"):
        for b, h, n in todo:
            q_tile = _tile(q[b, :, h], n * block, block)
            o = _fwd_unit_bf16(q_tile, k[b, :, h], v[b, :, h], kcp[b, :, h],
                               vcp[b, :, h], thr[b, n, h], n, T, N, block, s2,
                               sink_blocks, sink_q, group)
            r1 = min(T, (n + 1) * block)
            out[b, n * block:r1, h] = o[: r1 - n * block]
    if return_parts:
        return out, dict(kc=kc, vc=vc, thr=thr)
    return out


# ------------------------------------------------------------------ INT8 (a9-a13)

def _round_half_away(val: np.ndarray) -> np.ndarray:
    """where(val >= 0, trunc(val + 0.5), trunc(val - 0.5)) in fp32."""
    return np.where(val >= 0, np.trunc(val + F32(0.5)), np.trunc(val - F32(0.5))).astype(F32)


def quantize_bthd(x: np.ndarray, mean: np.ndarray | None = None):
    """Per-(token, head) symmetric int8 (_quant_kernel, _fused_quant.py:8-42).

    x [B,T,H,D] fp32 (bf16 values); mean [B,H,D] or None. Returns (xi int8, xs fp32
    [B,T,H]).
    """
    x = x.astype(F32)
    if mean is not None:
        x = x - mean[:, None, :, :].astype(F32)
    s = np.max(np.abs(x), axis=-1) / F32(127.0)
    s_safe = np.where(s > F32(1e-8), s, F32(1e-8)).astype(F32)
    val = x / s_safe[..., None]
    xi = np.minimum(np.maximum(_round_half_away(val), F32(-127.0)), F32(127.0))
    return xi.astype(np.int8), s_safe


def quantize_q(x: np.ndarray):
    """Q quant of _q_quant_threshold_kernel (_fused_prep.py:36-44): clamp first, then
    round half away from zero by truncation."""
    x = x.astype(F32)
    s = np.max(np.abs(x), axis=-1) / F32(127.0)
    s_safe = np.where(s > F32(1e-8), s, F32(1e-8)).astype(F32)
    xi = np.minimum(np.maximum(x / s_safe[..., None], F32(-127.0)), F32(127.0))
    xi = np.where(xi >= 0, xi + F32(0.5), xi - F32(0.5))
    return np.trunc(xi).astype(np.int8), s_safe


def v_scale(v_absmax: np.ndarray) -> np.ndarray:
    """clamp_min(absmax / 127, 1e-8) [B,H,D] (_fused_quant.py:103), torch calls."""
    return torch.from_numpy(v_absmax).float().div(127.0).clamp_min_(1e-8).numpy()


def quantize_v_per_channel(v: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """vi = clamp(round_half_away(v / scale[b,h,d]), +-127) (_quant_v_kernel,
    _fused_quant.py:61-88)."""
    val = v.astype(F32) / scale[:, None, :, :]
    xi = np.minimum(np.maximum(_round_half_away(val), F32(-127.0)), F32(127.0))
    return xi.astype(np.int8)


def fused_preprocess(q, k, v, tau, scale, tokens, block, int8_pv=True, group_pad=64,
                     reference_batch_stride=False):
    """The INT8 preprocess (_fused_prep.py:62-98): pooled K/V, k_mean from the pooled
    keys, kc centred in place (re-rounded to bf16), kc variance, K quant with the mean
    removed, per-channel V quant, Q quant and the tau*sigma threshold."""
    B, _, H, D = q.shape
    T = int(tokens)
    N = -(-T // block)
    kc, vc, vamax = pool_kv(k, v, T, block, group_pad, v_absmax=True,
                            reference_batch_stride=reference_batch_stride)
    v_absmax = torch.from_numpy(vamax).amax(dim=1).numpy()               # [B,H,D]
    kct = torch.from_numpy(kc).to(torch.bfloat16)
    k_mean = kct[:, :N].mean(dim=1, dtype=torch.float32)                  # [B,H,D]
    kct[:, :N] = (kct[:, :N].float() - k_mean.unsqueeze(1)).to(kct.dtype)
    centred = kct[:, :N].float().permute(0, 2, 1, 3)
    kc_var = centred.pow(2).mean(dim=2).contiguous().numpy()
    kc = kct.float().numpy()
    k_mean = k_mean.numpy()
    ki, ks = quantize_bthd(k[:, :T], mean=k_mean)
    if int8_pv:
        vsc = v_scale(v_absmax)
        vi = quantize_v_per_channel(v[:, :T], vsc)
    else:
        vsc = vi = None
    qi, qs = quantize_q(q[:, :T])
    c = q_centroids(q, T, block)
    s2 = _log2_scale(scale)
    taus = np.broadcast_to(np.asarray(tau, F32), (H,)).astype(F32)
    variance = np.sum(c * c * kc_var[:, None], axis=-1) * (s2 * s2)
    thr = (taus[None, None, :] * np.sqrt(variance + F32(1.0e-6))).astype(F32)
    return dict(kc=kc, vc=vc, thr=thr, qi=qi, qs=qs, ki=ki, ks=ks, vi=vi, vsc=vsc,
                k_mean=k_mean, kc_var=kc_var, v_absmax=v_absmax)


def _fwd_unit_int8(q_tile, qi_t, qs_t, ki_bh, ks_bh, vi_bh, v_bh, vsc_bh, kc_bh, vc_bh,
                   thr_val, q_block, T, N, block, s2, sink_blocks, sink_q, group, int8_pv):
    """One (b, h, q-block) of _forward_int8_ptr (_int8_fwd.py:232-372), BV = D."""
    q_len = F32(min(block, T - q_block * block))
    D = q_tile.shape[1]
    out = np.zeros((block, D), F32)
    row_sum = np.zeros(block, F32)
    row_max = np.full(block, -np.inf, F32)
    qs_log2 = qs_t * s2
    tail = F32(T - (N - 1) * block)
    q_in_sink = sink_q[0] <= q_block < sink_q[1]
    tok = np.arange(block)
    inv127 = F32(1.0 / 127.0)
    for g0 in range(0, N, group):
        idx = g0 + np.arange(group)
        valid = idx < N
        kc = kc_bh[g0:g0 + group]
        vc = vc_bh[g0:g0 + group]
        scores = _dot(q_tile, kc.T) * s2
        routed = ((np.sum(scores, axis=0) / q_len > thr_val)
                  | (np.abs(q_block - idx) <= 1)
                  | ((idx >= sink_blocks[0]) & (idx < sink_blocks[1]))) & valid
        exact = valid if q_in_sink else routed
        approx = valid & ~exact
        a_scores = np.where(approx[None, :], scores, F32(-np.inf))
        new_max = np.maximum(row_max, np.max(a_scores, axis=1))
        alpha = np.exp2(np.where(row_max == new_max, F32(0.0), row_max - new_max))
        a_prob = np.where(approx[None, :], np.exp2(a_scores - new_max[:, None]), F32(0.0))
        out = out * alpha[:, None] + _dot(bf16(a_prob), vc)
        lengths = np.where(idx == N - 1, tail, F32(block)).astype(F32)
        row_sum = row_sum * alpha + np.sum(a_prob * lengths[None, :], axis=1)
        row_max = new_max
        for off in np.nonzero(exact)[0]:
            kv0 = (g0 + int(off)) * block
            k_valid = kv0 + tok < T
            ki = _tile(ki_bh, kv0, block)
            ks = _tile(ks_bh, kv0, block)
            acc = np.matmul(qi_t.astype(np.int32), ki.T.astype(np.int32))
            e_scores = acc.astype(F32) * (qs_log2[:, None] * ks[None, :])
            e_scores = e_scores + np.where(k_valid[None, :], F32(0.0), F32(-np.inf))
            block_max = np.max(e_scores, axis=1)
            new_max = np.maximum(row_max, block_max)
            alpha = np.exp2(row_max - new_max)
            if int8_pv:
                vi = _tile(vi_bh, kv0, block)
                pe = np.exp2(e_scores - block_max[:, None])
                beta = np.exp2(block_max - new_max)
                row_sum = row_sum * alpha + beta * np.sum(pe, axis=1)
                pi = np.trunc(np.minimum(pe * F32(127.0) + F32(0.5), F32(127.0))).astype(np.int32)
                pv = np.matmul(pi, vi.astype(np.int32)).astype(F32) * (
                    (beta * inv127)[:, None] * vsc_bh[None, :])
            else:
                vb = _tile(v_bh, kv0, block)
                p = np.exp2(e_scores - new_max[:, None])
                row_sum = row_sum * alpha + np.sum(p, axis=1)
                pv = _dot(bf16(p), vb)
            out = out * alpha[:, None] + pv
            row_max = new_max
    return bf16(out / row_sum[:, None])


def sol_attn_int8(q, k, v, scale=None, tau=1.0, sink_blocks=(0, 0), sink_q=(0, 0),
                  int8_pv=True, block=64, group=64, units=None, return_parts=False,
                  reference_batch_stride=False):
    """INT8 Sol-Attn: ``sol_attn_int8`` (_int8_fwd.py:379-458) with
    _forward_int8_ptr, BV = D."""
    B, T, H, D = q.shape
    scale = D ** -0.5 if scale is None else float(scale)
    N = -(-T // block)
    parts = fused_preprocess(q, k, v, tau, scale, T, block, int8_pv,
                             reference_batch_stride=reference_batch_stride)
    kcp, vcp = _pad_rows(parts["kc"], group), _pad_rows(parts["vc"], group)
    s2 = _log2_scale(scale)
    out = np.zeros((B, T, H, D), F32)
    todo = units if units is not None else (
        (b, h, n) for b in range(B) for h in range(H) for n in range(N))
    qi, qs, ki, ks, vi, vsc = (parts[x] for x in ("qi", "qs", "ki", "ks", "vi", "vsc"))
    with np.errstate(invalid="ignore", over="ignore"):
        for b, h, n in todo:
            r0, r1 = n * block, min(T, (n + 1) * block)
            q_tile = _tile(q[b, :, h], r0, block)
            qi_t = _tile(qi[b, :, h], r0, block)
            qs_t = _tile(qs[b, :, h], r0, block)
            o = _fwd_unit_int8(q_tile, qi_t, qs_t, ki[b, :, h], ks[b, :, h],
                               vi[b, :, h] if int8_pv else None, v[b, :, h],
                               vsc[b, h] if int8_pv else None, kcp[b, :, h], vcp[b, :, h],
                               parts["thr"][b, n, h], n, T, N, block, s2, sink_blocks,
                               sink_q, group, int8_pv)
            out[b, r0:r1, h] = o[: r1 - r0]
    if return_parts:
        return out, parts
    return out


def route_mask_int8(q, parts, scale, tokens, block, sink_blocks=(0, 0), sink_q=(0, 0),
                    group=64):
    """Routing mask of the INT8 path: the BF16 rule on the centred kc and the
    tau*sigma threshold (_int8_fwd.py:288-295)."""
    return route_mask(q, parts["kc"], parts["thr"], scale, tokens, block, sink_blocks,
                      sink_q, group)


def dense_reference(q, k, v, scale=None):
    """fp32 softmax(q k^T * scale) v on [B,T,H,D] (torch CPU SDPA, the dense check)."""
    qt, kt, vt = (torch.from_numpy(np.ascontiguousarray(x)).float().permute(0, 2, 1, 3)
                  for x in (q, k, v))
    o = torch.nn.functional.scaled_dot_product_attention(qt, kt, vt, scale=scale)
    return o.permute(0, 2, 1, 3).contiguous().numpy()


# ------------------------------------------------------------- CPU timing arm

def unit_runner(q, k, v, *, tau, block, path="bf16", int8_pv=True, scale=None, group=64):
    """For timing the reference's algorithm on host cores (bench.py's CPU legs): run the
    call's preprocess once (``prepare`` / ``fused_preprocess``, the same code as
    ``sol_attn`` / ``sol_attn_int8``) and return ``run(units)``, which computes the output
    tiles of the given (b, h, q_block) units exactly as those functions do (a list of
    [block, D] float32 tiles, rows past T included)."""
    B, T, H, D = q.shape
    scale = D ** -0.5 if scale is None else float(scale)
    N = -(-T // block)
    s2 = _log2_scale(scale)
    no_sink = (0, 0)
    if path == "int8":
        parts = fused_preprocess(q, k, v, tau, scale, T, block, int8_pv)
        kcp, vcp = _pad_rows(parts["kc"], group), _pad_rows(parts["vc"], group)

        def run(units):
            tiles = []
            for b, h, n in units:
                r0 = n * block
                tiles.append(_fwd_unit_int8(_tile(q[b, :, h], r0, block), _tile(parts["qi"][b, :, h], r0, block),
                               _tile(parts["qs"][b, :, h], r0, block), parts["ki"][b, :, h],
                               parts["ks"][b, :, h], parts["vi"][b, :, h] if int8_pv else None, v[b, :, h],
                               parts["vsc"][b, h] if int8_pv else None, kcp[b, :, h], vcp[b, :, h],
                               parts["thr"][b, n, h], n, T, N, block, s2, no_sink, no_sink, group, int8_pv))
            return tiles
    else:
        kc, vc, thr = prepare(q, k, v, tau, scale, T, block)
        kcp, vcp = _pad_rows(kc, group), _pad_rows(vc, group)

        def run(units):
            return [_fwd_unit_bf16(_tile(q[b, :, h], n * block, block), k[b, :, h], v[b, :, h], kcp[b, :, h],
                                   vcp[b, :, h], thr[b, n, h], n, T, N, block, s2, no_sink, no_sink, group)
                    for b, h, n in units]
    return run
