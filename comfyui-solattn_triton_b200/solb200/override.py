"""The attention-override boundary: the callable ComfyUI invokes for every attention
call, with the reference extension's gates, layouts, fallbacks and counters, over
the sm_100a kernels.

Reference behaviour this module reproduces (kijai/ComfyUI-SolAttn_triton):
    make_override          __init__.py:256-320   mask / depth / sigma gates, sinks,
                                                 dense fallback on decline or error,
                                                 chaining to a previous override
    _run                   __init__.py:192-231   BND (heads*D packed) or BHND layouts
    _ineligible            __init__.py:170-189   cuda, bf16, D == 128, no mask,
                                                 self-attention, T >= min_tokens
    _sink_blocks           __init__.py:237-253   MiniMax-H3 conditioning sink
    parse_blocks           __init__.py:49-66     "0-3,47,-1" depth specs
    parse_tau_profile      __init__.py:69-91     "0-30=2.0; 39-42=0.9"
    make_probe_override    __init__.py:323-342   sparse-vs-dense block probe
    sol_attn_stats         __init__.py:144-152   dispatch counters
    attention_sol          __init__.py:649-663   registry entry with defaults

This build's additions: declined calls that the dense sm_100a kernel can take run there
(``_run``'s dense branch, counter ``dense_b200``), and so do masked calls (``_run_masked``,
counter ``masked_b200``), which the reference always hands to the host.

Nothing here imports ComfyUI: ``func`` (the host's dense attention) is passed in by
the caller, as the host does. The ComfyUI node classes live in the package's
top-level ``__init__.py``.
"""

from __future__ import annotations

import logging
import re
from functools import partial

import torch

from . import ops

HEAD_DIM = 128
BLOCK_SIZE = 64          # routing block of the override (the reference's constant)

_stats = {"sparse": 0, "dense_fallback": 0, "outside_range": 0, "dense_block": 0, "errors": 0,
          "dense_b200": 0, "masked_b200": 0}
_seen = set()
_probe = {}


def sol_attn_stats():
    """Dispatch counters since process start (or the last reset)."""
    return dict(_stats)


def reset_sol_attn_stats():
    for key in _stats:
        _stats[key] = 0
    _seen.clear()


def _log_once(key, message):
    if key not in _seen:
        _seen.add(key)
        logging.info(f"[sol_attn] {message}")


def _log_kernel_failure(exc):
    key = ("kernel_failure", type(exc).__name__, str(exc))
    first = key not in _seen
    _seen.add(key)
    logging.error(f"[sol_attn] kernel failed ({exc}); falling back", exc_info=first)


# ------------------------------------------------------------------ block specs

_SPEC = re.compile(r"(-?\d+)(?:-(-?\d+))?")


def parse_blocks(spec, count):
    """Absolute transformer-block indices from "0-3,47,-1"; negatives count from the
    end, ranges may be given in either order, whitespace is ignored, indices outside
    [0, count) are dropped."""
    chosen = set()
    for part in re.sub(r"\s+", "", str(spec)).split(","):
        if not part:
            continue
        m = _SPEC.fullmatch(part)
        if m is None:
            raise ValueError(f"cannot parse block spec {part!r}; use indices and ranges like "
                             "'0-3,47,-1'")
        lo = int(m.group(1))
        hi = lo if m.group(2) is None else int(m.group(2))
        lo = lo + count if lo < 0 else lo
        hi = hi + count if hi < 0 else hi
        lo, hi = min(lo, hi), max(lo, hi)
        chosen.update(range(max(lo, 0), min(hi, count - 1) + 1))
    return frozenset(chosen)


def parse_tau_profile(spec, count):
    """{block: tau} from "blocks=tau" entries separated by ';' or newlines ('#' starts a
    comment); later entries win."""
    profile = {}
    for raw in re.split(r"[;\n]", str(spec)):
        entry = raw.split("#", 1)[0].strip()
        if not entry:
            continue
        blocks, sep, value = entry.partition("=")
        if not sep:
            raise ValueError(f"tau_profile entry {entry!r} needs '=', e.g. '39-42=0.9'")
        try:
            level = float(value)
        except ValueError:
            raise ValueError(f"tau_profile entry {entry!r} has a non-numeric tau") from None
        for b in parse_blocks(blocks, count):
            profile[b] = level
    return profile


# ------------------------------------------------------------------ dispatch

def _ineligible(q, k, mask, dim_head, min_tokens):
    """Why this BTHD call cannot take the sparse path, or None."""
    if q.device.type != "cuda":
        return "not cuda"
    if q.dtype != torch.bfloat16:
        return f"dtype {q.dtype} (kernel is bf16-only)"
    if dim_head != HEAD_DIM:
        return f"head_dim {dim_head} != {HEAD_DIM}"
    if mask is not None:
        return "masked attention"
    if q.shape[1] != k.shape[1]:
        return "cross-attention (kept dense)"
    if q.shape != k.shape:
        return f"q/k shape mismatch {tuple(q.shape)} vs {tuple(k.shape)}"
    if q.shape[1] < min_tokens:
        return f"seq {q.shape[1]} < {min_tokens}"
    return None


def _dense_capable(q, k, v, dim_head):
    """Whether a declined BTHD call can run on the dense B200 kernel (``ops.dense_attn``)
    instead of the host's attention: bf16 on an sm_100 device, head_dim 64 or 128, k and v
    alike and q matching them in batch and heads (any sequence lengths)."""
    return (q.device.type == "cuda" and q.dtype == k.dtype == v.dtype == torch.bfloat16
            and dim_head in (64, 128) and k.shape == v.shape and q.shape[0] == k.shape[0]
            and q.shape[2:] == k.shape[2:] and torch.cuda.get_device_capability(q.device)[0] == 10)


def _run(q, k, v, heads, skip_reshape, skip_output_reshape, scale, tau, min_tokens, verbose,
         int8_qk=False, sink_blocks=(0, 0), sink_q=(0, 0), use_tma=False, int8_pv=True,
         block=BLOCK_SIZE):
    """The attention output in the caller's layout, or None to stay dense."""
    if skip_reshape:                         # BHND
        b, _, _, dim_head = q.shape
        qs, ks, vs = (t.transpose(1, 2) for t in (q, k, v))
    else:                                    # B, N, heads*dim_head
        b, _, width = q.shape
        dim_head = width // heads
        qs, ks, vs = (t.view(b, -1, heads, dim_head) for t in (q, k, v))
    reason = _ineligible(qs, ks, None, dim_head, min_tokens)
    if reason is not None:
        if _dense_capable(qs, ks, vs, dim_head):
            # this build's addition: the declined call runs dense on the same tensor cores
            out = ops.dense_attn(qs, ks, vs, scale=scale)
            _stats["dense_b200"] += 1
            if verbose:
                _log_once((tuple(qs.shape), reason, "b200"), f"dense sm_100a {tuple(qs.shape)}: {reason}")
            return out.transpose(1, 2) if skip_output_reshape else out.reshape(b, -1, heads * dim_head)
        _stats["dense_fallback"] += 1
        if verbose:
            _log_once((tuple(qs.shape), reason), f"dense {tuple(qs.shape)}: {reason}")
        return None
    if int8_qk:
        out = ops.sol_attn_int8(qs, ks, vs, scale=scale, tau=tau, sink_blocks=sink_blocks,
                                sink_q=sink_q, int8_pv=int8_pv, block=block)
    else:
        out = ops.sol_attn(qs, ks, vs, scale=scale, tau=tau, sink_blocks=sink_blocks,
                           sink_q=sink_q, block=block)
    _stats["sparse"] += 1
    if verbose:
        mode = "int8" if int8_qk else "bf16"
        _log_once((tuple(qs.shape), "sparse", mode), f"sparse {tuple(qs.shape)} tau={tau} {mode} sm_100a")
    if skip_output_reshape:
        return out.transpose(1, 2)
    return out.reshape(b, -1, heads * dim_head)


def _run_masked(q, k, v, heads, mask, skip_reshape, skip_output_reshape, scale, verbose):
    """A masked call on the dense B200 kernel (``ops.dense_attn`` with the mask), in the
    caller's layout, or None when the host must take it: the reference declines every
    masked call (``__init__.py:170-189``); this build runs the ones whose tensors the dense
    kernel takes and whose mask ``ops.mask_layout`` reads (bool or float, broadcastable
    to [B, H, Tq, Tk])."""
    if skip_reshape:                         # BHND
        b, _, _, dim_head = q.shape
        qs, ks, vs = (t.transpose(1, 2) for t in (q, k, v))
    else:                                    # B, N, heads*dim_head
        b, _, width = q.shape
        dim_head = width // heads
        qs, ks, vs = (t.view(b, -1, heads, dim_head) for t in (q, k, v))
    if not _dense_capable(qs, ks, vs, dim_head) or mask.device != q.device:
        return None
    try:
        ops.mask_layout(mask, qs.shape[0], heads, qs.shape[1], ks.shape[1])
    except ValueError:
        return None
    out = ops.dense_attn(qs, ks, vs, scale=scale, mask=mask)
    _stats["masked_b200"] += 1
    if verbose:
        _log_once((tuple(qs.shape), tuple(mask.shape), "masked"),
                  f"masked dense sm_100a {tuple(qs.shape)} mask {tuple(mask.shape)} {mask.dtype}")
    return out.transpose(1, 2) if skip_output_reshape else out.reshape(b, -1, heads * dim_head)


def _sink_blocks(transformer_options, tokens, mode, block=BLOCK_SIZE):
    """(exact-KV block range, dense-query block range) for MiniMax-H3's packed
    conditioning rows [text][cond][ref][audio][video]: every block up to the one holding
    the video span's first token."""
    if mode == "off":
        return (0, 0), (0, 0)
    span = (transformer_options or {}).get("sol_h3_video_span")
    if span is None:
        return (0, 0), (0, 0)
    start, stop = span
    if tokens < stop or start <= 0:
        return (0, 0), (0, 0)
    blocks = (0, -(-start // block))
    return blocks, (blocks if mode == "exact_kv_and_rows" else (0, 0))


def make_override(tau=1.0, min_tokens=4096, sigma_start=None, sigma_end=None, verbose=False,
                  int8_qk=False, sink_conditioning="exact_kv", use_tma=False,
                  dense_blocks=frozenset(), tau_profile=None, int8_pv=True, previous=None,
                  block=BLOCK_SIZE):
    """An ``optimized_attention_override`` callable. Declined calls go to ``previous``
    (an override installed earlier), else to the host's ``func``."""

    def override(func, q, k, v, heads, mask=None, attn_precision=None, skip_reshape=False,
                 skip_output_reshape=False, **kwargs):
        def dense():
            target = func if previous is None else partial(previous, func)
            return target(q, k, v, heads, mask=mask, attn_precision=attn_precision,
                          skip_reshape=skip_reshape, skip_output_reshape=skip_output_reshape,
                          **kwargs)

        if mask is not None:
            try:
                out = _run_masked(q, k, v, heads, mask, skip_reshape, skip_output_reshape,
                                  kwargs.get("scale", None), verbose)
            except Exception as exc:
                _stats["errors"] += 1
                _log_kernel_failure(exc)
                out = None
            if out is None:
                _stats["dense_fallback"] += 1
                return dense()
            return out
        options = kwargs.get("transformer_options", {}) or {}
        depth = options.get("sol_block") if (dense_blocks or tau_profile) else None
        if depth in dense_blocks:
            _stats["dense_block"] += 1
            return dense()
        block_tau = tau_profile.get(depth, tau) if tau_profile else tau
        if sigma_start is not None or sigma_end is not None:
            sigmas = options.get("sigmas")
            if sigmas is not None:
                sigma = float(sigmas[0])
                if (sigma_start is not None and sigma > sigma_start) or \
                        (sigma_end is not None and sigma < sigma_end):
                    _stats["outside_range"] += 1
                    return dense()
        tokens = q.shape[2] if skip_reshape else q.shape[1]
        sink, sink_q = _sink_blocks(kwargs.get("transformer_options"), tokens, sink_conditioning,
                                    block)
        if verbose and sink != (0, 0):
            _log_once((tokens, sink, sink_q),
                      f"conditioning sink: KV blocks {sink} exact, dense query blocks {sink_q}")
        try:
            out = _run(q, k, v, heads, skip_reshape, skip_output_reshape, kwargs.get("scale", None),
                       block_tau, min_tokens, verbose, int8_qk, sink, sink_q, use_tma, int8_pv,
                       block)
        except Exception as exc:
            _stats["errors"] += 1
            _log_kernel_failure(exc)
            return dense()
        return dense() if out is None else out

    return override


def _probe_record(block, sparse_out, reference):
    ref = reference.float()
    norm = ref.norm()
    if norm > 0:
        entry = _probe.setdefault(block, [0.0, 0])
        entry[0] += float((sparse_out.float() - ref).norm() / norm)
        entry[1] += 1


def log_probe_summary(*_args, **_kwargs):
    """Per-block relative error of the sparse path, worst first."""
    if not _probe:
        return
    rows = sorted(((tot / n, blk, n) for blk, (tot, n) in _probe.items()), reverse=True)
    logging.info("[sol_attn] block sensitivity to sparsification (worst first); "
                 "put the top entries in dense_blocks:")
    for err, blk, n in rows:
        logging.info(f"[sol_attn]   block {blk}  rel err {err:.4f}  ({n} calls)")
    _probe.clear()


def probe_results():
    return {blk: tot / n for blk, (tot, n) in _probe.items()}


def make_probe_override(inner):
    """Every call computed sparse and dense; the dense result is returned so errors
    do not compound across blocks."""

    def override(func, q, k, v, heads, mask=None, attn_precision=None, skip_reshape=False,
                 skip_output_reshape=False, **kwargs):
        common = dict(mask=mask, attn_precision=attn_precision, skip_reshape=skip_reshape,
                      skip_output_reshape=skip_output_reshape, **kwargs)
        sparse = inner(func, q, k, v, heads, **common)
        reference = func(q, k, v, heads, **common)
        _probe_record((kwargs.get("transformer_options") or {}).get("sol_block"), sparse, reference)
        return reference

    return override


def attention_sol(q, k, v, heads, mask=None, attn_precision=None, skip_reshape=False,
                  skip_output_reshape=False, dense=None, **kwargs):
    """Registry entry point with the defaults (tau 1.0, min_tokens 4096, no gates);
    ``dense`` is the host's fallback attention."""
    try:
        if mask is None:
            out = _run(q, k, v, heads, skip_reshape, skip_output_reshape, kwargs.get("scale", None),
                       1.0, 4096, False)
        else:
            out = _run_masked(q, k, v, heads, mask, skip_reshape, skip_output_reshape,
                              kwargs.get("scale", None), False)
        if out is not None:
            return out
    except Exception as exc:
        _stats["errors"] += 1
        _log_kernel_failure(exc)
    if dense is None:
        raise RuntimeError("solb200.attention_sol: no dense fallback given for a declined call")
    return dense(q, k, v, heads, mask=mask, skip_reshape=skip_reshape,
                 skip_output_reshape=skip_output_reshape, **kwargs)
