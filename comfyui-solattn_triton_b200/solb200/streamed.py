"""Sol-Attn on q/k/v that live in host memory, streamed through the GPU by head chunks.

Every stage of the path depends only on its own (batch, head), so the heads can be cut
into chunks and the three costs of a host-resident call overlap instead of adding up:

    copy stream     H2D q,k,v of chunk i+1          (PCIe, host -> device)
    compute stream  Sol-Attn of chunk i              (the same kernels as sol_attn)
    copy-out stream D2H output of chunk i-1          (PCIe, device -> host)

Host -> device and device -> host run on separate copy engines, so a call costs about
the host -> device transfer of q, k and v plus one chunk's compute and copy-out. Each
head's output is bit-identical to ``sol_attn`` / ``sol_attn_int8`` on device tensors.
Device memory: two chunk slots of q, k, v, out plus one workspace. They and the two copy
streams are kept per (device, geometry) across calls (``release_host_buffers`` frees
them), so a repeated call allocates nothing and creates no stream.

The reference has no host-memory entry point (its wrappers receive device tensors);
this is this build's addition for callers that keep activations in host memory.
"""

from __future__ import annotations

import torch

from ._lib import check, lib
from .ops import BLOCK, I64x2, I64x3, STAGES_ALL, _SYNC_CHECK, Workspace

H2D, D2H = 1, 0


def plan_chunks(heads: int, heads_per_chunk: int | None = None) -> list[tuple[int, int]]:
    """(first head, head count) of each chunk. Default: 2 heads from 16 heads up (at 40
    heads 2-head chunks measured 19.7 ms per host-to-host call against 20.3 ms for 5-head
    and 22.3 ms for 10-head chunks), single heads below, so that a rank with few heads
    still has at least four chunks in flight and only the first copy-in and the last
    copy-out are exposed."""
    if heads < 1:
        raise ValueError("heads must be positive")
    hc = heads_per_chunk if heads_per_chunk else min(heads, 2 if heads >= 16 else 1)
    if hc < 1:
        raise ValueError("heads_per_chunk must be positive")
    return [(h0, min(hc, heads - h0)) for h0 in range(0, heads, hc)]


_BUFFERS = {}


def _buffers(dev, B, T, hc, D, block, int8):
    """Copy streams, two chunk slots of q, k, v, out and a workspace for this geometry,
    created on first use and kept for later calls."""
    key = (str(dev), B, T, hc, D, block, bool(int8))
    hit = _BUFFERS.get(key)
    if hit is None:
        hit = dict(s_in=torch.cuda.Stream(dev), s_out=torch.cuda.Stream(dev),
                   slots=[[torch.empty((B, T, hc, D), dtype=torch.bfloat16, device=dev) for _ in range(4)]
                          for _ in range(2)],
                   ws=Workspace(B, T, hc, D, block, int8, dev))
        _BUFFERS[key] = hit
    return hit


def release_host_buffers():
    """Free the device buffers and streams kept by sol_attn_host (after a synchronize)."""
    torch.cuda.synchronize()
    _BUFFERS.clear()


def _check_host(t: torch.Tensor, name: str):
    if t.device.type != "cpu":
        raise RuntimeError(f"solb200.sol_attn_host: {name} must be a host (CPU) tensor")
    if t.dtype != torch.bfloat16:
        raise RuntimeError(f"solb200.sol_attn_host: {name} must be bfloat16")
    if t.dim() != 4 or not t.is_contiguous():
        raise RuntimeError(f"solb200.sol_attn_host: {name} must be a contiguous BTHD tensor")


def sol_attn_host(q, k, v, *, scale=None, tau=1.0, sink_blocks=(0, 0), sink_q=(0, 0), block=BLOCK,
                  int8=False, int8_pv=True, heads_per_chunk=None, out=None, device=None,
                  synchronize=True):
    """Sol-Attn of host BTHD bf16 q/k/v (contiguous; page-locked for overlap) into a host
    output (``out``, or a new page-locked tensor). ``int8`` selects the INT8 path. With
    ``synchronize`` the call returns once the output is in host memory; otherwise the
    current stream of ``device`` waits for it (stream-ordered)."""
    for t, n in ((q, "q"), (k, "k"), (v, "v")):
        _check_host(t, n)
    if q.shape != k.shape or q.shape != v.shape:
        raise RuntimeError("solb200.sol_attn_host: q/k/v shapes differ")
    B, T, H, D = q.shape
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    if out is None:
        out = torch.empty((B, T, H, D), dtype=torch.bfloat16, pin_memory=True)
    else:
        _check_host(out, "out")
        if out.shape != q.shape:
            raise RuntimeError("solb200.sol_attn_host: out has the wrong shape")
    chunks = plan_chunks(H, heads_per_chunk)
    hc = max(n for _, n in chunks)
    scale = D ** -0.5 if scale is None else float(scale)
    L = lib()
    with torch.cuda.device(dev):
        comp = torch.cuda.current_stream(dev)
        bufs = _buffers(dev, B, T, hc, D, block, int8)
        s_in, s_out, slots, ws = bufs["s_in"], bufs["s_out"], bufs["slots"], bufs["ws"]
        # the copy streams start after whatever the caller queued on its stream (which
        # includes the previous call's last copy-out, so the kept slots are free again)
        s_in.wait_stream(comp)
        s_out.wait_stream(comp)
        sk, sq = I64x2(int(sink_blocks[0]), int(sink_blocks[1])), I64x2(int(sink_q[0]), int(sink_q[1]))
        ev_in, ev_comp, ev_out = [], [], []
        for i, (h0, n) in enumerate(chunks):
            dq, dk, dv, do = slots[i % 2]
            e_in, e_comp, e_out = (torch.cuda.Event() for _ in range(3))
            # H2D of chunk i into its slot once chunk i-2's kernels have read that slot
            if i >= 2:
                s_in.wait_event(ev_comp[i - 2])
            for dst, src in ((dq, q), (dk, k), (dv, v)):
                check(L.solb200_copy_heads(dst.data_ptr(), src.data_ptr(), B, T, H, D, h0, n, H2D,
                                           s_in.cuda_stream), "copy_heads H2D")
            e_in.record(s_in)
            # the attention of chunk i once its inputs are in, and chunk i-2's output
            # has left the slot
            comp.wait_event(e_in)
            if i >= 2:
                comp.wait_event(ev_out[i - 2])
            st = I64x3(T * n * D, n * D, D)
            a = [dq.data_ptr(), st, dk.data_ptr(), st, dv.data_ptr(), st, do.data_ptr(), B, T, n, D, block,
                 scale, float(tau), sk, sq]
            tail = [STAGES_ALL, ws.ptr(), ws.nbytes, None, None, comp.cuda_stream]
            rc = (L.solb200_sol_attn_int8(*a, int(bool(int8_pv)), *tail) if int8
                  else L.solb200_sol_attn_bf16(*a, *tail))
            check(rc, "sol_attn_host chunk")
            if _SYNC_CHECK:
                ws.check_device_error()   # every call clears the error word: check each chunk
            e_comp.record(comp)
            # D2H of chunk i's output
            s_out.wait_event(e_comp)
            check(L.solb200_copy_heads(do.data_ptr(), out.data_ptr(), B, T, H, D, h0, n, D2H,
                                       s_out.cuda_stream), "copy_heads D2H")
            e_out.record(s_out)
            ev_in.append(e_in)
            ev_comp.append(e_comp)
            ev_out.append(e_out)
        # the caller's stream (and so the next call) waits for the last copy-out
        comp.wait_event(ev_out[-1])
        if synchronize:
            ev_out[-1].synchronize()
    return out
