"""Benchmark of the Sol-Attn hot path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--path bf16|int8] [--impl ours|reference]

Workload: the headline configuration (config 3): B=1, H=40, T=21x30x52=32760 tokens,
D=128, block 128, tau=0.9, seeded synthetic video-DiT q/k/v (solb200.workloads).
A step is one attention call through the C ABI: pooling, routing, the block-sparse
forward. value = dense-equivalent TFLOP/s of the whole job (4*B*H*T^2*D / time).
With N GPUs (torchrun) the 40 heads are split across ranks (H/N each, no
collective); time is the max over ranks.

Also on the line: the INT8 path at config 3 (``int8``), config 5 (T=111600) with the input
sequence-sharded over the N ranks and re-sharded by NCCL all-to-alls (``ulysses_c5``, BF16
and INT8), the end-to-end call from pinned host memory (``e2e``), the stage split, the
roofline of the forward kernel, the Morton reorder and dense SDPA on the same GPU.

--impl reference times the reference's algorithm on the host cores instead: the CPU
oracle port (oracle/solattn_oracle.py, a step-for-step restatement of the reference's
kernels, pinned bit-exact to them) on a bounded sample of query blocks per step,
extrapolated to the full call, with one process per host core.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "comfyui-solattn_triton_b200"))
sys.path.insert(0, str(REPO))

METRIC = "ms/attn call + dense-equiv TFLOPS @40h×32760tok×D128 bf16/int8, tau=0.9"
UNIT = "dense-equiv TFLOP/s"
L2_NOTE = "L2 flushed before every timed step (256 MB write, outside the step's CUDA-event pair)"


def bench_config(path, world):
    """The `config` of both arms (identical for the same arguments)."""
    return {"workload": "config3_video480p_B1_H40_T32760_D128_blk128_tau0.9", "path": path,
            "heads_per_rank": 40 // world, "parallelism": f"heads/{world}", "l2": L2_NOTE}


def load_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return dict(hbm=d["hbm_gbs"], bf16=d["bf16_tflops"], bf16_sus=d.get("bf16_tflops_sustained"),
                    source="measured")
    return dict(hbm=6650.0, bf16=1590.0, bf16_sus=1400.0, source="fallback")


def profiled_traffic(path, heads):
    """DRAM bytes (read + write) of one forward launch at `heads` heads, from the ncu
    capture summarised in profiles/sol_fwd_<path>_config3.md (a line
    `traffic_bytes_per_head: N`; every head's work is independent, so traffic scales
    with the head count). None when there is no capture for this path."""
    f = REPO / "profiles" / f"sol_fwd_{path}_config3.md"
    if not f.exists():
        return None
    for line in f.read_text().splitlines():
        if line.strip().startswith("traffic_bytes_per_head:"):
            return float(line.split(":", 1)[1].strip().strip("`")) * heads
    return None


class Clocks:
    """nvidia-smi sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.result = None
        if self.proc is None:
            return False
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out = ""
        sms, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sms.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if sms:
            self.result = {"sm_mhz": statistics.median(sms), "sm_max_mhz": mx,
                           "reasons": sorted(reasons), "samples": len(sms)}
        return False


class Timer:
    """CUDA-event timing on one stream with an L2 flush (a 256 MB write) before every
    timed step, outside the step's event pair; the mean over steps, max over ranks."""

    def __init__(self, torch, dist, dev, world):
        self.torch, self.dist, self.dev, self.world = torch, dist, dev, world
        self.flush_buf = torch.empty((256 << 20) // 4, dtype=torch.float32, device=dev)

    def __call__(self, fn, steps, stream=None):
        torch = self.torch
        stream = stream or torch.cuda.current_stream(self.dev)
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(steps)]
        if self.world > 1:
            self.dist.barrier()
        torch.cuda.synchronize()
        for ev0, ev1 in evs:
            self.flush_buf.zero_()
            ev0.record(stream)
            fn()
            ev1.record(stream)
        torch.cuda.synchronize()
        if self.world > 1:
            self.dist.barrier()
        ms = sum(ev0.elapsed_time(ev1) for ev0, ev1 in evs) / steps
        return self.max_over_ranks(ms)

    def max_over_ranks(self, x):
        t = self.torch.tensor([float(x)], device=self.dev)
        if self.world > 1:
            self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())


def executed_flops(torch, ws, B, H, T, D, blk):
    """Executed (algorithmic) flops of one forward launch from the routing in `ws`:
    4 D sum over routed pairs len(qb) len(kb) + 4 D B H T N (approximate branch); and the
    routed density."""
    counts = ws.view("count", torch.int32, (B, H, ws.N)).long()
    words = ws.view("mask", torch.int32, (B, H, ws.N, ws.nw))
    tail = T - (ws.N - 1) * blk
    n_pairs = int(counts.sum())
    bits = torch.arange(32, device=words.device, dtype=torch.int32)
    mask = ((words.unsqueeze(-1) >> bits) & 1).reshape(B, H, ws.N, -1)[..., :ws.N]
    last_col = int(mask[..., ws.N - 1].sum())        # routed pairs whose key block is the tail
    last_row = int(mask[:, :, ws.N - 1, :].sum())    # routed pairs whose query block is the tail
    corner = int(mask[:, :, ws.N - 1, ws.N - 1].sum())
    tok_pairs = (n_pairs * blk * blk - last_col * blk * (blk - tail) - last_row * blk * (blk - tail)
                 + corner * (blk - tail) ** 2)
    flops = 4.0 * D * tok_pairs + 4.0 * D * B * H * T * ws.N
    return flops, n_pairs / float(B * H * ws.N * ws.N)


# ------------------------------------------------------------------ our arm

def bind_gpu_local_cpus(torch, local_rank):
    """Run this process on the CPUs local to its GPU, so that the pinned host buffers of the
    e2e leg (placed on first touch) sit on the GPU's NUMA node. Returns the CPU list it
    bound to, or None when the PCI topology is not readable or shares no CPU with the
    allowed set."""
    try:
        p = torch.cuda.get_device_properties(local_rank)
        bus = f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        text = open(f"/sys/bus/pci/devices/{bus}/local_cpulist").read().strip()
        cpus = set()
        for part in text.split(","):
            lo, _, hi = part.partition("-")
            cpus.update(range(int(lo), int(hi or lo) + 1))
        cpus &= os.sched_getaffinity(0)
        if not cpus:
            return None
        os.sched_setaffinity(0, cpus)
        return text
    except Exception:
        return None


class Ctx:
    """What every measurement of our arm needs."""

    def __init__(self, args, rank, world, local_rank):
        import torch
        import torch.distributed as dist
        from solb200 import _lib
        self.torch, self.dist, self._lib = torch, dist, _lib
        self.args, self.rank, self.world, self.local_rank = args, rank, world, local_rank
        self.dev = torch.device("cuda", local_rank)
        torch.cuda.set_device(self.dev)
        self.host_cpus = bind_gpu_local_cpus(torch, local_rank)
        self.lib = _lib.lib()
        self.timer = Timer(torch, dist, self.dev, world)


def make_call(ctx, path, ws, q, k, v, out, tau):
    """One attention call through the C ABI on the current stream (stages selectable)."""
    from solb200.ops import I64x2, I64x3
    B, T, H, D = q.shape
    int8 = path == "int8"
    stream = ctx.torch.cuda.current_stream(ctx.dev).cuda_stream
    zero = I64x2(0, 0)

    def call(stages):
        a = [q.data_ptr(), I64x3(*q.stride()[:3]), k.data_ptr(), I64x3(*k.stride()[:3]), v.data_ptr(),
             I64x3(*v.stride()[:3]), out.data_ptr(), B, T, H, D, ws.block, D ** -0.5, tau, zero, zero]
        tail = [stages, ws.ptr(), ws.nbytes, None, None, stream]
        rc = (ctx.lib.solb200_sol_attn_int8(*a, 1, *tail) if int8
              else ctx.lib.solb200_sol_attn_bf16(*a, *tail))
        ctx._lib.check(rc, "bench call")
    return call


def measure_c3(ctx, path, q, k, v, cfg):
    """Config 3 on this rank's heads: the call, its stage split and the forward's
    executed flops; timed on the launching stream, max over ranks."""
    torch = ctx.torch
    from solb200.ops import STAGES_ALL, STAGES_PREPARE, Workspace
    from solb200._lib import STAGES_FORWARD
    B, T, H, D = q.shape
    ws = Workspace(B, T, H, D, cfg.block, path == "int8", ctx.dev)
    out = torch.empty((B, T, H, D), dtype=torch.bfloat16, device=ctx.dev)
    call = make_call(ctx, path, ws, q, k, v, out, cfg.tau)
    steps = ctx.args.steps
    for _ in range(ctx.args.warmup):
        call(STAGES_ALL)
    ws.check_device_error()
    with Clocks(ctx.local_rank) as clk:
        ms = ctx.timer(lambda: call(STAGES_ALL), steps)
    ws.check_device_error()
    for _ in range(2):
        call(STAGES_PREPARE)
    ms_prep = ctx.timer(lambda: call(STAGES_PREPARE), steps)
    for _ in range(2):
        call(STAGES_FORWARD)
    ms_fwd = ctx.timer(lambda: call(STAGES_FORWARD), steps)
    # PREPARE in its parts (each timed alone, so each carries its own launch latency)
    from solb200._lib import STAGES_POOL, STAGES_QUANT, STAGES_ROUTE
    parts = {"pool": STAGES_POOL, "route": STAGES_ROUTE}
    if path == "int8":
        parts["quant"] = STAGES_QUANT
    ms_parts = {}
    for name, st in parts.items():
        call(st)
        ms_parts[name] = ctx.timer(lambda st=st: call(st), steps)
    ws.check_device_error()
    flops, density = executed_flops(torch, ws, B, H, T, D, cfg.block)
    # the slowest rank's forward decides the job; flops summed over ranks
    flops_all = flops
    if ctx.world > 1:
        t = torch.tensor([flops], device=ctx.dev, dtype=torch.float64)
        ctx.dist.all_reduce(t)
        flops_all = float(t.item())
    return dict(ms=ms, ms_prep=ms_prep, ms_fwd=ms_fwd, ms_parts=ms_parts, flops=flops, flops_all=flops_all,
                density=density, clocks=clk.result, ws=ws, out=out)


def int8_block(ctx, m, cfg, peaks):
    """The INT8 path's sub-object (config 3): ms per call, stage split, executed-op
    roofline of the forward kernel and the clocks of its timed region."""
    achieved = m["flops_all"] / ctx.world / (m["ms_fwd"] * 1e-3) / 1e12   # one GPU's launch
    return {
        "ms_per_call": m["ms"], "value": cfg.dense_flops() / (m["ms"] * 1e-3) / 1e12, "unit": UNIT,
        "stages_ms": {"prep_route": m["ms_prep"], **m["ms_parts"], "forward": m["ms_fwd"]},
        "routed_density": m["density"],
        "roofline": {"bound": "tensor", "kernel": "sol_fwd_int8_kernel", "achieved": achieved,
                     "unit": "TOP/s", "peak_bf16": peaks["bf16"], "frac_of_bf16_peak": achieved / peaks["bf16"],
                     "peak_int8": 2 * peaks["bf16"], "frac_of_int8_peak": achieved / (2 * peaks["bf16"]),
                     "traffic": profiled_traffic("int8", 40 // ctx.world),
                     "note": "executed ops (int8 exact tiles + bf16 approximate tiles) of one GPU's launch "
                             "(all ranks' / N) / the slowest rank's forward time; int8 peak = 2 x the measured "
                             f"bf16 peak (nominal ratio), {peaks['source']}"},
        "clocks": m["clocks"],
    }


def e2e_block(ctx, q, k, v, cfg, path):
    """End to end through the public API for host-resident tensors: pinned host q/k/v ->
    solb200.sol_attn_host (head chunks streamed in, computed and streamed out) -> pinned
    host output, timed over the bench's steps."""
    torch = ctx.torch
    import solb200
    hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
    hout = torch.empty(q.shape, dtype=torch.bfloat16).pin_memory()

    def step():
        solb200.sol_attn_host(hq, hk, hv, tau=cfg.tau, block=cfg.block, int8=path == "int8", out=hout,
                              heads_per_chunk=ctx.args.e2e_chunk or None, synchronize=False)

    for _ in range(max(2, ctx.args.warmup)):
        step()
    ms = ctx.timer(step, ctx.args.steps)
    solb200.release_host_buffers()
    h2d = sum(t.numel() * t.element_size() for t in (hq, hk, hv))
    d2h = hout.numel() * hout.element_size()
    return {"value": cfg.dense_flops() / (ms * 1e-3) / 1e12, "unit": UNIT, "ms_per_step": ms,
            "h2d_bytes_per_step": h2d * ctx.world, "d2h_bytes_per_step": d2h * ctx.world,
            "h2d_gbs_per_rank": h2d / (ms * 1e-3) / 1e9,
            "host_cpus": ctx.host_cpus or "unbound",
            "api": "solb200.sol_attn_host (pinned host in and out, head chunks streamed)"}


def ulysses_block(ctx, path):
    """Config 5 (B1 H40 T111600 D128, block 128, tau 0.9): q/k/v arrive sequence-sharded
    (T/N tokens, all 40 heads per rank), NCCL all-to-alls re-shard them to H/N heads of
    the whole sequence, Sol-Attn runs locally, an all-to-all returns the output to the
    sequence shards. Timed: the whole step, the exchanges alone, the local call alone.
    Checked: this rank's shard of head 0 equals the single-GPU call on head 0's full
    sequence bit for bit (rank 0; heads are independent). At N = 1 the step is the plain
    call (no exchange)."""
    torch = ctx.torch
    import solb200
    from solb200.parallel import head_to_seq, seq_to_head
    from solb200.workloads import CONFIGS, make_qkv
    cfg = CONFIGS["c5"]
    T, W, r = cfg.tokens, ctx.world, ctx.rank
    Tl = T // W
    q, k, v = make_qkv(cfg, device=ctx.dev)
    ql, kl, vl = (t[:, r * Tl:(r + 1) * Tl].contiguous() for t in (q, k, v))
    q0, k0, v0 = (t[:, :, 0:1].contiguous() for t in (q, k, v))
    del q, k, v
    torch.cuda.empty_cache()
    fn = solb200.sol_attn_int8 if path == "int8" else solb200.sol_attn
    kw = dict(tau=cfg.tau, block=cfg.block)
    res = {}
    if W > 1:
        def step():
            qh, kh, vh = (seq_to_head(t) for t in (ql, kl, vl))
            return head_to_seq(fn(qh, kh, vh, **kw))
        qh, kh, vh = (seq_to_head(t) for t in (ql, kl, vl))
        oh = fn(qh, kh, vh, **kw)
        for _ in range(ctx.args.warmup):
            step()
        res["ms_per_call"] = ctx.timer(step, ctx.args.steps)
        res["exchange_ms"] = ctx.timer(lambda: ([seq_to_head(t) for t in (ql, kl, vl)], head_to_seq(oh)),
                                       ctx.args.steps)
        res["local_ms"] = ctx.timer(lambda: fn(qh, kh, vh, **kw), ctx.args.steps)
        out = step()
    else:
        for _ in range(ctx.args.warmup):
            fn(ql, kl, vl, **kw)
        res["ms_per_call"] = ctx.timer(lambda: fn(ql, kl, vl, **kw), ctx.args.steps)
        res["exchange_ms"] = 0.0
        res["local_ms"] = res["ms_per_call"]
        out = fn(ql, kl, vl, **kw)
    ok = True
    if r == 0:
        want = fn(q0, k0, v0, **kw)[:, :Tl, 0]
        ok = bool(torch.equal(out[:, :, 0], want))
    res["head0_bit_identical"] = bool(ctx.timer.max_over_ranks(0.0 if ok else 1.0) == 0.0)
    dense = 4.0 * cfg.batch * cfg.heads * T ** 2 * cfg.head_dim
    res.update({"value": dense / (res["ms_per_call"] * 1e-3) / 1e12, "unit": UNIT,
                "workload": "config5_B1_H40_T111600_D128_blk128_tau0.9_seq_sharded",
                "heads_per_rank": cfg.heads // W, "tokens_per_rank_in": Tl,
                "exchange": "NCCL all_to_all_single x3 in, x1 out" if W > 1 else "none (one rank)"})
    return res


def morton_block(ctx, q, k, v, out, cfg, path, sdpa, qt, kt, vt, density, plain_ms):
    """Morton (both curves): the gather passes' cost, the call with the gathers (Python API)
    and the reordered call that fuses them (C ABI, preallocated, next to the plain call's
    `plain_ms`), routed density and accuracy against dense SDPA (one GPU)."""
    torch = ctx.torch
    import solb200
    fn = solb200.sol_attn_int8 if path == "int8" else solb200.sol_attn
    dense_out = sdpa(qt, kt, vt).transpose(1, 2)

    def vs_dense(o):
        a, b = o.float().flatten(), dense_out.float().flatten()
        return {"max_abs": float((a - b).abs().max()), "cosine": float((a @ b) / (a.norm() * b.norm()))}

    kw = dict(tau=cfg.tau, block=cfg.block)
    res = {"none": {"routed_density": density, "vs_dense": vs_dense(fn(q, k, v, **kw))}}
    for curve in ("3d", "2d_frame"):
        pm, ivm = solb200.morton_perm(cfg.grid, ctx.dev, curve)
        for _ in range(2):
            solb200.permute_tokens_many([q, k, v], pm), solb200.permute_tokens(out, ivm)
        ms_r = ctx.timer(lambda: (solb200.permute_tokens_many([q, k, v], pm), solb200.permute_tokens(out, ivm)), 3)

        def unfused():
            qp, kp, vp = solb200.permute_tokens_many([q, k, v], pm)
            return solb200.permute_tokens(fn(qp, kp, vp, **kw), ivm)

        def fused():
            return fn(q, k, v, token_order=pm, **kw)

        for _ in range(2):
            unfused(), fused()
        ms_unfused = ctx.timer(unfused, ctx.args.steps)
        # the reordered call through the C ABI on a preallocated workspace, as the headline
        # call is timed (the Python-level calls above allocate their outputs)
        from solb200.ops import I64x2, I64x3, Workspace
        B, T, H, D = q.shape
        wsr = Workspace(B, T, H, D, cfg.block, path == "int8", ctx.dev, reordered=True)
        outr = torch.empty_like(out)
        stream = torch.cuda.current_stream(ctx.dev).cuda_stream

        def reordered_abi():
            ctx._lib.check(ctx.lib.solb200_sol_attn_reordered(
                q.data_ptr(), I64x3(*q.stride()[:3]), k.data_ptr(), I64x3(*k.stride()[:3]), v.data_ptr(),
                I64x3(*v.stride()[:3]), outr.data_ptr(), B, T, H, D, cfg.block, D ** -0.5, cfg.tau, I64x2(0, 0),
                I64x2(0, 0), pm.data_ptr(), int(path == "int8"), 1, wsr.ptr(), wsr.nbytes, stream), "reordered call")

        for _ in range(3):
            reordered_abi()
        ms_fused = ctx.timer(reordered_abi, ctx.args.steps)
        wsr.check_device_error()
        om = fused()
        qp, kp, vp = solb200.permute_tokens_many([q, k, v], pm)
        r = solb200.routing(qp, kp, vp, tau=cfg.tau, block=cfg.block, int8=path == "int8")
        res[curve] = {"reorder_ms": ms_r, "gather_call_gather_ms": ms_unfused, "reordered_call_ms": ms_fused,
                      "reordered_call_over_plain_ms": ms_fused - plain_ms,
                      "reordered_equals_gathers": bool(torch.equal(om, unfused())),
                      "routed_density": float(r["mask"].float().mean()), "vs_dense": vs_dense(om)}
        del qp, kp, vp, r, om
    return res


def run_ours(args, rank, world, local_rank):
    import dataclasses
    ctx = Ctx(args, rank, world, local_rank)
    torch = ctx.torch
    import solb200
    from solb200.workloads import CONFIGS, make_qkv

    cfg = CONFIGS["c3"]
    if args.heads:   # profiling only: a smaller launch of the same kernels
        cfg = dataclasses.replace(cfg, heads=args.heads)
    if cfg.heads % world:
        raise SystemExit(f"{cfg.heads} heads do not split over {world} ranks")
    H = cfg.heads // world
    q, k, v = make_qkv(cfg, device=ctx.dev, heads=slice(rank * H, (rank + 1) * H))
    torch.cuda.synchronize()
    peaks = load_peaks()

    m = measure_c3(ctx, args.path, q, k, v, cfg)
    ms, out = m["ms"], m["out"]
    int8 = None
    if args.path == "bf16" and not args.no_int8:
        int8 = int8_block(ctx, measure_c3(ctx, "int8", q, k, v, cfg), cfg, peaks)
    e2e = None if args.no_e2e else e2e_block(ctx, q, k, v, cfg, args.path)

    # Morton reorder stage: q, k, v into Z-order and O back (one gather launch each way)
    perm, inv = solb200.morton_perm(cfg.grid, ctx.dev, "3d")

    def reorder():
        return solb200.permute_tokens_many([q, k, v], perm), solb200.permute_tokens(out, inv)

    for _ in range(2):
        reorder()
    ms_reorder = ctx.timer(reorder, 3)

    # dense reference on the same GPU (torch SDPA, bf16): the "< 30% of dense" target
    ms_dense, morton = None, None
    sdpa = torch.nn.functional.scaled_dot_product_attention
    qt, kt, vt = (t.transpose(1, 2) for t in (q, k, v))
    if not args.no_dense:
        for _ in range(2):
            sdpa(qt, kt, vt)
        ms_dense = ctx.timer(lambda: sdpa(qt, kt, vt), 3)
        if world == 1:
            morton = morton_block(ctx, q, k, v, out, cfg, args.path, sdpa, qt, kt, vt, m["density"], ms)

    ulysses = None
    if not args.no_ulysses and not args.heads:
        del qt, kt, vt
        torch.cuda.empty_cache()
        ulysses = {p: ulysses_block(ctx, p) for p in ("bf16", "int8")}

    achieved = m["flops_all"] / world / (m["ms_fwd"] * 1e-3) / 1e12   # one GPU's launch
    config = bench_config(args.path, world)
    if args.heads:
        config.update(workload=f"config3_video480p_B1_H{cfg.heads}_T32760_D128_blk128_tau0.9",
                      heads_per_rank=H)
    launches_per_call = 6 if args.path == "int8" else 5   # pool, moments, (quant_kv), route, order, forward
    return {
        "metric": METRIC,
        "value": cfg.dense_flops() / (ms * 1e-3) / 1e12,
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": args.path,
        "data": "synthetic (seeded smooth+noise video-DiT q/k/v, solb200.workloads)",
        "config": config,
        "routed_density": m["density"],
        "stages_ms": {"prep_route": m["ms_prep"], **m["ms_parts"], "forward": m["ms_fwd"],
                      "reorder_qkv_and_o": ms_reorder},
        "dense_sdpa_ms": ms_dense,
        "sparse_over_dense": (ms / ms_dense) if ms_dense else None,
        "roofline": {"bound": "tensor", "kernel": f"sol_fwd_{args.path}_kernel",
                     "achieved": achieved, "peak": peaks["bf16"], "unit": "TFLOP/s",
                     "frac": achieved / peaks["bf16"],
                     "traffic": profiled_traffic(args.path, H),
                     "note": f"executed flops of one GPU's launch ({m['flops_all']:.4g} over all ranks / {world}) "
                             f"/ the slowest rank's forward kernel time (CUDA events on its stream); peak = bf16 dense "
                             f"burst, {peaks['source']}; traffic = DRAM bytes per launch from the ncu capture "
                             f"in profiles/, scaled to {H} heads"},
        "int8": int8,
        "ulysses_c5": ulysses,
        "e2e": e2e,
        "morton": morton,
        "gpu_launches": launches_per_call * args.steps,
        "clocks": m["clocks"],
    }


# ------------------------------------------------------------- CPU baseline

_SAMPLER = None


def _sampler_init(path, arrays, tau, block):
    """Pool worker set-up: the head's preprocess once (timed), kept for every step."""
    global _SAMPLER
    import threadpoolctl
    threadpoolctl.threadpool_limits(1)
    from oracle import solattn_oracle as O
    qn, kn, vn = arrays
    t0 = time.perf_counter()
    run = O.unit_runner(qn, kn, vn, tau=tau, block=block, path=path)
    _SAMPLER = (run, time.perf_counter() - t0)


def _sampler_units(units):
    """Seconds one worker takes for `units` (b, h, q_block) forward tiles, and its
    preprocess seconds."""
    run, prep_s = _SAMPLER
    t0 = time.perf_counter()
    run(units)
    return time.perf_counter() - t0, prep_s, len(units)


def cpu_sdpa_dense(rows=2048):
    """torch CPU SDPA (dense, fp32: the CPU path's dense attention) on head 0 of config 3:
    `rows` query rows against all 32760 keys, timed once after a warm-up on a smaller
    slice, extrapolated to the call's 40 heads x 32760 rows. Uses torch's intra-op
    threads."""
    import torch
    from solb200.workloads import CONFIGS, make_qkv
    cfg = CONFIGS["c3"]
    q, k, v = (t.float().transpose(1, 2) for t in make_qkv(cfg, heads=slice(0, 1)))   # [1, 1, T, D]
    sdpa = torch.nn.functional.scaled_dot_product_attention
    sdpa(q[:, :, :256], k, v)
    t0 = time.perf_counter()
    sdpa(q[:, :, :rows], k, v)
    sec = time.perf_counter() - t0
    ms = sec * 1e3 * (cfg.tokens / rows) * cfg.heads * cfg.batch
    return {"ms_per_call": ms, "value": cfg.dense_flops() / (ms * 1e-3) / 1e12, "unit": UNIT,
            "cores": torch.get_num_threads(),
            "sample": f"{rows} query rows of head 0 x {cfg.tokens} keys, fp32, extrapolated to "
                      f"{cfg.heads} heads x {cfg.tokens} rows"}


class CpuSampler:
    """The oracle port (the reference's algorithm restated on the CPU, pinned to the
    reference's own kernels) on `procs` spawned host processes, one thread each, over head
    0 of config 3. Each worker runs the head's preprocess once; a step times a bounded set
    of query blocks per worker. The call is extrapolated: preprocess x heads plus per-unit
    time x all units, spread over the processes."""

    def __init__(self, path, procs):
        import multiprocessing as mp
        from oracle import solattn_oracle as O
        from solb200.workloads import CONFIGS, make_qkv
        self.cfg = CONFIGS["c3"]
        q, k, v = make_qkv(self.cfg, heads=slice(0, 1))
        arrays = tuple(O.to_np(t) for t in (q, k, v))
        self.procs = procs
        self.pool = mp.get_context("spawn").Pool(procs, initializer=_sampler_init,
                                                 initargs=(path, arrays, self.cfg.tau, self.cfg.block))
        self.next_unit = 0

    def step(self, units_per_proc):
        N = self.cfg.blocks
        tasks = []
        for _ in range(self.procs):
            tasks.append([(0, 0, (self.next_unit + i * 37) % N) for i in range(units_per_proc)])
            self.next_unit = (self.next_unit + 11) % N
        t0 = time.perf_counter()
        res = self.pool.map(_sampler_units, tasks)
        wall = time.perf_counter() - t0
        prep = min(r[1] for r in res)
        per_unit = sum(r[0] for r in res) / sum(r[2] for r in res)
        cfg = self.cfg
        units = cfg.batch * cfg.heads * cfg.blocks
        ms = (prep * cfg.batch * cfg.heads + per_unit * units) * 1e3 / self.procs
        return ms, wall

    def info(self, units_per_proc):
        cfg = self.cfg
        return (f"{units_per_proc} query blocks per process per step (of {cfg.blocks} in head 0) plus "
                f"head 0's preprocess (once per process), oracle port, {self.procs} processes x 1 "
                f"thread, extrapolated to {cfg.batch * cfg.heads * cfg.blocks} units and {cfg.heads} heads")

    def close(self):
        self.pool.close()
        self.pool.join()


# --------------------------------------------------------------------- main

# stdout carries exactly one line, the JSON result: everything else written to file
# descriptor 1 (NCCL's version banner, library chatter, stray prints) goes to stderr
_RESULT_FD = None


def _isolate_stdout():
    global _RESULT_FD
    sys.stdout.flush()
    _RESULT_FD = os.dup(1)
    os.dup2(2, 1)


def emit(obj):
    line = (json.dumps(obj) + "\n").encode()
    if _RESULT_FD is None:
        sys.stdout.write(line.decode())
        sys.stdout.flush()
    else:
        os.write(_RESULT_FD, line)


def reference_arm(args, world):
    """The reference's algorithm on the host cores (rank 0 only): per step a bounded
    sample on every core, extrapolated to the config-3 call."""
    from solb200.workloads import CONFIGS
    cfg = CONFIGS["c3"]
    procs = max(1, len(os.sched_getaffinity(0)))
    sampler = CpuSampler(args.path, procs)
    try:
        for _ in range(args.warmup):
            sampler.step(1)
        times = [sampler.step(args.ref_units)[0] for _ in range(args.steps)]
    finally:
        sampler.close()
    ms = statistics.median(times)
    val = cfg.dense_flops() / (ms * 1e-3) / 1e12
    try:   # the dense half of the reference's CPU path: torch CPU SDPA
        dense_cpu = cpu_sdpa_dense()
    except Exception as exc:   # pragma: no cover
        dense_cpu = {"error": str(exc)[:200]}
    emit({
        "impl": "reference", "metric": METRIC, "value": val, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": args.path,
        "data": "synthetic (seeded smooth+noise video-DiT q/k/v, solb200.workloads)",
        "config": bench_config(args.path, world),
        "cpu_baseline": {"value": val, "unit": UNIT, "cores": procs, "kind": "port",
                         "sample": sampler.info(args.ref_units), "dense_sdpa_cpu": dense_cpu},
        "e2e": {"value": val, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    })


def triton_bar(args):
    """The Blackwell bar: the reference's own Triton kernels, JIT-compiled on this B200
    through its public API (``sol_attn``, _tri_fwd.py:354-434; ``sol_attn_int8``,
    _int8_fwd.py:379-458), at config 3 with 128-token blocks (the reference hard-codes
    64-token blocks as module constants; they are reassigned, as for the golden fixtures),
    next to this build's calls on the same tensors. The reference is imported from
    baseline/_ref (git-ignored; absent there, the line says so)."""
    import torch
    import solb200
    from solb200.workloads import CONFIGS, make_qkv
    sys.path.insert(0, str(REPO / "baseline" / "_ref"))
    try:
        import triton
        from solattn_ref import _fused_prep, _int8_fwd, _preprocess, _tri_fwd
    except Exception as exc:
        emit({"triton_reference": {"unavailable": f"reference not importable from baseline/_ref: {exc}"}})
        return
    for mod in (_preprocess, _fused_prep, _tri_fwd, _int8_fwd):
        for name in ("BLOCK", "BLOCK_SIZE"):
            if hasattr(mod, name):
                setattr(mod, name, 128)
    cfg = CONFIGS["c3"]
    dev = torch.device("cuda", 0)
    q, k, v = make_qkv(cfg, device=dev)
    ctx = Timer(torch, None, dev, 1)
    res = {"triton": triton.__version__, "workload": "config3_video480p_B1_H40_T32760_D128_blk128_tau0.9"}
    calls = {
        "reference_bf16": lambda: _tri_fwd.sol_attn(q, k, v, tau=cfg.tau),
        "reference_int8": lambda: _int8_fwd.sol_attn_int8(q, k, v, tau=cfg.tau),
        "ours_bf16": lambda: solb200.sol_attn(q, k, v, tau=cfg.tau, block=128),
        "ours_int8": lambda: solb200.sol_attn_int8(q, k, v, tau=cfg.tau, block=128),
    }
    outs = {}
    for name, fn in calls.items():
        try:
            t0 = time.perf_counter()
            outs[name] = fn()          # the reference's first call autotunes and compiles
            torch.cuda.synchronize()
            first_s = time.perf_counter() - t0
            for _ in range(args.warmup):
                fn()
            res[name] = {"ms_per_call": ctx(fn, args.steps), "first_call_s": first_s}
        except Exception as exc:
            res[name] = {"error": f"{type(exc).__name__}: {exc}"[:400]}
    for p in ("bf16", "int8"):
        a, b = outs.get(f"reference_{p}"), outs.get(f"ours_{p}")
        if a is not None and b is not None:
            x, y = a.float().flatten(), b.float().flatten()
            res[f"ours_vs_reference_{p}"] = {"max_abs": float((x - y).abs().max()),
                                            "cosine": float((x @ y) / (x.norm() * y.norm()))}
    emit({"triton_reference": res})


def h2d_probe(args):
    """The host link the e2e leg runs against: copy-engine rates for one config-3 tensor
    (40 heads x 32760 tokens x 128, bf16, 335 MB) between pinned host memory and the GPU,
    as one 1-D copy and as the head-chunk 2-D copies ``solb200_copy_heads`` issues for
    ``sol_attn_host`` (1, 2, 5 and 40 heads per row), each direction alone and the 2-head
    rows both ways at once (the e2e leg's overlap). One line, then exit."""
    import torch
    from solb200._lib import check, lib
    from solb200.workloads import CONFIGS
    cfg = CONFIGS["c3"]
    B, T, H, D = cfg.batch, cfg.tokens, cfg.heads, cfg.head_dim
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    host_in = torch.randn(B, T, H, D).to(torch.bfloat16).pin_memory()
    host_out = torch.empty_like(host_in).pin_memory()
    dbuf = torch.empty(B, T, H, D, dtype=torch.bfloat16, device=dev)
    dbuf2 = torch.empty_like(dbuf)
    nbytes = host_in.numel() * host_in.element_size()
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    L = lib()

    def chunks(hc, to_device, stream, dst_dev):
        for h0 in range(0, H, hc):
            n = min(hc, H - h0)
            d = dst_dev.data_ptr() + h0 * B * T * D * 2     # chunk slots back to back
            h = (host_in if to_device else host_out).data_ptr()
            check(L.solb200_copy_heads(d, h, B, T, H, D, h0, n, int(to_device), stream.cuda_stream), "copy_heads")

    def rate(fn, streams, moved):
        fn()
        torch.cuda.synchronize()
        best = float("inf")
        for _ in range(max(3, args.steps)):
            t0 = [torch.cuda.Event(enable_timing=True) for _ in streams]
            t1 = [torch.cuda.Event(enable_timing=True) for _ in streams]
            for s, e in zip(streams, t0):
                e.record(s)
            fn()
            for s, e in zip(streams, t1):
                e.record(s)
            torch.cuda.synchronize()
            best = min(best, max(a.elapsed_time(b) for a, b in zip(t0, t1)))
        return {"ms": best, "gbs": moved / (best * 1e-3) / 1e9}

    res = {"tensor_bytes": nbytes, "workload": "config3_video480p_B1_H40_T32760_D128 (one of q/k/v/out)"}
    res["h2d_1d"] = rate(lambda: dbuf.copy_(host_in, non_blocking=True), [torch.cuda.current_stream(dev)], nbytes)
    res["d2h_1d"] = rate(lambda: host_out.copy_(dbuf, non_blocking=True), [torch.cuda.current_stream(dev)], nbytes)
    for hc in (1, 2, 5, 40):
        res[f"h2d_{hc}head_rows"] = rate(lambda: chunks(hc, True, s_in, dbuf), [s_in], nbytes)
    res["d2h_2head_rows"] = rate(lambda: chunks(2, False, s_out, dbuf2), [s_out], nbytes)
    both = rate(lambda: (chunks(2, True, s_in, dbuf), chunks(2, False, s_out, dbuf2)), [s_in, s_out], 2 * nbytes)
    res["both_ways_2head_rows"] = {"ms": both["ms"], "gbs_each_way": both["gbs"] / 2}
    emit({"h2d_probe": res})


def main():
    _isolate_stdout()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--path", choices=["bf16", "int8"], default="bf16")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-dense", action="store_true")
    ap.add_argument("--no-int8", action="store_true", help="skip the INT8 sub-object")
    ap.add_argument("--no-ulysses", action="store_true", help="skip the config-5 sub-object")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-units", type=int, default=48,
                    help="query blocks of the one-core CPU baseline sample")
    ap.add_argument("--ref-units", type=int, default=2,
                    help="query blocks per host process per step of --impl reference")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--e2e-chunk", type=int, default=0,
                    help="heads per streamed chunk in the e2e leg (0 = the API default)")
    ap.add_argument("--heads", type=int, default=0,
                    help="profiling only: run this many of the 40 heads (0 = all)")
    ap.add_argument("--triton-bar", action="store_true",
                    help="time the reference's Triton kernels on this GPU (one line, then exit)")
    ap.add_argument("--h2d-probe", action="store_true",
                    help="time the host link the e2e leg uses (one line, then exit)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.h2d_probe:
        h2d_probe(args)
        return
    if args.triton_bar:
        triton_bar(args)
        return

    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))

    if args.impl == "reference":
        if rank == 0:
            reference_arm(args, world)
        return

    import torch
    import torch.distributed as dist
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    all_cpus = os.sched_getaffinity(0)
    try:
        result = run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            dist.destroy_process_group()
        os.sched_setaffinity(0, all_cpus)   # the CPU legs below use every allowed core
    if rank != 0:
        return
    if not args.no_cpu_baseline and world == 1:
        try:
            sampler = CpuSampler(args.path, 1)
            try:
                ms_cpu, _ = sampler.step(args.cpu_units)
            finally:
                sampler.close()
            from solb200.workloads import CONFIGS
            result["cpu_baseline"] = {
                "value": CONFIGS["c3"].dense_flops() / (ms_cpu * 1e-3) / 1e12, "unit": UNIT,
                "cores": 1, "kind": "port", "sample": sampler.info(args.cpu_units), "ms_per_call": ms_cpu}
            try:
                result["cpu_baseline"]["dense_sdpa_cpu"] = cpu_sdpa_dense()
            except Exception as exc:   # pragma: no cover
                result["cpu_baseline"]["dense_sdpa_cpu"] = {"error": str(exc)[:200]}
        except Exception as exc:   # pragma: no cover
            result["cpu_baseline"] = {"error": str(exc)}
    emit(result)


if __name__ == "__main__":
    main()
