"""Benchmark of the Sol-Attn hot path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--path bf16|int8] [--impl ours|reference]

Workload: the headline configuration (config 3): B=1, H=40, T=21x30x52=32760 tokens,
D=128, block 128, tau=0.9, seeded synthetic video-DiT q/k/v (solb200.workloads).
A step is one attention call through the C ABI: pooling, routing, the block-sparse
forward. value = dense-equivalent TFLOP/s of the whole job (4*B*H*T^2*D / time).
With N GPUs (torchrun) the 40 heads are split across ranks (H/N each, no
collective); time is the max over ranks.

--impl reference times the reference's algorithm on the host cores instead: the CPU
oracle port (oracle/solattn_oracle.py, a step-for-step restatement of the reference's
kernels, pinned bit-exact to them) on a bounded sample of query blocks, extrapolated
to the full call.
"""

from __future__ import annotations

import argparse
import json
import math
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


# ------------------------------------------------------------------ our arm

def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    import solb200
    from solb200 import _lib
    from solb200.ops import STAGES_ALL, STAGES_PREPARE, I64x2, I64x3, Workspace
    from solb200._lib import STAGES_FORWARD
    from solb200.workloads import CONFIGS, make_qkv

    cfg = CONFIGS["c3"]
    if args.heads:
        import dataclasses
        cfg = dataclasses.replace(cfg, heads=args.heads)
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    B, T, Hall, D, blk = cfg.batch, cfg.tokens, cfg.heads, cfg.head_dim, cfg.block
    if Hall % world:
        raise SystemExit(f"{Hall} heads do not split over {world} ranks")
    H = Hall // world
    h0 = rank * H
    # seeded inputs generated on the device; each rank keeps its head slice
    q, k, v = make_qkv(cfg, device=dev, heads=slice(h0, h0 + H))
    torch.cuda.synchronize()
    int8 = args.path == "int8"
    lib = _lib.lib()
    ws = Workspace(B, T, H, D, blk, int8, dev)
    out = torch.empty((B, T, H, D), dtype=torch.bfloat16, device=dev)
    stream = torch.cuda.current_stream(dev)
    sk, sq = I64x2(0, 0), I64x2(0, 0)
    scale = D ** -0.5

    def call(stages, qq=q, kk=k, vv=v, oo=out):
        a = [qq.data_ptr(), I64x3(*qq.stride()[:3]), kk.data_ptr(), I64x3(*kk.stride()[:3]),
             vv.data_ptr(), I64x3(*vv.stride()[:3]), oo.data_ptr(), B, T, H, D, blk, scale,
             cfg.tau, sk, sq]
        tail = [stages, ws.ptr(), ws.nbytes, None, None, stream.cuda_stream]
        rc = lib.solb200_sol_attn_int8(*a, 1, *tail) if int8 else lib.solb200_sol_attn_bf16(*a, *tail)
        _lib.check(rc, "bench call")

    # L2 is flushed before every timed step (a write larger than L2, outside the step's
    # event pair): a rank's inputs are not larger than L2 at every head count
    # (5 heads x 32760 tokens: 3 x 42 MB)
    l2_bytes = int(getattr(torch.cuda.get_device_properties(dev), "L2_cache_size", 0) or (126 << 20))
    flush_buf = torch.empty(max(2 * l2_bytes, 256 << 20) // 4, dtype=torch.float32, device=dev)

    def timed(fn, steps):
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(steps)]
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        for ev0, ev1 in evs:
            flush_buf.zero_()
            ev0.record(stream)
            fn()
            ev1.record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        ms = sum(ev0.elapsed_time(ev1) for ev0, ev1 in evs) / steps
        t = torch.tensor([ms], device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        call(STAGES_ALL)
    ws.check_device_error()
    with Clocks(local_rank) as clk:
        ms = timed(lambda: call(STAGES_ALL), args.steps)
    ws.check_device_error()
    clocks = clk.result
    # stage split (same stream, same inputs): preprocess + routing alone, then the
    # forward kernel alone over the workspace the last call left (CUDA events on the
    # stream the kernels are launched on)
    for _ in range(2):
        call(STAGES_PREPARE)
    ms_prep = timed(lambda: call(STAGES_PREPARE), args.steps)
    for _ in range(2):
        call(STAGES_FORWARD)
    ms_fwd = timed(lambda: call(STAGES_FORWARD), args.steps)
    ws.check_device_error()

    # executed (algorithmic) flops of the forward from the routing of this input
    counts = ws.view("count", torch.int32, (B, H, ws.N)).long()
    words = ws.view("mask", torch.int32, (B, H, ws.N, ws.nw))
    tail = T - (ws.N - 1) * blk
    # exact pairs: every routed block is blk x blk except those touching the tail
    n_pairs = int(counts.sum())
    bits = torch.arange(32, device=dev, dtype=torch.int32)
    mask = ((words.unsqueeze(-1) >> bits) & 1).reshape(B, H, ws.N, -1)[..., :ws.N]
    last_col = int(mask[..., ws.N - 1].sum())        # routed pairs whose key block is the tail
    last_row = int(mask[:, :, ws.N - 1, :].sum())    # routed pairs whose query block is the tail
    corner = int(mask[:, :, ws.N - 1, ws.N - 1].sum())
    tok_pairs = (n_pairs * blk * blk - last_col * blk * (blk - tail) - last_row * blk * (blk - tail)
                 + corner * (blk - tail) ** 2)
    exact_flops = 4.0 * D * tok_pairs
    approx_flops = 4.0 * D * B * H * T * ws.N
    density = n_pairs / float(B * H * ws.N * ws.N)
    fwd_flops = exact_flops + approx_flops
    dense_job = cfg.dense_flops()

    # e2e through the public API for host-resident tensors: pinned host q/k/v ->
    # solb200.sol_attn_host (head chunks streamed H2D / computed / streamed D2H on
    # three streams) -> pinned host output
    hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
    hout = torch.empty((B, T, H, D), dtype=torch.bfloat16).pin_memory()

    def e2e_step():
        solb200.sol_attn_host(hq, hk, hv, tau=cfg.tau, block=blk, int8=int8, out=hout,
                              heads_per_chunk=args.e2e_chunk or None, synchronize=False)

    ms_e2e = None
    if not args.no_e2e:
        for _ in range(2):
            e2e_step()
        ms_e2e = timed(e2e_step, max(2, min(args.steps, 5)))
    h2d = sum(t.numel() * t.element_size() for t in (hq, hk, hv))
    d2h = hout.numel() * hout.element_size()

    # Morton reorder stage: q, k, v into Z-order and O back (one gather launch each way)
    perm, inv = solb200.morton_perm(cfg.grid, dev, "3d")
    ms_reorder = timed(lambda: (solb200.permute_tokens_many([q, k, v], perm),
                                solb200.permute_tokens(out, inv)), 3)

    # dense reference on the same GPU (torch SDPA, bf16): the "< 30% of dense" target
    ms_dense = None
    if not args.no_dense:
        try:
            qt, kt, vt = (t.transpose(1, 2) for t in (q, k, v))
            sdpa = torch.nn.functional.scaled_dot_product_attention
            for _ in range(2):
                sdpa(qt, kt, vt)
            ms_dense = timed(lambda: sdpa(qt, kt, vt), 3)
        except Exception as exc:   # pragma: no cover - informational only
            ms_dense = f"failed: {exc}"

    # Morton (both curves): reorder cost, routed density and accuracy against dense SDPA,
    # next to the unpermuted call (one GPU only; needs the dense output)
    morton = None
    if world == 1 and isinstance(ms_dense, float):
        fn = solb200.sol_attn_int8 if int8 else solb200.sol_attn
        dense_out = sdpa(qt, kt, vt).transpose(1, 2)

        def vs_dense(o):
            a, b = o.float().flatten(), dense_out.float().flatten()
            return {"max_abs": float((a - b).abs().max()),
                    "cosine": float((a @ b) / (a.norm() * b.norm()))}

        morton = {"none": {"routed_density": density, "vs_dense": vs_dense(fn(q, k, v, tau=cfg.tau, block=blk))}}
        for curve in ("3d", "2d_frame"):
            pm, ivm = solb200.morton_perm(cfg.grid, dev, curve)
            ms_r = timed(lambda: (solb200.permute_tokens_many([q, k, v], pm),
                                  solb200.permute_tokens(out, ivm)), 3)
            qp, kp, vp = solb200.permute_tokens_many([q, k, v], pm)
            r = solb200.routing(qp, kp, vp, tau=cfg.tau, block=blk, int8=int8)
            om = solb200.permute_tokens(fn(qp, kp, vp, tau=cfg.tau, block=blk), ivm)
            morton[curve] = {"reorder_ms": ms_r, "routed_density": float(r["mask"].float().mean()),
                             "vs_dense": vs_dense(om)}
            del qp, kp, vp, r, om
        del dense_out

    peaks = load_peaks()
    achieved = fwd_flops / (ms_fwd * 1e-3) / 1e12
    result = {
        "metric": METRIC,
        "value": dense_job / (ms * 1e-3) / 1e12,
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "int8" if int8 else "bf16",
        "data": "synthetic (seeded smooth+noise video-DiT q/k/v, solb200.workloads)",
        "config": {"workload": "config3_video480p_B1_H%d_T32760_D128_blk128_tau0.9" % cfg.heads,
                   "path": args.path, "heads_per_rank": H, "parallelism": f"heads/{world}",
                   "l2": "L2 flushed before every timed step (%d MB write, outside the step's "
                         "CUDA-event pair)" % (flush_buf.numel() * 4 >> 20),
                   "routed_density": density},
        "stages_ms": {"prep_route": ms_prep, "forward": ms_fwd, "reorder_qkv_and_o": ms_reorder},
        "dense_sdpa_ms": ms_dense,
        "morton": morton,
        "sparse_over_dense": (ms / ms_dense) if isinstance(ms_dense, float) else None,
        "roofline": {"bound": "tensor", "kernel": "sol_fwd_%s_kernel" % ("int8" if int8 else "bf16"),
                     "achieved": achieved, "peak": peaks["bf16"], "unit": "TFLOP/s",
                     "frac": achieved / peaks["bf16"],
                     "traffic": profiled_traffic("int8" if int8 else "bf16", H),
                     "note": f"executed flops {fwd_flops:.4g} per launch / forward kernel time; "
                             f"peak = bf16 dense burst, {peaks['source']}; traffic = DRAM bytes "
                             f"per launch from the ncu capture in profiles/, scaled to {H} heads"},
        "e2e": ({"value": dense_job / (ms_e2e * 1e-3) / 1e12, "unit": UNIT, "ms_per_step": ms_e2e,
                 "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": d2h * world,
                 "api": "solb200.sol_attn_host (pinned host in and out, head chunks streamed)"}
                if ms_e2e else None),
        # per step: pool, moments, route, order, forward (+ quant_kv on the INT8 path)
        "gpu_launches": (5 + (1 if int8 else 0)) * args.steps,
        "clocks": clocks,
    }
    return result


# ------------------------------------------------------------- CPU baseline

def _oracle_sample_worker(task):
    """Time the oracle on some query blocks of one head (runs in a spawned process):
    (seconds of the whole-head preprocess, seconds of the units' forward, units)."""
    import threadpoolctl
    from oracle import solattn_oracle as O
    from solb200.workloads import CONFIGS

    path, units, (qn, kn, vn) = task
    cfg = CONFIGS["c3"]
    with threadpoolctl.threadpool_limits(1):
        t0 = time.perf_counter()
        if path == "int8":
            O.fused_preprocess(qn, kn, vn, cfg.tau, cfg.head_dim ** -0.5, cfg.tokens, cfg.block)
        else:
            O.prepare(qn, kn, vn, cfg.tau, cfg.head_dim ** -0.5, cfg.tokens, cfg.block)
        t1 = time.perf_counter()
        fn = O.sol_attn_int8 if path == "int8" else O.sol_attn
        fn(qn, kn, vn, tau=cfg.tau, block=cfg.block, units=[(0, 0, n) for n in units])
        t2 = time.perf_counter()
    # the forward call repeats the preprocess internally: subtract it
    return t1 - t0, max(t2 - t1 - (t1 - t0), 1e-9), len(units)


def cpu_baseline(path, procs, budget_units):
    """The oracle port on `procs` host processes over a bounded sample of query blocks
    of one head of config 3, extrapolated to the whole call (all B*H*N units plus the
    per-head preprocess), with the processes working in parallel. Returns
    (ms per call, info)."""
    import multiprocessing as mp
    from oracle import solattn_oracle as O
    from solb200.workloads import CONFIGS, make_qkv

    cfg = CONFIGS["c3"]
    N = cfg.blocks
    stride = max(1, N // budget_units)
    units = list(range(0, N, stride))[:budget_units]
    q, k, v = make_qkv(cfg, heads=slice(0, 1))
    arrays = tuple(O.to_np(t) for t in (q, k, v))
    chunks = [c for c in (units[i::procs] for i in range(procs)) if c]
    ctx = mp.get_context("spawn")
    t0 = time.perf_counter()
    with ctx.Pool(len(chunks)) as pool:
        res = pool.map(_oracle_sample_worker, [(path, c, arrays) for c in chunks])
    wall = time.perf_counter() - t0
    prep = min(r[0] for r in res)
    per_unit = sum(r[1] for r in res) / sum(r[2] for r in res)
    total_units = cfg.batch * cfg.heads * N
    core_ms = (prep * cfg.batch * cfg.heads + per_unit * total_units) * 1e3
    return core_ms / len(chunks), {
        "sample": f"{sum(r[2] for r in res)} of {N} query blocks of head 0 (every {stride}th) "
                  f"plus head 0's preprocess, oracle {path} port, extrapolated to "
                  f"{total_units} units and {cfg.heads} heads",
        "cores": len(chunks), "sample_wall_s": wall}


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


def main():
    _isolate_stdout()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--path", choices=["bf16", "int8"], default="bf16")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-dense", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-units", type=int, default=64)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--e2e-chunk", type=int, default=0,
                    help="heads per streamed chunk in the e2e leg (0 = the API default)")
    ap.add_argument("--heads", type=int, default=0,
                    help="profiling only: run this many of the 40 heads (0 = all)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))

    if args.impl == "reference":
        if rank != 0:
            return
        from solb200.workloads import CONFIGS
        cfg = CONFIGS["c3"]
        procs = max(1, len(os.sched_getaffinity(0)))
        times = []
        for _ in range(args.steps):
            ms, info = cpu_baseline(args.path, procs, max(8, args.cpu_units // 4))
            times.append(ms)
        ms = statistics.median(times)
        val = cfg.dense_flops() / (ms * 1e-3) / 1e12
        emit({
            "impl": "reference", "metric": METRIC, "value": val, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": args.path,
            "data": "synthetic (seeded, solb200.workloads)",
            "config": {"workload": "config3_video480p_B1_H40_T32760_D128_blk128_tau0.9",
                       "path": args.path},
            "cpu_baseline": {"value": val, "unit": UNIT, "cores": info["cores"], "kind": "port",
                             "sample": info["sample"]},
            "e2e": {"value": val, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        })
        return

    import torch
    import torch.distributed as dist
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        result = run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            dist.destroy_process_group()
    if rank != 0:
        return
    if not args.no_cpu_baseline:
        try:
            ms_cpu, info = cpu_baseline(args.path, 1, args.cpu_units)
            from solb200.workloads import CONFIGS
            result["cpu_baseline"] = {
                "value": CONFIGS["c3"].dense_flops() / (ms_cpu * 1e-3) / 1e12, "unit": UNIT,
                "cores": info["cores"], "kind": "port", "sample": info["sample"],
                "ms_per_call": ms_cpu}
        except Exception as exc:   # pragma: no cover
            result["cpu_baseline"] = {"error": str(exc)}
    emit(result)


if __name__ == "__main__":
    main()
