"""Parity of the sm_100a path with the CPU oracle (which is pinned bit-exact to the
reference's own kernels by test_oracle.py).

Bars:
* bit-exact: Morton permutations, pooled keys/values, int8 values and scales,
  thresholds; routing masks except decisions whose routing statistic lies within an
  fp32-rounding margin of the threshold (the reference sums per-row scores, this
  build dots the query-block mean; the two agree to ~1e-6 relative).
* attention outputs: max |diff| <= 2e-2 and cosine >= 0.999 against the oracle's
  BF16 / INT8 outputs and against fp32 SDPA when every block is exact (tau = -1e4).
"""

import numpy as np
import pytest
import torch

from conftest import golden_meta, load_golden
from oracle import solattn_oracle as O

import solb200
from solb200.workloads import CONFIGS, custom_config, make_qkv

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MIN_COS = 0.999
CASES = ["c1", "tiny", "ragged", "d128", "groups"]


def to_dev(*arrs, dtype=torch.bfloat16):
    return [torch.from_numpy(np.ascontiguousarray(a)).to(dtype).cuda() for a in arrs]


def cosine(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-30))


def assert_close_output(got, want, label):
    got = got.float().cpu().numpy() if torch.is_tensor(got) else got
    d = np.abs(got.astype(np.float64) - want.astype(np.float64))
    cos = cosine(got, want)
    assert np.isfinite(got).all(), f"{label}: non-finite output"
    assert d.max() <= MAX_ABS and cos >= MIN_COS, f"{label}: max|d|={d.max():.3e} cos={cos:.6f}"
    return d.max(), cos


def assert_bitexact(got, want, label):
    got = got.float().cpu().numpy() if torch.is_tensor(got) and got.is_floating_point() else (
        got.cpu().numpy() if torch.is_tensor(got) else got)
    want = np.asarray(want)
    assert got.shape == want.shape, f"{label}: shape {got.shape} vs {want.shape}"
    bad = got != want
    assert not bad.any(), f"{label}: {bad.sum()} of {bad.size} differ"


def assert_mask_parity(got_mask, want_mask, stat, thr, label, rel=1e-5):
    """Masks must agree except where the oracle's routing statistic is within an fp32
    rounding margin of the threshold."""
    got = got_mask.cpu().numpy()
    diff = got != want_mask
    if diff.any():
        B, H, N, _ = want_mask.shape
        thr_b = np.transpose(thr, (0, 2, 1))[..., None]          # [B,H,N,1]
        margin = np.abs(stat - thr_b)
        scale = np.abs(thr_b) + np.abs(stat) + 1e-3
        assert (margin[diff] <= rel * scale[diff]).all(), \
            f"{label}: {diff.sum()} routing flips, max margin {margin[diff].max():.3e}"
    return int(diff.sum())


# ------------------------------------------------------------------ Morton

@pytest.mark.parametrize("grid", [(2, 16, 16), (1, 5, 7), (3, 9, 13), (21, 30, 52), (31, 45, 80),
                                  (1, 64, 64), (7, 1, 1)])
@pytest.mark.parametrize("curve", ["3d", "2d_frame"])
def test_morton_perm_bitexact(cuda_device, grid, curve):
    perm, inv = solb200.morton_perm(grid, cuda_device, curve)
    wp, wi = O.morton_perm(grid, curve)
    assert_bitexact(perm, wp, f"perm{grid}{curve}")
    assert_bitexact(inv, wi, f"inverse{grid}{curve}")


@pytest.mark.parametrize("start", [0, 5, 77, 130, 4095])
def test_morton_block_aligned_roll(cuda_device, start):
    perm, inv = solb200.perm_for_span((2, 16, 16), "3d", cuda_device, start)
    wp, wi = O.morton_perm_for_span((2, 16, 16), "3d", start)
    assert_bitexact(perm, wp, "perm")
    assert_bitexact(inv, wi, "inverse")


def test_permute_tokens_roundtrip(cuda_device):
    g = torch.Generator(device="cuda").manual_seed(0)
    q = torch.randn(2, 2 * 16 * 16, 3, 64, device=cuda_device, generator=g).to(torch.bfloat16)
    k = torch.randn_like(q.float()).to(torch.bfloat16)
    perm, inv = solb200.morton_perm((2, 16, 16), cuda_device, "3d")
    pq, pk = solb200.permute_tokens_many([q, k], perm)
    assert torch.equal(pq, q.index_select(1, perm))
    assert torch.equal(pk, k.index_select(1, perm))
    back = solb200.permute_tokens(pq, inv)
    assert torch.equal(back, q)
    x = torch.randn(1, 512, 3 * 64, device=cuda_device).to(torch.bfloat16)   # [B, T, C]
    assert torch.equal(solb200.permute_tokens(x, perm), x.index_select(1, perm))


# ------------------------------------------------------------ preprocessing

def _golden_inputs(name):
    g = load_golden(name)
    B, T, H, D, blk = golden_meta(g)
    q, k, v = to_dev(g["q"], g["k"], g["v"])
    return g, (B, T, H, D, blk), (q, k, v)


@pytest.mark.parametrize("name", CASES)
def test_prepare_bitexact(cuda_device, name):
    g, (B, T, H, D, blk), (q, k, v) = _golden_inputs(name)
    tau = float(g["tau"])
    kc, vc, thr = solb200.prepare(q, k, v, tau=tau, scale=D ** -0.5, block=blk)
    wkc, wvc, wthr = O.prepare(g["q"], g["k"], g["v"], tau, D ** -0.5, T, blk)
    assert_bitexact(kc, wkc, "kc")
    assert_bitexact(vc, wvc, "vc")
    assert_bitexact(thr, wthr, "thr")
    if B == 1:   # and equal to the reference's own values
        assert_bitexact(kc, g["kc"], "kc vs reference")
        assert_bitexact(thr, g["thr"], "thr vs reference")


@pytest.mark.parametrize("name", CASES)
@pytest.mark.parametrize("int8_pv", [True, False])
def test_fused_preprocess_bitexact(cuda_device, name, int8_pv):
    g, (B, T, H, D, blk), (q, k, v) = _golden_inputs(name)
    tau = float(g["tau"])
    got = solb200.fused_preprocess(q, k, v, tau=tau, scale=D ** -0.5, int8_pv=int8_pv, block=blk)
    want = O.fused_preprocess(g["q"], g["k"], g["v"], tau, D ** -0.5, T, blk, int8_pv=int8_pv)
    names = ["kc", "vc", "thr", "qi", "qs", "ki", "ks", "vi", "vsc"]
    for nm, val in zip(names, got):
        if val is None:
            assert want[nm] is None
            continue
        w = want[nm]
        if nm == "vsc":
            w = w.reshape(-1, D)
        assert_bitexact(val, w, nm)
    if B == 1 and int8_pv:
        assert_bitexact(got[3], g["i8_qi"][:, :T], "qi vs reference")
        assert_bitexact(got[5], g["i8_ki"][:, :T], "ki vs reference")
        assert_bitexact(got[6], g["i8_ks"][:, :T], "ks vs reference")


@pytest.mark.parametrize("B,T,H,D", [(2, 1000, 5, 128), (1, 777, 3, 64), (3, 300, 7, 128)])
def test_quantiser_layouts_bitexact(cuda_device, B, T, H, D):
    """The Q/K/V quantiser's persistent stripes for head counts whose lanes do not fill a
    warp per token (warps spanning two tokens), batches > 1 (the row cursor crossing a
    batch) and ragged token counts: every code and scale equals the oracle's."""
    gen = torch.Generator().manual_seed(B * 1000 + T + H)
    q, k, v = ((torch.randn(B, T, H, D, generator=gen) * s).to(torch.bfloat16) for s in (1.0, 0.7, 1.3))
    blk = 64
    got = solb200.fused_preprocess(q.cuda(), k.cuda(), v.cuda(), tau=0.9, scale=D ** -0.5, int8_pv=True, block=blk)
    want = O.fused_preprocess(*(O.to_np(t) for t in (q, k, v)), 0.9, D ** -0.5, T, blk, int8_pv=True)
    for nm, val in zip(["kc", "vc", "thr", "qi", "qs", "ki", "ks", "vi", "vsc"], got):
        w = want[nm]
        if nm == "vsc":
            w = w.reshape(-1, D)
        assert_bitexact(val, w, f"{nm} B={B} T={T} H={H} D={D}")


@pytest.mark.parametrize("name", CASES)
@pytest.mark.parametrize("int8", [False, True])
def test_routing_mask_parity(cuda_device, name, int8):
    g, (B, T, H, D, blk), (q, k, v) = _golden_inputs(name)
    tau = float(g["tau"])
    r = solb200.routing(q, k, v, tau=tau, block=blk, int8=int8)
    if int8:
        parts = O.fused_preprocess(g["q"], g["k"], g["v"], tau, D ** -0.5, T, blk)
        kc, thr = parts["kc"], parts["thr"]
    else:
        kc, _, thr = O.prepare(g["q"], g["k"], g["v"], tau, D ** -0.5, T, blk)
    want, stat = O.route_mask(g["q"], kc, thr, D ** -0.5, T, blk)
    flips = assert_mask_parity(r["mask"], want, stat, thr, f"{name} int8={int8}")
    assert flips == 0, f"{flips} margin-level flips on a small fixture"
    # routing statistic itself agrees with the oracle's to fp32 rounding
    s = r["stat"].cpu().numpy()
    assert np.abs(s - stat).max() <= 1e-4 * (1 + np.abs(stat).max())
    # lists are the mask, ascending, -1 padded; counts are the row popcounts
    lists = r["lists"].cpu().numpy()
    counts = r["counts"].cpu().numpy()
    N = want.shape[-1]
    for b in range(B):
        for h in range(H):
            for n in range(N):
                idx = np.nonzero(r["mask"][b, h, n].cpu().numpy())[0]
                assert counts[b, h, n] == len(idx)
                assert (lists[b, h, n, :len(idx)] == idx).all()
                assert (lists[b, h, n, len(idx):] == -1).all()


def test_routing_sinks(cuda_device):
    g, (B, T, H, D, blk), (q, k, v) = _golden_inputs("c1")
    r = solb200.routing(q, k, v, tau=0.9, block=blk, sink_blocks=(0, 2), sink_q=(3, 5))
    m = r["mask"].cpu().numpy()
    assert m[:, :, :, 0:2].all()            # sink KV blocks exact for every query block
    assert m[:, :, 3:5, :].all()            # sink query blocks attend everything
    kc, _, thr = O.prepare(g["q"], g["k"], g["v"], 0.9, D ** -0.5, T, blk)
    want, stat = O.route_mask(g["q"], kc, thr, D ** -0.5, T, blk, (0, 2), (3, 5))
    assert assert_mask_parity(r["mask"], want, stat, thr, "sinks") == 0


# ----------------------------------------------------------------- forward

@pytest.mark.parametrize("name", CASES)
def test_sol_attn_bf16(cuda_device, name):
    g, (B, T, H, D, blk), (q, k, v) = _golden_inputs(name)
    tau = float(g["tau"])
    out = solb200.sol_attn(q, k, v, tau=tau, block=blk)
    want = O.sol_attn(g["q"], g["k"], g["v"], tau=tau, block=blk)
    assert out.shape == (B, T, H, D) and out.dtype == torch.bfloat16
    assert_close_output(out, want, f"bf16 {name}")
    if B == 1:
        assert_close_output(out, g["o_bf16"], f"bf16 {name} vs reference")


@pytest.mark.parametrize("name", CASES)
@pytest.mark.parametrize("int8_pv", [True, False])
def test_sol_attn_int8(cuda_device, name, int8_pv):
    g, (B, T, H, D, blk), (q, k, v) = _golden_inputs(name)
    tau = float(g["tau"])
    out = solb200.sol_attn_int8(q, k, v, tau=tau, block=blk, int8_pv=int8_pv)
    want = O.sol_attn_int8(g["q"], g["k"], g["v"], tau=tau, block=blk, int8_pv=int8_pv)
    assert_close_output(out, want, f"int8 {name} pv={int8_pv}")
    if B == 1:
        key = "o_int8" if int8_pv else "o_int8_nopv"
        assert_close_output(out, g[key], f"int8 {name} vs reference")


@pytest.mark.parametrize("name", ["c1", "tiny", "ragged", "d128"])
def test_dense_limit_matches_sdpa(cuda_device, name):
    g, (B, T, H, D, blk), (q, k, v) = _golden_inputs(name)
    ref = O.dense_reference(g["q"], g["k"], g["v"])
    out = solb200.sol_attn(q, k, v, tau=-1.0e4, block=blk)
    assert_close_output(out, ref, "bf16 dense")
    out8 = solb200.sol_attn_int8(q, k, v, tau=-1.0e4, block=blk)
    assert_close_output(out8, ref, "int8 dense")


@pytest.mark.parametrize("sink", [((0, 2), (0, 1)), ((1, 3), (0, 0)), ((0, 0), (0, 8))])
def test_sinks_forward(cuda_device, sink):
    g, (B, T, H, D, blk), (q, k, v) = _golden_inputs("c1")
    sk, sq = sink
    out = solb200.sol_attn(q, k, v, tau=0.9, block=blk, sink_blocks=sk, sink_q=sq)
    want = O.sol_attn(g["q"], g["k"], g["v"], tau=0.9, block=blk, sink_blocks=sk, sink_q=sq)
    assert_close_output(out, want, "bf16 sink")
    out8 = solb200.sol_attn_int8(q, k, v, tau=0.9, block=blk, sink_blocks=sk, sink_q=sq)
    want8 = O.sol_attn_int8(g["q"], g["k"], g["v"], tau=0.9, block=blk, sink_blocks=sk, sink_q=sq)
    assert_close_output(out8, want8, "int8 sink")


def test_strided_inputs(cuda_device):
    """BHND tensors transposed to BTHD views, and q/k/v slices of one packed qkv
    buffer, give the same result as contiguous copies."""
    g, (B, T, H, D, blk), (q, k, v) = _golden_inputs("c1")
    ref = solb200.sol_attn(q, k, v, tau=0.9, block=blk)
    bhnd = [t.transpose(1, 2).contiguous().transpose(1, 2) for t in (q, k, v)]
    assert not bhnd[0].is_contiguous()
    assert torch.equal(solb200.sol_attn(*bhnd, tau=0.9, block=blk), ref)
    qkv = torch.stack([q, k, v], dim=3)            # [B, T, H, 3, D] interleaved
    views = [qkv[:, :, :, i] for i in range(3)]
    assert torch.equal(solb200.sol_attn(*views, tau=0.9, block=blk), ref)


@pytest.mark.parametrize("cfg_name", ["c2"])
def test_config2_full(cuda_device, cfg_name):
    cfg = CONFIGS[cfg_name]
    q, k, v = make_qkv(cfg)
    qn, kn, vn = (O.to_np(t) for t in (q, k, v))
    qd, kd, vd = (t.cuda() for t in (q, k, v))
    out = solb200.sol_attn(qd, kd, vd, tau=cfg.tau, block=cfg.block)
    want = O.sol_attn(qn, kn, vn, tau=cfg.tau, block=cfg.block)
    assert_close_output(out, want, "config 2 bf16")
    r = solb200.routing(qd, kd, vd, tau=cfg.tau, block=cfg.block)
    kc, _, thr = O.prepare(qn, kn, vn, cfg.tau, 128 ** -0.5, cfg.tokens, cfg.block)
    wmask, stat = O.route_mask(qn, kc, thr, 128 ** -0.5, cfg.tokens, cfg.block)
    flips = assert_mask_parity(r["mask"], wmask, stat, thr, "config 2")
    assert flips <= 2


def test_config3_head_slice(cuda_device):
    """The headline shape (T = 32760, blk 128) on two heads of the seeded tensors."""
    cfg = CONFIGS["c3"]
    q, k, v = make_qkv(cfg, heads=slice(0, 2))
    qn, kn, vn = (O.to_np(t) for t in (q, k, v))
    qd, kd, vd = (t.cuda() for t in (q, k, v))
    out = solb200.sol_attn(qd, kd, vd, tau=cfg.tau, block=cfg.block)
    units = [(0, h, n) for h in range(2) for n in range(0, cfg.blocks, 17)]
    want = O.sol_attn(qn, kn, vn, tau=cfg.tau, block=cfg.block, units=units)
    rows = np.concatenate([np.arange(n * 128, min(cfg.tokens, n * 128 + 128))
                           for n in range(0, cfg.blocks, 17)])
    assert_close_output(out.float().cpu().numpy()[:, rows], want[:, rows], "config 3 slice")
    for pv in (True, False):
        out8 = solb200.sol_attn_int8(qd, kd, vd, tau=cfg.tau, block=cfg.block, int8_pv=pv)
        want8 = O.sol_attn_int8(qn, kn, vn, tau=cfg.tau, block=cfg.block, int8_pv=pv, units=units)
        assert_close_output(out8.float().cpu().numpy()[:, rows], want8[:, rows], f"config 3 slice int8 pv={pv}")
    kc, vc, thr = solb200.prepare(qd, kd, vd, tau=cfg.tau, scale=128 ** -0.5, block=cfg.block)
    wkc, wvc, wthr = O.prepare(qn, kn, vn, cfg.tau, 128 ** -0.5, cfg.tokens, cfg.block)
    assert_bitexact(kc, wkc, "kc")
    assert_bitexact(vc, wvc, "vc")
    assert_bitexact(thr, wthr, "thr")


def test_bad_arguments_raise(cuda_device):
    q = torch.zeros(1, 256, 2, 96, dtype=torch.bfloat16, device=cuda_device)
    with pytest.raises(RuntimeError, match="head_dim"):
        solb200.sol_attn(q, q, q)
    q = torch.zeros(1, 256, 2, 64, dtype=torch.float16, device=cuda_device)
    with pytest.raises(RuntimeError, match="bfloat16"):
        solb200.sol_attn(q, q, q)


def _slice_inputs(cfg_name, heads):
    """One or two heads of a config's seeded tensors, drawn on the GPU (the full draw
    of the long configs is slow on the host), plus host copies for the oracle."""
    cfg = CONFIGS[cfg_name]
    qd, kd, vd = make_qkv(cfg, device="cuda", heads=heads)
    qd, kd, vd = (t.contiguous() for t in (qd, kd, vd))
    qn, kn, vn = (O.to_np(t.cpu()) for t in (qd, kd, vd))
    return cfg, (qd, kd, vd), (qn, kn, vn)


def _sampled(cfg, step, nheads):
    units = [(0, h, n) for h in range(nheads) for n in range(0, cfg.blocks, step)]
    rows = np.concatenate([np.arange(n * cfg.block, min(cfg.tokens, n * cfg.block + cfg.block))
                           for n in range(0, cfg.blocks, step)])
    return units, rows


@pytest.mark.parametrize("tau", [0.8, 0.9, 0.95])
def test_config4_int8_head_slice(cuda_device, tau):
    """Config 4 (720p, T = 75600, INT8 at the three taus of the config) on one head:
    forward on sampled query blocks and the full routing mask against the oracle."""
    cfg, (qd, kd, vd), (qn, kn, vn) = _slice_inputs("c4", slice(3, 4))
    units, rows = _sampled(cfg, 41, 1)
    out8 = solb200.sol_attn_int8(qd, kd, vd, tau=tau, block=cfg.block)
    want8 = O.sol_attn_int8(qn, kn, vn, tau=tau, block=cfg.block, units=units)
    assert_close_output(out8.float().cpu().numpy()[:, rows], want8[:, rows], f"config 4 int8 tau={tau}")
    r = solb200.routing(qd, kd, vd, tau=tau, block=cfg.block, int8=True)
    parts = O.fused_preprocess(qn, kn, vn, tau, 128 ** -0.5, cfg.tokens, cfg.block)
    want, stat = O.route_mask(qn, parts["kc"], parts["thr"], 128 ** -0.5, cfg.tokens, cfg.block)
    flips = assert_mask_parity(r["mask"], want, stat, parts["thr"], f"config 4 tau={tau}")
    assert flips <= 2


def test_config5_head_slice(cuda_device):
    """Config 5 (T = 111600, N = 872 blocks) on one head, BF16 and INT8, sampled query
    blocks against the oracle."""
    cfg, (qd, kd, vd), (qn, kn, vn) = _slice_inputs("c5", slice(7, 8))
    units, rows = _sampled(cfg, 67, 1)
    out = solb200.sol_attn(qd, kd, vd, tau=cfg.tau, block=cfg.block)
    want = O.sol_attn(qn, kn, vn, tau=cfg.tau, block=cfg.block, units=units)
    assert_close_output(out.float().cpu().numpy()[:, rows], want[:, rows], "config 5 bf16")
    out8 = solb200.sol_attn_int8(qd, kd, vd, tau=cfg.tau, block=cfg.block)
    want8 = O.sol_attn_int8(qn, kn, vn, tau=cfg.tau, block=cfg.block, units=units)
    assert_close_output(out8.float().cpu().numpy()[:, rows], want8[:, rows], "config 5 int8")


def test_forward_schedule(cuda_device):
    """The forward's unit schedule: head by head, each head's query blocks once, by
    non-increasing exact-block count."""
    from solb200.ops import STAGES_PREPARE, _attn
    g, (B, T, H, D, blk), (q, k, v) = _golden_inputs("groups")
    _, ws, _, _ = _attn(q, k, v, scale=None, tau=0.5, sink_blocks=(0, 0), sink_q=(0, 0), block=blk,
                        int8=False, int8_pv=False, stages=STAGES_PREPARE)
    N = ws.N
    order = ws.view("order", torch.int32, (B * H * N,)).cpu().numpy()
    counts = ws.view("count", torch.int32, (B * H * N,)).cpu().numpy()
    for bh in range(B * H):
        seg = order[bh * N:(bh + 1) * N]
        assert sorted(seg.tolist()) == list(range(bh * N, (bh + 1) * N))
        c = counts[seg]
        assert (np.diff(c) <= 0).all(), "query blocks not by descending count"
    assert counts.min() < counts.max(), "fixture should have uneven counts"


@pytest.mark.parametrize("int8", [False, True])
def test_stage_parts_equal_one_call(cuda_device, int8):
    """POOL, QUANT (INT8), ROUTE and FORWARD run as separate C-ABI calls on one workspace
    produce the one-call output bit for bit (the per-stage timing of the bench uses them)."""
    from solb200._lib import (STAGES_ALL, STAGES_FORWARD, STAGES_POOL, STAGES_QUANT, STAGES_ROUTE, I64x2, I64x3,
                              check, lib)
    from solb200.ops import Workspace
    g = torch.Generator().manual_seed(21)
    B, T, H, D, blk = 1, 3000, 3, 128, 128
    q, k, v = (torch.randn(B, T, H, D, generator=g).to(torch.bfloat16).cuda() for _ in range(3))
    st = torch.cuda.current_stream().cuda_stream

    def run(stages_list):
        ws = Workspace(B, T, H, D, blk, int8, q.device)
        out = torch.zeros_like(q)
        for stages in stages_list:
            a = [q.data_ptr(), I64x3(*q.stride()[:3]), k.data_ptr(), I64x3(*k.stride()[:3]), v.data_ptr(),
                 I64x3(*v.stride()[:3]), out.data_ptr(), B, T, H, D, blk, D ** -0.5, 0.9, I64x2(0, 0), I64x2(0, 0)]
            tail = [stages, ws.ptr(), ws.nbytes, None, None, st]
            rc = lib().solb200_sol_attn_int8(*a, 1, *tail) if int8 else lib().solb200_sol_attn_bf16(*a, *tail)
            check(rc, f"stages {stages}")
        ws.check_device_error()
        return out

    whole = run([STAGES_ALL])
    parts = run([STAGES_POOL] + ([STAGES_QUANT] if int8 else []) + [STAGES_ROUTE, STAGES_FORWARD])
    assert torch.equal(whole, parts)
    ws = Workspace(B, T, H, D, blk, int8, q.device)
    a = [q.data_ptr(), I64x3(*q.stride()[:3]), k.data_ptr(), I64x3(*k.stride()[:3]), v.data_ptr(),
         I64x3(*v.stride()[:3]), whole.data_ptr(), B, T, H, D, blk, D ** -0.5, 0.9, I64x2(0, 0), I64x2(0, 0)]
    assert lib().solb200_sol_attn_bf16(*a, 6, ws.ptr(), ws.nbytes, None, None, st) == 1   # unknown stage: invalid
