"""The CPU oracle against the reference's own kernels.

The fixtures in ``tests/golden`` were produced by ``tests/golden/make_golden.py``,
which runs the reference's Triton kernels on CPU (TRITON_INTERPRET=1 with four
documented shims). Every comparison here is bit-exact: the oracle restates the
reference with the same numpy/torch operations in the same order.
"""

import numpy as np
import pytest

from conftest import golden_meta, load_golden
from oracle import solattn_oracle as O

CASES = ["c1", "tiny", "ragged", "d128", "groups"]


def _eq(a, b):
    a, b = np.asarray(a), np.asarray(b)
    assert a.shape == b.shape, (a.shape, b.shape)
    bad = ~((a == b) | (np.isnan(a.astype(np.float64)) & np.isnan(b.astype(np.float64))))
    assert not bad.any(), f"{bad.sum()} of {a.size} differ, max |d| = " \
        f"{np.abs(a.astype(np.float64) - b.astype(np.float64))[bad].max()}"


@pytest.mark.parametrize("name", CASES)
def test_bf16_path_bitexact(name):
    g = load_golden(name)
    B, T, H, D, blk = golden_meta(g)
    stride_bug = B > 1
    o, parts = O.sol_attn(g["q"], g["k"], g["v"], tau=float(g["tau"]), block=blk,
                          return_parts=True, reference_batch_stride=stride_bug)
    _eq(parts["kc"], g["kc"])
    _eq(parts["vc"], g["vc"])
    _eq(parts["thr"], g["thr"])
    _eq(o, g["o_bf16"])


@pytest.mark.parametrize("name", CASES)
def test_int8_path_bitexact(name):
    g = load_golden(name)
    B, T, H, D, blk = golden_meta(g)
    o, p = O.sol_attn_int8(g["q"], g["k"], g["v"], tau=float(g["tau"]), block=blk,
                           return_parts=True, reference_batch_stride=B > 1)
    for n in ("kc", "vc", "thr"):
        _eq(p[n], g[f"i8_{n}"])
    for n in ("qi", "qs", "ki", "ks", "vi"):
        _eq(p[n], g[f"i8_{n}"][:, :T])
    _eq(p["vsc"].reshape(-1, D), g["i8_vsc"])
    _eq(o, g["o_int8"])
    o2 = O.sol_attn_int8(g["q"], g["k"], g["v"], tau=float(g["tau"]), block=blk,
                         int8_pv=False, reference_batch_stride=B > 1)
    _eq(o2, g["o_int8_nopv"])


@pytest.mark.parametrize("name", ["c1", "d128"])
def test_sinks_and_taus_bitexact(name):
    g = load_golden(name)
    B, T, H, D, blk = golden_meta(g)
    q, k, v = g["q"], g["k"], g["v"]
    for key in g.files:
        if key.startswith("sink"):
            s = g[key]
            kw = dict(sink_blocks=(int(s[0]), int(s[1])), sink_q=(int(s[2]), int(s[3])),
                      tau=float(g["tau"]), block=blk, reference_batch_stride=B > 1)
            _eq(O.sol_attn(q, k, v, **kw), g[f"o_bf16_{key}"])
            _eq(O.sol_attn_int8(q, k, v, **kw), g[f"o_int8_{key}"])
        if key.startswith("o_bf16_tau"):
            tau = float(key[len("o_bf16_tau"):])
            _eq(O.sol_attn(q, k, v, tau=tau, block=blk), g[key])


@pytest.mark.parametrize("name", ["c1", "tiny", "ragged", "d128"])
def test_dense_limit_matches_sdpa(name):
    """tau = -1e4 makes every block exact: the reference equals fp32 SDPA (within the
    bf16 rounding of P and O) and the oracle equals the reference bit for bit."""
    g = load_golden(name)
    B, T, H, D, blk = golden_meta(g)
    od = O.sol_attn(g["q"], g["k"], g["v"], tau=-1.0e4, block=blk,
                    reference_batch_stride=B > 1)
    _eq(od, g["o_bf16_dense"])
    ref = O.dense_reference(g["q"], g["k"], g["v"])
    # batch 0 only: the reference's B > 1 pooling rows do not matter when every
    # block is exact, but keep the statement about what was measured precise.
    assert np.abs(od[0] - ref[0]).max() < 4e-3


def test_batch_divergence_is_the_reference_stride():
    """For B > 1 the reference's pooled rows are misplaced (batch stride N instead of
    Npad). With correct pooling, batch 0 is unchanged and equal to the fixture."""
    g = load_golden("d128")
    B, T, H, D, blk = golden_meta(g)
    o = O.sol_attn(g["q"], g["k"], g["v"], tau=float(g["tau"]), block=blk)
    _eq(o[0], g["o_bf16"][0])
    assert not np.array_equal(o[1], g["o_bf16"][1])


def test_morton_perm_bitexact():
    g = load_golden("morton")
    import hashlib
    for key in g.files:
        if key.endswith("_grid"):
            base = key[:-5]
            grid = tuple(int(x) for x in g[key])
            curve = "2d_frame" if base.endswith("2d_frame") else "3d"
            perm, inv = O.morton_perm(grid, curve)
            digest = np.frombuffer(hashlib.sha256(perm.astype("<i8").tobytes()).digest(),
                                   np.uint8)
            _eq(digest, g[base + "_sha"])
            if base + "_perm" in g.files:
                _eq(perm, g[base + "_perm"])
                _eq(inv, g[base + "_inv"])
    for start in (0, 5, 77, 130):
        perm, inv = O.morton_perm_for_span((2, 16, 16), "3d", start)
        _eq(perm, g[f"h3_start{start}_perm"])
        _eq(inv, g[f"h3_start{start}_inv"])


def test_routing_mask_restatement_consistent():
    """The oracle's materialised routing mask equals the decisions its own forward
    makes, and always contains the diagonal band."""
    g = load_golden("c1")
    B, T, H, D, blk = golden_meta(g)
    mask, stat = O.route_mask(g["q"], g["kc"], g["thr"], D ** -0.5, T, blk)
    N = mask.shape[-1]
    for n in range(N):
        for j in (n - 1, n, n + 1):
            if 0 <= j < N:
                assert mask[:, :, n, j].all()
    assert 0 < mask.mean() < 1


@pytest.mark.parametrize("path", ["bf16", "int8"])
def test_unit_runner_matches_full_call(path):
    """The CPU timing arm's unit runner computes the same tiles as the full oracle call."""
    g = load_golden("c1")
    B, T, H, D, blk = golden_meta(g)
    run = O.unit_runner(g["q"], g["k"], g["v"], tau=0.9, block=blk, path=path)
    units = [(0, 1, 2), (0, 0, T // blk - 1)]
    fn = O.sol_attn_int8 if path == "int8" else O.sol_attn
    full = fn(g["q"], g["k"], g["v"], tau=0.9, block=blk, units=units)
    for (b, h, n), tile in zip(units, run(units)):
        r1 = min(T, (n + 1) * blk)
        assert np.array_equal(tile[: r1 - n * blk], full[b, n * blk:r1, h])
