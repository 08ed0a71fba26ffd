"""The int8 quantisers divide without a division per element (one correctly rounded
reciprocal per scale, then two FMA remainder corrections: Markstein's theorem, two lanes
at a time) and round half away from zero as x / s + copysign(0.5) then a truncating
conversion. These tests compare both, on the GPU, with CUDA's IEEE division __fdiv_rn and
the reference's rounding, through the library's self-test entry point: random pairs over
the scale range the quantisers use, the exact tie points (k + 0.5) * s and their
neighbours, and edge scales."""

import numpy as np
import pytest
import torch


def _run(x: np.ndarray, s: np.ndarray):
    from solb200 import _lib

    dx = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    ds = torch.from_numpy(np.ascontiguousarray(s, np.float32)).cuda()
    bad = torch.zeros(2, dtype=torch.int64, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    _lib.check(_lib.lib().solb200_selftest_quotient(dx.data_ptr(), ds.data_ptr(), dx.numel(), bad.data_ptr(), st),
               "selftest")
    torch.cuda.synchronize()
    return [int(v) for v in bad.cpu()]


def _scales(rng, n):
    """log-uniform over [1e-8, 1e2] plus the floor 1e-8, powers of two and scales whose
    mantissa is all ones (the hardest reciprocals)."""
    s = np.exp(rng.uniform(np.log(1e-8), np.log(1e2), n)).astype(np.float32)
    edge = [np.float32(1e-8), np.float32(1.0), np.float32(0.5), np.float32(2.0 ** -20),
            np.nextafter(np.float32(2.0), np.float32(0.0)), np.nextafter(np.float32(1.0), np.float32(0.0)),
            np.float32(1.0 / 127.0), np.float32(3.0 / 127.0)]
    s[: len(edge) * 64] = np.repeat(np.array(edge, np.float32), 64)
    return s


@pytest.mark.gpu
def test_quotient_random_pairs(cuda_device):
    rng = np.random.default_rng(11)
    n = 1 << 24
    s = _scales(rng, n)
    u = rng.uniform(-140.0, 140.0, n)
    u = np.where(np.abs(u) < 1e-3, 1e-3, u)
    x = (s.astype(np.float64) * u).astype(np.float32)
    assert _run(x, s) == [0, 0]


@pytest.mark.gpu
def test_quotient_ties_and_neighbours(cuda_device):
    """x = RN((k + 0.5) * s) for k in [-130, 130) and its neighbours up to 2 ulp away:
    the pairs whose int8 code depends on the last bit of the quotient."""
    rng = np.random.default_rng(12)
    m = 1 << 16
    s = np.repeat(_scales(rng, m), 260)
    k = np.tile(np.arange(-130, 130, dtype=np.float64) + 0.5, m)
    base = (s.astype(np.float64) * k).astype(np.float32)
    xs, ss = [base], [s]
    for step in (1, 2):
        up, dn = base.copy(), base.copy()
        for _ in range(step):
            up = np.nextafter(up, np.float32(np.inf))
            dn = np.nextafter(dn, np.float32(-np.inf))
        xs += [up, dn]
        ss += [s, s]
    assert _run(np.concatenate(xs), np.concatenate(ss)) == [0, 0]


@pytest.mark.gpu
def test_quotient_quantiser_inputs(cuda_device):
    """The quantisers' own operands: bf16 values over s = max|x| / 127 of their group."""
    rng = np.random.default_rng(13)
    g = rng.standard_normal((1 << 16, 128)).astype(np.float32) * np.exp(rng.uniform(-8, 3, (1 << 16, 1)))
    g = torch.from_numpy(g).bfloat16().float().numpy()
    s = np.maximum(np.abs(g).max(axis=1, keepdims=True) / np.float32(127.0), np.float32(1e-8)).astype(np.float32)
    assert _run(g.ravel(), np.broadcast_to(s, g.shape).ravel()) == [0, 0]
