"""The dense B200 path (``solb200.dense_attn``, C ABI ``solb200_attn_dense``) for the calls the
Sol-Attn path declines (``__init__.py:170-189`` of the reference: cross-attention, head_dim
!= 128, short sequences), which the reference hands back to the host's attention.

* against fp32 SDPA on the same bf16 inputs (max |diff| <= 2e-2, cosine >= 0.999):
  cross-attention (text-length keys), head_dim 64 and 128, ragged and tiny lengths, batch 2,
  strided (BHND) views;
* self-attention equals the Sol-Attn kernel with every block exact (tau = -1e30), bit for bit
  (the same tiles in the same order);
* the attention override runs a cross-attention call on it (counter ``dense_b200``) instead
  of the host's function, and still hands masked calls to the host.
"""

import pytest
import torch

import solb200
from solb200 import override as ov

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MIN_COS = 0.999


def _sdpa(q, k, v):
    qt, kt, vt = (t.float().transpose(1, 2) for t in (q, k, v))
    return torch.nn.functional.scaled_dot_product_attention(qt, kt, vt).transpose(1, 2)


def _close(got, want, label):
    a, b = got.float().flatten().double(), want.float().flatten().double()
    d = (a - b).abs().max().item()
    cos = (a @ b / (a.norm() * b.norm())).item()
    assert torch.isfinite(a).all(), label
    assert d <= MAX_ABS and cos >= MIN_COS, f"{label}: max|d|={d:.3e} cos={cos:.6f}"


@pytest.mark.parametrize("B,Tq,Tk,H,D", [(1, 4096, 512, 4, 128), (2, 1000, 300, 3, 64), (1, 333, 333, 2, 128),
                                         (1, 200, 17, 2, 128), (1, 64, 4096, 2, 64)])
def test_dense_matches_sdpa(cuda_device, B, Tq, Tk, H, D):
    g = torch.Generator(device="cpu").manual_seed(Tq + Tk)
    q = (torch.randn(B, Tq, H, D, generator=g) * D ** -0.25).to(torch.bfloat16).cuda()
    k = (torch.randn(B, Tk, H, D, generator=g) * D ** -0.25).to(torch.bfloat16).cuda()
    v = torch.randn(B, Tk, H, D, generator=g).to(torch.bfloat16).cuda()
    out = solb200.dense_attn(q, k, v)
    assert out.shape == (B, Tq, H, D) and out.dtype == torch.bfloat16
    _close(out, _sdpa(q, k, v), f"dense {B}x{Tq}x{Tk}x{H}x{D}")
    # BHND views of the same tensors
    qv, kv, vv = (t.transpose(1, 2).contiguous().transpose(1, 2) for t in (q, k, v))
    assert torch.equal(solb200.dense_attn(qv, kv, vv), out)


def test_dense_self_attention_equals_all_exact_sparse(cuda_device):
    g = torch.Generator(device="cpu").manual_seed(9)
    q, k, v = (torch.randn(1, 1500, 3, 128, generator=g).to(torch.bfloat16).cuda() for _ in range(3))
    assert torch.equal(solb200.dense_attn(q, k, v), solb200.sol_attn(q, k, v, tau=-1e30, block=128))


def test_override_runs_cross_attention_dense_on_b200(cuda_device):
    ov.reset_sol_attn_stats()
    g = torch.Generator(device="cpu").manual_seed(4)
    heads, D = 4, 128
    q = torch.randn(1, 4096, heads * D, generator=g).to(torch.bfloat16).cuda()
    kv = torch.randn(1, 512, heads * D, generator=g).to(torch.bfloat16).cuda()

    def host(q, k, v, heads, **kw):
        raise AssertionError("the host's attention should not run")

    override = ov.make_override(tau=0.9, min_tokens=4096)
    out = override(host, q, kv, kv, heads)
    want = _sdpa(q.view(1, 4096, heads, D), kv.view(1, 512, heads, D), kv.view(1, 512, heads, D))
    _close(out.view(1, 4096, heads, D), want, "override cross-attention")
    assert ov.sol_attn_stats()["dense_b200"] == 1
    # a masked call still goes to the host
    mask = torch.zeros(4096, 512, device="cuda")
    assert override(lambda *a, **k: "host", q, kv, kv, heads, mask=mask) == "host"
