"""The dense B200 path (``solb200.dense_attn``, C ABI ``solb200_attn_dense``) for the calls the
Sol-Attn path declines (``__init__.py:170-189`` of the reference: cross-attention, head_dim
!= 128, short sequences), which the reference hands back to the host's attention.

* against fp32 SDPA on the same bf16 inputs (max |diff| <= 2e-2, cosine >= 0.999):
  cross-attention (text-length keys), head_dim 64 and 128, ragged and tiny lengths, batch 2,
  strided (BHND) views;
* self-attention equals the Sol-Attn kernel with every block exact (tau = -1e30), bit for bit
  (the same tiles in the same order);
* the attention override runs a cross-attention call on it (counter ``dense_b200``) instead
  of the host's function;
* masks (C ABI ``solb200_attn_dense_masked``), read as the host's attention reads them: bool
  and float32 / bfloat16 / float16 additive masks, 2-D [Tq, Tk], 3-D [B, Tq, Tk] and 4-D
  (key padding [B, 1, 1, Tk], full [B, H, Tq, Tk], expanded views) against fp32 SDPA with the
  same mask; an all-zero float mask gives the unmasked kernel's output bit for bit; a row whose
  keys are all masked is NaN; the override runs masked calls on it (counter ``masked_b200``)
  and hands a mask it cannot read (int64, or [B*H, Tq, Tk]) to the host.
"""

import pytest
import torch

import solb200
from solb200 import override as ov

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MIN_COS = 0.999


def _sdpa(q, k, v, mask=None):
    """fp32 SDPA on BTHD tensors; ``mask`` as the host's attention takes it (2-D [Tq, Tk],
    3-D [B, Tq, Tk], 4-D [B, H, Tq, Tk]; bool attends where true, float is added)."""
    qt, kt, vt = (t.float().transpose(1, 2) for t in (q, k, v))
    if mask is not None:
        if mask.dim() == 2:
            mask = mask.unsqueeze(0)
        if mask.dim() == 3:
            mask = mask.unsqueeze(1)
        if mask.dtype != torch.bool:
            mask = mask.float()
    return torch.nn.functional.scaled_dot_product_attention(qt, kt, vt, attn_mask=mask).transpose(1, 2)


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
    # a masked call runs on the dense kernel too, with the host's mask semantics
    mask = torch.randn(4096, 512, generator=g).cuda()
    out = override(host, q, kv, kv, heads, mask=mask)
    want = _sdpa(q.view(1, 4096, heads, D), kv.view(1, 512, heads, D), kv.view(1, 512, heads, D), mask)
    _close(out.view(1, 4096, heads, D), want, "override masked cross-attention")
    assert ov.sol_attn_stats()["masked_b200"] == 1
    # masks it cannot read stay with the host: an integer mask, and one per (batch x head)
    for bad in (torch.zeros(4096, 512, dtype=torch.int64, device="cuda"),
                torch.zeros(heads, 4096, 512, device="cuda")):
        assert override(lambda *a, **k: "host", q, kv, kv, heads, mask=bad) == "host"
    assert ov.sol_attn_stats()["masked_b200"] == 1


def _rows_with_a_key(mask):
    """bool mask with at least one attended key per query row (column 0 set)."""
    mask = mask.clone()
    mask[..., 0] = True
    return mask


@pytest.mark.parametrize("B,Tq,Tk,H,D", [(2, 1000, 300, 3, 64), (1, 333, 4096, 2, 128), (1, 200, 17, 2, 128)])
@pytest.mark.parametrize("form", ["key_padding_bool", "full_bool", "2d_f32", "3d_f16", "4d_bf16_head",
                                  "expanded_f32"])
def test_masked_dense_matches_sdpa(cuda_device, B, Tq, Tk, H, D, form):
    g = torch.Generator(device="cpu").manual_seed(Tq * 7 + Tk + len(form))
    q = (torch.randn(B, Tq, H, D, generator=g) * D ** -0.25).to(torch.bfloat16).cuda()
    k = (torch.randn(B, Tk, H, D, generator=g) * D ** -0.25).to(torch.bfloat16).cuda()
    v = torch.randn(B, Tk, H, D, generator=g).to(torch.bfloat16).cuda()
    if form == "key_padding_bool":          # [B, 1, 1, Tk]: the last keys of each batch padded out
        mask = torch.arange(Tk).view(1, 1, 1, Tk) < torch.tensor([Tk - Tk // 3, Tk])[:B].view(B, 1, 1, 1)
    elif form == "full_bool":
        mask = _rows_with_a_key(torch.rand(B, H, Tq, Tk, generator=g) < 0.4)
    elif form == "2d_f32":
        mask = torch.randn(Tq, Tk, generator=g) * 2
    elif form == "3d_f16":
        mask = (torch.randn(B, Tq, Tk, generator=g) * 2).half()
    elif form == "4d_bf16_head":            # one additive mask per head, shared over the batch
        mask = (torch.randn(1, H, Tq, Tk, generator=g) * 2).bfloat16()
        mask[..., Tk // 2:] = float("-inf")
    else:                                   # a stride-0 view, as expand() gives
        mask = torch.randn(1, 1, 1, Tk, generator=g).expand(B, H, Tq, Tk)
    mask = mask.cuda()
    out = solb200.dense_attn(q, k, v, mask=mask)
    _close(out, _sdpa(q, k, v, mask), f"masked {form} {B}x{Tq}x{Tk}x{H}x{D}")


def test_zero_mask_is_the_unmasked_kernel_and_masked_rows_are_nan(cuda_device):
    g = torch.Generator(device="cpu").manual_seed(12)
    q, k, v = (torch.randn(1, 700, 2, 128, generator=g).to(torch.bfloat16).cuda() for _ in range(3))
    plain = solb200.dense_attn(q, k, v)
    assert torch.equal(solb200.dense_attn(q, k, v, mask=torch.zeros(700, 700, device="cuda")), plain)
    assert torch.equal(solb200.dense_attn(q, k, v, mask=torch.ones(700, 700, dtype=torch.bool,
                                                                   device="cuda")), plain)
    mask = torch.ones(700, 700, dtype=torch.bool, device="cuda")
    mask[5] = False                          # query row 5 attends to nothing
    out = solb200.dense_attn(q, k, v, mask=mask)
    assert torch.isnan(out[0, 5]).all()
    keep = torch.ones(700, dtype=torch.bool)
    keep[5] = False
    assert torch.equal(out[0, keep.cuda()], plain[0, keep.cuda()])
