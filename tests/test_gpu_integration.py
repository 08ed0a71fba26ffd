"""A ComfyUI-style sampling loop on the B200 through the node's own entry points, with stub
``comfy`` modules (ComfyUI itself is not in the image): a small bf16 Wan-style block stack
whose attention goes through ``transformer_options["optimized_attention_override"]``, as
ComfyUI's attention call does, patched by "Patch Sol-Attn" (sigma window, dense_blocks,
Morton on a 3-D grid, BF16 or INT8) and measured by "Sol-Attn Block Probe", the per-block
sparse-vs-dense error table the reference logs at cleanup (``__init__.py:256-342, 422-684``).

* the counters of a 6-step loop follow the sigma window and dense_blocks exactly;
* with every block routed exact (tau = -1e30), the patched loop, Morton reorder included,
  ends where the unpatched (host SDPA) loop ends, within bf16 rounding;
* at tau 0.9 the probe records every block (the dense ones at zero error), returns the
  host's result, and its cleanup callback logs the table.
"""

import importlib.util
import logging

import pytest
import torch
import torch.nn.functional as F

from conftest import PKG
from test_override import FakeModel, _install_stub_comfy

from solb200 import override as ov

pytestmark = pytest.mark.gpu

GRID = (4, 16, 32)          # frames, height, width: 2048 tokens
HEADS, D = 4, 128
DIM = HEADS * D
SIGMAS = [1.0, 0.75, 0.6, 0.4, 0.2, 0.0]   # float32 like ComfyUI's (0.8 would read 0.80000001)


def _host_attention(q, k, v, heads, mask=None, attn_precision=None, skip_reshape=False,
                    skip_output_reshape=False, transformer_options=None, **kwargs):
    """The host's attention function (ComfyUI's attention_pytorch for this layout)."""
    B, T, C = q.shape
    qh, kh, vh = (t.view(B, -1, heads, C // heads).transpose(1, 2) for t in (q, k, v))
    return F.scaled_dot_product_attention(qh, kh, vh).transpose(1, 2).reshape(B, T, C)


class Block(torch.nn.Module):
    def __init__(self, gen):
        super().__init__()
        self.qkv = torch.nn.Linear(DIM, 3 * DIM, bias=False)
        self.out = torch.nn.Linear(DIM, DIM, bias=False)
        with torch.no_grad():
            self.qkv.weight.copy_(torch.randn(3 * DIM, DIM, generator=gen) * DIM ** -0.5)
            self.out.weight.copy_(torch.randn(DIM, DIM, generator=gen) * 0.5 * DIM ** -0.5)

    def forward(self, x, freqs=None, transformer_options=None):
        q, k, v = self.qkv(x).chunk(3, dim=-1)
        override = (transformer_options or {}).get("optimized_attention_override")
        if override is not None:
            a = override(_host_attention, q, k, v, HEADS, transformer_options=transformer_options)
        else:
            a = _host_attention(q, k, v, HEADS)
        return x + self.out(a)


class WanLike(torch.nn.Module):
    """Blocks called with (x, freqs=..., transformer_options=...) and a rope_encode method:
    what the node's hooks recognise as a Wan-style stack."""

    def __init__(self, blocks=4):
        super().__init__()
        gen = torch.Generator().manual_seed(3)
        self.blocks = torch.nn.ModuleList([Block(gen) for _ in range(blocks)])

    def rope_encode(self, *args):
        return None

    def forward(self, x, sigma, transformer_options):
        opts = dict(transformer_options)
        opts["sigmas"] = torch.tensor([sigma])
        opts["grid_sizes"] = GRID
        freqs = torch.zeros(1, x.shape[1], 1, 2, device=x.device)   # a RoPE table, one row per token
        for block in self.blocks:
            x = block(x, freqs=freqs, transformer_options=opts)
        return x


def _node_module(monkeypatch):
    _install_stub_comfy(monkeypatch)
    spec = importlib.util.spec_from_file_location("solattn_b200_node_gpu", PKG / "__init__.py",
                                                  submodule_search_locations=[str(PKG)])
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _latent():
    gen = torch.Generator().manual_seed(7)
    # smooth along the token axis plus noise, like a video latent's projections
    base = torch.randn(1, 256, DIM, generator=gen).repeat_interleave(8, dim=1)
    return (base + 0.3 * torch.randn(1, 2048, DIM, generator=gen)).to(torch.bfloat16).cuda()


def _sample(model, dm):
    """Euler-like loop over SIGMAS with the patched model's transformer_options."""
    x = _latent()
    opts = model.model_options["transformer_options"]
    with torch.no_grad():
        for sigma in SIGMAS:
            x = x - 0.1 * dm(x, sigma, opts)
    return x.float()


def _patch(mod, model, **kw):
    args = dict(tau=0.9, start_percent=0.2, end_percent=0.9, min_tokens=1024, int8_qk=False,
                sink_conditioning="off", morton=False, morton_curve="3d", dense_blocks="0,-1",
                verbose=False)
    args.update(kw)
    return mod.SolAttnPatch.execute(model, **args)


def _close(a, b):
    a, b = a.flatten().double(), b.flatten().double()
    return float((a - b).abs().max()), float(a @ b / (a.norm() * b.norm()))


def test_sampling_loop_counters(cuda_device, monkeypatch):
    mod = _node_module(monkeypatch)
    dm = WanLike().cuda().to(torch.bfloat16)
    m = _patch(mod, FakeModel(dm))
    _sample(m, dm)
    st = ov.sol_attn_stats()
    # window [0.1, 0.8]: sigmas 0.75, 0.6, 0.4, 0.2 run Sol-Attn on blocks 1 and 2
    assert st["sparse"] == 4 * 2, st
    assert st["dense_block"] == 6 * 2, st          # blocks 0 and -1 (checked before the window)
    assert st["outside_range"] == 2 * 2, st        # sigmas 1.0 and 0.0 on blocks 1 and 2
    assert st["errors"] == 0 and st["dense_fallback"] == 0, st


@pytest.mark.parametrize("int8,morton", [(False, False), (False, True), (True, True)])
def test_all_exact_loop_matches_host(cuda_device, monkeypatch, int8, morton):
    mod = _node_module(monkeypatch)
    dm = WanLike().cuda().to(torch.bfloat16)
    want = _sample(FakeModel(dm), dm)
    m = _patch(mod, FakeModel(dm), tau=-1e30, int8_qk=int8, morton=morton, dense_blocks="",
               start_percent=0.0, end_percent=1.0)
    if morton:
        assert m.model_options["transformer_options"].get("sol_morton") is True
    got = _sample(m, dm)
    assert ov.sol_attn_stats()["sparse"] == len(SIGMAS) * 4
    d, cos = _close(got, want)
    assert torch.isfinite(got).all()
    assert cos >= (0.998 if int8 else 0.9999) and d <= (0.25 if int8 else 0.1), (d, cos)


def test_block_probe_table(cuda_device, monkeypatch, caplog):
    mod = _node_module(monkeypatch)
    dm = WanLike().cuda().to(torch.bfloat16)
    want = _sample(FakeModel(dm), dm)
    m = _patch(mod, FakeModel(dm))
    probed = mod.SolAttnBlockProbe.execute(m)
    got = _sample(probed, dm)
    # the probe hands back the host's result, so the loop is the dense one
    d, cos = _close(got, want)
    assert cos >= 0.9999, (d, cos)
    errors = ov.probe_results()
    assert set(errors) == {0, 1, 2, 3}, errors
    assert errors[0] == 0.0 and errors[3] == 0.0, errors        # dense_blocks: host result
    # random-weight blocks attend broadly, so tau 0.9 leaves a visible error: bounded, not zero
    assert 0.0 < errors[1] < 0.5 and 0.0 < errors[2] < 0.5, errors
    with caplog.at_level(logging.INFO):
        for kind, fn in probed.callbacks:
            fn()
    assert any("block" in r.getMessage().lower() for r in caplog.records)
    assert ov.probe_results() == {}                  # the table is emitted once, then cleared
