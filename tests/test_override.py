"""The attention-override boundary: gates, layouts, fallbacks, counters and the ComfyUI
node wiring (with a stub ``comfy`` package; ComfyUI itself is not installed here).
Behaviour follows the reference's __init__.py:49-320, 422-684."""

import importlib.util
import sys
import types

import pytest
import torch

from conftest import PKG

from solb200 import override as ov


# ------------------------------------------------------------------ block specs

def test_parse_blocks():
    assert ov.parse_blocks("0-3,47,-1", 48) == frozenset({0, 1, 2, 3, 47})
    assert ov.parse_blocks(" 5 - 2 ", 10) == frozenset({2, 3, 4, 5})      # whitespace, reversed
    assert ov.parse_blocks("-3--1", 10) == frozenset({7, 8, 9})
    assert ov.parse_blocks("", 10) == frozenset()
    assert ov.parse_blocks("100,3", 10) == frozenset({3})                 # out of range dropped
    with pytest.raises(ValueError):
        ov.parse_blocks("a-b", 10)


def test_parse_tau_profile():
    prof = ov.parse_tau_profile("0-2=2.0; 1=0.5\n# comment\n9=1.1 # trailing", 10)
    assert prof == {0: 2.0, 1: 0.5, 2: 2.0, 9: 1.1}                       # later entries win
    with pytest.raises(ValueError):
        ov.parse_tau_profile("3", 10)
    with pytest.raises(ValueError):
        ov.parse_tau_profile("3=x", 10)


def test_sink_blocks():
    opts = {"sol_h3_video_span": (200, 5000)}
    assert ov._sink_blocks(opts, 5000, "exact_kv") == ((0, 4), (0, 0))
    assert ov._sink_blocks(opts, 5000, "exact_kv_and_rows") == ((0, 4), (0, 4))
    assert ov._sink_blocks(opts, 5000, "off") == ((0, 0), (0, 0))
    assert ov._sink_blocks(opts, 4000, "exact_kv") == ((0, 0), (0, 0))    # span beyond tokens
    assert ov._sink_blocks({"sol_h3_video_span": (0, 10)}, 10, "exact_kv") == ((0, 0), (0, 0))
    assert ov._sink_blocks({}, 10, "exact_kv") == ((0, 0), (0, 0))
    assert ov._sink_blocks(opts, 5000, "exact_kv", block=128) == ((0, 2), (0, 0))


# ---------------------------------------------------------------- fallbacks

class Dense:
    def __init__(self):
        self.calls = 0

    def __call__(self, q, k, v, heads, **kw):
        self.calls += 1
        return torch.zeros_like(q)


def _qkv(T=64, heads=2, D=128, device="cpu"):
    g = torch.Generator().manual_seed(0)
    return [torch.randn(1, T, heads * D, generator=g).to(torch.bfloat16).to(device) for _ in range(3)]


def test_gates_and_counters_cpu():
    ov.reset_sol_attn_stats()
    dense = Dense()
    q, k, v = _qkv()
    o = ov.make_override(tau=1.0, min_tokens=0)
    o(dense, q, k, v, 2, mask=torch.ones(1))                     # masked -> dense
    assert ov.sol_attn_stats()["dense_fallback"] == 1
    o(dense, q, k, v, 2)                                         # cpu tensors -> ineligible
    assert ov.sol_attn_stats()["dense_fallback"] == 2
    o2 = ov.make_override(dense_blocks=frozenset({3}))
    o2(dense, q, k, v, 2, transformer_options={"sol_block": 3})
    assert ov.sol_attn_stats()["dense_block"] == 1
    o3 = ov.make_override(sigma_start=10.0, sigma_end=1.0)
    o3(dense, q, k, v, 2, transformer_options={"sigmas": torch.tensor([12.0])})
    o3(dense, q, k, v, 2, transformer_options={"sigmas": torch.tensor([0.5])})
    assert ov.sol_attn_stats()["outside_range"] == 2
    assert dense.calls == 5


def test_previous_override_is_chained():
    seen = []

    def previous(func, q, k, v, heads, **kw):
        seen.append(heads)
        return func(q, k, v, heads, **kw)

    dense = Dense()
    q, k, v = _qkv()
    ov.make_override(previous=previous)(dense, q, k, v, 2, mask=torch.ones(1))
    assert seen == [2] and dense.calls == 1


def test_kernel_failure_falls_back_dense(monkeypatch):
    ov.reset_sol_attn_stats()

    def boom(*a, **k):
        raise RuntimeError("forced failure")

    monkeypatch.setattr(ov, "_run", boom)
    dense = Dense()
    q, k, v = _qkv()
    out = ov.make_override()(dense, q, k, v, 2)
    assert dense.calls == 1 and torch.count_nonzero(out) == 0
    assert ov.sol_attn_stats()["errors"] == 1


def test_ineligible_reasons():
    q = torch.zeros(1, 8, 2, 128, dtype=torch.bfloat16)
    assert ov._ineligible(q, q, None, 128, 0) == "not cuda"


def test_probe_returns_dense_and_records():
    ov._probe.clear()

    def inner(func, q, k, v, heads, **kw):
        return q + 1

    def dense(q, k, v, heads, **kw):
        return torch.ones_like(q)

    q, k, v = _qkv()
    out = ov.make_probe_override(inner)(dense, q.float(), k, v, 2, transformer_options={"sol_block": 7})
    assert torch.equal(out, torch.ones_like(out))         # the dense result is returned
    assert 7 in ov.probe_results() and ov.probe_results()[7] > 0


# ------------------------------------------------------------ the node module

def _install_stub_comfy(monkeypatch):
    registered = {}

    def wrap_attn(f):
        return f

    attn = types.ModuleType("comfy.ldm.modules.attention")
    attn.attention_pytorch = lambda q, k, v, heads, **kw: torch.zeros_like(q)
    attn.register_attention_function = lambda name, fn: registered.__setitem__(name, fn)
    attn.wrap_attn = wrap_attn
    patcher = types.ModuleType("comfy.patcher_extension")
    patcher.CallbacksMP = types.SimpleNamespace(ON_CLEANUP="on_cleanup")

    class _Any:
        def __init__(self, *a, **k):
            self.a, self.k = a, k

    io = types.SimpleNamespace(
        ComfyNode=object, Schema=_Any, NodeOutput=lambda m: m,
        Model=types.SimpleNamespace(Input=_Any, Output=_Any),
        Float=types.SimpleNamespace(Input=_Any), Int=types.SimpleNamespace(Input=_Any),
        Boolean=types.SimpleNamespace(Input=_Any), Combo=types.SimpleNamespace(Input=_Any),
        String=types.SimpleNamespace(Input=_Any))
    latest = types.ModuleType("comfy_api.latest")
    latest.ComfyExtension = object
    latest.io = io
    for name in ["comfy", "comfy.ldm", "comfy.ldm.modules", "comfy_api"]:
        monkeypatch.setitem(sys.modules, name, types.ModuleType(name))
    monkeypatch.setitem(sys.modules, "comfy.ldm.modules.attention", attn)
    monkeypatch.setitem(sys.modules, "comfy.patcher_extension", patcher)
    monkeypatch.setitem(sys.modules, "comfy_api.latest", latest)
    return registered


class FakeModel:
    def __init__(self, diffusion_model):
        self.diffusion_model = diffusion_model
        self.model_options = {"transformer_options": {}}
        self.object_patches = {}
        self.callbacks = []

    def get_model_object(self, name):
        if name == "diffusion_model":
            return self.diffusion_model
        return types.SimpleNamespace(percent_to_sigma=lambda p: 1.0 - p)

    def clone(self):
        c = FakeModel(self.diffusion_model)
        c.model_options = {"transformer_options": dict(self.model_options["transformer_options"])}
        return c

    def add_callback(self, kind, fn):
        self.callbacks.append((kind, fn))


def test_node_module_with_stub_comfy(monkeypatch):
    registered = _install_stub_comfy(monkeypatch)
    spec = importlib.util.spec_from_file_location("solattn_b200_node", PKG / "__init__.py",
                                                  submodule_search_locations=[str(PKG)])
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    assert "sol_attn" in registered
    blocks = torch.nn.ModuleList([torch.nn.Identity() for _ in range(4)])
    dm = types.SimpleNamespace(blocks=blocks, rope_encode=lambda *a: None)
    model = FakeModel(dm)
    m = mod.SolAttnPatch.execute(model, tau=1.3, start_percent=0.2, end_percent=0.9,
                                 min_tokens=4096, int8_qk=True, sink_conditioning="exact_kv",
                                 morton=False, morton_curve="2d_frame", dense_blocks="0,-1",
                                 verbose=False)
    opts = m.model_options["transformer_options"]
    assert callable(opts["optimized_attention_override"])
    assert opts["sol_compose"] == {"sigma_start": 0.8, "sigma_end": pytest.approx(0.1),
                                   "min_tokens": 4096}
    assert "sol_morton" not in opts
    probe = mod.SolAttnBlockProbe.execute(m)
    assert probe.callbacks and callable(probe.model_options["transformer_options"][
        "optimized_attention_override"])
    with pytest.raises(RuntimeError):
        mod.SolAttnBlockProbe.execute(model)     # no override to measure


def test_mask_layout_reads_masks_like_the_host():
    """``ops.mask_layout``: the host's 2-D / 3-D / 4-D mask conventions as element strides over
    [B, H, Tq, Tk], size-1 dimensions broadcast (stride 0); other shapes and dtypes refused."""
    from solb200 import ops
    B, H, Tq, Tk = 2, 3, 5, 7
    _, kind, st = ops.mask_layout(torch.zeros(Tq, Tk), B, H, Tq, Tk)
    assert (kind, st) == (2, [0, 0, Tk, 1])
    _, kind, st = ops.mask_layout(torch.zeros(B, Tq, Tk, dtype=torch.float16), B, H, Tq, Tk)
    assert (kind, st) == (4, [Tq * Tk, 0, Tk, 1])
    _, kind, st = ops.mask_layout(torch.zeros(B, 1, 1, Tk, dtype=torch.bool), B, H, Tq, Tk)
    assert (kind, st) == (1, [0 if B == 1 else Tk, 0, 0, 1])
    _, kind, st = ops.mask_layout(torch.zeros(1, H, Tq, Tk, dtype=torch.bfloat16), B, H, Tq, Tk)
    assert (kind, st) == (3, [0, Tq * Tk, Tk, 1])
    _, _, st = ops.mask_layout(torch.zeros(1, 1, 1, Tk).expand(B, H, Tq, Tk), B, H, Tq, Tk)
    assert st == [0, 0, 0, 1]
    _, _, st = ops.mask_layout(torch.zeros(Tk, Tq).t(), B, H, Tq, Tk)     # a transposed view
    assert st == [0, 0, 1, Tq]
    for bad in (torch.zeros(Tq, Tk, dtype=torch.int64), torch.zeros(Tq, Tk, dtype=torch.float64),
                torch.zeros(B * H, Tq, Tk), torch.zeros(Tq + 1, Tk), torch.zeros(Tk),
                torch.zeros(1, 1, 1, 1, Tk)):
        with pytest.raises(ValueError):
            ops.mask_layout(bad, B, H, Tq, Tk)


def test_masked_call_on_cpu_goes_to_the_host():
    ov.reset_sol_attn_stats()
    dense = Dense()
    q, k, v = _qkv()
    ov.make_override(tau=1.0, min_tokens=0)(dense, q, k, v, 2, mask=torch.zeros(64, 64))
    assert ov.sol_attn_stats()["dense_fallback"] == 1 and ov.sol_attn_stats()["masked_b200"] == 0
