"""ComfyUI custom-node entry of the B200 Sol-Attn extension.

Same nodes, inputs, defaults and transformer_options keys as the reference extension
(kijai/ComfyUI-SolAttn_triton, __init__.py:422-684), with the attention override
running the sm_100a kernels of ``solb200`` (C ABI in include/solb200.h):

    SolAttnPatch        "Patch Sol-Attn": installs the override on a model clone
    SolAttnBlockProbe   "Sol-Attn Block Probe": per-block sparse-vs-dense error
    attention_sol       registry entry ("sol_attn"); SOL_ATTN=1 makes it global

Model hooks (Morton reordering for Wan / MiniMax-H3, block-index publishing) use
the device-side Morton permutation and gather of ``solb200.morton`` / ``solb200.hooks``.
"""

import logging
import os
import sys
from pathlib import Path

_HERE = str(Path(__file__).resolve().parent)
if _HERE not in sys.path:
    sys.path.insert(0, _HERE)

from comfy.ldm.modules.attention import (  # noqa: E402
    attention_pytorch,
    register_attention_function,
    wrap_attn,
)
from comfy.patcher_extension import CallbacksMP  # noqa: E402
from comfy_api.latest import ComfyExtension, io  # noqa: E402

try:
    from solb200 import override as _ov  # noqa: E402
    from solb200 import hooks as _hooks  # noqa: E402
    from solb200 import _lib as _native  # noqa: E402
    _native.lib()
    _IMPORT_ERROR = None
except Exception as exc:  # library missing or not built
    _ov = _hooks = None
    _IMPORT_ERROR = exc

sol_attn_stats = _ov.sol_attn_stats if _ov else (lambda: {})
reset_sol_attn_stats = _ov.reset_sol_attn_stats if _ov else (lambda: None)


class SolAttnPatch(io.ComfyNode):
    @classmethod
    def define_schema(cls):
        return io.Schema(
            node_id="SolAttnPatch",
            display_name="Patch Sol-Attn",
            is_experimental=True,
            category="sol_attn",
            description="Sparsify self-attention with Sol-Attn on B200 (sm_100a kernels), with "
                        "optional Morton token reordering, INT8 QK and an exact-KV sink for "
                        "MiniMax-H3's packed conditioning rows. bf16 + head_dim 128 only; "
                        "everything else falls back to the existing attention backend.",
            inputs=[
                io.Model.Input("model"),
                io.Float.Input("tau", default=1.3, min=0.0, max=4.0, step=0.05,
                               tooltip="Routing threshold multiplier. Higher is sparser."),
                io.Float.Input("start_percent", default=0.2, min=0.0, max=1.0, step=0.01,
                               tooltip="Run dense before this point of sampling."),
                io.Float.Input("end_percent", default=0.9, min=0.0, max=1.0, step=0.01),
                io.Int.Input("min_tokens", default=4096, min=0, max=1 << 20, step=512,
                             tooltip="Sequences shorter than this stay dense."),
                io.Boolean.Input("int8_qk", default=True,
                                 tooltip="INT8 QK in the exact branch (smoothed K, per-token "
                                         "scales)."),
                io.Combo.Input("sink_conditioning", options=["exact_kv", "exact_kv_and_rows", "off"],
                               default="exact_kv_and_rows",
                               tooltip="MiniMax-H3 only: keep the packed conditioning rows exact "
                                       "as keys (exact_kv) or also as queries."),
                io.Boolean.Input("morton", default=False,
                                 tooltip="Reorder video tokens into Morton (Z-order) so each "
                                         "block is a compact 3D neighbourhood. Wan and "
                                         "MiniMax-H3 only."),
                io.Combo.Input("morton_curve", options=["3d", "2d_frame"], default="2d_frame"),
                io.Boolean.Input("int8_pv", default=True,
                                 tooltip="Also run the exact branch's P@V in INT8 (only with "
                                         "int8_qk)."),
                io.Boolean.Input("verbose", default=False),
                io.Boolean.Input("use_tma", default=False,
                                 tooltip="Accepted for workflow compatibility; the sm_100a "
                                         "kernels always stage tiles with TMA."),
                io.String.Input("tau_profile", optional=True, force_input=True,
                                tooltip="Per-block tau: 'blocks=tau' entries separated by ';' "
                                        "or newlines, e.g. '0-30=2.0; 39-42=0.9'."),
                io.String.Input("dense_blocks", default="",
                                tooltip="Transformer blocks to keep dense, e.g. '0-2,-1'."),
            ],
            outputs=[io.Model.Output()],
        )

    @classmethod
    def execute(cls, model, tau, start_percent, end_percent, min_tokens, int8_qk, sink_conditioning,
                morton, morton_curve, dense_blocks, verbose, tau_profile=None, use_tma=False,
                int8_pv=True) -> io.NodeOutput:
        if _ov is None:
            raise RuntimeError(f"Sol-Attn B200 kernels unavailable: {_IMPORT_ERROR}")
        diffusion_model = model.get_model_object("diffusion_model")
        setup = _hooks.install_for_model(diffusion_model, morton=morton,
                                         sink_conditioning=sink_conditioning)
        blocks = getattr(diffusion_model, "blocks", None)
        count = len(blocks) if blocks is not None else 0
        dense = _ov.parse_blocks(dense_blocks, count)
        profile = _ov.parse_tau_profile(tau_profile or "", count)
        if (dense or profile) and not _hooks.install_block_index(diffusion_model):
            logging.warning(f"[sol_attn] dense_blocks/tau_profile ignored: "
                            f"{type(diffusion_model).__name__} has no .blocks list to index")
            dense, profile = frozenset(), {}
        model_sampling = model.get_model_object("model_sampling")
        sigma_start = float(model_sampling.percent_to_sigma(start_percent))
        sigma_end = float(model_sampling.percent_to_sigma(end_percent))
        m = model.clone()
        options = m.model_options["transformer_options"]
        previous = options.get("optimized_attention_override")
        if previous is not None:
            logging.info("[sol_attn] chaining onto an existing attention override")
        _hooks.compose_object_patches(m, diffusion_model, setup)
        options["sol_compose"] = {"sigma_start": sigma_start, "sigma_end": sigma_end,
                                  "min_tokens": min_tokens}
        options["optimized_attention_override"] = _ov.make_override(
            tau=tau, min_tokens=min_tokens, sigma_start=sigma_start, sigma_end=sigma_end,
            verbose=verbose, int8_qk=int8_qk, sink_conditioning=sink_conditioning,
            use_tma=use_tma, dense_blocks=dense, tau_profile=profile, int8_pv=int8_pv,
            previous=previous)
        if setup.get("reorder"):
            options["sol_morton"] = True
            options["sol_morton_curve"] = morton_curve
        _ov.reset_sol_attn_stats()
        return io.NodeOutput(m)


class SolAttnBlockProbe(io.ComfyNode):
    @classmethod
    def define_schema(cls):
        return io.Schema(
            node_id="SolAttnBlockProbe",
            display_name="Sol-Attn Block Probe",
            is_experimental=True,
            category="sol_attn",
            description="Diagnostic: every attention call is computed sparse and dense and each "
                        "block's relative error is logged worst-first when sampling ends.",
            inputs=[io.Model.Input("model")],
            outputs=[io.Model.Output()],
        )

    @classmethod
    def execute(cls, model) -> io.NodeOutput:
        m = model.clone()
        options = m.model_options["transformer_options"]
        inner = options.get("optimized_attention_override")
        if inner is None:
            raise RuntimeError("Sol-Attn Block Probe needs an attention override to measure; "
                               "connect it after Patch Sol-Attn.")
        diffusion_model = m.get_model_object("diffusion_model")
        if not _hooks.install_block_index(diffusion_model):
            logging.warning("[sol_attn] probe: model has no .blocks list; errors land under None")
        options["optimized_attention_override"] = _ov.make_probe_override(inner)
        _ov._probe.clear()
        m.add_callback(CallbacksMP.ON_CLEANUP, _ov.log_probe_summary)
        return io.NodeOutput(m)


@wrap_attn
def attention_sol(q, k, v, heads, mask=None, attn_precision=None, skip_reshape=False,
                  skip_output_reshape=False, **kwargs):
    """Registry-visible entry point with the defaults (no sigma gating)."""
    if _ov is None:
        return attention_pytorch(q, k, v, heads, mask=mask, skip_reshape=skip_reshape,
                                 skip_output_reshape=skip_output_reshape, **kwargs)
    return _ov.attention_sol(q, k, v, heads, mask=mask, attn_precision=attn_precision,
                             skip_reshape=skip_reshape, skip_output_reshape=skip_output_reshape,
                             dense=attention_pytorch, **kwargs)


register_attention_function("sol_attn", attention_sol)

if os.environ.get("SOL_ATTN", "0") not in ("0", "", "false"):
    if _ov is None:
        logging.error(f"[sol_attn] SOL_ATTN set but the kernels failed to load: {_IMPORT_ERROR}")
    else:
        import comfy.ldm.modules.attention as _attn_mod
        _attn_mod.optimized_attention = attention_sol
        _attn_mod.optimized_attention_masked = attention_sol
        logging.info("[sol_attn] global override active (node patch is preferred)")


class SolAttnExtension(ComfyExtension):
    async def get_node_list(self):
        return [SolAttnPatch, SolAttnBlockProbe]


async def comfy_entrypoint() -> SolAttnExtension:
    return SolAttnExtension()
