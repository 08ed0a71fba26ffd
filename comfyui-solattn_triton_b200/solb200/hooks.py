"""Model hooks for the ComfyUI node: the running block index and the Morton reorder of a
Wan-style block stack.

Behaviour (the reference's, for the host-visible parts):
  * every block sees ``transformer_options["sol_block"]`` = its position in ``.blocks``
    (the reference publishes it from per-block pre-hooks, ``__init__.py:94-113``), which the
    override uses for ``dense_blocks`` and ``tau_profile``;
  * with ``transformer_options["sol_morton"]`` set, the hidden states ``x [B, T, C]`` and
    the RoPE table enter the first block in Z-order and leave the last block in the
    original order (``_morton.py:85-153``), so every attention call in between runs on
    Morton-ordered tokens.

Design of this build: one ``_StackHooks`` object per diffusion model, kept in a weak
registry (nothing is stored on the model). It registers exactly one forward-pre-hook per
block, which does both jobs, plus one forward hook on the last block. The reorder is a
small state machine:

    idle --(block 0, flag set, grid matches)--> active(plan) --(last block returns)--> idle

where ``plan`` holds the inverse permutation and the permuted RoPE table for the
current model call. x and the output are permuted on the device by the row-gather kernel
(``solb200.permute_tokens``); the small RoPE table by ``index_select``.

MiniMax-H3 span hooks and composition with foreign object patches are model-specific
glue that this build does not provide: the node logs that and Sol-Attn itself applies.
"""

from __future__ import annotations

import logging
import math
import weakref
from dataclasses import dataclass

import torch

from .morton import morton_perm, permute_tokens

_logged = set()


def _log_once(message, level=logging.INFO):
    if message not in _logged:
        _logged.add(message)
        logging.log(level, f"[sol_attn] {message}")


@dataclass
class _Plan:
    """Reorder plan of one model call."""
    inverse: torch.Tensor
    freqs: torch.Tensor


def _gather_rows(t: torch.Tensor, index: torch.Tensor) -> torch.Tensor:
    return permute_tokens(t, index) if t.is_cuda else t.index_select(1, index)


class _StackHooks:
    def __init__(self, model):
        blocks = getattr(model, "blocks", None)
        if blocks is None or len(blocks) == 0:
            raise RuntimeError("block hooks need a non-empty .blocks list on the diffusion model")
        self.count = len(blocks)
        self.publish_index = False
        self.reorder = False
        self.plan = None
        for position, block in enumerate(blocks):
            block.register_forward_pre_hook(self._pre_hook(position), with_kwargs=True)
        blocks[-1].register_forward_hook(self._after_last, with_kwargs=True)

    # -------------------------------------------------------------- planning

    @staticmethod
    def _why_not(x, freqs, grid):
        """None when the call can be reordered, else the reason it cannot."""
        if grid is None:
            return "transformer_options has no grid_sizes"
        tokens = math.prod(int(g) for g in grid)
        if not (torch.is_tensor(x) and x.dim() == 3 and x.shape[1] == tokens):
            return f"hidden states do not hold the {tuple(int(g) for g in grid)} video grid"
        if not (torch.is_tensor(freqs) and freqs.dim() >= 2 and freqs.shape[1] == tokens):
            return "the RoPE table does not match the video grid"
        return None

    def _start(self, x, freqs, options):
        grid = options.get("grid_sizes")
        reason = self._why_not(x, freqs, grid)
        if reason is not None:
            _log_once(f"Wan Morton inactive: {reason}")
            return None
        perm, inverse = morton_perm(grid, x.device, options.get("sol_morton_curve", "3d"))
        xp = _gather_rows(x, perm)
        fp = freqs.index_select(1, perm.to(freqs.device))   # the RoPE table is small
        self.plan = _Plan(inverse=inverse, freqs=fp)
        return xp

    # ----------------------------------------------------------------- hooks

    def _pre_hook(self, position):
        def hook(_module, args, kwargs):
            options = kwargs.get("transformer_options")
            if not isinstance(options, dict):
                return None
            if self.publish_index:
                options["sol_block"] = position
            if not (self.reorder and options.get("sol_morton") and args):
                return None
            if position == 0:
                self.plan = None   # a new model call starts; drop any unfinished plan
                xp = self._start(args[0], kwargs.get("freqs"), options)
                if xp is None:
                    return None
                return (xp, *args[1:]), {**kwargs, "freqs": self.plan.freqs}
            if self.plan is None:
                return None
            return args, {**kwargs, "freqs": self.plan.freqs}
        return hook

    def _after_last(self, _module, _args, _kwargs, output):
        plan, self.plan = self.plan, None
        if plan is None:
            return None
        if not (torch.is_tensor(output) and output.shape[1] == plan.inverse.numel()):
            _log_once("Wan Morton: the block stack changed the token count; order not restored",
                      logging.ERROR)
            return None
        return _gather_rows(output, plan.inverse)


# Hook objects, keyed by the model's first block (an nn.Module, which supports weak
# references even when the model object itself does not): they go away with the model.
_REGISTRY: "weakref.WeakKeyDictionary[object, _StackHooks]" = weakref.WeakKeyDictionary()


def _hooks_for(model) -> _StackHooks | None:
    blocks = getattr(model, "blocks", None)
    if not blocks:
        return None
    key = blocks[0]
    hooks = _REGISTRY.get(key)
    if hooks is None:
        hooks = _StackHooks(model)
        _REGISTRY[key] = hooks
    return hooks


def install_block_index(model) -> bool:
    """Publish transformer_options["sol_block"] from every block; False when the model has
    no .blocks list."""
    hooks = _hooks_for(model)
    if hooks is None:
        return False
    hooks.publish_index = True
    return True


def install_wan_morton(model):
    """Enable the Morton reorder on a Wan-style block stack (inert until the host sets
    transformer_options["sol_morton"]); idempotent."""
    hooks = _hooks_for(model)
    if hooks is None:
        raise RuntimeError("Morton reordering needs .blocks on the diffusion model")
    hooks.reorder = True


def install_for_model(diffusion_model, morton, sink_conditioning):
    """Install what the node's options need on this model; returns a small description."""
    is_h3 = hasattr(diffusion_model, "rope_freqs") and hasattr(diffusion_model, "_forward")
    is_wan = hasattr(diffusion_model, "rope_encode") and hasattr(diffusion_model, "blocks")
    reorder = False
    if is_h3 and (morton or sink_conditioning != "off"):
        logging.warning("[sol_attn] MiniMax-H3 span hooks are not provided by this build: Morton "
                        "and the conditioning sink stay inactive unless the host publishes "
                        "transformer_options['sol_h3_video_span']. Sol-Attn itself still applies.")
    elif is_wan and morton:
        install_wan_morton(diffusion_model)
        reorder = True
    elif morton:
        logging.warning(f"[sol_attn] Morton reordering skipped: {type(diffusion_model).__name__} is "
                        "neither Wan-style nor MiniMax-H3. Sol-Attn itself still applies.")
    return {"is_h3": is_h3, "is_wan": is_wan, "reorder": reorder}


def compose_object_patches(model_patcher, diffusion_model, setup):
    """Foreign object-patched attention forwards bypass the override; this build does
    not wrap them (model glue, out of scope) and says so."""
    patches = getattr(model_patcher, "object_patches", {}) or {}
    keys = [k for k in patches if k.endswith(".forward") and "attn" in k.rsplit(".", 2)[-2].lower()]
    if keys:
        logging.warning(f"[sol_attn] {len(keys)} object-patched attention forward(s) (e.g. "
                        f"{keys[0]}) bypass optimized_attention and keep their own kernel")
    return keys
