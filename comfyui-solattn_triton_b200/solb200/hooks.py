"""Model hooks used by the ComfyUI node: Morton reordering of a Wan-style block stack
and the running block index.

    install_wan_morton(model)    _morton.py:85-153: block-0 pre-hook permutes the hidden
                                 states x[B, T, C] and the RoPE table into Z-order (one
                                 decision point for both), later blocks reuse the
                                 permuted table, the last block's post-hook restores the
                                 token order. Gated on transformer_options["sol_morton"].
    install_block_index(model)   __init__.py:94-113: publishes transformer_options["sol_block"]

The permutation and the gathers run on the device (solb200.morton). MiniMax-H3 span
hooks and the composition with foreign object patches are model-specific glue that
this build does not provide: the node logs that and Sol-Attn itself still applies.
"""

from __future__ import annotations

import logging
import math

import torch

from .morton import morton_perm, permute_tokens

_INSTALLED = set()
_BLOCK_INDEX = set()
_logged = set()


def _log_once(message):
    if message not in _logged:
        _logged.add(message)
        logging.info(f"[sol_attn] {message}")


def install_block_index(model) -> bool:
    blocks = getattr(model, "blocks", None)
    if blocks is None:
        return False
    if id(model) in _BLOCK_INDEX:
        return True

    def make_hook(index):
        def hook(_module, _args, kwargs):
            options = kwargs.get("transformer_options")
            if isinstance(options, dict):
                options["sol_block"] = index
            return None
        return hook

    for index, block in enumerate(blocks):
        block.register_forward_pre_hook(make_hook(index), with_kwargs=True)
    _BLOCK_INDEX.add(id(model))
    return True


def install_wan_morton(model):
    """Idempotently install the reorder hooks; inert without the sol_morton flag."""
    if id(model) in _INSTALLED:
        return
    blocks = getattr(model, "blocks", None)
    if blocks is None:
        raise RuntimeError("Morton reordering needs .blocks on the diffusion model")
    first, last = blocks[0], blocks[-1]

    def decide(x, freqs, options):
        grid = options.get("grid_sizes")
        if grid is None:
            _log_once("Wan Morton: transformer_options has no grid_sizes; inactive")
            return None
        tokens = int(math.prod(int(g) for g in grid))
        if not torch.is_tensor(x) or x.ndim != 3 or x.shape[1] != tokens:
            _log_once(f"Wan Morton: token count does not match the video grid {tuple(grid)}; inactive")
            return None
        if not torch.is_tensor(freqs) or freqs.shape[1] != tokens:
            _log_once("Wan Morton: rope table does not match the video grid; inactive")
            return None
        perm, inverse = morton_perm(grid, x.device, options.get("sol_morton_curve", "3d"))
        return perm, inverse, freqs.index_select(1, perm)

    def pre_hook(module, args, kwargs):
        options = kwargs.get("transformer_options") or {}
        if not options.get("sol_morton") or not args:
            return None
        if module is first:
            model._sol_morton_state = None
            decision = decide(args[0], kwargs.get("freqs"), options)
            if decision is None:
                return None
            perm, inverse, freqs = decision
            model._sol_morton_state = (perm, inverse, freqs)
            x = args[0]
            xp = permute_tokens(x, perm) if x.is_cuda else x.index_select(1, perm)
            return (xp,) + tuple(args[1:]), {**kwargs, "freqs": freqs}
        state = getattr(model, "_sol_morton_state", None)
        if state is None:
            return None
        return args, {**kwargs, "freqs": state[2]}

    def post_hook(_module, _args, _kwargs, output):
        state = getattr(model, "_sol_morton_state", None)
        if state is None:
            return None
        model._sol_morton_state = None
        inverse = state[1]
        if not torch.is_tensor(output) or output.shape[1] != inverse.numel():
            logging.error("[sol_attn] Wan Morton: block stack changed the token count; "
                          "cannot restore order")
            return None
        return permute_tokens(output, inverse) if output.is_cuda else output.index_select(1, inverse)

    for block in blocks:
        block.register_forward_pre_hook(pre_hook, with_kwargs=True)
    last.register_forward_hook(post_hook, with_kwargs=True)
    _INSTALLED.add(id(model))


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
