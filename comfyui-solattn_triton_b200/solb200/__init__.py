"""solb200: B200-native (sm_100a) Sol-Attn block-sparse attention.

Drop-in for the hot path of kijai/ComfyUI-SolAttn_triton: the same kernel-level API
(``sol_attn``, ``sol_attn_int8``, ``prepare``, ``fused_preprocess``, ``morton_perm``)
backed by hand-written sm_100a kernels in ``libsolb200.so`` (C ABI in
``include/solb200.h``).
"""

from .morton import morton_perm, perm_for_span, permute_tokens, permute_tokens_many
from .ops import BLOCK, dense_attn, fused_preprocess, prepare, routing, sol_attn, sol_attn_int8, workspace_bytes
from .streamed import release_host_buffers, sol_attn_host

__all__ = ["sol_attn", "sol_attn_int8", "dense_attn", "prepare", "fused_preprocess", "routing", "morton_perm",
           "perm_for_span", "permute_tokens", "permute_tokens_many", "workspace_bytes", "BLOCK",
           "sol_attn_host", "release_host_buffers"]
