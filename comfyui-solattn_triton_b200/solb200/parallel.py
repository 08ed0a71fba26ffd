"""Multi-GPU layouts for the Sol-Attn path: one process per GPU.

Every stage of the path depends only on its own (batch, head) — pooling, kc moments,
routing, the forward — and the Morton permutation only on the token grid. So:

* ``head_shard(rank, world, heads)``: the head range a rank owns when the whole
  sequence is present on every rank. No exchange at all; the per-head results are
  identical to a single-GPU run.
* ``ulysses_attention(q, k, v, attn, group)``: inputs that arrive sequence-sharded
  ([B, T/W, H, D] per rank) are re-sharded to head-sharded ([B, T, H/W, D]) with one
  all-to-all per tensor (``torch.distributed``, NCCL over NVLink on GPUs), the local
  Sol-Attn runs on whole sequences, and one all-to-all returns the output to the
  sequence-sharded layout.

The reference has no multi-GPU code; these are this build's additions.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def head_shard(rank: int, world: int, heads: int) -> slice:
    if heads % world:
        raise ValueError(f"{heads} heads do not split evenly over {world} ranks")
    per = heads // world
    return slice(rank * per, (rank + 1) * per)


def seq_to_head(x: torch.Tensor, group=None) -> torch.Tensor:
    """[B, T/W, H, D] on each rank -> [B, T, H/W, D] (rank r gets heads r*H/W..)."""
    world = dist.get_world_size(group)
    B, Tl, H, D = x.shape
    if H % world:
        raise ValueError(f"{H} heads do not split over {world} ranks")
    hw = H // world
    send = x.reshape(B, Tl, world, hw, D).permute(2, 0, 1, 3, 4).contiguous()  # [W, B, Tl, hw, D]
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    # recv[j] = sequence chunk j of my heads
    return recv.permute(1, 0, 2, 3, 4).reshape(B, world * Tl, hw, D)


def head_to_seq(x: torch.Tensor, group=None) -> torch.Tensor:
    """[B, T, H/W, D] on each rank -> [B, T/W, H, D] (the inverse of seq_to_head)."""
    world = dist.get_world_size(group)
    B, T, hw, D = x.shape
    if T % world:
        raise ValueError(f"{T} tokens do not split over {world} ranks")
    Tl = T // world
    send = x.reshape(B, world, Tl, hw, D).permute(1, 0, 2, 3, 4).contiguous()  # [W, B, Tl, hw, D]
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    # recv[j] = my sequence chunk of rank j's heads
    return recv.permute(1, 2, 0, 3, 4).reshape(B, Tl, world * hw, D)


def ulysses_attention(q, k, v, attn, group=None, **kwargs):
    """Sequence-sharded q/k/v [B, T/W, H, D] -> attention over the full sequence ->
    sequence-sharded output [B, T/W, H, D]. ``attn`` is ``solb200.sol_attn`` (or
    ``sol_attn_int8``); it sees whole sequences and H/W heads."""
    qh, kh, vh = (seq_to_head(t, group) for t in (q, k, v))
    out = attn(qh, kh, vh, **kwargs)
    return head_to_seq(out, group)
