"""The node's model hooks on a stub Wan-style block stack (CPU): the block index that the
override reads, and the Morton reorder of hidden states and RoPE table around the block
stack (``_morton.py:85-153``, ``__init__.py:94-113`` of the reference). The permutation
comes from the oracle here (the device kernel needs a GPU; it is checked bit for bit
against the oracle in test_gpu_parity.py)."""

import torch
import torch.nn as nn

from oracle import solattn_oracle as O
from solb200 import hooks


class _Block(nn.Module):
    """Token-local block: y = 2 x + freqs (freqs broadcast over channels), recording what
    it saw. Token order does not change what a token computes, so the stack's output is
    the same whatever order the tokens arrive in, provided freqs travels with x."""

    def __init__(self, log):
        super().__init__()
        self.log = log

    def forward(self, x, freqs=None, transformer_options=None):
        self.log.append((transformer_options.get("sol_block"), x.clone()))
        return 2 * x + freqs[:, :, 0, :1]


class _Wan(nn.Module):
    def __init__(self, n):
        super().__init__()
        self.log = []
        self.blocks = nn.ModuleList(_Block(self.log) for _ in range(n))

    def rope_encode(self):   # marks the model Wan-style for install_for_model
        return None

    def forward(self, x, freqs, options):
        for b in self.blocks:
            x = b(x, freqs=freqs, transformer_options=options)
        return x


def _oracle_perm(grid, device, curve="3d"):
    p, i = O.morton_perm(tuple(grid), curve)
    return torch.from_numpy(p).to(device), torch.from_numpy(i).to(device)


def _inputs(grid, C=8):
    T = grid[0] * grid[1] * grid[2]
    g = torch.Generator().manual_seed(0)
    x = torch.randn(1, T, C, generator=g)
    freqs = torch.randn(1, T, 1, 4, generator=g)
    return x, freqs


def test_block_index_published():
    m = _Wan(3)
    assert hooks.install_block_index(m)
    assert hooks.install_block_index(m)        # idempotent: one hook per block
    x, freqs = _inputs((1, 4, 4))
    m(x, freqs, {})
    assert [s for s, _ in m.log] == [0, 1, 2]
    assert not hooks.install_block_index(nn.Linear(2, 2))


def test_morton_reorder_roundtrip(monkeypatch):
    monkeypatch.setattr(hooks, "morton_perm", _oracle_perm)
    grid = (2, 4, 8)
    m = _Wan(3)
    setup = hooks.install_for_model(m, morton=True, sink_conditioning="off")
    assert setup["reorder"] and setup["is_wan"]
    x, freqs = _inputs(grid)
    want = m(x, freqs, {})                      # flag off: plain order
    m.log.clear()
    opts = {"sol_morton": True, "sol_morton_curve": "3d", "grid_sizes": grid}
    got = m(x, freqs, opts)
    assert torch.equal(got, want)               # order restored after the last block
    perm, _ = _oracle_perm(grid, "cpu")
    assert torch.equal(m.log[0][1], x.index_select(1, perm))   # block 0 saw Z-order tokens
    # a call whose grid does not match the tokens runs unpermuted
    m.log.clear()
    got = m(x, freqs, {"sol_morton": True, "grid_sizes": (2, 4, 4)})
    assert torch.equal(got, want)
    assert torch.equal(m.log[0][1], x)


def test_morton_2d_frame_curve(monkeypatch):
    monkeypatch.setattr(hooks, "morton_perm", _oracle_perm)
    grid = (3, 4, 4)
    m = _Wan(2)
    hooks.install_wan_morton(m)
    x, freqs = _inputs(grid)
    want = 4 * x + 3 * freqs[:, :, 0, :1]
    got = m(x, freqs, {"sol_morton": True, "sol_morton_curve": "2d_frame", "grid_sizes": grid})
    assert torch.allclose(got, want)
    perm, _ = _oracle_perm(grid, "cpu", "2d_frame")
    assert torch.equal(m.log[0][1], x.index_select(1, perm))
