"""The C-ABI boundary without a GPU: the library loads, exports every entry point the
header declares, and rejects bad arguments with the documented status codes before
touching a device."""

import ctypes
import re
from pathlib import Path

import pytest
import torch

from conftest import REPO

import solb200
from solb200 import _lib


def header_symbols():
    text = (REPO / "include" / "solb200.h").read_text()
    return sorted(set(re.findall(r"\b(solb200_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    declared = header_symbols()
    assert declared, "no declarations found in include/solb200.h"
    for name in declared:
        assert hasattr(lib, name), f"{name} declared but not exported"
    assert set(declared) == set(_lib.exported_symbols())
    assert lib.solb200_abi_version() == 2


def test_workspace_plan_without_gpu():
    n = solb200.workspace_bytes(1, 32760, 40, 128, 128, False)
    # kc + vc dominate: 2 * 256 blocks * 40 heads * 128 * 2 bytes
    assert 2 * 256 * 40 * 128 * 2 < n < 16 * 1024 * 1024
    n8 = solb200.workspace_bytes(1, 32760, 40, 128, 128, True)
    assert n8 > 3 * 32760 * 40 * 128   # qi, ki, vi
    offs = [solb200.ops._offset((1, 4096, 24, 128, 128, 1), w) for w in _lib.BUF]
    assert offs == sorted(offs) and all(o % 256 == 0 for o in offs)


@pytest.mark.parametrize("args, code", [
    ((1, 512, 2, 96, 64, 0), 1),     # head_dim 96
    ((1, 512, 2, 64, 32, 0), 1),     # block 32
    ((0, 512, 2, 64, 64, 0), 1),     # empty batch
    ((1, 0, 2, 64, 64, 0), 1),       # no tokens
])
def test_plan_rejects_bad_geometry(args, code):
    n = ctypes.c_int64(0)
    rc = _lib.lib().solb200_workspace_bytes(*args, ctypes.byref(n))
    assert rc == code
    assert _lib.last_error()


def test_int8_workspace_holds_only_int8_operands():
    """The INT8 workspace holds the int8 codes and their scales, no bf16 copies of them:
    beyond the BF16 workspace it adds qi, ki, vi (1 byte per element), the per-token Q / K
    scales, the per-block |V| max and the V scales."""
    B, T, H, D, blk = 1, 4096, 4, 128, 128
    bf16 = solb200.workspace_bytes(B, T, H, D, blk, False)
    int8 = solb200.workspace_bytes(B, T, H, D, blk, True)
    N = T // blk
    extra = 3 * B * T * H * D + 2 * 4 * B * H * N * blk + 4 * B * N * H * D + 4 * B * H * D
    assert int8 - bf16 <= extra + 8 * 256          # plus 256-byte alignment of each buffer
    n = ctypes.c_int64(0)
    assert _lib.lib().solb200_workspace_offset(B, T, H, D, blk, 1, 17, ctypes.byref(n)) == 1
    assert _lib.lib().solb200_abi_version() == 2


def test_offset_of_int8_buffer_in_bf16_workspace_is_an_error():
    n = ctypes.c_int64(0)
    rc = _lib.lib().solb200_workspace_offset(1, 512, 2, 64, 64, 0, _lib.BUF["qi"], ctypes.byref(n))
    assert rc == 1


def test_ops_refuse_cpu_tensors():
    q = torch.zeros(1, 64, 2, 64, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        solb200.sol_attn(q, q, q)
    with pytest.raises(RuntimeError, match="CUDA"):
        solb200.sol_attn_int8(q, q, q)


def test_product_package_does_not_import_the_oracle():
    pkg = REPO / "comfyui-solattn_triton_b200"
    for f in pkg.rglob("*.py"):
        text = f.read_text()
        assert "oracle" not in re.sub(r"#.*", "", text).split("\"\"\"")[0] or "import oracle" not in text
        assert "from oracle" not in text and "import oracle" not in text, f
