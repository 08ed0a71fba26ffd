"""Generate the golden fixtures in this folder by running the REFERENCE's own Triton
kernels (kijai/ComfyUI-SolAttn_triton) on CPU under ``TRITON_INTERPRET=1``.

Run in a container that has the reference checked out (read-only is fine):

    python tests/golden/make_golden.py --reference /path/to/ComfyUI-SolAttn_triton

Nothing here runs at test time: the tests only read the ``.npz`` files this writes.
The reference is imported from where it lies; no source is copied.

Shims (none changes the reference's arithmetic; each makes the CPU interpreter
evaluate what the kernels mean on a GPU):

1. Package without the ComfyUI ``__init__``: the kernel modules are symlinked into a
   temporary package with an empty ``__init__`` so their relative imports resolve
   without ComfyUI installed.
2. Autotune pinned to one config per kernel (benchmarking needs a GPU driver). The
   configs only pick warps/stages/BV/GROUP; the forward kernels get BV = D and
   GROUP = 64.
3. bf16 ``tl.dot`` and ``tl.sum``: Triton 3.6's interpreter stores bf16 as uint16 and
   runs numpy on the raw bit patterns. Patched to multiply the exact bf16 values in
   fp32 (``np.matmul``) and to sum bf16 in fp32 with one final rounding.
4. fp32 -> bf16 casts: the interpreter truncates the low 16 bits; on a GPU the same
   ``fptrunc`` rounds to nearest even. Patched to round to nearest even.

Block size: the reference hard-codes 64; a 128 case is produced by reassigning the
module constants (``_preprocess.BLOCK_SIZE``, ``_fused_prep.BLOCK_SIZE``,
``_tri_fwd.BLOCK``, ``_int8_fwd.BLOCK``).
"""

from __future__ import annotations

import argparse
import hashlib
import importlib
import os
import sys
import tempfile
import time
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402
import triton  # noqa: E402
import triton.language as tl  # noqa: E402
from triton.runtime import interpreter as interp  # noqa: E402

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO / "comfyui-solattn_triton_b200"))
from solb200.workloads import custom_config, make_qkv  # noqa: E402

MODULES = ["_autotune_log", "_preprocess", "_fused_quant", "_fused_prep", "_tri_fwd",
           "_int8_fwd", "_morton", "_morton_h3"]


# ------------------------------------------------------------------ shims 3 and 4

def _bits_to_f32(u16: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray((u16.astype(np.uint32) << 16).view(np.float32))


def _f32_to_bits_rne(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF).astype(np.uint16)


def install_interpreter_patches():
    Builder = interp.InterpreterBuilder
    orig_dot = Builder.create_dot
    orig_cast = Builder.cast_impl
    orig_fp_to_fp = Builder.create_fp_to_fp
    orig_sum = interp.ReduceOps.sum

    def create_dot(self, a, b, d, input_precision, max_num_imprecise_acc):
        if a.dtype.scalar == tl.bfloat16 and b.dtype.scalar == tl.bfloat16:
            res = np.matmul(_bits_to_f32(a.data), _bits_to_f32(b.data), dtype=np.float32)
            return interp.TensorHandle(res + d.data, d.dtype.scalar)
        return orig_dot(self, a, b, d, input_precision, max_num_imprecise_acc)

    def cast_impl(self, src, dst_type):
        if src.dtype.scalar == tl.float32 and dst_type.scalar == tl.bfloat16:
            return interp.TensorHandle(_f32_to_bits_rne(src.data).reshape(src.data.shape),
                                       dst_type.scalar)
        return orig_cast(self, src, dst_type)

    def create_fp_to_fp(self, src, dst_type, rounding_mode):
        if src.dtype.scalar == tl.float32 and dst_type.scalar == tl.bfloat16:
            return cast_impl(self, src, dst_type)
        return orig_fp_to_fp(self, src, dst_type, rounding_mode)

    def reduce_sum(self, input):
        if input.dtype.scalar == tl.bfloat16:
            s = np.sum(_bits_to_f32(input.handle.data), axis=self.axis,
                       keepdims=self.keep_dims, dtype=np.float32)
            return self.to_tensor(_f32_to_bits_rne(np.asarray(s)).reshape(np.shape(s)),
                                  input.dtype)
        return orig_sum(self, input)

    Builder.create_dot = create_dot
    Builder.cast_impl = cast_impl
    Builder.create_fp_to_fp = create_fp_to_fp
    interp.ReduceOps.sum = reduce_sum


# ------------------------------------------------------------------ shims 1 and 2

def load_reference(ref_dir: Path):
    pkg_root = Path(tempfile.mkdtemp(prefix="solattn_ref_"))
    pkg = pkg_root / "solattn_ref"
    pkg.mkdir()
    (pkg / "__init__.py").write_text("")
    for m in MODULES:
        os.symlink(ref_dir / f"{m}.py", pkg / f"{m}.py")
    sys.path.insert(0, str(pkg_root))
    mods = {m: importlib.import_module(f"solattn_ref.{m}") for m in MODULES}
    return mods


def pin_autotune(mods, head_dim):
    pre, tri, i8 = mods["_preprocess"], mods["_tri_fwd"], mods["_int8_fwd"]
    for kern in (pre._reduce_kc_kernel, pre._reduce_vc_kernel, pre._diag_threshold_kernel):
        kern.configs = [triton.Config({}, num_warps=4, num_stages=2)]
    tri._forward_ptr.configs = [triton.Config({"BV": head_dim, "GROUP_SIZE": 64},
                                              num_warps=4, num_stages=1)]
    i8._forward_int8_ptr.configs = [triton.Config({"BV": head_dim, "GROUP_SIZE": 64},
                                                  num_warps=4, num_stages=1)]
    for kern in (tri._forward_ptr, i8._forward_int8_ptr, pre._reduce_kc_kernel,
                 pre._reduce_vc_kernel, pre._diag_threshold_kernel):
        kern.cache.clear()


def set_block(mods, block):
    mods["_preprocess"].BLOCK_SIZE = block
    mods["_fused_prep"].BLOCK_SIZE = block
    mods["_tri_fwd"].BLOCK = block
    mods["_int8_fwd"].BLOCK = block


# ------------------------------------------------------------------------ cases

def f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy().astype(np.float32)


def run_case(mods, cfg, taus=(), sinks=(), int8=True, dense=True):
    set_block(mods, cfg.block)
    pin_autotune(mods, cfg.head_dim)
    q, k, v = make_qkv(cfg)
    T = q.shape[1]
    scale = cfg.head_dim ** -0.5
    out = dict(q=f32(q), k=f32(k), v=f32(v),
               meta=np.array([cfg.batch, T, cfg.heads, cfg.head_dim, cfg.block]),
               tau=np.float32(cfg.tau))
    pre, fp = mods["_preprocess"], mods["_fused_prep"]
    t0 = time.time()
    kc, vc, thr = pre.prepare(q, k, v, tau=cfg.tau, scale=scale, tokens=T)
    out.update(kc=f32(kc), vc=f32(vc), thr=f32(thr))
    out["o_bf16"] = f32(mods["_tri_fwd"].sol_attn(q, k, v, tau=cfg.tau))
    t_bf16 = time.time() - t0
    if int8:
        t0 = time.time()
        parts = fp.fused_preprocess(q, k, v, tau=cfg.tau, scale=scale, tokens=T)
        names = ["kc", "vc", "thr", "qi", "qs", "ki", "ks", "vi", "vsc"]
        for name, val in zip(names, parts):
            arr = val.detach().cpu()
            out[f"i8_{name}"] = arr.numpy() if arr.dtype in (torch.int8,) else f32(arr)
        out["o_int8"] = f32(mods["_int8_fwd"].sol_attn_int8(q, k, v, tau=cfg.tau))
        out["o_int8_nopv"] = f32(mods["_int8_fwd"].sol_attn_int8(q, k, v, tau=cfg.tau,
                                                                  int8_pv=False))
        out["secs_int8"] = np.float64(time.time() - t0)
    if dense:
        out["o_bf16_dense"] = f32(mods["_tri_fwd"].sol_attn(q, k, v, tau=-1.0e4))
    for tau in taus:
        out[f"o_bf16_tau{tau}"] = f32(mods["_tri_fwd"].sol_attn(q, k, v, tau=tau))
    for i, (sk, sq) in enumerate(sinks):
        out[f"sink{i}"] = np.array([sk[0], sk[1], sq[0], sq[1]])
        out[f"o_bf16_sink{i}"] = f32(mods["_tri_fwd"].sol_attn(q, k, v, tau=cfg.tau,
                                                                sink_blocks=sk, sink_q=sq))
        if int8:
            out[f"o_int8_sink{i}"] = f32(mods["_int8_fwd"].sol_attn_int8(
                q, k, v, tau=cfg.tau, sink_blocks=sk, sink_q=sq))
    out["secs_bf16"] = np.float64(t_bf16)
    return out


def morton_cases(mods):
    mo, h3 = mods["_morton"], mods["_morton_h3"]
    out = {}
    small = [(2, 16, 16), (1, 5, 7), (3, 9, 13), (21, 30, 52)]
    for gi, grid in enumerate(small):
        for curve in ("3d", "2d_frame"):
            perm, inv = mo.morton_perm(grid, "cpu", curve)
            key = f"g{gi}_{curve}"
            out[f"{key}_grid"] = np.array(grid)
            if int(np.prod(grid)) <= 4096:
                out[f"{key}_perm"] = perm.numpy()
                out[f"{key}_inv"] = inv.numpy()
            out[f"{key}_sha"] = np.frombuffer(
                hashlib.sha256(perm.numpy().astype("<i8").tobytes()).digest(), np.uint8)
    # H3 block-aligned rolls (_morton_h3._perm_for) for a few span starts
    for start in (0, 5, 77, 130):
        perm, inv = h3._perm_for((2, 16, 16), "3d", "cpu", start)
        out[f"h3_start{start}_perm"] = perm.numpy()
        out[f"h3_start{start}_inv"] = inv.numpy()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("SOLATTN_REFERENCE"))
    ap.add_argument("--only", default="")
    args = ap.parse_args()
    if not args.reference:
        raise SystemExit("pass --reference <path to the reference checkout>")
    install_interpreter_patches()
    mods = load_reference(Path(args.reference))
    torch.set_num_threads(min(8, os.cpu_count() or 1))

    cases = {
        # config 1 of the headline metric, with the dense (tau=-1e4) and sink checks
        "c1": (custom_config("c1", 1, 2, 64, (2, 16, 16), 64, 0.9, (3, 3, 3), 0),
               dict(taus=(0.3, 1.3), sinks=[((0, 2), (0, 1)), ((1, 3), (0, 0))])),
        # ragged tail: T = 450 tokens, block 64 -> 8 blocks, 2-token tail
        "ragged": (custom_config("ragged", 1, 2, 64, (1, 9, 50), 64, 0.9, (1, 3, 3), 11),
                   dict()),
        # shorter than one block
        "tiny": (custom_config("tiny", 1, 2, 64, (1, 5, 8), 64, 0.9, (1, 2, 2), 12),
                 dict()),
        # D = 128, block 128 (the shape class of configs 2-5), 64-token tail, batch 2
        "d128": (custom_config("d128", 2, 2, 128, (1, 24, 40), 128, 0.9, (1, 3, 3), 13),
                 dict(sinks=[((0, 1), (0, 0))])),
        # more than one 64-block routing group (68 blocks)
        "groups": (custom_config("groups", 1, 1, 64, (1, 65, 66), 64, 0.9, (1, 3, 3), 14),
                   dict(dense=False)),
    }
    only = set(args.only.split(",")) if args.only else None
    for name, (cfg, kw) in cases.items():
        if only and name not in only:
            continue
        t0 = time.time()
        res = run_case(mods, cfg, **kw)
        np.savez_compressed(HERE / f"{name}.npz", **res)
        print(f"{name}: {time.time() - t0:.1f}s", flush=True)
    if not only or "morton" in only:
        np.savez_compressed(HERE / "morton.npz", **morton_cases(mods))
        print("morton: done")


if __name__ == "__main__":
    main()
