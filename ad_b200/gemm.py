"""Dot products (``DotProdNode`` / ``DPElwFuse``) on B200.

The reference computes ``C[ty, tx] = sum_k A(_x=ty, _y=k) * B(_x=k, _y=tx)``
one output per work item (opencl/kernels/dotprod.py:7-43) and runs the fused
epilogue with ``_x = ty, _y = tx, _global_id = ty * wB + tx``
(opencl/kernels/dp_elw_fuse.py:11-65).  This module picks the B200 schedule:

* ``simt``: fp32 CUDA-core kernels for tiny products where a tensor-core
  tile would be mostly padding: one warp per output for few outputs with a
  long K (``codegen.gen_dot_warp``), 64x64 register tiles otherwise
  (``codegen.gen_dot_simt``).
* ``tc``: tcgen05 tensor cores with 3xTF32 (see ``tcgen05.py``).
"""
from __future__ import annotations

import os
from typing import Dict, List

from . import codegen, ir


def use_tensor_cores(dev, M: int, N: int, K: int) -> bool:
    mode = getattr(dev, "gemm", "auto")
    if mode == "simt":
        return False
    if mode == "tc":
        return True
    if M * N * K < (1 << 21) or min(M, N) < 16 or K < 8:
        return False
    # too few output tiles to occupy the GPU: the CUDA-core kernel, which batches
    # across independent commands (e.g. per-head projections), does better
    from .tcgen05 import BM, pad, tile_n
    tiles = (pad(M, BM) // BM) * (pad(N, tile_n(N)) // tile_n(N))
    min_tiles = int(os.environ.get("AD_TC_MIN_TILES", "64"))
    return tiles >= min_tiles or (tiles >= 8 and M * N * K >= (1 << 27) and min_tiles <= 64)


def single_kernel_spec(dev, cmd, name: str, sizes: Dict[int, int]):
    """The CUDA-core kernel of a dot product that does not take the tensor-core
    path (one launch, pointer parameters only), else None."""
    dn, M, N, K = codegen.dot_shape(cmd)
    if use_tensor_cores(dev, M, N, K):
        return None
    return plan_dot(dev, cmd, name, sizes)[0]


def plan_dot(dev, cmd, name: str, sizes: Dict[int, int]) -> List[codegen.KernelSpec]:
    dn, M, N, K = codegen.dot_shape(cmd)
    if use_tensor_cores(dev, M, N, K):
        from . import tcgen05
        return tcgen05.plan(dev, cmd, name, sizes)
    if K >= 32 and M * N <= 4096:
        return [codegen.gen_dot_warp(cmd, name + "_warp", sizes)]
    return [codegen.gen_dot_simt(cmd, name + "_simt", sizes)]


def setup_scratch(dev, proc: ir.Proc) -> None:
    """Scratch for the tensor-core path (split operands), sized for the largest dot."""
    dev.scratch = {}
    need = 0
    for c in ir.iter_cmds(proc):
        if type(c).__name__ in ("DotProdNode", "DPElwFuse"):
            dn, M, N, K = codegen.dot_shape(c)
            if use_tensor_cores(dev, M, N, K):
                from . import tcgen05
                need = max(need, tcgen05.scratch_bytes(M, N, K))
    if need:
        base = dev.ctx.malloc(need)
        dev.scratch_allocs.append(base)
        dev.scratch_base = base
        dev.scratch_bytes = need
