"""Dot products (``DotProdNode`` / ``DPElwFuse``) on B200.

The reference computes ``C[ty, tx] = sum_k A(_x=ty, _y=k) * B(_x=k, _y=tx)``
one output per work item (opencl/kernels/dotprod.py:7-43) and runs the fused
epilogue with ``_x = ty, _y = tx, _global_id = ty * wB + tx``
(opencl/kernels/dp_elw_fuse.py:11-65).  This module picks the B200 schedule:

* ``simt``: fp32 CUDA-core kernels for tiny products where a tensor-core
  tile would be mostly padding (or with ``AD_DOT_SMALL=simt``): one warp per output for few outputs with a
  long K (``codegen.gen_dot_warp``), 64x64 register tiles otherwise
  (``codegen.gen_dot_simt``).
* ``tc``: tcgen05 tensor cores with 3xTF32: split operands + persistent GEMM
  for large products (``tcgen05.py``), one CTA per 128-row tile with the
  split done in shared memory for small ones (``dot_small.py``).
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
    # Larger products fill the GPU through grouping and split-K.  Smaller ones
    # (per-(sequence, head) attention blocks: 128 x 128 x 64) run on the
    # CUDA-core kernels batched across commands, measured faster than grouped
    # tensor-core launches (4.60 vs 4.98 ms for the 4-layer encoder step).
    tc_min = int(os.environ.get("AD_TC_MIN_MNK", str(1 << 22)))
    return M * N * K >= tc_min and min(M, N) >= 64 and K >= 32


def single_kernel_spec(dev, cmd, name: str, sizes: Dict[int, int]):
    """The CUDA-core kernel of a dot product that does not take the tensor-core
    path (one launch, pointer parameters only), else None."""
    dn, M, N, K = codegen.dot_shape(cmd)
    if use_tensor_cores(dev, M, N, K):
        return None
    return plan_dot(dev, cmd, name, sizes)[0]


def tc_signature(dev, cmd) -> str:
    """Commands with equal signatures can share one grouped tensor-core launch:
    same shapes, operand accesses and epilogue, only their buffers differ."""
    from . import tcgen05
    dn, M, N, K = codegen.dot_shape(cmd)
    bn = tcgen05.tile_n(N)
    gp = tcgen05.GroupPlan([cmd])
    g = tcgen05.gen_gemm(cmd, "k", M, N, K, bn, tcgen05.stages_for(bn))
    return "\n".join(["tc", gp.sa[0].src, gp.sb[0].src, g.src])


def plan_dot(dev, cmd, name: str, sizes: Dict[int, int]) -> List[codegen.KernelSpec]:
    dn, M, N, K = codegen.dot_shape(cmd)
    if use_tensor_cores(dev, M, N, K):
        from . import tcgen05
        return tcgen05.plan(dev, cmd, name, sizes)
    if K >= 32 and M * N <= 4096:
        return [codegen.gen_dot_warp(cmd, name + "_warp", sizes)]
    from . import dot_small
    if use_small_tc(dev, M, N, K):
        return [dot_small.gen_dot_tc(cmd, name + "_small", sizes)]
    return [codegen.gen_dot_simt(cmd, name + "_simt", sizes)]


def use_small_tc(dev, M: int, N: int, K: int) -> bool:
    """Products below the grouped-GEMM threshold run on the one-CTA tcgen05
    kernel (``dot_small``) unless the CUDA-core kernels are asked for."""
    from . import dot_small
    mode = os.environ.get("AD_DOT_SMALL", "tc")
    return mode == "tc" and getattr(dev, "gemm", "auto") != "simt" and dot_small.eligible(M, N, K)


def setup_scratch(dev, proc: ir.Proc) -> None:
    """Scratch for the tensor-core path (split operands), sized for the largest dot."""
    from . import tcgen05
    dev.scratch = {}
    need = 0
    for c in ir.iter_cmds(proc):
        if type(c).__name__ == "Batched" and type(c.cmds[0]).__name__ in ("DotProdNode", "DPElwFuse"):
            dn, M, N, K = codegen.dot_shape(c.cmds[0])
            if use_tensor_cores(dev, M, N, K):
                need = max(need, tcgen05.group_scratch_bytes(c.cmds, dev.ctx.sm_count))
        elif type(c).__name__ in ("DotProdNode", "DPElwFuse"):
            dn, M, N, K = codegen.dot_shape(c)
            if use_tensor_cores(dev, M, N, K):
                need = max(need, tcgen05.group_scratch_bytes([c], dev.ctx.sm_count))
    if need:
        base = dev.ctx.malloc(need)
        dev.scratch_allocs.append(base)
        dev.scratch_base = base
        dev.scratch_bytes = need
