"""The scratch-free dot-product entry point, called through the C ABI (B200 only).

``ad_dot_tf32x3_noalloc`` serves callers that cannot allocate device memory
(a host framework that owns every allocation, or a hot loop that must not
call cudaMalloc/cudaFree because they synchronise the device).  Its scratch is
a fixed array inside the library, shared by every call.  This test checks,
on two calls in a row with different shapes, that its output matches the
library's existing dot-product path (the device plug-in running the same
product through its generated split + tcgen05 kernels, with scratch from the
arena) within the elementwise error bound the dot-product tests use, and that oversize
problems are rejected with an error instead of running.

This file is named so that pytest collects it last.
"""
import ctypes

import numpy as np
import pytest

from tests.procgen import dot_proc

pytestmark = pytest.mark.gpu


def existing_path(A, B, transpose_b):
    from ad_b200.device import CudaB200Device
    d = CudaB200Device(gemm="tc")
    try:
        d.execute(dot_proc(A, B, transpose_b=transpose_b))
        assert any(L.spec.kind == "gemm_tcgen05" for ls in d.launches.values() for L in ls)
        return d.last_received[0]
    finally:
        d.close()


def noalloc_call(ctx, A, B, transpose_b):
    M, K = A.shape
    N = B.shape[0] if transpose_b else B.shape[1]
    a, b, c = ctx.malloc(A.nbytes), ctx.malloc(B.nbytes), ctx.malloc(4 * M * N)
    try:
        A32, B32 = np.ascontiguousarray(A, np.float32), np.ascontiguousarray(B, np.float32)
        ctx.h2d(a, A32.ctypes.data, A32.nbytes, 0)
        ctx.h2d(b, B32.ctypes.data, B32.nbytes, 0)
        ctx.memset(c, 0xFF, 4 * M * N, 0)   # NaN-fill: every output must be written
        ctx.sync()
        rc = ctx.L.ad_dot_tf32x3_noalloc(ctypes.c_void_p(a), ctypes.c_void_p(b), ctypes.c_void_p(c),
                                         M, N, K, int(transpose_b), None)
        assert rc == 0, ctx.L.ad_last_error().decode()
        out = np.empty((M, N), np.float32)
        ctx.d2h(out.ctypes.data, c, out.nbytes, 0)
        ctx.sync()
        return out
    finally:
        for p in (a, b, c):
            ctx.free(p)


def test_noalloc_matches_existing_path_twice():
    from ad_b200 import runtime as rt
    rng = np.random.default_rng(7)
    cases = [((384, 200, 300), True), ((130, 520, 96), False)]
    ctx = rt.Context(0)
    try:
        for (M, K, N), tb in cases:
            A = rng.uniform(-1, 1, (M, K)).astype(np.float32)
            B = rng.uniform(-1, 1, (N, K) if tb else (K, N)).astype(np.float32)
            want = existing_path(A, B, tb)
            got = noalloc_call(ctx, A, B, tb)
            assert np.isfinite(got).all()
            # both are 3xTF32 results with different summation orders (the
            # existing path may split K): compare with the dot-product tests'
            # elementwise bound, |C - C'| <= 1e-4 * (|A| @ |B|) + 1e-5
            Bm = (B.T if tb else B).astype(np.float64)
            bound = 1e-4 * (np.abs(A.astype(np.float64)) @ np.abs(Bm)) + 1e-5
            assert np.all(np.abs(got.astype(np.float64) - want) <= bound)
            assert np.all(np.abs(got - (A.astype(np.float64) @ Bm)) <= bound)
    finally:
        ctx.close()


def test_noalloc_rejects_oversize():
    from ad_b200 import runtime as rt
    ctx = rt.Context(0)
    try:
        # 8 * (4096 + 4096) * 4096 bytes of split operands > the 32 MiB array
        rc = ctx.L.ad_dot_tf32x3_noalloc(ctypes.c_void_p(256), ctypes.c_void_p(256), ctypes.c_void_p(256),
                                         4096, 4096, 4096, 0, None)
        assert rc != 0
        assert "scratch" in ctx.L.ad_last_error().decode()
    finally:
        ctx.close()
