"""The C-ABI library loads without a GPU and exports every symbol its header declares."""
import ctypes
import os
import re

from ad_b200 import runtime as rt

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared():
    src = open(os.path.join(ROOT, "include", "ad_b200.h")).read()
    return sorted(set(re.findall(r"^(?:int|void|const char\*)\s+(ad_\w+)\s*\(", src, re.M)))


def test_exports_every_declared_symbol():
    L = rt.lib()
    names = declared()
    assert len(names) >= 30
    for n in names:
        assert hasattr(L, n), n
    assert set(names) == set(rt.SIGNATURES), set(names) ^ set(rt.SIGNATURES)


def test_version_and_errors_without_gpu():
    L = rt.lib()
    assert L.ad_version() == 1
    # a call that must fail cleanly (null context) reports a message
    assert L.ad_stream_sync(None, 0) != 0
    assert b"null context" in L.ad_last_error()


def test_nvrtc_compiles_sm100a():
    cub = rt.compile_cubin('extern "C" __global__ void k(float* p) { p[threadIdx.x] = 1.0f; }', "t.cu")
    assert len(cub) > 100


def test_host_copy_threads():
    """ad_host_copy (the Feeder staging copy) on sizes around its split points."""
    import numpy as np
    from ad_b200 import runtime as rt
    rng = np.random.default_rng(3)
    for n in (0, 1, 4095, 1 << 20, (1 << 20) + 3, (7 << 20) + 12345, 33 << 20):
        src = rng.integers(0, 255, n, dtype=np.uint8)
        dst = np.zeros(n + 16, np.uint8)
        rt.host_copy(dst.ctypes.data, src.ctypes.data, n)
        assert np.array_equal(dst[:n], src) and not dst[n:].any()


def test_small_dot_kernel_compiles_for_sm100a():
    """The one-CTA tcgen05 dot kernel (dot_small) builds for the encoder's
    attention shapes, with ptxas's limits met (NVRTC straight to a cubin)."""
    from ad_b200 import dot_small
    from tests.procgen import dot_proc
    import numpy as np
    for M, N, K, tb in ((128, 128, 64, True), (128, 64, 128, False), (130, 300, 17, True)):
        proc = dot_proc(np.zeros((M, K), np.float32), np.zeros((N, K) if tb else (K, N), np.float32),
                        transpose_b=tb)
        cmd = next(c for c in proc.procedure if type(c).__name__ in ("DotProdNode", "DPElwFuse"))
        sp = dot_small.gen_dot_tc(cmd, "k_dot_tc", {})
        assert sp.kind == "dot_tc" and sp.smem <= 225 * 1024
        assert len(rt.compile_cubin(sp.src, "k_dot_tc.cu")) > 1000
