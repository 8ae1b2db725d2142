"""Every kernel that the benchmarked procs launch compiles for sm_100a (CPU).

The device passes and code generators run offline (no GPU context) over the
procs that ``bench.py`` times -- config 4's encoder (single GPU and the
data-parallel rewrite), config 3's 4096^3 product, config 2's LayerNorm +
softmax -- and each distinct generated source goes through NVRTC to an
sm_100a cubin, with ptxas's limits checked.  Tensor maps need the CUDA driver
and are not part of a kernel's source, so they are stubbed here.
"""
from concurrent.futures import ThreadPoolExecutor

import pytest

from ad_b200 import ir, memplan, runtime as rt
from ad_b200.device import CudaB200Device
from ad_b200.fixtures import load_case

NON_KERNEL = ("AllocEntry", "DeallocEntry", "ForNode", "AllReduce", "AllReduceWait", "Feeder", "Receiver")


def kernel_sources(case: str, world: int = 1, gemm: str = "auto"):
    p, _ = load_case(case, with_content=False)
    d = CudaB200Device.offline(gemm=gemm, world=world)
    proc = d.transform(p)
    d.slots, _ = memplan.plan(proc)
    d.err_ptr, d.scratch_base, d.scratch_bytes, d.scratch = 0, 0, 1 << 40, {}
    srcs = {}
    for c in ir.iter_cmds(proc):
        if type(c).__name__ in NON_KERNEL:
            continue
        for s in d._specs_for(c):
            srcs.setdefault(s.src, s)
    return list(srcs.values())


@pytest.mark.parametrize("case,world", [("enc_4_32_128_512_8_2048_100", 1),
                                        ("enc_4_32_128_512_8_2048_100", 2),
                                        ("dotsig_4096", 1),
                                        ("lnsm_8192_4096", 1)])
def test_bench_proc_kernels_compile(monkeypatch, case, world):
    monkeypatch.setattr(rt, "tmap_2d", lambda *a, **k: bytes(128))
    specs = kernel_sources(case, world)
    assert specs
    kinds = {s.kind for s in specs}
    if case.startswith("enc"):
        assert {"gemm_tcgen05", "split", "rowfused"} <= kinds, kinds
    with ThreadPoolExecutor(16) as ex:
        sizes = list(ex.map(lambda s: len(rt.compile_cubin(s.src, s.name + ".cu")), specs))
    assert all(n > 500 for n in sizes)
    assert all(s.smem <= 227 * 1024 for s in specs)
