"""Offset folding and dependency-level batching (CPU)."""
import numpy as np

from ad_b200 import batch, codegen, ir
from ad_b200.fixtures import load_case
from tests.test_ir import rand_expr


def test_split_offset_preserves_value():
    rng = np.random.default_rng(1)
    for _ in range(2000):
        e = rand_expr(rng)
        r, c = codegen.split_offset(e)
        for _ in range(8):
            g, x, y = (int(v) for v in rng.integers(0, 100, 3))
            assert ir.expr_eval(e, g, x, y) == ir.expr_eval(r, g, x, y) + c


def test_slice_offset_moves_into_pointer():
    X, Y = ir.Xv(), ir.Yv()
    e = ir.Bin("Add", ir.Bin("ShiftLeft", ir.Bin("Add", X, ir.Const(896)), ir.Const(6)), Y)
    k = ir.KMatrix(5, e, [128, 64])
    assert codegen.view_of(k, set()) == (5, 896 * 64)
    assert codegen.view_of(k, {5}) == (5, 0)       # written buffers keep offsets in the index


def _check_order(body, out):
    """Every conflicting pair (same buffer, at least one write) keeps its order,
    so members of one batched launch never conflict; host commands keep order."""
    newpos = {}
    for i, c in enumerate(out):
        for m in (c.cmds if isinstance(c, batch.Batched) else [c]):
            newpos[id(m)] = i
    assert sorted(newpos) == sorted(map(id, body))
    host = [newpos[id(c)] for c in body if type(c).__name__ in batch.HOST]
    assert host == sorted(host)
    last_w, readers = {}, {}
    for c in body:
        r, w = batch._rw(c)
        pc = newpos[id(c)]
        for b in r:
            assert last_w.get(b, -1) < pc
        for b in w:
            assert last_w.get(b, -1) < pc
            assert all(q < pc for q in readers.get(b, []))
        for b in r:
            readers.setdefault(b, []).append(pc)
        for b in w:
            last_w[b] = pc
            readers[b] = []


def test_schedule_respects_dependencies():
    """Re-scheduled commands never read a buffer before its writer nor overwrite
    one a pending reader needs; host commands keep their order."""
    p, _ = load_case("enc_1_8_128_512_8_2048_100", with_content=False)
    body = [c for c in next(c for c in p.procedure if isinstance(c, ir.ForNode)).proc.procedure
            if type(c).__name__ not in ("AllocEntry", "DeallocEntry")]
    out = batch.schedule(body, lambda c: type(c).__name__ if type(c).__name__ in ir.COMPUTE_KINDS else None)
    _check_order(body, out)


def test_device_passes_keep_dependencies_and_batch():
    """The device's pass pipeline (split horizontal groups, row fusion, then
    batching with the device's kernel signatures) on the 4-layer encoder:
    dependency order preserved, and ~10k per-(sequence, head) commands
    collapse into under 200 launches-worth of commands."""
    from ad_b200.device import CudaB200Device
    p, _ = load_case("enc_4_32_128_512_8_2048_100", with_content=False)
    dev = CudaB200Device.offline(batch=False)
    proc = dev.transform(p)
    body = [c for c in next(c for c in proc.procedure if isinstance(c, ir.ForNode)).proc.procedure
            if type(c).__name__ not in ("AllocEntry", "DeallocEntry")]
    sizes = {c.id: c.size for c in ir.iter_cmds(proc) if isinstance(c, ir.AllocEntry) and not c.is_temp}
    out = batch.schedule(body, lambda c: dev.batch_signature(c, sizes))
    _check_order(body, out)
    assert len(body) > 2000 and len(out) < 200


def test_hsplit_preserves_results():
    """Splitting horizontally fused elementwise groups into their components
    changes no result (oracle, bit-exact) on the small encoder."""
    from ad_b200 import hsplit
    from oracle.cexec import OracleDevice
    outs = []
    for split in (False, True):
        p, _ = load_case("enc_1_2_16_32_2_64_3")
        p = ir.conv_proc(p)
        if split:
            assert hsplit.split_groups(p) > 0
        o = OracleDevice(faithful_tree=False)
        o.execute(p)
        outs.append(o.last_received)
    for a, b in zip(*outs):
        np.testing.assert_array_equal(a, b)
