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


def test_schedule_respects_dependencies():
    """Re-scheduled commands never read a buffer before its writer nor overwrite
    one a pending reader needs; host commands keep their order."""
    p, _ = load_case("enc_1_8_128_512_8_2048_100", with_content=False)
    body = [c for c in next(c for c in p.procedure if isinstance(c, ir.ForNode)).proc.procedure
            if type(c).__name__ not in ("AllocEntry", "DeallocEntry")]
    out = batch.schedule(body, lambda c: type(c).__name__ if type(c).__name__ in ir.COMPUTE_KINDS else None)
    flat = []
    for c in out:
        flat += c.cmds if isinstance(c, batch.Batched) else [c]
    assert sorted(map(id, flat)) == sorted(map(id, body))
    pos = {id(c): i for i, c in enumerate(body)}
    # for every pair in original order with a conflict, relative order is kept
    rw = [batch._rw(c) for c in body]
    newpos = {}
    i = 0
    for c in out:
        for m in (c.cmds if isinstance(c, batch.Batched) else [c]):
            newpos[id(m)] = i
        i += 1
    for a in range(len(body)):
        for b in range(a + 1, min(len(body), a + 60)):
            ra, wa = rw[a]
            rb, wb = rw[b]
            if (wa & rb) or (ra & wb) or (wa & wb):
                assert newpos[id(body[a])] < newpos[id(body[b])]
