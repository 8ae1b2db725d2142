"""IR mirror: JSON round trip, expression semantics and analyses (CPU)."""
import glob
import os

import numpy as np
import pytest

from ad_b200 import exprs, ir, memplan
from ad_b200.fixtures import PROC_DIR, load_case

CASES = sorted(os.path.basename(f)[:-8] for f in glob.glob(os.path.join(PROC_DIR, "*.json.gz")))


@pytest.mark.parametrize("case", CASES)
def test_roundtrip(case, tmp_path):
    p, m = load_case(case, with_content=False)
    path = str(tmp_path / "p.json.gz")
    ir.save_proc(p, path, m)
    q, m2 = ir.load_proc(path)
    assert ir.proc_to_json(p) == ir.proc_to_json(q)
    assert m2 == m


def rand_expr(rng, depth=0):
    if depth > 3 or rng.random() < 0.3:
        r = rng.integers(0, 4)
        return [ir.Gid(), ir.Xv(), ir.Yv(), ir.Const(int(rng.integers(1, 64)))][r]
    op = ["Add", "Mult", "Div", "Remainder", "ShiftRight", "ShiftLeft", "BitwiseAnd"][rng.integers(0, 7)]
    a = rand_expr(rng, depth + 1)
    if op in ("Div", "Remainder", "ShiftRight", "ShiftLeft", "BitwiseAnd", "Mult"):
        c = int(rng.integers(1, 9)) if op in ("ShiftRight", "ShiftLeft") else int(rng.choice([1, 3, 4, 8, 16, 255, 256]))
        return ir.Bin(op, a, ir.Const(c))
    return ir.Bin(op, a, rand_expr(rng, depth + 1))


def test_bounds_and_lanes_sound():
    rng = np.random.default_rng(0)
    vec = 4
    for _ in range(400):
        e = rand_expr(rng)
        R = {"G": (0, 1023), "X": (0, 31), "Y": (0, 63)}
        lo, hi = exprs.bounds(e, R)
        for _ in range(40):
            g, x, y = int(rng.integers(0, 1024)), int(rng.integers(0, 32)), int(rng.integers(0, 64))
            v = ir.expr_eval(e, g, x, y)
            assert lo <= v <= hi
        ln = exprs.lanes(e, "G", vec)
        if ln.s is not None:
            for _ in range(20):
                base = int(rng.integers(0, 256)) * vec
                x, y = int(rng.integers(0, 32)), int(rng.integers(0, 64))
                v0 = ir.expr_eval(e, base, x, y)
                assert v0 % ln.a == 0 or ln.a == 1 or v0 == 0, (ir.expr_str(e), ln)
                for j in range(vec):
                    assert ir.expr_eval(e, base + j, x, y) == v0 + ln.s * j, (ir.expr_str(e), ln)


@pytest.mark.parametrize("case", ["lnsm_64_256", "mlp", "dotsig_256", "unary+tetris"])
def test_memplan_no_overlap(case):
    p, _ = load_case(case, with_content=False)
    slots, total = memplan.plan(p)
    s = list(slots.values())
    for i in range(len(s)):
        assert s[i].offset % memplan.ALIGN == 0
        assert s[i].offset + s[i].nbytes <= total
        for j in range(i + 1, len(s)):
            a, b = s[i], s[j]
            live = not (a.end < b.start or b.end < a.start)
            mem = not (a.offset + a.nbytes <= b.offset or b.offset + b.nbytes <= a.offset)
            assert not (live and mem), (a, b)
