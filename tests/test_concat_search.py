"""Nested KConcat chains emitted as a binary search over their thresholds (CPU):
the search selects the same piece as the reference's nested conditionals
(opencl/karg.py:52, ``cond ? two : one``) for every index."""

import numpy as np

from ad_b200 import codegen, ir

def nested_pick(k, x, y):
    if isinstance(k, ir.KConcat):
        return nested_pick(k.karg_two if ir.expr_eval(k.condition, 0, x, y) else k.karg_one, x, y)
    return k

def search_pick(k, x, y):
    flat = codegen.concat_pieces(k) if isinstance(k, ir.KConcat) else None
    if flat is None:
        if isinstance(k, ir.KConcat):
            return search_pick(k.karg_two if ir.expr_eval(k.condition, 0, x, y) else k.karg_one, x, y)
        return k
    var, pieces, ths = flat
    v = ir.expr_eval(var, 0, x, y)
    lo, hi = 0, len(pieces)
    while hi - lo > 1:            # the emitted code's search, step for step
        mid = (lo + hi) // 2
        if v > ths[mid]:
            lo = mid
        else:
            hi = mid
    return search_pick(pieces[lo], x, y)

def concat_tree(rng, var, lo, hi, leaf_id, depth=0):
    """Random concat tree over [lo, hi) of ``var``; inner trees over the other axis."""
    if hi - lo < 2 or depth > 6 or rng.random() < 0.15:
        if rng.random() < 0.3 and depth < 3:
            other = ir.Yv() if isinstance(var, ir.Xv) else ir.Xv()
            return concat_tree(rng, other, 0, 64, leaf_id, depth + 1)
        leaf_id[0] += 1
        return ir.KMatrix(leaf_id[0], ir.Gid(), [1])
    cut = int(rng.integers(lo, hi - 1))
    one = concat_tree(rng, var, lo, cut + 1, leaf_id, depth + 1)
    two = concat_tree(rng, var, cut + 1, hi, leaf_id, depth + 1)
    return ir.KConcat(one, two, ir.Bin("MoreThan", var, ir.Const(cut)), [1])

def test_binary_search_matches_nested_conditionals():
    rng = np.random.default_rng(3)
    flattened = 0
    for _ in range(300):
        k = concat_tree(rng, ir.Xv(), 0, 64, [0])
        if isinstance(k, ir.KConcat) and codegen.concat_pieces(k) is not None:
            flattened += 1
        for _ in range(40):
            x, y = (int(v) for v in rng.integers(0, 64, 2))
            assert search_pick(k, x, y) is nested_pick(k, x, y)
    assert flattened > 50

def test_left_deep_chain_flattens():
    X = ir.Xv()
    k = ir.KMatrix(0, ir.Gid(), [1])
    for i in range(1, 256):
        k = ir.KConcat(k, ir.KMatrix(i, ir.Gid(), [1]), ir.Bin("MoreThan", X, ir.Const(128 * i - 1)), [1])
    var, pieces, ths = codegen.concat_pieces(k)
    assert len(pieces) == 256 and ths[1:] == sorted(ths[1:])
    for x in (0, 127, 128, 5000, 32767):
        assert search_pick(k, x, 0) is nested_pick(k, x, 0)
