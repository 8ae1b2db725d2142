"""Sums of dot products folded into one dot over the concatenated K axis (CPU).

``ad_b200.kcat.fuse_ksums`` is a rewrite of the proc, so the oracle checks it
directly: the rewritten proc, executed by the oracle, gives the original
proc's results up to the rounding of the changed summation order, and is at
least as close to the float64 evaluation of the original.  On the traced
encoders every per-head input-gradient product of every layer but the first
is folded in, with the weight updates that sat between a product and the sum
moved after the sum.
"""
import numpy as np
import pytest

from ad_b200 import dist, ir, kcat
from ad_b200.fixtures import load_case, set_loop_count
from oracle.cexec import OracleDevice


def _run(proc, f64=False):
    o = OracleDevice(faithful_tree=False, f64=f64)
    o.execute(proc)
    return o.last_received


def _prepared(case, loops=None):
    p, _ = load_case(case)
    if loops is not None:
        set_loop_count(p, loops)
    return ir.copy_structure(ir.conv_proc(p))


def test_folded_proc_matches_original_on_the_oracle():
    case = "encdy_2_2_16_32_2_64_3_lr4"        # 2 layers, 2 heads, 3 SGD steps
    want = _run(_prepared(case))
    exact = _run(_prepared(case), f64=True)
    q = _prepared(case)
    before = {id(c): i for i, c in enumerate(_loop_body(q))}
    assert kcat.fuse_ksums(q) == 5             # 3 x 2 heads - 1 products, second layer
    # a weight update that sat between a product and the sum now runs after the sum
    order = [before[id(c)] for c in _loop_body(q) if id(c) in before]
    assert any(b < a for a, b in zip(order, order[1:]))
    got = _run(q)
    assert all(np.isfinite(w).all() for w in want)
    for g, w, e in zip(got, want, exact):
        np.testing.assert_allclose(g, w, rtol=1e-5, atol=1e-7)
        assert np.abs(g - e).max() <= 2 * np.abs(w - e).max() + 1e-7


def _loop_body(q):
    return next(c for c in q.procedure if isinstance(c, ir.ForNode)).proc.procedure


@pytest.mark.parametrize("case,world,n", [("enc_4_32_128_512_8_2048_100", 1, 69),
                                          ("enc_4_32_128_512_8_2048_100_p2", 2, 69),
                                          ("enc_12_256_512_1024_16_4096_50_p8", 8, 11 * 47)])
def test_encoder_products_folded(case, world, n):
    p, _ = load_case(case, with_content=False)
    q = ir.copy_structure(ir.conv_proc(p))
    if world > 1:
        dist.insert_grad_allreduce(q)
    before = sum(type(c).__name__ == "DotProdNode" for c in _loop_body(q))
    assert kcat.fuse_ksums(q) == n
    after = sum(type(c).__name__ == "DotProdNode" for c in _loop_body(q))
    assert before - after == n
    # the folded dots: K = 3 x heads x 64 (every Q/K/V projection of every head)
    heads = 16 if "1024" in case else 8
    folded = [c for c in _loop_body(q) if type(c).__name__ == "DPElwFuse"
              and c.init_node.children_shapes[0][1] == 3 * heads * 64]
    assert len(folded) == n // (3 * heads - 1)
