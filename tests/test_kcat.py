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


def _synthetic(reader_between: bool):
    """C = A0 @ W0 + A1 @ W1 as the reference's fusion emits it: the product
    A1 @ W1 as its own command, W1 updated in place (``W1 += 1``) after it, and
    a ``DPElwFuse`` whose dot A0 @ W0 heads an ADD of the product.  With
    ``reader_between`` a command between the update and the sum reads W1, so
    the update cannot move past it."""
    rng = np.random.default_rng(1)
    M, K, N = 64, 32, 48
    G = ir.Gid()

    def rm(ld):
        return ir.Bin("Add", ir.Bin("Mult", ir.Xv(), ir.Const(ld)), ir.Yv())

    arrs = {1: (M, K), 2: (K, N), 3: (M, K), 4: (K, N)}
    cmds = [ir.AllocEntry(i, a * b, rng.standard_normal(a * b).astype(np.float32)) for i, (a, b) in arrs.items()]
    cmds += [ir.AllocEntry(5, M * N), ir.AllocEntry(6, M * N), ir.AllocEntry(7, K * N)]
    cmds.append(ir.DotProdNode(5, [ir.KMatrix(3, rm(K), [M, K]), ir.KMatrix(4, rm(N), [K, N])],
                               ir.KMatrix(5, rm(N), [M, N]), [M, N], [[M, K], [K, N]]))
    cmds.append(ir.BinaryNode(4, "ADD", [ir.KMatrix(4, G, [K, N]), ir.KConstant(1.0)],
                              ir.KMatrix(4, G, [K, N]), [K, N], True))
    if reader_between:
        cmds.append(ir.BinaryNode(7, "MULT", [ir.KMatrix(4, G, [K, N]), ir.KConstant(2.0)],
                                  ir.KMatrix(7, G, [K, N]), [K, N]))
    nodes = [ir.AllocEntry(8, M * N, None, True),
             ir.DotProdNode(8, [ir.KMatrix(1, rm(K), [M, K]), ir.KMatrix(2, rm(N), [K, N])],
                            ir.KMatrix(8, None, [M, N], True), [M, N], [[M, K], [K, N]]),
             ir.BinaryNode(6, "ADD", [ir.KMatrix(8, None, [M, N], True), ir.KMatrix(5, G, [M, N])],
                           ir.KMatrix(6, G, [M, N]), [M, N])]
    cmds.append(ir.DPElwFuse(nodes, 1))
    outs = [ir.KMatrix(6, G, [M, N]), ir.KMatrix(4, G, [K, N])]
    if reader_between:
        outs.append(ir.KMatrix(7, G, [K, N]))
    cmds.append(ir.Receiver(99, outs, "out"))
    return ir.Proc(cmds)


@pytest.mark.parametrize("reader_between", [False, True])
def test_update_between_product_and_sum(monkeypatch, reader_between):
    monkeypatch.setattr(kcat, "MIN_TERMS", 1)
    want = _run(_synthetic(reader_between))
    q = _synthetic(reader_between)
    n = kcat.fuse_ksums(q)
    kinds = [type(c).__name__ for c in q.procedure]
    if reader_between:
        # the update must stay before its reader, so the product stays before the update
        assert n == 0 and kinds.count("DotProdNode") == 1
    else:
        # folded; the update now runs after the sum, which reads the weight before it
        assert n == 1 and "DotProdNode" not in kinds
        assert kinds.index("BinaryNode") > kinds.index("DPElwFuse")
    for g, w in zip(_run(q), want):
        np.testing.assert_allclose(g, w, rtol=1e-5, atol=1e-5)
