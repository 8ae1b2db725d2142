"""Tensor-core dots whose operands are concatenations (B200 only).

A traced transformer feeds the output projection with the heads' outputs
concatenated along the feature axis, each head's output itself concatenated
over the sequences of the batch (``nn/transformer.py:20-45``: one buffer per
(sequence, head)).  The split kernel reads such an operand a float4 at a time
when every concatenation boundary along the 4-wide lane axis is a multiple of
4 (one piece per float4, chosen by a binary search over the thresholds), and
element by element otherwise.  Both cases, for A and for a transposed B, are
checked against float64 with the 3xTF32 bound
``|C - C64| <= 1e-4 |A||B| + 1e-5``.
"""
import numpy as np
import pytest

from ad_b200 import ir
from tests.procgen import C, add, mul

pytestmark = pytest.mark.gpu

X, Y = ir.Xv(), ir.Yv()


def concat2d(ids, widths, heights, mats, transposed=False):
    """Operand ``[sum(heights), sum(widths)]`` as a concat along columns of
    concats along rows; piece (i, j) is buffer ``ids[i][j]`` (row-major
    ``heights[j] x widths[i]``).  ``transposed`` builds the same matrix seen
    as a ``.T()`` B operand: element (k = row, n = column) at (X = k, Y = n)
    with the roles of X and Y swapped in the conditions and accesses."""
    r_var, c_var = (Y, X) if transposed else (X, Y)

    def col_piece(i):
        node = None
        r0 = 0
        for j, h in enumerate(heights):
            acc = add(mul(ir.Bin("Minus", r_var, C(r0)), C(widths[i])), ir.Bin("Minus", c_var, C(sum(widths[:i]))))
            leaf = ir.KMatrix(ids[i][j], acc, [h, widths[i]])
            node = leaf if node is None else ir.KConcat(node, leaf, ir.Bin("MoreThan", r_var, C(r0 - 1)),
                                                        [r0 + h, widths[i]])
            r0 += h
        return node

    node = None
    c0 = 0
    for i, w in enumerate(widths):
        piece = col_piece(i)
        node = piece if node is None else ir.KConcat(node, piece, ir.Bin("MoreThan", c_var, C(c0 - 1)),
                                                     [sum(heights), c0 + w])
        c0 += w
    return node


def run_concat_dot(widths, heights, N, b_concat):
    from ad_b200.device import CudaB200Device
    rng = np.random.default_rng(len(widths) * 100 + len(heights))
    M, K = sum(heights), sum(widths)
    procs, ids, nxt = [], [], 100
    pieces = {}
    for i, w in enumerate(widths):
        ids.append([])
        for j, h in enumerate(heights):
            a = rng.standard_normal((h, w)).astype(np.float32)
            pieces[(i, j)] = a
            procs.append(ir.AllocEntry(nxt, a.size, a.reshape(-1)))
            ids[-1].append(nxt)
            nxt += 1
    A = np.block([[pieces[(i, j)] for i in range(len(widths))] for j in range(len(heights))])
    Bm = rng.standard_normal((K, N)).astype(np.float32)
    if b_concat:
        # the concatenated matrix is B^T: B(k, n) = A(n, k), N = M
        ka = ir.KMatrix(1, add(mul(X, C(K)), Y), [M, K])
        procs.append(ir.AllocEntry(1, A.size, A.reshape(-1)))
        kb = concat2d(ids, widths, heights, pieces, transposed=True)
        left, right, n_out = A, A.T, M
    else:
        ka = concat2d(ids, widths, heights, pieces)
        procs.append(ir.AllocEntry(2, Bm.size, Bm.reshape(-1)))
        kb = ir.KMatrix(2, add(mul(X, C(N)), Y), [K, N])
        left, right, n_out = A, Bm, N
    procs.append(ir.AllocEntry(3, M * n_out))
    procs.append(ir.DotProdNode(10, [ka, kb], ir.KMatrix(3, add(mul(X, C(n_out)), Y), [M, n_out]),
                                [M, n_out], [[M, K], [K, n_out]]))
    procs.append(ir.Receiver(20, [ir.KMatrix(3, ir.Gid(), [M, n_out])], "out"))
    d = CudaB200Device(gemm="tc")
    try:
        d.execute(ir.Proc(procs))
        got = d.last_received[0].reshape(M, n_out).astype(np.float64)
        kinds = {L.spec.kind for ls in d.launches.values() for L in ls}
    finally:
        d.close()
    assert "gemm_tcgen05" in kinds
    ref = left.astype(np.float64) @ right.astype(np.float64)
    bound = 1e-4 * (np.abs(left).astype(np.float64) @ np.abs(right).astype(np.float64)) + 1e-5
    assert np.all(np.abs(got - ref) <= bound)


@pytest.mark.parametrize("widths,heights", [
    ([64] * 8, [128] * 8),          # heads x sequences, every boundary on a float4
    ([20, 44, 12, 52], [100, 156]),  # ragged pieces, boundaries still multiples of 4
    ([6, 10, 48, 17], [64, 64, 3]),  # boundaries off the float4 grid: element-wise reads
])
@pytest.mark.parametrize("b_concat", [False, True])
def test_concat_operand_split(widths, heights, b_concat):
    run_concat_dot(widths, heights, 192, b_concat)
