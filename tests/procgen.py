"""Small hand-built procs in the reference's IR shape, for kernel-level tests.

They follow what the reference's kernalize emits for the same graphs:
row-major ``(X * ld) + Y`` accesses for dot/reduce operands, ``(Y * ld) + X``
for a ``.T()`` operand (kernalize.py:71-114 via helper.py:52-73), ``Global``
for elementwise results.
"""
import numpy as np

from ad_b200 import ir

G, X, Y = ir.Gid(), ir.Xv(), ir.Yv()


def C(v):
    return ir.Const(v)


def add(a, b):
    return ir.Bin("Add", a, b)


def mul(a, b):
    return ir.Bin("Mult", a, b)


def rowmaj(ld):
    return add(mul(X, C(ld)), Y)


def colmaj(ld):
    return add(mul(Y, C(ld)), X)


def dot_proc(A: np.ndarray, B: np.ndarray, transpose_b=False, bias=None, epi_scale=None):
    """C = A @ (B.T if transpose_b else B) [+ bias broadcast over rows] [* scale]."""
    M, K = A.shape
    N = B.shape[0] if transpose_b else B.shape[1]
    a = ir.AllocEntry(1, A.size, A.astype(np.float32).reshape(-1))
    b = ir.AllocEntry(2, B.size, B.astype(np.float32).reshape(-1))
    c = ir.AllocEntry(3, M * N)
    procs = [a, b, c]
    ka = ir.KMatrix(1, rowmaj(K), [M, K])
    kb = ir.KMatrix(2, colmaj(K) if transpose_b else rowmaj(N), [K, N])
    if bias is None and epi_scale is None:
        dn = ir.DotProdNode(10, [ka, kb], ir.KMatrix(3, rowmaj(N), [M, N]), [M, N], [[M, K], [K, N]])
        procs.append(dn)
    else:
        nodes = [ir.AllocEntry(10, M * N, None, True)]
        dn = ir.DotProdNode(10, [ka, kb], ir.KMatrix(10, None, [M, N], True), [M, N], [[M, K], [K, N]])
        nodes.append(dn)
        cur = ir.KMatrix(10, None, [M, N], True)
        if bias is not None:
            procs.append(ir.AllocEntry(4, N, bias.astype(np.float32)))
            nodes.append(ir.AllocEntry(11, M * N, None, True))
            nodes.append(ir.BinaryNode(11, "ADD", [cur, ir.KMatrix(4, ir.Bin("Remainder", G, C(N)), [N])],
                                       ir.KMatrix(11, None, [M, N], True), [M, N]))
            cur = ir.KMatrix(11, None, [M, N], True)
        nodes.append(ir.BinaryNode(12, "MULT", [cur, ir.KConstant(epi_scale or 1.0)],
                                   ir.KMatrix(3, G, [M, N]), [M, N]))
        procs.append(ir.DPElwFuse(nodes, 1))
    procs.append(ir.Receiver(20, [ir.KMatrix(3, G, [M, N])], "out"))
    return ir.Proc(procs)
