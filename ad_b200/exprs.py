"""Static analysis of the reference's integer access expressions.

Two analyses over ``ad_b200.ir`` expression trees (the index math that the
reference's ``kernalize`` folds Permute/View/Broadcast/Index/Concat into,
autodiff/kernalize/kernalize.py:71-128 and autodiff/helper.py:19-73):

* ``bounds``  -- interval arithmetic, to pick 32- or 64-bit index math and to
  find the address range a kernel touches in each buffer (hazard checks).
* ``lanes``   -- how an index varies across ``VEC`` consecutive values of one
  loop variable (the "lane" variable: Global for elementwise kernels, Y along
  a reduced row, X across rows).  The result classifies an access as
  *uniform* (same address for all lanes: a broadcast, load once), *unit*
  (``base + j`` with ``base`` a multiple of ``VEC``: one 128-bit load) or
  *other* (per-lane gather).  This is what turns the reference's scalar
  ``buf[expr]`` accesses into coalesced vector accesses.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Optional, Tuple

from .ir import Bin, Const, Expr, Gid, Xv, Yv

CAP = 1 << 30


def _var(e: Expr) -> Optional[str]:
    if isinstance(e, Gid):
        return "G"
    if isinstance(e, Xv):
        return "X"
    if isinstance(e, Yv):
        return "Y"
    return None


# ---------------------------------------------------------------- intervals

def bounds(e: Expr, rng: Dict[str, Tuple[int, int]]) -> Tuple[int, int]:
    """Inclusive [lo, hi] of ``e`` for variables in the inclusive ranges ``rng``."""
    if isinstance(e, Const):
        return e.val, e.val
    v = _var(e)
    if v is not None:
        return rng.get(v, (0, 0))
    alo, ahi = bounds(e.a, rng)
    blo, bhi = bounds(e.b, rng)
    op = e.op
    if op == "Add":
        return alo + blo, ahi + bhi
    if op == "Minus":
        return alo - bhi, ahi - blo
    if op == "Mult":
        c = [alo * blo, alo * bhi, ahi * blo, ahi * bhi]
        return min(c), max(c)
    if op == "ShiftLeft":
        return min(alo << blo, alo << bhi), max(ahi << blo, ahi << bhi)
    if op == "ShiftRight":
        return min(alo >> bhi, alo >> blo), max(ahi >> blo, ahi >> bhi)
    if op == "Div":
        if blo > 0:
            c = [int(alo / blo), int(alo / bhi), int(ahi / blo), int(ahi / bhi)]
            return min(c), max(c)
        m = max(abs(alo), abs(ahi))
        return -m, m
    if op == "Remainder":
        m = max(abs(blo), abs(bhi)) - 1
        if alo >= 0:
            return 0, min(m, ahi)
        return -m, m
    if op == "BitwiseAnd":
        if blo >= 0 and alo >= 0:
            return 0, min(ahi, bhi)
        if blo >= 0:
            return 0, bhi
        return min(alo, blo, 0), max(ahi, bhi)
    if op in ("MoreThan", "LessThan"):
        return 0, 1
    raise ValueError(op)


def max_abs(e: Expr, rng) -> int:
    lo, hi = bounds(e, rng)
    return max(abs(lo), abs(hi))


def subexpr_max(e: Expr, rng) -> int:
    """Largest magnitude of any subexpression (for choosing int vs 64-bit math)."""
    m = max_abs(e, rng)
    if isinstance(e, Bin):
        m = max(m, subexpr_max(e.a, rng), subexpr_max(e.b, rng))
    return m


# ---------------------------------------------------------------- lanes

@dataclass(frozen=True)
class Lane:
    """Value of an expression at lane ``j`` (0 <= j < VEC) = B + s*j, where B is a
    multiple of ``a``.  ``s is None`` means "no usable structure"."""
    s: Optional[int]
    a: int

    @property
    def uniform(self) -> bool:
        return self.s == 0

    def unit(self, vec: int) -> bool:
        return self.s == 1 and self.a % vec == 0


OTHER = Lane(None, 1)


def _p2(c: int) -> int:
    """Largest power of two dividing c (CAP for 0)."""
    if c == 0:
        return CAP
    c = abs(c)
    return min(c & -c, CAP)


def lanes(e: Expr, lane_var: str, vec: int, align: Optional[Dict[str, int]] = None) -> Lane:
    """Lane structure of ``e`` when ``lane_var`` takes the values ``base + j``
    (``base`` a multiple of ``vec``) and every other variable is uniform with
    alignment ``align.get(var, 1)``."""
    align = align or {}
    if isinstance(e, Const):
        return Lane(0, _p2(e.val))
    v = _var(e)
    if v is not None:
        if v == lane_var:
            return Lane(1, vec)
        return Lane(0, align.get(v, 1))
    A = lanes(e.a, lane_var, vec, align)
    B = lanes(e.b, lane_var, vec, align)
    op = e.op
    bc = e.b.val if isinstance(e.b, Const) else None
    ac = e.a.val if isinstance(e.a, Const) else None
    if A.s is None or B.s is None:
        return OTHER
    if op == "Add":
        return Lane(A.s + B.s, min(A.a, B.a))
    if op == "Minus":
        return Lane(A.s - B.s, min(A.a, B.a))
    if op == "Mult":
        if bc is not None:
            return Lane(A.s * bc, min(A.a * _p2(bc), CAP))
        if ac is not None:
            return Lane(B.s * ac, min(B.a * _p2(ac), CAP))
        if A.s == 0 and B.s == 0:
            return Lane(0, min(A.a * B.a, CAP))
        return OTHER
    if op == "ShiftLeft":
        if bc is not None:
            return Lane(A.s << bc, min(A.a << bc, CAP))
        return Lane(0, 1) if (A.s == 0 and B.s == 0) else OTHER
    if op == "ShiftRight":
        if A.s == 0 and B.s == 0:
            if bc is not None:
                return Lane(0, max(1, A.a >> bc))
            return Lane(0, 1)
        if bc is not None and A.s == 1 and A.a % vec == 0:
            if bc == 0:
                return A
            if (1 << bc) % vec == 0:
                return Lane(0, max(1, A.a >> bc))
        return OTHER
    if op == "Div":
        if A.s == 0 and B.s == 0:
            if bc and bc > 0 and A.a % bc == 0:
                return Lane(0, max(1, _p2(A.a // bc)))
            return Lane(0, 1)
        if bc is not None and bc > 0 and A.s == 1 and A.a % vec == 0 and bc % vec == 0:
            return Lane(0, 1)
        if bc == 1:
            return A
        return OTHER
    if op == "Remainder":
        if A.s == 0 and B.s == 0:
            return Lane(0, min(A.a, _p2(bc)) if bc else 1)
        if bc is not None and bc > 0 and A.s == 1 and A.a % vec == 0 and bc % vec == 0:
            return Lane(1, min(A.a, _p2(bc)))
        return OTHER
    if op == "BitwiseAnd":
        if A.s == 0 and B.s == 0:
            if bc is not None:
                return Lane(0, min(A.a, _p2(bc)) if bc else CAP)
            return Lane(0, 1)
        if bc is not None and bc >= 0 and A.s == 1 and A.a % vec == 0 and (bc & (vec - 1)) == vec - 1:
            return Lane(1, vec)
        return OTHER
    if op in ("MoreThan", "LessThan"):
        if A.s == 0 and B.s == 0:
            return Lane(0, 1)
        return OTHER
    raise ValueError(op)


# ---------------------------------------------------------------- affine form

def affine(e: Expr) -> Optional[Dict[str, int]]:
    """``e`` as ``{"1": c, "X": sx, "Y": sy, "G": sg}`` when it is affine, else None."""
    if isinstance(e, Const):
        return {"1": e.val}
    v = _var(e)
    if v is not None:
        return {v: 1}
    a = affine(e.a)
    b = affine(e.b)
    if a is None or b is None:
        return None
    op = e.op

    def add(p, q, sign=1):
        r = dict(p)
        for k, val in q.items():
            r[k] = r.get(k, 0) + sign * val
        return {k: val for k, val in r.items() if val != 0}

    if op == "Add":
        return add(a, b)
    if op == "Minus":
        return add(a, b, -1)
    if op in ("Mult", "ShiftLeft"):
        if op == "ShiftLeft":
            if set(b) - {"1"}:
                return None
            b = {"1": 1 << b.get("1", 0)}
        if set(b) <= {"1"}:
            c = b.get("1", 0)
            return {k: val * c for k, val in a.items() if val * c != 0}
        if set(a) <= {"1"}:
            c = a.get("1", 0)
            return {k: val * c for k, val in b.items() if val * c != 0}
        return None
    return None
