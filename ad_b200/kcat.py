"""Sums of dot products as one dot product over the concatenated K axis.

The reference accumulates the gradients that reach one node from several
consumers with a chain of ADD nodes (autodiff/node.py:125-133).  For the input
of a traced multi-head attention layer (one ``Linear`` per head and per
Q/K/V, nn/transformer.py:20-45) that chain sums 3 x heads products
``dQ_h @ W_h`` of the same shape; its fusion pass puts one of them at the head
of a ``DPElwFuse`` (autodiff/fusion/ops.py:14-26) whose ADD chain reads the
others, each written to HBM by its own dot command.  On the config-4 encoder
that is 23 products of 4096 x 512 (K = 64) written as 8 MB each and read back
by one epilogue, per layer.

``fuse_ksums`` rewrites such a ``DPElwFuse`` so that its dot computes
``A_0 @ B_0 + sum_i A_i @ B_i`` as ``[A_0 | A_1 | ...] @ [B_0; B_1; ...]``:
the operands become concatenations along K (the split kernel gathers them
into one K-major operand), the ADD nodes that read a product are replaced by
``x * 1`` (so the chain and every later statement keep their inputs), and the
product commands are removed.  The products are summed in a different order
than the reference's chain (inside one accumulation instead of one rounding
per ADD), which changes the result by rounding only.

A product is folded in only when

* it is a plain ``DotProdNode`` of the same body, writing a non-temporary
  buffer row-major with the head dot's M and N;
* that buffer is read by this ``DPElwFuse`` alone, written by the product
  alone, and is not a view of another buffer;
* nothing between the product and the ``DPElwFuse`` writes or frees what the
  product reads (a weight updated in between keeps its product where it is,
  so every read sees the value the reference's order gives it).
"""
from __future__ import annotations

import os
from typing import Dict, List, Optional, Set

from . import exprs, ir
from .memplan import _accesses

MIN_TERMS = int(os.environ.get("AD_KCAT_MIN", "2"))     # products folded in, at least


def _subst(e, var: str, off: int):
    """``e`` with variable ``var`` replaced by ``var - off``."""
    if e is None:
        return None
    if exprs._var(e) == var:
        return ir.Bin("Minus", e, ir.Const(off)) if off else e
    if isinstance(e, ir.Bin):
        return ir.Bin(e.op, _subst(e.a, var, off), _subst(e.b, var, off))
    return e


def _shift(k, var: str, off: int):
    """Argument ``k`` read at ``var - off`` (every access and condition)."""
    if isinstance(k, ir.KMatrix):
        return ir.KMatrix(k.id, _subst(k.access, var, off), list(k.shape), k.is_temp)
    if isinstance(k, ir.KConcat):
        return ir.KConcat(_shift(k.karg_one, var, off), _shift(k.karg_two, var, off),
                          _subst(k.condition, var, off), list(k.shape))
    return k


def _cat(pieces, var: str, other_dim: int, along_rows: bool):
    """Concatenation of ``(karg, width)`` pieces along ``var`` (a nested chain:
    piece i is selected when ``var > start_i - 1``)."""
    node, start = None, 0
    for k, w in pieces:
        sk = _shift(k, var, start)
        shape = [start + w, other_dim] if along_rows else [other_dim, start + w]
        node = sk if node is None else ir.KConcat(node, sk, ir.Bin("MoreThan", ir.Xv() if var == "X" else ir.Yv(),
                                                                    ir.Const(start - 1)), shape)
        start += w
    return node, start


def _no_gid(e) -> bool:
    if isinstance(e, ir.Gid):
        return False
    if isinstance(e, ir.Bin):
        return _no_gid(e.a) and _no_gid(e.b)
    return True


def _plain_kmats(k) -> bool:
    """Buffers (no temporaries) and constants, addressed by X and Y only."""
    if isinstance(k, ir.KMatrix):
        return not k.is_temp and k.access is not None and _no_gid(k.access)
    if isinstance(k, ir.KConcat):
        return _plain_kmats(k.karg_one) and _plain_kmats(k.karg_two) and _no_gid(k.condition)
    return isinstance(k, ir.KConstant)


def _ids_read(n) -> Set[int]:
    if type(n).__name__ in ("AllocEntry", "DeallocEntry"):
        return set()
    return {i for k in n.kargs for i in k.ids(True)}


def _row_major(k: ir.KMatrix, N: int) -> bool:
    if isinstance(k.access, ir.Gid):
        return True
    return exprs.affine(k.access) == {"X": N, "Y": 1}


def _fuse_body(body: ir.Proc, readers: Dict[int, int], writers: Dict[int, int], views: Set[int]) -> int:
    cmds = body.procedure
    pos = {id(c): i for i, c in enumerate(cmds)}
    producer: Dict[int, ir.DotProdNode] = {}
    for c in cmds:
        if type(c).__name__ == "DotProdNode" and not c.kres.is_temp:
            producer[c.kres.id] = c
    removed: Set[int] = set()
    move: Dict[int, Dict[int, object]] = {}     # id(f) -> commands to place right after f
    folded = 0
    for f in cmds:
        if type(f).__name__ != "DPElwFuse" or type(f.init_node).__name__ != "DotProdNode":
            continue
        d0 = f.init_node
        M, K0 = d0.children_shapes[0]
        N = d0.children_shapes[1][1]
        if not (_plain_kmats(d0.kargs[0]) and _plain_kmats(d0.kargs[1])):
            continue
        fi = pos[id(f)]
        terms = []                         # (node index in f, ADD operand index, product)
        for ni, n in enumerate(f.nodes):
            if type(n).__name__ != "BinaryNode" or n.op != "ADD" or n.in_place:
                continue
            for ai, k in enumerate(n.kargs):
                if not (isinstance(k, ir.KMatrix) and not k.is_temp and k.id in producer):
                    continue
                p = producer[k.id]
                if id(p) in removed or pos[id(p)] >= fi or list(p.shape) != [M, N]:
                    continue
                if not (_row_major(k, N) and _row_major(p.kres, N) and list(k.shape) == [M, N]):
                    continue
                if readers.get(k.id, 0) != 1 or writers.get(k.id, 0) != 1 or k.id in views:
                    continue
                if sum(k.id in _ids_read(m) for m in f.nodes) != 1:
                    continue
                if p.children_shapes[0][0] != M or p.children_shapes[1][1] != N:
                    continue
                if not (_plain_kmats(p.kargs[0]) and _plain_kmats(p.kargs[1])):
                    continue
                src = set(p.kargs[0].ids(True)) | set(p.kargs[1].ids(True))
                if src & views:
                    continue
                movers = _movers(cmds, pos[id(p)], fi, src, f, removed | {id(t[2]) for t in terms}, views)
                if movers is not None and any(id(c) in m for g, m in move.items() if g != id(f) for c in movers):
                    movers = None           # already placed after another command
                if movers is not None:
                    terms.append((ni, ai, p))
                    for c in movers:
                        move.setdefault(id(f), {})[id(c)] = c
                break
        if len(terms) < MIN_TERMS:
            move.pop(id(f), None)
            continue
        a_pieces = [(d0.kargs[0], K0)] + [(p.kargs[0], p.children_shapes[0][1]) for _, _, p in terms]
        b_pieces = [(d0.kargs[1], K0)] + [(p.kargs[1], p.children_shapes[0][1]) for _, _, p in terms]
        a_cat, K = _cat(a_pieces, "Y", M, along_rows=False)
        b_cat, _ = _cat(b_pieces, "X", N, along_rows=True)
        f.nodes[f.init] = ir.DotProdNode(d0.id, [a_cat, b_cat], d0.kres, list(d0.shape), [[M, K], [K, N]],
                                         d0.program_id)
        for ni, ai, p in terms:
            n = f.nodes[ni]
            keep = n.kargs[1 - ai]
            f.nodes[ni] = ir.BinaryNode(n.id, "MULT", [keep, ir.KConstant(1.0)], n.kres, list(n.shape), False,
                                        getattr(n, "program_id", -1))
            removed.add(id(p))
        folded += len(terms)
    if removed:
        gone = {c.kres.id for c in cmds if id(c) in removed}
        moved = {i for m in move.values() for i in m}
        out = []
        for c in cmds:
            if id(c) in removed or id(c) in moved or (
                    type(c).__name__ in ("AllocEntry", "DeallocEntry") and c.id in gone):
                continue
            out.append(c)
            if id(c) in move:
                out += [x for x in cmds if id(x) in move[id(c)]]      # original order
        body.procedure = out
    return folded


def _rw(c):
    r, w = _accesses(c)
    return set(r), set(w)


def _movers(cmds, pi: int, fi: int, src: Set[int], f, removed: Set[int], views: Set[int]):
    """The commands between the product at ``pi`` and ``f`` at ``fi`` that write
    what the product reads, when each of them can run right after ``f``
    instead (then the product can be computed at ``f``); else None.

    A command moves past the commands after it up to ``f`` (products folded
    into ``f`` excepted: they leave) and past ``f`` itself when none of them
    reads or writes what it writes, writes what it reads, or allocates or
    frees a buffer it touches; ``f`` reads the product's operands after the
    rewrite.  Moved commands keep their order among themselves."""
    out = []
    f_r, f_w = _rw(f)          # before the rewrite
    for ci in range(pi + 1, fi):
        c = cmds[ci]
        kind = type(c).__name__
        if kind in ("AllocEntry", "DeallocEntry"):
            if c.id in src:
                return None
            continue
        r, w = _rw(c)
        if not (w & src):
            continue
        if kind not in ("ElwFuse", "ReduceElwFuse", "DPElwFuse", "DotProdNode", "BinaryNode", "UnaryNode",
                        "ReduceNode", "ContigiousNode") or (r | w) & views:
            return None
        touched = r | w
        for x in cmds[ci + 1:fi]:
            if id(x) in removed:
                continue
            if type(x).__name__ in ("AllocEntry", "DeallocEntry"):
                if x.id in touched:
                    return None
                continue
            xr, xw = _rw(x)
            if (w & (xr | xw)) or (r & xw):
                return None
        if (w & (f_r | f_w)) or (r & f_w):
            return None
        out.append(c)
    return out


def fuse_ksums(proc: ir.Proc) -> int:
    """Rewrite ``proc`` in place (module docstring); returns how many products
    were folded into the dot of another command."""
    readers: Dict[int, int] = {}
    writers: Dict[int, int] = {}
    views: Set[int] = set()
    for c in ir.iter_cmds(proc):
        kind = type(c).__name__
        if kind == "AllocEntry" and getattr(c, "alias", None):
            views.add(c.id)
            views.add(c.alias[0])
        if kind in ("AllocEntry", "DeallocEntry", "ForNode"):
            continue
        r, w = _accesses(c)
        for b in set(r):
            readers[b] = readers.get(b, 0) + 1
        for b in set(w):
            writers[b] = writers.get(b, 0) + 1
    bodies = [proc] + [c.proc for c in ir.iter_cmds(proc) if isinstance(c, ir.ForNode)]
    return sum(_fuse_body(b, readers, writers, views) for b in bodies)
