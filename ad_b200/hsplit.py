"""Split horizontally fused elementwise groups into independent commands.

The reference's fusion pass (autodiff/fusion/elw.py) fuses every elementwise
node of equal element count into one ``ElwFuse``, whether or not the nodes
depend on one another.  A per-(sequence, head) transformer step therefore holds
groups of 256 to 2304 statements that are 256 independent copies of one short
chain, each on its own slice: one kernel with as many threads as a single
slice has elements (16 CTAs of 256 threads on the config-4 encoder), every
thread running all of the copies in sequence.

``split_groups`` rewrites such a group into its connected components -- nodes
are connected when one writes a buffer (temp or not) that the other reads or
writes -- each a separate ``ElwFuse`` in the order of its first statement.
Components share only buffers that none of them writes, so running them one
after another computes exactly what the single kernel computed (every
element's statements still run in their original order).  The batching pass
then groups the identical components into one launch.
"""
from __future__ import annotations

from typing import Dict, List

from . import ir


def _ids(k) -> List[int]:
    """Buffer ids (temps included) an argument reads."""
    if isinstance(k, ir.KMatrix):
        return [k.id]
    if isinstance(k, ir.KConcat):
        return _ids(k.karg_one) + _ids(k.karg_two)
    return []


def _compute(n) -> bool:
    return type(n).__name__ not in ("AllocEntry", "DeallocEntry")


def _components(g: ir.ElwFuse) -> List[List[int]]:
    """Indices into ``g.nodes`` of each component (compute nodes and the temp
    Alloc/Dealloc entries of the temps they use), in program order."""
    nodes = g.nodes
    comp = [i for i, n in enumerate(nodes) if _compute(n)]
    parent = {i: i for i in comp}

    def find(i):
        while parent[i] != i:
            parent[i] = parent[parent[i]]
            i = parent[i]
        return i

    written = set()
    for i in comp:
        written.add(nodes[i].kres.id)
    owner: Dict[int, int] = {}          # written buffer id -> a node touching it
    for i in comp:
        n = nodes[i]
        ids = {n.kres.id} | {b for a in n.kargs for b in _ids(a)}
        for b in ids:
            if b not in written:
                continue                # read-only inside the group: no edge
            if b in owner:
                ra, rb = find(owner[b]), find(i)
                if ra != rb:
                    parent[rb] = ra
            else:
                owner[b] = i
    groups: Dict[int, List[int]] = {}
    for i in comp:
        groups.setdefault(find(i), []).append(i)
    if len(groups) == 1:
        return [list(range(len(nodes)))]
    temp_of: Dict[int, int] = {}        # temp id -> component root
    for i in comp:
        n = nodes[i]
        if n.kres.is_temp:
            temp_of[n.kres.id] = find(i)
    out: Dict[int, List[int]] = {r: [] for r in groups}
    for i, n in enumerate(nodes):
        if _compute(n):
            out[find(i)].append(i)
        else:
            r = temp_of.get(n.id)
            if r is None:               # an entry no statement uses: keep it with the first component
                r = find(comp[0])
            out[r].append(i)
    return sorted(out.values(), key=lambda ix: min(j for j in ix if _compute(nodes[j])))


def split_groups(proc: ir.Proc, min_nodes: int = 2) -> int:
    """Rewrite every ``ElwFuse`` of ``proc`` (loop bodies included) with more than
    one component; returns how many groups were split."""
    count = 0

    def rewrite(p: ir.Proc):
        nonlocal count
        out = []
        for c in p.procedure:
            if isinstance(c, ir.ForNode):
                rewrite(c.proc)
                out.append(c)
                continue
            if type(c).__name__ != "ElwFuse" or len(c.nodes) < min_nodes:
                out.append(c)
                continue
            parts = _components(c)
            if len(parts) == 1:
                out.append(c)
                continue
            count += 1
            for ix in parts:
                nodes = [c.nodes[j] for j in ix]
                init = next(k for k, n in enumerate(nodes) if _compute(n))
                out.append(ir.ElwFuse(nodes, init, c.program_id, c.fuse_id))
        p.procedure = out

    rewrite(proc)
    return count
