"""Horizontal batching: independent commands with the same kernel -> one launch.

The reference's DotProd is 2-D only (autodiff/graph/compute/dotprod.py:10-16),
so a batched transformer is traced per (sequence, head): a 4-layer, batch-32,
8-head encoder step holds thousands of tiny dot products, softmaxes and
elementwise commands that differ only in which buffers (or which slice of a
buffer) they touch.  Launched one by one each would occupy a handful of SMs
for a few microseconds.

This pass re-schedules a command list by dependency level (as-soon-as-possible
levels of the read/write dependency graph on buffer ids: read-after-write,
write-after-read, write-after-write; host commands -- Feeder, Receiver -- keep
their original relative order; a nested ``ForNode`` is a barrier) and groups
the commands of one level whose generated kernel source is identical into a
``Batched`` command.  A batched kernel receives a device table of pointer
parameters and ``blockIdx.z`` selects the instance; its body is the unchanged
per-command kernel.  Slice offsets of read-only buffers are already folded
into those pointers (``codegen.view_of``), so per-sequence slices share a
source.
"""
from __future__ import annotations

import re
from dataclasses import dataclass
from typing import Callable, Dict, List, Optional, Set, Tuple

from . import ir

HOST = ("Feeder", "Receiver")


@dataclass
class Batched:
    cmds: List
    program_id: int = -1

    def accesses(self) -> Tuple[List[int], List[int]]:
        from .memplan import _accesses
        r, w = [], []
        for c in self.cmds:
            a, b = _accesses(c)
            r += a
            w += b
        return sorted(set(r)), sorted(set(w))


def _rw(c) -> Tuple[Set[int], Set[int]]:
    from .memplan import _accesses
    r, w = _accesses(c)
    return set(r), set(w)


def schedule(body: List, signature: Callable[[object], Optional[str]]) -> List:
    """Reorder + group ``body`` (a list of commands without Alloc/Dealloc)."""
    out: List = []
    seg: List = []
    for c in body:
        if isinstance(c, ir.ForNode):
            out += _schedule_segment(seg, signature)
            seg = []
            out.append(c)
        else:
            seg.append(c)
    out += _schedule_segment(seg, signature)
    return out


def _edges(cmds: List) -> List[Set[int]]:
    """Predecessors of each command: read-after-write, write-after-read and
    write-after-write on buffer ids; host commands in their original order."""
    preds: List[Set[int]] = []
    last_write: Dict[int, int] = {}
    readers: Dict[int, List[int]] = {}      # buffer -> readers since its last write
    last_host = -1
    for i, c in enumerate(cmds):
        r, w = _rw(c)
        p: Set[int] = set()
        for b in r:
            if b in last_write:
                p.add(last_write[b])
        for b in w:
            if b in last_write:
                p.add(last_write[b])
            p.update(readers.get(b, ()))
        if type(c).__name__ in HOST:
            if last_host >= 0:
                p.add(last_host)
            last_host = i
        p.discard(i)
        preds.append(p)
        for b in r:
            readers.setdefault(b, []).append(i)
        for b in w:
            last_write[b] = i
            readers[b] = []
    return preds


def _levels(cmds: List, signature) -> List[int]:
    """A level per command such that every predecessor sits on a lower level,
    within the critical-path depth, chosen so that commands with equal
    signatures share levels: each command may go anywhere in its window
    [as soon as possible, as late as possible]; repeatedly the (signature,
    level) covering the most unplaced commands is fixed and the windows of
    their predecessors and successors narrowed, until no two unplaced commands
    of one signature can share a level; the rest take their earliest level."""
    n = len(cmds)
    preds = _edges(cmds)
    succs: List[List[int]] = [[] for _ in range(n)]
    for i, ps in enumerate(preds):
        for j in ps:
            succs[j].append(i)
    lo = [0] * n
    for i in range(n):
        for j in preds[i]:
            lo[i] = max(lo[i], lo[j] + 1)
    depth = max(lo) if n else 0
    hi = [depth] * n
    for i in range(n - 1, -1, -1):
        for j in succs[i]:
            hi[i] = min(hi[i], hi[j] - 1)
    # commands marked ``late`` (joins of asynchronous collectives) go as late as
    # their successors allow, so the work between fork and join overlaps
    late = [i for i, c in enumerate(cmds) if getattr(c, "late", False)]
    sigs = [signature(c) for c in cmds]
    classes: Dict[str, List[int]] = {}
    for i, sg in enumerate(sigs):
        if sg is not None:
            classes.setdefault(sg, []).append(i)
    fixed = [False] * n

    def narrow(starts: List[int]) -> None:
        work = list(starts)
        while work:
            i = work.pop()
            for j in succs[i]:
                if lo[j] < lo[i] + 1:
                    lo[j] = lo[i] + 1
                    work.append(j)
        work = list(starts)
        while work:
            i = work.pop()
            for j in preds[i]:
                if hi[j] > hi[i] - 1:
                    hi[j] = hi[i] - 1
                    work.append(j)

    for i in late:
        lo[i] = hi[i]
        fixed[i] = True
    narrow(late)

    while True:
        best = (1, None, None)
        for sg, members in classes.items():
            ev = []
            for i in members:
                if not fixed[i]:
                    ev.append((lo[i], 0))
                    ev.append((hi[i], 1))
            if len(ev) < 4:
                continue
            ev.sort()
            cur = 0
            for lv, kind in ev:
                if kind == 0:
                    cur += 1
                    if cur > best[0]:
                        best = (cur, sg, lv)
                else:
                    cur -= 1
        count, sg, lv = best
        if sg is None:
            break
        chosen = [i for i in classes[sg] if not fixed[i] and lo[i] <= lv <= hi[i]]
        for i in chosen:
            lo[i] = hi[i] = lv
            fixed[i] = True
        narrow(chosen)
        classes[sg] = [i for i in classes[sg] if not fixed[i]]
    return lo


def _schedule_segment(cmds: List, signature) -> List:
    if len(cmds) < 2:
        return list(cmds)
    level = _levels(cmds, signature)
    out: List = []
    for lv in range(max(level) + 1):
        groups: Dict[str, List] = {}
        order: List = []
        for c, l in zip(cmds, level):
            if l != lv:
                continue
            sig = signature(c)
            if sig is None:
                order.append(c)
                continue
            if sig not in groups:
                groups[sig] = []
                order.append(("group", sig))
            groups[sig].append(c)
        for item in order:
            if isinstance(item, tuple):
                g = groups[item[1]]
                out.append(g[0] if len(g) == 1 else Batched(g))
            else:
                out.append(item)
    return out


def batch_proc(proc: ir.Proc, signature) -> ir.Proc:
    def rewrite(p: ir.Proc):
        body = [c for c in p.procedure if type(c).__name__ not in ("AllocEntry", "DeallocEntry")]
        for c in body:
            if isinstance(c, ir.ForNode):
                rewrite(c.proc)
        head = [c for c in p.procedure if type(c).__name__ == "AllocEntry"]
        tail = [c for c in p.procedure if type(c).__name__ == "DeallocEntry"]
        p.procedure = head + schedule(body, signature) + tail

    rewrite(proc)
    return proc


_SIG = re.compile(r'extern "C" __global__ void (__launch_bounds__\([^)]*\) )?(\w+)\(([^)]*)\)\s*\{')


def batched_source(src: str, name: str) -> Tuple[str, int]:
    """Turn ``extern "C" __global__ void K(T0* p0, ..., Tn* pn) { body }`` into a
    kernel that reads its n pointer parameters from ``ad_tab[blockIdx.z * n + i]``."""
    m = _SIG.search(src)
    if m is None:
        raise ValueError("kernel signature not found")
    params = [x.strip() for x in m.group(3).split(",") if x.strip()]
    body = src[m.end():]
    decls = []
    for i, prm in enumerate(params):
        typ, pname = prm.rsplit(" ", 1)
        if "*" not in typ:
            raise ValueError(f"non-pointer parameter {prm}")
        base = typ.replace("__restrict__", "").strip()
        slot = f"ad_tab[(unsigned long long)blockIdx.z * {len(params)} + {i}]"
        uses = re.findall(rf"\b{pname}\b(.)", body)
        if len(params) > 16 and uses and all(u == "[" for u in uses):
            # many pointers (a concatenation's pieces): read each from the table
            # where it is indexed, so only the pieces actually selected are loaded
            body = re.sub(rf"\b{pname}\[", f"(reinterpret_cast<{base}>({slot}))[", body)
            continue
        decls.append(f"    {typ} {pname} = reinterpret_cast<{base}>({slot});")
    lb = m.group(1) or ""
    head = (f'extern "C" __global__ void {lb}{name}(const unsigned long long* __restrict__ ad_tab) {{\n'
            + "\n".join(decls) + "\n")
    return src[:m.start()] + head + body, len(params)
