"""Arena planning: every buffer of a proc placed in ONE device allocation.

Replaces the reference's ``tetris_opt`` (autodiff/alloc/tetris_opt.py:69-192)
for the device side.  Differences, each deliberate:

* Offsets are aligned to 256 bytes (the reference packs at float
  granularity), so every buffer base is valid for 128-bit vector access and
  TMA (16-byte) descriptors.
* Lifetimes are computed at *kernel* granularity from the commands' own
  reads and writes: a buffer read by command k is live through the end of
  k, and a buffer written by command k is live from the start of k.  So an
  output never shares memory with an input of the same kernel.  (The
  reference computes lifetimes from Alloc/Dealloc positions *inside* fused
  groups, which lets a fused kernel's output overlap a buffer that other
  threads of the same kernel still read -- a data race; e.g. the row-mean
  slot in the LayerNorm chain.)
* A buffer used inside a ``For`` body lives for the whole loop unless its
  first access in the body is a write and it is not used outside the loop
  (then it is iteration-local).
* Buffers with content (parameters, ``Tensor`` leaves) live for the whole
  program.

Accepts procs with or without the reference's own tetris arena (then the
arena id is simply one more buffer).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

from . import ir

ALIGN = 256


@dataclass
class Slot:
    id: int
    size: int          # floats
    start: int
    end: int
    offset: int = 0    # bytes
    pinned: bool = False

    @property
    def nbytes(self) -> int:
        return self.size * 4


def _accesses(c) -> Tuple[List[int], List[int]]:
    """(reads, writes) buffer ids of one command."""
    kind = type(c).__name__
    if hasattr(c, "accesses"):
        return c.accesses()
    if kind == "Feeder":
        return [], c.kres.ids(True)
    if kind == "Receiver":
        r = []
        for k in c.kargs:
            r += k.ids(True)
        return r, []
    nodes = c.nodes if isinstance(c, ir.FuseGroup) else [c]
    reads, writes = [], []
    for n in nodes:
        if isinstance(n, (ir.AllocEntry, ir.DeallocEntry)):
            continue
        for k in n.kargs:
            reads += k.ids(True)
        writes += n.kres.ids(True)
    return reads, writes


def plan(proc: ir.Proc) -> Tuple[Dict[int, Slot], int]:
    """Returns ({buffer id: Slot}, arena bytes)."""
    sizes: Dict[int, int] = {}
    content: Dict[int, bool] = {}
    alias: Dict[int, tuple] = {}
    for c in ir.iter_cmds(proc):
        if isinstance(c, ir.AllocEntry) and not c.is_temp and getattr(c, "alias", None):
            alias[c.id] = (c.alias[0], c.alias[1], c.size)
            continue
        if isinstance(c, ir.AllocEntry) and not c.is_temp:
            sizes[c.id] = max(sizes.get(c.id, 0), c.size)
            content[c.id] = content.get(c.id, False) or c.content is not None

    first: Dict[int, int] = {}
    last: Dict[int, int] = {}
    pos = [0]

    def touch(b: int, p: int) -> None:
        if b in alias:           # a view: its accesses keep the base buffer alive
            b = alias[b][0]
        first[b] = min(first.get(b, p), p)
        last[b] = max(last.get(b, p), p)

    def walk(p: ir.Proc) -> None:
        for c in p.procedure:
            if isinstance(c, ir.ForNode):
                start = pos[0]
                # which buffers does the loop touch, and is the first touch a write?
                body_first: Dict[int, str] = {}
                inner_outer_touch: Dict[int, bool] = {}
                mark_before = dict(first)
                walk(c.proc)
                end = pos[0]
                for cc in ir.iter_cmds(c.proc):
                    if isinstance(cc, ir.ForNode) or type(cc).__name__ in ("AllocEntry", "DeallocEntry"):
                        continue
                    r, w = _accesses(cc)
                    for b in r:
                        body_first.setdefault(b, "r")
                    for b in w:
                        body_first.setdefault(b, "w")
                for b, kind in body_first.items():
                    if b in alias:
                        b = alias[b][0]
                        kind = "r"        # partial writes through views: keep the base loop-live
                    local = kind == "w" and b not in mark_before
                    if not local:
                        touch(b, start)
                        touch(b, end)
                    else:
                        # may still be read after the loop: handled by later touches
                        inner_outer_touch[b] = True
                pos[0] += 1
                continue
            if type(c).__name__ in ("AllocEntry", "DeallocEntry"):
                continue
            r, w = _accesses(c)
            for b in r + w:
                touch(b, pos[0])
            pos[0] += 1

    walk(proc)
    end_all = pos[0] + 1
    slots: Dict[int, Slot] = {}
    for b, n in sizes.items():
        if not content.get(b) and b not in first:
            continue   # never touched by a launch or a host copy (e.g. kept in registers)
        if content.get(b) or b not in first:
            s, e = 0, end_all
        else:
            s, e = first[b], last[b]
        slots[b] = Slot(b, n, s, e, pinned=content.get(b, False))
    # any buffer referenced without an AllocEntry is an error in the proc
    for b in list(first):
        if b not in slots:
            raise ValueError(f"buffer {b} is used but never allocated")

    total = _place(slots, end_all)
    for a, (base, off, n) in alias.items():
        if base in slots:
            slots[a] = Slot(a, n, slots[base].start, slots[base].end, slots[base].offset + 4 * off)
    return slots, total


def _place(slots: Dict[int, Slot], end_all: int) -> int:
    """Offsets for ``slots`` (sets ``Slot.offset``); returns the arena bytes.

    Buffers that live for the whole program (parameters) are packed first, by
    decreasing size, at the bottom.  The others are placed in order of their
    first use (larger first among equal starts) by a simulated best-fit
    allocator: a buffer's range is released after its last use, free ranges are
    coalesced, and a request takes the smallest free range that holds it, else
    grows the top.  O(n log n + n * free ranges): tens of thousands of buffers
    plan in well under a second."""
    import bisect
    import heapq

    def rounded(sl):
        return (sl.nbytes + ALIGN - 1) // ALIGN * ALIGN

    whole = [sl for sl in slots.values() if sl.start <= 0 and sl.end >= end_all]
    rest = [sl for sl in slots.values() if not (sl.start <= 0 and sl.end >= end_all)]
    off = 0
    for sl in sorted(whole, key=lambda x: (-x.size, x.id)):
        sl.offset = off
        off += rounded(sl)
    base = top = total = off
    free_off: List[int] = []       # free ranges above ``base``, sorted by offset
    free_len: List[int] = []
    live: List[Tuple[int, int, int, int]] = []      # heap of (end, id, offset, bytes)

    def release(o: int, n: int) -> None:
        nonlocal top
        i = bisect.bisect_left(free_off, o)
        if i > 0 and free_off[i - 1] + free_len[i - 1] == o:      # merge with the range below
            i -= 1
            o, n = free_off[i], free_len[i] + n
            del free_off[i], free_len[i]
        if i < len(free_off) and o + n == free_off[i]:            # and the one above
            n += free_len[i]
            del free_off[i], free_len[i]
        if o + n == top:
            top = o
        else:
            free_off.insert(i, o)
            free_len.insert(i, n)

    for sl in sorted(rest, key=lambda x: (x.start, -x.size, x.id)):
        while live and live[0][0] < sl.start:
            _, _, o, n = heapq.heappop(live)
            release(o, n)
        need = rounded(sl)
        best = -1
        for i, n in enumerate(free_len):
            if n >= need and (best < 0 or n < free_len[best]):
                best = i
                if n == need:
                    break
        if best >= 0:
            sl.offset = free_off[best]
            if free_len[best] == need:
                del free_off[best], free_len[best]
            else:
                free_off[best] += need
                free_len[best] -= need
        else:
            sl.offset = top
            top += need
            total = max(total, top)
        heapq.heappush(live, (sl.end, sl.id, sl.offset, need))
    return max(total, base)
