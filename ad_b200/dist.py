"""Data parallelism: per-rank batch shards + one gradient all-reduce per step.

The reference has no multi-device code (TODO.md:68-69).  Its SGD update
``p -= lr * grad`` (autodiff/nn/optimizers/SGD.py:13-16) becomes an in-place
``ADD`` whose result id is the parameter's (autodiff/opt/in_place.py:7-31);
linearize fuses it as the last statement of the kernel that computes the
gradient, so in a single-device proc the gradient never exists on its own.

``insert_grad_allreduce`` rewrites a rank's proc (traced with the rank's share
of the global batch) so that

1. every in-place parameter update ``W[G] = W[G] + T`` (``T = -lr * grad``)
   instead writes ``T`` into the parameter's slice of one contiguous gradient
   bucket ``GB`` (``g_W[G] = T + 0``; ``g_W`` is a buffer aliased to
   ``GB[off_W:]``, so that independent gradient kernels stay independent for
   scheduling while the all-reduce sees one contiguous range);
2. finished slices are summed over ranks in buckets: once the pending
   slices reach ``AD_DP_BUCKET_MB`` (8 MiB), an ``AllReduce`` of their
   contiguous range of ``GB`` starts on the device's communication stream
   while the backward pass goes on; an ``AllReduceWait``, placed as late as
   possible, joins it back, and then one update per parameter,
   ``W[G] = W[G] + g_W[G]``, runs -- before the first later command that reads
   one of those parameters, else at the end of the loop body.

The loss is a sum over examples, so the summed ``-lr * grad`` of the shards
equals the full-batch update: no division by the world size.  Flushing before
the next reader keeps the reference's semantics exactly: its linearize can
place an update before a read of the same weight (the attention output
projection is updated before the kernel that back-propagates through it, so
the head gradients see the updated weight); a reader after the update sees
the updated value here too, and one before it the old value.  Without such
readers all parameters share one all-reduce at the end of the step.
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

from . import ir

_next_id = [10 ** 9]


def _fresh_id() -> int:
    _next_id[0] += 1
    return _next_id[0]


@dataclass
class AllReduce:
    """Sum ``count`` floats of buffer ``buf`` starting at element ``offset`` over
    all ranks, in place.  ``members`` are the per-parameter slice buffers
    (aliases into ``buf``) the range covers, for dependency tracking.  With
    ``async_start`` the device runs it on its communication stream, forked from
    the compute stream at this point; an ``AllReduceWait`` joins it back."""
    buf: int
    count: int
    offset: int = 0
    members: Tuple[int, ...] = ()
    program_id: int = -1
    comm: object = None
    async_start: bool = False

    def accesses(self) -> Tuple[List[int], List[int]]:
        ids = list(self.members) or [self.buf]
        return ids, ids


@dataclass
class AllReduceWait:
    """The compute stream waits for the all-reduces ``starts``.  Scheduled as
    late as its successors allow (``late``), so the reduction overlaps the
    compute between its start and the first command that needs its result."""
    starts: List[AllReduce]
    program_id: int = -1
    late: bool = True

    def accesses(self) -> Tuple[List[int], List[int]]:
        ids = [m for s in self.starts for m in (list(s.members) or [s.buf])]
        return ids, ids


BUCKET_BYTES = int(float(os.environ.get("AD_DP_BUCKET_MB", "8")) * (1 << 20))


def _is_update(n, content_ids) -> bool:
    return (type(n).__name__ == "BinaryNode" and n.in_place and n.op == "ADD"
            and not n.kres.is_temp and n.kres.id in content_ids
            and isinstance(n.kres.access, ir.Gid)
            and isinstance(n.kargs[0], ir.KMatrix) and n.kargs[0].id == n.kres.id
            and isinstance(n.kargs[0].access, ir.Gid))


def insert_grad_allreduce(proc: ir.Proc, comm=None, bucket_bytes: Optional[int] = None) -> Optional[int]:
    """Rewrite ``proc`` in place (see module docstring).  Returns the bucket's
    buffer id of the last rewritten body, or None when the proc has no in-place
    parameter update.  Loop bodies and the top level are rewritten alike."""
    from .memplan import _accesses
    cap = BUCKET_BYTES if bucket_bytes is None else bucket_bytes
    content = {c.id: c.size for c in ir.iter_cmds(proc)
               if isinstance(c, ir.AllocEntry) and c.content is not None}
    loops = [c for c in proc.procedure if isinstance(c, ir.ForNode)]
    bodies = [l.proc for l in loops] + [proc]
    gb = None
    for body in bodies:
        has = any(_is_update(n, content) for c in body.procedure
                  for n in (c.nodes if isinstance(c, ir.FuseGroup) else [c]))
        if not has:
            continue
        gb = _fresh_id()
        total = 0
        pending: List[Tuple[int, int, int, int]] = []     # (param, offset, n_el, slice id): not started
        inflight: List[Tuple[AllReduce, list]] = []        # started, updates not applied
        new_body: List = []
        slices: List[ir.AllocEntry] = []

        def start(async_start: bool, which=None):
            """Start the all-reduce of ``which`` (default: every pending slice),
            one collective per run of adjacent slices in the bucket."""
            nonlocal pending
            which = pending if which is None else which
            if not which:
                return
            runs, cur = [], [which[0]]
            for x in which[1:]:
                prev = cur[-1]
                if x[1] == prev[1] + (prev[2] + 63) // 64 * 64:
                    cur.append(x)
                else:
                    runs.append(cur)
                    cur = [x]
            runs.append(cur)
            for run in runs:
                start_off = run[0][1]
                end_off = run[-1][1] + (run[-1][2] + 63) // 64 * 64
                ar = AllReduce(gb, end_off - start_off, start_off,
                               tuple(sid for _, _, _, sid in run), comm=comm, async_start=async_start)
                new_body.append(ar)
                inflight.append((ar, run))
            ids = {id(x) for x in which}
            pending = [x for x in pending if id(x) not in ids]

        def finish(which):
            """Wait for the started buckets ``which`` and apply their updates."""
            nonlocal inflight
            if not which:
                return
            asyncs = [ar for ar, _ in which if ar.async_start]
            if asyncs:
                new_body.append(AllReduceWait(asyncs))
            for _, members in which:
                for w, off, n_el, sid in members:
                    new_body.append(ir.BinaryNode(_fresh_id(), "ADD",
                                                  [ir.KMatrix(w, ir.Gid(), [n_el]), ir.KMatrix(sid, ir.Gid(), [n_el])],
                                                  ir.KMatrix(w, ir.Gid(), [n_el]), [n_el], True))
            inflight = [x for x in inflight if all(x is not y for y in which)]

        def need(params):
            """Every update of ``params`` must be applied before the next command."""
            if any(x[0] in params for x in pending):
                # everything pending goes with it: per-parameter collectives for
                # the per-head weights would put dozens of latencies on the path
                start(True)
            finish([x for x in inflight if any(w in params for w, _, _, _ in x[1])])

        for c in body.procedure:
            kind = type(c).__name__
            if kind == "ForNode":
                start(True)
                finish(list(inflight))
            elif kind not in ("AllocEntry", "DeallocEntry") and (pending or inflight):
                reads, writes = _accesses(c)
                need(set(reads) | set(writes))
            nodes = c.nodes if isinstance(c, ir.FuseGroup) else [c]
            for i, n in enumerate(nodes):
                if not _is_update(n, content):
                    continue
                w = n.kres.id
                need({w})
                n_el = math.prod(n.shape)
                off = total
                total += (n_el + 63) // 64 * 64      # 256-byte aligned slices
                sid = _fresh_id()
                slices.append(ir.AllocEntry(sid, n_el, None, False, (gb, off)))
                new = ir.BinaryNode(n.id, "ADD", [n.kargs[1], ir.KConstant(0.0)],
                                    ir.KMatrix(sid, ir.Gid(), list(n.shape)), list(n.shape), False,
                                    getattr(n, "program_id", -1))
                if isinstance(c, ir.FuseGroup):
                    c.nodes[i] = new
                else:
                    c = new
                pending.append((w, off, n_el, sid))
            new_body.append(c)
            if 4 * sum(x[2] for x in pending) >= cap:
                start(True)
        start(True)
        finish(list(inflight))
        body.procedure = new_body
        proc.procedure[0:0] = [ir.AllocEntry(gb, total)] + slices
    return gb


def nccl_unique_id() -> bytes:
    """128-byte NCCL id (call on rank 0, send to the other ranks)."""
    import ctypes
    from . import runtime as rt
    buf = ctypes.create_string_buffer(128)
    rt.check(rt.lib().ad_nccl_unique_id(buf), "ad_nccl_unique_id")
    return buf.raw
