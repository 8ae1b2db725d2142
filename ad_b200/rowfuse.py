"""Row fusion: several procedural-IR commands over the same row structure -> one kernel.

The reference fuses only an elementwise *epilogue* into a reduction
(autodiff/fusion/ops.py:27-38) and launches every other command on its own,
so a LayerNorm + softmax forward/backward is ~12 kernels and ~26 full passes
over HBM.  This pass finds maximal runs of consecutive commands that all live
on one ``[V, R]`` row structure:

* reductions ``ReduceNode``/``ReduceElwFuse`` over ``[V, R]``,
* elementwise commands of size ``V * R`` (``_global_id = x * R + c``) or of
  size ``V`` (one value per row, ``_global_id = x``),

such that every buffer the run *writes* is only ever accessed by the run at
the canonical position of the current row (``x * R + c`` for full rows, ``x``
for per-row scalars), so rows never depend on each other.  Buffers the run
only reads may be accessed with any expression (broadcast columns such as
LayerNorm's gamma, transposes, ...).

The run becomes one kernel: ``GS`` threads own one row (``NC`` 128-bit
chunks each); values of full-size buffers produced in the run stay in
registers, per-row scalars are broadcast, reductions are shuffle +
shared-memory trees inside the row's thread group.  Buffers that nothing
outside the run touches are never written to HBM.  For the config-2 proc
this turns 12 kernels / ~26 passes into 1 kernel that reads x, dy, gamma,
beta and writes y, dx.

Command semantics (statement order, arithmetic, in-place updates) are those
of the individual kernels; reductions are exact (see ``codegen.gen_reduce``).
"""
from __future__ import annotations

import os

import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Set, Tuple

import numpy as np

from . import codegen, exprs, ir
from .codegen import Emitter, KernelSpec, binary_expr, flit, unary_expr

ELW = ("ElwFuse", "BinaryNode", "UnaryNode", "ContigiousNode")
RED = ("ReduceNode", "ReduceElwFuse")
VEC = 4
MAX_CHUNKS = 8


@dataclass
class RowFused:
    """A run of commands executed as one row-fused kernel."""
    cmds: List
    V: int
    R: int
    internal: Set[int]                    # buffers that never reach HBM
    program_id: int = -1

    def accesses(self) -> Tuple[List[int], List[int]]:
        """External (reads, writes), for the arena planner."""
        reads, writes = [], []
        for c in self.cmds:
            for n in codegen.chain_nodes(c):
                for k in n.kargs:
                    reads += [b for b in k.ids(True) if b not in self.internal]
                writes += [b for b in n.kres.ids(True) if b not in self.internal]
        return sorted(set(reads)), sorted(set(writes))


# ---------------------------------------------------------------- numeric expression checks

def eval_np(e: ir.Expr, G=None, X=None, Y=None):
    if isinstance(e, ir.Const):
        return np.int64(e.val)
    if isinstance(e, ir.Gid):
        return G
    if isinstance(e, ir.Xv):
        return X
    if isinstance(e, ir.Yv):
        return Y
    a = eval_np(e.a, G, X, Y)
    b = eval_np(e.b, G, X, Y)
    op = e.op
    if op == "Add":
        return a + b
    if op == "Minus":
        return a - b
    if op == "Mult":
        return a * b
    if op in ("Div", "Remainder"):
        q = np.abs(a) // np.abs(b)
        q = np.where((a >= 0) == (b >= 0), q, -q)
        return q if op == "Div" else a - b * q
    if op == "ShiftRight":
        return a >> b
    if op == "ShiftLeft":
        return a << b
    if op == "BitwiseAnd":
        return a & b
    if op == "MoreThan":
        return (a > b).astype(np.int64)
    if op == "LessThan":
        return (a < b).astype(np.int64)
    raise ValueError(op)


def _pow2(n: int) -> bool:
    return n > 0 and n & (n - 1) == 0


def classify_full(e: ir.Expr, V: int, R: int) -> Optional[str]:
    """Access ``e(G)`` inside a full-size command (G = x*R + c): 'row' if
    e == G (this row's element), 'scalar' if e == x (this row's scalar), else None."""
    xs = np.arange(V, dtype=np.int64)
    base = eval_np(e, G=xs * R)
    if not _pow2(R):
        # fall back to sampling every column of a few rows plus all rows at c = 0, R-1
        cs = np.arange(R, dtype=np.int64)
        for x in sorted({0, 1, V // 2, V - 1}):
            if x < 0 or x >= V:
                continue
            v = eval_np(e, G=x * R + cs)
            if np.array_equal(v, x * R + cs):
                continue
            if np.all(v == x):
                continue
            return None
        last = eval_np(e, G=xs * R + (R - 1))
        if np.array_equal(base, xs * R) and np.array_equal(last, xs * R + R - 1):
            return "row"
        if np.array_equal(base, xs) and np.array_equal(last, xs):
            return "scalar"
        return None
    ln = exprs.lanes(e, "G", R)
    if ln.s == 1 and np.array_equal(base, xs * R):
        return "row"
    if ln.s == 0 and np.array_equal(base, xs):
        return "scalar"
    return None


def classify_rowscalar(e: ir.Expr, V: int) -> bool:
    xs = np.arange(V, dtype=np.int64)
    return bool(np.array_equal(eval_np(e, G=xs, X=xs, Y=np.int64(0)), xs))


def classify_reduce_src(e: ir.Expr, V: int, R: int) -> bool:
    """Reduce input ``e(X, Y)`` is this row's canonical element ``x*R + y``."""
    xs = np.arange(V, dtype=np.int64)
    if not np.array_equal(eval_np(e, X=xs, Y=np.int64(0), G=np.int64(0)), xs * R):
        return False
    if _pow2(R):
        return exprs.lanes(e, "Y", R).s == 1
    ys = np.arange(R, dtype=np.int64)
    for x in sorted({0, V // 2, V - 1}):
        if not np.array_equal(eval_np(e, X=np.int64(x), Y=ys, G=np.int64(0)), x * R + ys):
            return False
    return True


# ---------------------------------------------------------------- region detection

def _kmats(k) -> List[ir.KMatrix]:
    if isinstance(k, ir.KMatrix) and not k.is_temp:
        return [k]
    if isinstance(k, ir.KConcat):
        return _kmats(k.karg_one) + _kmats(k.karg_two)
    return []


def _cmd_kind(c, V: int, R: int) -> Optional[str]:
    k = type(c).__name__
    if k in RED:
        rn = c if k == "ReduceNode" else c.init_node
        return "reduce" if list(rn.children_shapes[0]) == [V, R] else None
    if k in ELW:
        n = math.prod(c.init_node.shape if k == "ElwFuse" else c.shape)
        if n == V * R:
            return "full"
        if n == V:
            return "scalar"
    return None


class RunState:
    """Incremental legality check of a row run (commands added in program order).

    Rules: every command lives on [V, R]; a buffer written in the run is only
    accessed at this row's canonical position (``x*R + c`` for 'row' buffers,
    ``x`` for 'scalar' buffers), both before and after its write; buffers
    never written in the run may be read with any expression."""

    def __init__(self, V: int, R: int):
        self.V, self.R = V, R
        self.kinds: Dict[int, str] = {}
        self.written: Set[int] = set()
        self.read_pattern: Dict[int, Optional[str]] = {}   # first-read class of not-yet-written buffers
        self.n_reduce = 0

    def _cls_full(self, e):
        return classify_full(e, self.V, self.R)

    def _cls_scalar(self, e):
        return "scalar" if classify_rowscalar(e, self.V) else None

    def _read(self, km: ir.KMatrix, cls: Optional[str]) -> bool:
        b = km.id
        if b in self.written:
            return cls is not None and cls == self.kinds[b]
        prev = self.read_pattern.get(b, "unset")
        if prev == "unset":
            self.read_pattern[b] = cls
        elif prev != cls:
            self.read_pattern[b] = None
        return True

    def _write(self, km: ir.KMatrix, cls: Optional[str]) -> bool:
        if cls is None:
            return False
        b = km.id
        if self.kinds.setdefault(b, cls) != cls:
            return False
        if b in self.read_pattern and self.read_pattern[b] != cls:
            return False   # read with another pattern earlier in the run: cross-row hazard
        self.written.add(b)
        return True

    def add(self, c) -> bool:
        V, R = self.V, self.R
        ck = _cmd_kind(c, V, R)
        if ck is None:
            return False
        snapshot = (dict(self.kinds), set(self.written), dict(self.read_pattern))
        ok = self._add(c, ck)
        if not ok:
            self.kinds, self.written, self.read_pattern = snapshot
        elif ck == "reduce":
            self.n_reduce += 1
        return ok

    def _add(self, c, ck: str) -> bool:
        V, R = self.V, self.R
        for n in codegen.chain_nodes(c):
            nk = type(n).__name__
            if nk == "ReduceNode":
                src = n.kargs[0]
                for km in _kmats(src):
                    canon = isinstance(src, ir.KMatrix) and classify_reduce_src(km.access, V, R)
                    if not self._read(km, "row" if canon else None):
                        return False
                if not n.kres.is_temp and not self._write(n.kres, self._cls_scalar(n.kres.access)):
                    return False
                continue
            for karg in n.kargs:
                for km in _kmats(karg):
                    cls = self._cls_full(km.access) if ck == "full" else self._cls_scalar(km.access)
                    if isinstance(karg, ir.KConcat) and km.id in self.written:
                        return False
                    if not self._read(km, cls):
                        return False
            if not n.kres.is_temp:
                cls = self._cls_full(n.kres.access) if ck == "full" else self._cls_scalar(n.kres.access)
                if ck == "full" and cls != "row":
                    return False
                if not self._write(n.kres, cls):
                    return False
        return True


def _depends_on_run(c, written: Set[int]) -> bool:
    for n in codegen.chain_nodes(c):
        for k in n.kargs:
            if any(km.id in written for km in _kmats(k)):
                return True
    return False


def _rw(c) -> Tuple[Set[int], Set[int]]:
    from .memplan import _accesses
    r, w = _accesses(c)
    return set(r), set(w)


WINDOW = 640    # how far ahead a run looks for dependent commands


def _anchor_shape(body: List, i: int, rws) -> Optional[Tuple[int, int]]:
    c = body[i]
    k = type(c).__name__
    if k in RED:
        rn = c if k == "ReduceNode" else c.init_node
        return tuple(rn.children_shapes[0])
    if k not in ELW:
        return None
    n_el = math.prod(c.init_node.shape if k == "ElwFuse" else c.shape)
    w = rws[i][1]
    for j in range(i + 1, min(len(body), i + WINDOW)):
        d = body[j]
        if isinstance(d, ir.ForNode):
            return None
        if type(d).__name__ in RED and rws[j][0] & w:
            rn = d if type(d).__name__ == "ReduceNode" else d.init_node
            V, R = rn.children_shapes[0]
            return (V, R) if V * R == n_el or V == n_el else None
    return None


def _fully_connected(c, run_w: Set[int]) -> bool:
    """Every statement of ``c`` reads something the run (or an earlier statement
    of ``c`` that does) produced.  Keeps out commands that only partly belong to
    the run, e.g. the reference's horizontal ElwFuse of all attention heads."""
    live = set(run_w)
    live_t: Set[int] = set()
    for n in codegen.chain_nodes(c):
        hit = False
        for k in n.kargs:
            for km in _kmats(k):
                hit |= km.id in live
            if isinstance(k, ir.KMatrix) and k.is_temp and k.id in live_t:
                hit = True
        if not hit:
            return False
        if n.kres.is_temp:
            live_t.add(n.kres.id)
        else:
            live.add(n.kres.id)
    return True


def grow_run(body: List, rws, i: int) -> Optional[Tuple[List[int], int, int, int]]:
    """Try to grow a row run from anchor ``body[i]`` (a reduction, or an
    elementwise command feeding one).  Later commands that read something the
    run wrote may join.  The run executes at position ``P``: while no skipped
    command conflicts with the run, members are *sunk* to the newest member
    (P moves there); once one conflicts (reads what the run writes, or writes
    what it reads or writes), later candidates must be *hoisted* to P, which
    needs them not to read what a command skipped after P writes, nor write
    what one reads or writes.  Independent siblings (the same softmax of other
    attention heads) are skipped and form their own runs, which the batching
    pass launches side by side.  Returns (members, P, V, R) or None."""
    n = len(body)
    shape = _anchor_shape(body, i, rws)
    if shape is None:
        return None
    V, R = shape
    if R % VEC != 0 or R < 32 or R // VEC > 1024 * MAX_CHUNKS:
        return None
    st = RunState(V, R)
    if not st.add(body[i]):
        return None
    members = [i]
    P = i
    run_r, run_w = set(rws[i][0]), set(rws[i][1])
    skip_r: Set[int] = set()
    skip_w: Set[int] = set()
    blocked = False
    for j in range(i + 1, min(n, i + WINDOW)):
        d = body[j]
        if isinstance(d, ir.ForNode):
            break
        r, w = rws[j]
        if type(d).__name__ in ELW + RED and (r & run_w) and _fully_connected(d, run_w):
            ok = (not blocked) or (not (r & skip_w) and not (w & (skip_r | skip_w)))
            if ok and st.add(d):
                members.append(j)
                run_r |= r
                run_w |= w
                if not blocked:
                    P = j
                    skip_r, skip_w = set(), set()
                continue
        if (r & run_w) or (w & (run_r | run_w)):
            blocked = True
        skip_r |= r
        skip_w |= w
    if st.n_reduce and len(members) >= 2:
        return members, P, V, R
    return None


def run_state(cmds, V, R) -> RunState:
    st = RunState(V, R)
    for c in cmds:
        assert st.add(c)
    return st


def run_kinds(cmds, V, R) -> Dict[int, str]:
    return run_state(cmds, V, R).kinds


# ---------------------------------------------------------------- the pass

def _flat_positions(proc: ir.Proc):
    """buffer -> list of (position, command object) over the whole program, and
    command id -> position; For bodies are flattened in order."""
    pos_of: Dict[int, int] = {}
    uses: Dict[int, List[int]] = {}
    counter = [0]

    def walk(p):
        for c in p.procedure:
            k = type(c).__name__
            if k == "ForNode":
                walk(c.proc)
                continue
            if k in ("AllocEntry", "DeallocEntry"):
                continue
            pos_of[id(c)] = counter[0]
            from .memplan import _accesses
            r, w = _accesses(c)
            bufs = sorted(set(r) | set(w))
            for b in bufs:
                uses.setdefault(b, []).append(counter[0])
            counter[0] += 1

    walk(proc)
    return pos_of, uses


def fuse_rows(proc: ir.Proc) -> ir.Proc:
    """Rewrite ``proc`` in place, replacing fusible runs by ``RowFused`` commands."""
    pos_of, uses = _flat_positions(proc)

    def rewrite(p: ir.Proc):
        body = p.procedure
        compute_idx = [i for i, c in enumerate(body) if type(c).__name__ not in ("AllocEntry", "DeallocEntry")]
        seq = [body[i] for i in compute_idx]
        for c in seq:
            if type(c).__name__ == "ForNode":
                rewrite(c.proc)
        rws = [(_rw(c) if not isinstance(c, ir.ForNode) else (set(), set())) for c in seq]
        i = 0
        changed = False
        while i < len(seq):
            if type(seq[i]).__name__ not in ELW + RED:
                i += 1
                continue
            got = grow_run(seq, rws, i)
            if got is None:
                i += 1
                continue
            members, P, V, R = got
            cmds = [seq[m] for m in members]
            mpos = {pos_of[id(c)] for c in cmds}
            kinds = run_kinds(cmds, V, R)
            internal = {b for b in kinds if all(u in mpos for u in uses.get(b, []))}
            rf = RowFused(cmds, V, R, internal, getattr(cmds[0], "program_id", -1))
            rr, ww = set(), set()
            for m in members:
                rr |= rws[m][0]
                ww |= rws[m][1]
            mset = set(members)
            assert P in mset
            # splice in place: the run takes its anchor's slot, the other members go
            seq[P] = rf
            rws[P] = (rr, ww)
            for k in sorted(mset - {P}, reverse=True):
                del seq[k]
                del rws[k]
            changed = True
            # the anchor slot now holds the next command (or the run itself)
        if not changed:
            return
        others = [c for c in body if type(c).__name__ in ("AllocEntry", "DeallocEntry")]
        p.procedure = [c for c in others if type(c).__name__ == "AllocEntry"] + seq + \
            [c for c in others if type(c).__name__ == "DeallocEntry"]

    rewrite(proc)
    return proc


# ---------------------------------------------------------------- code generation

STAGE_SMEM_MAX = 96 * 1024   # per block, all ring slots
# ring depth: 3 slots measured slower than 2 on config 2 (4358 vs ~4550 GB/s)
MAX_SLOTS = 2
# threads per row (at most; 256 measured 5.9 vs 4.7 TB/s for 512 on config 2):
# fewer threads hold more of the row in registers
# and make each reduction's shuffle/shared-memory exchange cheaper per element
GS_MAX = int(os.environ.get("AD_RF_GS", "256"))
GRID_PER_SM = int(os.environ.get("AD_RF_GRID", "2"))     # persistent blocks per SM (staged schedule)


def gen_rowfused(rf: RowFused, name: str, sizes: Dict[int, int], sm_count: int = 148) -> KernelSpec:
    """Two schedules.  *Staged* (one row per thread group, rows streamed): a
    persistent loop over rows in which thread 0 prefetches the next row's
    row-canonical inputs with ``cp.async.bulk`` (TMA, 1-D) into a ``MAX_SLOTS``-slot
    shared-memory ring while the block computes the current row.  *Direct*
    (short rows, several rows per block): inputs are loaded straight from
    global memory."""
    V, R = rf.V, rf.R
    units = R // VEC
    gs = 1
    while gs * 2 <= min(GS_MAX, units) and units % (gs * 2) == 0:
        gs *= 2
    nc = units // gs
    if nc > MAX_CHUNKS:
        raise ValueError("row too long for row fusion")
    rows_pb = max(1, 256 // gs) if gs < 256 else 1
    block = gs * rows_pb
    written_all: Set[int] = set()
    for c in rf.cmds:
        written_all |= codegen.cmd_written(c)
    views = set()
    for c in rf.cmds:
        views |= set(codegen.cmd_views(c, written_all))
    bufs = sorted(v for v in views if v[0] not in rf.internal)
    rng = {"G": (0, V * R - 1), "X": (0, V - 1), "Y": (0, R - 1)}
    it = "int"
    for c in rf.cmds:
        if codegen.index_type(c, rng) != "int":
            it = "long long"
    if V * R >= (1 << 31) - 64:
        it = "long long"
    em = Emitter(bufs, it, written_all)
    lines: List[str] = []
    st_run = run_state(rf.cmds, V, R)
    kinds = st_run.kinds
    staged = sorted(b for b, pat in st_run.read_pattern.items()
                    if pat == "row" and b not in kinds and b not in rf.internal)
    slot_bytes = len(staged) * R * 4
    nslot = max(2, min(MAX_SLOTS, STAGE_SMEM_MAX // max(slot_bytes, 1)))
    stage_bytes = nslot * slot_bytes
    staged_mode = rows_pb == 1 and staged and stage_bytes <= STAGE_SMEM_MAX
    if not staged_mode:
        staged = []
    sidx = {b: i for i, b in enumerate(staged)}
    U = R // VEC   # float4 units per row
    # register state
    row_regs: Dict[int, List[List[str]]] = {}     # full-size buffer -> [chunk][lane] var names
    sc_regs: Dict[int, str] = {}                   # per-row scalar buffer -> var
    decl: List[str] = []
    # register names by position, not buffer id: runs that differ only in their
    # buffers get identical sources (and batch into one launch)
    for v, (b, kind) in enumerate(sorted(kinds.items())):
        if kind == "row":
            row_regs[b] = [[f"r{v}_{k}_{j}" for j in range(VEC)] for k in range(nc)]
            decl.append("float " + ", ".join(f"r{v}_{k}_{j} = 0.0f" for k in range(nc) for j in range(VEC)) + ";")
        else:
            sc_regs[b] = f"s{v}"
            decl.append(f"float s{v} = 0.0f;")

    defined: Set = set()   # (buffer, chunk) for row buffers, buffer for scalars: value is in registers
    staged_loaded: Set = set()

    def staged_reg(b: int, k: int) -> str:
        """The row's chunk k of staged input b, read from shared memory once per row."""
        name_ = f"c{b}_{k}"
        if (b, k) not in staged_loaded:
            staged_loaded.add((b, k))
            decl.append(f"float4 {name_};")
            lines.append(f"{name_} = stg[(slot * {len(staged)} + {sidx[b]}) * {U} + {k} * {gs} + tig];")
        return name_

    def gbase(k: int) -> str:
        return f"(rowbase + ((({it}){k} * {gs} + tig) * {VEC}))"

    # --- full-size statements for chunk k
    def emit_full(c, k: int):
        temps = [dict() for _ in range(VEC)]
        env0 = {"G": f"g{k}"}

        def val(karg, out: List[str]):
            if isinstance(karg, ir.KConstant):
                for j in range(VEC):
                    out.append(flit(karg.constant))
                return
            if isinstance(karg, ir.KMatrix):
                if karg.is_temp:
                    for j in range(VEC):
                        out.append(temps[j][karg.id])
                    return
                if karg.id in row_regs and (karg.id, k) in defined:
                    for j in range(VEC):
                        out.append(row_regs[karg.id][k][j])
                    return
                if karg.id in sc_regs and karg.id in defined:
                    for j in range(VEC):
                        out.append(sc_regs[karg.id])
                    return
                if karg.id in sidx:
                    q = staged_reg(karg.id, k)
                    out.extend(f"{q}.{cmp}" for cmp in "xyzw")
                    return
                ln = exprs.lanes(karg.access, "G", VEC)
                if ln.unit(VEC):
                    q = em.tmp("q")
                    lines.append(f"const float4 {q} = *reinterpret_cast<const float4*>(&{em.at(karg, env0)});")
                    out.extend(f"{q}.{cmp}" for cmp in "xyzw")
                elif ln.uniform:
                    u = em.tmp("u")
                    lines.append(f"const float {u} = {em.at(karg, env0)};")
                    out.extend([u] * VEC)
                else:
                    for j in range(VEC):
                        u = em.tmp("u")
                        lines.append(f"const float {u} = {em.at(karg, {'G': f'(g{k} + ({it}){j})'})};")
                        out.append(u)
                return
            for j in range(VEC):   # KConcat on an input buffer: per-lane select
                u = em.tmp("u")
                lines.append(f"const float {u} = {em.scalar_karg(karg, {'G': f'(g{k} + ({it}){j})'}, temps[j])};")
                out.append(u)

        for n in codegen.chain_nodes(c):
            nk = type(n).__name__
            args = []
            for karg in n.kargs:
                vs: List[str] = []
                val(karg, vs)
                args.append(vs)
            res = []
            for j in range(VEC):
                if nk == "BinaryNode":
                    res.append(binary_expr(n.op, args[0][j], args[1][j]))
                elif nk == "UnaryNode":
                    res.append(unary_expr(n.op, args[0][j]))
                else:
                    res.append(args[0][j])
            if n.kres.is_temp:
                for j in range(VEC):
                    t = em.tmp("t")
                    lines.append(f"const float {t} = {res[j]};")
                    temps[j][n.kres.id] = t
                continue
            b = n.kres.id
            if b in row_regs:
                tv = [em.tmp("w") for _ in range(VEC)]
                for j in range(VEC):
                    lines.append(f"const float {tv[j]} = {res[j]};")
                for j in range(VEC):
                    lines.append(f"{row_regs[b][k][j]} = {tv[j]};")
                defined.add((b, k))
                if b not in rf.internal:
                    lines.append(f"if (live) *reinterpret_cast<float4*>(&{em.at(n.kres, env0)}) = "
                                 f"make_float4({', '.join(tv)});")
            else:
                raise AssertionError("full-size write to a non-row buffer")

    # --- per-row scalar statements (uniform across the row's threads)
    def emit_scalar_chain(nodes, head_value: Optional[str] = None):
        temps: Dict[int, str] = {}
        env = {"G": "xr", "X": "xr", "Y": f"(({it})0)"}
        for n in nodes:
            nk = type(n).__name__
            if nk == "ReduceNode":
                r = head_value
            else:
                args = []
                for karg in n.kargs:
                    if isinstance(karg, ir.KMatrix) and not karg.is_temp and karg.id in defined:
                        args.append(sc_regs[karg.id])
                    elif isinstance(karg, ir.KMatrix) and not karg.is_temp:
                        u = em.tmp("u")
                        lines.append(f"const float {u} = live ? {em.at(karg, env)} : 0.0f;")
                        args.append(u)
                    else:
                        args.append(em.scalar_karg(karg, env, temps))
                r = binary_expr(n.op, args[0], args[1]) if nk == "BinaryNode" else \
                    (unary_expr(n.op, args[0]) if nk == "UnaryNode" else args[0])
            if n.kres.is_temp:
                t = em.tmp("e")
                lines.append(f"const float {t} = {r};")
                temps[n.kres.id] = t
                continue
            b = n.kres.id
            tv = em.tmp("w")
            lines.append(f"const float {tv} = {r};")
            lines.append(f"{sc_regs[b]} = {tv};")
            defined.add(b)
            if b not in rf.internal:
                lines.append(f"if (live && tig == 0) {em.at(n.kres, env)} = {tv};")

    # consecutive reductions are independent of each other (a reduction reads a full
    # row buffer and writes per-row scalars), so a group of them shares one
    # shared-memory exchange and one barrier; their epilogues then run in order.
    groups: List[List] = []
    for c in rf.cmds:
        ck = _cmd_kind(c, V, R)
        if ck == "reduce" and groups and groups[-1][0] == "reduce":
            groups[-1][1].append(c)
        else:
            groups.append([ck, [c]])
    max_group = max([len(g[1]) for g in groups if g[0] == "reduce"] or [1])
    n_red = 0
    for ck, members in groups:
        if ck == "full":
            c = members[0]
            for k in range(nc):
                lines.append(f"{{ // chunk {k}")
                emit_full(c, k)
                lines.append("}")
            continue
        if ck == "scalar":
            lines.append("{")
            emit_scalar_chain(codegen.chain_nodes(members[0]))
            lines.append("}")
            continue
        accs = []
        combs = []
        for c in members:
            rn = c if type(c).__name__ == "ReduceNode" else c.init_node
            op = rn.op
            ident = "0.0f" if op == "SUM" else "(__int_as_float(0xff800000))"
            comb = (lambda a, b: f"({a} + {b})") if op == "SUM" else (lambda a, b: f"fmaxf({a}, {b})")
            src = rn.kargs[0]
            acc = em.tmp("acc")
            accs.append(acc)
            combs.append(comb)
            lines.append(f"float {acc} = {ident};")
            for k in range(nc):
                env0 = {"X": "xr", "Y": f"((({it}){k} * {gs} + tig) * {VEC})", "G": "xr"}
                if isinstance(src, ir.KMatrix) and not src.is_temp and (src.id, k) in defined:
                    vs = row_regs[src.id][k]
                    lines.append(f"{acc} = {comb(acc, comb(comb(vs[0], vs[1]), comb(vs[2], vs[3])))};")
                elif isinstance(src, ir.KMatrix) and not src.is_temp and src.id in sidx:
                    q = staged_reg(src.id, k)
                    lines.append(f"{acc} = {comb(acc, comb(comb(q + '.x', q + '.y'), comb(q + '.z', q + '.w')))};")
                elif isinstance(src, ir.KConstant):
                    lines.append(f"{acc} = {comb(acc, flit(src.constant))};" if op == "MAX" else
                                 f"{acc} = {acc} + {VEC}.0f * {flit(src.constant)};")
                else:
                    ly = exprs.lanes(src.access, "Y", VEC) if isinstance(src, ir.KMatrix) else exprs.OTHER
                    if ly.unit(VEC):
                        q = em.tmp("q")
                        lines.append(f"const float4 {q} = live ? *reinterpret_cast<const float4*>(&{em.at(src, env0)})"
                                     f" : make_float4({ident}, {ident}, {ident}, {ident});")
                        lines.append(f"{acc} = {comb(acc, comb(comb(q + '.x', q + '.y'), comb(q + '.z', q + '.w')))};")
                    else:
                        for j in range(VEC):
                            envj = {"X": "xr", "Y": f"(((({it}){k} * {gs} + tig) * {VEC}) + {j})", "G": "xr"}
                            lines.append(f"if (live) {acc} = {comb(acc, em.scalar_karg(src, envj, {}))};")
        # group reduction, results broadcast to all threads of the row group
        w = min(gs, 32)
        lines.append(f"#pragma unroll\nfor (int o = {w // 2}; o > 0; o >>= 1) {{")
        for acc, comb in zip(accs, combs):
            lines.append(f"    {acc} = {comb(acc, f'__shfl_xor_sync(0xffffffffu, {acc}, o)')};")
        lines.append("}")
        if gs > 32:
            nw = gs // 32
            slot_r = n_red % 2
            for ai, acc in enumerate(accs):
                lines.append(f"if ((threadIdx.x & 31) == 0) red[{slot_r}][{ai}][threadIdx.x >> 5] = {acc};")
            lines.append("__syncthreads();")
            nw_all = max(1, block // 32)
            for ai, (acc, comb) in enumerate(zip(accs, combs)):
                if nw % 4 == 0 and nw_all % 4 == 0:
                    # 16-byte reads of the warp partials, summed in the same order
                    parts = []
                    for q4 in range(nw // 4):
                        v = f"rq{n_red}_{ai}_{q4}"
                        lines.append(f"const float4 {v} = *reinterpret_cast<const float4*>"
                                     f"(&red[{slot_r}][{ai}][grp * {nw} + {4 * q4}]);")
                        parts += [f"{v}.x", f"{v}.y", f"{v}.z", f"{v}.w"]
                else:
                    parts = [f"red[{slot_r}][{ai}][grp * {nw} + {i}]" for i in range(nw)]
                tot = parts[0]
                for pp in parts[1:]:
                    tot = comb(tot, pp)
                lines.append(f"{acc} = {tot};")
        n_red += 1
        for c, acc in zip(members, accs):
            lines.append("{")
            emit_scalar_chain(codegen.chain_nodes(c), acc)
            lines.append("}")
    params = ", ".join([f"float* __restrict__ p{i}" for i in range(len(bufs))] + ["int* __restrict__ err"])
    nw_tot = max(1, block // 32)
    body_lines = decl + [f"const {it} g{k} = {gbase(k)};" for k in range(nc)] + lines
    if not staged_mode:
        body = "\n    ".join(body_lines)
        src = f"""extern "C" __global__ void __launch_bounds__({block}) {name}({params}) {{
    __shared__ __align__(16) float red[2][{max_group}][{nw_tot}];
    const int tig = threadIdx.x % {gs};
    const int grp = threadIdx.x / {gs};
    (void)grp; (void)red; (void)err;
    const {it} xr = ({it})blockIdx.x * {rows_pb} + grp;
    const bool live = xr < ({it}){V};
    const {it} rowbase = (live ? xr : ({it})0) * ({it}){R};
    {body}
}}
"""
        grid = ((V + rows_pb - 1) // rows_pb, 1, 1)
        smem = 0
    else:
        body = "\n        ".join(body_lines)
        row_bytes = R * 4
        issue = "\n            ".join(
            f"bulk_g2s(&stg[(s * {len(staged)} + {i}) * {U}], {em.p(b, 0)} + ({it})row * {R}, {row_bytes}u, &bar[s]);"
            for i, b in enumerate(staged))
        src = f"""
__device__ __forceinline__ unsigned rf_smem(const void* p) {{ return (unsigned)__cvta_generic_to_shared(p); }}
__device__ __forceinline__ void bulk_g2s(void* dst, const float* src, unsigned bytes, unsigned long long* bar) {{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 :: "r"(rf_smem(dst)), "l"(src), "r"(bytes), "r"(rf_smem(bar)) : "memory");
}}
__device__ __forceinline__ bool rf_try(unsigned long long* b, unsigned ph) {{
    unsigned ok;
    asm volatile("{{\\n .reg .pred p;\\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\\n selp.u32 %0, 1, 0, p;\\n}}"
                 : "=r"(ok) : "r"(rf_smem(b)), "r"(ph) : "memory");
    return ok != 0;
}}
__device__ __noinline__ bool rf_wait(unsigned long long* b, unsigned ph) {{
    if (rf_try(b, ph)) return true;
    unsigned long long t0, t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    while (true) {{
        for (int i = 0; i < 64; ++i) if (rf_try(b, ph)) return true;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        if (t - t0 > 2000000000ull) return false;
    }}
}}

extern "C" __global__ void __launch_bounds__({block}) {name}({params}) {{
    extern __shared__ __align__(128) float4 stg[];
    __shared__ __align__(16) float red[2][{max_group}][{nw_tot}];
    __shared__ __align__(8) unsigned long long bar[{nslot}];
    const int tig = threadIdx.x;
    const int grp = 0;
    (void)grp;
    const bool live = true;
    if (threadIdx.x == 0) {{
        for (int s = 0; s < {nslot}; ++s)
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" :: "r"(rf_smem(&bar[s])));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }}
    __syncthreads();
    auto issue = [&](int s, {it} row) {{
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(rf_smem(&bar[s])), "r"({len(staged) * row_bytes}u) : "memory");
            {issue}
    }};
    // ring of {nslot} slots: row i of this block goes to slot i % {nslot}, {nslot - 1} rows ahead
    if (threadIdx.x == 0)
        for (int j = 0; j < {nslot - 1}; ++j)
            if (({it})blockIdx.x + ({it})j * gridDim.x < ({it}){V}) issue(j, ({it})blockIdx.x + ({it})j * gridDim.x);
    int iter = 0;
    for ({it} xr = blockIdx.x; xr < ({it}){V}; xr += gridDim.x, ++iter) {{
        const int slot = iter % {nslot};
        const {it} nxt = xr + ({it}){nslot - 1} * gridDim.x;
        // this barrier also ends every thread's use of the previous row's slot, which
        // the prefetch below overwrites (so no barrier is needed at the end of a row)
        const bool ok = __syncthreads_and(rf_wait(&bar[slot], (iter / {nslot}) & 1));
        if (!ok) {{
            if (threadIdx.x == 0) {{
                atomicExch(err, 5);
                // bounded drain of the copies still in flight before the block exits
                for (int j = 1; j < {nslot - 1}; ++j)
                    if (xr + ({it})j * gridDim.x < ({it}){V})
                        rf_wait(&bar[(iter + j) % {nslot}], ((iter + j) / {nslot}) & 1);
            }}
            break;
        }}
        if (threadIdx.x == 0 && nxt < ({it}){V}) issue((iter + {nslot - 1}) % {nslot}, nxt);
        const {it} rowbase = xr * ({it}){R};
        {body}
    }}
}}
"""
        grid = (min(V, GRID_PER_SM * sm_count), 1, 1)
        smem = stage_bytes
    # algorithmic bytes: external reads + external writes (extents)
    nbytes = 0
    reads, writes = rf.accesses()
    for c in rf.cmds:
        pass
    seen_r: Dict[int, Tuple[int, int]] = {}
    seen_w: Dict[int, Tuple[int, int]] = {}
    for c in rf.cmds:
        ck = _cmd_kind(c, V, R)
        for n in codegen.chain_nodes(c):
            if type(n).__name__ == "ReduceNode":
                rg = {"X": (0, V - 1), "Y": (0, R - 1), "G": (0, V - 1)}
            elif ck == "full":
                rg = {"G": (0, V * R - 1)}
            else:
                rg = {"G": (0, V - 1), "X": (0, V - 1), "Y": (0, 0)}
            for k in n.kargs:
                for km in _kmats(k):
                    if km.id in rf.internal or km.id in seen_w:
                        continue
                    lo, hi = exprs.bounds(km.access, rg)
                    o = seen_r.get(km.id)
                    seen_r[km.id] = (lo, hi) if o is None else (min(o[0], lo), max(o[1], hi))
            if not n.kres.is_temp and n.kres.id not in rf.internal:
                rgw = {"G": (0, V * R - 1)} if ck == "full" and type(n).__name__ != "ReduceNode" else \
                    {"G": (0, V - 1), "X": (0, V - 1), "Y": (0, 0)}
                lo, hi = exprs.bounds(n.kres.access, rgw)
                o = seen_w.get(n.kres.id)
                seen_w[n.kres.id] = (lo, hi) if o is None else (min(o[0], lo), max(o[1], hi))
    for d in (seen_r, seen_w):
        for b, (lo, hi) in d.items():
            nbytes += 4 * min(hi - lo + 1, sizes.get(b, hi - lo + 1))
    return KernelSpec(name, src, bufs, grid, (block, 1, 1), smem, "rowfused", nbytes)
