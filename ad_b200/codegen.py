"""CUDA C++ source generation for the procedural IR (one kernel per command).

Each compute command of the reference's proc -- ``ElwFuse``, ``BinaryNode``,
``UnaryNode``, ``ContigiousNode``, ``ReduceNode``, ``ReduceElwFuse``,
``DotProdNode``, ``DPElwFuse`` (dispatch list autodiff/device/opencl/device.py:52-86)
-- becomes one hand-written sm_100a template instantiated with the command's
straight-line body, then compiled by NVRTC.  The math of every statement
follows the reference's lowering (autodiff/device/opencl/karg.py:8-54,
opencl/kernels/*.py); the *schedule* is B200-native:

* elementwise: ``VEC`` = 4 consecutive elements per thread.  Each access is
  classified by ``exprs.lanes``: contiguous accesses become one 128-bit
  load/store, broadcasts (``G >> k``, ``G & m``) one scalar load, the rest a
  per-element gather.  Permute/View/Broadcast/Concat stay folded into the
  address math exactly as the reference's expressions say.
* reduce: a *row* schedule (warp or CTA per reduced row, 128-bit loads along
  the row, shuffle + shared-memory tree) when the row is contiguous, a
  *column* schedule (lanes across rows, warps along the reduced dim) when
  consecutive rows are contiguous (the ``Permute[1,0]`` bias-gradient case),
  and a per-element gather otherwise.  The fused epilogue runs once per row
  with ``_global_id = row`` (reduce_elw_fuse.py:57-62).
* dot products: see ``gemm.py`` (tcgen05/TMEM, 3xTF32) and the SIMT kernel
  here, used for tiny products and as a general fallback on the GPU.

Kernels take positional ``float*`` parameters (p0, p1, ...), one per distinct
buffer; buffer ids never appear in the source, so structurally identical
commands share one compiled kernel.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

from . import exprs
from . import ir

VEC = 4
THREADS = 256


def flit(v: float) -> str:
    """fp32 literal.  (The reference prints unsuffixed, i.e. double, literals:
    karg.py:53-54; fp32 arithmetic here is a deliberate choice, covered by the
    rel 1e-4 tolerance.)"""
    v = float(v)
    if math.isinf(v):
        return "(__int_as_float(0x7f800000))" if v > 0 else "(__int_as_float(0xff800000))"
    if math.isnan(v):
        return "(__int_as_float(0x7fffffff))"
    s = repr(v)
    if "e" not in s and "." not in s:
        s += ".0"
    return s + "f"


def unary_expr(op: str, a: str) -> str:
    """opencl/kernels/unary.py:19-33 in fp32."""
    return {
        "EXP2": f"exp2f({a})", "LOG2": f"log2f({a})", "SIN": f"sinf({a})",
        "RECIP": f"(1.0f / ({a}))", "SQRT": f"sqrtf(fabsf({a}))",
        "EQUAL": f"(({a}) == 0.0f ? 1.0f : 0.0f)", "MORE_ZERO": f"(({a}) > 0.0f ? 1.0f : 0.0f)",
        "LESS_ZERO": f"(({a}) < 0.0f ? 1.0f : 0.0f)",
        "MORE_OR_EQ_ZERO": f"(({a}) >= 0.0f ? 1.0f : 0.0f)",
        "LESS_OR_EQ_ZERO": f"(({a}) <= 0.0f ? 1.0f : 0.0f)",
    }[op]


def binary_expr(op: str, a: str, b: str) -> str:
    return f"(({a}) + ({b}))" if op == "ADD" else f"(({a}) * ({b}))"


# ---------------------------------------------------------------- kernel spec

@dataclass
class KernelSpec:
    """What the device needs to launch one generated kernel."""
    name: str
    src: str
    buffers: List[int]            # buffer ids in parameter order
    grid: Tuple[int, int, int]
    block: Tuple[int, int, int]
    smem: int = 0
    kind: str = ""
    bytes_moved: int = 0          # algorithmic bytes (unique extents read + written)
    flops: int = 0
    extra: Dict = field(default_factory=dict)


def distribute(e: ir.Expr) -> ir.Expr:
    """Move constant terms out of ``(a + c) * m`` and ``(a + c) << s``:
    ``a*m + c*m`` / ``(a << s) + (c << s)``.  Same integer value."""
    if not isinstance(e, ir.Bin):
        return e
    if e.op == "Add":
        return ir.Bin("Add", distribute(e.a), distribute(e.b))
    if e.op in ("Mult", "ShiftLeft") and isinstance(e.b, ir.Const) and e.b.val >= 0:
        inner = distribute(e.a)
        terms = _sum_terms(inner)
        if len(terms) == 1:
            return ir.Bin(e.op, inner, e.b)
        scale = e.b.val if e.op == "Mult" else (1 << e.b.val)
        out = None
        for t in terms:
            u = ir.Const(t.val * scale) if isinstance(t, ir.Const) else ir.Bin(e.op, t, e.b)
            out = u if out is None else ir.Bin("Add", out, u)
        return out
    return e


def _sum_terms(x: ir.Expr) -> List[ir.Expr]:
    if isinstance(x, ir.Bin) and x.op == "Add":
        return _sum_terms(x.a) + _sum_terms(x.b)
    return [x]


def split_offset(e: ir.Expr) -> Tuple[ir.Expr, int]:
    """``e`` as ``(rest, C)`` with ``e == rest + C``: C collects the constant terms
    of the sum after ``distribute`` (the folded Index/slice start)."""
    terms = _sum_terms(distribute(e))
    c = sum(t.val for t in terms if isinstance(t, ir.Const))
    rest = [t for t in terms if not isinstance(t, ir.Const)]
    if not rest:
        return ir.Const(0), c
    r = rest[0]
    for t in rest[1:]:
        r = ir.Bin("Add", r, t)
    return r, c


def _kmats_of(k) -> List[ir.KMatrix]:
    if isinstance(k, ir.KMatrix) and not k.is_temp:
        return [k]
    if isinstance(k, ir.KConcat):
        return _kmats_of(k.karg_one) + _kmats_of(k.karg_two)
    return []


def view_of(k: ir.KMatrix, written: set) -> Tuple[int, int]:
    """Pointer view (buffer id, element offset) for an access.  The constant
    offset of a read-only buffer moves into the pointer when that keeps 16-byte
    alignment, so commands that differ only in which slice they read share one
    kernel source (and can be batched, see ``batch.py``)."""
    if k.id in written:
        return (k.id, 0)
    _, c = split_offset(k.access)
    if c > 0 and c % 4 == 0:
        return (k.id, c)
    return (k.id, 0)


class Emitter:
    """Lowers kargs/expressions to C++ over positional pointer params.  Params
    are *views* ``(buffer id, element offset)``: see ``view_of``."""

    def __init__(self, views: Sequence, idx_t: str, written: Optional[set] = None):
        views = [v if isinstance(v, tuple) else (v, 0) for v in views]
        self.pos = {v: i for i, v in enumerate(views)}
        self.written = set(written or ())
        self.idx_t = idx_t
        self.n = 0

    def tmp(self, prefix="v") -> str:
        self.n += 1
        return f"{prefix}{self.n}"

    def p(self, buf_id: int, off: int = 0) -> str:
        return f"p{self.pos[(buf_id, off)]}"

    def ref(self, k: ir.KMatrix) -> Tuple[str, ir.Expr]:
        """(param name, index expression relative to that param) for an access."""
        v = view_of(k, self.written)
        if v[1]:
            return f"p{self.pos[v]}", split_offset(k.access)[0]
        return f"p{self.pos[v]}", k.access

    def at(self, k: ir.KMatrix, env: Dict[str, str]) -> str:
        pn, e = self.ref(k)
        return f"{pn}[{self.expr(e, env)}]"

    def expr(self, e: ir.Expr, env: Dict[str, str]) -> str:
        if isinstance(e, ir.Const):
            return f"(({self.idx_t}){e.val})"
        if isinstance(e, ir.Gid):
            return env["G"]
        if isinstance(e, ir.Xv):
            return env["X"]
        if isinstance(e, ir.Yv):
            return env["Y"]
        sym = {"Add": "+", "Minus": "-", "Mult": "*", "Div": "/", "Remainder": "%",
               "ShiftRight": ">>", "ShiftLeft": "<<", "BitwiseAnd": "&",
               "MoreThan": ">", "LessThan": "<"}[e.op]
        a = self.expr(e.a, env)
        b = self.expr(e.b, env)
        if e.op in ("MoreThan", "LessThan"):
            return f"(({self.idx_t})({a} {sym} {b}))"
        return f"({a} {sym} {b})"

    def scalar_karg(self, k: ir.KernelArg, env: Dict[str, str], temps: Dict[int, str]) -> str:
        if isinstance(k, ir.KConstant):
            return flit(k.constant)
        if isinstance(k, ir.KMatrix):
            if k.is_temp:
                return temps[k.id]
            return self.at(k, env)
        flat = concat_pieces(k)
        if flat is not None:
            var, pieces, ths = flat
            v = self.expr(var, env)

            def search(lo: int, hi: int) -> str:
                # pieces[lo:hi]; piece i is selected when var > ths[i] (ths[0] = -inf)
                if hi - lo == 1:
                    return self.scalar_karg(pieces[lo], env, temps)
                mid = (lo + hi) // 2
                return f"(({v}) > {ths[mid]} ? ({search(mid, hi)}) : ({search(lo, mid)}))"
            return search(0, len(pieces))
        c = self.expr(k.condition, env)
        return (f"({c} ? ({self.scalar_karg(k.karg_two, env, temps)}) : "
                f"({self.scalar_karg(k.karg_one, env, temps)}))")


def _gt_const(cond):
    if isinstance(cond, ir.Bin) and cond.op == "MoreThan" and isinstance(cond.b, ir.Const):
        return cond.a, cond.b.val
    return None


def concat_pieces(k):
    """A tree of ``KConcat`` whose conditions all read ``v > c`` for one
    expression ``v`` (the reference's nested concatenations along one axis,
    opencl/karg.py:52) as its in-order pieces and thresholds: piece i is the
    value where ``ths[i] < v <= ths[i + 1]``.  None unless there are at least
    4 pieces with strictly increasing thresholds.  Selecting by binary search
    over the thresholds picks the same piece as the nested conditionals."""
    gc = _gt_const(k.condition)
    if gc is None:
        return None
    var = gc[0]
    pieces, ths = [], [None]

    def walk(n) -> bool:
        if isinstance(n, ir.KConcat):
            g = _gt_const(n.condition)
            if g is not None and g[0] == var:
                if not walk(n.karg_one):
                    return False
                ths.append(g[1])
                return walk(n.karg_two)
        pieces.append(n)
        return True

    if not walk(k) or len(pieces) < 4:
        return None
    if any(b <= a for a, b in zip(ths[1:], ths[2:])):
        return None
    return var, pieces, ths


def cmd_written(c) -> set:
    w = set()
    for n in chain_nodes(c):
        w |= set(n.kres.ids(True))
    return w


def cmd_views(c, written: Optional[set] = None) -> List[Tuple[int, int]]:
    """Sorted pointer views of a command (see ``view_of``)."""
    written = cmd_written(c) if written is None else written
    vs = set()
    for n in chain_nodes(c):
        for k in n.kargs:
            for km in _kmats_of(k):
                vs.add(view_of(km, written))
        for km in _kmats_of(n.kres):
            vs.add(view_of(km, written))
    return sorted(vs)


def make_emitter(c, idx_t: str):
    w = cmd_written(c)
    views = cmd_views(c, w)
    return views, Emitter(views, idx_t, w)


def karg_buffers(k: ir.KernelArg) -> List[int]:
    return k.ids(True)


def cmd_buffers(c) -> List[int]:
    ids: List[int] = []
    nodes = c.nodes if isinstance(c, ir.FuseGroup) else [c]
    for n in nodes:
        if isinstance(n, (ir.AllocEntry, ir.DeallocEntry)):
            continue
        for k in n.kargs:
            ids += karg_buffers(k)
        ids += n.kres.ids(True)
    return sorted(set(ids))


def chain_nodes(c) -> List:
    nodes = c.nodes if isinstance(c, ir.FuseGroup) else [c]
    return [n for n in nodes if not isinstance(n, (ir.AllocEntry, ir.DeallocEntry))]


def all_exprs(c):
    out = []

    def kexprs(k):
        if isinstance(k, ir.KMatrix) and not k.is_temp:
            out.append(k.access)
        elif isinstance(k, ir.KConcat):
            out.append(k.condition)
            kexprs(k.karg_one)
            kexprs(k.karg_two)

    for n in chain_nodes(c):
        for k in n.kargs:
            kexprs(k)
        kexprs(n.kres)
    return out


def index_type(c, rng) -> str:
    m = 0
    for e in all_exprs(c):
        m = max(m, exprs.subexpr_max(e, rng))
    for v in rng.values():
        m = max(m, abs(v[0]), abs(v[1]))
    return "int" if m < (1 << 31) - 64 else "long long"


def written_reads_bytes(c, rng, sizes: Dict[int, int]) -> int:
    """Algorithmic HBM bytes of one launch: for each buffer, the extent of the
    address range it touches (capped at the buffer size), once if read and once
    if written.  A read of a buffer that an earlier statement of the same
    kernel already wrote (same thread, read-after-write) costs no DRAM traffic
    and is not counted."""
    reads: Dict[int, Tuple[int, int]] = {}
    writes: Dict[int, Tuple[int, int]] = {}

    def note(d, k, skip=()):
        if isinstance(k, ir.KMatrix) and not k.is_temp:
            if k.id in skip:
                return
            lo, hi = exprs.bounds(k.access, rng)
            o = d.get(k.id)
            d[k.id] = (lo, hi) if o is None else (min(o[0], lo), max(o[1], hi))
        elif isinstance(k, ir.KConcat):
            note(d, k.karg_one, skip)
            note(d, k.karg_two, skip)

    for n in chain_nodes(c):
        for k in n.kargs:
            note(reads, k, skip=writes)
        note(writes, n.kres)
    total = 0
    for d in (reads, writes):
        for b, (lo, hi) in d.items():
            total += 4 * min(hi - lo + 1, sizes.get(b, hi - lo + 1))
    return total


# ---------------------------------------------------------------- elementwise

def gen_elementwise(c, name: str, sizes: Dict[int, int]) -> KernelSpec:
    """ElwFuse / BinaryNode / UnaryNode / ContigiousNode
    (opencl/kernels/{elw_fuse,binary,unary,contigious}.py): one logical work
    item per element of ``prod(shape)`` with ``_global_id`` = element index."""
    kind = type(c).__name__
    n_el = math.prod(c.init_node.shape if kind == "ElwFuse" else c.shape)
    rng = {"G": (0, max(n_el - 1, 0))}
    it = index_type(c, rng)
    bufs, em = make_emitter(c, it)
    nodes = chain_nodes(c)

    def body_vec() -> List[str]:
        """VEC lanes per thread; g0 = first element (a multiple of VEC)."""
        lines: List[str] = []
        temps_l: List[Dict[int, str]] = [dict() for _ in range(VEC)]
        env0 = {"G": "g0"}

        def load(k, out_vars: List[str]) -> None:
            """Emit statements that set out_vars[j] to the value of karg k at lane j."""
            if isinstance(k, ir.KConstant):
                for j in range(VEC):
                    lines.append(f"const float {out_vars[j]} = {flit(k.constant)};")
                return
            if isinstance(k, ir.KMatrix):
                if k.is_temp:
                    for j in range(VEC):
                        lines.append(f"const float {out_vars[j]} = {temps_l[j][k.id]};")
                    return
                ln = exprs.lanes(k.access, "G", VEC)
                if ln.unit(VEC):
                    v = em.tmp("q")
                    lines.append(f"const float4 {v} = *reinterpret_cast<const float4*>(&{em.at(k, env0)});")
                    for j, comp in enumerate("xyzw"):
                        lines.append(f"const float {out_vars[j]} = {v}.{comp};")
                elif ln.uniform:
                    v = em.tmp("u")
                    lines.append(f"const float {v} = {em.at(k, env0)};")
                    for j in range(VEC):
                        lines.append(f"const float {out_vars[j]} = {v};")
                else:
                    for j in range(VEC):
                        env = {"G": f"(g0 + ({it}){j})"}
                        lines.append(f"const float {out_vars[j]} = {em.at(k, env)};")
                return
            # KConcat: cond ? two : one (opencl/karg.py:52)
            lc = exprs.lanes(k.condition, "G", VEC)
            one = [em.tmp("c") for _ in range(VEC)]
            two = [em.tmp("c") for _ in range(VEC)]
            if lc.uniform:
                cond = em.tmp("b")
                lines.append(f"const bool {cond} = {em.expr(k.condition, env0)} != 0;")
                for j in range(VEC):
                    lines.append(f"float {out_vars[j]};")
                lines.append(f"if ({cond}) {{")
                load(k.karg_two, two)
                for j in range(VEC):
                    lines.append(f"{out_vars[j]} = {two[j]};")
                lines.append("} else {")
                load(k.karg_one, one)
                for j in range(VEC):
                    lines.append(f"{out_vars[j]} = {one[j]};")
                lines.append("}")
            else:
                for j in range(VEC):
                    env = {"G": f"(g0 + ({it}){j})"}
                    lines.append(f"const float {out_vars[j]} = {em.scalar_karg(k, env, temps_l[j])};")

        for nd in nodes:
            kk = type(nd).__name__
            args = []
            for k in nd.kargs:
                vs = [em.tmp("a") for _ in range(VEC)]
                load(k, vs)
                args.append(vs)
            res = []
            for j in range(VEC):
                if kk == "BinaryNode":
                    res.append(binary_expr(nd.op, args[0][j], args[1][j]))
                elif kk == "UnaryNode":
                    res.append(unary_expr(nd.op, args[0][j]))
                else:  # ContigiousNode: plain copy
                    res.append(args[0][j])
            kres = nd.kres
            if kres.is_temp:
                for j in range(VEC):
                    t = em.tmp("t")
                    lines.append(f"const float {t} = {res[j]};")
                    temps_l[j][kres.id] = t
                continue
            ln = exprs.lanes(kres.access, "G", VEC)
            if ln.unit(VEC):
                lines.append(f"*reinterpret_cast<float4*>(&{em.at(kres, env0)}) = "
                             f"make_float4({', '.join(res)});")
            else:
                for j in range(VEC):
                    env = {"G": f"(g0 + ({it}){j})"}
                    lines.append(f"{em.at(kres, env)} = {res[j]};")
        return lines

    def body_scalar() -> List[str]:
        lines: List[str] = []
        temps: Dict[int, str] = {}
        env = {"G": "g"}
        for nd in nodes:
            kk = type(nd).__name__
            args = [em.scalar_karg(k, env, temps) for k in nd.kargs]
            if kk == "BinaryNode":
                r = binary_expr(nd.op, args[0], args[1])
            elif kk == "UnaryNode":
                r = unary_expr(nd.op, args[0])
            else:
                r = args[0]
            if nd.kres.is_temp:
                t = em.tmp("s")
                lines.append(f"const float {t} = {r};")
                temps[nd.kres.id] = t
            else:
                lines.append(f"{em.at(nd.kres, env)} = {r};")
        return lines

    vec_ok = n_el >= VEC
    params = ", ".join(f"float* __restrict__ p{i}" for i in range(len(bufs)))
    n_groups = (n_el + VEC - 1) // VEC if vec_ok else n_el
    if vec_ok:
        main = "\n        ".join(body_vec())
        tail = "\n            ".join(body_scalar())
        body = f"""
    const {it} g0 = ({it})(blockIdx.x * (long long){THREADS} + threadIdx.x) * {VEC};
    if (g0 + {VEC} <= ({it}){n_el}) {{
        {main}
    }} else if (g0 < ({it}){n_el}) {{
        for ({it} g = g0; g < ({it}){n_el}; ++g) {{
            {tail}
        }}
    }}"""
    else:
        tail = "\n        ".join(body_scalar())
        body = f"""
    const {it} g = ({it})(blockIdx.x * (long long){THREADS} + threadIdx.x);
    if (g < ({it}){n_el}) {{
        {tail}
    }}"""
    src = f"""extern "C" __global__ void __launch_bounds__({THREADS}) {name}({params}) {{{body}
}}
"""
    grid = (max(1, (n_groups + THREADS - 1) // THREADS), 1, 1)
    return KernelSpec(name, src, bufs, grid, (THREADS, 1, 1), 0, "elementwise",
                      written_reads_bytes(c, rng, sizes))


# ---------------------------------------------------------------- reduce

REDUCE_BLOCK = 256


def gen_reduce(c, name: str, sizes: Dict[int, int]) -> KernelSpec:
    """ReduceNode / ReduceElwFuse (opencl/kernels/{reduce,reduce_elw_fuse}.py).

    Row ``_x`` in [0, V) reduces ``karg(_x, _y)`` over ``_y`` in [0, R) with SUM
    or MAX.  The reference's zero-padded halving tree drops elements when
    ``ceil(R/2)*2`` is not a power of two and pads MAX with 0; this kernel
    computes the exact reduction instead (deliberate fix, identical for the
    power-of-two R the benchmarks use)."""
    kind = type(c).__name__
    rn = c if kind == "ReduceNode" else c.init_node
    V, R = rn.children_shapes[0]
    op = rn.op
    src_k = rn.kargs[0]
    rng = {"X": (0, V - 1), "Y": (0, max(R - 1, 0)), "G": (0, V - 1)}
    it = index_type(c, rng)
    bufs, em = make_emitter(c, it)
    ident = "0.0f" if op == "SUM" else "(__int_as_float(0xff800000))"
    comb = (lambda a, b: f"({a} + {b})") if op == "SUM" else (lambda a, b: f"fmaxf({a}, {b})")

    # epilogue: the fused chain after the reduce node, with _global_id = _x
    def epilogue(acc: str) -> str:
        lines = []
        temps: Dict[int, str] = {}
        env = {"G": "xr", "X": "xr", "Y": f"(({it})0)"}
        for nd in chain_nodes(c):
            kk = type(nd).__name__
            if kk == "ReduceNode":
                r = acc
            else:
                args = [em.scalar_karg(k, env, temps) for k in nd.kargs]
                r = binary_expr(nd.op, args[0], args[1]) if kk == "BinaryNode" else unary_expr(nd.op, args[0])
            if nd.kres.is_temp:
                t = em.tmp("e")
                lines.append(f"const float {t} = {r};")
                temps[nd.kres.id] = t
            else:
                lines.append(f"{em.at(nd.kres, env)} = {r};")
        return "\n            ".join(lines)

    params = ", ".join(f"float* __restrict__ p{i}" for i in range(len(bufs)))

    # classify the input access
    schedule = "row"
    row_vec = False
    col_vec = False
    if isinstance(src_k, ir.KMatrix) and not src_k.is_temp:
        ly = exprs.lanes(src_k.access, "Y", VEC)
        lx = exprs.lanes(src_k.access, "X", VEC)
        if ly.unit(VEC) and R % VEC == 0:
            row_vec = True
        elif ly.s == 1:
            pass
        elif lx.s == 1 and V >= 32:
            schedule = "col"
            col_vec = lx.unit(VEC) and V % VEC == 0
    elif isinstance(src_k, ir.KConstant):
        schedule = "const"

    if schedule == "const":
        # every element of the row is the same constant
        val = flit(src_k.constant)
        acc = f"({flit(float(R))} * {val})" if op == "SUM" else val
        if R == 0:
            acc = ident
        src = f"""extern "C" __global__ void __launch_bounds__({REDUCE_BLOCK}) {name}({params}) {{
    const {it} xr = ({it})(blockIdx.x * (long long){REDUCE_BLOCK} + threadIdx.x);
    if (xr < ({it}){V}) {{
            {epilogue(acc)}
    }}
}}
"""
        grid = ((V + REDUCE_BLOCK - 1) // REDUCE_BLOCK, 1, 1)
        return KernelSpec(name, src, bufs, grid, (REDUCE_BLOCK, 1, 1), 0, "reduce",
                          written_reads_bytes(c, rng, sizes))

    if schedule == "row":
        per = VEC if row_vec else 1
        units = (R + per - 1) // per
        gs = 32
        while gs < 512 and gs * 4 < units:
            gs *= 2
        rows_per_block = max(1, REDUCE_BLOCK // gs)
        block = gs * rows_per_block
        warps_per_group = gs // 32
        env = {"X": "xr", "Y": "yy", "G": "xr"}
        upt_all = (units + gs - 1) // gs
        upt = min(upt_all, 8)          # loads per thread in flight before combining
        chunks = (upt_all + upt - 1) // upt
        if row_vec:
            ldv = (f"*reinterpret_cast<const float4*>(&{em.at(src_k, env)})")
            load_stmt = f"if (yy < ({it}){R}) q[u] = {ldv};"
            fold = f"acc = {comb(comb('acc', 'q[u].x'), comb('q[u].y', comb('q[u].z', 'q[u].w')))};"
            qdecl = f"float4 q[{upt}];"
            qinit = f"q[u] = make_float4({ident}, {ident}, {ident}, {ident});"
        else:
            load_stmt = f"if (yy < ({it}){R}) q[u] = {em.scalar_karg(src_k, env, {})};"
            fold = f"acc = {comb('acc', 'q[u]')};"
            qdecl = f"float q[{upt}];"
            qinit = f"q[u] = {ident};"
        shfl = comb("acc", "__shfl_xor_sync(0xffffffffu, acc, o)")
        cross = ""
        if warps_per_group > 1:
            cross = f"""
        __shared__ float red[{REDUCE_BLOCK // 32}];
        if (lane == 0) red[wid] = acc;
        __syncthreads();
        if (tig < 32) {{
            const int g0w = (threadIdx.x / {gs}) * {warps_per_group};
            acc = (lane < {warps_per_group}) ? red[g0w + lane] : {ident};
            #pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc = {shfl};
        }}"""
        src = f"""extern "C" __global__ void __launch_bounds__({block}) {name}({params}) {{
    const int tig = threadIdx.x % {gs};
    const int lane = threadIdx.x & 31;
    const int wid = threadIdx.x >> 5;
    (void)wid;
    const {it} xr = ({it})blockIdx.x * {rows_per_block} + threadIdx.x / {gs};
    const bool live = xr < ({it}){V};
    float acc = {ident};
    {qdecl}
    for (int ch = 0; ch < {chunks}; ++ch) {{
        #pragma unroll
        for (int u = 0; u < {upt}; ++u) {{ {qinit} }}
        if (live) {{
            #pragma unroll
            for (int u = 0; u < {upt}; ++u) {{
                const {it} yy = (({it})tig + ({it})(ch * {upt} + u) * {gs}) * {per};
                {load_stmt}
            }}
        }}
        #pragma unroll
        for (int u = 0; u < {upt}; ++u) {{ {fold} }}
    }}
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc = {shfl};{cross}
    if (live && tig == 0) {{
            {epilogue('acc')}
    }}
}}
"""
        grid = ((V + rows_per_block - 1) // rows_per_block, 1, 1)
        return KernelSpec(name, src, bufs, grid, (block, 1, 1), 0, "reduce",
                          written_reads_bytes(c, rng, sizes))

    # column schedule: lanes across rows (contiguous), warps along the reduced dim
    per = VEC if col_vec else 1
    cols_per_block = 32 * per
    ny = 32 if R >= 256 else 8
    env = {"X": "xq", "Y": "yy", "G": "xq"}
    if col_vec:
        ld = (f"{{ const float4 q = *reinterpret_cast<const float4*>(&{em.at(src_k, env)});\n"
              f"            a0 = {comb('a0', 'q.x')}; a1 = {comb('a1', 'q.y')}; a2 = {comb('a2', 'q.z')}; a3 = {comb('a3', 'q.w')}; }}")
        accs = ["a0", "a1", "a2", "a3"]
    else:
        ld = f"a0 = {comb('a0', em.scalar_karg(src_k, env, {}))};"
        accs = ["a0"]
    decl = " ".join(f"float {a} = {ident};" for a in accs)
    stores = "\n    ".join(f"red[threadIdx.y][threadIdx.x * {per} + {j}] = {a};" for j, a in enumerate(accs))
    src = f"""extern "C" __global__ void __launch_bounds__({32 * ny}) {name}({params}) {{
    __shared__ float red[{ny}][{cols_per_block + 1}];
    const {it} xq = ({it})blockIdx.x * {cols_per_block} + threadIdx.x * {per};
    {decl}
    if (xq < ({it}){V}) {{
        for ({it} yy = threadIdx.y; yy < ({it}){R}; yy += {ny}) {{
            {ld}
        }}
    }}
    {stores}
    __syncthreads();
    for (int cidx = threadIdx.y * 32 + threadIdx.x; cidx < {cols_per_block}; cidx += {32 * ny}) {{
        const {it} xr = ({it})blockIdx.x * {cols_per_block} + cidx;
        if (xr < ({it}){V}) {{
            float acc = red[0][cidx];
            for (int r = 1; r < {ny}; ++r) acc = {comb('acc', 'red[r][cidx]')};
            {epilogue('acc')}
        }}
    }}
}}
"""
    grid = ((V + cols_per_block - 1) // cols_per_block, 1, 1)
    return KernelSpec(name, src, bufs, grid, (32, ny, 1), 0, "reduce",
                      written_reads_bytes(c, rng, sizes))


# ---------------------------------------------------------------- dot (SIMT)

def dot_epilogue(c, em: Emitter, it: str, acc: str, env: Dict[str, str]) -> str:
    """DotProd: ``kres = _value``; DPElwFuse: the chain with
    ``_x = ty, _y = tx, _global_id = ty * wB + tx`` (dp_elw_fuse.py:51-56)."""
    lines = []
    temps: Dict[int, str] = {}
    for nd in chain_nodes(c):
        kk = type(nd).__name__
        if kk == "DotProdNode":
            r = acc
        else:
            args = [em.scalar_karg(k, env, temps) for k in nd.kargs]
            r = binary_expr(nd.op, args[0], args[1]) if kk == "BinaryNode" else unary_expr(nd.op, args[0])
        if nd.kres.is_temp:
            t = em.tmp("e")
            lines.append(f"const float {t} = {r};")
            temps[nd.kres.id] = t
        else:
            lines.append(f"{em.at(nd.kres, env)} = {r};")
    return "\n".join(lines)


def dot_shape(c):
    dn = c if type(c).__name__ == "DotProdNode" else c.init_node
    M, K = dn.children_shapes[0]
    N = dn.children_shapes[1][1]
    return dn, M, N, K


def gen_dot_simt(c, name: str, sizes: Dict[int, int]) -> KernelSpec:
    """General fp32 CUDA-core dot product: 64x64 tile, 16-deep k slices staged
    in shared memory through the operands' access expressions (any
    Permute/Concat/constant), fp32 FMA accumulation, fused epilogue."""
    dn, M, N, K = dot_shape(c)
    rng = {"X": (0, max(M, K) - 1), "Y": (0, max(N, K) - 1), "G": (0, M * N - 1)}
    it = index_type(c, rng)
    bufs, em = make_emitter(c, it)
    A, B = dn.kargs
    la = em.scalar_karg(A, {"X": "gm", "Y": "gk"}, {})
    lb = em.scalar_karg(B, {"X": "gk", "Y": "gn"}, {})
    epi = dot_epilogue(c, em, it, "accv", {"X": "om", "Y": "on", "G": f"(om * ({it}){N} + on)"})
    epi = "\n                ".join(epi.split("\n"))
    params = ", ".join(f"float* __restrict__ p{i}" for i in range(len(bufs)))

    def contiguous(k, var):
        return isinstance(k, ir.KMatrix) and not k.is_temp and exprs.lanes(k.access, var, 4).s == 1

    # staging order: consecutive threads walk the operand's contiguous dimension
    a_k_fast = not (contiguous(A, "X") and not contiguous(A, "Y"))
    b_n_fast = not (contiguous(B, "X") and not contiguous(B, "Y"))
    a_idx = "const int kk = e % 16, mm = e / 16;" if a_k_fast else "const int mm = e % 64, kk = e / 64;"
    b_idx = "const int nn = e % 64, kb = e / 64;" if b_n_fast else "const int kb = e % 16, nn = e / 16;"
    full_mk = M % 64 == 0 and K % 16 == 0
    full_nk = N % 64 == 0 and K % 16 == 0
    a_val = la if full_mk else f"(gm < ({it}){M} && gk < ({it}){K}) ? ({la}) : 0.0f"
    b_val = lb if full_nk else f"(gn < ({it}){N} && gk < ({it}){K}) ? ({lb}) : 0.0f"
    out_guard = "true" if (M % 64 == 0 and N % 64 == 0) else f"om < ({it}){M} && on < ({it}){N}"
    nk = (K + 15) // 16
    src = f"""extern "C" __global__ void __launch_bounds__(256) {name}({params}) {{
    // double-buffered 16-deep k slices: slice t+1 is fetched into registers
    // while slice t is multiplied out of shared memory
    __shared__ __align__(16) float As[2][16][64 + 4];
    __shared__ __align__(16) float Bs[2][16][64 + 4];
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    const {it} m0 = ({it})blockIdx.y * 64, n0 = ({it})blockIdx.x * 64;
    float acc[4][4];
    #pragma unroll
    for (int i = 0; i < 4; ++i)
        #pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
    float ra[4], rb[4];
    auto fetch = [&]({it} k0) {{
        #pragma unroll
        for (int u = 0; u < 4; ++u) {{
            const int e = threadIdx.x + u * 256;
            {{ {a_idx}
               const {it} gm = m0 + mm, gk = k0 + kk;
               ra[u] = {a_val}; }}
            {{ {b_idx}
               const {it} gn = n0 + nn, gk = k0 + kb;
               rb[u] = {b_val}; }}
        }}
    }};
    auto stash = [&](int buf) {{
        #pragma unroll
        for (int u = 0; u < 4; ++u) {{
            const int e = threadIdx.x + u * 256;
            {{ {a_idx} As[buf][kk][mm] = ra[u]; }}
            {{ {b_idx} Bs[buf][kb][nn] = rb[u]; }}
        }}
    }};
    fetch(0);
    stash(0);
    __syncthreads();
    for (int t = 0; t < {nk}; ++t) {{
        const int cur = t & 1;
        if (t + 1 < {nk}) fetch(({it})(t + 1) * 16);
        #pragma unroll
        for (int kk = 0; kk < 16; ++kk) {{
            const float4 a = *reinterpret_cast<const float4*>(&As[cur][kk][ty * 4]);
            const float4 b = *reinterpret_cast<const float4*>(&Bs[cur][kk][tx * 4]);
            const float av[4] = {{a.x, a.y, a.z, a.w}}, bv[4] = {{b.x, b.y, b.z, b.w}};
            #pragma unroll
            for (int i = 0; i < 4; ++i)
                #pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }}
        if (t + 1 < {nk}) stash(cur ^ 1);
        __syncthreads();
    }}
    #pragma unroll
    for (int i = 0; i < 4; ++i)
        #pragma unroll
        for (int j = 0; j < 4; ++j) {{
            const {it} om = m0 + ty * 4 + i, on = n0 + tx * 4 + j;
            if ({out_guard}) {{
                const float accv = acc[i][j];
                {epi}
            }}
        }}
}}
"""
    grid = ((N + 63) // 64, (M + 63) // 64, 1)
    rngw = {"X": (0, M - 1), "Y": (0, N - 1), "G": (0, M * N - 1)}
    return KernelSpec(name, src, bufs, grid, (256, 1, 1), 0, "dot_simt",
                      written_reads_bytes(c, rngw, sizes), 2 * M * N * K)


def gen_dot_warp(c, name: str, sizes: Dict[int, int]) -> KernelSpec:
    """Skinny dot products (few outputs, long K: e.g. the batch-2 MLP of
    examples/linear.py): one warp per output element, lanes stride over K,
    shuffle reduction, lane 0 runs the fused epilogue."""
    dn, M, N, K = dot_shape(c)
    rng = {"X": (0, max(M, K) - 1), "Y": (0, max(N, K) - 1), "G": (0, M * N - 1)}
    it = index_type(c, rng)
    bufs, em = make_emitter(c, it)
    A, B = dn.kargs
    la = em.scalar_karg(A, {"X": "om", "Y": "kk"}, {})
    lb = em.scalar_karg(B, {"X": "kk", "Y": "on"}, {})
    epi = dot_epilogue(c, em, it, "accv", {"X": "om", "Y": "on", "G": f"(om * ({it}){N} + on)"})
    epi = "\n            ".join(epi.split("\n"))
    params = ", ".join(f"float* __restrict__ p{i}" for i in range(len(bufs)))
    src = f"""extern "C" __global__ void __launch_bounds__(256) {name}({params}) {{
    const long long w = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (w >= {M * N}LL) return;
    const {it} om = ({it})(w / {N}), on = ({it})(w % {N});
    float acc = 0.0f;
    for ({it} kk = lane; kk < ({it}){K}; kk += 32) acc = fmaf({la}, {lb}, acc);
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) {{
            const float accv = acc;
            {epi}
    }}
}}
"""
    grid = ((M * N + 7) // 8, 1, 1)
    rngw = {"X": (0, M - 1), "Y": (0, N - 1), "G": (0, M * N - 1)}
    return KernelSpec(name, src, bufs, grid, (256, 1, 1), 0, "dot_warp",
                      written_reads_bytes(c, rngw, sizes), 2 * M * N * K)
