"""CPU oracle: a C restatement of the reference's device kernels.  TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this module, and only as the checker / the timed CPU baseline.
The product path (``ad_b200``) never calls it.

What it restates (reference project file:line):

* index-expression and kernel-arg lowering   autodiff/device/opencl/karg.py:8-54
  (``buf_<id>[expr]``, ``temp_<id>`` locals, ``cond ? two : one`` for KConcat,
  constants as *double* literals exactly as the reference prints them)
* binary / unary / contigious / elw_fuse     opencl/kernels/{binary,unary,contigious,elw_fuse}.py
  (one work item per element of ``prod(shape)``; for ElwFuse the size of the
  init node; SQRT is ``sqrt(fabs(x))``; comparisons give 1.0 / 0.0)
* reduce / reduce_elw_fuse                   opencl/kernels/{reduce,reduce_elw_fuse}.py
  (one work-group per row ``_x``; ``local = ceil(R/2)*2`` zero-padded scratch,
  halving tree ``for off = local/2; off > 0; off >>= 1``, result from
  ``scratch[0]``; the fused epilogue runs with ``_global_id = _x``)
* dotprod / dp_elw_fuse                      opencl/kernels/{dotprod,dp_elw_fuse}.py
  (fp32 accumulation in k order; epilogue with ``_x = ty, _y = tx,
  _global_id = ty * wB + tx``)
* device walk                                autodiff/device/opencl/device.py:46-130
  (init pass, then run pass with ForNode bodies replayed ``len(r)`` times)
* Feeder offset semantics                    autodiff/device/cuda/cuda_helper.py:113-119
  (the Feeder writes at ``kres`` offset; the OpenCL path's offset 0 at
  cl_helper.py:326 is a bug and is not reproduced)
* Receiver offsets                           autodiff/kernalize/__init__.py:74-83

The kernel bodies are C; ``<tgmath.h>`` gives OpenCL C's type-generic math
(``exp2`` on a float is the float function, ``1.0/x`` is a double division),
so the arithmetic follows the OpenCL source.  Parallel loops use OpenMP.

Set ``faithful_tree=False`` to replace the reference's halving tree by a plain
sequential reduction (used to check the deliberate fix for non-power-of-two
reduce sizes, where the reference tree drops elements).
"""
from __future__ import annotations

import ctypes
import re
import hashlib
import math
import os
import subprocess
import sys
import tempfile
from typing import Dict, List, Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
from ad_b200 import ir  # noqa: E402  (IR data classes only)

CACHE = os.environ.get("AD_ORACLE_CACHE", os.path.join(HERE, "_cache"))

# ---------------------------------------------------------------- lowering


def lower_expr(e: ir.Expr) -> str:
    """opencl/karg.py:8-43."""
    if isinstance(e, ir.Const):
        return f"{e.val}LL"
    if isinstance(e, ir.Gid):
        return "_global_id"
    if isinstance(e, ir.Xv):
        return "_x"
    if isinstance(e, ir.Yv):
        return "_y"
    sym = {"Add": "+", "Minus": "-", "Mult": "*", "Div": "/", "Remainder": "%",
           "ShiftRight": ">>", "ShiftLeft": "<<", "BitwiseAnd": "&",
           "MoreThan": ">", "LessThan": "<"}[e.op]
    return f"({lower_expr(e.a)} {sym} {lower_expr(e.b)})"


def lit(v: float) -> str:
    """A constant exactly as the reference prints it: Python ``str(float)``
    (opencl/karg.py:53-54) -- an unsuffixed, i.e. double, literal."""
    s = repr(float(v))
    if s in ("inf", "-inf", "nan"):
        return {"inf": "INFINITY", "-inf": "(-INFINITY)", "nan": "NAN"}[s]
    return s


def lower_karg(k: ir.KernelArg) -> str:
    """opencl/karg.py:45-54."""
    if isinstance(k, ir.KMatrix):
        return f"temp_{k.id}" if k.is_temp else f"buf_{k.id}[{lower_expr(k.access)}]"
    if isinstance(k, ir.KConcat):
        return f"({lower_expr(k.condition)} ? ({lower_karg(k.karg_two)}) : ({lower_karg(k.karg_one)}))"
    return lit(k.constant)


def lower_unary(c: ir.UnaryNode) -> str:
    """opencl/kernels/unary.py:8-33."""
    a = lower_karg(c.kargs[0])
    e = {
        "EXP2": f"exp2({a})", "LOG2": f"log2({a})", "SIN": f"sin({a})",
        "RECIP": f"1.0/{a}", "SQRT": f"sqrt(fabs({a}))",
        "EQUAL": f"({a} == 0.0f) ? 1.0 : 0.0", "MORE_ZERO": f"({a} > 0.0f) ? 1.0 : 0.0",
        "LESS_ZERO": f"({a} < 0.0f) ? 1.0 : 0.0", "MORE_OR_EQ_ZERO": f"({a} >= 0.0f) ? 1.0 : 0.0",
        "LESS_OR_EQ_ZERO": f"({a} <= 0.0f) ? 1.0 : 0.0",
    }[c.op]
    return f"{lower_karg(c.kres)} = {e};"


def lower_binary(c: ir.BinaryNode) -> str:
    """opencl/kernels/binary.py:8-17."""
    op = "+" if c.op == "ADD" else "*"
    return f"{lower_karg(c.kres)} = {lower_karg(c.kargs[0])} {op} {lower_karg(c.kargs[1])};"


def lower_chain(nodes, head_stmt) -> str:
    """Straight-line body of a fused group (opencl/kernels/elw_fuse.py:13-25,
    reduce_elw_fuse.py:12-26, dp_elw_fuse.py:11-25).  ``head_stmt(node)``
    lowers the group's init node (reduce / dot)."""
    out = []
    for n in nodes:
        if isinstance(n, ir.BinaryNode):
            out.append(lower_binary(n))
        elif isinstance(n, ir.UnaryNode):
            out.append(lower_unary(n))
        elif isinstance(n, ir.AllocEntry):
            if n.is_temp:
                out.append(f"float temp_{n.id} = 0.0;")  # karg.py:87-89
        elif isinstance(n, (ir.ReduceNode, ir.DotProdNode)):
            out.append(head_stmt(n))
    return "\n        ".join(out)


def arg_ids(c) -> List[int]:
    """Buffers a command touches, in a fixed order (opencl/karg.py:56-85 keeps a set)."""
    ids: List[int] = []
    nodes = c.nodes if isinstance(c, ir.FuseGroup) else [c]
    for n in nodes:
        if isinstance(n, (ir.AllocEntry, ir.DeallocEntry)):
            continue
        for k in n.kargs:
            ids += k.ids(True)
        ids += n.kres.ids(True)
    return sorted(set(ids))


def gen_kernel(c, name: str, faithful_tree: bool = True, dot_rows: Optional[int] = None) -> str:
    ids = arg_ids(c)
    head = "".join(f"    float *buf_{i} = B[{j}];\n" for j, i in enumerate(ids))
    kind = type(c).__name__
    if kind in ("BinaryNode", "UnaryNode", "ContigiousNode", "ElwFuse"):
        if kind == "ElwFuse":
            n = math.prod(c.init_node.shape)
            body = lower_chain(c.nodes, None)
        else:
            n = math.prod(c.shape)
            body = {"BinaryNode": lower_binary, "UnaryNode": lower_unary,
                    "ContigiousNode": lambda x: f"{lower_karg(x.kres)} = {lower_karg(x.kargs[0])};"}[kind](c)
        return f"""void {name}(float **B) {{
{head}    #pragma omp parallel for schedule(static)
    for (long long _global_id = 0; _global_id < {n}LL; ++_global_id) {{
        {body}
    }}
}}
"""
    if kind in ("ReduceNode", "ReduceElwFuse"):
        rn = c if kind == "ReduceNode" else c.init_node
        vec, red = rn.children_shapes[0]
        local = int(math.ceil(red / 2) * 2)
        if kind == "ReduceNode":
            epi = f"{lower_karg(rn.kres)} = scratch[0];"
        else:
            epi = lower_chain(c.nodes, lambda n: f"{lower_karg(n.kres)} = scratch[0];")
        combine = ("scratch[_y] += scratch[_y + _off];" if rn.op == "SUM"
                   else "scratch[_y] = fmax(scratch[_y], scratch[_y + _off]);")
        if faithful_tree:
            tree = f"""for (long long _off = {local} / 2; _off > 0; _off >>= 1)
            for (long long _y = 0; _y < _off; ++_y) {combine}"""
        else:
            acc = "scratch[0] += scratch[_y];" if rn.op == "SUM" else "scratch[0] = fmax(scratch[0], scratch[_y]);"
            tree = f"for (long long _y = 1; _y < {red}; ++_y) {acc}"
        src = lower_karg(rn.kargs[0])
        return f"""void {name}(float **B) {{
{head}    #pragma omp parallel for schedule(static)
    for (long long _x = 0; _x < {vec}LL; ++_x) {{
        float scratch[{max(local, 1)}];
        for (long long _y = 0; _y < {local}; ++_y) scratch[_y] = (_y < {red}) ? {src} : 0.0f;
        {tree}
        long long _y = 0; (void)_y;
        long long _global_id = _x; (void)_global_id;
        {epi}
    }}
}}
"""
    if kind in ("DotProdNode", "DPElwFuse"):
        dn = c if kind == "DotProdNode" else c.init_node
        m, kdim = dn.children_shapes[0]
        if dot_rows is not None:
            m = min(m, dot_rows)   # bounded CPU-baseline sample: first rows only
        ncol = dn.children_shapes[1][1]
        if kind == "DotProdNode":
            epi = f"{lower_karg(dn.kres)} = _value;"
        else:
            epi = lower_chain(c.nodes, lambda n: f"{lower_karg(n.kres)} = _value;")
        # Same arithmetic as the reference's per-output loop (fp32 products added in
        # k order, no FMA contraction), restated with dense gathered operands and the
        # output row as the inner loop so the compiler vectorises across outputs.
        return f"""void {name}(float **B) {{
{head}    float *_A = (float *)malloc(sizeof(float) * {m}LL * {kdim}LL);
    float *_Bm = (float *)malloc(sizeof(float) * {kdim}LL * {ncol}LL);
    #pragma omp parallel for schedule(static)
    for (long long _x = 0; _x < {m}LL; ++_x)
        for (long long _y = 0; _y < {kdim}LL; ++_y) _A[_x * {kdim}LL + _y] = {lower_karg(dn.kargs[0])};
    #pragma omp parallel for schedule(static)
    for (long long _x = 0; _x < {kdim}LL; ++_x)
        for (long long _y = 0; _y < {ncol}LL; ++_y) _Bm[_x * {ncol}LL + _y] = {lower_karg(dn.kargs[1])};
    #pragma omp parallel
    {{
        float *_acc = (float *)malloc(sizeof(float) * {ncol}LL);
        #pragma omp for schedule(static)
        for (long long _ty = 0; _ty < {m}LL; ++_ty) {{
            for (long long _tx = 0; _tx < {ncol}LL; ++_tx) _acc[_tx] = 0.0f;
            for (long long _k = 0; _k < {kdim}LL; ++_k) {{
                const float _a = _A[_ty * {kdim}LL + _k];
                const float *_b = _Bm + _k * {ncol}LL;
                for (long long _tx = 0; _tx < {ncol}LL; ++_tx) _acc[_tx] += _a * _b[_tx];
            }}
            for (long long _tx = 0; _tx < {ncol}LL; ++_tx) {{
                const float _value = _acc[_tx];
                long long _x = _ty, _y = _tx;
                long long _global_id = _ty * {ncol}LL + _tx; (void)_global_id;
                {epi}
            }}
        }}
        free(_acc);
    }}
    free(_A);
    free(_Bm);
}}
"""
    raise TypeError(kind)


# ---------------------------------------------------------------- build


def default_flags() -> List[str]:
    """``-O3`` for AVX2 hosts (x86-64-v3, which every current server CPU
    implements, so a library built on one host runs on another), else ``-O2``.
    No FMA contraction and no fast-math: each product and sum is rounded to fp32
    exactly as in the reference kernels."""
    try:
        with open("/proc/cpuinfo") as f:
            cpu = f.read(1 << 16)
    except OSError:
        cpu = ""
    isa = ["-march=x86-64-v3"] if all(f" {x}" in cpu for x in ("avx2", "fma", "bmi2", "movbe")) else []
    return ["-O3" if isa else "-O2", *isa, "-fopenmp", "-fno-fast-math", "-ffp-contract=off"]


def compile_kernels(srcs: Dict[str, str], flags: Optional[List[str]] = None) -> ctypes.CDLL:
    """Compile the kernels into one shared library (cached by source, flags and
    host CPU).  Large programs are split into one translation unit per host
    core, compiled in parallel and linked."""
    hdr = "#include <tgmath.h>\n#include <math.h>\n#include <float.h>\n#include <stdlib.h>\n\n"
    bodies = list(srcs.values())
    flags = flags or default_flags()
    key = hashlib.sha1((hdr + "\n".join(bodies) + " ".join(flags)).encode()).hexdigest()[:20]
    os.makedirs(CACHE, exist_ok=True)
    so = os.path.join(CACHE, f"k_{key}.so")
    if not os.path.exists(so):
        nparts = max(1, min(os.cpu_count() or 1, len(bodies) // 64))
        with tempfile.TemporaryDirectory() as td:
            jobs, objs = [], []
            for i in range(nparts):
                c = os.path.join(td, f"k{i}.c")
                with open(c, "w") as f:
                    f.write(hdr + "\n".join(bodies[i::nparts]))
                o = os.path.join(td, f"k{i}.o")
                objs.append(o)
                jobs.append(subprocess.Popen(["gcc", *flags, "-fPIC", "-c", "-o", o, c],
                                             stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True))
            for j in jobs:
                _, err = j.communicate()
                if j.returncode != 0:
                    raise RuntimeError("oracle C compile failed:\n" + err[-4000:])
            tmp = so + f".{os.getpid()}.tmp"
            r = subprocess.run(["gcc", "-fopenmp", "-shared", "-o", tmp, *objs, "-lm"],
                               capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError("oracle C link failed:\n" + r.stderr[-4000:])
            os.replace(tmp, so)
    return ctypes.CDLL(so)


# ---------------------------------------------------------------- executor


class OracleDevice:
    """CPU executor with the reference device's walk (opencl/device.py:46-130)."""

    def __init__(self, faithful_tree: bool = True, threads: Optional[int] = None,
                 dot_rows: Optional[int] = None, f64: bool = False):
        """``f64=True``: the same kernels with every float (buffers, temporaries,
        accumulators) widened to double -- a near-exact value of what the
        reference computes, used to judge rounding differences between two fp32
        results (never as the checked result itself)."""
        self.f64 = f64
        self.dtype = np.float64 if f64 else np.float32
        self.faithful_tree = faithful_tree
        self.dot_rows = dot_rows
        self.buffers: Dict[int, np.ndarray] = {}
        self.kernels = {}
        if threads is not None:
            os.environ["OMP_NUM_THREADS"] = str(threads)

    # init pass: allocate buffers and build every kernel once
    def prepare(self, proc: ir.Proc) -> None:
        proc = ir.conv_proc(proc)
        self.proc = proc
        srcs = {}
        self._cmds = []
        aliases = []
        for c in ir.iter_cmds(proc):
            if isinstance(c, ir.AllocEntry) and not c.is_temp and getattr(c, "alias", None):
                aliases.append(c)
            elif isinstance(c, ir.AllocEntry) and not c.is_temp:
                buf = np.zeros(c.size, dtype=self.dtype)
                if c.content is not None:
                    buf[:] = np.asarray(c.content, dtype=np.float32).reshape(-1)
                self.buffers[c.id] = buf
            elif type(c).__name__ in ir.COMPUTE_KINDS:
                name = f"k{len(srcs)}"
                srcs[name] = gen_kernel(c, name, self.faithful_tree, self.dot_rows)
                self._cmds.append((c, name))
        for c in aliases:   # views into another buffer (ad_b200.dist gradient slices)
            base, off = c.alias
            self.buffers[c.id] = self.buffers[base][off:off + c.size]
        if self.f64:
            srcs = {k: re.sub(r"\bfloat\b", "double", v) for k, v in srcs.items()}
        lib = compile_kernels(srcs) if srcs else None
        for c, name in self._cmds:
            fn = getattr(lib, name)
            fn.argtypes = [ctypes.POINTER(ctypes.c_void_p)]
            fn.restype = None
            ids = arg_ids(c)
            ptrs = (ctypes.c_void_p * max(len(ids), 1))(*[self.buffers[i].ctypes.data for i in ids])
            self.kernels[id(c)] = (fn, ptrs)

    def run_cmd(self, c) -> None:
        kind = type(c).__name__
        if kind in ir.COMPUTE_KINDS:
            fn, ptrs = self.kernels[id(c)]
            fn(ptrs)
        elif kind == "Feeder":
            arr = c.func()
            assert isinstance(arr, np.ndarray) and list(arr.shape) == list(c.shape), "Invalid function"
            off = offset_of(c.kres)
            self.buffers[c.kres.id][off:off + arr.size] = arr.reshape(-1)
        elif kind == "AllReduceWait":
            pass                      # the oracle's all-reduce is synchronous
        elif kind == "AllReduce":
            # data-parallel gradient sum (ad_b200.dist): the test supplies c.comm
            c.comm(self.buffers[c.buf][c.offset:c.offset + c.count])
        elif kind == "Receiver":
            outs = []
            for k in c.kargs:
                off = offset_of(k)
                n = math.prod(k.shape)
                outs.append(self.buffers[k.id][off:off + n].reshape(k.shape).copy())
            if c.func is not None:
                c.func(*outs)
            self.last_received = outs

    def run_proc(self, proc: ir.Proc) -> None:
        for c in proc.procedure:
            if isinstance(c, ir.ForNode):
                for _ in c.r:
                    self.run_proc(c.proc)
            else:
                self.run_cmd(c)

    def execute(self, proc) -> None:
        self.prepare(proc)
        self.run_proc(self.proc)


def offset_of(k: ir.KMatrix) -> int:
    """``KMatrix.calc_offset`` (autodiff/kernalize/__init__.py:74-83)."""
    a = k.access
    if isinstance(a, ir.Gid):
        return 0
    if isinstance(a, ir.Bin) and a.op == "Add" and isinstance(a.a, ir.Gid) and isinstance(a.b, ir.Const):
        return a.b.val
    if isinstance(a, ir.Const) and math.prod(k.shape) == 1:
        return a.val
    raise ValueError(f"Invalid Feeder/Receiver access: {ir.expr_str(a)}")
