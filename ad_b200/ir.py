"""Procedural IR consumed by the CUDA device: a plain mirror of the reference's.

The reference compiler (Eshaancoding/ad) hands its device a ``Proc``: a linear
list of commands produced by ``kernalize`` + ``linearize`` + ``alloc``
(autodiff/__init__.py:34-85).  This module restates that structure as small
Python classes with the *same class names and attribute names*, so that

* the device can consume the reference's live objects unchanged (it only
  duck-types on class name and attributes, like ``OpenCLDevice.init`` does at
  autodiff/device/opencl/device.py:46-86), and
* a proc can be serialised to JSON and re-loaded on a machine where the
  reference front-end is absent (fixtures for tests and benchmarks).

Mirrored reference types (file:line in the reference project):

* index expressions ``Constant/Global/X/Y/Val/Add/Minus/Mult/Div/Remainder/
  ShiftRight/ShiftLeft/BitwiseAnd/MoreThan/LessThan``  autodiff/expr/__init__.py:16-155
* kernel args ``KMatrix/KConcat/KConstant``           autodiff/kernalize/__init__.py:42-128
* ``AllocEntry/DeallocEntry``                         autodiff/alloc/__init__.py:34-57
* compute nodes ``BinaryNode/UnaryNode/ReduceNode/DotProdNode/ContigiousNode``
  autodiff/graph/compute/*.py, autodiff/graph/data/contigious.py
* ``Feeder``/``Receiver``                             autodiff/graph/data/feeder.py, receiver.py
* ``ForNode``                                         autodiff/graph/control/ir_for.py:6-18
* fused groups ``ElwFuse/ReduceElwFuse/DPElwFuse``    autodiff/fusion/ops.py:14-50
* ``Proc``                                            autodiff/context.py:7-47

Expressions are normalised on conversion: ``Val(v)`` wrappers are dropped, so a
leaf is one of ``Const(c)``, ``Gid()``, ``Xv()``, ``Yv()`` and an inner node is
``Bin(op, a, b)`` with ``op`` one of ``BIN_OPS``.
"""
from __future__ import annotations

import base64
import gzip
import json
import zlib
from dataclasses import dataclass, field
from typing import Any, Callable, Dict, List, Optional, Union

import numpy as np

# --------------------------------------------------------------------------
# Integer index expressions (autodiff/expr/__init__.py:16-155)
# --------------------------------------------------------------------------

BIN_OPS = ("Add", "Minus", "Mult", "Div", "Remainder", "ShiftRight",
           "ShiftLeft", "BitwiseAnd", "MoreThan", "LessThan")


class Expr:
    __slots__ = ()


@dataclass(frozen=True)
class Const(Expr):
    val: int


@dataclass(frozen=True)
class Gid(Expr):
    """``Global``: the flat element index of an elementwise launch."""


@dataclass(frozen=True)
class Xv(Expr):
    """``X``: row index (reduce row / dot-product output row)."""


@dataclass(frozen=True)
class Yv(Expr):
    """``Y``: column index (reduce position / dot-product output column)."""


@dataclass(frozen=True)
class Bin(Expr):
    op: str
    a: Expr
    b: Expr


def expr_eval(e: Expr, g: int = 0, x: int = 0, y: int = 0) -> int:
    """Evaluate with C semantics on non-negative ints (integer / and %)."""
    if isinstance(e, Const):
        return int(e.val)
    if isinstance(e, Gid):
        return g
    if isinstance(e, Xv):
        return x
    if isinstance(e, Yv):
        return y
    a = expr_eval(e.a, g, x, y)
    b = expr_eval(e.b, g, x, y)
    op = e.op
    if op == "Add":
        return a + b
    if op == "Minus":
        return a - b
    if op == "Mult":
        return a * b
    if op in ("Div", "Remainder"):
        q = abs(a) // abs(b)
        q = q if (a >= 0) == (b >= 0) else -q
        return q if op == "Div" else a - b * q
    if op == "ShiftRight":
        return a >> b
    if op == "ShiftLeft":
        return a << b
    if op == "BitwiseAnd":
        return a & b
    if op == "MoreThan":
        return int(a > b)
    if op == "LessThan":
        return int(a < b)
    raise ValueError(op)


def expr_vars(e: Expr) -> set:
    if isinstance(e, Gid):
        return {"G"}
    if isinstance(e, Xv):
        return {"X"}
    if isinstance(e, Yv):
        return {"Y"}
    if isinstance(e, Bin):
        return expr_vars(e.a) | expr_vars(e.b)
    return set()


def expr_str(e: Expr) -> str:
    if isinstance(e, Const):
        return str(e.val)
    if isinstance(e, Gid):
        return "G"
    if isinstance(e, Xv):
        return "X"
    if isinstance(e, Yv):
        return "Y"
    sym = {"Add": "+", "Minus": "-", "Mult": "*", "Div": "/", "Remainder": "%",
           "ShiftRight": ">>", "ShiftLeft": "<<", "BitwiseAnd": "&",
           "MoreThan": ">", "LessThan": "<"}[e.op]
    return f"({expr_str(e.a)} {sym} {expr_str(e.b)})"


# --------------------------------------------------------------------------
# Kernel arguments (autodiff/kernalize/__init__.py:42-128)
# --------------------------------------------------------------------------

class KernelArg:
    __slots__ = ()


@dataclass
class KMatrix(KernelArg):
    id: int
    access: Optional[Expr]
    shape: List[int]
    is_temp: bool = False

    def ids(self, filter_temp: bool = True) -> List[int]:
        return [] if (filter_temp and self.is_temp) else [self.id]


@dataclass
class KConcat(KernelArg):
    """``condition ? karg_two : karg_one`` (autodiff/device/opencl/karg.py:52)."""
    karg_one: KernelArg
    karg_two: KernelArg
    condition: Expr
    shape: List[int]

    def ids(self, filter_temp: bool = True) -> List[int]:
        out = self.karg_one.ids(filter_temp) + self.karg_two.ids(filter_temp)
        return list(dict.fromkeys(out))


@dataclass
class KConstant(KernelArg):
    constant: float

    def ids(self, filter_temp: bool = True) -> List[int]:
        return []


def karg_ids(k: KernelArg, filter_temp: bool = True) -> List[int]:
    return k.ids(filter_temp)


# --------------------------------------------------------------------------
# Commands
# --------------------------------------------------------------------------

@dataclass
class AllocEntry:
    id: int
    size: int
    content: Optional[np.ndarray] = None
    is_temp: bool = False
    alias: Optional[tuple] = None     # (base id, element offset): a view into another buffer


@dataclass
class DeallocEntry:
    id: int
    size: int
    is_temp: bool = False


@dataclass
class Feeder:
    id: int
    shape: List[int]
    kres: KMatrix
    name: str = ""
    func: Optional[Callable[[], np.ndarray]] = None


@dataclass
class Receiver:
    id: int
    kargs: List[KMatrix]
    name: str = ""
    func: Optional[Callable[..., Any]] = None


@dataclass
class BinaryNode:
    id: int
    op: str                 # "ADD" | "MULT"
    kargs: List[KernelArg]
    kres: KMatrix
    shape: List[int]
    in_place: bool = False
    program_id: int = -1


UNARY_OPS = ("EXP2", "LOG2", "SIN", "RECIP", "SQRT", "EQUAL", "MORE_ZERO",
             "LESS_ZERO", "MORE_OR_EQ_ZERO", "LESS_OR_EQ_ZERO")


@dataclass
class UnaryNode:
    id: int
    op: str
    kargs: List[KernelArg]
    kres: KMatrix
    shape: List[int]
    program_id: int = -1


@dataclass
class ContigiousNode:
    id: int
    kargs: List[KernelArg]
    kres: KMatrix
    shape: List[int]
    program_id: int = -1


@dataclass
class ReduceNode:
    id: int
    op: str                 # "SUM" | "MAX"
    kargs: List[KernelArg]
    kres: KMatrix
    shape: List[int]
    children_shapes: List[List[int]]
    program_id: int = -1


@dataclass
class DotProdNode:
    id: int
    kargs: List[KernelArg]
    kres: KMatrix
    shape: List[int]
    children_shapes: List[List[int]]
    program_id: int = -1


@dataclass
class FuseGroup:
    """Common shape of ``ElwFuse``/``ReduceElwFuse``/``DPElwFuse``
    (autodiff/fusion/base.py:13-77): ``nodes`` in program order, with
    temp Alloc/Dealloc entries interleaved; ``init_node`` is ``nodes[init]``."""
    nodes: List[Any]
    init: int = 0
    program_id: int = -1
    fuse_id: int = -1

    @property
    def init_node(self):
        return self.nodes[self.init]


class ElwFuse(FuseGroup):
    pass


class ReduceElwFuse(FuseGroup):
    pass


class DPElwFuse(FuseGroup):
    pass


@dataclass
class Proc:
    procedure: List[Any]
    id: int = 0


@dataclass
class ForNode:
    id: int
    proc: Proc
    r: range


COMPUTE_KINDS = ("BinaryNode", "UnaryNode", "ContigiousNode", "ReduceNode",
                 "DotProdNode", "ElwFuse", "ReduceElwFuse", "DPElwFuse", "RowFused", "Batched")

# --------------------------------------------------------------------------
# Conversion from the reference's live objects (duck-typed by class name)
# --------------------------------------------------------------------------


def _cls(o) -> str:
    return type(o).__name__


def conv_expr(e) -> Expr:
    """Reference ``Expression``/``Value`` -> normalised ``Expr``."""
    n = _cls(e)
    if n == "Val":
        return conv_expr(e.v)
    if n == "Constant":
        return Const(int(e.val))
    if n == "Global":
        return Gid()
    if n == "X":
        return Xv()
    if n == "Y":
        return Yv()
    if n in BIN_OPS:
        return Bin(n, conv_expr(e.a), conv_expr(e.b))
    if n in ("Const", "Gid", "Xv", "Yv", "Bin"):
        return e
    raise TypeError(f"unsupported expression node {n}")


def conv_karg(k) -> KernelArg:
    n = _cls(k)
    if n == "KMatrix":
        acc = None if k.is_temp else conv_expr(k.access)
        return KMatrix(int(k.id), acc, [int(s) for s in k.shape], bool(k.is_temp))
    if n == "KConcat":
        return KConcat(conv_karg(k.karg_one), conv_karg(k.karg_two),
                       conv_expr(k.condition), [int(s) for s in k.shape])
    if n == "KConstant":
        return KConstant(float(k.constant))
    raise TypeError(f"unsupported kernel arg {n}")


def _opname(op) -> str:
    return op if isinstance(op, str) else op.name


def conv_cmd(c):
    n = _cls(c)
    pid = int(getattr(c, "program_id", -1) if getattr(c, "program_id", None) is not None else -1)
    if n == "AllocEntry":
        content = None if c.content is None else np.ascontiguousarray(
            np.asarray(c.content, dtype=np.float32).reshape(-1))
        return AllocEntry(int(c.id), int(c.size), content, bool(c.is_temp))
    if n == "DeallocEntry":
        return DeallocEntry(int(c.id), int(c.size), bool(c.is_temp))
    if n == "Feeder":
        return Feeder(int(c.id), [int(s) for s in c.shape], conv_karg(c.kres),
                      str(getattr(c, "name", "")), getattr(c, "func", None))
    if n == "Receiver":
        return Receiver(int(c.id), [conv_karg(k) for k in c.kargs],
                        str(getattr(c, "name", "")), getattr(c, "func", None))
    if n == "ForNode":
        return ForNode(int(c.id), conv_proc(c.proc), range(c.r.start, c.r.stop, c.r.step))
    if n == "BinaryNode":
        return BinaryNode(int(c.id), _opname(c.op), [conv_karg(k) for k in c.kargs],
                          conv_karg(c.kres), list(c.shape), bool(c.in_place), pid)
    if n == "UnaryNode":
        return UnaryNode(int(c.id), _opname(c.op), [conv_karg(k) for k in c.kargs],
                         conv_karg(c.kres), list(c.shape), pid)
    if n == "ContigiousNode":
        return ContigiousNode(int(c.id), [conv_karg(k) for k in c.kargs],
                              conv_karg(c.kres), list(c.shape), pid)
    if n == "ReduceNode":
        return ReduceNode(int(c.id), _opname(c.op), [conv_karg(k) for k in c.kargs],
                          conv_karg(c.kres), list(c.shape),
                          [list(s) for s in c.children_shapes], pid)
    if n == "DotProdNode":
        return DotProdNode(int(c.id), [conv_karg(k) for k in c.kargs], conv_karg(c.kres),
                           list(c.shape), [list(s) for s in c.children_shapes], pid)
    if n in ("ElwFuse", "ReduceElwFuse", "DPElwFuse"):
        if isinstance(c, FuseGroup):
            return c
        nodes = [conv_cmd(x) for x in c.nodes]
        init = 0
        for i, x in enumerate(c.nodes):
            if x is c.init_node:
                init = i
                break
        cls = {"ElwFuse": ElwFuse, "ReduceElwFuse": ReduceElwFuse, "DPElwFuse": DPElwFuse}[n]
        return cls(nodes, init, pid, int(getattr(c, "fuse_id", -1)))
    raise TypeError(f"unsupported proc entry {n}")


def copy_structure(p: Proc) -> Proc:
    """A new Proc (and new ForNode/Proc containers) sharing the commands, so that
    device-side rewrites of the command list never touch the caller's proc."""
    out = []
    for c in p.procedure:
        if isinstance(c, ForNode):
            out.append(ForNode(c.id, copy_structure(c.proc), c.r))
        else:
            out.append(c)
    return Proc(out, p.id)


def conv_proc(p) -> Proc:
    """Convert a reference ``Proc`` (or one of ours) to this module's IR."""
    if isinstance(p, Proc):
        return p
    return Proc([conv_cmd(c) for c in p.procedure], int(getattr(p, "id", 0)))


# --------------------------------------------------------------------------
# JSON (de)serialisation
# --------------------------------------------------------------------------


def _ej(e: Optional[Expr]):
    if e is None:
        return None
    if isinstance(e, Const):
        return e.val
    if isinstance(e, Gid):
        return "G"
    if isinstance(e, Xv):
        return "X"
    if isinstance(e, Yv):
        return "Y"
    return [e.op, _ej(e.a), _ej(e.b)]


def _dj(j) -> Optional[Expr]:
    if j is None:
        return None
    if isinstance(j, int):
        return Const(j)
    if j == "G":
        return Gid()
    if j == "X":
        return Xv()
    if j == "Y":
        return Yv()
    return Bin(j[0], _dj(j[1]), _dj(j[2]))


def _kj(k: KernelArg):
    if isinstance(k, KMatrix):
        return {"M": k.id, "a": _ej(k.access), "s": k.shape, "t": int(k.is_temp)}
    if isinstance(k, KConcat):
        return {"C": [_kj(k.karg_one), _kj(k.karg_two)], "c": _ej(k.condition), "s": k.shape}
    return {"K": k.constant}


def _dk(j) -> KernelArg:
    if "M" in j:
        return KMatrix(j["M"], _dj(j["a"]), j["s"], bool(j["t"]))
    if "C" in j:
        return KConcat(_dk(j["C"][0]), _dk(j["C"][1]), _dj(j["c"]), j["s"])
    return KConstant(j["K"])


def _arr_j(a: np.ndarray):
    raw = zlib.compress(np.ascontiguousarray(a, dtype=np.float32).tobytes(), 6)
    return {"n": int(a.size), "z": base64.b64encode(raw).decode()}


def _arr_d(j) -> np.ndarray:
    return np.frombuffer(zlib.decompress(base64.b64decode(j["z"])), dtype=np.float32).copy()


def cmd_to_json(c) -> dict:
    n = _cls(c)
    if n == "AllocEntry":
        return {"k": n, "id": c.id, "size": c.size, "t": int(c.is_temp),
                "content": None if c.content is None else _arr_j(c.content)}
    if n == "DeallocEntry":
        return {"k": n, "id": c.id, "size": c.size, "t": int(c.is_temp)}
    if n == "Feeder":
        return {"k": n, "id": c.id, "shape": c.shape, "kres": _kj(c.kres), "name": c.name}
    if n == "Receiver":
        return {"k": n, "id": c.id, "kargs": [_kj(k) for k in c.kargs], "name": c.name}
    if n == "ForNode":
        return {"k": n, "id": c.id, "r": [c.r.start, c.r.stop, c.r.step],
                "proc": proc_to_json(c.proc)}
    if n in ("ElwFuse", "ReduceElwFuse", "DPElwFuse"):
        return {"k": n, "pid": c.program_id, "fid": c.fuse_id, "init": c.init,
                "nodes": [cmd_to_json(x) for x in c.nodes]}
    d = {"k": n, "id": c.id, "pid": c.program_id, "kargs": [_kj(k) for k in c.kargs],
         "kres": _kj(c.kres), "shape": c.shape}
    if n in ("BinaryNode", "UnaryNode", "ReduceNode"):
        d["op"] = c.op
    if n == "BinaryNode":
        d["in_place"] = int(c.in_place)
    if n in ("ReduceNode", "DotProdNode"):
        d["cs"] = c.children_shapes
    return d


def cmd_from_json(j):
    k = j["k"]
    if k == "AllocEntry":
        return AllocEntry(j["id"], j["size"], None if j["content"] is None else _arr_d(j["content"]),
                          bool(j["t"]))
    if k == "DeallocEntry":
        return DeallocEntry(j["id"], j["size"], bool(j["t"]))
    if k == "Feeder":
        return Feeder(j["id"], j["shape"], _dk(j["kres"]), j.get("name", ""))
    if k == "Receiver":
        return Receiver(j["id"], [_dk(x) for x in j["kargs"]], j.get("name", ""))
    if k == "ForNode":
        return ForNode(j["id"], proc_from_json(j["proc"]), range(*j["r"]))
    if k in ("ElwFuse", "ReduceElwFuse", "DPElwFuse"):
        cls = {"ElwFuse": ElwFuse, "ReduceElwFuse": ReduceElwFuse, "DPElwFuse": DPElwFuse}[k]
        return cls([cmd_from_json(x) for x in j["nodes"]], j["init"], j["pid"], j["fid"])
    kargs = [_dk(x) for x in j["kargs"]]
    kres = _dk(j["kres"])
    if k == "BinaryNode":
        return BinaryNode(j["id"], j["op"], kargs, kres, j["shape"], bool(j["in_place"]), j["pid"])
    if k == "UnaryNode":
        return UnaryNode(j["id"], j["op"], kargs, kres, j["shape"], j["pid"])
    if k == "ContigiousNode":
        return ContigiousNode(j["id"], kargs, kres, j["shape"], j["pid"])
    if k == "ReduceNode":
        return ReduceNode(j["id"], j["op"], kargs, kres, j["shape"], j["cs"], j["pid"])
    if k == "DotProdNode":
        return DotProdNode(j["id"], kargs, kres, j["shape"], j["cs"], j["pid"])
    raise ValueError(k)


def proc_to_json(p: Proc) -> dict:
    return {"id": p.id, "procedure": [cmd_to_json(c) for c in p.procedure]}


def proc_from_json(j: dict) -> Proc:
    return Proc([cmd_from_json(c) for c in j["procedure"]], j.get("id", 0))


def save_proc(p: Proc, path: str, meta: Optional[dict] = None) -> None:
    doc = {"format": "ad_b200.proc/1", "meta": meta or {}, "proc": proc_to_json(conv_proc(p))}
    data = json.dumps(doc, separators=(",", ":")).encode()
    with (gzip.open(path, "wb") if path.endswith(".gz") else open(path, "wb")) as f:
        f.write(data)


def load_proc(path: str):
    """Returns ``(proc, meta)``."""
    with (gzip.open(path, "rb") if path.endswith(".gz") else open(path, "rb")) as f:
        doc = json.loads(f.read())
    assert doc.get("format") == "ad_b200.proc/1", "not an ad_b200 proc file"
    return proc_from_json(doc["proc"]), doc.get("meta", {})


# --------------------------------------------------------------------------
# Walk helpers
# --------------------------------------------------------------------------


def iter_cmds(proc: Proc, into_loops: bool = True):
    for c in proc.procedure:
        yield c
        if into_loops and isinstance(c, ForNode):
            yield from iter_cmds(c.proc, True)


def bind_io(proc: Proc, feeders: Optional[Dict[str, Callable]] = None,
            receivers: Optional[Dict[str, Callable]] = None) -> Proc:
    """Attach host callables to Feeders/Receivers by ``name`` (loaded procs carry none)."""
    for c in iter_cmds(proc):
        if isinstance(c, Feeder) and feeders and c.name in feeders:
            c.func = feeders[c.name]
        if isinstance(c, Receiver) and receivers and c.name in receivers:
            c.func = receivers[c.name]
    return proc
