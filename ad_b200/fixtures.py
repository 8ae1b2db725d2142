"""Load committed proc fixtures and regenerate their seeded parameter contents.

A fixture is a proc produced by the reference front-end (see
``tests/golden/gen_fixtures.py``) plus ``meta``.  Large ``AllocEntry`` contents
are stored as generator specs (``meta["content_specs"]``, keyed by alloc id) so
that fixtures stay small; ``make_array`` turns a spec back into the exact same
float32 array on any machine (numpy ``default_rng`` streams are portable).
"""
import os
from typing import Dict, Optional

import numpy as np

from . import ir

PROC_DIR = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                        "tests", "golden", "procs")


def make_array(spec: Dict) -> np.ndarray:
    """``spec["part_rows"]`` (optional) selects rows ``[part*part_rows, (part+1)*part_rows)``
    of the full array: one data-parallel rank's share of a global batch."""
    a = _make_full(spec)
    if "part_rows" in spec:
        r = spec["part_rows"]
        k = spec.get("part", 0)
        a = np.ascontiguousarray(a[k * r:(k + 1) * r])
    return a


def _make_full(spec: Dict) -> np.ndarray:
    rng = np.random.default_rng(spec["seed"])
    shape = tuple(spec["shape"])
    if spec["dist"] == "normal":
        return rng.standard_normal(shape, dtype=np.float32)
    if spec["dist"] == "uniform":
        return rng.uniform(spec["lo"], spec["hi"], size=shape).astype(np.float32)
    if spec["dist"] == "fill":
        return np.full(shape, spec["value"], dtype=np.float32)
    raise ValueError(spec["dist"])


def load_case(case: str, path: Optional[str] = None, with_content: bool = True, rank: int = 0,
              feeder_seed_offset: int = 0):
    """Returns ``(proc, meta)`` with every AllocEntry content materialised.  For a
    data-parallel fixture (``meta["dp_parts"] > 1``) ``rank`` picks that rank's rows
    of the per-example data (inputs and the fixed loss weights).
    ``feeder_seed_offset`` shifts the seeds of the Feeders' data only (weights
    unchanged): each rank of a weak-scaling data-parallel run feeds its own batch."""
    proc, meta = ir.load_proc(path or os.path.join(PROC_DIR, f"{case}.json.gz"))

    def with_rank(sp):
        return dict(sp, part=rank) if "part_rows" in sp else sp

    if with_content:
        specs = meta.get("content_specs", {})
        for c in ir.iter_cmds(proc):
            if isinstance(c, ir.AllocEntry) and str(c.id) in specs:
                c.content = make_array(with_rank(specs[str(c.id)])).reshape(-1)
    for c in ir.iter_cmds(proc):
        if isinstance(c, ir.Feeder):
            f = meta.get("feeders", {}).get(c.name)
            if f is not None and "fill" in f:
                val, shape = f["fill"], tuple(f["shape"])
                c.func = lambda val=val, shape=shape: np.full(shape, val, dtype=np.float32)
            elif f is not None and "spec" in f:
                sp = with_rank(f["spec"])
                if feeder_seed_offset and "seed" in sp:
                    sp = dict(sp, seed=sp["seed"] + feeder_seed_offset)
                arr = make_array(sp)
                c.func = lambda arr=arr: arr
    return proc, meta


def set_loop_count(proc: ir.Proc, n: int) -> ir.Proc:
    """Replace the range of every top-level ForNode by ``range(n)``."""
    for c in proc.procedure:
        if isinstance(c, ir.ForNode):
            c.r = range(0, n)
    return proc
