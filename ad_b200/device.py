"""``CudaB200Device``: the reference's device plug-in, backed by sm_100a kernels.

Drop-in for ``autodiff.device.opencl.OpenCLDevice`` (autodiff/device/opencl/
device.py:9-146): same duck-typed methods ``init(cmd)``, ``run(cmd)``,
``_run_proc(proc, func, init)``, ``execute(proc)``, and the same observable
behaviour -- Feeder ``func()`` called once per iteration and its result
asserted to be an ``np.ndarray`` of the declared shape (device.py:98-101),
Receiver callbacks called with freshly allocated numpy arrays in program order
(device.py:102-110), exceptions from callbacks propagate out of ``execute``.

What is different (B200-native):

* one arena allocation planned by ``memplan`` (256-byte aligned, kernel-
  granularity lifetimes) instead of one buffer per AllocEntry;
* every compute command becomes a generated sm_100a kernel (``codegen``,
  ``gemm``) compiled by NVRTC in parallel during ``init``;
* ``ForNode`` bodies are captured once into a CUDA graph and replayed
  (``len(r)`` launches instead of ``len(r) * n_kernels`` Python launches); the
  Feeder's host-to-device copy is a node of that graph reading a pinned
  staging buffer, double-buffered so the host prepares iteration i+1 while
  the GPU runs iteration i;
* optional data parallelism: ``dist`` inserts gradient all-reduces.

There is no CPU fallback: if the CUDA library or a GPU is missing, the
constructor raises.
"""
from __future__ import annotations

import ctypes
import math
import os
import time
from concurrent.futures import ThreadPoolExecutor
from typing import Callable, Dict, List, Optional

import numpy as np

from . import codegen, ir, memplan
from . import runtime as rt

ELEMENTWISE = ("ElwFuse", "BinaryNode", "UnaryNode", "ContigiousNode")
REDUCE = ("ReduceNode", "ReduceElwFuse")
DOT = ("DotProdNode", "DPElwFuse")
COMM_STREAM = 3          # the context's communication stream (include/ad_b200.h)


class Launch:
    """A compiled kernel with its bound arguments (the reference's ``funcs[pid]``
    closure from build_kernel, cl_helper.py:445-455)."""
    __slots__ = ("spec", "kernel", "args", "argv", "holders")

    def __init__(self, spec: codegen.KernelSpec, kernel: rt.Kernel, ptrs: List[int], extra=None):
        self.spec = spec
        self.kernel = kernel
        extra = extra or {}
        holders = list(extra.get("prefix", [])) + [ctypes.c_uint64(p) for p in ptrs] + \
            list(extra.get("suffix", []))
        self.holders = holders
        self.argv = (ctypes.c_void_p * max(1, len(holders)))(
            *[ctypes.addressof(h) for h in holders])


class CudaB200Device:
    """Device plug-in with the reference's interface (device/__init__.py:1-6)."""

    def __init__(self, device: int = 0, use_graphs: bool = True, gemm: str = "auto",
                 verbose: bool = False, comm=None, rowfuse: bool = True, batch: bool = True,
                 dp: Optional[tuple] = None, nccl_timeout_s: float = 120.0, hsplit: bool = True):
        """``dp = (rank, world, uid)``: data-parallel rank of ``world``; ``uid`` is
        the 128-byte NCCL id from ``ad_b200.dist.nccl_unique_id()`` on rank 0,
        shared with every rank by the caller.  The proc is then this rank's shard
        and gradients are summed over ranks (``ad_b200.dist``)."""
        # host copy threads (pageable Feeder/Receiver staging): share the cores
        # among the processes of this node
        lw = int(os.environ.get("LOCAL_WORLD_SIZE", "1"))
        if lw > 1 and "AD_COPY_THREADS" not in os.environ:
            os.environ["AD_COPY_THREADS"] = str(max(1, (os.cpu_count() or 2) // (2 * lw)))
        self.ctx = rt.Context(device)
        self.world = 1
        if dp is not None and dp[1] > 1:
            rank, world, uid = dp
            buf = ctypes.create_string_buffer(bytes(uid), 128)
            rt.check(self.ctx.L.ad_nccl_init(self.ctx.h, rank, world, buf, nccl_timeout_s), "ad_nccl_init")
            self.rank, self.world = rank, world
        self.rowfuse = rowfuse and os.environ.get("AD_ROWFUSE", "1") != "0"
        self.batch = batch and os.environ.get("AD_BATCH", "1") != "0"
        self.hsplit = hsplit and os.environ.get("AD_HSPLIT", "1") != "0"
        self._spec_cache: Dict[int, codegen.KernelSpec] = {}
        self.use_graphs = use_graphs and os.environ.get("AD_GRAPH", "1") != "0"
        self.gemm = os.environ.get("AD_GEMM", gemm)
        self.verbose = verbose
        self.comm = comm
        self.arena = 0
        self.arena_bytes = 0
        self.slots: Dict[int, memplan.Slot] = {}
        self.launches: Dict[int, List[Launch]] = {}   # id(cmd) -> launches
        self.kernels: Dict[str, rt.Kernel] = {}
        self._graphs: Dict[int, list] = {}
        self._staging: Dict[int, list] = {}
        self.n_launches = 0
        self.compile_seconds = 0.0
        self.proc: Optional[ir.Proc] = None
        # diagnostics: per all-reduce (bytes, async, start event, end event) when
        # a list; AD_DP_SKIP_COMM=1 leaves the collectives out (timing only:
        # ranks then diverge)
        self.comm_trace = None
        self.skip_comm = os.environ.get("AD_DP_SKIP_COMM", "0") == "1"
        # gradient sums: NCCL, or the library's peer-memory kernel (AD_DP_COMM=peer)
        self.peer_comm = os.environ.get("AD_DP_COMM", "nccl") == "peer"

    # ------------------------------------------------------------ memory
    def ptr(self, buf_id: int) -> int:
        return self.arena + self.slots[buf_id].offset

    def _setup_memory(self, proc: ir.Proc) -> None:
        self.slots, total = memplan.plan(proc)
        self.scratch_bytes = 0
        self.arena_bytes = total
        self.arena = self.ctx.malloc(max(total, 256))
        for c in ir.iter_cmds(proc):
            if isinstance(c, ir.AllocEntry) and not c.is_temp and c.content is not None:
                a = np.ascontiguousarray(np.asarray(c.content, dtype=np.float32).reshape(-1))
                assert a.size <= c.size
                self.ctx.h2d_pageable(self.ptr(c.id), a.ctypes.data, a.nbytes, 0)
        self.ctx.sync(0)

    def upload(self, buf_id: int, arr: np.ndarray, offset: int = 0) -> None:
        a = np.ascontiguousarray(arr, dtype=np.float32)
        self.ctx.h2d(self.ptr(buf_id) + 4 * offset, a.ctypes.data, a.nbytes, 0)
        self.ctx.sync(0)

    def download(self, buf_id: int, n: Optional[int] = None, offset: int = 0) -> np.ndarray:
        n = self.slots[buf_id].size - offset if n is None else n
        out = np.empty(n, dtype=np.float32)
        self.ctx.sync(0)
        self.ctx.d2h(out.ctypes.data, self.ptr(buf_id) + 4 * offset, out.nbytes, 0)
        self.ctx.sync(0)
        return out

    # ------------------------------------------------------------ init pass
    def _single_spec(self, cmd, sizes) -> Optional[codegen.KernelSpec]:
        """The one pointer-only kernel of ``cmd``, or None when it needs several
        launches or non-pointer arguments (the tensor-core dot path)."""
        key = id(cmd)
        if key in self._spec_cache:
            return self._spec_cache[key]
        kind = type(cmd).__name__
        name = f"k_{kind}"
        spec = None
        if kind in ELEMENTWISE:
            spec = codegen.gen_elementwise(cmd, name, sizes)
        elif kind in REDUCE:
            spec = codegen.gen_reduce(cmd, name, sizes)
        elif kind in DOT:
            from . import gemm
            spec = gemm.single_kernel_spec(self, cmd, name, sizes)
        elif kind == "RowFused":
            from . import rowfuse
            spec = rowfuse.gen_rowfused(cmd, "k_RowFused", sizes, self.ctx.sm_count)
            spec.extra["err_param"] = True
        self._spec_cache[key] = spec
        return spec

    def _specs_for(self, cmd) -> List[codegen.KernelSpec]:
        kind = type(cmd).__name__
        sizes = {b: s.size for b, s in self.slots.items()}
        name = f"k_{kind}"
        if kind == "Batched" and type(cmd.cmds[0]).__name__ in DOT and \
                self._single_spec(cmd.cmds[0], sizes) is None:
            from . import tcgen05
            return tcgen05.plan_group(self, cmd.cmds, name, sizes)
        if kind == "Batched":
            from . import batch
            members = [self._single_spec(c, sizes) for c in cmd.cmds]
            first = members[0]
            src, nparam = batch.batched_source(first.src, first.name + "_x")
            spec = codegen.KernelSpec(first.name + "_x", src, [], (first.grid[0], first.grid[1], len(members)),
                                      first.block, first.smem, first.kind + "_batched",
                                      sum(m.bytes_moved for m in members), sum(m.flops for m in members))
            spec.extra["table"] = [(m.buffers, bool(m.extra.get("err_param"))) for m in members]
            spec.extra["nparam"] = nparam
            return [spec]
        single = self._single_spec(cmd, sizes)
        if single is not None:
            if single.extra.get("err_param"):
                single.extra["suffix"] = [ctypes.c_uint64(self.err_ptr)]
            return [single]
        if kind in DOT:
            from . import gemm
            return gemm.plan_dot(self, cmd, name, sizes)
        raise TypeError(f"Encountered unexpected cmd: {kind}")

    def _upload_table(self, spec) -> int:
        """Device table of pointer parameters of a batched launch (instance-major)."""
        rows = []
        for entry in spec.extra["table"]:
            bufs, err = entry[0], entry[1]
            pre, post = (entry[2], entry[3]) if len(entry) > 2 else ([], [])
            row = list(pre) + [self.view_ptr(v) for v in bufs] + ([self.err_ptr] if err else []) + list(post)
            assert spec.extra["nparam"] is None or len(row) == spec.extra["nparam"]
            rows += row
        a = np.asarray(rows, dtype=np.uint64)
        p = self.ctx.malloc(a.nbytes)
        self.scratch_allocs.append(p)
        self.ctx.h2d(p, a.ctypes.data, a.nbytes, 0)
        self.ctx.sync(0)
        return p

    def init(self, cmd) -> None:
        """Per-command init (opencl/device.py:46-86): kernels are generated here
        and compiled in one parallel batch by ``_compile_pending``."""
        kind = type(cmd).__name__
        if kind in ("Feeder", "Receiver"):
            ks = [cmd.kres] if kind == "Feeder" else cmd.kargs
            for k in ks:
                off = offset_of(k)
                n = math.prod(k.shape)
                if off < 0 or off + n > self.slots[k.id].size:
                    raise ValueError(f"{kind} access out of range for buffer {k.id}")
            return
        if kind == "AllReduce":
            self._comm_slot[id(cmd)] = len(self._comm_slot)
        if kind == "AllReduce" and cmd.async_start:
            # fork/join events of the communication stream (recorded again by
            # every replay; inside a graph capture they become dependencies)
            self._comm_events[id(cmd)] = (self.ctx.event(False), self.ctx.event(False))
            return
        if kind in ("AllocEntry", "DeallocEntry", "ForNode", "AllReduce", "AllReduceWait"):
            return
        self._pending.append((cmd, self._specs_for(cmd)))

    def _compile_pending(self) -> None:
        todo = {}
        for _, specs in self._pending:
            for s in specs:
                if s.src not in self.kernels and s.src not in todo:
                    todo[s.src] = s
        t0 = time.time()
        srcs = list(todo.values())
        with ThreadPoolExecutor(max_workers=min(16, max(1, len(srcs)))) as ex:
            cubins = list(ex.map(lambda s: rt.compile_cubin(s.src,
                                                            s.name + ".cu"), srcs))
        for s, cub in zip(srcs, cubins):
            k = self.ctx.load(cub, s.name)
            if s.smem > 48 * 1024:
                k.set_smem(s.smem)
            self.kernels[s.src] = k
        self.compile_seconds += time.time() - t0
        for cmd, specs in self._pending:
            ls = []
            for s in specs:
                if "table" in s.extra:
                    ls.append(Launch(s, self.kernels[s.src], [self._upload_table(s)],
                                     {"prefix": s.extra.get("prefix", []), "suffix": s.extra.get("suffix", [])}))
                    continue
                ptrs = [self.view_ptr(v) for v in s.buffers]
                ls.append(Launch(s, self.kernels[s.src], ptrs, s.extra))
            self.launches[id(cmd)] = ls
        self._pending = []

    def view_ptr(self, v) -> int:
        """Device address of a kernel pointer parameter: a buffer, or a
        (buffer, element offset) view of one."""
        if isinstance(v, tuple):
            return self.ptr(v[0]) + 4 * v[1]
        return self.ptr(v)

    # ------------------------------------------------------------ run pass
    def _launch(self, L: Launch, stream: int = 0) -> None:
        s = L.spec
        self.ctx.launch(L.kernel, s.grid, s.block, s.smem, L.argv, stream)
        self.n_launches += 1

    def run(self, cmd) -> None:
        """Per-command run (opencl/device.py:88-112)."""
        kind = type(cmd).__name__
        if kind in ("AllocEntry", "DeallocEntry", "ForNode"):
            return
        if kind == "Feeder":
            arr = cmd.func()
            assert isinstance(arr, np.ndarray) and list(arr.shape) == list(cmd.shape), "Invalid function"
            a = np.ascontiguousarray(arr, dtype=np.float32)
            # staged through pinned memory; the array may be freed once this returns
            self.ctx.h2d_pageable(self.ptr(cmd.kres.id) + 4 * offset_of(cmd.kres), a.ctypes.data, a.nbytes, 0)
            return
        if kind == "Receiver":
            outs = []
            for k in cmd.kargs:
                n = math.prod(k.shape)
                o = np.empty(n, dtype=np.float32)
                if 4 * n >= (1 << 20):
                    self.ctx.d2h_pageable(o.ctypes.data, self.ptr(k.id) + 4 * offset_of(k), 4 * n, 0)
                else:
                    self.ctx.d2h(o.ctypes.data, self.ptr(k.id) + 4 * offset_of(k), 4 * n, 0)
                outs.append(o)
            self.ctx.sync(0)
            outs = [o.reshape(k.shape) for o, k in zip(outs, cmd.kargs)]
            self.last_received = outs
            if cmd.func is not None:
                cmd.func(*outs)
            return
        if kind == "AllReduce":
            p = self.ptr(cmd.buf) + 4 * cmd.offset
            stream = COMM_STREAM if cmd.async_start else 0
            if cmd.async_start:
                fork, join = self._comm_events[id(cmd)]
                fork.record(0)
                fork.wait_on(COMM_STREAM)
            trace = self.comm_trace
            if trace is not None:
                t0, t1 = self.ctx.event(True), self.ctx.event(True)
                t0.record(stream)
            if self.skip_comm:
                pass
            elif self.peer_comm:
                rt.check(self.ctx.L.ad_peer_allreduce_f32(self.ctx.h, p, cmd.count, self._comm_slot[id(cmd)],
                                                          stream, self.err_ptr), "ad_peer_allreduce_f32")
            else:
                rt.check(self.ctx.L.ad_allreduce_f32(self.ctx.h, p, p, cmd.count, 0, stream),
                         "ad_allreduce_f32")
            if trace is not None:
                t1.record(stream)
                trace.append((cmd.count * 4, cmd.async_start, t0, t1))
            if cmd.async_start:
                join.record(COMM_STREAM)
            return
        if kind == "AllReduceWait":
            for st in cmd.starts:
                self._comm_events[id(st)][1].wait_on(0)
            return
        for L in self.launches[id(cmd)]:
            self._launch(L)

    def _run_proc(self, proc: ir.Proc, func: Callable, init: bool = False) -> None:
        """opencl/device.py:114-124, with ForNode bodies replayed as CUDA graphs."""
        for cmd in proc.procedure:
            if isinstance(cmd, ir.ForNode):
                if init:
                    self._run_proc(cmd.proc, func, init)
                elif self.use_graphs and graphable(cmd.proc):
                    self._replay_graph(cmd)
                else:
                    for _ in cmd.r:
                        self._run_proc(cmd.proc, func, init)
            else:
                func(cmd)

    # ------------------------------------------------------------ graphs
    def _capture(self, body: ir.Proc, stagings: List[Dict[int, np.ndarray]]):
        """Capture ``len(stagings)`` consecutive replays of ``body`` (no Receivers)
        into one CUDA graph; replay i's Feeder copies read ``stagings[i]``
        (pinned host arrays)."""
        rt.graph_begin(self.ctx, 0)
        try:
            for staging in stagings:
                self._capture_inline(body, staging)
        except Exception:
            try:
                rt.graph_end(self.ctx, 0)
            except Exception:
                pass
            raise
        return rt.graph_end(self.ctx, 0)

    def _capture_inline(self, body, staging):
        for cmd in body.procedure:
            kind = type(cmd).__name__
            if kind == "Feeder":
                a = staging[id(cmd)]
                self.ctx.h2d(self.ptr(cmd.kres.id) + 4 * offset_of(cmd.kres), a.ctypes.data, a.nbytes, 0)
            elif kind == "ForNode":
                for _ in cmd.r:
                    self._capture_inline(cmd.proc, staging)
            elif kind not in ("AllocEntry", "DeallocEntry"):
                self.run(cmd)

    def _pinned(self, nbytes: int) -> np.ndarray:
        p = ctypes.c_void_p()
        rt.check(self.ctx.L.ad_pinned_alloc(nbytes, ctypes.byref(p)), "ad_pinned_alloc")
        self._pinned_ptrs.append(p.value)
        return np.ctypeslib.as_array((ctypes.c_float * (nbytes // 4)).from_address(p.value))

    LOOP_UNROLL = 16
    FIRST_CHUNK = 2

    def _loop_graphs(self, loop: ir.ForNode, feeders, u: int):
        """Two graphs (ping-pong) of ``u`` iterations each, with their own pinned
        Feeder staging, so the host fills one while the GPU runs the other."""
        key = (id(loop), u)
        if key not in self._graphs:
            pairs = []
            for _ in range(2 if feeders else 1):
                stagings = [{id(f): self._pinned(4 * math.prod(f.shape)) for f in feeders} for _ in range(u)]
                g = self._capture(loop.proc, stagings)
                pairs.append((g, stagings, self.ctx.event(False), [False]))
            self._graphs[key] = pairs
        return self._graphs[key]

    def _replay_graph(self, loop: ir.ForNode) -> None:
        """Run ``len(loop.r)`` iterations as launches of graphs that each hold
        LOOP_UNROLL iterations.  Feeder functions are still called once per
        iteration, in order, before the graph that consumes their data."""
        feeders = [c for c in ir.iter_cmds(loop.proc) if type(c).__name__ == "Feeder"]
        n = len(loop.r)
        u = max(1, min(n, self.LOOP_UNROLL))
        # a short first chunk: its Feeder data is staged on the host before the
        # GPU has anything to run, later chunks are staged while the previous one runs
        first = min(n, self.FIRST_CHUNK) if feeders and n > u else 0
        rest = n - first
        chunks = ([first] if first else []) + [u] * (rest // u) + ([rest % u] if rest % u else [])
        n_kern = sum(len(self.launches.get(id(c), [])) for c in ir.iter_cmds(loop.proc))
        for ci, cu in enumerate(chunks):
            pairs = self._loop_graphs(loop, feeders, cu)
            g, stagings, done, used = pairs[ci % len(pairs)]
            if feeders:
                if used[0]:
                    done.sync()  # the copies that read these staging slots have finished
                for i in range(cu):
                    for f in feeders:
                        arr = f.func()
                        assert isinstance(arr, np.ndarray) and list(arr.shape) == list(f.shape), "Invalid function"
                        a = np.ascontiguousarray(arr, dtype=np.float32)
                        st = stagings[i][id(f)]
                        rt.host_copy(st.ctypes.data, a.ctypes.data, min(a.nbytes, st.nbytes))
            g.launch(0)
            self.n_launches += n_kern * cu
            if feeders:
                done.record(0)
                used[0] = True

    # ------------------------------------------------------------ entry point
    def prepare(self, proc) -> ir.Proc:
        """Init pass: plan + allocate memory, upload contents, build all kernels."""
        proc = self.transform(proc)
        self.proc = proc
        self._pinned_ptrs: List[int] = []
        self._setup_memory(proc)
        self.err_ptr = self.ctx.malloc(256)
        self.ctx.memset(self.err_ptr, 0, 256, 0)
        self.scratch_allocs = [self.err_ptr]
        from . import gemm
        gemm.setup_scratch(self, proc)
        self._pending = []
        self._comm_events = {}
        self._comm_slot = {}
        if self.world > 1 and self.peer_comm:
            rt.check(self.ctx.L.ad_peer_init(self.ctx.h, self.arena, self.arena_bytes), "ad_peer_init")
        self._run_proc(proc, self.init, init=True)
        self._compile_pending()
        return proc

    @classmethod
    def offline(cls, gemm: str = "auto", rowfuse: bool = True, batch: bool = True,
                hsplit: bool = True, sm_count: int = 148, world: int = 1) -> "CudaB200Device":
        """A device object without a GPU context, for the command-level passes
        only (``transform``; inspection and CPU tests)."""
        import types
        self = cls.__new__(cls)
        self.ctx = types.SimpleNamespace(sm_count=sm_count)
        self.gemm, self.rowfuse, self.batch, self.hsplit, self.world = gemm, rowfuse, batch, hsplit, world
        self._spec_cache = {}
        return self

    @classmethod
    def passes_only(cls, proc, **kw) -> ir.Proc:
        """``transform`` on a copy of ``proc`` without a GPU (see ``offline``)."""
        return cls.offline(**kw).transform(proc)

    def batch_signature(self, c, sizes: Dict[int, int]) -> Optional[str]:
        """Commands with equal signatures run as one launch when independent:
        the generated kernel source (tensor-core dots: split + GEMM sources)."""
        if type(c).__name__ not in ir.COMPUTE_KINDS:
            return None
        cache = self.__dict__.setdefault("_sig_cache", {})
        if id(c) in cache:
            return cache[id(c)]
        cache[id(c)] = sig = self._batch_signature(c, sizes)
        return sig

    def _batch_signature(self, c, sizes: Dict[int, int]) -> Optional[str]:
        sp = self._single_spec(c, sizes)
        if sp is None and type(c).__name__ in DOT:
            from . import gemm
            return gemm.tc_signature(self, c)
        return None if sp is None else sp.src

    def transform(self, proc) -> ir.Proc:
        """Command-level passes: a private copy of the proc, then the gradient
        all-reduce rewrite (data parallel), sums of dot products folded into
        one dot over the concatenated K axis, splitting of horizontally fused
        elementwise groups, row fusion, and batching."""
        proc = ir.copy_structure(ir.conv_proc(proc))
        if self.world > 1 or os.environ.get("AD_DP_FORCE_REWRITE") == "1":
            # (forced on one GPU with AD_DP_SKIP_COMM=1: profiles the rewrite's own cost)
            from . import dist
            dist.insert_grad_allreduce(proc)
        if os.environ.get("AD_KCAT", "1") != "0":
            from . import kcat
            kcat.fuse_ksums(proc)
        if self.hsplit:
            from . import hsplit
            hsplit.split_groups(proc)
        if self.rowfuse:
            from . import rowfuse
            rowfuse.fuse_rows(proc)
        if self.batch:
            from . import batch
            sizes: Dict[int, int] = {}
            for c in ir.iter_cmds(proc):
                if isinstance(c, ir.AllocEntry) and not c.is_temp:
                    sizes[c.id] = max(sizes.get(c.id, 0), c.size)

            batch.batch_proc(proc, lambda c: self.batch_signature(c, sizes))
        return proc

    def execute(self, proc) -> None:
        """opencl/device.py:126-130: init pass, run pass, wait for the queue."""
        proc = self.prepare(proc)
        self._run_proc(proc, self.run, init=False)
        self.ctx.sync()
        self.check_errors()

    def check_errors(self) -> None:
        """Raise if a kernel recorded a device-side error (a bounded wait that
        expired: 1 = TMA ring stalled, 2 = operand tile never arrived,
        3 = accumulator never completed)."""
        flag = np.zeros(1, dtype=np.int32)
        self.ctx.sync()
        self.ctx.d2h(flag.ctypes.data, self.err_ptr, 4, 0)
        self.ctx.sync(0)
        if flag[0] != 0:
            raise rt.ADError(f"device kernel reported error code {int(flag[0])} (bounded wait expired)")

    def capture(self, cmds: Optional[List] = None) -> rt.Graph:
        """One CUDA graph that launches every kernel of ``cmds`` (default: the
        compute commands of the prepared main proc) in program order."""
        rt.graph_begin(self.ctx, 0)
        try:
            self.replay(cmds)
        except Exception:
            rt.graph_end(self.ctx, 0)
            raise
        return rt.graph_end(self.ctx, 0)

    def capture_launches(self, launches: List["Launch"], repeat: int = 1) -> rt.Graph:
        rt.graph_begin(self.ctx, 0)
        try:
            for _ in range(repeat):
                for L in launches:
                    self._launch(L)
        except Exception:
            rt.graph_end(self.ctx, 0)
            raise
        return rt.graph_end(self.ctx, 0)

    def replay(self, cmds: Optional[List] = None) -> None:
        """Re-launch the compute commands of the prepared proc (no host I/O)."""
        for c in (cmds if cmds is not None else self.proc.procedure):
            if id(c) in self.launches:
                self.run(c)

    def close(self) -> None:
        if getattr(self, "ctx", None) is None:
            return
        self._graphs = {}
        try:
            self.ctx.sync()
        except Exception:
            pass
        for p in getattr(self, "_pinned_ptrs", []):
            self.ctx.L.ad_pinned_free(ctypes.c_void_p(p))
        self._pinned_ptrs = []
        for k in self.kernels.values():
            self.ctx.L.ad_kernel_free(k.h)
        self.kernels = {}
        if self.arena:
            self.ctx.free(self.arena)
            self.arena = 0
        for p in getattr(self, "scratch_allocs", []):
            self.ctx.free(p)
        self.scratch_allocs = []
        self.ctx.close()
        self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def graphable(p: ir.Proc) -> bool:
    """A loop body can be replayed as a graph if it has no Receiver (host callback)
    and no nested loop that feeds host data."""
    if any(type(c).__name__ == "Receiver" for c in ir.iter_cmds(p)):
        return False
    for c in p.procedure:
        if isinstance(c, ir.ForNode) and any(type(x).__name__ == "Feeder" for x in ir.iter_cmds(c.proc)):
            return False
    return True


def offset_of(k) -> int:
    """``KMatrix.calc_offset`` (autodiff/kernalize/__init__.py:74-83)."""
    a = k.access
    if isinstance(a, ir.Gid):
        return 0
    if isinstance(a, ir.Bin) and a.op == "Add" and isinstance(a.a, ir.Gid) and isinstance(a.b, ir.Const):
        return a.b.val
    if isinstance(a, ir.Const) and math.prod(k.shape) == 1:
        return a.val
    raise Exception(f"Invalid Feeder setting: {ir.expr_str(a)}. Make sure to call .contigious before Global() ")
