"""Benchmark of the B200 device backend on BASELINE.json's configurations.

Default: the transformer-encoder training step of config 4 (4 layers, d512,
8 heads, ff2048, S128, batch 32, fp32, SGD), run as the proc the reference
front-end produces for it (tests/golden/procs/enc_4_32_128_512_8_2048_100).
One step = one iteration of the proc's training loop (Feeder copy of the
batch, forward, backward, SGD update), replayed as CUDA graphs.

* N=1: config 4 itself.
* N>1 (torchrun, one rank per GPU): data parallel, weak scaling -- every rank
  runs the batch-32 step on its own inputs and the NCCL all-reduce of the
  gradients before each SGD update (``ad_b200.dist``) makes it one global step
  of 32*N sequences.  ``value`` is sequences/s of the whole job, device-timed
  (CUDA events), max over ranks.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME]
    python bench.py --impl reference ...   # the reference's kernels on the host CPU

Other workloads: ``lnsm`` (config 2, LayerNorm+softmax fwd+bwd, fused-kernel
HBM GB/s), ``dotsig`` (config 3, TFLOP/s), ``mlp`` (config 1), ``enc12``
(config 5's per-GPU shard: 12 layers, d1024, 16 heads, ff4096, S512, batch 32
per GPU; at 8 GPUs it is config 5's global batch of 256), ``enc3_d1024``,
``enc`` (strong scaling of config 4's global batch of 32), ``enc_small``.

``e2e`` is the same metric through the device's public run pass with host
data: the Feeder's ``func()`` returns a pageable numpy array each step, the
device stages and copies it, and the Receiver hands freshly allocated numpy
arrays to its callback (host wall clock around the whole call, after a device
synchronize on both sides).
"""
import argparse
import json
import math
import os
import re
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOADS = {
    "lnsm": {"case": "lnsm_8192_4096", "data": "synthetic: x ~ N(0,1) seed 0, dy ~ N(0,1) seed 1 (numpy default_rng)", "metric": "fused-kernel HBM GB/s (LayerNorm+softmax fwd+bwd, fp32 [8192,4096])",
             "unit": "GB/s", "min_bytes": 4 * 8192 * 4096 * 4,
             "profile": ("rowfused", "rowfused_lnsm_8192x4096.md")},
    "mlp": {"case": "mlp", "metric": "Linear MLP train steps/s (examples/linear.py: 255-255-255, batch 2, SGD)",
            "unit": "steps/s", "loop": True, "cpu_iters": 300,
            "data": "Feeder of np.full((2,255), 0.2); weights from np.random.seed(0) randn (reference init)"},
    "enc": {"case": "enc_4_32_128_512_8_2048_100",
            "metric": "encoder train steps/s (4 layers, d512, 8 heads, ff2048, S128, B32, fp32, SGD)",
            "unit": "steps/s", "loop": True, "cpu_iters": 1, "dp": True, "global_batch": 32,
            "data": "synthetic: x ~ N(0,1) [4096, 512] seed 0 via Feeder; Xavier-uniform weights (seeded)"},
    "enc_weak": {"case": "enc_4_32_128_512_8_2048_100",
                 "profile": ("gemm_tcgen05", "gemm_tcgen05_enc_4l_b32_top.md"),
                 "metric": "encoder train sequences/s (config 4: 4 layers, d512, 8 heads, ff2048, S128, batch 32 per GPU, fp32, SGD; data parallel over N GPUs)",
                 "unit": "sequences/s", "loop": True, "cpu_iters": 1, "dp": "weak", "batch_per_gpu": 32,
                 "data": "synthetic: x ~ N(0,1) [4096, 512] per rank (seed 1000*rank) via Feeder; Xavier-uniform weights (seeded, same on every rank)"},
    "enc12": {"case": "enc_12_256_512_1024_16_4096_50_p8",
              "metric": "encoder train sequences/s (config 5 shard: 12 layers, d1024, 16 heads, ff4096, S512, batch 32 per GPU, fp32, SGD; data parallel over N GPUs)",
              "unit": "sequences/s", "loop": True, "cpu_iters": 0, "dp": "weak", "batch_per_gpu": 32,
              "data": "synthetic: x ~ N(0,1) [32*512, 1024] per rank (seed 1000*rank) via Feeder; Xavier-uniform weights (seeded, same on every rank)"},
    "enc3_d1024": {"case": "enc_3_96_512_1024_16_4096_50_p3",
                   "metric": "encoder train sequences/s (3 layers, d1024, 16 heads, ff4096, S512, batch 32 per GPU, fp32, SGD)",
                   "unit": "sequences/s", "loop": True, "cpu_iters": 0, "dp": "weak", "batch_per_gpu": 32,
                   "data": "synthetic: x ~ N(0,1) [32*512, 1024] per rank (seed 1000*rank) via Feeder; Xavier-uniform weights (seeded, same on every rank)"},
    "enc_small": {"case": "enc_1_8_128_512_8_2048_100",
                  "metric": "encoder train steps/s (1 layer, d512, 8 heads, ff2048, S128, B8, fp32, SGD)",
                  "unit": "steps/s", "loop": True, "cpu_iters": 1,
                  "data": "synthetic: x ~ N(0,1) [1024, 512] seed 0 via Feeder; Xavier-uniform weights (seeded)"},
    "dotsig": {"case": "dotsig_4096", "data": "synthetic: X, W, b ~ U(-1/64, 1/64), dz ~ N(0,1), seeded numpy default_rng", "metric": "fused DotProd+sigmoid fwd+bwd TFLOP/s (fp32 4096^3)",
               "unit": "TFLOP/s", "flops": 3 * 2 * 4096 ** 3, "inputs": ("X_id", "dz_id"),
               "cpu_dot_rows": 16, "dot_m": 4096,
               "profile": ("gemm_tcgen05", "gemm_tcgen05_dotsig_4096.md")},
}


def profile_traffic(wl, kind):
    """DRAM bytes (read + write) per launch of the dominant kernel, from the
    committed ncu summary of that kernel on this workload (one ncu capture of
    the same bench command; ``dram__bytes_read.sum`` + ``dram__bytes_write.sum``)."""
    prof = wl.get("profile")
    if not prof or prof[0] != kind:
        return None, None
    path = os.path.join(ROOT, "profiles", prof[1])
    if not os.path.exists(path):
        return None, None
    units = {"byte": 1, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9}
    total, seen = 0.0, 0
    with open(path) as f:
        for line in f:
            m = re.match(r"\|\s*dram__bytes_(read|write)\.sum\s*\|\s*([0-9.]+)\s*(\w+)", line)
            if m and m.group(3) in units:
                total += float(m.group(2)) * units[m.group(3)]
                seen += 1
    return (int(total), f"profiles/{prof[1]} (ncu)") if seen == 2 else (None, None)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    def __init__(self, index: int):
        self.index = index
        self.rows = []
        self.proc = None

    def __enter__(self):
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=2)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[0]) for r in self.rows if r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4)
                          if len(r) > 3 + i and r[3 + i].lower().startswith("active")})
        return {"sm_mhz": float(np.median(sm)) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(self.rows)}


def dist_env():
    return int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("LOCAL_RANK", "0"))


def host_group(world):
    if world == 1:
        return None
    import torch.distributed as td
    td.init_process_group("gloo")
    return td


def allmax(td, v: float) -> float:
    if td is None:
        return v
    import torch
    t = torch.tensor([v], dtype=torch.float64)
    td.all_reduce(t, op=td.ReduceOp.MAX)
    return float(t.item())


def barrier(td):
    if td is not None:
        td.barrier()


def cpu_measure(wl, p, max_steps=2, budget_s=20.0):
    """Time the reference's kernels (oracle/cexec.py: the C restatement of its
    OpenCL kernel bodies) on all host threads over a bounded sample of the
    workload.  Returns (value, seconds per full step, threads, sample text)."""
    from oracle.cexec import OracleDevice
    threads = os.cpu_count() or 1
    frac = 1.0
    dot_rows = wl.get("cpu_dot_rows")
    if dot_rows:
        frac = dot_rows / wl["dot_m"]
    d = OracleDevice(threads=threads, dot_rows=dot_rows)
    d.prepare(p)
    cmds = [c for c in p.procedure if type(c).__name__ not in ("AllocEntry", "DeallocEntry", "Receiver")]
    for c in cmds:
        d.run_cmd(c)
    t0 = time.perf_counter()
    n = 0
    while n < max_steps and (n == 0 or time.perf_counter() - t0 < budget_s):
        for c in cmds:
            d.run_cmd(c)
        n += 1
    dt = (time.perf_counter() - t0) / n
    if wl["unit"] == "GB/s":
        value = step_value(wl, wl.get("min_bytes") or alg_bytes_of(p), dt)
        sample = f"{n} full step(s) of {wl['case']}"
    else:
        value = wl["flops"] * frac / dt / 1e12
        sample = (f"{n} step(s) of {wl['case']} with each dot product restricted to its first "
                  f"{dot_rows} output rows ({frac:.4f} of the FLOPs)")
    return value, dt, threads, sample + f"; C restatement of the reference kernels, OpenMP x{threads}"


def cpu_reference(args, wl, rank, world):
    """``--impl reference``: the reference's CPU implementation of the path, rank 0 only."""
    if rank != 0:
        return
    from ad_b200.fixtures import load_case
    if wl.get("cpu_iters") == 0:
        print(json.dumps({"impl": "reference", "metric": wl["metric"], "unavailable":
                          "one step of this workload on the host restatement exceeds the bounded-sample budget"}),
              flush=True)
        return
    if wl.get("loop"):
        cb = cpu_loop_baseline(wl)
        value, dt, threads, sample = cb["value"], 1.0 / cb["value"], cb["cores"], cb["sample"]
    else:
        p, m = load_case(wl["case"])
        value, dt, threads, sample = cpu_measure(wl, p, max_steps=max(1, min(args.steps, args.cpu_steps)))
    line = {"impl": "reference", "metric": wl["metric"], "value": value, "unit": wl["unit"],
            "n_gpus": world, "steps": max(1, min(args.steps, args.cpu_steps)), "warmup": 1,
            "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": wl.get("data", "synthetic"), "config": {"workload": wl["case"]},
            "cpu_baseline": {"value": value, "unit": wl["unit"], "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": wl["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def feeder_proc(proc, dev, in_ids):
    """The prepared ``proc`` with its input buffers fed by Feeders (placed
    before the first command) whose ``func()`` returns a pageable numpy array,
    as a user of ``execute()`` supplies data.  Returns (proc, h2d, d2h bytes)."""
    from ad_b200 import ir
    feeders, h2d = [], 0
    for i, b in enumerate(in_ids):
        n = dev.slots[b].size
        arr = np.random.default_rng(100 + i).standard_normal(n, dtype=np.float32)
        k = ir.KMatrix(b, ir.Gid(), [n])
        feeders.append(ir.Feeder(-1 - i, [n], k, f"in{i}", func=lambda a=arr: a))
        h2d += arr.nbytes
    recv = [c for c in proc.procedure if type(c).__name__ == "Receiver"]
    d2h = sum(4 * int(np.prod(k.shape)) for r in recv for k in r.kargs)
    return ir.Proc(feeders + list(proc.procedure)), h2d, d2h


def alg_bytes_of(p):
    from ad_b200 import codegen, ir, memplan
    slots, _ = memplan.plan(p)
    sizes = {b: s.size for b, s in slots.items()}
    total = 0
    for c in ir.iter_cmds(p):
        k = type(c).__name__
        if k in ("ElwFuse", "BinaryNode", "UnaryNode", "ContigiousNode"):
            total += codegen.gen_elementwise(c, "k", sizes).bytes_moved
        elif k in ("ReduceNode", "ReduceElwFuse"):
            total += codegen.gen_reduce(c, "k", sizes).bytes_moved
        elif k in ("DotProdNode", "DPElwFuse"):
            _, M, N, K = codegen.dot_shape(c)
            total += 4 * (M * K + K * N + M * N)
    return total


def step_value(wl, alg_bytes, seconds):
    if wl["unit"] == "GB/s":
        return alg_bytes / seconds / 1e9
    return wl["flops"] / seconds / 1e12


def build_parser():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="enc_weak", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-steps", type=int, default=2)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--comm-profile", action="store_true",
                    help="data parallel: time each gradient all-reduce of one eager iteration")
    ap.add_argument("--no-kernel-timing", action="store_true",
                    help="skip the per-kernel isolated timings (loop workloads)")
    return ap


def main():
    args = build_parser().parse_args()
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        # NCCL's init lines name the communicator's rank count and its algorithms (NVLS);
        # set outright: an inherited NCCL_DEBUG=VERSION would hide them
        os.environ["NCCL_DEBUG"] = "INFO"
    args.warmup = max(args.warmup, 3)
    wl = WORKLOADS[args.workload]
    rank, world, local = dist_env()
    if args.impl == "reference":
        cpu_reference(args, wl, rank, world)
        return

    td = host_group(world)
    if wl.get("loop"):
        return bench_loop(args, wl, rank, world, local, td)
    from ad_b200 import ir
    from ad_b200.device import CudaB200Device
    from ad_b200.fixtures import load_case
    from ad_b200 import runtime as rt

    p, meta = load_case(wl["case"])
    dev = CudaB200Device(local)
    proc = dev.prepare(p)
    cmds = [c for c in proc.procedure if type(c).__name__ in ir.COMPUTE_KINDS]
    launches = [L for c in cmds for L in dev.launches[id(c)]]
    alg_bytes = sum(L.spec.bytes_moved for L in launches)
    ctx = dev.ctx

    # the step as one CUDA graph (no per-kernel host launch overhead)
    step_graph = dev.capture(cmds)
    for _ in range(args.warmup):
        step_graph.launch(0)
    ctx.sync()
    barrier(td)
    start, end = ctx.event(True), ctx.event(True)
    with ClockSampler(local) as clk:
        ctx.sync()
        start.record(0)
        for s in range(args.steps):
            step_graph.launch(0)
        end.record(0)
        end.sync()
    total_ms = start.elapsed_ms(end)
    ms = allmax(td, total_ms / args.steps)
    dev.check_errors()

    # each kernel timed alone: CUDA events around a graph of `rep` back-to-back launches
    rep = 5
    per_kernel = np.zeros(len(launches))
    for i, L in enumerate(launches):
        g = dev.capture_launches([L], rep)
        g.launch(0)
        e0, e1 = ctx.event(True), ctx.event(True)
        e0.record(0)
        for _ in range(3):
            g.launch(0)
        e1.record(0)
        e1.sync()
        per_kernel[i] = e0.elapsed_ms(e1) / (3 * rep)
    # the step's data was clobbered by the repeated launches (in-place kernels): re-prepare
    # is not needed for timing; correctness is covered by the parity tests.

    if wl["unit"] == "GB/s":
        value = step_value(wl, wl.get("min_bytes", alg_bytes), ms / 1e3) * world
    else:
        value = step_value(wl, None, ms / 1e3) * world

    # roofline of the dominant kernel
    hbm, bf16, peak_kind = peaks()
    top = int(np.argmax(per_kernel))
    Lt = launches[top]
    traffic, traffic_src = profile_traffic(wl, Lt.spec.kind)
    if Lt.spec.kind == "gemm_tcgen05":
        from ad_b200 import tcgen05
        tf32 = tcgen05.measure_tf32_peak(ctx, dev.err_ptr)
        executed = 3 * Lt.spec.flops   # 3xTF32: three MMAs per product
        achieved = executed / (per_kernel[top] / 1e3) / 1e12
        roof = {"bound": "tensor", "achieved": achieved, "peak": tf32, "unit": "TFLOP/s",
                "frac": achieved / tf32, "traffic": traffic,
                "peak_kind": "measured: kind::tf32 tcgen05 probe in this run (smem-resident operands)",
                "algorithmic_fp32_TFLOPs": Lt.spec.flops / (per_kernel[top] / 1e3) / 1e12,
                "bf16_peak_measured": bf16}
    else:
        achieved = Lt.spec.bytes_moved / (per_kernel[top] / 1e3) / 1e9
        roof = {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                "frac": achieved / hbm, "traffic": traffic, "peak_kind": peak_kind}
    roof.update({"kernel": f"{top}:{Lt.spec.kind}", "kernel_ms": float(per_kernel[top]),
                 "alg_bytes": Lt.spec.bytes_moved, "traffic_source": traffic_src})

    # e2e through the device's public run pass: the inputs enter as Feeders
    # whose func() returns pageable numpy arrays, the proc's Receiver hands
    # fresh numpy arrays to its callback
    in_ids = [meta[k] for k in wl.get("inputs", ("x_id", "dy_id")) if k in meta]
    fproc, h2d, d2h = feeder_proc(proc, dev, in_ids)
    e2e_steps = max(3, args.steps // 2)
    got = []
    for c in fproc.procedure:
        if type(c).__name__ == "Receiver":
            c.func = lambda *outs: got.append(len(outs))
    dev._run_proc(fproc, dev.run)
    ctx.sync()
    barrier(td)
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        dev._run_proc(fproc, dev.run)
    ctx.sync()
    e2e_ms = allmax(td, (time.perf_counter() - t0) * 1e3 / e2e_steps)
    assert len(got) == e2e_steps + 1

    if rank == 0:
        line = {
            "metric": wl["metric"], "value": value, "unit": wl["unit"], "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": wl.get("data", "synthetic: x ~ N(0,1) seed 0, dy ~ N(0,1) seed 1 (numpy default_rng)"),
            "config": {"workload": wl["case"], "alg_bytes_per_step": alg_bytes,
                       "min_bytes_per_step": wl.get("min_bytes"),
                       "kernel_bytes_GBps": alg_bytes / (ms / 1e3) / 1e9,
                       "kernels_per_step": len(launches), "l2": "inputs larger than L2 (128 MiB each)",
                       "parallelism": f"replicas x{world}"},
            "gpu_launches": len(launches) * args.steps,
            "roofline": roof,
            "per_kernel_ms": [round(float(x), 4) for x in per_kernel],
            "per_kernel_kind": [L.spec.kind for L in launches],
            "per_kernel_GBps": [round(L.spec.bytes_moved / (t / 1e3) / 1e9, 1) for L, t in zip(launches, per_kernel)],
            "clocks": clk.summary(),
            "e2e": {"value": step_value(wl, wl.get("min_bytes", alg_bytes), e2e_ms / 1e3) * world, "unit": wl["unit"],
                    "ms_per_step": e2e_ms, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "note": "per step one call of the device's run pass: Feeders of the inputs (pageable "
                            "numpy arrays), the step's kernels, the Receiver's copies into fresh numpy "
                            "arrays and its callback; host wall clock"},
            "compile_s": round(dev.compile_seconds, 2),
        }
        if not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(wl, p)
        print(json.dumps(line), flush=True)
    dev.close()
    barrier(td)


def bench_loop(args, wl, rank, world, local, td):
    """Loop workloads (config 1): one step = one iteration of the proc's ForNode
    body, replayed as a CUDA graph with the Feeder's host-to-device copy inside."""
    from ad_b200 import ir
    from ad_b200.device import CudaB200Device
    from ad_b200.fixtures import load_case, set_loop_count
    case = wl["case"]
    dp = None
    weak = wl.get("dp") == "weak"
    if world > 1 and wl.get("dp"):
        # data parallel, gradients summed with NCCL.  Strong: this rank's shard of
        # the fixed global batch.  Weak: the full per-GPU batch on every rank, each
        # with its own data (global batch = batch_per_gpu x world).
        if not weak:
            case = f"{case}_p{world}"
        from ad_b200 import dist
        box = [dist.nccl_unique_id() if rank == 0 else None]
        td.broadcast_object_list(box, src=0)
        dp = (rank, world, box[0])
    # weak scaling: each rank feeds its own batch (the fixture's seed shifted by rank)
    offset = 1000 * rank if weak else 0
    p, meta = load_case(case, rank=0 if weak else rank, feeder_seed_offset=offset)
    set_loop_count(p, args.warmup)
    dev = CudaB200Device(local, dp=dp)
    proc = dev.prepare(p)
    loop = next(c for c in proc.procedure if isinstance(c, ir.ForNode))
    body_cmds = [c for c in loop.proc.procedure if id(c) in dev.launches]
    launches = [L for c in body_cmds for L in dev.launches[id(c)]]
    ctx = dev.ctx
    dev._run_proc(proc, dev.run)          # warm-up: W iterations + final Receiver
    loop.r = range(args.steps)
    dev._replay_graph(loop)               # captures the graphs for this loop length outside the timing
    ctx.sync()
    barrier(td)
    e0, e1 = ctx.event(True), ctx.event(True)
    with ClockSampler(local) as clk:
        ctx.sync()
        e0.record(0)
        dev._replay_graph(loop)
        e1.record(0)
        e1.sync()
    ms = allmax(td, e0.elapsed_ms(e1) / args.steps)
    dev.check_errors()
    per_kernel = np.zeros(len(launches))
    for i, L in enumerate(launches if not args.no_kernel_timing else []):
        g = dev.capture_launches([L], 5)
        g.launch(0)
        a, b = ctx.event(True), ctx.event(True)
        a.record(0)
        for _ in range(3):
            g.launch(0)
        b.record(0)
        b.sync()
        per_kernel[i] = a.elapsed_ms(b) / 15
    top = int(np.argmax(per_kernel))
    Lt = launches[top]
    hbm, bf16, peak_kind = peaks()
    kt = max(per_kernel[top], 1e-9) / 1e3
    timed = not args.no_kernel_timing
    if timed and os.environ.get("AD_PROFILE_TOP") == "1":
        profile_one(dev, Lt)
    if Lt.spec.kind == "gemm_tcgen05" and not args.no_kernel_timing:
        from ad_b200 import tcgen05
        tf32 = tcgen05.measure_tf32_peak(ctx, dev.err_ptr)
        achieved = 3 * Lt.spec.flops / kt / 1e12      # 3xTF32: three MMAs per product
        roof = {"bound": "tensor", "achieved": achieved, "peak": tf32, "unit": "TFLOP/s",
                "frac": achieved / tf32, "traffic": None,
                "peak_kind": "measured: kind::tf32 tcgen05 probe in this run (smem-resident operands)",
                "algorithmic_fp32_TFLOPs": Lt.spec.flops / kt / 1e12, "bf16_peak_measured": bf16}
    else:
        achieved = Lt.spec.bytes_moved / kt / 1e9
        roof = {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                "frac": achieved / hbm, "traffic": None, "peak_kind": peak_kind}
    traffic, traffic_src = profile_traffic(wl, Lt.spec.kind)
    roof.update({"kernel": f"{top}:{Lt.spec.kind}", "kernel_ms": float(per_kernel[top]),
                 "alg_bytes": Lt.spec.bytes_moved, "traffic": traffic, "traffic_source": traffic_src,
                 "gflop": round(Lt.spec.flops / 1e9, 3)})
    if not timed:
        roof = None                     # --no-kernel-timing: no per-kernel figures
    work_set = dev.arena_bytes + getattr(dev, "scratch_bytes", 0)
    l2_note = (f"step working set {work_set / 1e6:.0f} MB (arena + dot-operand scratch) "
               + ("exceeds the 126 MB L2" if work_set > 126e6 else "fits in the 126 MB L2 (small model)"))
    feed_bytes = sum(4 * int(np.prod(c.shape)) for c in ir.iter_cmds(loop.proc) if type(c).__name__ == "Feeder")
    comm = comm_profile(dev, loop, td) if (args.comm_profile and dp) else None
    e2e = e2e_loop(dev, proc, loop, args.steps, td)
    if weak:
        value = 1e3 / ms * wl["batch_per_gpu"] * world       # sequences per second, whole job
    else:
        value = 1e3 / ms * (1 if dp else world)
    if rank == 0:
        line = {
            "metric": wl["metric"], "value": value, "unit": wl["unit"], "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong" if (dp and not weak) else "weak", "vs_baseline": None, "dtype": "f32", "data": wl["data"],
            "config": {"workload": case, "kernels_per_step": len(launches),
                       "global_batch": wl.get("global_batch") or wl.get("batch_per_gpu", 0) * world or None,
                       "step": "one ForNode iteration as a CUDA graph (Feeder H2D + kernels)",
                       "l2": l2_note,
                       "parallelism": (f"data parallel x{world} (NCCL all-reduce of gradients)" if dp
                                       else f"replicas x{world}")},
            "gpu_launches": len(launches) * args.steps,
            "roofline": roof,
            **({} if not timed else {
                "per_kernel_ms": [round(float(x), 4) for x in per_kernel],
                "per_kernel_kind": [L.spec.kind for L in launches],
                "per_kernel_gflop": [round(L.spec.flops / 1e9, 3) for L in launches],
                "per_kernel_GBps": [round(L.spec.bytes_moved / (t / 1e3) / 1e9, 1) if t > 0 else None
                                    for L, t in zip(launches, per_kernel)]}),
            "clocks": clk.summary(),
            "comm_profile": comm,
            "e2e": {"value": (value * ms / e2e["ms_per_step"]), "unit": wl["unit"],
                    "ms_per_step": e2e["ms_per_step"], "h2d_bytes_per_step": feed_bytes,
                    "d2h_bytes_per_step": e2e["d2h_bytes"] / args.steps,
                    "note": "one call of the device's run pass over the proc with the loop set to the timed "
                            "step count: each step calls the Feeder (a pageable numpy batch), which the device "
                            "stages into pinned memory and copies inside the step's graph; after the loop the "
                            "Receiver copies every parameter back into fresh numpy arrays and calls its "
                            "callback (d2h bytes amortised over the steps); host wall clock, max over ranks"},
        }
        if not args.no_cpu_baseline and wl["cpu_iters"] > 0 and world == 1:
            line["cpu_baseline"] = cpu_loop_baseline(wl)
        print(json.dumps(line), flush=True)
    dev.close()
    barrier(td)


def profile_one(dev, L):
    """One launch of ``L`` inside a profiler range (``ncu --profile-from-start off``
    then captures exactly this launch of the dominant kernel)."""
    from ad_b200 import runtime as rt
    dev.ctx.sync()
    rt.check(rt.lib().ad_profiler_range(1), "ad_profiler_range")
    dev._launch(L)
    dev.ctx.sync()
    rt.check(rt.lib().ad_profiler_range(0), "ad_profiler_range")


def comm_profile(dev, loop, td):
    """One eager (not graph) iteration of the loop body with CUDA events around
    every gradient all-reduce; then the same all-reduces alone, back to back."""
    from ad_b200 import runtime as rt
    ctx = dev.ctx
    for _ in range(2):
        dev.comm_trace = []
        barrier(td)
        a, b = ctx.event(True), ctx.event(True)
        a.record(0)
        dev._run_proc(loop.proc, dev.run)
        b.record(0)
        ctx.sync()
    it_ms = a.elapsed_ms(b)
    ops = [{"bytes": n, "async": asy, "ms": round(t0.elapsed_ms(t1), 4),
            "start_ms": round(a.elapsed_ms(t0), 4)} for n, asy, t0, t1 in dev.comm_trace]
    dev.comm_trace = None
    alone = []
    for op in ops:
        n = op["bytes"] // 4
        ctx.sync()
        barrier(td)
        e0, e1 = ctx.event(True), ctx.event(True)
        e0.record(0)
        for _ in range(5):
            rt.check(ctx.L.ad_allreduce_f32(ctx.h, dev.arena, dev.arena, n, 0, 0), "ad_allreduce_f32")
        e1.record(0)
        e1.sync()
        alone.append(round(e0.elapsed_ms(e1) / 5, 4))
    # the allreduces above summed arena contents over ranks; this run is for timing only
    return {"eager_iteration_ms": round(it_ms, 3), "ops": ops, "alone_ms": alone,
            "total_bytes": sum(o["bytes"] for o in ops)}


def e2e_loop(dev, proc, loop, steps, td):
    """The public run pass (``CudaB200Device._run_proc`` with ``run``, as
    ``execute`` calls it after init) over ``steps`` loop iterations, with the
    Feeder returning pageable numpy arrays; host wall clock."""
    import time as _t
    from ad_b200 import ir
    feeders = [c for c in ir.iter_cmds(loop.proc) if type(c).__name__ == "Feeder"]
    saved = [(f, f.func) for f in feeders]
    for f, fn in saved:
        first = np.array(fn(), dtype=np.float32, copy=True)
        pool = [first, first[::-1].copy()]          # two distinct pageable host arrays
        cnt = [0]

        def feed(pool=pool, cnt=cnt):
            cnt[0] += 1
            return pool[cnt[0] % 2]
        f.func = feed
    recv = [c for c in ir.iter_cmds(proc) if type(c).__name__ == "Receiver"]
    d2h = sum(4 * int(np.prod(k.shape)) for r in recv for k in r.kargs)
    loop.r = range(steps)
    dev._run_proc(proc, dev.run)             # graphs for this loop length exist after the first call
    dev.ctx.sync()
    barrier(td)
    t0 = _t.perf_counter()
    dev._run_proc(proc, dev.run)
    dev.ctx.sync()
    dt = allmax(td, _t.perf_counter() - t0)
    for f, fn in saved:
        f.func = fn
    return {"ms_per_step": dt * 1e3 / steps, "d2h_bytes": d2h}


def cpu_loop_baseline(wl):
    from ad_b200.fixtures import load_case, set_loop_count
    from oracle.cexec import OracleDevice
    n = wl["cpu_iters"]
    p, _ = load_case(wl["case"])
    set_loop_count(p, n)
    threads = os.cpu_count() or 1
    d = OracleDevice(threads=threads)
    d.prepare(p)
    t0 = time.perf_counter()
    d.run_proc(d.proc)
    dt = time.perf_counter() - t0
    per_step = wl.get("batch_per_gpu", 1) if wl["unit"] == "sequences/s" else 1
    return {"value": n * per_step / dt, "unit": wl["unit"], "cores": threads, "kind": "port",
            "sample": f"{n} iterations of {wl['case']} (C restatement of the reference kernels, OpenMP x{threads})"}


def cpu_baseline(wl, p):
    value, dt, threads, sample = cpu_measure(wl, p)
    return {"value": value, "unit": wl["unit"], "cores": threads, "kind": "port", "sample": sample}


if __name__ == "__main__":
    main()
