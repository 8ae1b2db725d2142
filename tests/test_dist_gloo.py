"""Data-parallel rewrite on CPU: 2 gloo ranks, each with half the batch, vs one
process with the full batch (the oracle executes both; no GPU)."""
import os
import socket

import numpy as np
import pytest
import torch.distributed as td
import torch.multiprocessing as mp

from ad_b200 import dist
from ad_b200.fixtures import load_case
from oracle.cexec import OracleDevice

FULL = "encdy_1_2_16_32_2_64_3"
PART = "encdy_1_2_16_32_2_64_3_p2"


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank(rank, world, port, out_q):
    import torch
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    td.init_process_group("gloo", rank=rank, world_size=world)
    try:
        p, _ = load_case(PART, rank=rank)

        def allreduce(a):
            t = torch.from_numpy(a)           # shares memory with the oracle buffer
            td.all_reduce(t, op=td.ReduceOp.SUM)

        gb = dist.insert_grad_allreduce(p, comm=allreduce)
        assert gb is not None
        d = OracleDevice(faithful_tree=False, threads=1)
        d.execute(p)
        out_q.put((rank, [o.copy() for o in d.last_received]))
    finally:
        td.destroy_process_group()


def test_two_ranks_match_full_batch():
    want_p, _ = load_case(FULL)
    o = OracleDevice(faithful_tree=False, threads=1)
    o.execute(want_p)
    want = o.last_received
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for pr in procs:
        pr.start()
    res = dict(q.get(timeout=300) for _ in range(2))
    for pr in procs:
        pr.join(timeout=60)
        assert pr.exitcode == 0
    for r in range(2):
        for g, w in zip(res[r], want):
            np.testing.assert_allclose(g, w, rtol=1e-3, atol=1e-4)
    for g0, g1 in zip(res[0], res[1]):
        np.testing.assert_array_equal(g0, g1)     # ranks stay bit-identical


def test_rewrite_structure():
    p, _ = load_case(PART)          # parameters are the AllocEntries with content
    gb = dist.insert_grad_allreduce(p)
    loop = next(c for c in p.procedure if type(c).__name__ == "ForNode")
    kinds = [type(c).__name__ for c in loop.proc.procedure]
    ars = [c for c in loop.proc.procedure if type(c).__name__ == "AllReduce"]
    assert 1 <= len(ars) <= 3
    # the all-reduces tile the bucket exactly once
    spans = sorted((a.offset, a.offset + a.count) for a in ars)
    assert spans[0][0] == 0 and all(spans[i][1] == spans[i + 1][0] for i in range(len(spans) - 1))
    ups = [c for c in loop.proc.procedure if type(c).__name__ == "BinaryNode" and c.in_place]
    assert len(ups) == 15
    assert kinds.index("AllReduce") < min(loop.proc.procedure.index(u) for u in ups)


def test_rewrite_without_peers_is_identity():
    """With a no-op all-reduce the rewritten proc computes exactly what the
    reference's order computes (updates still land before their next reader)."""
    p, _ = load_case(FULL)
    o = OracleDevice(faithful_tree=False, threads=1)
    o.execute(p)
    q, _ = load_case(FULL)
    dist.insert_grad_allreduce(q, comm=lambda a: None)
    o2 = OracleDevice(faithful_tree=False, threads=1)
    o2.execute(q)
    for g, w in zip(o2.last_received, o.last_received):
        np.testing.assert_array_equal(g, w)


def test_async_buckets_overlap_backward():
    """Bucketed all-reduces start as soon as their gradients exist and are
    joined as late as the next reader allows: on the 4-layer encoder's rank
    proc some join sits several commands after its start, every join precedes
    the updates of its members, and the buckets tile the gradient buffer."""
    from ad_b200.device import CudaB200Device
    p, _ = load_case("enc_4_32_128_512_8_2048_100_p2")
    q = CudaB200Device.passes_only(p, world=2)
    loop = next(c for c in q.procedure if type(c).__name__ == "ForNode")
    body = loop.proc.procedure
    starts = {id(c): i for i, c in enumerate(body) if type(c).__name__ == "AllReduce"}
    assert starts and all(c.async_start for c in body if type(c).__name__ == "AllReduce")
    gaps, n_updates = [], [0]
    for i, c in enumerate(body):
        if type(c).__name__ != "AllReduceWait":
            continue
        for s in c.starts:
            assert starts[id(s)] < i
            gaps.append(i - starts[id(s)])
            members = set(s.members)
            for j, u in enumerate(body):
                for v in (u.cmds if type(u).__name__ == "Batched" else [u]):
                    if type(v).__name__ == "BinaryNode" and v.in_place and \
                            any(getattr(k, "id", None) in members for k in v.kargs):
                        assert j > i
                        n_updates[0] += 1
    assert max(gaps) >= 5 and n_updates[0] == 4 * 33
    ars = sorted((c.offset, c.offset + c.count) for c in body if type(c).__name__ == "AllReduce")
    assert ars[0][0] == 0 and all(a[1] == b[0] for a, b in zip(ars, ars[1:]))
