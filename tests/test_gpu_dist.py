"""Data parallelism on 2 GPUs with NCCL (skipped with fewer GPUs): each rank runs
its half of the batch through the device, gradients are summed with
``ad_allreduce_f32`` inside the CUDA-graph loop replay; parameters must match
the single-process full-batch oracle (rel 1e-3)."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

FULL = "encdy_1_2_16_32_2_64_3"
PART = "encdy_1_2_16_32_2_64_3_p2"


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank(rank, world, port, q, comm="nccl"):
    import torch.distributed as td
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0",
                      AD_DP_COMM=comm)
    td.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from ad_b200 import dist
        from ad_b200.device import CudaB200Device
        from ad_b200.fixtures import load_case
        box = [dist.nccl_unique_id() if rank == 0 else None]
        td.broadcast_object_list(box, src=0)
        p, _ = load_case(PART, rank=rank)
        d = CudaB200Device(rank, dp=(rank, world, box[0]))
        d.execute(p)
        q.put((rank, [o.copy() for o in d.last_received]))
        d.close()
    except Exception as e:          # report instead of hanging the parent
        q.put((rank, repr(e)))
    finally:
        td.destroy_process_group()


@pytest.mark.parametrize("comm", ["nccl", "peer"])
def test_two_gpu_data_parallel_matches_full_batch(comm):
    """``peer``: the library's own all-reduce kernel over CUDA IPC mappings."""
    from ad_b200 import runtime as rt
    if rt.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    from ad_b200.fixtures import load_case
    from oracle.cexec import OracleDevice
    p, _ = load_case(FULL)
    o = OracleDevice(faithful_tree=False)
    o.execute(p)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q, comm)) for r in range(2)]
    for pr in procs:
        pr.start()
    res = dict(q.get(timeout=600) for _ in range(2))
    for pr in procs:
        pr.join(timeout=120)
    for r in range(2):
        assert not isinstance(res[r], str), res[r]
        for g, w in zip(res[r], o.last_received):
            np.testing.assert_allclose(g, w, rtol=1e-3, atol=1e-4)
    for g0, g1 in zip(res[0], res[1]):
        np.testing.assert_array_equal(g0, g1)        # every rank holds the same parameters
