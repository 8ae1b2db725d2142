"""Host-side pieces of bench.py and the fixture loader (CPU)."""
import numpy as np

import bench
from ad_b200 import ir
from ad_b200.fixtures import load_case


def test_profile_traffic_reads_committed_ncu_summary():
    """roofline.traffic = dram read + write bytes of the dominant kernel, parsed
    from its committed ncu summary; other kernels / workloads get None."""
    t, src = bench.profile_traffic(bench.WORKLOADS["lnsm"], "rowfused")
    assert src.startswith("profiles/rowfused_lnsm_8192x4096.md")
    assert 4e8 < t < 6e8                      # ~0.49 GB per launch vs 0.54 GB algorithmic
    assert bench.profile_traffic(bench.WORKLOADS["lnsm"], "elementwise") == (None, None)
    assert bench.profile_traffic(bench.WORKLOADS["mlp"], "rowfused") == (None, None)


def test_feeder_seed_offset_changes_only_feeder_data():
    """Weak-scaling ranks feed their own batch; weights stay identical."""
    p0, _ = load_case("enc_1_2_16_32_2_64_3")
    p1, _ = load_case("enc_1_2_16_32_2_64_3", feeder_seed_offset=1000)

    def feeds(p):
        return [c.func() for c in ir.iter_cmds(p) if isinstance(c, ir.Feeder)]

    def params(p):
        return [np.asarray(c.content) for c in ir.iter_cmds(p)
                if isinstance(c, ir.AllocEntry) and c.content is not None]

    f0, f1 = feeds(p0), feeds(p1)
    assert f0 and all(a.shape == b.shape and not np.array_equal(a, b) for a, b in zip(f0, f1))
    for a, b in zip(params(p0), params(p1)):
        np.testing.assert_array_equal(a, b)


def test_feeder_proc_feeds_inputs_before_first_command():
    """Config 2's e2e leg: the inputs enter through Feeders (pageable numpy
    arrays of the input buffers' size) placed before every other command."""
    import types
    from ad_b200 import memplan
    p, m = load_case("lnsm_16_4096")
    slots, _ = memplan.plan(p)
    dev = types.SimpleNamespace(slots=slots)
    fp, h2d, d2h = bench.feeder_proc(p, dev, [m["x_id"], m["dy_id"]])
    head = fp.procedure[:2]
    assert [type(c).__name__ for c in head] == ["Feeder", "Feeder"]
    assert [c.kres.id for c in head] == [m["x_id"], m["dy_id"]]
    for c in head:
        a = c.func()
        assert isinstance(a, np.ndarray) and a.dtype == np.float32 and list(a.shape) == c.shape
    assert h2d == 2 * 16 * 4096 * 4 and d2h == 2 * 16 * 4096 * 4
    assert fp.procedure[2:] == p.procedure


def test_default_workload_is_config4_encoder():
    args = bench.build_parser().parse_args([])
    assert args.workload == "enc_weak" and args.gpus == 1 and args.warmup >= 3
    assert bench.WORKLOADS["enc_weak"]["case"] == "enc_4_32_128_512_8_2048_100"
    assert bench.WORKLOADS["enc_weak"]["dp"] == "weak"
