"""Host-side pieces of bench.py on CPU: topologies, expert splits, the routing generators (config 2 sigmoid,
config 4 softmax, config 5 Zipf), the clock-sample filter and the config-1 CPU timing."""

import time

import numpy as np
import pytest
import torch

import bench


def test_topology_and_expert_bounds():
    assert bench.topology("half", 2) == (1, 1)
    assert bench.topology("half", 8) == (4, 4)
    assert bench.topology("2a6f", 8) == (2, 6)
    assert bench.topology("2a4f", 6) == (2, 4)
    with pytest.raises(SystemExit):
        bench.topology("2a6f", 6)
    b = bench.expert_bounds(6)
    assert b[0] == 0 and b[-1] == 256 and sorted(np.diff(b)) == [42, 42, 43, 43, 43, 43]
    assert bench.expert_bounds(4) == [0, 64, 128, 192, 256]


def test_routing_generators():
    saved = {k: getattr(bench, k) for k in ("E", "K_TOP", "ROUTING")}
    try:
        for routing, E, k in (("sigmoid", 256, 8), ("softmax", 64, 6)):
            bench.E, bench.K_TOP, bench.ROUTING = E, k, routing
            ids, w = bench.make_routing(512, 3, "cpu")
            assert ids.shape == (512, k) and ids.dtype == torch.int32 and w.dtype == torch.float32
            assert torch.all((ids >= 0) & (ids < E))
            assert torch.all(torch.tensor([len(set(r.tolist())) == k for r in ids]))  # distinct experts per token
            assert torch.allclose(w.sum(1), torch.ones(512), atol=1e-5)
        bench.E, bench.K_TOP = 256, 8
        ids, w = bench.zipf_routing(20000, 1, "cpu")
        ids2, _ = bench.zipf_routing(20000, 2, "cpu")
        c1 = torch.bincount(ids.flatten().long(), minlength=256)
        c2 = torch.bincount(ids2.flatten().long(), minlength=256)
        assert int(c1.argmax()) == int(c2.argmax())  # popularity is a property of the model, not of the seed
        assert c1.max() > 0.8 * 20000  # the top expert of Zipf(1.2) is in most tokens' top-8
        assert torch.all(torch.tensor([len(set(r.tolist())) == 8 for r in ids[:500]]))
        assert torch.allclose(w.sum(1), torch.ones(20000), atol=1e-5)
    finally:
        for k, v in saved.items():
            setattr(bench, k, v)


def test_clock_sampler_window():
    c = bench.ClockSampler(0)
    now = time.time()
    c.t_start, c.t_end = now, now + 0.2
    line = "0, {}, 1965, 700.0, 0x0, Not Active, Not Active, Not Active, {}"
    c.lines = [(now - 1.0, line.format(1000, "Active")), (now + 0.05, line.format(1965, "Not Active")),
               (now + 0.15, line.format(1950, "Active"))]
    s = c.summary()
    assert s["samples"] == 2 and s["sm_mhz"] == pytest.approx(1957.5) and s["reasons"] == ["sw_power_cap"]
    c.t_start, c.t_end = now + 0.3, now + 0.31  # no sample inside (a region shorter than the period): nearest
    s = c.summary()
    assert s["samples"] == 2 and s["window"].startswith("nearest")


def test_cpu_config1_runs():
    r = bench.cpu_config1(reps=1)
    assert r["value"] > 0 and r["unit"] == "tokens/s"


def test_placement():
    assert bench.placement(8, 4, "block") == ([0, 1, 2, 3], [4, 5, 6, 7])
    assert bench.placement(8, 4, "interleave") == ([0, 2, 4, 6], [1, 3, 5, 7])
    assert bench.placement(8, 2, "interleave") == ([0, 4], [1, 2, 3, 5, 6, 7])
    for world, n_a in ((2, 1), (4, 2), (6, 2), (8, 2), (8, 4)):
        for how in ("block", "interleave"):
            a, f = bench.placement(world, n_a, how)
            assert a[0] == 0 and len(a) == n_a and sorted(a + f) == list(range(world))


def test_layer_roofline_4a4f():
    """The per-layer roofline at 4A4F (config 2): each F rank receives the 90.36% of each replica's tokens that
    route to its 64 experts, 11.54 TFLOP of expert GEMMs."""
    peaks = {"hbm_gbs": 6547.5, "bf16_tflops_sustained": 1361.5}
    rows = round(4 * 16384 * 0.9036)
    r = bench.layer_roofline(4, 16384, [rows] * 4, [0, 64, 128, 192, 256], 8.06, peaks, "measured", nvlink_gbs=770.0)
    assert r["bound"] == "tensor" and r["peaks"]["nvlink_gbs"] == 770.0
    assert r["t_flop_ms"] == pytest.approx(11.544e12 / 2723e12 * 1e3, rel=1e-3)   # 4.24 ms
    assert r["t_in_ms"] == pytest.approx(rows * (2 * 7168 + 64) / 770e9 * 1e3, abs=1e-4)  # 1.11 ms
    assert r["t_out_ms"] == pytest.approx(rows * 2 * 7168 / 770e9 * 1e3, abs=1e-4)
    assert r["t_serial_ms"] == pytest.approx(r["t_in_ms"] + r["t_out_ms"] + r["t_flop_ms"], abs=1e-3)
    assert 6.3 < r["t_serial_ms"] < 6.5
    assert r["frac"] == pytest.approx(r["t_bound_ms"] / 8.06, abs=1e-4)
    # uneven F ranks: the most loaded one sets the bound
    r2 = bench.layer_roofline(2, 16384, [30000, 50000], [0, 100, 256], 5.0, peaks, "measured")
    assert r2["t_flop_ms"] == pytest.approx(2 * 16384 * 8 * 156 / 256 * 6 * 7168 * 2048 / 2723e12 * 1e3, rel=1e-3)
    # no link rate measured: the nominal NVLink 5 figure, labelled as such
    r3 = bench.layer_roofline(4, 16384, [rows] * 4, [0, 64, 128, 192, 256], 8.06, peaks, "measured")
    assert r3["peaks"]["nvlink_gbs"] == 900.0 and "nominal" in r3["peaks"]["source"]


def test_hbm_kernel_gbs():
    T, pairs = 16384, 131072
    r = bench.hbm_kernel_gbs(T, pairs, {"quantise_permute": 0.42, "reduce_reply": 0.45})
    qp = T * 2 * 7168 + pairs * (7168 + 7168 // 32)
    assert r["bytes"]["quantise_permute"] == qp  # 1.20 GB
    assert r["quantise_permute"] == pytest.approx(qp / 0.42e-3 / 1e9, abs=0.1)
    assert r["bytes"]["reduce_reply"] == pairs * 2 * 7168 + T * 2 * 7168
    assert bench.hbm_kernel_gbs(T, pairs, {"quantise_permute": 0.0, "reduce_reply": 0.45})["quantise_permute"] is None


def test_f_job_launches():
    """wait + route count/scan/place + quantise + GEMM1 + GEMM2 + reduce (+ gather for joined jobs)."""
    assert bench.f_job_launches() == 8 and bench.f_job_launches(4) == 9


def test_first_then_rest_policy():
    """--serve auto: the first ready message alone and the rest joined when three or more replicas send and a
    message brings an F rank fewer than FTR_PAIRS expected pairs; per-message jobs otherwise."""
    from types import SimpleNamespace

    args = SimpleNamespace(serve="auto", join_replicas=False)
    assert bench.E == 256 and bench.K_TOP == 8
    assert not bench.first_then_rest(args, 4, 16384, 64)  # config 2 at 4A4F: 32768 pairs per message
    assert bench.first_then_rest(args, 4, 4096, 64)
    assert not bench.first_then_rest(args, 1, 256, 256)  # one replica: nothing to join
    assert not bench.first_then_rest(args, 2, 4096, 43)  # two replicas: the rest is a single message
    assert bench.first_then_rest(SimpleNamespace(serve="first-then-rest", join_replicas=False), 4, 16384, 64)
    assert not bench.first_then_rest(SimpleNamespace(serve="per-message", join_replicas=False), 4, 256, 64)
    assert not bench.first_then_rest(SimpleNamespace(serve="auto", join_replicas=True), 4, 256, 64)
