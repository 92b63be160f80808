"""The whole A->F->A round trip on one GPU (one A rank and one F rank, loopback arenas), through the
reference-facing API (AsapMoE.forward / AsapDispatcher.dispatch + combine / AsapBuffer), against the oracle:
relative L2 <= 1e-2 of the reference semantics with the same MXFP8 activation quantisation; the F rank's
region bytes, the doorbell word in its host page and the per-F-rank token table bit-exact."""

import numpy as np
import pytest
import torch

from asap_b200.dispatcher import AsapDispatcher
from asap_b200.experts import Mxfp4Experts
from asap_b200.layer import AsapMoE
from asap_b200.loopback import Loopback
from asap_b200.quant import mxfp4_quantize
from asap_b200.sglang_shim import StandardTopKOutput
from asap_b200.transport.layout import Geometry, pack_doorbell
from gpu_util import bf16_tensor_from_np, experts_to_oracle, np_from_bf16
from oracle import moe, mx

pytestmark = pytest.mark.gpu
TOL = 1e-2


def config1_experts(rng, E=16, H=1024, I=512):
    w13 = rng.standard_normal((E, 2 * I, H)).astype(np.float32) * 0.02
    w2 = rng.standard_normal((E, H, I)).astype(np.float32) * 0.02
    c13, s13 = mxfp4_quantize(w13)
    c2, s2 = mxfp4_quantize(w2)
    return Mxfp4Experts.from_logical(c13, s13, c2, s2)


@pytest.fixture(scope="module")
def pair(cuda_ok):
    rng = np.random.default_rng(0)
    experts = {0: config1_experts(rng), 5: config1_experts(rng)}
    lb = Loopback(Geometry(1, 1, 2, 512, 1024, 2, 1), experts, timeout_s=5.0)
    lb.install()
    oracle_w = {lid: experts_to_oracle(e) for lid, e in experts.items()}
    yield lb, oracle_w
    lb.close()
    for e in experts.values():
        e.release()


def run_layer(lb, layer_id, x, ids, w, shared=None, micro_batch=None):
    disp = AsapDispatcher(layer_id)
    topk = StandardTopKOutput(torch.from_numpy(w).cuda(), torch.from_numpy(ids).cuda())
    out = disp.dispatch(bf16_tensor_from_np(x), topk, micro_batch=micro_batch)
    res = disp.combine(out, shared=None if shared is None else bf16_tensor_from_np(shared))
    torch.cuda.synchronize()
    lb.check()
    return np_from_bf16(res)


def test_config1_round_trip(pair):
    """Benchmark config 1 (T=512, H=1024, 16 experts, top-2 softmax, I=512), plus a bf16 shared expert output."""
    lb, ow = pair
    rng = np.random.default_rng(1)
    T = 512
    x = mx.bf16_round(rng.standard_normal((T, 1024)).astype(np.float32))
    ids, w = moe.topk_routing(rng.standard_normal((T, 16)), 2, "softmax")
    shared = mx.bf16_round(rng.standard_normal((T, 1024)).astype(np.float32) * 0.1)
    got = run_layer(lb, 0, x, ids, w, shared)
    ref = moe.round_trip(x, ids, w, [0, 16], [ow[0]], shared=shared)
    assert moe.rel_l2(got, ref) < TOL
    plain = moe.round_trip(x, ids, w, [0, 16], [ow[0]], shared=shared, act_quant=False)
    assert moe.rel_l2(got, plain) < 8e-2
    # wire bytes of the message: region rows, doorbell word, routing table
    g = lb.g
    seq = lb.channel._last_sent[0]
    reg = torch.as_tensor(lb.sched.recv_arena[g.region_off(0, 0): g.region_off(0, 1)]).cpu().numpy()
    np.testing.assert_array_equal(reg[: T * 1024 * 2].view(np.uint16).reshape(T, 1024), mx.bf16_bits(x))
    np.testing.assert_array_equal(reg[g.ids_off: g.ids_off + T * 2 * 4].view(np.int32).reshape(T, 2), ids)
    word = int(lb.server.bell_words[0])
    assert word == pack_doorbell(seq, T, 0, lb.channel.epochs[0])
    row_of = lb.channel.route_ws(0)[512: 512 + 4 * T].view(torch.int32).cpu().numpy()
    np.testing.assert_array_equal(row_of, np.arange(T))


def test_asap_moe_forward_layers_and_slots(pair):
    """AsapMoE.forward on two layers (different weights) and both slots, many messages (seq advances,
    backpressure on each slot is satisfied by the previous answer)."""
    lb, ow = pair
    rng = np.random.default_rng(2)
    for it in range(6):
        layer = (0, 5)[it % 2]
        T = int(rng.integers(1, 513))
        x = mx.bf16_round(rng.standard_normal((T, 1024)).astype(np.float32))
        ids, w = moe.topk_routing(rng.standard_normal((T, 16)), 2, "softmax")
        if it % 3 == 0:
            moe_layer = AsapMoE(16, 1024, 512, layer, top_k=2)
            topk = StandardTopKOutput(torch.from_numpy(w).cuda(), torch.from_numpy(ids).cuda())
            got = np_from_bf16(moe_layer(bf16_tensor_from_np(x), topk))
            torch.cuda.synchronize()
            lb.check()
        else:
            got = run_layer(lb, layer, x, ids, w, micro_batch=it % 2)
        ref = moe.round_trip(x, ids, w, [0, 16], [ow[layer]])
        assert moe.rel_l2(got, ref) < TOL, (it, T)


def test_tokens_routed_nowhere_and_empty_batch(pair):
    lb, ow = pair
    rng = np.random.default_rng(3)
    T = 64
    x = mx.bf16_round(rng.standard_normal((T, 1024)).astype(np.float32))
    ids = np.full((T, 2), -1, np.int32)
    w = np.zeros((T, 2), np.float32)
    shared = mx.bf16_round(rng.standard_normal((T, 1024)).astype(np.float32))
    got = run_layer(lb, 0, x, ids, w, shared)
    np.testing.assert_array_equal(got, shared)  # F got one padding row; every token's routed output is 0
    ids[::2, 0] = 3  # half the tokens routed
    w[::2, 0] = 1.0
    got = run_layer(lb, 0, x, ids, w)
    ref = moe.round_trip(x, ids, w, [0, 16], [ow[0]])
    assert moe.rel_l2(got, ref) < TOL
    assert not got[1::2].any()
    # an empty batch never reaches the transport
    disp = AsapDispatcher(0)
    empty = torch.empty(0, 1024, dtype=torch.bfloat16, device="cuda")
    topk = StandardTopKOutput(torch.empty(0, 2, device="cuda"), torch.empty(0, 2, dtype=torch.int32, device="cuda"))
    assert disp.combine(disp.dispatch(empty, topk)).shape == (0, 1024)


def test_exchange_splits_batches_larger_than_n_max(pair):
    lb, ow = pair
    rng = np.random.default_rng(4)
    T = 1100  # > n_max = 512: three pieces
    x = mx.bf16_round(rng.standard_normal((T, 1024)).astype(np.float32))
    ids, w = moe.topk_routing(rng.standard_normal((T, 16)), 2, "softmax")
    got = run_layer(lb, 5, x, ids, w)
    ref = moe.round_trip(x, ids, w, [0, 16], [ow[5]])
    assert moe.rel_l2(got, ref) < TOL


def test_deepseek_v3_layer_shape(cuda_ok):
    """A DeepSeek-V3-shape layer (H=7168, I=2048, top-8 sigmoid) on 16 routed experts, 192 tokens."""
    rng = np.random.default_rng(5)
    E, H, I, T, k = 16, 7168, 2048, 192, 8
    e = Mxfp4Experts.random(E, H, I, seed=5, scale_lo=117, scale_hi=120)
    lb = Loopback(Geometry(1, 1, 1, 256, H, k, 1), {0: e}, timeout_s=5.0)
    lb.install()
    try:
        gate, up, w2 = experts_to_oracle(e)
        x = mx.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
        ids, w = moe.topk_routing(rng.standard_normal((T, E)), k, "sigmoid")
        shared = mx.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
        got = run_layer(lb, 0, x, ids, w, shared)
        ref = moe.round_trip(x, ids, w, [0, E], [(gate, up, w2)], shared=shared)
        assert moe.rel_l2(got, ref) < TOL
    finally:
        lb.close()
        e.release()


def _from_fp32(rng, E, H, I, base):
    w13 = rng.standard_normal((E, 2 * I, H)).astype(np.float32) * 0.02
    w2 = rng.standard_normal((E, H, I)).astype(np.float32) * 0.02
    c13, s13 = mxfp4_quantize(w13)
    c2, s2 = mxfp4_quantize(w2)
    return Mxfp4Experts.from_logical(c13, s13, c2, s2, expert_base=base)


def test_config1_two_f_ranks(cuda_ok):
    """Benchmark config 1 exactly: 1 A replica + 2 F ranks with 8 experts each (T=512, H=1024, top-2 softmax over
    16 experts, I=512, fp32 N(0, 0.02) weights as MXFP4, x ~ N(0,1) bf16, seed 0)."""
    rng = np.random.default_rng(0)
    T, H, I = 512, 1024, 512
    per_f = [{0: _from_fp32(rng, 8, H, I, 0)}, {0: _from_fp32(rng, 8, H, I, 8)}]
    lb = Loopback(Geometry(1, 1, 2, T, H, 2, 2), per_f, timeout_s=5.0)
    lb.install()
    try:
        ow = [experts_to_oracle(d[0]) for d in per_f]
        x = mx.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
        ids, w = moe.topk_routing(rng.standard_normal((T, 16)), 2, "softmax")
        got = run_layer(lb, 0, x, ids, w)
        ref = moe.round_trip(x, ids, w, [0, 8, 16], ow)
        assert moe.rel_l2(got, ref) < TOL
        # every token to F rank 0 only: F rank 1 gets the one padding row and answers it with zeros
        ids0 = np.stack([rng.permutation(8)[:2] for _ in range(T)]).astype(np.int32)
        got0 = run_layer(lb, 0, x, ids0, w)
        ref0 = moe.round_trip(x, ids0, w, [0, 8, 16], ow)
        assert moe.rel_l2(got0, ref0) < TOL
        row_of = lb.channel.route_ws(0)[512: 512 + 4 * 2 * T].view(torch.int32).view(2, T).cpu().numpy()
        np.testing.assert_array_equal(row_of, moe.f_rank_tables(ids0, [0, 8, 16])[0])
    finally:
        lb.close()
        for d in per_f:
            d[0].release()


def test_uneven_six_f_ranks(cuda_ok):
    """The 2A6F-style uneven contiguous split (here 6/6/5/5/5/5 of 32 experts), top-8 sigmoid routing."""
    rng = np.random.default_rng(7)
    T, H, I, k = 300, 256, 128, 8
    sizes = [6, 6, 5, 5, 5, 5]
    bases = np.concatenate([[0], np.cumsum(sizes)])
    per_f = [{3: Mxfp4Experts.random(sz, H, I, expert_base=int(b), seed=10 + f)}
             for f, (sz, b) in enumerate(zip(sizes, bases[:-1]))]
    lb = Loopback(Geometry(1, 1, 1, T, H, k, 6), per_f, timeout_s=5.0)
    lb.install()
    try:
        ow = [experts_to_oracle(d[3]) for d in per_f]
        x = mx.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
        ids, w = moe.topk_routing(rng.standard_normal((T, 32)), k, "sigmoid")
        shared = mx.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
        got = run_layer(lb, 3, x, ids, w, shared)
        ref = moe.round_trip(x, ids, w, [int(b) for b in bases], ow, shared=shared)
        assert moe.rel_l2(got, ref) < TOL
        counts = [lb.scheds[f].debug_tensors()["expert_counts"].cpu().numpy() for f in range(6)]
        for f in range(6):
            sel = moe.f_rank_tables(ids, [int(b) for b in bases])[0][f] >= 0
            np.testing.assert_array_equal(counts[f], moe.expert_counts(ids[sel], int(bases[f]), sizes[f]))
    finally:
        lb.close()
        for d in per_f:
            d[3].release()


def test_zipf_skew_four_f_ranks_and_timestamps(cuda_ok):
    """Routing skew (config 5's shape, scaled down): Zipf(s=1.2) expert popularity over a seeded permutation of 32
    experts, top-8 without replacement, 4 F ranks of 8 -- the most popular expert takes most tokens (a segment of
    several 128-row tiles), some experts none.  Per-F row counts announced by the dispatch, per-expert counts
    (bit-exact) and the output (rel L2) against the oracle; the device timestamps are ordered."""
    rng = np.random.default_rng(11)
    T, H, I, k, E_, n_f = 700, 256, 128, 8, 32, 4
    per_f = [{0: Mxfp4Experts.random(8, H, I, expert_base=8 * f, seed=30 + f)} for f in range(n_f)]
    bounds = [0, 8, 16, 24, 32]
    lb = Loopback(Geometry(1, 1, 2, T, H, k, n_f), per_f, timeout_s=5.0)
    lb.install()
    try:
        ow = [experts_to_oracle(d[0]) for d in per_f]
        logp = np.empty(E_)
        logp[rng.permutation(E_)] = -1.2 * np.log(np.arange(1, E_ + 1))
        scores = logp[None, :] - np.log(-np.log(rng.uniform(1e-12, 1.0, (T, E_))))
        ids = np.argsort(-scores, axis=1)[:, :k].astype(np.int32)
        w = 1.0 / (1.0 + np.exp(-rng.standard_normal((T, k))))
        w = (w / w.sum(1, keepdims=True)).astype(np.float32)
        x = mx.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
        got = run_layer(lb, 0, x, ids, w)
        ref = moe.round_trip(x, ids, w, bounds, ow)
        assert moe.rel_l2(got, ref) < TOL
        tables = moe.f_rank_tables(ids, bounds)[0]
        stream = torch.cuda.current_stream().cuda_stream
        info = lb.channel.dispatch_info(0, stream)
        assert info["counts"] == [int((tables[f] >= 0).sum()) for f in range(n_f)]
        top = np.bincount(ids.ravel(), minlength=E_).max()
        assert top > 3 * 128  # the skew really spans several tiles of one expert
        for f in range(n_f):
            sel = tables[f] >= 0
            c = lb.scheds[f].debug_tensors()["expert_counts"].cpu().numpy()
            np.testing.assert_array_equal(c, moe.expert_counts(ids[sel], bounds[f], 8))
        jobs = [sc.job_info(stream) for sc in lb.scheds]
        assert 0 < info["t_ring_ns"] <= jobs[0]["t_seen_ns"]
        for j in jobs:
            assert j["t_seen_ns"] <= j["t_reply_ns"] <= info["t_replies_ns"]
    finally:
        lb.close()
        for d in per_f:
            d[0].release()


def test_cuda_graph_mode_matches_eager(cuda_ok):
    """F jobs as CUDA-graph replays (one graph per (slot, layer), captured on first use; the doorbell wait keeps its
    sequence word on the device): bit-identical to the eager chain, over several messages on two slots and three
    layers, including an eager job in between (the device word is re-synchronised before the next replay)."""
    rng = np.random.default_rng(8)
    T, H, I, k, E = 96, 256, 128, 4, 8
    layers = {l: Mxfp4Experts.random(E, H, I, seed=40 + l) for l in range(3)}
    outs = {}
    for graphs in (False, True):
        lb = Loopback(Geometry(1, 1, 2, T, H, k, 1), layers, timeout_s=5.0, graphs=graphs)
        lb.install()
        try:
            r = np.random.default_rng(9)
            got = []
            for step in range(4):
                for layer in range(3):
                    slot = (step + layer) % 2
                    x = mx.bf16_round(r.standard_normal((T - step, H)).astype(np.float32))
                    ids, w = moe.topk_routing(r.standard_normal((T - step, E)), k, "sigmoid")
                    if graphs and step == 2 and layer == 1:  # one eager job between replays on this slot
                        lb.local.graphs = False
                        got.append(run_layer(lb, layer, x, ids, w, micro_batch=slot))
                        lb.local.graphs = True
                    else:
                        got.append(run_layer(lb, layer, x, ids, w, micro_batch=slot))
            lb.check()
            outs[graphs] = got
            if graphs:
                assert lb.sched.graph_replays == 11 and len(lb.sched._graphs) == 6
        finally:
            lb.close()
    for e in layers.values():
        e.release()
    assert len(outs[False]) == len(outs[True]) == 12
    for a, b in zip(outs[False], outs[True]):
        np.testing.assert_array_equal(a, b)  # the eager chain is checked against the oracle by the tests above
