"""The MoE oracle against independent restatements: brute-force loops for the routing tables and the
expert-major permutation, a float64 torch evaluation of the reference's expert formula
(srt/managers/scheduler.py:410-412), and the reference's own send-everything-to-every-F semantics
(transport/channel.py:340-355 + token_dispatcher/asap.py:178-184), which per-F bucketing must reproduce exactly."""

import numpy as np
import pytest
import torch

from asap_b200.quant import mxfp4_quantize
from oracle import moe, mx


def brute_tables(ids, bounds):
    F, n = len(bounds) - 1, len(ids)
    row_of = [[-1] * n for _ in range(F)]
    for f in range(F):
        r = 0
        for t in range(n):
            if any(bounds[f] <= e < bounds[f + 1] for e in ids[t]):
                row_of[f][t] = r
                r += 1
    return row_of


def brute_perm(ids, e0, P):
    n, k = len(ids), len(ids[0])
    counts = [0] * P
    for t in range(n):
        for j in range(k):
            if e0 <= ids[t][j] < e0 + P:
                counts[ids[t][j] - e0] += 1
    start, acc = [], 0
    for c in counts:
        start.append(acc)
        acc += -(-c // 128) * 128
    pos = [[-1] * k for _ in range(n)]
    nxt = list(start)
    for e in range(P):
        for t in range(n):
            for j in range(k):
                if ids[t][j] == e0 + e:
                    pos[t][j] = nxt[e]
                    nxt[e] += 1
    return pos, counts


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_tables_and_permutation_match_brute_force(seed):
    rng = np.random.default_rng(seed)
    n, k, E = 50, 4, 24
    ids = rng.integers(-2, E + 2, (n, k))  # includes ids that go nowhere
    ids[3] = [5, 5, 5, 5]  # duplicates count twice (FusedMoE semantics)
    bounds = [0, 7, 7, 16, 24]  # uneven, one empty F rank
    row_of, count, pad = moe.f_rank_tables(ids, bounds)
    assert row_of.tolist() == brute_tables(ids.tolist(), bounds)
    assert count[1] == 1 and pad[1] == 1
    for f in range(4):
        sel = row_of[f] >= 0
        e0, P = bounds[f], bounds[f + 1] - bounds[f]
        if P == 0:
            continue
        pos, mstart, counts = moe.expert_permutation(ids[sel], e0, P)
        bpos, bcounts = brute_perm(ids[sel].tolist(), e0, P)
        assert pos.tolist() == bpos
        assert counts.tolist() == bcounts
        assert (np.diff(mstart) == -(-np.array(bcounts) // 128)).all()


def _random_experts(rng, P, H, I):
    w13 = rng.standard_normal((P, 2 * I, H)).astype(np.float32) * 0.05
    w2 = rng.standard_normal((P, H, I)).astype(np.float32) * 0.05
    return w13, w2


def test_ffn_formula_against_torch_float64():
    rng = np.random.default_rng(5)
    P, H, I, n, k = 6, 64, 32, 40, 3
    w13, w2 = _random_experts(rng, P, H, I)
    gate, up = w13[:, :I], w13[:, I:]
    x = mx.bf16_round(rng.standard_normal((n, H)).astype(np.float32))
    ids = rng.integers(0, P + 3, (n, k))  # some non-local
    w = rng.random((n, k)).astype(np.float32)
    got = moe.ffn_rank(x, ids, w, gate, up, w2, 0, P, act_quant=False)
    X = torch.from_numpy(x).double()
    ref = torch.zeros(n, H, dtype=torch.float64)
    for t in range(n):
        for j in range(k):
            e = int(ids[t, j])
            if 0 <= e < P:
                g = torch.from_numpy(gate[e]).double() @ X[t]
                u = torch.from_numpy(up[e]).double() @ X[t]
                h = torch.nn.functional.silu(g) * u
                ref[t] += float(w[t, j]) * (torch.from_numpy(w2[e]).double() @ h)
    assert moe.rel_l2(got, ref.numpy()) < 4e-3  # bf16 rounding of rows and of the sum


def test_bucketed_round_trip_equals_send_everything():
    """Sending each F rank only its tokens changes no output value: the reference sends every token to every F
    rank and sums all partials (tokens without a local expert contribute exact zeros)."""
    rng = np.random.default_rng(6)
    H, I, n, k = 64, 32, 30, 2
    bounds = [0, 4, 8, 12]
    experts = []
    for f in range(3):
        w13, w2 = _random_experts(rng, 4, H, I)
        experts.append((w13[:, :I], w13[:, I:], w2))
    x = mx.bf16_round(rng.standard_normal((n, H)).astype(np.float32))
    ids = rng.integers(0, 12, (n, k))
    w = rng.random((n, k)).astype(np.float32)
    shared = mx.bf16_round(rng.standard_normal((n, H)).astype(np.float32))
    got = moe.round_trip(x, ids, w, bounds, experts, shared=shared)
    parts = [moe.ffn_rank(x, ids, w, *experts[f], bounds[f], 4) for f in range(3)]
    acc = parts[0].astype(np.float32).copy()
    for p in parts[1:]:
        acc += p
    ref = mx.bf16_round(mx.bf16_round(acc) + shared)
    np.testing.assert_array_equal(got, ref)


def test_activation_quant_error_is_the_mxfp8_level():
    rng = np.random.default_rng(7)
    P, H, I, n, k = 4, 256, 128, 64, 2
    w13, w2 = _random_experts(rng, P, H, I)
    x = mx.bf16_round(rng.standard_normal((n, H)).astype(np.float32))
    ids = rng.integers(0, P, (n, k))
    w = rng.random((n, k)).astype(np.float32)
    a = moe.ffn_rank(x, ids, w, w13[:, :I], w13[:, I:], w2, 0, P, act_quant=True)
    b = moe.ffn_rank(x, ids, w, w13[:, :I], w13[:, I:], w2, 0, P, act_quant=False)
    err = moe.rel_l2(a, b)
    assert 5e-3 < err < 8e-2


def test_mxfp4_weight_quantizer():
    rng = np.random.default_rng(8)
    w = rng.standard_normal((8, 64)).astype(np.float32) * 0.02
    codes, sb = mxfp4_quantize(w)
    deq = mx.e2m1_decode(codes).reshape(8, 2, 32) * mx.e8m0_value(sb)[..., None]
    deq = deq.reshape(8, 64)
    amax = np.abs(w).reshape(8, 2, 32).max(-1)
    # shared exponent floor(log2 amax) - 2: amax / scale in [4, 8)
    r = amax / mx.e8m0_value(sb)
    assert np.all((r >= 4) & (r < 8))
    assert moe.rel_l2(deq, w) < 0.15
    # exact grid values survive unchanged
    grid = np.array([[0, .5, 1, 1.5, 2, 3, 4, 6] * 4], np.float32)
    c, s = mxfp4_quantize(grid)
    np.testing.assert_array_equal(mx.e2m1_decode(c) * mx.e8m0_value(s).repeat(32, -1), grid)


def test_topk_routing():
    rng = np.random.default_rng(9)
    logits = rng.standard_normal((16, 32))
    for kind in ("softmax", "sigmoid"):
        ids, w = moe.topk_routing(logits, 4, kind)
        assert ids.shape == (16, 4) and np.allclose(w.sum(1), 1, atol=1e-6)
        assert all(len(set(r)) == 4 for r in ids.tolist())
