"""The torch CPU restatement of the expert math (oracle/torch_cpu.py, the timed CPU baseline) against the numpy
oracle: MXFP8 and FP8 round trips bit-exact, per-pair rows and the reply reduce within fp32 summation-order
noise."""

import numpy as np
import torch

from oracle import moe, mx
from oracle import torch_cpu as tc


def test_mx_roundtrip_matches_numpy():
    rng = np.random.default_rng(0)
    v = (rng.standard_normal((64, 256)) * np.exp(rng.uniform(-20, 20, (64, 1)))).astype(np.float32)
    v[0, :32] = 0.0  # an all-zero block
    v[1, 5] = 1e30   # saturating block
    np.testing.assert_array_equal(tc.mx_roundtrip(torch.from_numpy(v)).numpy(), mx.mx_roundtrip(v))


def test_fp8_roundtrip_matches_numpy():
    rng = np.random.default_rng(1)
    v = (rng.standard_normal((16, 512)) * 3.0).astype(np.float32)
    v[2, :128] = 0.0
    np.testing.assert_array_equal(tc.fp8_roundtrip(torch.from_numpy(v)).numpy(), mx.fp8_act_roundtrip(v))


def test_ffn_pairs_and_reduce_match_numpy():
    rng = np.random.default_rng(2)
    n, k, P, H, I = 48, 4, 6, 256, 128
    x = mx.bf16_round(rng.standard_normal((n, H)).astype(np.float32))
    ids, w = moe.topk_routing(rng.standard_normal((n, P + 2)), k, "softmax")
    gate = (rng.standard_normal((P, I, H)) * 0.05).astype(np.float32)
    up = (rng.standard_normal((P, I, H)) * 0.05).astype(np.float32)
    w2 = (rng.standard_normal((P, H, I)) * 0.05).astype(np.float32)
    for act in (True, "fp8", False):
        y_np, used_np = moe.ffn_pairs(x, ids, w, gate, up, w2, 1, P, act_quant=act)
        y_t, used_t = tc.ffn_pairs(torch.from_numpy(x), torch.from_numpy(ids.astype(np.int64)), torch.from_numpy(w),
                                   torch.from_numpy(gate), torch.from_numpy(up), torch.from_numpy(w2), 1, range(P),
                                   act_quant=act)
        np.testing.assert_array_equal(used_t.numpy(), used_np)
        assert moe.rel_l2(y_t.numpy(), y_np) < 1e-3  # activation codes may tip where fp32 sums differ by an ulp
        r_np = moe.reduce_pairs(y_np, used_np)
        r_t = tc.reduce_pairs(torch.from_numpy(y_np), torch.from_numpy(used_np)).numpy()
        np.testing.assert_array_equal(r_t, r_np)  # same rows, same order: the reduce is bit-exact
