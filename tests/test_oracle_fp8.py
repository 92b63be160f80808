"""The oracle's FP8 pieces on CPU: the E4M3 encoder against torch's own float8_e4m3fn conversion (an independent
implementation of the same round-to-nearest-even rule), the per-1x128 activation quantisation's defining
properties, the block dequantisation, and the host-side FP8 weight quantiser (product code) against them."""

import numpy as np
import torch

from asap_b200.quant import fp8_block_quantize
from oracle import moe, mx


def test_e4m3_encode_matches_torch_float8():
    rng = np.random.default_rng(0)
    # every representable magnitude, the midpoints between neighbours (ties), and random values over the range
    grid = np.unique(np.abs(mx.e4m3_decode(np.arange(0, 0x7F, dtype=np.uint8))))
    mids = (grid[:-1] + grid[1:]) / 2
    rand = rng.standard_normal(20000).astype(np.float32) * np.float32(2.0) ** rng.integers(-12, 9, 20000)
    v = np.concatenate([grid, -grid, mids, -mids, rand, [447.9, 448.0, -448.0]]).astype(np.float32)
    v = v[np.abs(v) <= 448.0]
    ours = mx.e4m3_encode(v)
    ref = torch.from_numpy(v).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    # torch keeps the sign of a zero result; so does the encoder
    np.testing.assert_array_equal(ours, ref)


def test_fp8_act_quantize_properties():
    rng = np.random.default_rng(1)
    x = (rng.standard_normal((7, 512)) * 3).astype(np.float32)
    x[2, :128] = 0.0  # an all-zero block
    q, s = mx.fp8_act_quantize(x)
    assert q.shape == x.shape and s.shape == (7, 4) and s.dtype == np.float32
    amax = np.abs(x.reshape(7, 4, 128)).max(-1)
    np.testing.assert_array_equal(s, (np.maximum(amax, np.float32(1e-10)) / np.float32(448.0)).astype(np.float32))
    deq = mx.fp8_act_dequantize(q, s)
    assert np.all(deq[2, :128] == 0)
    # the block maximum maps to +-448 exactly; every element within half an E4M3 step (relative 2^-4)
    blocks = np.abs(mx.e4m3_decode(q)).reshape(7, 4, 128)
    assert np.all(blocks.max(-1)[amax > 0] == 448.0)
    err = np.abs(deq - x)
    assert np.all(err <= np.abs(x) * 2.0 ** -4 + s.repeat(128, axis=1) * 2.0 ** -9 + 1e-30)


def test_fp8_block_quantizer_and_dequant():
    rng = np.random.default_rng(2)
    w = (rng.standard_normal((2, 256, 384)) * 0.02).astype(np.float32)
    q, s = fp8_block_quantize(torch.from_numpy(w))
    q, s = q.numpy(), s.numpy()
    assert q.dtype == np.uint8 and s.shape == (2, 2, 3)
    deq = mx.fp8_block_dequantize(q, s)
    blocks = np.abs(w).reshape(2, 2, 128, 3, 128).max(axis=(2, 4))
    np.testing.assert_allclose(s, blocks / 448.0, rtol=1e-6)
    assert moe.rel_l2(deq, w) < 0.03
    # the codes are the oracle's E4M3 rounding of w / scale
    expect = mx.e4m3_encode((w.reshape(2, 2, 128, 3, 128) / s[:, :, None, :, None]).reshape(w.shape))
    assert np.mean(expect == q) > 0.999  # division vs the oracle's float64 path may tip an exact tie
    gate, up, w2 = moe.dequant_fp8(q, s, q[:, :, :256], s[:, :, :2])
    assert gate.shape == (2, 128, 384) and up.shape == (2, 128, 384)
    np.testing.assert_array_equal(gate, deq[:, :128])


def test_ffn_rank_fp8_mode_close_to_unquantised():
    rng = np.random.default_rng(3)
    P, H, I, n, k = 3, 256, 128, 40, 2
    gate = (rng.standard_normal((P, I, H)) * 0.05).astype(np.float32)
    up = (rng.standard_normal((P, I, H)) * 0.05).astype(np.float32)
    w2 = (rng.standard_normal((P, H, I)) * 0.05).astype(np.float32)
    x = mx.bf16_round(rng.standard_normal((n, H)).astype(np.float32))
    ids, w = moe.topk_routing(rng.standard_normal((n, P)), k, "softmax")
    exact = moe.ffn_rank(x, ids, w, gate, up, w2, 0, P, act_quant=False)
    fp8 = moe.ffn_rank(x, ids, w, gate, up, w2, 0, P, act_quant="fp8")
    assert 1e-4 < moe.rel_l2(fp8, exact) < 0.05
