"""The oracle's microscaling codecs against independent implementations (torch's float8_e4m3fn cast, the E2M1
value table, torch's bf16 rounding) and the OCP MX scale rule's properties."""

import numpy as np
import pytest
import torch

from oracle import mx


def test_e4m3_encode_matches_torch_cast():
    rng = np.random.default_rng(0)
    vals = np.concatenate([
        rng.standard_normal(20000).astype(np.float32) * 50,
        rng.uniform(-448, 448, 20000).astype(np.float32),
        np.ldexp(rng.uniform(-1, 1, 5000), rng.integers(-12, -5, 5000)).astype(np.float32),  # subnormal range
        np.array([0.0, -0.0, 448.0, -448.0, 2.0 ** -9, 2.0 ** -10, 1.0625, 1.1875, 15.5, 240.0, 232.0],
                 dtype=np.float32),
    ])
    ours = mx.e4m3_encode(vals)
    ref = torch.from_numpy(vals).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.testing.assert_array_equal(ours, ref)
    np.testing.assert_array_equal(mx.e4m3_decode(ours), torch.from_numpy(ref).view(torch.float8_e4m3fn).float().numpy())


def test_e4m3_saturates():
    codes = mx.e4m3_encode(np.array([500.0, -1e6, 449.0, 463.9], dtype=np.float32))
    np.testing.assert_array_equal(mx.e4m3_decode(codes), [448.0, -448.0, 448.0, 448.0])


def test_e2m1_table():
    expect = [0, .5, 1, 1.5, 2, 3, 4, 6]
    np.testing.assert_array_equal(mx.e2m1_decode(np.arange(8)), expect)
    np.testing.assert_array_equal(mx.e2m1_decode(np.arange(8) + 8), [-v for v in expect])
    packed = mx.pack_nibbles(np.array([[1, 2, 15, 0]]))
    assert packed.tolist() == [[0x21, 0x0F]]
    np.testing.assert_array_equal(mx.unpack_nibbles(packed), [[1, 2, 15, 0]])


def test_bf16_round_matches_torch():
    rng = np.random.default_rng(1)
    v = (rng.standard_normal(100000) * np.exp(rng.uniform(-20, 20, 100000))).astype(np.float32)
    ref = torch.from_numpy(v).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(mx.bf16_round(v), ref)


def test_mx_scale_rule():
    # shared exponent = floor(log2(amax)) - 8 (E4M3 emax), so amax / 2^shared lies in [256, 512)
    rng = np.random.default_rng(2)
    v = rng.standard_normal((64, 32)).astype(np.float32) * np.exp(rng.uniform(-10, 10, (64, 1))).astype(np.float32)
    q, sb = mx.mx_quantize(v)
    amax = np.abs(v).max(axis=1)
    ratio = amax / mx.e8m0_value(sb[:, 0])
    assert np.all((ratio >= 256) & (ratio < 512))
    deq = mx.mx_dequantize(q, sb)
    rel = np.abs(deq - v) / np.maximum(np.abs(v), 1e-30)
    scaled = np.abs(v) / mx.e8m0_value(sb[:, 0])[:, None]
    normal = (scaled >= 2.0 ** -6) & (scaled <= 448)
    assert np.all(rel[normal] <= 2.0 ** -4 + 1e-6)  # 3 mantissa bits: half an ulp
    sat = scaled > 448  # the OCP rule lets the top of a block saturate at 448 (< 512)
    assert np.all(rel[sat] <= 0.125 + 1e-6)


def test_mx_zero_block_and_tiny():
    q, sb = mx.mx_quantize(np.zeros((1, 32), np.float32))
    assert sb[0, 0] == 0 and not q.any()
    tiny = np.full((1, 32), 1e-40, np.float32)
    q, sb = mx.mx_quantize(tiny)
    assert sb[0, 0] == 0
    assert np.all(np.isfinite(mx.mx_dequantize(q, sb)))


def test_sf_atoms_roundtrip():
    rng = np.random.default_rng(3)
    sf = rng.integers(0, 256, (256, 8), dtype=np.uint8)
    atoms = mx.sf_to_atoms(sf)
    np.testing.assert_array_equal(mx.sf_from_atoms(atoms, 256, 8), sf)
    # atom byte (r%32)*16 + ((r/32)%4)*4 + kb%4 within atom [r/128][kb/4]
    assert atoms[512 * 1 + 5 * 16 + 2 * 4 + 3] == sf[64 + 5, 4 + 3]
    katoms = mx.sf_to_kmajor_atoms(sf)
    np.testing.assert_array_equal(mx.sf_from_kmajor_atoms(katoms, 256, 8), sf)
    assert katoms[(1 * 2 + 1) * 512 + 7 * 16 + 3 * 4 + 1] == sf[128 + 96 + 7, 4 + 1]


@pytest.mark.parametrize("shape", [(3, 64), (128, 1024)])
def test_mx_quantize_is_deterministic_and_idempotent(shape):
    rng = np.random.default_rng(4)
    v = rng.standard_normal(shape).astype(np.float32)
    a = mx.mx_roundtrip(v)
    np.testing.assert_array_equal(a, mx.mx_roundtrip(v))
    np.testing.assert_array_equal(mx.mx_roundtrip(a), a)
