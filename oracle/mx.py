"""Microscaling codecs in numpy -- test infrastructure only (see oracle/__init__.py).

* E2M1 (FP4) values: sign bit 3, magnitudes {0, 0.5, 1, 1.5, 2, 3, 4, 6}; two per byte, low nibble first.
* E4M3 (FP8, "fn": no infinities, 0x7f/0xff NaN, max 448), bias 7.
* E8M0 scale byte s means 2^(s - 127).
* Activation block quantisation (32 values, one E8M0 scale): OCP Microscaling Formats v1.0 section 6.3 --
  shared exponent = floor(log2(amax)) - emax_elem with emax_elem = 8 for E4M3, clamped to the E8M0 range;
  elements = RNE(v / 2^shared) saturated to +-448.  The CUDA kernels apply exactly this rule, with the same
  fp32 operations, so the codes match bit for bit for identical inputs.

The reference quantises its activations to MXFP8 inside FlashInfer (srt/layers/quantization/
mxfp4_flashinfer_trtllm_moe.py:50-53 "runs MXFP8 activations"); that kernel is closed, so the rule above is
the published OCP one, not a copy of FlashInfer's.
"""

from __future__ import annotations

import numpy as np

E2M1_VALUES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                        -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], dtype=np.float32)


def e2m1_decode(codes: np.ndarray) -> np.ndarray:
    return E2M1_VALUES[codes.astype(np.int64) & 15]


def unpack_nibbles(packed: np.ndarray) -> np.ndarray:
    """[..., K/2] bytes -> [..., K] codes (element 2i in the low nibble of byte i)."""
    lo = packed & 0x0F
    hi = packed >> 4
    return np.stack([lo, hi], axis=-1).reshape(*packed.shape[:-1], packed.shape[-1] * 2)


def pack_nibbles(codes: np.ndarray) -> np.ndarray:
    c = codes.astype(np.uint8).reshape(*codes.shape[:-1], codes.shape[-1] // 2, 2)
    return (c[..., 0] | (c[..., 1] << 4)).astype(np.uint8)


def e8m0_value(s: np.ndarray) -> np.ndarray:
    return np.ldexp(np.float32(1.0), s.astype(np.int32) - 127).astype(np.float32)


def e4m3_decode(codes: np.ndarray) -> np.ndarray:
    c = codes.astype(np.int64)
    sign = np.where(c & 0x80, -1.0, 1.0)
    e = (c >> 3) & 15
    m = c & 7
    mag = np.where(e == 0, m * 2.0 ** -9, (1.0 + m / 8.0) * np.ldexp(1.0, e - 7))
    mag = np.where((c & 0x7F) == 0x7F, np.nan, mag)
    return (sign * mag).astype(np.float32)


def e4m3_encode(v: np.ndarray) -> np.ndarray:
    """fp32 -> E4M3 codes, round to nearest even, saturating to +-448 (cvt.rn.satfinite.e4m3x2.f32)."""
    v = np.asarray(v, dtype=np.float32)
    sign = (np.signbit(v)).astype(np.uint8) << 7
    a = np.minimum(np.abs(v).astype(np.float64), 448.0)
    code = np.zeros(a.shape, dtype=np.int64)
    sub = a < 2.0 ** -6
    code = np.where(sub, np.rint(a / 2.0 ** -9).astype(np.int64), code)  # 8 -> 0x08 = 2^-6, consistent
    with np.errstate(divide="ignore", invalid="ignore"):
        e = np.floor(np.log2(np.where(sub, 1.0, a))).astype(np.int64)
        # guard log2 rounding at exact powers of two
        e = np.where(np.ldexp(1.0, e) > a, e - 1, e)
        e = np.where(np.ldexp(1.0, e + 1) <= a, e + 1, e)
        m = np.rint((a / np.ldexp(1.0, e) - 1.0) * 8.0).astype(np.int64)
    carry = m == 8
    e = np.where(carry, e + 1, e)
    m = np.where(carry, 0, m)
    normal = ((e + 7) << 3) | m
    code = np.where(sub, code, normal)
    code = np.minimum(code, 0x7E)
    return (code.astype(np.uint8) | sign).astype(np.uint8)


def _biased_exponent(x: np.ndarray) -> np.ndarray:
    return ((np.asarray(x, dtype=np.float32).view(np.uint32) >> 23) & 0xFF).astype(np.int64)


def mx_scale_bytes(amax: np.ndarray) -> np.ndarray:
    """E8M0 scale byte of a block with absolute maximum ``amax`` (E4M3 elements, emax_elem = 8)."""
    return np.maximum(_biased_exponent(amax) - 8, 0).astype(np.uint8)


def mx_inv_scale(sbytes: np.ndarray) -> np.ndarray:
    """2^(127 - s) as fp32 (exact)."""
    return np.ldexp(np.float32(1.0), 127 - sbytes.astype(np.int32)).astype(np.float32)


def mx_quantize(v: np.ndarray):
    """[..., K] fp32 (K % 32 == 0) -> (E4M3 codes [..., K], E8M0 bytes [..., K/32])."""
    v = np.asarray(v, dtype=np.float32)
    blocks = v.reshape(*v.shape[:-1], v.shape[-1] // 32, 32)
    amax = np.max(np.abs(blocks), axis=-1)
    sb = mx_scale_bytes(amax)
    scaled = (blocks * mx_inv_scale(sb)[..., None]).astype(np.float32)
    q = e4m3_encode(scaled)
    return q.reshape(v.shape), sb


def mx_dequantize(q: np.ndarray, sb: np.ndarray) -> np.ndarray:
    vals = e4m3_decode(q).reshape(*q.shape[:-1], q.shape[-1] // 32, 32)
    return (vals * e8m0_value(sb)[..., None]).reshape(q.shape).astype(np.float32)


def mx_roundtrip(v: np.ndarray) -> np.ndarray:
    q, sb = mx_quantize(v)
    return mx_dequantize(q, sb)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """fp32 -> nearest bf16 (ties to even), returned as fp32."""
    u = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return r.astype(np.uint32).view(np.float32)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


def bf16_from_bits(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


# ---- scale-factor atoms: the device layout of E8M0 scales the tcgen05 scale-factor copy reads
def sf_atom_offset(r, kb, kblocks):
    """Byte offset of the scale of (row r, 32-block kb) in an array [r/128][kblocks/4][512]."""
    r = np.asarray(r, dtype=np.int64)
    kb = np.asarray(kb, dtype=np.int64)
    return ((r >> 7) * (kblocks >> 2) + (kb >> 2)) * 512 + (r & 31) * 16 + ((r >> 5) & 3) * 4 + (kb & 3)


def sf_to_atoms(sf: np.ndarray) -> np.ndarray:
    """[rows, kblocks] scale bytes (rows % 128 == 0, kblocks % 4 == 0) -> flat atom array."""
    rows, kblocks = sf.shape
    out = np.zeros(rows * kblocks, dtype=np.uint8)
    r, kb = np.meshgrid(np.arange(rows), np.arange(kblocks), indexing="ij")
    out[sf_atom_offset(r, kb, kblocks)] = sf
    return out


def sf_from_atoms(atoms: np.ndarray, rows: int, kblocks: int) -> np.ndarray:
    r, kb = np.meshgrid(np.arange(rows), np.arange(kblocks), indexing="ij")
    return atoms.reshape(-1)[sf_atom_offset(r, kb, kblocks)].astype(np.uint8)


def sf_to_kmajor_atoms(sf: np.ndarray) -> np.ndarray:
    """Weight scales [N, kblocks] -> atoms ordered [kblocks/4][N/128][512] (k-chunk outer), the weight layout."""
    n, kblocks = sf.shape
    out = np.zeros(n * kblocks, dtype=np.uint8)
    r, kb = np.meshgrid(np.arange(n), np.arange(kblocks), indexing="ij")
    off = ((kb >> 2) * (n >> 7) + (r >> 7)) * 512 + (r & 31) * 16 + ((r >> 5) & 3) * 4 + (kb & 3)
    out[off] = sf
    return out


def sf_from_kmajor_atoms(atoms: np.ndarray, n: int, kblocks: int) -> np.ndarray:
    r, kb = np.meshgrid(np.arange(n), np.arange(kblocks), indexing="ij")
    off = ((kb >> 2) * (n >> 7) + (r >> 7)) * 512 + (r & 31) * 16 + ((r >> 5) & 3) * 4 + (kb & 3)
    return atoms.reshape(-1)[off].astype(np.uint8)


# ---------------------------------------------------------------- FP8 per 1 x 128 (fp32 scale)
FP8_MAX = np.float32(448.0)


def fp8_act_quantize(v: np.ndarray):
    """[..., K] fp32 (K % 128 == 0) -> (E4M3 codes [..., K], fp32 scales [..., K/128]).  SGLang's per-token-group
    FP8 quantisation (group 128): amax clamped to 1e-10, scale = amax / 448, codes = e4m3(v * (448 / amax)),
    every operation one fp32 rounding (as libasap's quant_permute_fp8 kernel and FP8 GEMM1 epilogue compute it)."""
    v = np.asarray(v, dtype=np.float32)
    blocks = v.reshape(*v.shape[:-1], v.shape[-1] // 128, 128)
    amax = np.maximum(np.max(np.abs(blocks), axis=-1), np.float32(1e-10)).astype(np.float32)
    scale = (amax / FP8_MAX).astype(np.float32)
    inv = (FP8_MAX / amax).astype(np.float32)
    q = e4m3_encode((blocks * inv[..., None]).astype(np.float32))
    return q.reshape(v.shape), scale


def fp8_act_dequantize(q: np.ndarray, scale: np.ndarray) -> np.ndarray:
    vals = e4m3_decode(q).reshape(*q.shape[:-1], q.shape[-1] // 128, 128)
    return (vals * scale[..., None]).reshape(q.shape).astype(np.float32)


def fp8_act_roundtrip(v: np.ndarray) -> np.ndarray:
    return fp8_act_dequantize(*fp8_act_quantize(v))


def fp8_block_dequantize(codes: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """E4M3 weights [..., N, K] with fp32 scales [..., N/128, K/128] -> fp32 (weight = e4m3 * scale)."""
    vals = e4m3_decode(codes)
    *lead, n, k = vals.shape
    b = vals.reshape(*lead, n // 128, 128, k // 128, 128) * np.asarray(scale, np.float32)[..., :, None, :, None]
    return b.reshape(*lead, n, k).astype(np.float32)
