"""Host-side weight quantisation (weight ingest of dense fp32/bf16 expert weights): MXFP4, and FP8 E4M3 with one
fp32 scale per 128 x 128 block.

FP8 block quantisation (the DeepSeek-V3 / SGLang block-FP8 checkpoint format, weight = e4m3 * scale_inv): per
128 x 128 block, scale = amax / 448 and codes = e4m3(w / scale), round to nearest even.

OCP Microscaling Formats v1.0, section 6.3, for E2M1 elements: per block of 32 values along K, shared exponent
X = floor(log2(amax)) - 2 (emax of E2M1), stored as E8M0 byte X + 127 (clamped to [0, 254]); elements are
v / 2^X rounded to the nearest E2M1 value {0, 0.5, 1, 1.5, 2, 3, 4, 6} (ties to the even code), saturating at 6.
"""

from __future__ import annotations

import numpy as np

_GRID = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])


def e2m1_round_codes(a: np.ndarray) -> np.ndarray:
    """Magnitudes (>= 0) -> E2M1 magnitude codes 0..7, round to nearest, ties to the even code, saturating."""
    a = np.minimum(np.asarray(a, np.float64), 6.0)
    hi = np.clip(np.searchsorted(_GRID, a, side="left"), 0, 7)
    lo = np.clip(hi - 1, 0, 7)
    dlo, dhi = a - _GRID[lo], _GRID[hi] - a
    pick_hi = (dhi < dlo) | ((dhi == dlo) & (hi % 2 == 0))
    return np.where(pick_hi, hi, lo).astype(np.uint8)


def mxfp4_quantize(w: np.ndarray):
    """[..., K] float (K % 32 == 0) -> (codes uint8 [..., K] with the sign in bit 3, scales uint8 [..., K/32])."""
    w = np.asarray(w, np.float32)
    blocks = w.reshape(*w.shape[:-1], w.shape[-1] // 32, 32)
    amax = np.abs(blocks).max(axis=-1)
    biased = ((amax.view(np.uint32) >> 23) & 0xFF).astype(np.int64)
    sb = np.clip(biased - 2, 0, 254).astype(np.uint8)
    scaled = blocks.astype(np.float64) / np.ldexp(1.0, sb.astype(np.int64) - 127)[..., None]
    codes = e2m1_round_codes(np.abs(scaled)) | (np.signbit(scaled).astype(np.uint8) << 3)
    return codes.reshape(w.shape), sb


def fp8_block_quantize(w):
    """[..., N, K] float (N, K multiples of 128) -> (E4M3 codes as uint8 [..., N, K], fp32 scales
    [..., N/128, K/128]); a torch tensor in, torch tensors out on its device."""
    import torch

    w = torch.as_tensor(w).float()
    *lead, n, k = w.shape
    b = w.reshape(*lead, n // 128, 128, k // 128, 128)
    amax = b.abs().amax(dim=(-3, -1))
    scale = torch.clamp(amax, min=1e-12) / 448.0
    q = (b / scale[..., :, None, :, None]).clamp_(-448.0, 448.0).to(torch.float8_e4m3fn)
    return q.view(torch.uint8).reshape(*lead, n, k).contiguous(), scale.contiguous()
