"""The F rank's expert math as torch CPU code -- TEST INFRASTRUCTURE ONLY (the timed CPU baseline).

The reference runs its experts through torch (SGLang FusedMoE, srt/managers/scheduler.py:410-412); it has no
CPU path of its own.  This module restates ``oracle.moe.ffn_pairs`` / ``reduce_pairs`` with torch fp32 tensors on
the host cores, so that the benchmark's CPU baseline is the reference's torch semantics timed with every thread
``torch.set_num_threads`` allows.  Arithmetic per pair, as oracle/moe.py states it:

    y2[t, j] = bf16( w[t, j] * W2_e act( silu(W1_e act(x_t)) * W3_e act(x_t) ) ),  e = ids[t, j] local
    reply[t] = bf16( sum_j y2[t, j] )  (fp32, ascending j)

with act = the MXFP8 round trip (OCP Microscaling v1.0 section 6.3: E8M0 scale 2^(floor(log2 amax) - 8) per 32
values, E4M3 elements by round-to-nearest-even, saturated at 448), the E4M3 per-1x128 round trip (fp32 scale
amax / 448), or none.  tests/test_oracle_torch.py pins it against the numpy oracle.
"""

from __future__ import annotations

import torch

_FP8_MAX = 448.0


def _bf16(v: torch.Tensor) -> torch.Tensor:
    return v.to(torch.bfloat16).to(torch.float32)


def mx_roundtrip(v: torch.Tensor) -> torch.Tensor:
    """fp32 [..., K] -> the fp32 values of its MXFP8 encoding (see the module docstring)."""
    blocks = v.reshape(*v.shape[:-1], v.shape[-1] // 32, 32)
    amax = blocks.abs().amax(dim=-1)
    # biased fp32 exponent of amax, minus emax(E4M3) = 8, clamped at the bottom of the E8M0 range
    biased = (amax.view(torch.int32) >> 23) & 0xFF
    s = torch.clamp(biased - 8, min=0)
    scale = torch.ldexp(torch.ones_like(amax), (s - 127).to(torch.float32))
    inv = torch.ldexp(torch.ones_like(amax), (127 - s).to(torch.float32))
    q = (blocks * inv[..., None]).clamp(-_FP8_MAX, _FP8_MAX).to(torch.float8_e4m3fn).to(torch.float32)
    return (q * scale[..., None]).reshape(v.shape)


def fp8_roundtrip(v: torch.Tensor) -> torch.Tensor:
    """fp32 [..., K] -> the fp32 values of its E4M3 per-1x128 encoding (fp32 scale amax / 448)."""
    blocks = v.reshape(*v.shape[:-1], v.shape[-1] // 128, 128)
    amax = blocks.abs().amax(dim=-1).clamp(min=1e-10)
    scale = amax / _FP8_MAX
    inv = torch.full_like(amax, _FP8_MAX) / amax  # a true division: python_scalar / tensor is reciprocal * scalar
    q = (blocks * inv[..., None]).clamp(-_FP8_MAX, _FP8_MAX).to(torch.float8_e4m3fn).to(torch.float32)
    return (q * scale[..., None]).reshape(v.shape)


def _act(v: torch.Tensor, act_quant) -> torch.Tensor:
    if act_quant == "fp8":
        return fp8_roundtrip(v)
    return mx_roundtrip(v) if act_quant else v


def ffn_pairs(x, ids, w, gate, up, w2, e0: int, experts, *, act_quant=True):
    """torch CPU tensors: x [n, H] fp32 (bf16 values), ids [n, k] int, w [n, k] fp32; gate/up [len(experts), I, H],
    w2 [len(experts), H, I] fp32 for the local experts ``experts`` (indices relative to e0).
    -> (y2 [n, k, H] fp32 bf16 values, used [n, k] bool)."""
    n, k = ids.shape
    y2 = torch.zeros(n, k, x.shape[1], dtype=torch.float32)
    used = torch.zeros(n, k, dtype=torch.bool)
    for slot, e in enumerate(experts):
        tt, jj = torch.nonzero(ids == e0 + e, as_tuple=True)
        if tt.numel() == 0:
            continue
        xa = _act(x[tt], act_quant)
        g = xa @ gate[slot].T
        u = xa @ up[slot].T
        h = _act(torch.nn.functional.silu(g) * u, act_quant)
        y2[tt, jj] = _bf16((h @ w2[slot].T) * w[tt, jj][:, None])
        used[tt, jj] = True
    return y2, used


def reduce_pairs(y2: torch.Tensor, used: torch.Tensor) -> torch.Tensor:
    out = torch.zeros(y2.shape[0], y2.shape[2], dtype=torch.float32)
    for j in range(y2.shape[1]):
        out += torch.where(used[:, j, None], y2[:, j], 0.0)
    return _bf16(out)
