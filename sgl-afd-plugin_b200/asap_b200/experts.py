"""Routed-expert weights of one layer on one F rank, in the device layout libasap's tcgen05 GEMMs read.

MXFP4: E2M1 values (two per byte, low nibble first) with one E8M0 scale per 32 values along K (the
``flashinfer_mxfp4`` weights of the reference's F ranks, scripts/run_asap.sh:99).  Layout (include/asap.h,
asap_mxfp4_experts_t):

  w13     uint8 [P, 2I, H/2]  gate (W1) and up (W3) rows interleaved in blocks of 128 (rows 256b..256b+127 are
                              gate rows 128b.., rows 256b+128.. are up rows 128b..), so one 256-row GEMM tile
                              holds matching gate and up columns and the SwiGLU runs in the GEMM epilogue
  w13_sf  uint8 [P, H/128, 2I/128, 512]  scale atoms (k-chunk outer)
  w2      uint8 [P, H, I/2]
  w2_sf   uint8 [P, I/128, H/128, 512]

``from_logical`` builds that layout from plain [P, rows, K] codes and [P, rows, K/32] scale bytes (the
checkpoint layout after SGLang's loader, W13 = [W1; W3]); ``random`` makes seeded synthetic weights.

FP8 (``Fp8Experts``): E4M3 weights with one fp32 scale per 128 x 128 block, in the checkpoint's own layout
(include/asap.h, asap_fp8_experts_t): w13 [P, 2I, H] (gate rows then up rows), w13_scale [P, 2I/128, H/128],
w2 [P, H, I], w2_scale [P, H/128, I/128].
"""

from __future__ import annotations

import ctypes
from typing import Optional

import numpy as np
import torch

from . import _native as N


def _aligned_empty(nbytes: int, device, align: int = 1024) -> tuple[torch.Tensor, torch.Tensor]:
    """A uint8 buffer of nbytes whose address is ``align``-aligned -> (owner, view)."""
    owner = torch.empty(nbytes + align, dtype=torch.uint8, device=device)
    off = (-owner.data_ptr()) % align
    return owner, owner[off: off + nbytes]


class Mxfp4Experts:
    def __init__(self, w13: torch.Tensor, w13_sf: torch.Tensor, w2: torch.Tensor, w2_sf: torch.Tensor, *,
                 num_local: int, expert_base: int, hidden: int, inter: int):
        self.num_local, self.expert_base, self.hidden, self.inter = num_local, expert_base, hidden, inter
        P, H, I = num_local, hidden, inter
        expect = {"w13": P * 2 * I * H // 2, "w13_sf": P * 2 * I * H // 32, "w2": P * H * I // 2,
                  "w2_sf": P * H * I // 32}
        for name, t in (("w13", w13), ("w13_sf", w13_sf), ("w2", w2), ("w2_sf", w2_sf)):
            if t.dtype != torch.uint8 or not t.is_cuda or not t.is_contiguous() or t.numel() != expect[name]:
                raise ValueError(f"{name}: need a contiguous CUDA uint8 tensor of {expect[name]} bytes")
        self.w13, self.w13_sf, self.w2, self.w2_sf = w13, w13_sf, w2, w2_sf
        desc = N.Mxfp4Experts_t(P, expert_base, H, I, w13.data_ptr(), w13_sf.data_ptr(), w2.data_ptr(),
                                w2_sf.data_ptr())
        h = ctypes.c_uint64()
        N.call("asap_experts_register", ctypes.byref(desc), ctypes.byref(h))
        self.handle = h.value

    @property
    def nbytes(self) -> int:
        return sum(t.numel() for t in (self.w13, self.w13_sf, self.w2, self.w2_sf))

    def release(self) -> None:
        if self.handle:
            N.call("asap_experts_release", self.handle)
            self.handle = 0

    @classmethod
    def random(cls, num_local: int, hidden: int, inter: int, *, expert_base: int = 0, device="cuda",
               seed: int = 0, scale_lo: int = 118, scale_hi: int = 121) -> "Mxfp4Experts":
        """Uniform random E2M1 codes and E8M0 scales in [scale_lo, scale_hi] (2^-9 .. 2^-6 with the defaults),
        generated on the device.  Any arrangement of uniform random bytes is uniform, so no packing is needed."""
        P, H, I = num_local, hidden, inter
        gen = torch.Generator(device=device).manual_seed(seed)

        def rnd(n, lo, hi):
            owner, view = _aligned_empty(n, device)
            view.copy_(torch.randint(lo, hi + 1, (n,), dtype=torch.uint8, device=device, generator=gen))
            return view

        w13 = rnd(P * 2 * I * H // 2, 0, 255)
        w13_sf = rnd(P * 2 * I * H // 32, scale_lo, scale_hi)
        w2 = rnd(P * H * I // 2, 0, 255)
        w2_sf = rnd(P * H * I // 32, scale_lo, scale_hi)
        return cls(w13, w13_sf, w2, w2_sf, num_local=P, expert_base=expert_base, hidden=H, inter=I)

    @classmethod
    def from_logical(cls, w13_codes: np.ndarray, w13_scales: np.ndarray, w2_codes: np.ndarray,
                     w2_scales: np.ndarray, *, expert_base: int = 0, device="cuda") -> "Mxfp4Experts":
        """w13_codes [P, 2I, H] (rows: I gate then I up), w13_scales [P, 2I, H/32], w2_codes [P, H, I],
        w2_scales [P, H, I/32] -> device layout."""
        P, two_i, H = w13_codes.shape
        I = two_i // 2
        r = np.arange(two_i)
        b, within = r // 256, r % 256
        src_rows = np.where(within < 128, 128 * b + within, I + 128 * b + (within - 128))
        w13_dev = w13_codes[:, src_rows, :]
        s13_dev = w13_scales[:, src_rows, :]
        packed13 = (w13_dev[..., 0::2] | (w13_dev[..., 1::2] << 4)).astype(np.uint8)
        packed2 = (w2_codes[..., 0::2] | (w2_codes[..., 1::2] << 4)).astype(np.uint8)
        atoms13 = np.stack([_kmajor_atoms(s13_dev[e]) for e in range(P)])
        atoms2 = np.stack([_kmajor_atoms(w2_scales[e]) for e in range(P)])

        def dev(a):
            owner, view = _aligned_empty(a.size, device)
            view.copy_(torch.from_numpy(np.ascontiguousarray(a).reshape(-1)))
            return view

        return cls(dev(packed13), dev(atoms13), dev(packed2), dev(atoms2), num_local=P, expert_base=expert_base,
                   hidden=H, inter=I)


class Fp8Experts:
    """FP8 block-scaled routed experts of one layer on one F rank (used with FfnScheduler like Mxfp4Experts)."""

    def __init__(self, w13: torch.Tensor, w13_scale: torch.Tensor, w2: torch.Tensor, w2_scale: torch.Tensor, *,
                 num_local: int, expert_base: int, hidden: int, inter: int):
        self.num_local, self.expert_base, self.hidden, self.inter = num_local, expert_base, hidden, inter
        P, H, I = num_local, hidden, inter
        if H % 256 or I % 128:
            raise ValueError("FP8 experts need hidden % 256 == 0 and inter % 128 == 0")
        w13, w2 = (t.view(torch.uint8) if t.dtype == torch.float8_e4m3fn else t for t in (w13, w2))
        expect = {"w13": (torch.uint8, P * 2 * I * H), "w13_scale": (torch.float32, P * (2 * I // 128) * (H // 128)),
                  "w2": (torch.uint8, P * H * I), "w2_scale": (torch.float32, P * (H // 128) * (I // 128))}
        for name, t in (("w13", w13), ("w13_scale", w13_scale), ("w2", w2), ("w2_scale", w2_scale)):
            dt, n = expect[name]
            if t.dtype != dt or not t.is_cuda or not t.is_contiguous() or t.numel() != n:
                raise ValueError(f"{name}: need a contiguous CUDA {dt} tensor of {n} elements")
        self.w13, self.w13_scale, self.w2, self.w2_scale = w13, w13_scale, w2, w2_scale
        desc = N.Fp8Experts_t(P, expert_base, H, I, w13.data_ptr(), w13_scale.data_ptr(), w2.data_ptr(),
                              w2_scale.data_ptr())
        h = ctypes.c_uint64()
        N.call("asap_experts_register_fp8", ctypes.byref(desc), ctypes.byref(h))
        self.handle = h.value

    kind = "fp8"

    @property
    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.w13, self.w13_scale, self.w2, self.w2_scale))

    def release(self) -> None:
        if self.handle:
            N.call("asap_experts_release", self.handle)
            self.handle = 0

    @classmethod
    def from_float(cls, w13, w2, *, expert_base: int = 0, device="cuda") -> "Fp8Experts":
        """Dense w13 [P, 2I, H] (gate rows then up rows) and w2 [P, H, I] -> block-quantised FP8 on ``device``."""
        from .quant import fp8_block_quantize

        w13 = torch.as_tensor(w13, device=device)
        w2 = torch.as_tensor(w2, device=device)
        P, two_i, H = w13.shape
        q13, s13, q2, s2 = [], [], [], []
        for e in range(P):  # one expert at a time: bounded fp32 temporaries
            a, b = fp8_block_quantize(w13[e])
            c, d = fp8_block_quantize(w2[e])
            q13.append(a), s13.append(b), q2.append(c), s2.append(d)
        return cls(torch.stack(q13).contiguous(), torch.stack(s13).contiguous(), torch.stack(q2).contiguous(),
                   torch.stack(s2).contiguous(), num_local=P, expert_base=expert_base, hidden=H, inter=two_i // 2)

    @classmethod
    def random(cls, num_local: int, hidden: int, inter: int, *, expert_base: int = 0, device="cuda", seed: int = 0,
               std: float = 0.02) -> "Fp8Experts":
        """N(0, std) weights generated on the device, block-quantised one expert at a time."""
        from .quant import fp8_block_quantize

        P, H, I = num_local, hidden, inter
        gen = torch.Generator(device=device).manual_seed(seed)
        w13 = torch.empty(P, 2 * I, H, dtype=torch.uint8, device=device)
        s13 = torch.empty(P, 2 * I // 128, H // 128, dtype=torch.float32, device=device)
        w2 = torch.empty(P, H, I, dtype=torch.uint8, device=device)
        s2 = torch.empty(P, H // 128, I // 128, dtype=torch.float32, device=device)
        for e in range(P):
            w13[e], s13[e] = fp8_block_quantize(torch.randn(2 * I, H, device=device, generator=gen) * std)
            w2[e], s2[e] = fp8_block_quantize(torch.randn(H, I, device=device, generator=gen) * std)
        return cls(w13, s13, w2, s2, num_local=P, expert_base=expert_base, hidden=H, inter=I)


def _kmajor_atoms(sf: np.ndarray) -> np.ndarray:
    """[N, K/32] scale bytes -> atoms [K/128][N/128][512]: byte (r%32)*16 + ((r/32)%4)*4 + kb%4 of atom
    (kb/4, r/128), the order the tcgen05 scale-factor copy (32x128b, 4 warps) reads."""
    n, kblocks = sf.shape
    out = np.zeros(n * kblocks, dtype=np.uint8)
    r, kb = np.meshgrid(np.arange(n), np.arange(kblocks), indexing="ij")
    off = ((kb >> 2) * (n >> 7) + (r >> 7)) * 512 + (r & 31) * 16 + ((r >> 5) & 3) * 4 + (kb & 3)
    out[off] = sf
    return out
