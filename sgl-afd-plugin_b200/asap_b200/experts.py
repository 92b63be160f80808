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

``from_packed`` builds that layout from the checkpoint's tensors stacked per layer ([P, rows, K/2] E2M1 pairs,
[P, rows, K/32] scale bytes, W13 = [W1; W3] as SGLang's loader stacks them; ``asap_b200.ingest`` reads them from
safetensors shards); ``from_logical`` does the same from unpacked codes; ``random`` makes seeded synthetic
weights.

FP8 (``Fp8Experts``): E4M3 weights with one fp32 scale per 128 x 128 block, in the checkpoint's own layout
(include/asap.h, asap_fp8_experts_t): w13 [P, 2I, H] (gate rows then up rows), w13_scale [P, 2I/128, H/128],
w2 [P, H, I], w2_scale [P, H/128, I/128].
"""

from __future__ import annotations

import ctypes

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
    def from_packed(cls, w13: torch.Tensor, w13_scales: torch.Tensor, w2: torch.Tensor, w2_scales: torch.Tensor, *,
                    expert_base: int = 0, device="cuda") -> "Mxfp4Experts":
        """Checkpoint-order tensors -> device layout on ``device``: w13 [P, 2I, H/2] E2M1 pairs (rows: I gate then
        I up), w13_scales [P, 2I, H/32] E8M0 bytes, w2 [P, H, I/2], w2_scales [P, H, I/32].  The repacking runs
        where the inputs are (CPU, or the device for large layers)."""
        d13, s13, d2, s2 = mxfp4_device_layout(w13, w13_scales, w2, w2_scales)
        P, two_i, half_h = w13.shape

        def dev(t):
            owner, view = _aligned_empty(t.numel(), device)
            view.copy_(t.reshape(-1))
            return view

        return cls(dev(d13), dev(s13), dev(d2), dev(s2), num_local=P, expert_base=expert_base, hidden=2 * half_h,
                   inter=two_i // 2)

    @classmethod
    def from_logical(cls, w13_codes: np.ndarray, w13_scales: np.ndarray, w2_codes: np.ndarray,
                     w2_scales: np.ndarray, *, expert_base: int = 0, device="cuda") -> "Mxfp4Experts":
        """w13_codes [P, 2I, H] (rows: I gate then I up), w13_scales [P, 2I, H/32], w2_codes [P, H, I],
        w2_scales [P, H, I/32] -> device layout."""
        def pack(c):
            return torch.from_numpy((c[..., 0::2] | (c[..., 1::2] << 4)).astype(np.uint8))

        return cls.from_packed(pack(w13_codes), torch.from_numpy(np.ascontiguousarray(w13_scales, np.uint8)),
                               pack(w2_codes), torch.from_numpy(np.ascontiguousarray(w2_scales, np.uint8)),
                               expert_base=expert_base, device=device)


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


def _sf_atoms(sf: torch.Tensor) -> torch.Tensor:
    """[P, N, K/32] scale bytes -> [P, K/128 * N/128 * 512] atoms: byte (r%32)*16 + ((r/32)%4)*4 + kb%4 of atom
    (kb/4, r/128), the order the tcgen05 scale-factor copy (32x128b, 4 warps) reads."""
    P, n, kblocks = sf.shape
    r = torch.arange(n, device=sf.device).view(n, 1)
    kb = torch.arange(kblocks, device=sf.device).view(1, kblocks)
    off = ((kb >> 2) * (n >> 7) + (r >> 7)) * 512 + (r & 31) * 16 + ((r >> 5) & 3) * 4 + (kb & 3)
    out = torch.empty(P, n * kblocks, dtype=torch.uint8, device=sf.device)
    out[:, off.reshape(-1)] = sf.reshape(P, -1)
    return out


def w13_device_rows(inter: int, device=None) -> torch.Tensor:
    """Device row r of w13 -> row of the checkpoint's [W1; W3] stack: blocks of 256 device rows hold gate rows
    128b..128b+127 then up rows 128b..128b+127."""
    r = torch.arange(2 * inter, device=device)
    b, within = r // 256, r % 256
    return torch.where(within < 128, 128 * b + within, inter + 128 * b + (within - 128))


def mxfp4_device_layout(w13: torch.Tensor, w13_scales: torch.Tensor, w2: torch.Tensor, w2_scales: torch.Tensor):
    """Checkpoint-order MXFP4 tensors (see Mxfp4Experts.from_packed) -> the four device-layout byte tensors
    (w13 [P, 2I, H/2] in 128-row gate/up blocks, w13 scale atoms, w2 [P, H, I/2], w2 scale atoms), on the inputs'
    device.  Raises ValueError on shapes or dtypes the GEMMs cannot take."""
    w13, w13_scales, w2, w2_scales = (_as_bytes(t) for t in (w13, w13_scales, w2, w2_scales))
    if w13.dim() != 3 or w2.dim() != 3:
        raise ValueError("w13 / w2 must be [P, rows, K/2]")
    P, two_i, half_h = w13.shape
    H, I = 2 * half_h, two_i // 2
    if H % 256 or I % 128 or I < 128:
        raise ValueError(f"MXFP4 experts need hidden % 256 == 0 and inter % 128 == 0 (got H={H}, I={I})")
    want = {"w13_scales": (w13_scales, (P, 2 * I, H // 32)), "w2": (w2, (P, H, I // 2)),
            "w2_scales": (w2_scales, (P, H, I // 32))}
    for name, (t, shape) in want.items():
        if tuple(t.shape) != shape:
            raise ValueError(f"{name}: expected shape {shape}, got {tuple(t.shape)}")
    rows = w13_device_rows(I, w13.device)
    d13 = w13.index_select(1, rows).contiguous()
    s13 = _sf_atoms(w13_scales.index_select(1, rows))
    return d13, s13, w2.contiguous(), _sf_atoms(w2_scales)


def _as_bytes(t: torch.Tensor) -> torch.Tensor:
    """E2M1 pairs / E8M0 scales as stored in checkpoints (uint8, int8, float8_e8m0fnu) -> a uint8 view."""
    t = torch.as_tensor(t)
    if t.dtype == torch.uint8:
        return t
    if t.dtype in (torch.int8,) + _BYTE_FLOATS:
        return t.view(torch.uint8)
    raise ValueError(f"expected a one-byte dtype for MXFP4 codes / scales, got {t.dtype}")


_BYTE_FLOATS = tuple(getattr(torch, n) for n in ("float8_e8m0fnu",) if hasattr(torch, n))
