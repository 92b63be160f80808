"""Shared helpers of the GPU parity tests (not a test module)."""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from asap_b200 import _native as N
from asap_b200.experts import Mxfp4Experts, _aligned_empty
from asap_b200.transport.server import _raw_bytes
from oracle import moe, mx


def bf16_tensor_from_np(a: np.ndarray, device="cuda") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(device).to(torch.bfloat16)


def np_from_bf16(t: torch.Tensor) -> np.ndarray:
    return t.float().cpu().numpy()


def device_bytes(ptr: int, nbytes: int) -> np.ndarray:
    return _raw_bytes(ptr, nbytes, torch.cuda.current_device()).cpu().numpy()


def experts_to_oracle(e):
    """Dequantised (gate, up, w2) of device-layout experts (MXFP4 or FP8 block-scaled), read back from the GPU."""
    if getattr(e, "kind", "mxfp4") == "fp8":
        return moe.dequant_fp8(e.w13.cpu().numpy(), e.w13_scale.cpu().numpy(), e.w2.cpu().numpy(),
                               e.w2_scale.cpu().numpy())
    P, H, I = e.num_local, e.hidden, e.inter
    gate, up = moe.dequant_w13(e.w13.cpu().numpy(), e.w13_sf.cpu().numpy(), P, H, I)
    w2 = moe.dequant_w2(e.w2.cpu().numpy(), e.w2_sf.cpu().numpy(), P, H, I)
    return gate, up, w2


class FfnHarness:
    """The F chain through the C ABI on plain torch buffers: x/ids/w as a RecvArena row, a reply segment and a
    done flag as an A rank's ResultArena would hold them."""

    def __init__(self, experts: Mxfp4Experts, n_max: int, topk: int):
        self.e, self.n_max, self.topk = experts, n_max, topk
        nbytes = N.lib().asap_ffn_ws_bytes(n_max, topk, experts.num_local, experts.hidden, experts.inter)
        self._owner, self.ws = _aligned_empty(nbytes, "cuda")
        h = ctypes.c_uint64()
        N.call("asap_ffn_ws_register", self.ws.data_ptr(), n_max, topk, experts.num_local, experts.hidden,
               experts.inter, ctypes.byref(h))
        self.handle = h.value
        self.status = torch.zeros(1, dtype=torch.int64, device="cuda")
        self.reply = torch.zeros(n_max, experts.hidden, dtype=torch.bfloat16, device="cuda")
        self.done = torch.zeros(16, dtype=torch.int32, device="cuda")
        vals = [ctypes.c_uint64() for _ in range(7)]
        N.call("asap_ffn_debug_ptrs", self.handle, *[ctypes.byref(v) for v in vals])
        self.ptrs = dict(zip(("ecnt", "pair_pos", "xq", "xq_sf", "hq", "hq_sf", "y2"), [v.value for v in vals]))

    def run(self, x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor, seq: int = 7, layer: int = 3,
            swiglu_limit: float = 0.0, timeout_s: float = 5.0):
        n = x.shape[0]
        stream = torch.cuda.current_stream().cuda_stream
        N.call("asap_ffn_post", self.handle, seq, n, layer, 1, ctypes.c_void_p(stream))
        N.call("asap_ffn_job", self.e.handle, self.handle, x.data_ptr(), ids.data_ptr(), w.data_ptr(),
               self.reply.data_ptr(), self.done.data_ptr(), ctypes.c_float(swiglu_limit), self.status.data_ptr(),
               int(timeout_s * 1e9), ctypes.c_void_p(stream))
        torch.cuda.synchronize()
        st = int(self.status.item())
        assert st == 0, N.decode_status(st)

    def release(self):
        N.call("asap_ffn_ws_release", self.handle)


def random_inputs(rng, n, H, k, e_lo, e_hi, *, bias_expert=None):
    x = mx.bf16_round(rng.standard_normal((n, H)).astype(np.float32))
    ids = np.stack([rng.permutation(np.arange(e_lo, e_hi))[:k] for _ in range(n)]).astype(np.int32)
    if bias_expert is not None:
        ids[: n // 2, 0] = bias_expert
        for t in range(n // 2):  # keep the row's ids distinct
            row = ids[t]
            dup = np.nonzero(row[1:] == bias_expert)[0]
            for d in dup:
                row[1 + d] = e_hi - 1 if bias_expert != e_hi - 1 else e_lo
    w = rng.random((n, k)).astype(np.float32)
    w /= w.sum(1, keepdims=True)
    return x, ids, w
