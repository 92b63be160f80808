"""This build's F-side expert chain against the reference's own expert backend.

The golden outputs (tests/golden/flashinfer_moe_golden.npz) are FlashInfer's trtllm-gen MXFP4 MoE -- the kernel
the reference's F ranks call (srt/layers/quantization/mxfp4_flashinfer_trtllm_moe.py:68-99) -- on a seeded
DeepSeek-V3-shape case.  asap_ffn_job runs the same case through the C ABI (checkpoint-order weights packed by
Mxfp4Experts.from_packed, bf16-rounded routing weights as FlashInfer packs them) and must agree within the
north-star tolerance, relative L2 1e-2.  Where the prebuilt FlashInfer module is present, it is also run live and
must reproduce the stored outputs."""

import json
import pathlib
import sys

import numpy as np
import pytest
import torch

from asap_b200.experts import Mxfp4Experts
from gpu_util import FfnHarness, bf16_tensor_from_np, np_from_bf16
from oracle import moe, mx

pytestmark = pytest.mark.gpu
GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))

import make_flashinfer_golden as fg  # noqa: E402

TOL = 1e-2


def _golden():
    d = np.load(GOLDEN / "flashinfer_moe_golden.npz")
    return d["out_bits"], json.loads(str(d["meta"]))


def test_ffn_chain_matches_flashinfer_backend(cuda_ok):
    bits, meta = _golden()
    c = fg.case(meta["seed"])
    e = Mxfp4Experts.from_packed(*(torch.from_numpy(c[n]) for n in ("w13", "s13", "w2", "s2")), expert_base=0)
    h = FfnHarness(e, n_max=fg.T, topk=fg.K)
    h.run(bf16_tensor_from_np(c["x"]), torch.from_numpy(c["ids"]).cuda(), torch.from_numpy(c["w"]).cuda(), seq=3)
    out = np_from_bf16(h.reply[: fg.T])
    err = moe.rel_l2(out, mx.bf16_from_bits(bits))
    h.release()
    e.release()
    assert err < TOL, f"asap_ffn_job vs FlashInfer trtllm-gen MoE: relative L2 {err:.4g}"


def test_flashinfer_live_reproduces_golden(cuda_ok):
    import flashinfer_ref

    why = flashinfer_ref.available()
    if why:
        pytest.skip(why)
    bits, meta = _golden()
    got = fg.run_flashinfer(fg.case(meta["seed"]))
    err = moe.rel_l2(mx.bf16_from_bits(got), mx.bf16_from_bits(bits))
    assert err < 1e-3, f"FlashInfer now vs stored golden: relative L2 {err:.4g}"
