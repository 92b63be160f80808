"""The oracle's expert math against the reference's own expert backend: golden outputs of FlashInfer's trtllm-gen
MXFP4 MoE (what the reference's F ranks run, srt/layers/quantization/mxfp4_flashinfer_trtllm_moe.py:68-99) on a
seeded DeepSeek-V3-shape case, generated on a B200 by tests/golden/make_flashinfer_golden.py.  The oracle gets the
same inputs (MXFP8 activations by the OCP rule, bf16-rounded routing weights) and must agree within the north-star
tolerance, relative L2 1e-2."""

import json
import pathlib
import sys

import numpy as np
import pytest

from oracle import moe, mx

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))

import make_flashinfer_golden as fg  # noqa: E402

TOL = 1e-2


def load_golden():
    path = GOLDEN / "flashinfer_moe_golden.npz"
    if not path.exists():
        pytest.skip("no FlashInfer golden outputs (tests/golden/make_flashinfer_golden.py writes them on a B200)")
    d = np.load(path)
    return mx.bf16_from_bits(d["out_bits"]), json.loads(str(d["meta"]))


def oracle_reply(c):
    """The oracle over the case, one expert at a time (bounded memory)."""
    y2 = np.zeros((fg.T, fg.K, fg.H), np.float32)
    used = np.zeros((fg.T, fg.K), bool)
    for e in range(fg.E):
        one = {n: c[n][e: e + 1] for n in ("w13", "s13", "w2", "s2")}
        gate, up, w2 = _deq_one(one)
        y, u = moe.ffn_pairs(c["x"], c["ids"], c["w"], gate, up, w2, 0, fg.E, act_quant=True, experts=[e])
        y2[u] = y[u]
        used |= u
    return moe.reduce_pairs(y2, used)


def _deq_one(one):
    def deq(codes, sf):
        vals = mx.e2m1_decode(mx.unpack_nibbles(codes))
        return (vals.reshape(*sf.shape, 32) * mx.e8m0_value(sf)[..., None]).reshape(vals.shape)

    w13 = deq(one["w13"], one["s13"])
    return w13[:, : fg.I], w13[:, fg.I:], deq(one["w2"], one["s2"])


def test_golden_meta():
    got, meta = load_golden()
    assert (meta["T"], meta["E"], meta["K"], meta["H"], meta["I"]) == (fg.T, fg.E, fg.K, fg.H, fg.I)
    assert got.shape == (fg.T, fg.H) and np.isfinite(got).all() and np.abs(got).max() > 0


def test_oracle_matches_flashinfer_backend():
    got, meta = load_golden()
    ref = oracle_reply(fg.case(meta["seed"]))
    err = moe.rel_l2(ref, got)
    assert err < TOL, f"oracle vs FlashInfer trtllm-gen MoE: relative L2 {err:.4g}"
