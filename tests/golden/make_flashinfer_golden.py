"""Generate tests/golden/flashinfer_moe_golden.npz: the reference's expert backend (FlashInfer's trtllm-gen MXFP4
MoE, flashinfer_ref.py) run on a small seeded case, as golden outputs for the F-side expert math.

    python tests/golden/make_flashinfer_golden.py --out tests/golden/flashinfer_moe_golden.npz   (on a B200)

The case has the DeepSeek-V3 expert shape (hidden 7168, intermediate 2048) with 16 experts and top-4 routing over
64 tokens; ``case(seed)`` rebuilds every input from the seed with numpy alone, so the tests regenerate them and only
the outputs are stored.  FlashInfer receives the MXFP8 activation codes of the OCP rule (oracle/mx.py), the same
codes this build's kernels compute, so the comparison isolates the expert GEMMs, the SwiGLU, the intermediate
requantisation and the weighted sum; the routing weights are bf16-rounded on both sides (FlashInfer packs them as
bf16).  The generating run also records the relative L2 of the oracle and of FlashInfer's own MXFP8 quantiser
(flashinfer.mxfp8_quantize, when it can be used) for the log.
"""

from __future__ import annotations

import argparse
import json
import pathlib
import sys

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
ROOT = HERE.parent.parent
for p in (str(HERE), str(ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)

SEED, T, E, K, H, I = 0, 64, 16, 4, 7168, 2048


def case(seed: int = SEED):
    """-> dict of numpy inputs: x (bf16 values, fp32) [T, H], ids int32 [T, K], w fp32 [T, K] (bf16 values),
    w13 uint8 [E, 2I, H/2] (E2M1 pairs, rows gate then up), s13 uint8 [E, 2I, H/32] (E8M0), w2 [E, H, I/2],
    s2 [E, H, I/32]."""
    from oracle import moe, mx

    rng = np.random.default_rng(seed)
    x = mx.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
    ids, w = moe.topk_routing(rng.standard_normal((T, E)), K, "softmax")
    w = mx.bf16_round(w)
    return {"x": x, "ids": ids.astype(np.int32), "w": w,
            "w13": rng.integers(0, 256, (E, 2 * I, H // 2), dtype=np.uint8),
            "s13": rng.integers(117, 121, (E, 2 * I, H // 32), dtype=np.uint8),
            "w2": rng.integers(0, 256, (E, H, I // 2), dtype=np.uint8),
            "s2": rng.integers(117, 121, (E, H, I // 32), dtype=np.uint8)}


def oracle_weights(c):
    """Dequantised gate/up/w2 [E, I, H] / [E, I, H] / [E, H, I] fp32 of the case (checkpoint order)."""
    from oracle import mx

    def deq(codes, sf):
        vals = mx.e2m1_decode(mx.unpack_nibbles(codes))
        return (vals.reshape(*sf.shape, 32) * mx.e8m0_value(sf)[..., None]).reshape(vals.shape)

    w13 = np.stack([deq(c["w13"][e], c["s13"][e]) for e in range(E)])
    return w13[:, :I], w13[:, I:], np.stack([deq(c["w2"][e], c["s2"][e]) for e in range(E)])


def run_flashinfer(c):
    import torch

    import flashinfer_ref
    from oracle import mx

    dev = "cuda"
    q, sf = mx.mx_quantize(c["x"])
    weights = flashinfer_ref.weights_for_kernel(*(torch.from_numpy(c[n]).to(dev) for n in ("w13", "s13", "w2", "s2")))
    out = flashinfer_ref.run(torch.from_numpy(q).to(dev).view(torch.float8_e4m3fn), torch.from_numpy(sf).to(dev),
                             torch.from_numpy(c["ids"]).to(dev), torch.from_numpy(c["w"]).to(dev), weights, E, I)
    torch.cuda.synchronize()
    return out.view(torch.int16).cpu().numpy().view(np.uint16)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=str(HERE / "flashinfer_moe_golden.npz"))
    a = ap.parse_args()
    import flashinfer

    from oracle import moe, mx

    c = case()
    bits = run_flashinfer(c)
    got = mx.bf16_from_bits(bits)
    gate, up, w2 = oracle_weights(c)
    ref = moe.ffn_rank(c["x"], c["ids"], c["w"], gate, up, w2, 0, E, act_quant=True)
    plain = moe.ffn_rank(c["x"], c["ids"], c["w"], gate, up, w2, 0, E, act_quant=False)
    meta = {"seed": SEED, "T": T, "E": E, "K": K, "H": H, "I": I, "flashinfer": flashinfer.__version__,
            "rel_l2_oracle_mxfp8": moe.rel_l2(ref, got), "rel_l2_oracle_no_act_quant": moe.rel_l2(plain, got),
            "finite": bool(np.isfinite(got).all())}
    np.savez_compressed(a.out, out_bits=bits, meta=json.dumps(meta))
    print(json.dumps(meta))


if __name__ == "__main__":
    main()
