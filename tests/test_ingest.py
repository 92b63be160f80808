"""F-rank weight ingest on the CPU: which checkpoint tensors a rank reads (the reference's name filters), the
selective safetensors read, and the repacking of one layer's experts into the device layout, checked against the
oracle's dequantisation of that layout and an independent dequantisation of the checkpoint tensors."""

import numpy as np
import pytest
import torch

from asap_b200 import ingest
from asap_b200.experts import mxfp4_device_layout
from oracle import moe, mx

DSV4 = "layers.{l}.ffn.experts.{e}.{p}.{k}"          # DeepSeek-V4 checkpoint names
HF = "model.layers.{l}.mlp.experts.{e}.{p}.{k}"      # Hugging Face names
DSV4_PROJ = {"gate": "w1", "up": "w3", "down": "w2"}
HF_PROJ = {"gate": "gate_proj", "up": "up_proj", "down": "down_proj"}


def test_routed_expert_names():
    """srt/model_loader/weight_utils.py:1-13's examples and the cases around them."""
    assert ingest.routed_expert("layers.3.ffn.experts.17.w1.weight") == (3, 17)
    assert ingest.routed_expert("model.layers.3.mlp.experts.17.gate_proj.weight") == (3, 17)
    assert ingest.routed_expert("layers.3.ffn.shared_experts.w1.weight") is None
    assert ingest.routed_expert("layers.3.attn.wq_a.weight") is None
    assert ingest.routed_expert("embed.weight") is None
    keep = ingest.routed_experts_only(range(16, 32), num_layers=61)
    assert keep("layers.3.ffn.experts.17.w1.weight")
    assert keep("model.layers.60.mlp.experts.31.down_proj.weight_scale_inv")
    assert not keep("layers.3.ffn.experts.5.w1.weight")         # another rank's expert
    assert not keep("layers.3.ffn.experts.32.w1.weight")
    assert not keep("layers.61.ffn.experts.17.w1.weight")       # MTP layer
    assert not keep("layers.3.ffn.shared_experts.w1.weight")
    assert not keep("layers.3.attn.wq_a.weight")
    for name in ("layers.3.ffn.experts.17.w1.weight", "layers.3.ffn.shared_experts.w1.weight", "norm.weight"):
        assert ingest.skip_routed_experts(name) == (ingest.routed_expert(name) is None)


def test_read_tensors_selective(tmp_path):
    from safetensors.torch import save_file

    g = torch.Generator().manual_seed(0)
    tensors = {
        "layers.0.ffn.experts.0.w1.weight": torch.randint(0, 255, (4, 8), dtype=torch.uint8, generator=g),
        "layers.0.ffn.experts.1.w1.weight": torch.randint(0, 255, (4, 8), dtype=torch.uint8, generator=g),
        "layers.0.ffn.shared_experts.w1.weight": torch.randn(4, 8, generator=g),
        "layers.1.attn.wq_a.weight": torch.randn(4, 8, generator=g),
        "layers.2.ffn.experts.1.w2.scale": torch.randint(0, 255, (4, 2), dtype=torch.uint8, generator=g),
    }
    a, b = str(tmp_path / "a.safetensors"), str(tmp_path / "b.safetensors")
    save_file({k: v for i, (k, v) in enumerate(tensors.items()) if i % 2 == 0}, a)
    save_file({k: v for i, (k, v) in enumerate(tensors.items()) if i % 2 == 1}, b)
    got = dict(ingest.read_tensors([a, b], ingest.routed_experts_only(range(1, 2), num_layers=2)))
    assert set(got) == {"layers.0.ffn.experts.1.w1.weight"}
    assert torch.equal(got["layers.0.ffn.experts.1.w1.weight"], tensors["layers.0.ffn.experts.1.w1.weight"])
    rest = dict(ingest.read_tensors([a, b], ingest.skip_routed_experts))
    assert set(rest) == {"layers.0.ffn.shared_experts.w1.weight", "layers.1.attn.wq_a.weight"}


def _mxfp4_checkpoint(rng, experts, layer, H, I, names, proj):
    """Per-expert MXFP4 checkpoint tensors (some int8 weights, some float8_e8m0fnu scales) and their logical
    codes / scale bytes."""
    items, logical = [], {}
    for e in experts:
        for p, (rows, k) in (("gate", (I, H)), ("up", (I, H)), ("down", (H, I))):
            codes = rng.integers(0, 16, (rows, k)).astype(np.uint8)
            scales = rng.integers(118, 124, (rows, k // 32)).astype(np.uint8)
            w = torch.from_numpy(mx.pack_nibbles(codes))
            s = torch.from_numpy(scales)
            if (e + len(p)) % 2:
                w = w.view(torch.int8)
            if (e + len(p)) % 3 == 0 and hasattr(torch, "float8_e8m0fnu"):
                s = s.view(torch.float8_e8m0fnu)
            items.append((names.format(l=layer, e=e, p=proj[p], k="weight"), w))
            items.append((names.format(l=layer, e=e, p=proj[p], k="scale"), s))
            logical[e, p] = mx.e2m1_decode(codes) * np.repeat(mx.e8m0_value(scales), 32, axis=-1)
    return items, logical


@pytest.mark.parametrize("names,proj", [(DSV4, DSV4_PROJ), (HF, HF_PROJ)])
def test_mxfp4_layer_matches_oracle(names, proj):
    rng = np.random.default_rng(3)
    H, I, layer = 256, 128, 2
    experts = range(4, 7)
    items, logical = _mxfp4_checkpoint(rng, experts, layer, H, I, names, proj)
    other, _ = _mxfp4_checkpoint(rng, [2, 7], layer, H, I, names, proj)  # another rank's experts
    shifted, _ = _mxfp4_checkpoint(rng, experts, layer + 1, H, I, names, proj)  # the next layer
    collected = ingest.collect_layer(items + other + shifted, layer, experts)
    assert sorted(collected) == list(experts)
    kind, w13, s13, w2, s2 = ingest.layer_tensors(collected, experts)
    assert kind == "mxfp4"
    d13, a13, d2, a2 = mxfp4_device_layout(w13, s13, w2, s2)
    P = len(experts)
    gate, up = moe.dequant_w13(d13.numpy(), a13.numpy(), P, H, I)
    down = moe.dequant_w2(d2.numpy(), a2.numpy(), P, H, I)
    for i, e in enumerate(experts):
        np.testing.assert_array_equal(gate[i], logical[e, "gate"])
        np.testing.assert_array_equal(up[i], logical[e, "up"])
        np.testing.assert_array_equal(down[i], logical[e, "down"])


def test_fp8_layer_matches_oracle():
    g = torch.Generator().manual_seed(5)
    H, I, layer = 256, 256, 0
    experts = range(0, 2)
    items, dense = [], {}
    for e in experts:
        for p, (rows, k) in (("gate", (I, H)), ("up", (I, H)), ("down", (H, I))):
            q = (torch.randn(rows, k, generator=g) * 100).clamp(-448, 448).to(torch.float8_e4m3fn)
            s = torch.rand(rows // 128, k // 128, generator=g) * 1e-3 + 1e-4
            items.append((HF.format(l=layer, e=e, p=HF_PROJ[p], k="weight"), q))
            items.append((HF.format(l=layer, e=e, p=HF_PROJ[p], k="weight_scale_inv"), s))
            dense[e, p] = (q.float() * s.repeat_interleave(128, 0).repeat_interleave(128, 1)).numpy()
    kind, w13, s13, w2, s2 = ingest.layer_tensors(ingest.collect_layer(items, layer, experts), experts)
    assert kind == "fp8" and w13.dtype == torch.float8_e4m3fn and s13.dtype == torch.float32
    gate, up, down = moe.dequant_fp8(w13.view(torch.uint8).numpy(), s13.numpy(), w2.view(torch.uint8).numpy(),
                                     s2.numpy())
    for i, e in enumerate(experts):
        np.testing.assert_allclose(gate[i], dense[e, "gate"], rtol=1e-6)
        np.testing.assert_allclose(up[i], dense[e, "up"], rtol=1e-6)
        np.testing.assert_allclose(down[i], dense[e, "down"], rtol=1e-6)


def test_ingest_errors():
    rng = np.random.default_rng(1)
    H, I = 256, 128
    items, _ = _mxfp4_checkpoint(rng, [0, 1], 0, H, I, DSV4, DSV4_PROJ)
    collected = ingest.collect_layer(items, 0, range(0, 3))
    with pytest.raises(ValueError, match="missing"):
        ingest.layer_tensors(collected, range(0, 3))
    del collected[1]["down"]["scale"]
    with pytest.raises(ValueError, match="no down scale"):
        ingest.layer_tensors(collected, range(0, 2))
    with pytest.raises(ValueError, match="two w1 weight"):
        ingest.collect_layer(items + items[:1], 0, range(0, 2))
    bad = torch.zeros(1, 2 * 96, H // 2, dtype=torch.uint8)  # inter 96: not a multiple of 128
    with pytest.raises(ValueError, match="inter % 128"):
        mxfp4_device_layout(bad, torch.zeros(1, 192, H // 32, dtype=torch.uint8),
                            torch.zeros(1, H, 48, dtype=torch.uint8), torch.zeros(1, H, 3, dtype=torch.uint8))
    with pytest.raises(ValueError, match="one-byte dtype"):
        mxfp4_device_layout(torch.zeros(1, 256, H // 2), torch.zeros(1, 256, H // 32, dtype=torch.uint8),
                            torch.zeros(1, H, 64, dtype=torch.uint8), torch.zeros(1, H, 4, dtype=torch.uint8))
    with pytest.raises(ValueError, match="not a decoder layer"):
        ingest.load_layer([], 61, range(0, 2), num_layers=61, device="cpu")


def test_ingest_shape_checks():
    rng = np.random.default_rng(2)
    H, I = 256, 128
    items, _ = _mxfp4_checkpoint(rng, [0, 1], 0, H, I, DSV4, DSV4_PROJ)
    collected = ingest.collect_layer(items, 0, range(0, 2))
    with pytest.raises(ValueError, match="no experts"):
        ingest.layer_tensors(collected, range(0, 0))
    collected[1]["gate"]["weight"] = collected[1]["gate"]["weight"][:64]
    with pytest.raises(ValueError, match="differ in shape across experts"):
        ingest.layer_tensors(collected, range(0, 2))
    collected = ingest.collect_layer(items, 0, range(0, 2))
    collected[0]["up"]["weight"] = collected[0]["up"]["weight"][:, :64]
    collected[1]["up"]["weight"] = collected[1]["up"]["weight"][:, :64]
    with pytest.raises(ValueError, match="gate and up weight shapes differ"):
        ingest.layer_tensors(collected, range(0, 2))
