"""Weight ingest on the F rank: read only the routed experts this rank serves from the checkpoint's safetensors
shards, and pack one decoder layer's experts into the device layout of ``Mxfp4Experts`` / ``Fp8Experts``.

Reference behaviour: ``read_routed_experts_only`` / ``skip_routed_experts`` (srt/model_loader/weight_utils.py:
33-53) select tensors by checkpoint name before any byte is read.  A routed expert is ``.experts.<E>.`` in a
name, its decoder layer ``layers.<L>.``.  An FFN rank keeps the experts of its range in layers below
``num_layers`` (an MTP layer's experts are not its), and an attention rank keeps every other tensor.  The F rank's
model then loads them through FusedMoE's expert mapping, gate = ``w1`` / ``gate_proj``, up = ``w3`` /
``up_proj``, down = ``w2`` / ``down_proj`` (srt/models/deepseek_v4.py:126-166).

Tensor formats taken, per expert and projection (``<proj>.weight`` plus one scale tensor ``<proj>.scale``,
``.weight_scale`` or ``.weight_scale_inv``):

  MXFP4  weight uint8 / int8 [rows, K/2], two E2M1 values per byte, low nibble first;
         scale uint8 / float8_e8m0fnu [rows, K/32]
  FP8    weight float8_e4m3fn [rows, K]; scale float32 [rows/128, K/128] (value = e4m3 x scale)

with rows x K = I x H for gate and up, H x I for down.
"""

from __future__ import annotations

import re
from typing import Callable, Dict, Iterable, Iterator, Optional, Sequence, Tuple

import torch

from .experts import Fp8Experts, Mxfp4Experts, _as_bytes

_ROUTED_EXPERT = re.compile(r"\.experts\.(\d+)\.")
_LAYER = re.compile(r"(?:^|\.)layers\.(\d+)\.")
_PROJ = {"w1": "gate", "gate_proj": "gate", "w3": "up", "up_proj": "up", "w2": "down", "down_proj": "down"}
_KIND = {"weight": "weight", "scale": "scale", "weight_scale": "scale", "weight_scale_inv": "scale"}
_PROJ_TENSOR = re.compile(r"\.experts\.\d+\.(w1|w2|w3|gate_proj|up_proj|down_proj)\.(weight|scale|weight_scale|"
                          r"weight_scale_inv)$")


def routed_expert(name: str) -> Optional[Tuple[int, int]]:
    """(decoder layer, expert id) of a routed-expert tensor name, None for any other tensor."""
    e, l = _ROUTED_EXPERT.search(name), _LAYER.search(name)
    if e is None or l is None:
        return None
    return int(l.group(1)), int(e.group(1))


def routed_experts_only(experts: range, num_layers: int) -> Callable[[str], bool]:
    """FFN ranks: the routed experts in ``experts`` of the decoder layers below ``num_layers``, nothing else."""
    def keep(name: str) -> bool:
        le = routed_expert(name)
        return le is not None and le[0] < num_layers and le[1] in experts

    return keep


def skip_routed_experts(name: str) -> bool:
    """Attention ranks: every tensor but the routed experts."""
    return _ROUTED_EXPERT.search(name) is None


def read_tensors(files: Sequence[str], keep: Callable[[str], bool], device: str = "cpu") -> Iterator[
        Tuple[str, torch.Tensor]]:
    """The tensors of the safetensors ``files`` whose names ``keep`` accepts; no other tensor is read."""
    from safetensors import safe_open

    for path in files:
        with safe_open(path, framework="pt", device=device) as f:
            for name in f.keys():
                if keep(name):
                    yield name, f.get_tensor(name)


def collect_layer(tensors: Iterable[Tuple[str, torch.Tensor]], layer: int, experts: range) -> Dict[
        int, Dict[str, Dict[str, torch.Tensor]]]:
    """{expert: {"gate"|"up"|"down": {"weight": t, "scale": t}}} for ``layer``'s experts in ``experts``; tensors
    of other layers / experts and non-projection tensors (e.g. biases) are ignored."""
    out: Dict[int, Dict[str, Dict[str, torch.Tensor]]] = {}
    for name, t in tensors:
        le = routed_expert(name)
        m = _PROJ_TENSOR.search(name)
        if le is None or m is None or le[0] != layer or le[1] not in experts:
            continue
        slot = out.setdefault(le[1], {}).setdefault(_PROJ[m.group(1)], {})
        kind = _KIND[m.group(2)]
        if kind in slot:
            raise ValueError(f"layer {layer} expert {le[1]}: two {m.group(1)} {kind} tensors ({name})")
        slot[kind] = t
    return out


def layer_tensors(collected: Dict[int, Dict[str, Dict[str, torch.Tensor]]], experts: range, *,
                  device: str = "cpu"):
    """One layer's experts (``collect_layer``'s output; every expert of the contiguous ``experts`` range present)
    stacked in checkpoint order on ``device``: ("mxfp4" | "fp8", w13 [P, 2I, .] (gate rows then up rows), w13
    scales, w2, w2 scales)."""
    if len(experts) == 0:
        raise ValueError("no experts to load")
    missing = [e for e in experts if e not in collected]
    if missing:
        raise ValueError(f"experts missing from the checkpoint: {missing[:8]}{'...' if len(missing) > 8 else ''}")

    def part(e: int, proj: str, kind: str) -> torch.Tensor:
        try:
            t = collected[e][proj][kind].to(device)
        except KeyError:
            raise ValueError(f"expert {e}: no {proj} {kind} tensor") from None
        if t.dtype == torch.float8_e4m3fn or (kind == "scale" and t.dtype in (torch.float32, torch.bfloat16,
                                                                              torch.float16)):
            return t
        return _as_bytes(t)  # E2M1 pairs, E8M0 scales: one byte each, whatever dtype the checkpoint used

    parts = {(e, p, k): part(e, p, k) for e in experts for p in ("gate", "up", "down") for k in ("weight", "scale")}
    if len({parts[e, p, "weight"].dtype == torch.float8_e4m3fn for e in experts for p in ("gate", "up", "down")}) != 1:
        raise ValueError("the layer mixes FP8 and MXFP4 expert weights")
    for p in ("gate", "up", "down"):
        for k in ("weight", "scale"):
            shapes = {tuple(parts[e, p, k].shape) for e in experts}
            if len(shapes) != 1:
                raise ValueError(f"{p} {k} tensors differ in shape across experts: {sorted(shapes)}")
    for k in ("weight", "scale"):
        if parts[experts[0], "gate", k].shape != parts[experts[0], "up", k].shape:
            raise ValueError(f"gate and up {k} shapes differ: {tuple(parts[experts[0], 'gate', k].shape)} vs "
                             f"{tuple(parts[experts[0], 'up', k].shape)}")
    w13 = torch.stack([torch.cat([parts[e, "gate", "weight"], parts[e, "up", "weight"]]) for e in experts])
    s13 = torch.stack([torch.cat([parts[e, "gate", "scale"], parts[e, "up", "scale"]]) for e in experts])
    w2 = torch.stack([parts[e, "down", "weight"] for e in experts])
    s2 = torch.stack([parts[e, "down", "scale"] for e in experts])
    if w13.dtype == torch.float8_e4m3fn:
        return "fp8", w13, s13.float(), w2, s2.float()
    return "mxfp4", w13, s13, w2, s2


def layer_experts(collected: Dict[int, Dict[str, Dict[str, torch.Tensor]]], experts: range, *,
                  device: str = "cuda"):
    """``layer_tensors`` registered: ``Mxfp4Experts`` or ``Fp8Experts`` on ``device``, by the weights' dtype."""
    kind, w13, s13, w2, s2 = layer_tensors(collected, experts, device=device)
    if kind == "fp8":
        P, two_i, H = w13.shape
        return Fp8Experts(w13.contiguous(), s13.contiguous(), w2.contiguous(), s2.contiguous(), num_local=P,
                          expert_base=experts[0], hidden=H, inter=two_i // 2)
    return Mxfp4Experts.from_packed(w13, s13, w2, s2, expert_base=experts[0], device=device)


def load_layer(files: Sequence[str], layer: int, experts: range, num_layers: int, *, device: str = "cuda"):
    """Read ``layer``'s routed experts in ``experts`` from the safetensors ``files`` (no other tensor is read)
    and register them: the F rank's ingest of one layer."""
    if layer >= num_layers:
        raise ValueError(f"layer {layer} is not a decoder layer below num_layers={num_layers}")
    keep = routed_experts_only(experts, num_layers)
    return layer_experts(collect_layer(read_tensors(files, lambda n: keep(n) and routed_expert(n)[0] == layer),
                                       layer, experts), experts, device=device)
