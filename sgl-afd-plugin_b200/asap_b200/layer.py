"""The MoE layer of an attention rank whose routed experts run on the FFN ranks.

Same API as the reference's python/sgl_asap_plugin/srt/layers/moe/ep_moe/layer.py: ``get_moe_impl_class``
returns ``AsapMoE``, a FusedMoE stand-in without expert weights whose forward hands the routed experts to the
FFN ranks through ``AsapDispatcher``.  ``should_fuse_routed_scaling_factor_in_topk`` is True (the weights on the
wire already include the routed scale) and ``quant_method`` is None (layer.py:36-81).
"""

from __future__ import annotations

from typing import Optional

import torch

from .dispatcher import AsapDispatcher
from .sglang_shim import MoeRunnerConfig


def get_moe_impl_class(quant_config=None, *, context=None):
    """REPLACE of sglang.srt.layers.moe.ep_moe.layer.get_moe_impl_class (layer.py:19-21)."""
    return AsapMoE


class AsapMoE(torch.nn.Module):
    should_fuse_routed_scaling_factor_in_topk = True
    quant_method = None

    def __init__(self, num_experts: int, hidden_size: int, intermediate_size: int, layer_id: int,
                 top_k: Optional[int] = None, num_fused_shared_experts: int = 0,
                 params_dtype: Optional[torch.dtype] = None, routed_scaling_factor: Optional[float] = None, **kwargs):
        super().__init__()
        if num_fused_shared_experts:
            raise ValueError("ASAP keeps the shared experts on the attention ranks: disable shared experts fusion")
        self.num_experts = num_experts
        self.num_local_experts = 0
        self.num_fused_shared_experts = 0
        self.top_k = top_k
        self.hidden_size = hidden_size
        self.layer_id = layer_id
        self.moe_runner_config = MoeRunnerConfig(
            num_experts=num_experts, num_local_experts=0, hidden_size=hidden_size,
            intermediate_size_per_partition=intermediate_size, layer_id=layer_id, top_k=top_k,
            params_dtype=params_dtype, inplace=False, routed_scaling_factor=routed_scaling_factor)
        self.dispatcher = AsapDispatcher(layer_id)
        self.shared_experts_overlap = None

    def forward(self, hidden_states: torch.Tensor, topk_output, pre_quant_input=None) -> torch.Tensor:
        overlap = self.shared_experts_overlap
        if overlap is not None and getattr(overlap, "active", False):
            overlap.pre_quant_input = pre_quant_input
        dispatch_output = self.dispatcher.dispatch(hidden_states, topk_output)
        return self.dispatcher.combine(dispatch_output)
