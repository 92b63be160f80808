"""The few SGLang types the dispatcher and MoE layer are written against, for use without SGLang.

When ``sglang`` is importable its own classes are used (the drop-in case); otherwise these stand-ins with the
same names and fields are: ``BaseDispatcher`` (pre-combine hooks), ``StandardTopKOutput`` /
``TopKOutputChecker`` (sglang.srt.layers.moe.topk), ``MoeRunnerConfig`` (sglang.srt.layers.moe.moe_runner.base)
and ``get_parallel`` (sglang.srt.runtime_context: this rank's attention DP and TP ranks; the stand-in reads
ASAP_DP_RANK / ASAP_TP_RANK, 0 when unset).
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Any, Callable, List, NamedTuple, Optional

try:  # pragma: no cover - exercised only where SGLang is installed
    from sglang.srt.layers.moe.moe_runner.base import MoeRunnerConfig  # type: ignore
    from sglang.srt.layers.moe.token_dispatcher.base import BaseDispatcher  # type: ignore
    from sglang.srt.layers.moe.topk import StandardTopKOutput, TopKOutput, TopKOutputChecker  # type: ignore
    from sglang.srt.runtime_context import get_parallel  # type: ignore

    HAVE_SGLANG = True
except Exception:  # noqa: BLE001
    HAVE_SGLANG = False

    class StandardTopKOutput(NamedTuple):
        topk_weights: Any
        topk_ids: Any
        router_logits: Any = None

    TopKOutput = StandardTopKOutput

    class TopKOutputChecker:
        @staticmethod
        def format_is_standard(topk_output) -> bool:
            return isinstance(topk_output, StandardTopKOutput)

    class _HookHandle:
        def __init__(self, hooks: List[Callable], hook: Callable):
            self._hooks, self._hook = hooks, hook

        def remove(self) -> None:
            if self._hook in self._hooks:
                self._hooks.remove(self._hook)

    class BaseDispatcher:
        """Holds pre-combine hooks ``hook(dispatcher, combine_input)``; subclasses call
        ``_run_pre_combine_hooks`` at the start of combine()."""

        def __init__(self):
            self._pre_combine_hooks: List[Callable] = []

        def register_pre_combine_hook(self, hook: Callable) -> _HookHandle:
            self._pre_combine_hooks.append(hook)
            return _HookHandle(self._pre_combine_hooks, hook)

        def _run_pre_combine_hooks(self, combine_input) -> None:
            for hook in list(self._pre_combine_hooks):
                hook(self, combine_input)

    @dataclass
    class MoeRunnerConfig:
        num_experts: Optional[int] = None
        num_local_experts: Optional[int] = None
        hidden_size: Optional[int] = None
        intermediate_size_per_partition: Optional[int] = None
        layer_id: Optional[int] = None
        top_k: Optional[int] = None
        params_dtype: Any = None
        inplace: bool = False
        routed_scaling_factor: Optional[float] = None
        activation: str = "silu"

    class ParallelRanks(NamedTuple):
        dp_rank: Optional[int]
        tp_rank: int

    def get_parallel() -> ParallelRanks:
        """This process's attention data-parallel and tensor-parallel ranks."""
        return ParallelRanks(int(os.environ.get("ASAP_DP_RANK", "0")), int(os.environ.get("ASAP_TP_RANK", "0")))
