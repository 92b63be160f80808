"""Token dispatcher of an attention rank whose routed experts run on the FFN ranks.

Same API as the reference's python/sgl_asap_plugin/srt/layers/moe/token_dispatcher/asap.py:
``AsapDispatcher(layer_id).dispatch(hidden_states, topk_output, micro_batch=None) -> AsapDispatchOutput`` and
``.combine(out) -> Tensor`` (asap.py:43-78); ``AsapBuffer.{get, connect, send, recv, exchange, send_stream,
n_max}`` (asap.py:81-206).  dispatch() enqueues libasap's dispatch kernels on the buffer's send stream;
combine() runs the pre-combine hooks (the shared experts, computed while the F ranks work) and enqueues the
combine kernel on the compute stream, which waits for the F ranks' done flags on the device and sums their
partial rows in fp32.  The CPU never waits for the F ranks.
"""

from __future__ import annotations

import logging
from typing import NamedTuple, Optional

import torch

from .sglang_shim import BaseDispatcher, TopKOutputChecker

logger = logging.getLogger(__name__)

SLOT = 0  # the slot of a whole batch; micro-batch i of two-batch overlap uses slot i


class AsapDispatchOutput(NamedTuple):
    ticket: Optional[object]
    hidden_states: Optional[torch.Tensor]
    keepalive: tuple = ()


class AsapDispatcher(BaseDispatcher):
    def __init__(self, layer_id: int):
        super().__init__()
        self.layer_id = layer_id

    def dispatch(self, hidden_states: torch.Tensor, topk_output, micro_batch: Optional[int] = None
                 ) -> AsapDispatchOutput:
        """asap.py:48-73: empty -> empty; non-standard top-k -> RuntimeError; more than n_max tokens -> exchange()
        in pieces; else one send on slot ``micro_batch`` (0 for a whole batch)."""
        if hidden_states.shape[0] == 0:
            return AsapDispatchOutput(None, hidden_states.new_empty(hidden_states.shape))
        if not TopKOutputChecker.format_is_standard(topk_output):
            raise RuntimeError(f"ASAP sends explicit top-k ids and weights, got {type(topk_output).__name__}")
        buffer = AsapBuffer.get()
        ids, weights = topk_output.topk_ids, topk_output.topk_weights
        if hidden_states.shape[0] > buffer.n_max:
            return AsapDispatchOutput(None, buffer.exchange(self.layer_id, hidden_states, ids, weights))
        ticket, keepalive = buffer.send(self.layer_id, hidden_states, ids, weights, micro_batch)
        return AsapDispatchOutput(ticket, None, keepalive)

    def combine(self, combine_input: AsapDispatchOutput, shared: Optional[torch.Tensor] = None) -> torch.Tensor:
        """The routed output (plus ``shared`` when given, fused into the combine kernel)."""
        if hasattr(self, "_run_pre_combine_hooks"):
            self._run_pre_combine_hooks(combine_input)
        if combine_input.hidden_states is not None:
            out = combine_input.hidden_states
            return out if shared is None else out + shared
        return AsapBuffer.get().recv(combine_input.ticket, shared=shared)


class AsapBuffer:
    """The attention rank's channel to the FFN ranks (asap.py:81-206)."""

    _buffer: Optional["AsapBuffer"] = None

    def __init__(self, channel, device: int, local_ffn=None):
        """``local_ffn``: the F side living in this process on this GPU (the 1-GPU deployment); its jobs are
        ordered between send and recv with stream events instead of cross-kernel spins."""
        self.channel, self.device = channel, device
        self.n_max = channel.g.n_max
        self.hidden = channel.g.hidden
        self._send_stream = None
        self.local_ffn = local_ffn

    @property
    def send_stream(self) -> torch.cuda.Stream:
        """The stream every dispatch runs on (made on first use, on this buffer's device)."""
        if self._send_stream is None:
            self._send_stream = torch.cuda.Stream(self.device)
        return self._send_stream

    @classmethod
    def get(cls) -> "AsapBuffer":
        if cls._buffer is None:
            raise RuntimeError("This attention rank is not connected to the FFN ranks")
        return cls._buffer

    @classmethod
    def install(cls, buffer: Optional["AsapBuffer"]) -> Optional["AsapBuffer"]:
        cls._buffer = buffer
        return buffer

    @classmethod
    def connect(cls, model_runner) -> "AsapBuffer":
        """Connect this attention rank to every FFN rank and install the buffer (asap.py:99-147).  Called after
        the model is loaded and before the KV cache is sized, so the ResultArena exists before SGLang hands the
        free memory to the KV pool.

        The geometry comes from the --asap-* flags (``args.transport_geometry``: attention DP x TP ranks, micro-
        batch slots, max dispatch tokens, F ranks) and the model's AsapMoE layers (hidden size, top-k); the F
        endpoints are --asap-bootstrap-addr's port + f; the A rank is (base replica + DP rank) x TP size + TP rank;
        the hello carries the model fingerprint the F ranks check.  ASAP_WAITING_TIMEOUT (s, default 60) bounds
        every device wait, ASAP_BOOTSTRAP_TIMEOUT (s, default 1800) the wait for the F ranks to listen."""
        import os

        from .args import bootstrap_endpoints, get_asap_args, transport_geometry
        from .sglang_shim import get_parallel
        from .transport.channel import AttnChannel

        layers = sorted((m for m in model_runner.model.modules()
                         if isinstance(getattr(m, "dispatcher", None), AsapDispatcher)), key=lambda m: m.layer_id)
        if not layers:
            raise RuntimeError("--asap-ffn-size is set, but the model has no AsapMoE layer")
        args, parallel = get_asap_args(), get_parallel()
        if args.asap_ffn_size is None or args.asap_attn_dp_size is None or args.asap_attn_tp_size is None:
            raise RuntimeError("AsapBuffer.connect needs --asap-ffn-size, --asap-attn-dp-size and --asap-attn-tp-size")
        # the global replica number: other attention instances may share the F ranks
        replica = args.asap_attn_base_replica + (parallel.dp_rank or 0)
        rank = replica * args.asap_attn_tp_size + parallel.tp_rank
        first = layers[0]
        model = {"hidden": first.hidden_size, "topk": first.top_k, "n_experts": first.num_experts,
                 "moe_layers": [m.layer_id for m in layers]}
        channel = AttnChannel(rank, transport_geometry(args, model["hidden"], model["topk"]),
                              bootstrap_endpoints(args), device=model_runner.gpu_id, memory=args.asap_transport_mem,
                              hello={"model": model},
                              timeout_s=float(os.environ.get("ASAP_WAITING_TIMEOUT", "60")),
                              connect_timeout_s=float(os.environ.get("ASAP_BOOTSTRAP_TIMEOUT", "1800"))).connect()
        buffer = cls.install(cls(channel, model_runner.gpu_id))
        served = [{k: answer.get(k) for k in ("f", "experts", "quant_method")} for answer in channel.replies]
        logger.info(f"[ASAP] attention rank {rank} connected to {len(served)} FFN ranks over {channel.mem.kind} "
                    f"memory ({channel.mem.reason}): {served}")
        return buffer

    @classmethod
    def attach(cls, channel, device: int, local_ffn=None) -> "AsapBuffer":
        """Install a buffer over an existing AttnChannel (connecting it first if needed): deployments that build
        the channel themselves (benchmarks, one-GPU loopback, tests)."""
        if channel.result_base is None:
            channel.connect()
        return cls.install(cls(channel, device, local_ffn))

    def send(self, layer_id: int, x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor, micro_batch=None):
        """Enqueue one message on the send stream, after the work that produced its input -> (ticket, the tensors
        the dispatch kernels read; keep them until the answer)."""
        if x.dtype != torch.bfloat16:
            raise TypeError(f"ASAP carries bf16 activations, got {x.dtype}")
        if ids.dtype not in (torch.int32, torch.int64):
            ids = ids.to(torch.int32)
        if weights.dtype not in (torch.float32, torch.bfloat16):
            weights = weights.to(torch.float32)
        x, ids, weights = x.contiguous(), ids.contiguous(), weights.contiguous()
        slot = SLOT if micro_batch is None else micro_batch
        self.send_stream.wait_stream(torch.cuda.current_stream(self.device))
        if self.local_ffn is not None:  # same GPU: backpressure by stream order, never by a cross-kernel spin
            self.local_ffn.before_send(slot, self.send_stream)
        ticket = self.channel.send(layer_id, slot, x.data_ptr(), ids.data_ptr(), weights.data_ptr(), x.shape[0],
                                   self.send_stream.cuda_stream, ids_is_int64=ids.dtype == torch.int64,
                                   w_is_bf16=weights.dtype == torch.bfloat16)
        if self.local_ffn is not None:
            self.local_ffn.serve(ticket, self.send_stream)
        return ticket, (x, ids, weights)

    def recv(self, ticket, shared: Optional[torch.Tensor] = None) -> torch.Tensor:
        """The sum of the FFN ranks' partial outputs (+ shared), as a new tensor."""
        stream = torch.cuda.current_stream(self.device)
        if self.local_ffn is not None:
            self.local_ffn.before_combine(ticket, stream)
        out = torch.empty(ticket.n_tokens, self.hidden, dtype=torch.bfloat16, device=f"cuda:{self.device}")
        sp = 0
        if shared is not None:
            if shared.dtype != torch.bfloat16 or shared.shape != out.shape:
                raise TypeError("shared must be bf16 [n_tokens, hidden]")
            shared = shared.contiguous()
            sp = shared.data_ptr()
        self.channel.combine(ticket, out.data_ptr(), stream.cuda_stream, sp)
        return out

    def exchange(self, layer_id: int, x, ids, weights) -> torch.Tensor:
        """send + recv in pieces of at most n_max tokens (asap.py:186-193)."""
        pieces = []
        for i in range(0, x.shape[0], self.n_max):
            end = i + self.n_max
            ticket, _ = self.send(layer_id, x[i:end], ids[i:end], weights[i:end])
            pieces.append(self.recv(ticket))
        return torch.cat(pieces)
