"""A side of the transport: one AttnChannel per A rank, connected to every F rank.

API and protocol are the reference's (python/sgl_asap_plugin/transport/channel.py:186-377: connect, send, wait,
check, close, reconnect; the JSON-line handshake; epochs; a sequence number per slot; backpressure).  The data path
runs on the SMs:

* send() launches the dispatch kernels on the caller's stream (libasap asap_dispatch): a bounded device spin for
  backpressure (channel.py:337-339), the per-F-rank bucketing of the top-k, 16-byte P2P stores of the routed rows
  straight into each F rank's RecvArena, and the 64-bit doorbell released by the last CTA (channel.py:340-355,
  where the reference used three copy-engine copies and a stream memop per F rank).
* combine() launches the combine kernel: a bounded spin on the F done flags (channel.py:364-377) fused with the
  fp32 sum of the partials and the shared-expert add (token_dispatcher/asap.py:174-184).
* A device wait never blocks forever: it gives up after ``timeout_s``, writes a status word into pinned host
  memory and returns.  check() reads that word with a plain load (no sync) and raises ChannelPoisoned, as the
  reference's Watchdog does after it released a parked stream (channel.py:100-167, 301-311).

Connecting is organised per F rank: ``_greet`` runs the handshake with one F rank (TCP through ``wire.exchange``,
or an in-process ``_connector``), ``_FLink`` holds what came back (the mapped RecvArena and doorbell page, the
epoch, the answer), and ``connect`` undoes every finished link when a later one fails.
"""

from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from .. import _native as N
from .layout import PROTO_VERSION, SEQ_MASK, ChannelPoisoned, Geometry, HandshakeError
from .memory import Shared
from .memory import select as select_memory
from .wire import exchange


@dataclass
class Ticket:
    """One message in flight (channel.py:170-180)."""

    slot: int
    seq: int
    layer_id: int
    n_tokens: int
    result_ptrs: List[int] = field(default_factory=list)


@dataclass
class _FLink:
    """This A rank's view of one F rank after the handshake."""

    f: int
    epoch: int
    answer: dict
    recv: Shared   # the F rank's RecvArena, mapped here
    bells: Shared  # its doorbell page, mapped here

    def release(self) -> None:
        self.recv.release()
        self.bells.release()


class AttnChannel:
    """A rank ``a``'s connection to every F rank (``endpoints[f]`` is F rank f's handshake address).

    ``expert_bounds`` (num_f + 1 ints): F rank f owns experts [bounds[f], bounds[f+1]).  Default: the
    reference's contiguous equal split of ``num_experts`` (srt/managers/scheduler.py:206-218), given through
    ``hello["model"]["n_experts"]``.  ``_backpressure`` / ``_epoch_override`` exist only for tests that provoke
    protocol violations (the reference's own hooks, channel.py:198-203); ``_connector(f, hello)`` replaces the TCP
    handshake in one-process deployments."""

    def __init__(self, a: int, geometry: Geometry, endpoints: Sequence[Tuple[str, int]], *, device: int,
                 seq_base: int = 0, timeout_s: float = 60.0, connect_timeout_s: float = 60.0, memory: str = "auto",
                 hello: Optional[dict] = None, expert_bounds: Optional[Sequence[int]] = None,
                 _backpressure: bool = True, _epoch_override: Optional[int] = None, _connector=None):
        if len(endpoints) != geometry.num_f:
            raise ValueError(f"need one endpoint per F rank ({geometry.num_f}), got {len(endpoints)}")
        if not 0 <= a < geometry.num_a:
            raise ValueError(f"A rank {a} is outside [0, {geometry.num_a})")
        if geometry.num_f > N.MAX_F:
            raise ValueError(f"{geometry.num_f} F ranks; this build addresses at most {N.MAX_F}")
        self.a, self.g, self.endpoints, self.seq_base = a, geometry, list(endpoints), seq_base
        self.device, self.timeout_s, self.connect_timeout_s = device, timeout_s, connect_timeout_s
        self.hello = dict(hello or {})
        self._backpressure, self._epoch_override, self._connector = _backpressure, _epoch_override, _connector
        self.memory, self.mem = memory, None
        self.expert_bounds = list(expert_bounds) if expert_bounds is not None else None
        self.links: List[_FLink] = []
        self.status = None
        self._arena: Optional[Shared] = None
        self._route_ws: List[torch.Tensor] = []
        self._last_sent: Dict[int, int] = {}
        self._poison: Optional[ChannelPoisoned] = None

    # ---------------------------------------------------------------- connect / close
    def _split(self) -> List[int]:
        """Expert bounds per F rank: the given ones, or the equal contiguous split of hello.model.n_experts."""
        nf = self.g.num_f
        if self.expert_bounds is not None:
            bounds = list(self.expert_bounds)
        else:
            n_exp = (self.hello.get("model") or {}).get("n_experts")
            if n_exp is None or n_exp % nf:
                raise ValueError("expert_bounds is required unless hello['model']['n_experts'] is a multiple of "
                                 "num_f (the reference's equal contiguous split)")
            bounds = [f * (n_exp // nf) for f in range(nf + 1)]
        if len(bounds) != nf + 1:
            raise ValueError("expert_bounds needs num_f + 1 entries")
        return bounds

    def _greet(self, f: int, hello: dict) -> _FLink:
        """Handshake with F rank f and map what it shares."""
        if self._connector is not None:
            answer = self._connector(f, hello)
        else:
            host, port = self.endpoints[f]
            answer = exchange(host, port, hello, connect_timeout=self.connect_timeout_s)
        if answer["seq_base"] != self.seq_base:
            raise HandshakeError(f"seq_base A={self.seq_base} F={answer['seq_base']}")
        recv = self.mem.open(answer["recv"])
        try:
            bells = self.mem.open_doorbells(answer["doorbells"], self.g.host_bytes)
        except BaseException:
            recv.release()
            raise
        return _FLink(f, int(answer["epoch"]), answer, recv, bells)

    def connect(self) -> "AttnChannel":
        """Allocate the ResultArena (every done flag at seq_base), hand it to every F rank, map their RecvArenas
        and doorbell pages.  On any failure nothing stays allocated or mapped."""
        g = self.g
        if self.mem is None:
            self.mem = select_memory(self.memory, self.device)
        self.mem.activate()
        self.expert_bounds = self._split()
        arena = self.mem.device(g.result_bytes)
        self.mem.fill32(arena.ptr, self.seq_base & SEQ_MASK, g.flags_bytes // 4)
        hello = dict(self.hello)
        hello.update(proto=PROTO_VERSION, a=self.a, geometry=g.as_dict(), pid=os.getpid(), memory=self.mem.kind,
                     peer=self.mem.identity(), result=arena.desc)
        links: List[_FLink] = []
        try:
            for f in range(g.num_f):
                links.append(self._greet(f, hello))
        except BaseException:
            for link in links:
                link.release()
            arena.release()
            raise
        self._arena, self.links = arena, links
        self._last_sent = {}
        self._poison = None
        self.status = self.mem.status_words(1)
        ws_bytes = N.lib().asap_route_ws_bytes(ctypes.byref(N.geometry_struct(g)))
        self._route_ws = [self.mem.workspace(ws_bytes) for _ in range(g.slots)]
        self._gs = N.geometry_struct(g)
        F = g.num_f
        self._c_epochs = (ctypes.c_int32 * F)(*self.epochs)
        self._c_bounds = (ctypes.c_int32 * (F + 1))(*self.expert_bounds)
        self._c_recv = (ctypes.c_uint64 * F)(*self.recv_bases)
        self._c_bells = (ctypes.c_uint64 * F)(*self.bell_bases)
        return self

    def reconnect(self) -> "AttnChannel":
        """The only way out of a poisoned channel: a new epoch and a fresh ResultArena on every F rank."""
        self.close()
        return self.connect()

    @property
    def epochs(self) -> List[int]:
        return [link.epoch for link in self.links]

    @property
    def recv_bases(self) -> List[int]:
        """Device addresses (mapped here) of every F rank's RecvArena."""
        return [link.recv.ptr for link in self.links]

    @property
    def bell_bases(self) -> List[int]:
        """Device addresses (mapped here) of every F rank's doorbell page."""
        return [link.bells.ptr for link in self.links]

    @property
    def replies(self) -> List[dict]:
        """The F ranks' handshake answers (what each one serves, for logs)."""
        return [link.answer for link in self.links]

    def unmap_peers(self) -> None:
        """Unmap every F rank's RecvArena and doorbell page (first step of an orderly multi-process shutdown: every
        process unmaps its peers' memory before any process frees its own)."""
        for link in self.links:
            link.release()

    def close(self) -> None:
        """Release everything. Synchronize the streams that used the channel first."""
        self.unmap_peers()
        self.links = []
        if self._arena is not None:
            self._arena.release()
            self._arena = None
        self._route_ws = []
        if self.status is not None:
            self.status.close()
            self.status = None

    # ---------------------------------------------------------------- failure state
    def check(self) -> None:
        """Raise ChannelPoisoned if a device wait ran out (the reference's watchdog semantics)."""
        if self._poison is None and self.status is not None:
            word = self.status.read()
            if word:
                st = N.decode_status(word)
                self._poison = ChannelPoisoned(
                    f"A rank {self.a}: {st['what']} (F rank {st['f']}, slot {st['slot']}, seq {st['seq']}) did not "
                    f"complete within {self.timeout_s}s, F is dead or stuck; the results of every pending message "
                    "are garbage until reconnect()")
        if self._poison is not None:
            raise self._poison

    @property
    def result_base(self) -> int:
        return self._arena.ptr if self._arena is not None else None

    def route_ws(self, slot: int) -> torch.Tensor:
        return self._route_ws[slot]

    def dispatch_info(self, slot: int, stream: int) -> dict:
        """Rows announced to each F rank by the last dispatch on ``slot``, the device time (globaltimer ns) its
        doorbells were released and the one at which the combine's wait saw every reply (synchronizes
        ``stream``)."""
        counts = (ctypes.c_int32 * self.g.num_f)()
        t, t_back = ctypes.c_uint64(), ctypes.c_uint64()
        N.call("asap_dispatch_info", self._ws_ptr(slot), self.g.num_f, counts, ctypes.byref(t), ctypes.byref(t_back),
               ctypes.c_void_p(stream))
        return {"counts": list(counts), "t_ring_ns": t.value, "t_replies_ns": t_back.value}

    def _ws_ptr(self, slot: int) -> int:
        return self._route_ws[slot].data_ptr()

    # ---------------------------------------------------------------- data path
    def send(self, layer_id: int, slot: int, x_ptr: int, ids_ptr: int, w_ptr: int, n_tokens: int, stream: int, *,
             ids_is_int64: bool = False, w_is_bf16: bool = False) -> Ticket:
        """Enqueue one message on ``stream``: ``n_tokens`` contiguous rows of x (bf16 [n, hidden]), top-k ids
        (int32 or int64 [n, topk]) and top-k weights (fp32 or bf16 [n, topk]) at the given device addresses."""
        self.check()
        g = self.g
        if not (0 <= slot < g.slots and 1 <= n_tokens <= g.n_max):
            raise ValueError(f"slot {slot} / n_tokens {n_tokens} outside the geometry {g}")
        seq = self._last_sent[slot] = (self._last_sent.get(slot, self.seq_base) + 1) & SEQ_MASK
        epochs = self._c_epochs
        if self._epoch_override is not None:
            epochs = (ctypes.c_int32 * g.num_f)(*([self._epoch_override] * g.num_f))
        args = (ctypes.byref(self._gs), self.a, slot, seq, layer_id, epochs, x_ptr, ids_ptr, int(ids_is_int64), w_ptr,
                int(w_is_bf16), n_tokens, self._c_bounds, self._c_recv, self._c_bells, self.result_base,
                self._ws_ptr(slot), int(self._backpressure), self.status.ptr, int(self.timeout_s * 1e9),
                ctypes.c_void_p(stream))
        N.call("asap_dispatch", *args)
        return Ticket(slot, seq, layer_id, n_tokens)

    def wait(self, ticket: Ticket, stream: int) -> List[int]:
        """Enqueue on ``stream`` the bounded wait for every F rank's answer to ``ticket``; returns the A-device
        addresses of the F partial sums (bf16 rows, F rank f's row j answers its region row j)."""
        self.check()
        g = self.g
        base = self.result_base
        N.call("asap_wait_replies", ctypes.byref(self._gs), ticket.slot, ticket.seq, base, self.status.ptr,
               int(self.timeout_s * 1e9), ctypes.c_void_p(stream))
        ticket.result_ptrs = [base + g.seg_off(f, ticket.slot) for f in range(g.num_f)]
        return ticket.result_ptrs

    def combine(self, ticket: Ticket, out_ptr: int, stream: int, shared_ptr: int = 0) -> None:
        """Enqueue the bounded reply wait fused with out = bf16(sum_f partial_f) (+ shared): the A-side combine."""
        self.check()
        N.call("asap_combine", ctypes.byref(self._gs), ticket.slot, ticket.seq, ticket.n_tokens, self.result_base,
               self._ws_ptr(ticket.slot), shared_ptr, out_ptr, self.status.ptr,
               int(self.timeout_s * 1e9), ctypes.c_void_p(stream))


def send_order(a: int, num_a: int, num_f: int) -> List[int]:
    """The F ranks in the order A rank a's dispatch fills them (each F rank's doorbell rings when its rows are
    stored): starting at a * num_f // num_a, so that concurrent A ranks start on different F ranks."""
    off = a * num_f // max(1, num_a)
    return [(off + i) % num_f for i in range(num_f)]


def serve_order(f: int, num_a: int, num_f: int) -> List[int]:
    """The A ranks in the order their messages complete at F rank f (the order a fixed-order F rank should answer
    them)."""
    return sorted(range(num_a), key=lambda a: (send_order(a, num_a, num_f).index(f), a))
