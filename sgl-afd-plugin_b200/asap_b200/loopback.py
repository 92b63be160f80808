"""One GPU holding one A rank and one F rank: the 1-GPU deployment of the round trip.

The A side and the F side use the same transport as across GPUs -- the dispatch kernels store into the F
rank's RecvArena and ring its doorbell page, the F chain starts with the device-side doorbell wait and stores
its reply rows and done flag into the A rank's ResultArena, and the combine kernel checks the done flags -- but
kernels of one GPU never spin on each other: the F chain runs on its own stream after an event recorded behind
the dispatch, and the combine waits for an event recorded behind the F chain.  Every device wait therefore
finds its flag already set.
"""

from __future__ import annotations

import tempfile
from typing import Dict, Optional

import torch

from .dispatcher import AsapBuffer
from .experts import Mxfp4Experts
from .scheduler import FfnScheduler
from .transport.channel import AttnChannel
from .transport.layout import Geometry
from .transport.server import FfnServer


class LocalFfn:
    """The F rank of a loopback pair, driven from the A rank's send/recv calls."""

    def __init__(self, scheduler: FfnScheduler, a: int, slots: int, device: int):
        self.sched, self.a, self.device = scheduler, a, device
        self.stream = torch.cuda.Stream(device)
        self.sent = [torch.cuda.Event() for _ in range(slots)]
        self.done = [torch.cuda.Event() for _ in range(slots)]

    def before_send(self, slot: int, send_stream: torch.cuda.Stream) -> None:
        """The dispatch of a slot's next message waits for the F job of its previous one (an event, so that the
        dispatch kernel's backpressure spin finds the done flag already set)."""
        send_stream.wait_event(self.done[slot])

    def serve(self, ticket, send_stream: torch.cuda.Stream) -> None:
        s = ticket.slot
        self.sent[s].record(send_stream)
        self.stream.wait_event(self.sent[s])
        self.sched.run_device_wait(self.a, s, ticket.seq, ticket.layer_id, self.stream.cuda_stream)
        self.done[s].record(self.stream)

    def before_combine(self, ticket, stream: torch.cuda.Stream) -> None:
        stream.wait_event(self.done[ticket.slot])


class Loopback:
    """A + F on ``device``.  ``experts[layer_id]`` are all routed experts [0, n_experts) of that layer."""

    def __init__(self, geometry: Geometry, experts: Dict[int, Mxfp4Experts], *, device: int = 0,
                 timeout_s: float = 10.0, swiglu_limit: float = 0.0, run_dir: Optional[str] = None,
                 timing: bool = False):
        if geometry.num_a != 1 or geometry.num_f != 1 or geometry.group != 1:
            raise ValueError("a loopback pair is one A rank and one F rank (num_a = num_f = group = 1)")
        first = next(iter(experts.values()))
        self.g, self.device = geometry, device
        self.n_experts = first.num_local
        run_dir = run_dir or ("/dev/shm" if _writable("/dev/shm") else tempfile.gettempdir())
        self.server = FfnServer(0, geometry, device=device, run_dir=run_dir, listen=False).start()
        self.channel = AttnChannel(0, geometry, [("in-process", 0)], device=device, timeout_s=timeout_s,
                                   expert_bounds=[first.expert_base, first.expert_base + first.num_local],
                                   _connector=lambda f, hello: self.server.handshake(hello)).connect()
        self.sched = FfnScheduler(self.server, experts, swiglu_limit=swiglu_limit, timeout_s=timeout_s,
                                  timing=timing)
        self.local = LocalFfn(self.sched, 0, geometry.slots, device)
        self.buffer = AsapBuffer(self.channel, device, local_ffn=self.local)

    def install(self) -> AsapBuffer:
        """Make this pair's buffer the process's AsapBuffer (what AsapDispatcher uses)."""
        return AsapBuffer.install(self.buffer)

    def check(self) -> None:
        self.channel.check()
        self.sched.check()

    def close(self) -> None:
        torch.cuda.synchronize(self.device)
        if AsapBuffer._buffer is self.buffer:
            AsapBuffer.install(None)
        self.sched.close()
        self.channel.close()
        self.server.close()


def _writable(path: str) -> bool:
    import os

    return os.path.isdir(path) and os.access(path, os.W_OK)
