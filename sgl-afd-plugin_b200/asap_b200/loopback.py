"""One GPU holding one A rank and one or more F ranks: the 1-GPU deployment of the round trip.

The A side and the F side use the same transport as across GPUs -- the dispatch kernels store into the F
rank's RecvArena and ring its doorbell page, the F chain starts with the device-side doorbell wait and stores
its reply rows and done flag into the A rank's ResultArena, and the combine kernel checks the done flags -- but
kernels of one GPU never spin on each other: the F chain runs on its own stream after an event recorded behind
the dispatch, and the combine waits for an event recorded behind the F chain.  Every device wait therefore
finds its flag already set.
"""

from __future__ import annotations

import tempfile
from typing import Dict, List, Optional, Union

import torch

from .dispatcher import AsapBuffer
from .experts import Mxfp4Experts
from .scheduler import FfnScheduler
from .transport.channel import AttnChannel
from .transport.layout import Geometry
from .transport.server import FfnServer


class LocalFfn:
    """The F ranks of a loopback deployment, driven from the A rank's send/recv calls; their jobs run one after
    the other on one stream.  That stream has the highest priority: the F chain is the critical path of the step,
    so its kernels take SMs ahead of A-side work queued beside them (the shared expert)."""

    def __init__(self, schedulers: List[FfnScheduler], a: int, slots: int, device: int, graphs: bool = False,
                 priority: int = -1):
        self.scheds, self.a, self.device, self.graphs = schedulers, a, device, graphs
        self.stream = torch.cuda.Stream(device, priority=priority)
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
        for sched in self.scheds:
            if self.graphs:  # one CUDA-graph replay per F rank
                sched.run_graph([(self.a, s, ticket.seq)], ticket.layer_id, self.stream.cuda_stream)
            else:
                sched.run_device_wait(self.a, s, ticket.seq, ticket.layer_id, self.stream.cuda_stream)
        self.done[s].record(self.stream)

    def before_combine(self, ticket, stream: torch.cuda.Stream) -> None:
        stream.wait_event(self.done[ticket.slot])


class Loopback:
    """One A rank and ``num_f`` F ranks on ``device``.  ``experts``: for one F rank, ``{layer_id: Mxfp4Experts}``;
    for several, a list of such dicts, F rank f owning its experts' [expert_base, expert_base + num_local) --
    contiguous, in F order, possibly uneven (the 2A6F split 43/43/43/43/42/42).  ``graphs``: every F job is one
    replay of a CUDA graph of its chain (FfnScheduler.run_graph)."""

    def __init__(self, geometry: Geometry, experts: Union[Dict[int, Mxfp4Experts], List[Dict[int, Mxfp4Experts]]],
                 *, device: int = 0, timeout_s: float = 10.0, swiglu_limit: float = 0.0,
                 run_dir: Optional[str] = None, timing: bool = False, graphs: bool = False, ffn_priority: int = -1):
        per_f = [experts] if isinstance(experts, dict) else list(experts)
        if geometry.num_a != 1 or geometry.group != 1 or geometry.num_f != len(per_f):
            raise ValueError("a loopback deployment is one A rank (num_a = group = 1) and num_f F ranks, one experts "
                             "dict per F rank")
        firsts = [next(iter(d.values())) for d in per_f]
        bounds = [firsts[0].expert_base]
        for f, e in enumerate(firsts):
            if e.expert_base != bounds[-1]:
                raise ValueError(f"F rank {f}'s experts start at {e.expert_base}, expected {bounds[-1]} (contiguous)")
            bounds.append(e.expert_base + e.num_local)
        self.g, self.device, self.expert_bounds = geometry, device, bounds
        self.n_experts = bounds[-1] - bounds[0]
        run_dir = run_dir or ("/dev/shm" if _writable("/dev/shm") else tempfile.gettempdir())
        self.servers = [FfnServer(f, geometry, device=device, run_dir=run_dir, listen=False).start()
                        for f in range(len(per_f))]
        self.server = self.servers[0]
        self.channel = AttnChannel(0, geometry, [("in-process", f) for f in range(len(per_f))], device=device,
                                   timeout_s=timeout_s, expert_bounds=bounds,
                                   _connector=lambda f, hello: self.servers[f].handshake(hello)).connect()
        self.scheds = [FfnScheduler(srv, d, swiglu_limit=swiglu_limit, timeout_s=timeout_s, timing=timing)
                       for srv, d in zip(self.servers, per_f)]
        self.sched = self.scheds[0]
        self.local = LocalFfn(self.scheds, 0, geometry.slots, device, graphs=graphs, priority=ffn_priority)
        self.buffer = AsapBuffer(self.channel, device, local_ffn=self.local)

    def install(self) -> AsapBuffer:
        """Make this deployment's buffer the process's AsapBuffer (what AsapDispatcher uses)."""
        return AsapBuffer.install(self.buffer)

    def check(self) -> None:
        self.channel.check()
        for sched in self.scheds:
            sched.check()

    def close(self) -> None:
        torch.cuda.synchronize(self.device)
        if AsapBuffer._buffer is self.buffer:
            AsapBuffer.install(None)
        for sched in self.scheds:
            sched.close()
        self.channel.close()
        for srv in self.servers:
            srv.close()


def _writable(path: str) -> bool:
    import os

    return os.path.isdir(path) and os.access(path, os.W_OK)
