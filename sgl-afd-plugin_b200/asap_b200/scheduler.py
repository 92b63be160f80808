"""The F rank's job runner: the routed experts of every layer behind one FfnServer.

Replaces what the reference's FfnScheduler (python/sgl_asap_plugin/srt/managers/scheduler.py:162-453) does per
job, without SGLang: ``run_job`` (scheduler.py:387-436) launches libasap's fused chain -- expert-major
permutation + MXFP8 quantisation, GEMM1 (+SwiGLU + requant), GEMM2 (+top-k weight), the weighted reduce that
stores the reply rows straight into the A rank's ResultArena and releases its done flag (server.py:340-350) --
and ``rows_of`` (scheduler.py:438-450) gives torch views of a row's arena region.  ``JobTimer``
(scheduler.py:109-159) keeps its fields: per power-of-two bucket, host launch us, expert GPU ms (alone /
queued) and reply ms (here part of the expert chain, reported as 0).

Everything a job needs on the GPU is derived on the device from the job descriptor (n, seq), so a job can be
enqueued before its doorbell rings (``run_device_wait``) and the chain can be captured in a CUDA graph.

A job may answer several messages of one layer at once (``join`` > 1): the reference's ``Job`` already carries a
list of ``Row``s (the A ranks of a group, server.py:322-337, concatenated by ``run_job``, scheduler.py:399-405);
here the rows may also come from different A replicas (``run_device_wait_rows``), so that small messages share
one read of the experts' weights.
"""

from __future__ import annotations

import collections
import ctypes
import statistics
import time
from typing import Dict, Optional

import torch

from . import _native as N
from .experts import Mxfp4Experts, _aligned_empty
from .transport.layout import SEQ_MASK
from .transport.memory import HostWords
from .transport.server import FfnServer, Job, Row, _raw_bytes


class JobTimer:
    """scheduler.py:109-159: per job-size bucket, host launch time, experts GPU time (alone / queued)."""

    def __init__(self, keep: int = 4096):
        self.keep = keep
        self.pending = collections.deque()
        self.samples = collections.defaultdict(lambda: collections.defaultdict(list))
        self.free = []

    def event(self) -> torch.cuda.Event:
        event = self.free.pop() if self.free else torch.cuda.Event(enable_timing=True)
        event.record()
        return event

    def start(self) -> tuple:
        alone = not self.pending or self.pending[-1][3].query()
        return alone, self.event()

    def add(self, n_tokens: int, started: tuple, host_s: float) -> None:
        bucket = 1 << (n_tokens - 1).bit_length()
        self.pending.append((bucket, *started, self.event(), host_s))
        self.drain()

    def drain(self) -> None:
        while self.pending and self.pending[0][3].query():
            bucket, alone, start, done, host_s = self.pending.popleft()
            rows = self.samples[bucket]
            if len(rows["host_us"]) < self.keep:
                rows["host_us"].append(host_s * 1e6)
                rows["reply_ms"].append(0.0)
                rows[f"experts_ms_{'alone' if alone else 'queued'}"].append(start.elapsed_time(done))
            self.free += [start, done]

    def summary(self) -> dict:
        torch.cuda.synchronize()
        self.drain()
        out = {}
        for bucket, rows in sorted(self.samples.items()):
            out[bucket] = {"jobs": len(rows["host_us"])}
            for name, values in sorted(rows.items()):
                out[bucket][f"{name}_p50"] = round(statistics.median(values), 4)
                out[bucket][f"{name}_n"] = len(values)
        return out


class FfnScheduler:
    """The experts of one F rank (``experts[layer_id]``) answering the jobs of ``server``."""

    def __init__(self, server: FfnServer, experts: Dict[int, Mxfp4Experts], *, swiglu_limit: float = 0.0,
                 timeout_s: float = 60.0, timing: bool = False, join: int = 1, overlap_replies: int = 0):
        g = server.g
        if g.group != 1:
            raise NotImplementedError("AFD supports attention TP size 1 only (group=1), as the reference's "
                                      "deployment check does (srt/arg_groups/asap_hook.py:175-176)")
        first = next(iter(experts.values()))
        for lid, e in experts.items():
            if (e.num_local, e.hidden, e.inter, e.expert_base) != (first.num_local, first.hidden, first.inter,
                                                                    first.expert_base):
                raise ValueError(f"layer {lid} serves other experts than layer {next(iter(experts))}")
        if first.hidden != g.hidden:
            raise ValueError(f"experts hidden {first.hidden} != geometry hidden {g.hidden}")
        self.server, self.g, self.experts = server, g, experts
        self.f = server.f
        self.device = server.device
        self.swiglu_limit = float(swiglu_limit or 0.0)
        self.timeout_ns = int(timeout_s * 1e9)
        self.local = range(first.expert_base, first.expert_base + first.num_local)
        if not 1 <= join <= N.MAX_JOB_ROWS:
            raise ValueError(f"join must be in [1, {N.MAX_JOB_ROWS}]")
        self.join = join
        cap = g.n_max * join  # tokens of one (joined) job
        nbytes = N.lib().asap_ffn_ws_bytes(cap, g.topk, first.num_local, first.hidden, first.inter)
        self._ws_owner, self.ws = _aligned_empty(nbytes, f"cuda:{self.device}")
        h = ctypes.c_uint64()
        N.call("asap_ffn_ws_register", self.ws.data_ptr(), cap, g.topk, first.num_local, first.hidden,
               first.inter, ctypes.byref(h))
        self.ws_handle = h.value
        # overlap_replies = k > 0: device-wait jobs that ask for it send their reduce + reply from a side stream on
        # k SMs (the GEMMs keep the others) while the next job computes; jobs alternate between two workspaces so
        # that a reply still reading one never meets the next job writing it
        self.reserve = int(overlap_replies)
        self._wss, self._owners = [self.ws_handle], [self._ws_owner]
        self._ws_i = 0
        self._reply_done = [None, None]
        self._reply_stream = None
        if self.reserve:
            if not 0 < self.reserve < 64:
                raise ValueError("overlap_replies: SMs left to the replies, in [1, 63]")
            owner2, ws2 = _aligned_empty(nbytes, f"cuda:{self.device}")
            h2 = ctypes.c_uint64()
            N.call("asap_ffn_ws_register", ws2.data_ptr(), cap, g.topk, first.num_local, first.hidden,
                   first.inter, ctypes.byref(h2))
            self._wss.append(h2.value)
            self._owners.append(owner2)
            self._reply_stream = torch.cuda.Stream(self.device)
        self.status = HostWords(1)
        # CUDA-graph mode: per (A rank, slot) the last consumed seq lives on the device (asap_ffn_wait_state), so a
        # chain captured once replays for every message; _dev_seq mirrors what those words will hold
        self.seq_state = torch.zeros(g.num_a * g.slots, dtype=torch.int32, device=f"cuda:{self.device}")
        self.rr_state = torch.full((1,), -1, dtype=torch.int32, device=f"cuda:{self.device}")
        self._dev_seq: Dict[tuple, Optional[int]] = {}
        self._dev_owned = set()  # (a, slot) whose last seq only the device knows (after round-robin jobs)
        self._graphs: Dict[tuple, int] = {}
        self._capture = None
        self.graph_replays = 0
        self.layer_calls = collections.Counter()
        self.job_timer = JobTimer() if timing else None
        arena = _raw_bytes(server.recv_base, g.recv_bytes, self.device)
        self.recv_arena = arena

    def close(self) -> None:
        for h in self._graphs.values():
            N.call("asap_graph_release", h)
        self._graphs.clear()
        if self.ws_handle:
            for h in self._wss:
                N.call("asap_ffn_ws_release", h)
            self.ws_handle = 0
        self.status.close()

    def _next_ws(self, stream: int) -> None:
        """Overlapped replies: the next job takes the other workspace, after the reply that last read it."""
        if not self.reserve:
            return
        self._ws_i ^= 1
        self.ws_handle = self._wss[self._ws_i]
        ev = self._reply_done[self._ws_i]
        if ev is not None:
            torch.cuda.ExternalStream(stream, device=self.device).wait_event(ev)

    def enable_timing(self, on: bool) -> None:
        """Per-stage CUDA events of every job (asap_ffn_enable_timing on each workspace)."""
        for h in self._wss:
            N.call("asap_ffn_enable_timing", h, 1 if on else 0)

    def last_timing(self) -> Optional[list]:
        """Mean per-stage ms (routing, quantise+permute, gemm1, gemm2, reduce+reply) of the recorded jobs, over
        the workspaces that recorded any; None if none did."""
        got = []
        for h in self._wss:
            kms = (ctypes.c_float * 5)()
            if N.lib().asap_ffn_last_timing(h, kms, 5) == 0:
                got.append([float(v) for v in kms])
        return [sum(v[i] for v in got) / len(got) for i in range(5)] if got else None

    def check(self) -> None:
        word = self.status.read()
        if word:
            st = N.decode_status(word)
            raise RuntimeError(f"F rank {self.f}: device {st['what']} (slot {st['slot']}, seq {st['seq']})")

    # ---------------------------------------------------------------- one job
    def _launch(self, experts: Mxfp4Experts, row: Row, reply, stream: int) -> None:
        seg, done = reply
        N.call("asap_ffn_job", experts.handle, self.ws_handle, row.x_ptr, row.ids_ptr, row.w_ptr, seg, done,
               ctypes.c_float(self.swiglu_limit), self.status.ptr, self.timeout_ns, ctypes.c_void_p(stream))

    def _launch_rows(self, experts, rows, targets, stream: int, overlap: bool = False) -> None:
        views = (N.FfnRow_t * len(rows))(*[N.FfnRow_t(r.x_ptr, r.ids_ptr, r.w_ptr, seg, done)
                                            for r, (seg, done) in zip(rows, targets)])
        if self.reserve and overlap:
            sms = torch.cuda.get_device_properties(self.device).multi_processor_count
            N.call("asap_ffn_job_rows_overlap", experts.handle, self.ws_handle, len(rows), views,
                   ctypes.c_float(self.swiglu_limit), self.status.ptr, self.timeout_ns, ctypes.c_void_p(stream),
                   ctypes.c_void_p(self._reply_stream.cuda_stream), sms - self.reserve, 2 * self.reserve)
            ev = torch.cuda.Event()
            ev.record(self._reply_stream)
            self._reply_done[self._ws_i] = ev
            return
        N.call("asap_ffn_job_rows", experts.handle, self.ws_handle, len(rows), views,
               ctypes.c_float(self.swiglu_limit), self.status.ptr, self.timeout_ns, ctypes.c_void_p(stream))
        if self.reserve:
            self._reply_done[self._ws_i] = None  # this job's reply is ordered on the job's own stream

    def run_job(self, job: Job, stream: Optional[int] = None) -> None:
        """One expert chain for the rows of one job (host-poll mode; the rows' tokens are answered together, as
        scheduler.py:399-405 concatenates them); enqueues GPU work only."""
        tic, timer = time.perf_counter(), self.job_timer
        started = timer.start() if timer else None
        if stream is None:
            stream = torch.cuda.current_stream(self.device).cuda_stream
        self._next_ws(stream)
        live = [(row, self.server.reply_target(row)) for row in job.rows]
        live = [(row, t) for row, t in live if t is not None]  # reconnected A ranks: dropped (server.py:343-346)
        if not live:
            return
        if len(live) > self.join:
            raise ValueError(f"a job of {len(live)} rows needs join >= {len(live)} (this scheduler: {self.join})")
        rows = [r for r, _ in live]
        if len(rows) == 1:
            row, target = live[0]
            N.call("asap_ffn_post", self.ws_handle, row.seq & SEQ_MASK, row.n_tokens, row.layer_id, row.epoch,
                   ctypes.c_void_p(stream))
            self._launch(self.experts[job.layer_id], row, target, stream)
        else:
            R = len(rows)
            N.call("asap_ffn_post_rows", self.ws_handle, R, (ctypes.c_uint32 * R)(*[r.seq & SEQ_MASK for r in rows]),
                   (ctypes.c_int32 * R)(*[r.n_tokens for r in rows]), job.layer_id,
                   (ctypes.c_int32 * R)(*[r.epoch for r in rows]), ctypes.c_void_p(stream))
            self._launch_rows(self.experts[job.layer_id], rows, [t for _, t in live], stream)
        self.layer_calls[job.layer_id] += 1
        if timer:
            timer.add(sum(r.n_tokens for r in rows), started, time.perf_counter() - tic)

    def run_device_wait(self, a: int, slot: int, seq: int, layer_id: int, stream: int,
                        overlap: bool = False) -> None:
        """Enqueue a job for the next message of (a, slot) before it arrives: the chain starts with a bounded
        device spin on the doorbell (libasap asap_ffn_wait), which also validates epoch and size.  The token count
        comes from the doorbell on the device; ``seq`` is the message the host expects (backpressure forbids
        skipping one)."""
        server = self.server
        peer = server.peers[a]
        row = server.row_for(a, slot, seq, self.g.n_max, layer_id)
        target = server.reply_target(row)
        if target is None:
            return
        self._next_ws(stream)
        N.call("asap_ffn_wait", self.ws_handle, server.bell_dev(a, slot), (seq - 1) & SEQ_MASK, peer.epoch,
               self.g.n_max, self.status.ptr, self.timeout_ns, ctypes.c_void_p(stream))
        if self.reserve:
            self._launch_rows(self.experts[layer_id], [row], [target], stream, overlap)
        else:
            self._launch(self.experts[layer_id], row, target, stream)
        server.advance(a, slot, seq)
        self._dev_seq[(a, slot)] = None  # the device word was not used: re-sync before the next graph replay
        self._dev_owned.discard((a, slot))
        self.layer_calls[layer_id] += 1

    def run_graph(self, messages, layer_id: int, stream: int) -> None:
        """``run_device_wait`` / ``run_device_wait_rows`` for ``messages`` = [(a, slot, seq), ...] as one replay of a
        CUDA graph captured on first use per (their (a, slot) pairs, layer, epochs) -- the device-side doorbell
        wait (sequence words on the device) and the whole expert chain in one launch."""
        if self.reserve:
            raise ValueError("CUDA-graph jobs do not overlap their replies (overlap_replies=0)")
        server = self.server
        rows, targets = [], []
        for a, slot, seq in messages:
            row = server.row_for(a, slot, seq, self.g.n_max, layer_id)
            target = server.reply_target(row)
            if target is not None:
                rows.append(row)
                targets.append(target)
        if not rows:
            return
        if len(rows) > self.join:
            raise ValueError(f"a job of {len(rows)} rows needs join >= {len(rows)} (this scheduler: {self.join})")
        for r in rows:  # the device words must hold the seq before this message
            if self._dev_seq.get((r.a, r.slot)) != (r.seq - 1) & SEQ_MASK:
                N.call("asap_write32", self._state_ptr(r.a, r.slot), (r.seq - 1) & SEQ_MASK, ctypes.c_void_p(stream))
            self._dev_owned.discard((r.a, r.slot))
        key = (tuple((r.a, r.slot) for r in rows), layer_id, tuple(server.peers[r.a].epoch for r in rows))
        graph = self._graphs.get(key)
        if graph is None:
            graph = self._graphs[key] = self._capture_chain(rows, targets, layer_id)
        N.call("asap_graph_launch", graph, ctypes.c_void_p(stream))
        self.graph_replays += 1
        for r in rows:
            server.advance(r.a, r.slot, r.seq)
            self._dev_seq[(r.a, r.slot)] = r.seq & SEQ_MASK
        self.layer_calls[layer_id] += 1

    def run_device_wait_any(self, sources, layer_id: int, stream: int, graph: bool = False,
                            overlap: bool = False) -> None:
        """One job answering ONE message of layer ``layer_id``: the first of ``sources`` = [(a, slot), ...] with a new
        message, in round-robin order after the source answered last -- the reference's poll order over ready
        doorbells (server.py:270-275), decided on the device (asap_ffn_wait_any), so one slow replica does not
        hold up the others' answers.  Enqueue one such job per expected message.  With ``graph`` the wait and the
        chain are one CUDA-graph replay (captured once per sources, layer and epochs)."""
        server = self.server
        rows, targets = [], []
        for a, slot in sources:
            row = server.row_for(a, slot, 0, self.g.n_max, layer_id)
            target = server.reply_target(row)
            if target is None:
                raise RuntimeError(f"A rank {a} is not connected to F rank {self.f}")
            rows.append(row)
            targets.append(target)
            if (a, slot) not in self._dev_owned:  # the device word takes over from the host's bookkeeping
                last = server.last_seq(a, slot)
                N.call("asap_write32", self._state_ptr(a, slot), last & SEQ_MASK, ctypes.c_void_p(stream))
                self._dev_owned.add((a, slot))
                self._dev_seq[(a, slot)] = None
        R = len(rows)
        if R > N.MAX_JOB_ROWS:
            raise ValueError(f"at most {N.MAX_JOB_ROWS} sources")
        epochs = [server.peers[r.a].epoch for r in rows]

        if graph and self.reserve:
            raise ValueError("CUDA-graph jobs do not overlap their replies (overlap_replies=0)")
        if not graph:
            self._next_ws(stream)

        def enqueue(st: int) -> None:
            N.call("asap_ffn_wait_any", self.ws_handle, R,
                   (ctypes.c_uint64 * R)(*[server.bell_dev(r.a, r.slot) for r in rows]),
                   (ctypes.c_uint64 * R)(*[self._state_ptr(r.a, r.slot) for r in rows]),
                   (ctypes.c_int32 * R)(*epochs), self.g.n_max, self.rr_state.data_ptr(), self.status.ptr,
                   self.timeout_ns, ctypes.c_void_p(st))
            self._launch_rows(self.experts[layer_id], rows, targets, st, overlap)

        if graph:
            key = ("any", tuple(sources), layer_id, tuple(epochs))
            h = self._graphs.get(key)
            if h is None:
                if self._capture is None:
                    self._capture = torch.cuda.Stream(self.device)
                cap = self._capture.cuda_stream
                N.call("asap_graph_begin", ctypes.c_void_p(cap))
                out = ctypes.c_uint64()
                try:
                    enqueue(cap)
                finally:
                    N.call("asap_graph_end", ctypes.c_void_p(cap), ctypes.byref(out))
                h = self._graphs[key] = out.value
            N.call("asap_graph_launch", h, ctypes.c_void_p(stream))
            self.graph_replays += 1
        else:
            enqueue(stream)
        self.layer_calls[layer_id] += 1

    def run_device_wait_rest(self, messages, layer_id: int, stream: int, overlap: bool = False) -> None:
        """One joined job over the messages of this round not answered yet, ``messages`` = [(a, slot, seq), ...]
        with ``seq`` each source's message of the round: a source whose device sequence word already reached it
        (answered by an earlier run_device_wait_any job) is left out on the device (asap_ffn_wait_rest), the others'
        doorbells are awaited and their messages answered by one chain.  Enqueued after one run_device_wait_any
        per round, an F rank serving several replicas starts on the first message to arrive and answers the rest
        with one larger job."""
        server = self.server
        rows, targets = [], []
        for a, slot, _ in messages:
            row = server.row_for(a, slot, 0, self.g.n_max, layer_id)
            target = server.reply_target(row)
            if target is None:
                raise RuntimeError(f"A rank {a} is not connected to F rank {self.f}")
            rows.append(row)
            targets.append(target)
            if (a, slot) not in self._dev_owned:  # the device word takes over from the host's bookkeeping
                last = server.last_seq(a, slot)
                N.call("asap_write32", self._state_ptr(a, slot), last & SEQ_MASK, ctypes.c_void_p(stream))
                self._dev_owned.add((a, slot))
                self._dev_seq[(a, slot)] = None
        R = len(rows)
        if R > min(self.join, N.MAX_JOB_ROWS):
            raise ValueError(f"a job of {R} rows needs join >= {R} (this scheduler: {self.join})")
        self._next_ws(stream)
        N.call("asap_ffn_wait_rest", self.ws_handle, R,
               (ctypes.c_uint64 * R)(*[server.bell_dev(r.a, r.slot) for r in rows]),
               (ctypes.c_uint64 * R)(*[self._state_ptr(r.a, r.slot) for r in rows]),
               (ctypes.c_uint32 * R)(*[seq & SEQ_MASK for _, _, seq in messages]),
               (ctypes.c_int32 * R)(*[server.peers[r.a].epoch for r in rows]), self.g.n_max, self.status.ptr,
               self.timeout_ns, ctypes.c_void_p(stream))
        self._launch_rows(self.experts[layer_id], rows, targets, stream, overlap)
        self.layer_calls[layer_id] += 1

    def _state_ptr(self, a: int, slot: int) -> int:
        return self.seq_state.data_ptr() + 4 * (a * self.g.slots + slot)

    def _capture_chain(self, rows, targets, layer_id: int) -> int:
        if self._capture is None:
            self._capture = torch.cuda.Stream(self.device)
        cap = ctypes.c_void_p(self._capture.cuda_stream)
        server, R = self.server, len(rows)
        N.call("asap_graph_begin", cap)
        h = ctypes.c_uint64()
        try:
            N.call("asap_ffn_wait_state", self.ws_handle, R,
                   (ctypes.c_uint64 * R)(*[server.bell_dev(r.a, r.slot) for r in rows]),
                   (ctypes.c_uint64 * R)(*[self._state_ptr(r.a, r.slot) for r in rows]),
                   (ctypes.c_int32 * R)(*[server.peers[r.a].epoch for r in rows]), self.g.n_max, self.status.ptr,
                   self.timeout_ns, cap)
            self._launch_rows(self.experts[layer_id], rows, targets, cap.value)
        finally:
            N.call("asap_graph_end", cap, ctypes.byref(h))
        return h.value

    def run_device_wait_rows(self, messages, layer_id: int, stream: int) -> None:
        """One joined job over the next messages of several (a, slot) pairs, ``messages`` = [(a, slot, seq), ...]
        (all of layer ``layer_id``), enqueued before they arrive: the chain starts with one bounded device wait for
        all their doorbells; every row's reply goes to its own A rank."""
        server = self.server
        rows, targets = [], []
        for a, slot, seq in messages:
            row = server.row_for(a, slot, seq, self.g.n_max, layer_id)
            target = server.reply_target(row)
            if target is not None:
                rows.append(row)
                targets.append(target)
        if not rows:
            return
        R = len(rows)
        if R > self.join:
            raise ValueError(f"a job of {R} rows needs join >= {R} (this scheduler: {self.join})")
        self._next_ws(stream)
        N.call("asap_ffn_wait_rows", self.ws_handle, R,
               (ctypes.c_uint64 * R)(*[server.bell_dev(r.a, r.slot) for r in rows]),
               (ctypes.c_uint32 * R)(*[(r.seq - 1) & SEQ_MASK for r in rows]),
               (ctypes.c_int32 * R)(*[server.peers[r.a].epoch for r in rows]), self.g.n_max, self.status.ptr,
               self.timeout_ns, ctypes.c_void_p(stream))
        self._launch_rows(self.experts[layer_id], rows, targets, stream)
        for r in rows:
            server.advance(r.a, r.slot, r.seq)
            self._dev_seq[(r.a, r.slot)] = None
            self._dev_owned.discard((r.a, r.slot))
        self.layer_calls[layer_id] += 1

    def rows_of(self, row: Row):
        """x, topk_ids and topk_weights of one row: views into the RecvArena (scheduler.py:438-450)."""
        g, arena = self.g, self.recv_arena
        n, off = row.n_tokens, row.x_ptr - self.server.recv_base
        x = arena[off: off + n * g.hidden * 2].view(torch.bfloat16).view(n, g.hidden)
        ids_off, w_off = off + g.ids_off, off + g.w_off
        topk_ids = arena[ids_off: ids_off + n * g.topk * 4].view(torch.int32).view(n, g.topk)
        topk_weights = arena[w_off: w_off + n * g.topk * 4].view(torch.float32).view(n, g.topk)
        return x, topk_ids, topk_weights

    def debug_tensors(self) -> dict:
        """Device buffers of the last job (tests): per-local-expert counts and the pair permutation."""
        vals = [ctypes.c_uint64() for _ in range(7)]
        N.call("asap_ffn_debug_ptrs", self.ws_handle, *[ctypes.byref(v) for v in vals])
        g, P = self.g, len(self.local)
        e = self.experts[next(iter(self.experts))]
        return {
            "expert_counts": _raw_bytes(vals[0].value, 4 * P, self.device).view(torch.int32),
            "pair_pos": _raw_bytes(vals[1].value, 4 * g.n_max * g.topk, self.device).view(torch.int32).view(
                g.n_max, g.topk),
            "xq": vals[2].value, "xq_sf": vals[3].value, "hq": vals[4].value, "hq_sf": vals[5].value,
            "y2": vals[6].value, "hidden": e.hidden, "inter": e.inter,
        }

    def job_info(self, stream: Optional[int] = None) -> dict:
        if stream is None:
            stream = torch.cuda.current_stream(self.device).cuda_stream
        n, layer, epoch, valid = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
        seq, t_seen, t_reply = ctypes.c_uint32(), ctypes.c_uint64(), ctypes.c_uint64()
        N.call("asap_ffn_job_info", self.ws_handle, ctypes.byref(n), ctypes.byref(layer), ctypes.byref(seq),
               ctypes.byref(epoch), ctypes.byref(valid), ctypes.byref(t_seen), ctypes.byref(t_reply),
               ctypes.c_void_p(stream))
        return {"n": n.value, "layer": layer.value, "seq": seq.value, "epoch": epoch.value, "valid": valid.value,
                "t_seen_ns": t_seen.value, "t_reply_ns": t_reply.value}
