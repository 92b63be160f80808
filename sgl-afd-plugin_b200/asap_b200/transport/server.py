"""F side of the transport: one FfnServer per F rank.  It owns the RecvArena (where the A ranks' dispatch kernels
store their rows) and the doorbell page (where they release the 64-bit doorbell words), admits A ranks through the
JSON-line handshake, and tells the expert chain where each message is and where its answer goes.

The API and the wire contract are the reference's (python/sgl_asap_plugin/transport/server.py:87-390): the
handshake fields and rejection texts, ``PROTO_VERSION``, epochs cycling ``old % 31 + 1`` on every reconnect,
sequence numbers compared as a cyclic 32-bit difference, lost messages counted as the gap minus one, round robin
over ready doorbells starting after the last one served, TP rows joined into one job per (replica, slot), and the
stats counter names.  The code is organised around how this build serves messages:

* the hot path never polls on the host: ``bell_dev`` gives the GPU address of a doorbell and libasap's
  asap_ffn_wait / asap_ffn_wait_any spin on it inside the F job's first kernel (see ``FfnScheduler``), and the
  reply rows plus the done flag are stored by the job's last kernel;
* ``poll`` / ``serve_forever`` remain as the host fallback (the reference's discovery mode), built from two small
  parts: ``BellScanner`` (which doorbells moved, in round-robin order) and ``GroupAssembler`` (which jobs are
  complete);
* the handshake runs in ``wire.HelloListener`` and goes through ``_admit``, a list of checks.
"""

from __future__ import annotations

import collections
import ctypes
import os
import threading
import time
from dataclasses import dataclass
from typing import Callable, Dict, List, Optional, Tuple

import numpy as np
import torch

from .. import _native as N
from .layout import BELL_STRIDE, MAX_EPOCH, PROTO_VERSION, SEQ_MASK, Geometry, HandshakeError, unpack_doorbell
from .memory import Shared
from .memory import select as select_memory
from .wire import HelloListener


def next_epoch(previous: Optional[int]) -> int:
    """Epoch of an A rank's next connection: 1 for the first, then 2, ..., MAX_EPOCH (31), 1, ... (the doorbell
    word has 5 epoch bits and 0 is never used)."""
    return 1 if previous is None else previous % MAX_EPOCH + 1


@dataclass
class Peer:
    """A connected A rank: where its ResultArena is mapped and which epoch its messages must carry."""

    a: int
    result_base: int
    epoch: int
    pid: int
    mapping: Optional[Shared] = None
    host: Optional[str] = None


@dataclass
class Row:
    """One A rank's part of a job; the pointers address this F rank's RecvArena."""

    a: int
    slot: int
    seq: int
    epoch: int
    layer_id: int
    n_tokens: int
    x_ptr: int
    ids_ptr: int
    w_ptr: int


@dataclass
class Job:
    """One micro-batch of one layer of one replica, ready to compute."""

    replica: int
    slot: int
    layer_id: int
    rows: List[Row]
    t_detect_ns: int


class BellScanner:
    """The last sequence number seen per (A rank, slot) and where the next scan starts.  ``scan(words)`` returns
    the doorbells whose sequence number moved forward, as (index, seq, messages skipped), starting after the index
    that moved last time and wrapping around, so no A rank is always served first."""

    def __init__(self, count: int, seq_base: int):
        self.seen = np.full(count, seq_base & SEQ_MASK, dtype=np.int64)
        self.start = 0

    def reset(self, lo: int, hi: int, seq_base: int) -> None:
        self.seen[lo:hi] = seq_base & SEQ_MASK

    def scan(self, words: np.ndarray) -> List[Tuple[int, int, int]]:
        seq = (words & np.uint64(SEQ_MASK)).astype(np.int64)
        gap = (seq - self.seen) % (1 << 32)  # forward distance on the 32-bit circle
        moved = (gap > 0) & (gap < (1 << 31))
        count = len(seq)
        order = (np.arange(count) + self.start) % count
        hits = order[moved[order]]
        for idx in hits:
            self.seen[idx] = seq[idx]
        if hits.size:
            self.start = int(hits[-1]) + 1 if int(hits[-1]) + 1 < count else 0
        return [(int(i), int(seq[i]), int(gap[i]) - 1) for i in hits]


class GroupAssembler:
    """Rows of one (replica, slot) message arrive one TP rank at a time; a job is complete when every rank's row
    is there."""

    def __init__(self, group: int):
        self.group = group
        self.partial: Dict[Tuple[int, int], List[Optional[Row]]] = {}

    def add(self, key: Tuple[int, int], member: int, row: Row) -> Optional[List[Row]]:
        have = self.partial.setdefault(key, [None] * self.group)
        have[member] = row
        if any(r is None for r in have):
            return None
        del self.partial[key]
        return have

    def forget_replica(self, replica: int) -> None:
        for key in [k for k in self.partial if k[0] == replica]:
            del self.partial[key]


class FfnServer:
    """One F rank's end of the transport (start -> serve or device-wait jobs -> close)."""

    def __init__(self, f_rank: int, geometry: Geometry, *, device: int, run_dir: str, host: str = "127.0.0.1",
                 port: int = 0, seq_base: int = 0, memory: str = "auto", model: Optional[dict] = None,
                 info: Optional[dict] = None, trace_len: int = 4096, listen: bool = True):
        """``memory``: how the RecvArena and the doorbell page are shared (auto / ipc; every A rank must resolve to
        the same).  ``run_dir``: where the doorbell page's file lives (/dev/shm).  ``model``: the fingerprint every
        hello must carry (None: not checked).  ``info``: extra fields of the handshake answer.  ``listen``: False
        for in-process deployments (``handshake`` is called directly)."""
        self.f, self.g, self.seq_base = f_rank, geometry, seq_base
        self.memory, self.mem = memory, None
        self.model, self.info = model, dict(info or {})
        self.device, self.run_dir, self.host, self.listen = device, run_dir, host, listen
        self._port_req = port
        self.port: Optional[int] = None
        self.stats: collections.Counter = collections.Counter()
        self.trace: collections.deque = collections.deque(maxlen=trace_len)
        self.peers: Dict[int, Peer] = {}
        self._lock = threading.RLock()  # peers, scanner and assembler are shared with the handshake thread
        self._listener: Optional[HelloListener] = None
        self._last_replica: Optional[int] = None

    # ---------------------------------------------------------------- life cycle
    def start(self) -> "FfnServer":
        """Allocate and zero the RecvArena and the doorbell page, then accept A ranks."""
        g = self.g
        if self.mem is None:
            self.mem = select_memory(self.memory, self.device)
        self.mem.activate()
        self._recv = self.mem.device(g.recv_bytes)
        self.recv_base = self._recv.ptr
        self.mem.fill32(self.recv_base, 0, g.recv_bytes // 4)
        self._page = self.mem.doorbells(g.host_bytes,
                                        os.path.join(self.run_dir, f"asap_f{self.f}_{os.getpid()}.slots"))
        page = np.ctypeslib.as_array((ctypes.c_uint64 * (g.host_bytes // 8)).from_address(self._page.ptr))
        per_line = BELL_STRIDE // 8
        self.bell_words = page[: g.num_a * g.slots * per_line][::per_line]  # word 0 of each doorbell line
        self.bell_words[:] = self.seq_base
        self._scanner = BellScanner(g.num_a * g.slots, self.seq_base)
        self._assembler = GroupAssembler(g.group)
        if self.listen:
            self._listener = HelloListener(self.host, self._port_req, self._admit, f"asap-handshake-f{self.f}")
            self.port = self._listener.port
        return self

    def unmap_peers(self) -> None:
        """Unmap every connected A rank's ResultArena (first step of an orderly multi-process shutdown)."""
        for peer in self.peers.values():
            peer.mapping.release()

    def close(self) -> None:
        """Stop accepting, unmap the A arenas, free the doorbell page and the RecvArena."""
        if self._listener is not None:
            self._listener.stop()
            self._listener = None
        self.unmap_peers()
        self.peers.clear()
        self.bell_words = None
        self._page.release()
        self._recv.release()

    # ---------------------------------------------------------------- admission
    def handshake(self, hello: dict) -> dict:
        """In-process handshake with the TCP one's checks: the answer, or HandshakeError."""
        try:
            return self._admit(hello)
        except HandshakeError:
            raise
        except Exception as exc:
            raise HandshakeError(f"{type(exc).__name__}: {exc}") from exc

    def _admit(self, hello: dict) -> dict:
        """Check the hello, map the A rank's ResultArena, give it a new epoch and clear its slots."""
        for check in (self._check_protocol, self._check_memory, self._check_geometry, self._check_model,
                      self._check_rank):
            problem = check(hello)
            if problem:
                raise HandshakeError(problem)
        a = int(hello["a"])
        self.mem.activate()
        result = self.mem.open(hello["result"])  # may fail: keep the old mapping until it succeeded
        g = self.g
        with self._lock:
            old = self.peers.get(a)
            if old is not None:
                old.mapping.release()
                self.stats["reconnects"] += 1
            peer = Peer(a, result.ptr, next_epoch(old.epoch if old else None), int(hello.get("pid", 0)), result,
                        (hello.get("peer") or {}).get("host"))
            self.peers[a] = peer
            first, stop = a * g.slots, (a + 1) * g.slots
            self.bell_words[first:stop] = self.seq_base
            self._scanner.reset(first, stop, self.seq_base)
            self._assembler.forget_replica(a // g.group)  # half-joined jobs of the previous incarnation
        answer = {"ok": True, "f": self.f, "epoch": peer.epoch, "seq_base": self.seq_base, "memory": self.mem.kind,
                  "recv": self._recv.desc, "doorbells": self._page.desc}
        answer.update(self.info)
        return answer

    def _check_protocol(self, hello: dict) -> Optional[str]:
        if hello.get("proto") != PROTO_VERSION:
            return f"protocol version A={hello.get('proto')} F={PROTO_VERSION}"
        return None

    def _check_memory(self, hello: dict) -> Optional[str]:
        if hello.get("memory") != self.mem.kind:
            return (f"transport memory A={hello.get('memory')} F={self.mem.kind} ({self.mem.reason}): "
                    "give both roles the same --asap-transport-mem")
        self.mem.check_peer(hello.get("peer") or {})  # raises HandshakeError itself
        return None

    @staticmethod
    def _mismatches(theirs: dict, ours: dict) -> str:
        return ", ".join(f"{k}: A={theirs.get(k)} F={v}" for k, v in ours.items() if theirs.get(k) != v)

    def _check_geometry(self, hello: dict) -> Optional[str]:
        diff = self._mismatches(hello.get("geometry", {}), self.g.as_dict())
        return f"geometry mismatch ({diff})" if diff else None

    def _check_model(self, hello: dict) -> Optional[str]:
        if self.model is None:
            return None
        diff = self._mismatches(hello.get("model") or {}, self.model)
        return f"the A model and the experts served here differ ({diff})" if diff else None

    def _check_rank(self, hello: dict) -> Optional[str]:
        a = int(hello["a"])
        if not 0 <= a < self.g.num_a:
            return f"A rank {a} is outside [0, {self.g.num_a})"
        host = (hello.get("peer") or {}).get("host")
        with self._lock:
            holder = self.peers.get(a)
        if holder is not None and holder.host != host:  # not a reconnect: two A instances number a rank alike
            return (f"A rank {a} is connected from {holder.host} (pid {holder.pid}), and {host} claims it too: "
                    "the attention instances sharing the FFN ranks need disjoint --asap-attn-base-replica ranges")
        return None

    # ---------------------------------------------------------------- where messages are
    def bell_dev(self, a: int, s: int) -> int:
        """GPU address of A rank a's slot-s doorbell (the device waits spin on it)."""
        return self._page.dev + self.g.bell_off(a, s)

    def row_for(self, a: int, s: int, seq: int, n_tokens: int, layer_id: int) -> Row:
        """The Row of (a, s)'s message ``seq`` (device-wait mode: the device reads the real count)."""
        x = self.recv_base + self.g.region_off(a, s)
        return Row(a, s, seq, self.peers[a].epoch, layer_id, n_tokens, x, x + self.g.ids_off, x + self.g.w_off)

    def last_seq(self, a: int, s: int) -> int:
        """The last sequence number of (a, s) consumed here (host poll or ``advance``)."""
        with self._lock:
            return int(self._scanner.seen[a * self.g.slots + s])

    def advance(self, a: int, s: int, seq: int) -> None:
        """Device-wait mode: the GPU consumed (a, s)'s messages up to ``seq``."""
        with self._lock:
            self._scanner.seen[a * self.g.slots + s] = seq & SEQ_MASK

    def reply_target(self, row: Row) -> Optional[Tuple[int, int]]:
        """(segment address, done-flag address) of the row's answer in its A rank, or None when that A rank
        reconnected after sending it (the answer is dropped and counted)."""
        peer = self.peers.get(row.a)
        if peer is None or peer.epoch != row.epoch:
            self.stats["dropped_replies"] += 1
            return None
        return peer.result_base + self.g.seg_off(self.f, row.slot), peer.result_base + self.g.done_off(self.f,
                                                                                                       row.slot)

    # ---------------------------------------------------------------- host fallback: poll and serve
    def poll(self) -> List[Job]:
        """Jobs whose rows all arrived since the last call (never blocks)."""
        g, jobs = self.g, []
        with self._lock:
            words = self.bell_words.copy()
            for idx, seq, skipped in self._scanner.scan(words):
                self.stats["lost_messages"] += skipped  # overwritten before anyone read them; 0 with backpressure
                a, s = divmod(idx, g.slots)
                row = self._decode(a, s, int(words[idx]))
                if row is None:
                    continue
                rows = self._assembler.add((a // g.group, s), a % g.group, row)
                job = self._job(a // g.group, s, rows) if rows is not None else None
                if job is not None:
                    jobs.append(job)
        return jobs

    def _decode(self, a: int, s: int, word: int) -> Optional[Row]:
        seq, n_tokens, layer_id, epoch = unpack_doorbell(word)
        peer = self.peers.get(a)
        problem = ("unknown_peer" if peer is None else "stale_epoch" if epoch != peer.epoch else
                   "bad_doorbell" if not 1 <= n_tokens <= self.g.n_max else None)
        if problem:
            self.stats[problem] += 1
            return None
        x = self.recv_base + self.g.region_off(a, s)
        return Row(a, s, seq, epoch, layer_id, n_tokens, x, x + self.g.ids_off, x + self.g.w_off)

    def _job(self, replica: int, slot: int, rows: List[Row]) -> Optional[Job]:
        layers = {r.layer_id for r in rows}
        if len(layers) != 1:  # the TP ranks of one replica disagree on the layer: a protocol bug upstream
            self.stats["group_mismatch"] += 1
            return None
        layer = layers.pop()
        self.stats["jobs"] += 1
        if self._last_replica not in (None, replica):
            self.stats["replica_switches"] += 1
        self._last_replica = replica
        self.trace.append((replica, slot, layer))
        return Job(replica, slot, layer, rows, time.monotonic_ns())

    def reply(self, row: Row, src_ptr: int, nbytes: int, stream: int) -> None:
        """Enqueue on ``stream`` a copy of a partial sum computed elsewhere (nbytes at src_ptr) into the A rank's
        segment, then its done flag; dropped if that A rank reconnected since (the expert chain of this build
        stores its own replies, so only external handlers need this)."""
        target = self.reply_target(row)
        if target is None:
            return
        seg, done = target
        with torch.cuda.stream(torch.cuda.ExternalStream(stream)):
            _raw_bytes(seg, nbytes, self.device).copy_(_raw_bytes(src_ptr, nbytes, self.device), non_blocking=True)
        N.call("asap_write32", done, row.seq & SEQ_MASK, ctypes.c_void_p(stream))

    def serve_forever(self, handler: Callable[[Job], None], stop: threading.Event, spin_s: float = 0.005,
                      idle_sleep_s: float = 0.0002) -> None:
        """Host fallback loop: hand every complete job to ``handler`` (which should only enqueue GPU work) until
        ``stop`` is set.  It polls without pause for ``spin_s`` after a job, then naps ``idle_sleep_s`` between
        polls (on ``stop``, so closing never waits for a nap)."""
        self.mem.activate()
        busy_until = time.monotonic() + spin_s
        while not stop.is_set():
            jobs = self.poll()
            for job in jobs:
                handler(job)
            now = time.monotonic()
            if jobs:
                busy_until = now + spin_s
            elif idle_sleep_s and now > busy_until:
                stop.wait(idle_sleep_s)


class _CudaArray:
    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 2}


def _raw_bytes(ptr: int, nbytes: int, device: int) -> torch.Tensor:
    """A uint8 tensor aliasing raw device memory (not owned)."""
    return torch.as_tensor(_CudaArray(ptr, nbytes), device=f"cuda:{device}")
