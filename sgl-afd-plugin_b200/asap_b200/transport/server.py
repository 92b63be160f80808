"""F side of the transport: one FfnServer per F rank owns a RecvArena and a doorbell page, discovers messages,
and answers each with a partial sum written into the sender's ResultArena.

Same API and protocol as the reference's python/sgl_asap_plugin/transport/server.py: start, the handshake
thread (JSON line in / out, validation of proto, memory, geometry, model and host, epoch cycling
``(old % 31) + 1``), poll (cyclic int32 seq comparison, round robin, lost-message count ``ahead - 1``), _row
(unknown peer / stale epoch / bad size counters), _job (TP rows joined, group-mismatch counter), reply,
serve_forever and close.

Two discovery modes feed the same job handler:
* host poll (the reference's): the serving thread reads the doorbell words with plain loads (numpy);
* device wait: ``bell_dev(a, s)`` is the GPU address of a doorbell, which libasap's asap_ffn_wait spins on in
  a kernel, so a job can be queued on the GPU before its message arrives (the page is registered for this).
The reply itself is fused into the expert job (asap_ffn_job writes the rows and the done flag); ``reply()``
remains for callers that computed the partial sum elsewhere.
"""

from __future__ import annotations

import collections
import ctypes
import json
import os
import socket
import sys
import threading
import time
from dataclasses import dataclass
from typing import Callable, Dict, List, Optional

import numpy as np
import torch

from .. import _native as N
from .channel import MAX_HANDSHAKE_BYTES
from .layout import BELL_STRIDE, MAX_EPOCH, PROTO_VERSION, SEQ_MASK, Geometry, HandshakeError, unpack_doorbell
from .memory import Shared
from .memory import select as select_memory


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


class FfnServer:
    """One F rank's end of the transport (start -> serve_forever -> close)."""

    def __init__(self, f_rank: int, geometry: Geometry, *, device: int, run_dir: str, host: str = "127.0.0.1",
                 port: int = 0, seq_base: int = 0, memory: str = "auto", model: Optional[dict] = None,
                 info: Optional[dict] = None, trace_len: int = 4096, listen: bool = True):
        self.f, self.g, self.seq_base = f_rank, geometry, seq_base
        self.memory, self.mem = memory, None
        self.model, self.info = model, dict(info or {})
        self.device, self.run_dir, self.host, self._port_req = device, run_dir, host, port
        self.listen = listen
        self.stats: collections.Counter = collections.Counter()
        self.trace: collections.deque = collections.deque(maxlen=trace_len)
        self.peers: Dict[int, Peer] = {}
        self._pending: Dict[tuple, Dict[int, Row]] = {}
        self._lock = threading.RLock()
        self._rr = 0
        self._prev_replica = None
        self._srv = None
        self._hs_thread = None

    def start(self) -> "FfnServer":
        """Allocate and zero the RecvArena and the doorbell page, then listen for A ranks."""
        g = self.g
        if self.mem is None:
            self.mem = select_memory(self.memory, self.device)
        self.mem.activate()
        self._recv = self.mem.device(g.recv_bytes)
        self.recv_base = self._recv.ptr
        self.mem.fill32(self.recv_base, 0, g.recv_bytes // 4)
        self._page = self.mem.doorbells(g.host_bytes, os.path.join(self.run_dir, f"asap_f{self.f}_{os.getpid()}.slots"))
        words = np.ctypeslib.as_array((ctypes.c_uint64 * (g.host_bytes // 8)).from_address(self._page.ptr))
        self._bells = words[: g.num_a * g.slots * (BELL_STRIDE // 8)].reshape(-1, BELL_STRIDE // 8)[:, 0]
        self._bells[:] = self.seq_base
        self._last = np.full(g.num_a * g.slots, self.seq_base, dtype=np.uint32)
        self.port = None
        if self.listen:
            self._srv = socket.socket()
            self._srv.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
            self._srv.bind((self.host, self._port_req))
            self._srv.listen(64)
            self._srv.settimeout(0.2)
            self.port = self._srv.getsockname()[1]
            self._hs_stop = threading.Event()
            self._hs_thread = threading.Thread(target=self._accept_loop, name=f"asap-handshake-f{self.f}",
                                               daemon=True)
            self._hs_thread.start()
        return self

    def bell_dev(self, a: int, s: int) -> int:
        """GPU address of A rank a's slot-s doorbell (device-wait mode)."""
        return self._page.dev + self.g.bell_off(a, s)

    # ---- handshake (handshake thread) ----
    def _accept_loop(self) -> None:
        while not self._hs_stop.is_set():
            try:
                conn, _ = self._srv.accept()
            except (socket.timeout, OSError):
                continue
            with conn, conn.makefile("rwb") as f:
                conn.settimeout(10.0)
                try:
                    reply = self._on_hello(json.loads(f.readline(MAX_HANDSHAKE_BYTES)))
                except Exception as exc:  # reject with the reason; the thread survives any bad peer
                    reply = {"ok": False, "reason": f"{type(exc).__name__}: {exc}"}
                try:
                    f.write(json.dumps(reply).encode() + b"\n")
                    f.flush()
                except OSError:
                    pass

    def handshake(self, hello: dict) -> dict:
        """In-process handshake (same validation as the TCP one): the reply dict, or raises HandshakeError."""
        try:
            return self._on_hello(hello)
        except HandshakeError:
            raise
        except Exception as exc:
            raise HandshakeError(f"{type(exc).__name__}: {exc}") from exc

    def _on_hello(self, hello: dict) -> dict:
        """server.py:181-259: check protocol, memory, geometry, model and host; map A's ResultArena; new epoch."""
        g = self.g
        if hello.get("proto") != PROTO_VERSION:
            raise HandshakeError(f"protocol version A={hello.get('proto')} F={PROTO_VERSION}")
        if hello.get("memory") != self.mem.kind:
            raise HandshakeError(f"transport memory A={hello.get('memory')} F={self.mem.kind} ({self.mem.reason}): "
                                 "give both roles the same --asap-transport-mem")
        self.mem.check_peer(hello.get("peer") or {})
        theirs = hello.get("geometry", {})
        diff = [f"{k}: A={theirs.get(k)} F={v}" for k, v in g.as_dict().items() if theirs.get(k) != v]
        if diff:
            raise HandshakeError("geometry mismatch (" + ", ".join(diff) + ")")
        if self.model is not None:
            got = hello.get("model") or {}
            diff = [f"{k}: A={got.get(k)} F={v}" for k, v in self.model.items() if got.get(k) != v]
            if diff:
                raise HandshakeError("the A model and the experts served here differ (" + ", ".join(diff) + ")")
        a = int(hello["a"])
        if not 0 <= a < g.num_a:
            raise HandshakeError(f"A rank {a} is outside [0, {g.num_a})")
        host = (hello.get("peer") or {}).get("host")
        with self._lock:
            old = self.peers.get(a)
        if old is not None and old.host != host:
            raise HandshakeError(
                f"A rank {a} is connected from {old.host} (pid {old.pid}), and {host} claims it too: "
                "the attention instances sharing the FFN ranks need disjoint --asap-attn-base-replica ranges")
        self.mem.activate()
        result = self.mem.open(hello["result"])
        with self._lock:
            old = self.peers.get(a)
            if old is not None:
                old.mapping.release()
                self.stats["reconnects"] += 1
            peer = Peer(a, result.ptr, (old.epoch % MAX_EPOCH) + 1 if old else 1, int(hello.get("pid", 0)), result,
                        host)
            self.peers[a] = peer
            lo = a * g.slots
            self._bells[lo: lo + g.slots] = self.seq_base
            self._last[lo: lo + g.slots] = self.seq_base
            for s in range(g.slots):
                self._pending.pop((a // g.group, s), None)
        return {"ok": True, "f": self.f, "epoch": peer.epoch, "seq_base": self.seq_base, "memory": self.mem.kind,
                "recv": self._recv.desc, "doorbells": self._page.desc, **self.info}

    # ---- discovery (serving thread) ----
    def poll(self) -> List[Job]:
        """Jobs whose rows have all arrived since the last call; never blocks (server.py:262-294)."""
        g, jobs = self.g, []
        with self._lock:
            words = self._bells.copy()
            seq = (words & np.uint64(SEQ_MASK)).astype(np.uint32)
            ahead = (seq - self._last).view(np.int32)
            ready = np.flatnonzero(ahead > 0)
            if ready.size > 1:
                ready = np.concatenate([ready[ready >= self._rr], ready[ready < self._rr]])
            for idx in ready.tolist():
                a, s = divmod(idx, g.slots)
                self.stats["lost_messages"] += int(ahead[idx]) - 1
                self._last[idx] = seq[idx]
                self._rr = idx + 1
                row = self._row(a, s, int(words[idx]))
                if row is None:
                    continue
                rows = self._pending.setdefault((a // g.group, s), {})
                rows[a % g.group] = row
                if len(rows) == g.group:
                    job = self._job(a // g.group, s, self._pending.pop((a // g.group, s)))
                    if job is not None:
                        jobs.append(job)
        return jobs

    def advance(self, a: int, s: int, seq: int) -> None:
        """Device-wait mode: the GPU consumed the doorbell of (a, s) up to ``seq``."""
        with self._lock:
            self._last[a * self.g.slots + s] = seq & SEQ_MASK

    def row_for(self, a: int, s: int, seq: int, n_tokens: int, layer_id: int) -> Row:
        """The Row of a message whose doorbell the device read (device-wait mode)."""
        base = self.recv_base + self.g.region_off(a, s)
        peer = self.peers[a]
        return Row(a, s, seq, peer.epoch, layer_id, n_tokens, base, base + self.g.ids_off, base + self.g.w_off)

    def _row(self, a: int, s: int, word: int) -> Optional[Row]:
        seq, n_tokens, layer_id, epoch = unpack_doorbell(word)
        peer = self.peers.get(a)
        if peer is None:
            self.stats["unknown_peer"] += 1
            return None
        if epoch != peer.epoch:
            self.stats["stale_epoch"] += 1
            return None
        if not 1 <= n_tokens <= self.g.n_max:
            self.stats["bad_doorbell"] += 1
            return None
        base = self.recv_base + self.g.region_off(a, s)
        return Row(a, s, seq, epoch, layer_id, n_tokens, base, base + self.g.ids_off, base + self.g.w_off)

    def _job(self, replica: int, slot: int, rows: Dict[int, Row]) -> Optional[Job]:
        ordered = [rows[j] for j in range(self.g.group)]
        if len({r.layer_id for r in ordered}) > 1:
            self.stats["group_mismatch"] += 1
            return None
        self.stats["jobs"] += 1
        if self._prev_replica is not None and replica != self._prev_replica:
            self.stats["replica_switches"] += 1
        self._prev_replica = replica
        self.trace.append((replica, slot, ordered[0].layer_id))
        return Job(replica, slot, ordered[0].layer_id, ordered, time.monotonic_ns())

    # ---- answer ----
    def reply_target(self, row: Row):
        """(segment address, done-flag address) of the row's answer in its A rank, or None when that A rank
        reconnected since the message was sent (the reply is dropped, server.py:343-346)."""
        peer, g = self.peers.get(row.a), self.g
        if peer is None or peer.epoch != row.epoch:
            self.stats["dropped_replies"] += 1
            return None
        return peer.result_base + g.seg_off(self.f, row.slot), peer.result_base + g.done_off(self.f, row.slot)

    def reply(self, row: Row, src_ptr: int, nbytes: int, stream: int) -> None:
        """Enqueue on ``stream``: copy ``nbytes`` at src_ptr into the A rank's segment, then its done flag."""
        target = self.reply_target(row)
        if target is None:
            return
        seg, done = target
        with torch.cuda.stream(torch.cuda.ExternalStream(stream)):
            _raw_bytes(seg, nbytes, self.device).copy_(_raw_bytes(src_ptr, nbytes, self.device), non_blocking=True)
        N.call("asap_write32", done, row.seq & SEQ_MASK, ctypes.c_void_p(stream))

    def serve_forever(self, handler: Callable[[Job], None], stop: threading.Event, spin_s: float = 0.005,
                      idle_sleep_s: float = 0.0002) -> None:
        """Poll and hand every complete job to ``handler`` until ``stop`` is set (server.py:352-377)."""
        sys.setswitchinterval(1e-5)
        self.mem.activate()
        last_job = time.monotonic()
        while not stop.is_set():
            jobs = self.poll()
            for job in jobs:
                handler(job)
            if jobs:
                last_job = time.monotonic()
            elif idle_sleep_s and time.monotonic() - last_job > spin_s:
                time.sleep(idle_sleep_s)

    def unmap_peers(self) -> None:
        """Unmap every connected A rank's ResultArena (see AttnChannel.unmap_peers)."""
        for peer in self.peers.values():
            peer.mapping.release()

    def close(self) -> None:
        """Stop the handshake thread, unmap the A arenas, free the doorbell page and the RecvArena."""
        if self._hs_thread is not None:
            self._hs_stop.set()
            self._hs_thread.join(timeout=2.0)
            self._srv.close()
            self._hs_thread = None
        for peer in self.peers.values():
            peer.mapping.release()
        self.peers.clear()
        self._bells = None
        self._page.release()
        self._recv.release()


class _CudaArray:
    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 2}


def _raw_bytes(ptr: int, nbytes: int, device: int) -> torch.Tensor:
    """A uint8 tensor aliasing raw device memory (not owned)."""
    return torch.as_tensor(_CudaArray(ptr, nbytes), device=f"cuda:{device}")
