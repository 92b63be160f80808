"""The F rank's host poll and handshake in one process (FfnServer over plain host buffers, no GPU, no sockets):
the behaviours the reference's transport/server.py pins -- epoch cycling (old % 31) + 1 on reconnect
(server.py:237), the cyclic int32 seq comparison with lost messages counted as ahead - 1 (server.py:278-280),
round robin over the ready doorbells starting after the last one served (server.py:270-275), stale epochs,
unknown A ranks and out-of-range token counts dropped, and group-joined jobs (server.py:296-337)."""

import ctypes

import pytest

from asap_b200.transport.layout import MAX_EPOCH, PROTO_VERSION, Geometry, pack_doorbell
from asap_b200.transport.memory import Shared
from asap_b200.transport.server import FfnServer


class FakeMem:
    """Host buffers in place of device arenas and the doorbell page."""

    kind, reason = "ipc", "host test stand-in"

    def __init__(self):
        self.keep = []

    def _buf(self, nbytes):
        b = (ctypes.c_uint8 * nbytes)()
        self.keep.append(b)
        return ctypes.addressof(b)

    def activate(self):
        pass

    def device(self, nbytes):
        return Shared(self._buf(nbytes), lambda: None, {"bytes": nbytes})

    def doorbells(self, nbytes, path, device_access=True):
        addr = self._buf(nbytes)
        return Shared(addr, lambda: None, {"path": path}, dev=addr)

    def fill32(self, ptr, value, count):
        (ctypes.c_uint32 * count).from_address(ptr)[:] = [value & 0xFFFFFFFF] * count

    def check_peer(self, peer):
        pass

    def open(self, desc):
        return Shared(self._buf(4096), lambda: None)


def server(g):
    srv = FfnServer(0, g, device=0, run_dir="/tmp", listen=False, model={"hidden": g.hidden})
    srv.mem = FakeMem()
    return srv.start()


def hello(g, a):
    return {"proto": PROTO_VERSION, "a": a, "geometry": g.as_dict(), "memory": "ipc", "peer": {}, "result": {},
            "model": {"hidden": g.hidden}, "pid": 1}


def ring(srv, a, s, seq, n, layer, epoch):
    srv.bell_words[a * srv.g.slots + s] = pack_doorbell(seq, n, layer, epoch)


def test_epoch_cycles_through_31():
    g = Geometry(num_a=1, group=1, slots=1, n_max=16, hidden=64, topk=2, num_f=1)
    srv = server(g)
    epochs = [srv.handshake(hello(g, 0))["epoch"] for _ in range(MAX_EPOCH + 2)]
    assert epochs[:3] == [1, 2, 3]
    assert epochs[MAX_EPOCH - 1] == MAX_EPOCH and epochs[MAX_EPOCH] == 1 and epochs[MAX_EPOCH + 1] == 2
    assert srv.stats["reconnects"] == MAX_EPOCH + 1


def test_round_robin_after_last_served():
    g = Geometry(num_a=4, group=1, slots=1, n_max=16, hidden=64, topk=2, num_f=1)
    srv = server(g)
    for a in range(4):
        srv.handshake(hello(g, a))
    ring(srv, 2, 0, 1, 3, 0, 1)
    assert [j.replica for j in srv.poll()] == [2]           # next poll starts after index 2
    for a in range(4):
        ring(srv, a, 0, 2 if a == 2 else 1, 3, 0, 1)
    assert [j.replica for j in srv.poll()] == [3, 0, 1, 2]  # 3 first, then wrap around
    ring(srv, 0, 0, 2, 3, 0, 1)
    ring(srv, 1, 0, 2, 3, 0, 1)
    assert [j.replica for j in srv.poll()] == [0, 1]        # after 2: 3 is idle, so 0 then 1
    assert srv.stats["lost_messages"] == 0


def test_cyclic_seq_lost_messages_and_drops():
    g = Geometry(num_a=2, group=1, slots=2, n_max=16, hidden=64, topk=2, num_f=1)
    srv = FfnServer(0, g, device=0, run_dir="/tmp", listen=False, seq_base=0xFFFFFFFE, model={"hidden": 64})
    srv.mem = FakeMem()
    srv.start()
    srv.handshake(hello(g, 1))
    ring(srv, 1, 0, 0xFFFFFFFF, 4, 7, 1)            # one past seq_base: the next message
    jobs = srv.poll()
    assert [(j.replica, j.slot, j.layer_id, j.rows[0].n_tokens) for j in jobs] == [(1, 0, 7, 4)]
    ring(srv, 1, 0, 2, 4, 7, 1)                     # 0xFFFFFFFF -> 2 across the wrap: seqs 0 and 1 never rang
    assert len(srv.poll()) == 1 and srv.stats["lost_messages"] == 2
    ring(srv, 1, 0, 1, 4, 7, 1)                     # behind the last seen (int32 difference < 0): ignored
    assert srv.poll() == [] and srv.stats["lost_messages"] == 2
    ring(srv, 1, 1, 0xFFFFFFFF, 4, 7, 9)            # wrong epoch
    ring(srv, 0, 0, 0xFFFFFFFF, 4, 7, 1)            # A rank 0 never connected
    assert srv.poll() == []
    assert srv.stats["stale_epoch"] == 1 and srv.stats["unknown_peer"] == 1
    ring(srv, 1, 1, 0, 17, 7, 1)                    # n_tokens above n_max
    assert srv.poll() == [] and srv.stats["bad_doorbell"] == 1


def test_group_joined_jobs():
    """An attention TP group of 2: one job per (replica, slot) once both ranks' rows arrived; rows of different
    layers are dropped as a group mismatch."""
    g = Geometry(num_a=4, group=2, slots=1, n_max=16, hidden=64, topk=2, num_f=1)
    srv = server(g)
    for a in range(4):
        srv.handshake(hello(g, a))
    ring(srv, 1, 0, 1, 5, 3, 1)
    assert srv.poll() == []                          # rank 0 of replica 0 not there yet
    ring(srv, 0, 0, 1, 5, 3, 1)
    jobs = srv.poll()
    assert [(j.replica, [r.a for r in j.rows]) for j in jobs] == [(0, [0, 1])]
    ring(srv, 2, 0, 1, 5, 3, 1)
    ring(srv, 3, 0, 1, 5, 4, 1)                      # same replica, other layer
    assert srv.poll() == [] and srv.stats["group_mismatch"] == 1
    assert srv.stats["jobs"] == 1


def test_handshake_rejections():
    g = Geometry(num_a=2, group=1, slots=1, n_max=16, hidden=64, topk=2, num_f=1)
    srv = server(g)
    from asap_b200.transport.layout import HandshakeError

    with pytest.raises(HandshakeError, match="protocol version"):
        srv.handshake({**hello(g, 0), "proto": PROTO_VERSION - 1})
    with pytest.raises(HandshakeError, match="geometry mismatch"):
        srv.handshake({**hello(g, 0), "geometry": {**g.as_dict(), "topk": 4}})
    with pytest.raises(HandshakeError, match="differ"):
        srv.handshake({**hello(g, 0), "model": {"hidden": 128}})
    with pytest.raises(HandshakeError, match="outside"):
        srv.handshake(hello(g, 2))
    assert srv.handshake(hello(g, 1))["epoch"] == 1
