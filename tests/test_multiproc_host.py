"""The N>1 host path on CPU: an A rank and an F rank in two processes (world size 2, gloo for coordination),
talking the real protocol -- the JSON-over-TCP handshake (transport/server.py:181-259 validation, epochs), the
doorbell page shared through /dev/shm, the F poll (cyclic seq, lost messages, stale epochs, round robin), replies
into the A rank's ResultArena, reconnect -- with a host-memory stand-in for the device arenas (no GPU: the kernels'
stores are emulated by plain host stores of the same words at the same offsets)."""

import ctypes
import os
import socket
import tempfile

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as tmp

from asap_b200.transport.layout import Geometry, HandshakeError, pack_doorbell
from host_mem import HostMem

G = Geometry(num_a=2, group=1, slots=2, n_max=64, hidden=256, topk=2, num_f=1)
MODEL = {"hidden": 256, "topk": 2, "n_experts": 8}


def u64(addr):
    return ctypes.c_uint64.from_address(addr)


def u32(addr):
    return ctypes.c_uint32.from_address(addr)


def _run(rank, world, port0, run_dir, errq):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port0))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        if rank == 0:
            _f_rank(run_dir)
        else:
            _a_rank(run_dir)
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as exc:  # noqa: BLE001
        import traceback

        errq.put(f"rank {rank}: {exc!r}\n{traceback.format_exc()}")
        raise


def _f_rank(run_dir):
    from asap_b200.transport.server import FfnServer

    srv = FfnServer(0, G, device=0, run_dir=run_dir, host="127.0.0.1", port=0, model=MODEL)
    srv.mem = HostMem(run_dir)
    srv.start()
    obj = [srv.port]
    dist.broadcast_object_list(obj, src=0)
    dist.barrier()  # A rank 1 connected, rang slot 0 and slot 1
    jobs = srv.poll()
    assert [(j.replica, j.slot, j.layer_id) for j in jobs] == [(1, 0, 3), (1, 1, 4)], jobs
    row = jobs[0].rows[0]
    assert (row.a, row.seq, row.epoch, row.n_tokens) == (1, 1, 1, 5)
    assert row.x_ptr == srv.recv_base + G.region_off(1, 0)
    assert row.ids_ptr == row.x_ptr + G.ids_off and row.w_ptr == row.x_ptr + G.w_off
    # reply: F writes the partial row and the done flag into A's ResultArena through its mapping
    seg, done = srv.reply_target(row)
    np.ctypeslib.as_array((ctypes.c_uint16 * 4).from_address(seg))[:] = [1, 2, 3, 4]
    u32(done).value = row.seq
    assert srv.poll() == []  # nothing new
    dist.barrier()  # replied
    dist.barrier()  # A: skipped a seq, sent a stale epoch, an unknown rank rang
    jobs = srv.poll()
    assert [(j.replica, j.slot) for j in jobs] == [(1, 0)], jobs
    assert srv.stats["lost_messages"] == 1
    assert srv.stats["stale_epoch"] == 1
    assert srv.stats["unknown_peer"] == 1
    dist.barrier()  # polled: A may reconnect now
    dist.barrier()  # A reconnected
    assert srv.peers[1].epoch == 2 and srv.stats["reconnects"] == 1
    jobs = srv.poll()
    assert [j.rows[0].epoch for j in jobs] == [2]
    assert srv.reply_target(row) is None and srv.stats["dropped_replies"] == 1  # old-epoch reply is dropped
    dist.barrier()
    srv.unmap_peers()
    dist.barrier()
    srv.close()


def _a_rank(run_dir):
    from asap_b200.transport.channel import AttnChannel
    from asap_b200.transport.wire import exchange as request

    obj = [None]
    dist.broadcast_object_list(obj, src=0)
    port = obj[0]
    ch = AttnChannel(1, G, [("127.0.0.1", port)], device=0, hello={"model": MODEL}, connect_timeout_s=20.0)
    ch.mem = HostMem(run_dir)
    ch.connect()
    assert ch.epochs == [1] and ch.expert_bounds == [0, 8]
    flags = np.ctypeslib.as_array((ctypes.c_uint32 * (G.flags_bytes // 4)).from_address(ch.result_base))
    assert (flags == 0).all()  # seq_base
    bell = ch.bell_bases[0]
    u64(bell + G.bell_off(1, 0)).value = pack_doorbell(1, 5, 3, 1)
    u64(bell + G.bell_off(1, 1)).value = pack_doorbell(1, 7, 4, 1)
    dist.barrier()
    dist.barrier()  # F replied
    assert u32(ch.result_base + G.done_off(0, 0)).value == 1
    assert list(np.ctypeslib.as_array((ctypes.c_uint16 * 4).from_address(ch.result_base + G.seg_off(0, 0)))) == [
        1, 2, 3, 4]
    u64(bell + G.bell_off(1, 0)).value = pack_doorbell(3, 2, 3, 1)    # seq 2 never rang: one lost message
    u64(bell + G.bell_off(1, 1)).value = pack_doorbell(2, 2, 4, 9)    # epoch 9 is not this rank's
    u64(bell + G.bell_off(0, 0)).value = pack_doorbell(1, 2, 3, 1)    # A rank 0 never connected
    # handshake rejections carry the reason back
    bad = {"proto": 4, "a": 1, "geometry": {**G.as_dict(), "hidden": 512}, "memory": "ipc",
           "peer": {"host": socket.gethostname()}, "result": {}, "model": MODEL}
    with pytest.raises(HandshakeError, match="geometry mismatch"):
        request("127.0.0.1", port, bad, connect_timeout=5)
    other = {**bad, "geometry": G.as_dict(), "peer": {"host": "another-host"}}
    with pytest.raises(HandshakeError, match="needs one host|claims it too"):
        request("127.0.0.1", port, other, connect_timeout=5)
    with pytest.raises(HandshakeError, match="protocol version"):
        request("127.0.0.1", port, {**bad, "proto": 3}, connect_timeout=5)
    dist.barrier()  # F polls the doorbells above
    dist.barrier()
    ch.reconnect()
    assert ch.epochs == [2]
    u64(ch.bell_bases[0] + G.bell_off(1, 0)).value = pack_doorbell(1, 3, 5, 2)
    dist.barrier()
    dist.barrier()
    ch.unmap_peers()
    dist.barrier()
    ch.close()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_two_process_handshake_doorbells_replies_reconnect():
    run_dir = tempfile.mkdtemp(dir="/dev/shm" if os.access("/dev/shm", os.W_OK) else None)
    ctx = tmp.get_context("spawn")
    errq = ctx.Queue()
    port0 = _free_port()
    procs = [ctx.Process(target=_run, args=(r, 2, port0, run_dir, errq)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    errors = []
    while not errq.empty():
        errors.append(errq.get())
    assert not alive, "a rank did not finish"
    assert not errors, "\n".join(errors)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
