"""Joined F jobs: one expert chain answering several messages at once (asap_ffn_post_rows / asap_ffn_wait_rows /
asap_ffn_job_rows).  Each message's reply must equal the oracle's answer to that message alone (the output of a
token depends on that token only), its done flag must carry its own seq, and the expert counts are those of all
rows' pairs together (bit-exact).  Then two A replicas' messages through the real transport answered by one job
on one F rank (one GPU: the F chain runs after events recorded behind both dispatches, so no kernel spins on
another kernel of this GPU)."""

import ctypes

import numpy as np
import pytest
import torch

from asap_b200 import _native as N
from asap_b200.experts import Fp8Experts, Mxfp4Experts, _aligned_empty
from asap_b200.scheduler import FfnScheduler
from asap_b200.transport.channel import AttnChannel
from asap_b200.transport.layout import Geometry, pack_doorbell
from asap_b200.transport.server import FfnServer
from gpu_util import bf16_tensor_from_np, device_bytes, experts_to_oracle, np_from_bf16, random_inputs
from oracle import moe, mx

pytestmark = pytest.mark.gpu
TOL = 1e-2


class Rows:
    """Several messages' x/ids/w as separate device buffers, with a reply segment and done flag each."""

    def __init__(self, rng, sizes, H, k, e_lo, e_hi):
        self.msgs = [random_inputs(rng, n, H, k, e_lo, e_hi) for n in sizes]
        self.dev = [(bf16_tensor_from_np(x), torch.from_numpy(i).cuda(), torch.from_numpy(w).cuda())
                    for x, i, w in self.msgs]
        self.reply = [torch.zeros(n, H, dtype=torch.bfloat16, device="cuda") for n in sizes]
        self.done = torch.zeros(16 * len(sizes), dtype=torch.int32, device="cuda")

    def views(self):
        R = len(self.msgs)
        return (N.FfnRow_t * R)(*[N.FfnRow_t(x.data_ptr(), i.data_ptr(), w.data_ptr(), self.reply[r].data_ptr(),
                                             self.done.data_ptr() + 64 * r)
                                  for r, (x, i, w) in enumerate(self.dev)])


def make_ws(e, cap, k):
    nbytes = N.lib().asap_ffn_ws_bytes(cap, k, e.num_local, e.hidden, e.inter)
    owner, ws = _aligned_empty(nbytes, "cuda")
    h = ctypes.c_uint64()
    N.call("asap_ffn_ws_register", ws.data_ptr(), cap, k, e.num_local, e.hidden, e.inter, ctypes.byref(h))
    return owner, ws, h.value


def check_rows(rows, e, e0, P, act, seqs):
    gate, up, w2 = experts_to_oracle(e)
    for r, (x, ids, w) in enumerate(rows.msgs):
        ref = moe.ffn_rank(x, ids, w, gate, up, w2, e0, P, act_quant=act)
        assert moe.rel_l2(np_from_bf16(rows.reply[r]), ref) < TOL, r
        assert int(rows.done[16 * r].item()) == seqs[r]


@pytest.mark.parametrize("kind", ["mxfp4", "fp8"])
def test_posted_rows_each_answered_alone(cuda_ok, kind):
    rng = np.random.default_rng(3)
    H, I, k, P, e0 = 256, 128, 4, 8, 0
    sizes = [50, 1, 200]
    e = (Mxfp4Experts.random(P, H, I, seed=2) if kind == "mxfp4" else Fp8Experts.random(P, H, I, seed=2))
    rows = Rows(rng, sizes, H, k, e0 - 2, e0 + P + 2)
    owner, ws, wh = make_ws(e, sum(sizes), k)
    status = torch.zeros(1, dtype=torch.int64, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    seqs = [11, 7, 901]
    R = len(sizes)
    N.call("asap_ffn_post_rows", wh, R, (ctypes.c_uint32 * R)(*seqs), (ctypes.c_int32 * R)(*sizes), 3,
           (ctypes.c_int32 * R)(1, 1, 1), stream)
    N.call("asap_ffn_job_rows", e.handle, wh, R, rows.views(), ctypes.c_float(0.0), status.data_ptr(), int(5e9),
           stream)
    torch.cuda.synchronize()
    assert int(status.item()) == 0, N.decode_status(int(status.item()))
    check_rows(rows, e, e0, P, "fp8" if kind == "fp8" else True, seqs)
    # counts over every row's pairs together, bit-exact
    ecnt = ctypes.c_uint64()
    N.call("asap_ffn_debug_ptrs", wh, ctypes.byref(ecnt), *[None] * 6)
    all_ids = np.concatenate([m[1] for m in rows.msgs])
    np.testing.assert_array_equal(device_bytes(ecnt.value, 4 * P).view(np.int32), moe.expert_counts(all_ids, e0, P))
    N.call("asap_ffn_ws_release", wh)
    e.release()


def test_device_wait_rows_and_layer_mismatch(cuda_ok):
    rng = np.random.default_rng(4)
    H, I, k, P = 256, 128, 2, 4
    sizes = [30, 70]
    e = Mxfp4Experts.random(P, H, I, seed=3)
    rows = Rows(rng, sizes, H, k, 0, P)
    owner, ws, wh = make_ws(e, sum(sizes), k)
    status = torch.zeros(1, dtype=torch.int64, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    # the doorbells are already rung when the wait runs (device words written before the launch)
    bells = torch.zeros(16, dtype=torch.int64, device="cuda")
    bells[0] = pack_doorbell(5, sizes[0], 2, 1)
    bells[8] = pack_doorbell(9, sizes[1], 2, 1)
    R = 2
    addrs = (ctypes.c_uint64 * R)(bells.data_ptr(), bells.data_ptr() + 64)
    N.call("asap_ffn_wait_rows", wh, R, addrs, (ctypes.c_uint32 * R)(4, 8), (ctypes.c_int32 * R)(1, 1), sum(sizes),
           status.data_ptr(), int(2e9), stream)
    N.call("asap_ffn_job_rows", e.handle, wh, R, rows.views(), ctypes.c_float(0.0), status.data_ptr(), int(5e9),
           stream)
    torch.cuda.synchronize()
    assert int(status.item()) == 0, N.decode_status(int(status.item()))
    check_rows(rows, e, 0, P, True, [5, 9])
    # rows naming different layers: the job is refused (BAD_JOB) and answers nothing
    rows.done.zero_()
    bells[0] = pack_doorbell(6, sizes[0], 2, 1)
    bells[8] = pack_doorbell(10, sizes[1], 3, 1)
    N.call("asap_ffn_wait_rows", wh, R, addrs, (ctypes.c_uint32 * R)(5, 9), (ctypes.c_int32 * R)(1, 1), sum(sizes),
           status.data_ptr(), int(2e9), stream)
    N.call("asap_ffn_job_rows", e.handle, wh, R, rows.views(), ctypes.c_float(0.0), status.data_ptr(), int(5e9),
           stream)
    torch.cuda.synchronize()
    st = N.decode_status(int(status.item()))
    assert st["what"] == "bad job", st
    assert int(rows.done.abs().sum().item()) == 0
    N.call("asap_ffn_ws_release", wh)
    e.release()


def test_two_replicas_one_joined_job(cuda_ok):
    """Two A replicas (two AttnChannels, A ranks 0 and 1) send to one F rank; one joined job answers both."""
    import os
    import tempfile

    # the doorbell page must be a tmpfs file: a disk-backed mapping cannot be registered with the GPU
    run_dir = tempfile.mkdtemp(dir="/dev/shm" if os.access("/dev/shm", os.W_OK) else None)
    rng = np.random.default_rng(5)
    T, H, I, k, E = 120, 256, 128, 4, 8
    g = Geometry(2, 1, 2, T, H, k, 1)
    experts = Mxfp4Experts.random(E, H, I, seed=6)
    srv = FfnServer(0, g, device=0, run_dir=run_dir, listen=False).start()
    chans = [AttnChannel(a, g, [("in-process", 0)], device=0, timeout_s=5.0, expert_bounds=[0, E],
                         _connector=lambda f, hello: srv.handshake(hello)).connect() for a in range(2)]
    sched = FfnScheduler(srv, {0: experts}, timeout_s=5.0, join=2)
    try:
        gate, up, w2 = experts_to_oracle(experts)
        f_stream = torch.cuda.Stream()
        send = [torch.cuda.Stream() for _ in range(2)]
        stream = torch.cuda.current_stream()
        for seq in (1, 2):  # two rounds on slot 1
            msgs = [random_inputs(rng, n, H, k, 0, E) for n in (T, T // 3)]
            dev = [(bf16_tensor_from_np(x), torch.from_numpy(i).cuda(), torch.from_numpy(w).cuda()) for x, i, w in msgs]
            tickets, sent = [], []
            for a in range(2):
                x, i, w = dev[a]
                send[a].wait_stream(stream)
                tickets.append(chans[a].send(0, 1, x.data_ptr(), i.data_ptr(), w.data_ptr(), x.shape[0],
                                             send[a].cuda_stream))
                ev = torch.cuda.Event()
                ev.record(send[a])
                sent.append(ev)
            for ev in sent:
                f_stream.wait_event(ev)
            sched.run_device_wait_rows([(0, 1, seq), (1, 1, seq)], 0, f_stream.cuda_stream)
            done = torch.cuda.Event()
            done.record(f_stream)
            stream.wait_event(done)
            outs = []
            for a in range(2):
                out = torch.empty(dev[a][0].shape, dtype=torch.bfloat16, device="cuda")
                chans[a].combine(tickets[a], out.data_ptr(), stream.cuda_stream)
                outs.append(out)
            torch.cuda.synchronize()
            sched.check()
            for a in range(2):
                chans[a].check()
                x, ids, w = msgs[a]
                ref = moe.round_trip(x, ids, w, [0, E], [(gate, up, w2)])
                assert moe.rel_l2(np_from_bf16(outs[a]), ref) < TOL, (seq, a)
            assert sched.job_info()["n"] == T + T // 3
    finally:
        torch.cuda.synchronize()
        sched.close()
        for ch in chans:
            ch.close()
        srv.close()
        experts.release()


@pytest.mark.parametrize("graph", [False, True])
def test_round_robin_any_ready_message(cuda_ok, graph):
    """asap_ffn_wait_any: each job answers the first ready message among the sources, in round-robin order after
    the source answered last.  Only A rank 1 has sent -> the job answers A1 (A0's flag untouched); then A0 sends ->
    the next job answers A0; then both send -> A1 first (round robin after A0), then A0."""
    import os
    import tempfile

    run_dir = tempfile.mkdtemp(dir="/dev/shm" if os.access("/dev/shm", os.W_OK) else None)
    rng = np.random.default_rng(12)
    T, H, I, k, E = 64, 256, 128, 2, 8
    g = Geometry(2, 1, 2, T, H, k, 1)
    experts = Mxfp4Experts.random(E, H, I, seed=7)
    srv = FfnServer(0, g, device=0, run_dir=run_dir, listen=False).start()
    chans = [AttnChannel(a, g, [("in-process", 0)], device=0, timeout_s=5.0, expert_bounds=[0, E],
                         _connector=lambda f, hello: srv.handshake(hello)).connect() for a in range(2)]
    sched = FfnScheduler(srv, {0: experts}, timeout_s=5.0)
    gate, up, w2 = experts_to_oracle(experts)
    f_stream = torch.cuda.Stream()
    stream = torch.cuda.current_stream()
    sources = [(0, 0), (1, 0)]
    keep = []

    def send(a):
        x, ids, w = random_inputs(rng, T - 3 * a, H, k, 0, E)
        dev = (bf16_tensor_from_np(x), torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda())
        keep.append(dev)
        t = chans[a].send(0, 0, dev[0].data_ptr(), dev[1].data_ptr(), dev[2].data_ptr(), dev[0].shape[0],
                          stream.cuda_stream)
        return t, (x, ids, w)

    def answer():  # one round-robin job, ordered after everything sent so far (no cross-kernel spin)
        f_stream.wait_stream(stream)
        sched.run_device_wait_any(sources, 0, f_stream.cuda_stream, graph=graph)
        torch.cuda.synchronize()
        sched.check()

    def check(a, t, msg):
        out = torch.empty(msg[0].shape, dtype=torch.bfloat16, device="cuda")
        chans[a].combine(t, out.data_ptr(), stream.cuda_stream)
        torch.cuda.synchronize()
        chans[a].check()
        ref = moe.round_trip(*msg, [0, E], [(gate, up, w2)])
        assert moe.rel_l2(np_from_bf16(out), ref) < TOL

    try:
        t1, m1 = send(1)
        answer()
        info = sched.job_info()
        assert info["n"] == T - 3 and info["seq"] == 1  # A rank 1's message
        check(1, t1, m1)
        t0, m0 = send(0)
        answer()
        assert sched.job_info()["n"] == T
        check(0, t0, m0)
        t0, m0 = send(0)
        t1, m1 = send(1)
        answer()
        assert sched.job_info()["n"] == T - 3  # round robin: A1 after A0
        answer()
        assert sched.job_info()["n"] == T
        check(0, t0, m0)
        check(1, t1, m1)
        if graph:
            assert sched.graph_replays == 4 and len(sched._graphs) == 1
    finally:
        torch.cuda.synchronize()
        sched.close()
        for ch in chans:
            ch.close()
        srv.close()
        experts.release()


def test_first_message_then_the_rest(cuda_ok):
    """asap_ffn_wait_rest after asap_ffn_wait_any: three A replicas send one message each; the first job answers
    one of them, the second answers the other two together (its token count is theirs), every combined output
    matches the oracle.  In a second round three any-jobs answer all three messages, so the rest-job that follows
    finds nothing left: an empty job, with no error and no reply."""
    import os
    import tempfile

    run_dir = tempfile.mkdtemp(dir="/dev/shm" if os.access("/dev/shm", os.W_OK) else None)
    rng = np.random.default_rng(21)
    T, H, I, k, E = 96, 256, 128, 4, 8
    sizes = (T, T - 5, T - 11)
    g = Geometry(3, 1, 1, T, H, k, 1)
    experts = Mxfp4Experts.random(E, H, I, seed=8)
    srv = FfnServer(0, g, device=0, run_dir=run_dir, listen=False).start()
    chans = [AttnChannel(a, g, [("in-process", 0)], device=0, timeout_s=5.0, expert_bounds=[0, E],
                         _connector=lambda f, hello: srv.handshake(hello)).connect() for a in range(3)]
    sched = FfnScheduler(srv, {0: experts}, timeout_s=5.0, join=3)
    gate, up, w2 = experts_to_oracle(experts)
    f_stream = torch.cuda.Stream()
    stream = torch.cuda.current_stream()
    sources = [(a, 0) for a in range(3)]
    keep = []

    def send_all():
        sent = []
        for a in range(3):
            x, ids, w = random_inputs(rng, sizes[a], H, k, 0, E)
            dev = (bf16_tensor_from_np(x), torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda())
            keep.append(dev)
            t = chans[a].send(0, 0, dev[0].data_ptr(), dev[1].data_ptr(), dev[2].data_ptr(), sizes[a],
                              stream.cuda_stream)
            sent.append((t, (x, ids, w)))
        f_stream.wait_stream(stream)  # the F jobs run after every send (no kernel spins on another of this GPU)
        return sent

    def check_all(sent):
        for a, (t, msg) in enumerate(sent):
            out = torch.empty(sizes[a], H, dtype=torch.bfloat16, device="cuda")
            chans[a].combine(t, out.data_ptr(), stream.cuda_stream)
            torch.cuda.synchronize()
            chans[a].check()
            ref = moe.round_trip(*msg, [0, E], [(gate, up, w2)])
            assert moe.rel_l2(np_from_bf16(out), ref) < TOL, a

    try:
        sent = send_all()
        sched.run_device_wait_any(sources, 0, f_stream.cuda_stream)
        torch.cuda.synchronize()
        first = sched.job_info()["n"]
        assert first in sizes
        sched.run_device_wait_rest([(a, 0, 1) for a in range(3)], 0, f_stream.cuda_stream)
        torch.cuda.synchronize()
        sched.check()
        info = sched.job_info()
        assert info["valid"] == 1 and info["n"] == sum(sizes) - first
        check_all(sent)
        sent = send_all()
        for _ in range(3):
            sched.run_device_wait_any(sources, 0, f_stream.cuda_stream)
        sched.run_device_wait_rest([(a, 0, 2) for a in range(3)], 0, f_stream.cuda_stream)
        torch.cuda.synchronize()
        sched.check()
        assert sched.job_info()["valid"] == 0  # nothing left this round: an empty job
        check_all(sent)
    finally:
        torch.cuda.synchronize()
        sched.close()
        for ch in chans:
            ch.close()
        srv.close()
        experts.release()


def test_overlapped_replies_alternate_workspaces(cuda_ok):
    """FfnScheduler(overlap_replies=k): a job's reduce + reply runs on a side stream (k SMs left to it, the GEMMs
    on the rest) while the next job computes, and consecutive jobs alternate between two workspaces.  Three A
    replicas, two rounds of three round-robin jobs (the first two of each round overlapped): every combined output
    matches the oracle and every done flag carries its message's seq."""
    import os
    import tempfile

    run_dir = tempfile.mkdtemp(dir="/dev/shm" if os.access("/dev/shm", os.W_OK) else None)
    rng = np.random.default_rng(33)
    T, H, I, k, E = 128, 256, 128, 4, 8
    sizes = (T, T - 7, T - 20)
    g = Geometry(3, 1, 1, T, H, k, 1)
    experts = Mxfp4Experts.random(E, H, I, seed=9)
    srv = FfnServer(0, g, device=0, run_dir=run_dir, listen=False).start()
    chans = [AttnChannel(a, g, [("in-process", 0)], device=0, timeout_s=5.0, expert_bounds=[0, E],
                         _connector=lambda f, hello: srv.handshake(hello)).connect() for a in range(3)]
    sched = FfnScheduler(srv, {0: experts}, timeout_s=5.0, overlap_replies=8)
    gate, up, w2 = experts_to_oracle(experts)
    f_stream = torch.cuda.Stream()
    stream = torch.cuda.current_stream()
    sources = [(a, 0) for a in range(3)]
    keep = []
    try:
        assert len(sched._wss) == 2
        for rnd in range(2):
            sent = []
            for a in range(3):
                x, ids, w = random_inputs(rng, sizes[a], H, k, 0, E)
                dev = (bf16_tensor_from_np(x), torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda())
                keep.append(dev)
                t = chans[a].send(0, 0, dev[0].data_ptr(), dev[1].data_ptr(), dev[2].data_ptr(), sizes[a],
                                  stream.cuda_stream)
                sent.append((t, (x, ids, w)))
            f_stream.wait_stream(stream)  # the F jobs run after every send (no kernel spins on another here)
            for i in range(3):
                sched.run_device_wait_any(sources, 0, f_stream.cuda_stream, overlap=i < 2)
            torch.cuda.synchronize()
            sched.check()
            for a, (t, msg) in enumerate(sent):
                out = torch.empty(sizes[a], H, dtype=torch.bfloat16, device="cuda")
                chans[a].combine(t, out.data_ptr(), stream.cuda_stream)
                torch.cuda.synchronize()
                chans[a].check()
                ref = moe.round_trip(*msg, [0, E], [(gate, up, w2)])
                assert moe.rel_l2(np_from_bf16(out), ref) < TOL, (rnd, a)
    finally:
        torch.cuda.synchronize()
        sched.close()
        for ch in chans:
            ch.close()
        srv.close()
        experts.release()
