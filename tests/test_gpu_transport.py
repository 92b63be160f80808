"""A-side dispatch and combine kernels through the C ABI, against the oracle: arena bytes of every F rank's
region (compacted rows of x, ids, weights) and the doorbell words bit-exact, the routing table bit-exact, the
combine bit-exact given the F replies; plus the bounded device waits (backpressure, reply, doorbell) running
out on a flag nothing sets and reporting their status instead of hanging."""

import ctypes

import numpy as np
import pytest
import torch

from asap_b200 import _native as N
from asap_b200.transport.layout import Geometry, pack_doorbell
from gpu_util import bf16_tensor_from_np, np_from_bf16
from oracle import moe, mx

pytestmark = pytest.mark.gpu


class FakeDeployment:
    """One A rank and ``num_f`` F ranks' memory in this process: RecvArenas and doorbell pages as plain device
    buffers, the A rank's ResultArena, a routing workspace."""

    def __init__(self, g: Geometry, bounds, a=0):
        self.g, self.bounds, self.a = g, list(bounds), a
        dev = "cuda"
        self.recv = [torch.zeros(g.recv_bytes, dtype=torch.uint8, device=dev) for _ in range(g.num_f)]
        self.bells = [torch.zeros(g.host_bytes // 8, dtype=torch.int64, device=dev) for _ in range(g.num_f)]
        self.result = torch.zeros(g.result_bytes, dtype=torch.uint8, device=dev)
        gs = N.geometry_struct(g)
        self.gs = gs
        self.ws = torch.zeros(N.lib().asap_route_ws_bytes(ctypes.byref(gs)), dtype=torch.uint8, device=dev)
        self.status = torch.zeros(1, dtype=torch.int64, device=dev)

    def dispatch(self, seq, layer, x, ids, w, epochs=None, backpressure=True, timeout_s=2.0, ids64=False,
                 wbf16=False):
        g, F = self.g, self.g.num_f
        epochs = epochs or [1] * F
        args = (ctypes.byref(self.gs), self.a, 0, seq, layer, (ctypes.c_int32 * F)(*epochs),
                x.data_ptr(), ids.data_ptr(), int(ids64), w.data_ptr(), int(wbf16), x.shape[0],
                (ctypes.c_int32 * (F + 1))(*self.bounds), (ctypes.c_uint64 * F)(*[r.data_ptr() for r in self.recv]),
                (ctypes.c_uint64 * F)(*[b.data_ptr() for b in self.bells]), self.result.data_ptr(),
                self.ws.data_ptr(), int(backpressure), self.status.data_ptr(), int(timeout_s * 1e9),
                ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        N.call("asap_dispatch", *args)

    def done_flags(self):
        return self.result[: self.g.flags_bytes].view(torch.int32)

    def set_done(self, f, slot, seq):
        self.done_flags()[self.g.done_off(f, slot) // 4] = seq

    def region(self, f, slot=0):
        g = self.g
        base = g.region_off(self.a, slot)
        return self.recv[f][base: base + g.region_bytes]

    def seg(self, f, slot=0):
        g = self.g
        off = g.seg_off(f, slot)
        return self.result[off: off + g.n_max * g.hidden * 2].view(torch.bfloat16).view(g.n_max, g.hidden)

    def combine(self, seq, n, shared=None, timeout_s=2.0):
        out = torch.empty(n, self.g.hidden, dtype=torch.bfloat16, device="cuda")
        N.call("asap_combine", ctypes.byref(self.gs), 0, seq, n, self.result.data_ptr(), self.ws.data_ptr(),
               0 if shared is None else shared.data_ptr(), out.data_ptr(), self.status.data_ptr(),
               int(timeout_s * 1e9), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        return out


@pytest.mark.parametrize("n,H,k,bounds", [
    (100, 256, 4, [0, 8, 8, 20, 32]),        # uneven ranges, one F rank owns nothing (padding row)
    (1, 512, 2, [0, 16, 32]),               # a single token
    (2048, 7168, 8, [0, 64, 128, 192, 256]),  # 4A4F-shaped dispatch (DeepSeek-V3 hidden, top-8)
])
@pytest.mark.parametrize("ids64", [False, True])
def test_dispatch_arena_bytes_and_combine(cuda_ok, n, H, k, bounds, ids64):
    rng = np.random.default_rng(n + 7 * len(bounds))
    F = len(bounds) - 1
    E = bounds[-1]
    g = Geometry(1, 1, 2, max(n, 4), H, k, F)
    d = FakeDeployment(g, bounds)
    x = mx.bf16_round(rng.standard_normal((n, H)).astype(np.float32))
    ids = np.stack([rng.permutation(E + 2)[:k] - 1 for _ in range(n)]).astype(np.int64)  # -1 and E: nowhere
    w = rng.random((n, k)).astype(np.float32)
    xt = bf16_tensor_from_np(x)
    it = torch.from_numpy(ids if ids64 else ids.astype(np.int32)).cuda()
    wt = torch.from_numpy(w).cuda()
    seq, layer = 1, 37
    d.dispatch(seq, layer, xt, it, wt, epochs=[3] * F, ids64=ids64)
    torch.cuda.synchronize()
    assert int(d.status.item()) == 0
    row_of, count, pad = moe.f_rank_tables(ids, bounds)
    tables = d.ws[512: 512 + 8 * F * g.n_max].view(torch.int32).view(2, F, g.n_max).cpu().numpy()
    np.testing.assert_array_equal(tables[0][:, :n], row_of)
    for f in range(F):  # each F rank's row -> token list: the inverse of its row_of
        if not pad[f]:
            np.testing.assert_array_equal(tables[1][f, : count[f]], np.nonzero(row_of[f] >= 0)[0])
    for f in range(F):
        reg = d.region(f).cpu().numpy()
        c = int(count[f])
        if not pad[f]:
            sel = row_of[f] >= 0
            xs = reg[: c * H * 2].view(np.uint16).reshape(c, H)
            np.testing.assert_array_equal(xs, mx.bf16_bits(x[sel]))
            np.testing.assert_array_equal(reg[g.ids_off: g.ids_off + 4 * c * k].view(np.int32).reshape(c, k),
                                          ids[sel].astype(np.int32))
            np.testing.assert_array_equal(reg[g.w_off: g.w_off + 4 * c * k].view(np.float32).reshape(c, k), w[sel])
        else:
            assert c == 1
            np.testing.assert_array_equal(reg[g.ids_off: g.ids_off + 4 * k].view(np.int32), [-1] * k)
        word = int(d.bells[f][g.bell_off(0, 0) // 8].item()) & 0xFFFFFFFFFFFFFFFF
        assert word == pack_doorbell(seq, c, layer, 3)
    # F replies: row j of F rank f's segment answers its region row j
    parts = []
    for f in range(F):
        part = mx.bf16_round(rng.standard_normal((int(count[f]), H)).astype(np.float32))
        d.seg(f)[: len(part)] = bf16_tensor_from_np(part)
        d.set_done(f, 0, seq)
        parts.append(part)
    shared = mx.bf16_round(rng.standard_normal((n, H)).astype(np.float32))
    out = d.combine(seq, n, shared=bf16_tensor_from_np(shared))
    torch.cuda.synchronize()
    assert int(d.status.item()) == 0
    np.testing.assert_array_equal(np_from_bf16(out), moe.combine(parts, row_of, n, shared))
    out2 = d.combine(seq, n)
    np.testing.assert_array_equal(np_from_bf16(out2), moe.combine(parts, row_of, n))


def test_dispatch_bf16_weights(cuda_ok):
    rng = np.random.default_rng(3)
    n, H, k = 64, 256, 2
    g = Geometry(1, 1, 1, n, H, k, 1)
    d = FakeDeployment(g, [0, 8])
    x = bf16_tensor_from_np(rng.standard_normal((n, H)).astype(np.float32))
    ids = torch.randint(0, 8, (n, k), dtype=torch.int32, device="cuda")
    w = torch.rand(n, k, device="cuda").to(torch.bfloat16)
    d.dispatch(1, 0, x, ids, w, wbf16=True)
    torch.cuda.synchronize()
    reg = d.region(0)
    got = reg[g.w_off: g.w_off + 4 * n * k].view(torch.float32).view(n, k)
    assert torch.equal(got, w.float())


def test_backpressure_wait_runs_out(cuda_ok):
    """done[f][slot] is never advanced to seq-1: the dispatch gives up, reports, and sends nothing."""
    g = Geometry(1, 1, 2, 16, 256, 2, 2)
    d = FakeDeployment(g, [0, 4, 8])
    x = torch.zeros(4, 256, dtype=torch.bfloat16, device="cuda")
    ids = torch.zeros(4, 2, dtype=torch.int32, device="cuda")
    w = torch.zeros(4, 2, device="cuda")
    d.dispatch(5, 0, x, ids, w, timeout_s=0.02)  # expects done >= 4; flags are 0
    torch.cuda.synchronize()
    st = N.decode_status(int(d.status.item()))
    assert st["what"] == "backpressure timeout" and st["seq"] == 5
    assert all(int(b[0].item()) == 0 for b in d.bells)  # no doorbell


def test_reply_wait_runs_out(cuda_ok):
    g = Geometry(1, 1, 2, 16, 256, 2, 2)
    d = FakeDeployment(g, [0, 4, 8])
    x = torch.zeros(4, 256, dtype=torch.bfloat16, device="cuda")
    ids = torch.zeros(4, 2, dtype=torch.int32, device="cuda")
    w = torch.zeros(4, 2, device="cuda")
    d.dispatch(1, 0, x, ids, w)
    d.set_done(0, 0, 1)  # F rank 1 never answers
    d.combine(1, 4, timeout_s=0.02)
    torch.cuda.synchronize()
    st = N.decode_status(int(d.status.item()))
    assert st["what"] == "reply timeout" and st["f"] == 1 and st["seq"] == 1
    # the separate wait entry point reports the same way
    d.status.zero_()
    N.call("asap_wait_replies", ctypes.byref(d.gs), 0, 1, d.result.data_ptr(), d.status.data_ptr(), int(0.02e9),
           ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert N.decode_status(int(d.status.item()))["what"] == "reply timeout"


def test_seq_wraps(cuda_ok):
    """seq is compared as a cyclic int32 difference: 0 follows 0xFFFFFFFF (layout.py:51-52)."""
    g = Geometry(1, 1, 1, 8, 256, 2, 1)
    d = FakeDeployment(g, [0, 4])
    x = torch.zeros(2, 256, dtype=torch.bfloat16, device="cuda")
    ids = torch.zeros(2, 2, dtype=torch.int32, device="cuda")
    w = torch.zeros(2, 2, device="cuda")
    d.set_done(0, 0, 0xFFFFFFFF - 2**32)  # previous message 0xFFFFFFFF answered (stored as int32 -1)
    d.dispatch(0, 0, x, ids, w, timeout_s=0.5)  # seq 0 after the wrap
    torch.cuda.synchronize()
    assert int(d.status.item()) == 0
    word = int(d.bells[0][0].item()) & 0xFFFFFFFFFFFFFFFF
    assert word == pack_doorbell(0, 2, 0, 1)


def test_doorbell_wait_runs_out_and_rejects_stale_epoch(cuda_ok):
    from asap_b200.experts import Mxfp4Experts
    from gpu_util import FfnHarness

    e = Mxfp4Experts.random(4, 256, 128, seed=1)
    h = FfnHarness(e, n_max=8, topk=2)
    bell = torch.zeros(8, dtype=torch.int64, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    N.call("asap_ffn_wait", h.handle, bell.data_ptr(), 0, 1, 8, h.status.data_ptr(), int(0.02e9), stream)
    torch.cuda.synchronize()
    assert N.decode_status(int(h.status.item()))["what"] == "doorbell timeout"
    # a doorbell of another epoch is rejected and the job does nothing (no reply, no done flag)
    h.status.zero_()
    bell[0] = pack_doorbell(1, 4, 2, 7)
    N.call("asap_ffn_wait", h.handle, bell.data_ptr(), 0, 1, 8, h.status.data_ptr(), int(1e9), stream)
    x = torch.ones(8, 256, dtype=torch.bfloat16, device="cuda")
    ids = torch.zeros(8, 2, dtype=torch.int32, device="cuda")
    w = torch.ones(8, 2, device="cuda")
    N.call("asap_ffn_job", e.handle, h.handle, x.data_ptr(), ids.data_ptr(), w.data_ptr(), h.reply.data_ptr(),
           h.done.data_ptr(), ctypes.c_float(0), h.status.data_ptr(), int(1e9), stream)
    torch.cuda.synchronize()
    st = N.decode_status(int(h.status.item()))
    assert st["what"] == "bad doorbell" and st["seq"] == 1
    assert int(h.done[0].item()) == 0
    # the right epoch: a valid job
    h.status.zero_()
    bell[0] = pack_doorbell(2, 4, 2, 1)
    N.call("asap_ffn_wait", h.handle, bell.data_ptr(), 1, 1, 8, h.status.data_ptr(), int(1e9), stream)
    N.call("asap_ffn_job", e.handle, h.handle, x.data_ptr(), ids.data_ptr(), w.data_ptr(), h.reply.data_ptr(),
           h.done.data_ptr(), ctypes.c_float(0), h.status.data_ptr(), int(1e9), stream)
    torch.cuda.synchronize()
    assert int(h.status.item()) == 0 and int(h.done[0].item()) == 2
    h.release()
    e.release()


@pytest.mark.parametrize("a,num_a", [(0, 2), (1, 2), (2, 3)])
def test_dispatch_rotation_same_bytes(cuda_ok, a, num_a):
    """A ranks fill the F ranks in turn from a*num_f/num_a (each doorbell rung when its own rows are stored): the
    routing table, arena bytes and doorbell words are the same whichever F rank comes first, including an F rank
    that gets only the padding row."""
    rng = np.random.default_rng(21)
    n, H, k, bounds = 300, 512, 4, [0, 10, 10, 24]
    x = bf16_tensor_from_np(mx.bf16_round(rng.standard_normal((n, H)).astype(np.float32)))
    ids = torch.from_numpy(np.stack([rng.permutation(26)[:k] - 1 for _ in range(n)]).astype(np.int32)).cuda()
    w = torch.from_numpy(rng.random((n, k)).astype(np.float32)).cuda()
    ref = FakeDeployment(Geometry(1, 1, 2, n, H, k, 3), bounds, a=0)
    rot = FakeDeployment(Geometry(num_a, 1, 2, n, H, k, 3), bounds, a=a)
    ref.dispatch(1, 9, x, ids, w, epochs=[2, 2, 2])  # seq 1: backpressure needs done >= 0, already true
    rot.dispatch(1, 9, x, ids, w, epochs=[2, 2, 2])
    torch.cuda.synchronize()
    assert int(ref.status.item()) == 0 and int(rot.status.item()) == 0
    assert torch.equal(ref.ws[:320], rot.ws[:320]) and torch.equal(ref.ws[512:], rot.ws[512:])
    for f in range(3):
        assert torch.equal(ref.region(f), rot.region(f)), f
        word_ref = int(ref.bells[f][ref.g.bell_off(0, 0) // 8].item())
        word_rot = int(rot.bells[f][rot.g.bell_off(a, 0) // 8].item())
        assert word_ref == word_rot, f


def test_dispatch_sixteen_f_ranks(cuda_ok):
    """The largest F count (ASAP_MAX_F = 16), uneven and empty ranges: routing table, arena bytes and doorbells."""
    rng = np.random.default_rng(41)
    n, H, k = 200, 256, 8
    bounds = [0, 3, 3, 9, 12, 20, 21, 30, 31, 40, 41, 48, 49, 50, 60, 63, 64]
    F = len(bounds) - 1
    g = Geometry(1, 1, 1, n, H, k, F)
    d = FakeDeployment(g, bounds)
    x = mx.bf16_round(rng.standard_normal((n, H)).astype(np.float32))
    ids = np.stack([rng.permutation(64)[:k] for _ in range(n)]).astype(np.int32)
    w = rng.random((n, k)).astype(np.float32)
    d.dispatch(1, 2, bf16_tensor_from_np(x), torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda())
    torch.cuda.synchronize()
    assert int(d.status.item()) == 0
    row_of, count, pad = moe.f_rank_tables(ids, bounds)
    tables = d.ws[512: 512 + 8 * F * g.n_max].view(torch.int32).view(2, F, g.n_max).cpu().numpy()
    np.testing.assert_array_equal(tables[0][:, :n], row_of)
    for f in range(F):  # each F rank's row -> token list: the inverse of its row_of
        if not pad[f]:
            np.testing.assert_array_equal(tables[1][f, : count[f]], np.nonzero(row_of[f] >= 0)[0])
    for f in range(F):
        c = int(count[f])
        reg = d.region(f).cpu().numpy()
        if not pad[f]:
            sel = row_of[f] >= 0
            np.testing.assert_array_equal(reg[: c * H * 2].view(np.uint16).reshape(c, H), mx.bf16_bits(x[sel]))
        word = int(d.bells[f][g.bell_off(0, 0) // 8].item()) & 0xFFFFFFFFFFFFFFFF
        assert word == pack_doorbell(1, c, 2, 1)


def test_host_pages_and_release(cuda_ok, tmp_path):
    """asap_host_page_create / _open / asap_release: a page written on the device is seen by the host and by a
    second mapping of the same file; release unmaps both and removes the file; arenas and IPC-free pointers go
    through asap_release too, and a second release is refused."""
    import os
    import tempfile

    lib = N.lib()
    d = tempfile.mkdtemp(dir="/dev/shm" if os.access("/dev/shm", os.W_OK) else None)
    path = os.path.join(d, "bells").encode()
    host, dev = ctypes.c_uint64(), ctypes.c_uint64()
    N.call("asap_host_page_create", path, 4096, ctypes.byref(host), ctypes.byref(dev))
    host2, dev2 = ctypes.c_uint64(), ctypes.c_uint64()
    N.call("asap_host_page_open", path, 4096, ctypes.byref(host2), ctypes.byref(dev2))
    assert host2.value != host.value
    N.call("asap_write32", dev.value + 64, 0xC0FFEE, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert ctypes.c_uint32.from_address(host.value + 64).value == 0xC0FFEE
    assert ctypes.c_uint32.from_address(host2.value + 64).value == 0xC0FFEE
    N.call("asap_release", host2.value)
    assert os.path.exists(path)       # the opener does not remove the owner's file
    N.call("asap_release", host.value)
    assert not os.path.exists(path)   # the creator does
    assert lib.asap_release(host.value) == N.ASAP_EINVAL
    arena = ctypes.c_uint64()
    N.call("asap_arena_alloc", 1 << 20, ctypes.byref(arena), None)
    N.call("asap_release", arena.value)
    assert lib.asap_release(arena.value) == N.ASAP_EINVAL
    os.rmdir(d)


def test_channel_fault_hooks_stale_epoch_and_lost_messages(cuda_ok):
    """The reference's test hooks AttnChannel(_epoch_override=, _backpressure=False) (channel.py:198-203) provoke
    the protocol violations the F poll counts (server.py:278-280, 303-305): a doorbell with another epoch is
    dropped as stale; with backpressure off, a second message on a slot the F rank has not answered overwrites
    the first, which the F rank counts as lost and serves the newer one."""
    import os
    import shutil
    import tempfile

    from asap_b200.transport.channel import AttnChannel
    from asap_b200.transport.server import FfnServer

    g = Geometry(1, 1, 2, 64, 256, 2, 1)
    run_dir = tempfile.mkdtemp(dir="/dev/shm" if os.access("/dev/shm", os.W_OK) else None)
    x = torch.zeros(8, 256, dtype=torch.bfloat16, device="cuda")
    ids = torch.tensor([[0, 1]] * 8, dtype=torch.int32, device="cuda")
    w = torch.full((8, 2), 0.5, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream

    def deployment(**hooks):
        srv = FfnServer(0, g, device=0, run_dir=run_dir, listen=False).start()
        ch = AttnChannel(0, g, [("in-process", 0)], device=0, expert_bounds=[0, 8], timeout_s=2.0,
                         _connector=lambda f, hello: srv.handshake(hello), **hooks).connect()
        return srv, ch

    srv, ch = deployment(_epoch_override=9)
    ch.send(3, 0, x.data_ptr(), ids.data_ptr(), w.data_ptr(), 8, stream)
    torch.cuda.synchronize()
    assert srv.poll() == [] and srv.stats["stale_epoch"] == 1
    ch.check()
    ch.close()
    srv.close()

    srv, ch = deployment(_backpressure=False)
    ch.send(3, 0, x.data_ptr(), ids.data_ptr(), w.data_ptr(), 8, stream)
    ch.send(4, 0, x.data_ptr(), ids.data_ptr(), w.data_ptr(), 5, stream)  # slot 0 again, nothing answered
    torch.cuda.synchronize()
    jobs = srv.poll()
    assert [(j.slot, j.layer_id, j.rows[0].seq, j.rows[0].n_tokens) for j in jobs] == [(0, 4, 2, 5)]
    assert srv.stats["lost_messages"] == 1
    ch.check()
    ch.close()
    srv.close()
    shutil.rmtree(run_dir, ignore_errors=True)
