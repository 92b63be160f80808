"""asap_dispatch_noalloc, the allocation-free dispatch, against asap_dispatch through the C ABI.

Callers that cannot allocate device memory (an attention rank whose free memory already went to the KV-cache
pool, or a foreign-language host that only holds the transport's mapped arenas) use asap_dispatch_noalloc: its
routing table lives in a static device array inside the library.  This test sends the same two messages in a row
through both entry points into two separate sets of arenas and checks that everything they produce is identical:
every F rank's region bytes, the doorbell words, the routing table, and the combined output computed from it.
The comparison is exact (integer and byte data, and the combine of identical inputs).
Collected last on purpose (tests/test_zz_*), so a run that stops at the first failure has run everything else."""

import ctypes

import numpy as np
import pytest
import torch

from asap_b200 import _native as N
from asap_b200.transport.layout import Geometry

pytestmark = pytest.mark.gpu


class Arenas:
    """One A rank's ResultArena and num_f F ranks' RecvArenas and doorbell pages, as plain device buffers."""

    def __init__(self, g: Geometry):
        self.g = g
        self.recv = [torch.zeros(g.recv_bytes, dtype=torch.uint8, device="cuda") for _ in range(g.num_f)]
        self.bells = [torch.zeros(g.host_bytes // 8, dtype=torch.int64, device="cuda") for _ in range(g.num_f)]
        self.result = torch.zeros(g.result_bytes, dtype=torch.uint8, device="cuda")
        self.status = torch.zeros(1, dtype=torch.int64, device="cuda")

    def seg(self, f, slot):
        off = self.g.seg_off(f, slot)
        return self.result[off: off + self.g.n_max * self.g.hidden * 2].view(torch.bfloat16).view(
            self.g.n_max, self.g.hidden)

    def set_done(self, f, slot, seq):
        self.result[: self.g.flags_bytes].view(torch.int32)[self.g.done_off(f, slot) // 4] = seq


def _args(g, ar, slot, seq, x, ids, w, bounds, epochs):
    F = g.num_f
    return (ctypes.byref(N.geometry_struct(g)), 0, slot, seq, 9, (ctypes.c_int32 * F)(*epochs), x.data_ptr(),
            ids.data_ptr(), 0, w.data_ptr(), 0, x.shape[0], (ctypes.c_int32 * (F + 1))(*bounds),
            (ctypes.c_uint64 * F)(*[r.data_ptr() for r in ar.recv]),
            (ctypes.c_uint64 * F)(*[b.data_ptr() for b in ar.bells]), ar.result.data_ptr())


def _combine(g, ar, slot, seq, n, route_ws):
    out = torch.empty(n, g.hidden, dtype=torch.bfloat16, device="cuda")
    N.call("asap_combine", ctypes.byref(N.geometry_struct(g)), slot, seq, n, ar.result.data_ptr(), route_ws, 0,
           out.data_ptr(), ar.status.data_ptr(), int(2e9), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    return out


def test_noalloc_dispatch_matches_dispatch(cuda_ok):
    g = Geometry(1, 1, 2, 256, 512, 4, 3)
    bounds, epochs = [0, 8, 8, 20], [2, 2, 2]  # F rank 1 owns no expert: its padding row path is covered too
    ref, noa = Arenas(g), Arenas(g)
    route_ws = torch.zeros(N.lib().asap_route_ws_bytes(ctypes.byref(N.geometry_struct(g))), dtype=torch.uint8,
                           device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rng = np.random.default_rng(0)
    for call, (slot, n) in enumerate([(0, 200), (0, 77)]):  # two calls in a row, same slot
        seq = call + 1
        x = torch.from_numpy(rng.standard_normal((n, 512)).astype(np.float32)).cuda().to(torch.bfloat16)
        ids = torch.from_numpy(np.stack([rng.permutation(22)[:4] - 1 for _ in range(n)]).astype(np.int32)).cuda()
        w = torch.from_numpy(rng.random((n, 4)).astype(np.float32)).cuda()
        N.call("asap_dispatch", *_args(g, ref, slot, seq, x, ids, w, bounds, epochs), route_ws.data_ptr(), 1,
               ref.status.data_ptr(), int(2e9), stream)
        got_ws = ctypes.c_uint64()
        N.call("asap_dispatch_noalloc", *_args(g, noa, slot, seq, x, ids, w, bounds, epochs), 1,
               noa.status.data_ptr(), int(2e9), stream, ctypes.byref(got_ws))
        torch.cuda.synchronize()
        assert int(ref.status.item()) == 0 and int(noa.status.item()) == 0
        assert got_ws.value != 0 and got_ws.value % 256 == 0
        for f in range(g.num_f):
            assert torch.equal(ref.recv[f], noa.recv[f]), f"region bytes of F rank {f}, call {call}"
            assert torch.equal(ref.bells[f], noa.bells[f]), f"doorbells of F rank {f}, call {call}"
        nbytes = 512 + 4 * g.num_f * g.n_max
        table = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
        src = torch.as_tensor(_DevBytes(got_ws.value, nbytes), device="cuda")
        table.copy_(src)
        rows = slice(512, 512 + 4 * g.num_f * g.n_max)
        ref_rows = route_ws[rows].view(torch.int32).view(g.num_f, g.n_max)[:, :n]
        noa_rows = table[rows].view(torch.int32).view(g.num_f, g.n_max)[:, :n]
        assert torch.equal(ref_rows, noa_rows)
        assert torch.equal(route_ws[:256].view(torch.int32)[: g.num_f], table[:256].view(torch.int32)[: g.num_f])
        # identical replies in both ResultArenas; the combine reads each entry point's routing table
        for f in range(g.num_f):
            part = torch.randn(n, 512, device="cuda").to(torch.bfloat16)
            ref.seg(f, slot)[:n] = part
            noa.seg(f, slot)[:n] = part
            ref.set_done(f, slot, seq)
            noa.set_done(f, slot, seq)
        out_ref = _combine(g, ref, slot, seq, n, route_ws.data_ptr())
        out_noa = _combine(g, noa, slot, seq, n, got_ws.value)
        torch.cuda.synchronize()
        assert int(ref.status.item()) == 0 and int(noa.status.item()) == 0
        assert torch.equal(out_ref, out_noa)


def test_noalloc_dispatch_last_slot_at_the_maximum(cuda_ok):
    """Slot 7 (the last static table) with num_f * n_max = 131072 (the maximum): the full table equals
    asap_dispatch's, its address is the 8th slot's, and the neighbouring slot 6 is left untouched."""
    g = Geometry(1, 1, 8, 32768, 512, 4, 4)
    assert g.num_f * g.n_max == 1 << 17
    bounds, epochs, slot, n = [0, 6, 12, 18, 24], [1, 1, 1, 1], 7, 32768
    ref, noa = Arenas(g), Arenas(g)
    ws_bytes = N.lib().asap_route_ws_bytes(ctypes.byref(N.geometry_struct(g)))
    route_ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rng = np.random.default_rng(7)
    x = torch.from_numpy(rng.standard_normal((n, 512)).astype(np.float32)).cuda().to(torch.bfloat16)
    ids = torch.from_numpy(np.stack([rng.permutation(24)[:4] for _ in range(n)]).astype(np.int32)).cuda()
    w = torch.from_numpy(rng.random((n, 4)).astype(np.float32)).cuda()
    # one small call on slot 6 gives its table's address; snapshot that table
    small = Geometry(1, 1, 8, 8, 512, 4, 4)
    ar0 = Arenas(small)
    slot6_addr = ctypes.c_uint64()
    N.call("asap_dispatch_noalloc", *_args(small, ar0, 6, 1, x[:8], ids[:8], w[:8], bounds, epochs), 1,
           ar0.status.data_ptr(), int(2e9), stream, ctypes.byref(slot6_addr))
    torch.cuda.synchronize()
    slot_bytes = N.lib().asap_route_ws_bytes(ctypes.byref(N.geometry_struct(g)))  # 512 + 4 * 131072
    slot6 = torch.as_tensor(_DevBytes(slot6_addr.value, slot_bytes), device="cuda").clone()
    N.call("asap_dispatch", *_args(g, ref, slot, 1, x, ids, w, bounds, epochs), route_ws.data_ptr(), 1,
           ref.status.data_ptr(), int(2e9), stream)
    got = ctypes.c_uint64()
    N.call("asap_dispatch_noalloc", *_args(g, noa, slot, 1, x, ids, w, bounds, epochs), 1, noa.status.data_ptr(),
           int(2e9), stream, ctypes.byref(got))
    torch.cuda.synchronize()
    assert int(ref.status.item()) == 0 and int(noa.status.item()) == 0
    assert got.value == slot6_addr.value + slot_bytes  # slot 7 follows slot 6
    table = torch.as_tensor(_DevBytes(got.value, slot_bytes), device="cuda").clone()
    rows = slice(512, slot_bytes)
    assert torch.equal(route_ws[rows], table[rows])  # every row of the table, the last F rank's included
    assert torch.equal(route_ws[:256].view(torch.int32)[: g.num_f], table[:256].view(torch.int32)[: g.num_f])
    assert torch.equal(torch.as_tensor(_DevBytes(slot6_addr.value, slot_bytes), device="cuda"), slot6)
    for f in range(g.num_f):
        assert torch.equal(ref.recv[f], noa.recv[f]) and torch.equal(ref.bells[f], noa.bells[f])


def test_noalloc_dispatch_rejects_sizes_beyond_its_maximum(cuda_ok):
    out = ctypes.c_uint64()
    x = torch.zeros(4, 512, dtype=torch.bfloat16, device="cuda")
    ids = torch.zeros(4, 4, dtype=torch.int32, device="cuda")
    w = torch.zeros(4, 4, device="cuda")
    for g, slot in ((Geometry(1, 1, 2, 65536, 512, 4, 3), 0), (Geometry(1, 1, 9, 256, 512, 4, 3), 8)):
        ar = Arenas(Geometry(1, 1, 1, 8, 512, 4, 3))
        rc = N.lib().asap_dispatch_noalloc(*_args(g, ar, slot, 1, x, ids, w, [0, 8, 8, 20], [1, 1, 1]), 0,
                                           ar.status.data_ptr(), int(1e9), None, ctypes.byref(out))
        assert rc == N.ASAP_EINVAL
        msg = N.lib().asap_last_error_string().decode()
        assert "static maximum" in msg or "static routing tables" in msg


class _DevBytes:
    def __init__(self, ptr, nbytes):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 2}
