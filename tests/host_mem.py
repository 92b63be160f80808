"""A host-memory stand-in for the transport's shared memory (CPU tests of the multi-process host logic): /dev/shm
files in place of CUDA IPC arenas, so "device" pointers are host addresses both processes map."""

import ctypes
import mmap
import os
import socket

import numpy as np

from asap_b200.transport.layout import HandshakeError
from asap_b200.transport.memory import Shared


class HostMem:
    """Shared host memory (/dev/shm files) in place of CUDA IPC arenas; 'device' pointers are host addresses."""

    kind = "ipc"
    reason = "host test stand-in"

    def __init__(self, run_dir):
        self.ordinal, self.run_dir, self._n = 0, run_dir, 0

    def activate(self):
        pass

    def fill32(self, ptr, value, count):
        np.ctypeslib.as_array((ctypes.c_uint32 * count).from_address(ptr))[:] = value & 0xFFFFFFFF

    def identity(self):
        return {"host": socket.gethostname()}

    def check_peer(self, peer):
        if peer.get("host") not in (None, socket.gethostname()):
            raise HandshakeError(f"the ipc transport needs one host, peer on {peer['host']}")

    def _map(self, path, nbytes, create):
        fd = os.open(path, os.O_RDWR | (os.O_CREAT | os.O_TRUNC if create else 0), 0o600)
        try:
            if create:
                os.ftruncate(fd, nbytes)
            mm = mmap.mmap(fd, nbytes)
        finally:
            os.close(fd)
        buf = ctypes.c_char.from_buffer(mm)
        addr = ctypes.addressof(buf)
        del buf
        return mm, addr

    def device(self, nbytes):
        self._n += 1
        path = os.path.join(self.run_dir, f"arena_{os.getpid()}_{self._n}")
        mm, addr = self._map(path, nbytes, True)
        return Shared(addr, mm.close, {"shm": path, "bytes": nbytes})

    def doorbells(self, nbytes, path, device_access=True):
        mm, addr = self._map(path, nbytes, True)
        s = Shared(addr, mm.close, {"path": path}, dev=addr)
        s.mmap = mm
        return s

    def open(self, desc):
        mm, addr = self._map(desc["shm"], desc["bytes"], False)
        return Shared(addr, mm.close)

    def open_doorbells(self, desc, nbytes):
        mm, addr = self._map(desc["path"], nbytes, False)
        return Shared(addr, mm.close)

    def status_words(self, count):
        class Words:
            def __init__(self):
                self.buf = (ctypes.c_uint64 * count)()
                self.ptr = ctypes.addressof(self.buf)

            def read(self, i=0):
                return self.buf[i]

            def close(self):
                pass

        return Words()

    def workspace(self, nbytes):
        class Ws:
            def __init__(self):
                self.buf = (ctypes.c_uint8 * nbytes)()

            def data_ptr(self):
                return ctypes.addressof(self.buf)

        return Ws()
