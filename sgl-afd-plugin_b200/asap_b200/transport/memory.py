"""Where the transport's shared memory lives and how a peer maps it (replaces python/sgl_asap_plugin/transport/
memory.py for a single B200 node).

Every message goes into memory owned by its receiver: F rank f owns its RecvArena (device) and its doorbell
page (host memory its CPU polls and, in device-wait mode, its GPU polls); A rank a owns its ResultArena. The
owner allocates it and sends a descriptor in the handshake; the peer opens the descriptor and gets an address
its GPU stores to over NVLink (P2P stores from the dispatch / reply kernels, not copy engines).

* ``ipc``: cudaMalloc + cudaIpcGetMemHandle for device memory (memory.py:48-116); the doorbell page is a /dev/shm
  file the peer maps and registers (cudaHostRegister, mapped).  Within one process (the 1-GPU loopback
  deployment) a descriptor of the own process is opened as the plain pointer, because CUDA IPC cannot open a
  handle in the process that exported it.
* ``fabric`` (GB200 multi-node NVLink, IMEX) is not part of this B200 build: selecting it raises.
"""

from __future__ import annotations

import ctypes
import mmap
import os
import socket
from typing import Callable, Optional

from .. import _native as N
from .layout import HandshakeError, TransportError

KINDS = ("auto", "ipc", "fabric")


class Shared:
    """Shared memory as this process sees it. ``ptr``: the device address, except for an own doorbell page, where
    it is the CPU address. ``dev``: the device address of an own doorbell page (registered here), else ptr."""

    def __init__(self, ptr: int, release: Callable[[], None], desc: Optional[dict] = None, dev: Optional[int] = None):
        self.ptr, self.desc, self._release = ptr, desc, release
        self.dev = ptr if dev is None else dev

    def release(self) -> None:
        release, self._release = self._release, None
        if release is not None:
            release()


def _mmap_address(mm: mmap.mmap) -> int:
    buf = ctypes.c_char.from_buffer(mm)
    addr = ctypes.addressof(buf)
    del buf
    return addr


class IpcMemory:
    kind = "ipc"

    def __init__(self, ordinal: int, reason: str = "requested"):
        self.ordinal, self.reason = ordinal, reason

    def activate(self) -> None:
        """Make this backend's device current for the calling thread."""
        N.call("asap_init", self.ordinal)

    def fill32(self, ptr: int, value: int, count: int) -> None:
        """Set ``count`` 32-bit words of device memory at ``ptr`` to ``value`` and wait for it."""
        import torch

        stream = torch.cuda.current_stream(self.ordinal)
        N.call("asap_memset32", ptr, value & 0xFFFFFFFF, count, ctypes.c_void_p(stream.cuda_stream))
        stream.synchronize()

    def identity(self) -> dict:
        return {"host": socket.gethostname()}

    def status_words(self, count: int) -> "HostWords":
        """Registered host words the device writes status into."""
        return HostWords(count)

    def workspace(self, nbytes: int):
        """Private device scratch of this rank (torch-allocated)."""
        import torch

        return torch.empty(nbytes, dtype=torch.uint8, device=f"cuda:{self.ordinal}")

    def check_peer(self, peer: dict) -> None:
        mine = socket.gethostname()
        if peer.get("host") not in (None, mine):
            raise HandshakeError(
                f"the ipc transport needs one host, but the peer runs on {peer['host']} and this rank on {mine}")

    def device(self, nbytes: int) -> Shared:
        ptr = ctypes.c_uint64()
        handle = (ctypes.c_uint8 * 64)()
        N.call("asap_arena_alloc", nbytes, ctypes.byref(ptr), handle)
        p = ptr.value
        desc = {"ipc": bytes(handle).hex(), "pid": os.getpid(), "ptr": p, "bytes": nbytes}
        return Shared(p, lambda: N.call("asap_arena_free", p), desc)

    def doorbells(self, nbytes: int, path: str, device_access: bool = True) -> Shared:
        """A zeroed file of nbytes at ``path`` (in /dev/shm), mapped here; with device_access also registered so
        that this GPU can poll it (device-wait mode).  release() unregisters, unmaps and removes it."""
        fd = os.open(path, os.O_RDWR | os.O_CREAT | os.O_TRUNC, 0o600)
        try:
            os.ftruncate(fd, nbytes)
            mm = mmap.mmap(fd, nbytes)
        finally:
            os.close(fd)
        addr = _mmap_address(mm)
        dev = None
        if device_access:
            d = ctypes.c_uint64()
            try:
                N.call("asap_host_register", addr, nbytes, ctypes.byref(d))
            except BaseException:
                mm.close()
                raise
            dev = d.value

        def release():
            if dev is not None:
                N.call("asap_host_unregister", addr)
            mm.close()
            try:
                os.unlink(path)
            except FileNotFoundError:
                pass

        desc = {"path": path, "pid": os.getpid(), "dev": dev}
        shared = Shared(addr, release, desc, dev=dev)
        shared.mmap = mm
        return shared

    def open(self, desc: dict) -> Shared:
        if desc.get("pid") == os.getpid():  # own allocation (loopback): IPC cannot reopen it here
            return Shared(int(desc["ptr"]), lambda: None)
        ptr = ctypes.c_uint64()
        raw = (ctypes.c_uint8 * 64).from_buffer_copy(bytes.fromhex(desc["ipc"]))
        N.call("asap_arena_open", raw, ctypes.byref(ptr))
        p = ptr.value
        return Shared(p, lambda: N.call("asap_arena_close", p))

    def open_doorbells(self, desc: dict, nbytes: int) -> Shared:
        """mmap the owner's /dev/shm file and register it, so that this GPU can write the doorbells."""
        if desc.get("pid") == os.getpid() and desc.get("dev"):  # own page (loopback): already registered
            return Shared(int(desc["dev"]), lambda: None)
        fd = os.open(desc["path"], os.O_RDWR)
        try:
            mm = mmap.mmap(fd, nbytes)
        finally:
            os.close(fd)
        addr = _mmap_address(mm)
        d = ctypes.c_uint64()
        try:
            N.call("asap_host_register", addr, nbytes, ctypes.byref(d))
        except BaseException:
            mm.close()
            raise

        def release():
            N.call("asap_host_unregister", addr)
            mm.close()

        return Shared(d.value, release)


class HostWords:
    """``count`` 64-bit words of page-aligned host memory registered for device access: kernels store status
    words there, the host reads them with plain loads and no synchronisation."""

    def __init__(self, count: int = 1):
        self.nbytes = max(4096, -(-count * 8 // 4096) * 4096)
        self._mm = mmap.mmap(-1, self.nbytes)
        self.host = _mmap_address(self._mm)
        d = ctypes.c_uint64()
        N.call("asap_host_register", self.host, self.nbytes, ctypes.byref(d))
        self.ptr = d.value  # device address
        self.count = count

    def read(self, i: int = 0) -> int:
        return ctypes.c_uint64.from_address(self.host + 8 * i).value

    def clear(self) -> None:
        ctypes.memset(self.host, 0, 8 * self.count)

    def close(self) -> None:
        if self._mm is not None:
            N.call("asap_host_unregister", self.host)
            self._mm.close()
            self._mm = None


def select(kind: str, ordinal: int) -> IpcMemory:
    """memory.py:249-261 for a single node: auto and ipc give IpcMemory; fabric (GB200 IMEX) raises."""
    if kind not in KINDS:
        raise ValueError(f"transport memory must be one of {KINDS}, got {kind!r}")
    if kind == "fabric":
        raise TransportError(f"the fabric transport is not usable on GPU {ordinal}: this build serves one B200 node "
                             "(CUDA IPC); fabric handles need a GB200 NVLink domain with IMEX")
    return IpcMemory(ordinal, reason="requested" if kind == "ipc" else "auto: single node")
