"""The handshake wire: one JSON object per line over TCP, one request and one answer per connection.

Both ends of the transport use this module: ``exchange`` is the A rank's client (it retries the connect until the F
rank listens -- an F rank loads tens of GB of experts before it does), ``HelloListener`` is the F rank's server,
a ``socketserver`` thread that answers every connection with whatever its handler returns (or a rejection carrying
the handler's exception).  What the objects mean is the contract of the reference's handshake
(python/sgl_asap_plugin/transport/channel.py:43-83 on A, transport/server.py:162-179 on F); the error texts a
caller sees are the reference's, so logs read the same with either implementation on either end.
"""

from __future__ import annotations

import json
import socket
import socketserver
import threading
import time
from typing import Callable, Optional

from .layout import HandshakeError

MAX_LINE = 1 << 20  # longest accepted line (a hello or an answer)


def _write_obj(stream, obj: dict) -> None:
    stream.write(json.dumps(obj).encode() + b"\n")
    stream.flush()


def _dial(host: str, port: int, deadline: float) -> socket.socket:
    """Connect, retrying every 0.2 s until ``deadline`` (monotonic seconds)."""
    last = None
    while time.monotonic() <= deadline:
        try:
            return socket.create_connection((host, port), timeout=2.0)
        except OSError as exc:
            last = exc
            time.sleep(0.2)
    raise HandshakeError(f"cannot reach F at {host}:{port}: {last}")


def exchange(host: str, port: int, msg: dict, *, connect_timeout: float = 60.0, io_timeout: float = 30.0) -> dict:
    """Send ``msg`` to the F rank at host:port and return its answer; HandshakeError when it cannot be reached,
    hangs up, or rejects the hello (with the F rank's reason)."""
    sock = _dial(host, port, time.monotonic() + connect_timeout)
    where = f"F at {host}:{port}"
    try:
        sock.settimeout(io_timeout)
        stream = sock.makefile("rwb")
        try:
            _write_obj(stream, msg)
            line = stream.readline(MAX_LINE)
        except OSError as exc:
            raise HandshakeError(f"handshake with {where} failed: {exc}") from exc
        finally:
            stream.close()
    finally:
        sock.close()
    if not line:
        raise HandshakeError(f"{where} closed the connection without answering")
    answer = json.loads(line)
    if not answer.get("ok"):
        raise HandshakeError(f"{where} rejected the connection: {answer.get('reason')}")
    return answer


class _OneLine(socketserver.StreamRequestHandler):
    timeout = 10.0  # per connection: a peer that never finishes its line is dropped

    def handle(self) -> None:
        try:
            answer = self.server.on_hello(json.loads(self.rfile.readline(MAX_LINE)))
        except Exception as exc:  # the reason goes back to A; the listener keeps serving
            answer = {"ok": False, "reason": f"{type(exc).__name__}: {exc}"}
        try:
            _write_obj(self.wfile, answer)
        except OSError:
            pass


class HelloListener(socketserver.ThreadingTCPServer):
    """F side: serve hellos on (host, port) from a daemon thread; ``port`` is the bound port (0 picks one)."""

    daemon_threads = True
    allow_reuse_address = True
    request_queue_size = 64

    def __init__(self, host: str, port: int, on_hello: Callable[[dict], dict], name: str):
        super().__init__((host, port), _OneLine)
        self.on_hello = on_hello
        self.port = self.server_address[1]
        self._thread: Optional[threading.Thread] = threading.Thread(
            target=self.serve_forever, kwargs={"poll_interval": 0.2}, name=name, daemon=True)
        self._thread.start()

    def stop(self) -> None:
        if self._thread is not None:
            self.shutdown()
            self._thread.join(timeout=2.0)
            self._thread = None
        self.server_close()
