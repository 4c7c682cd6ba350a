"""Hop frames over TCP: the cross-host stand-in for the reference's WebRTC data
channel (rtc.js:7-22 frames, pipeline.js:226-253 hop, script.js:163-172 stage
side). A stage host serves HIDDEN_REQ / FINAL_REQ frames with a handler (usually
`pipeline.handle_stage_frame` bound to its Stage); the leader's `TcpTransport`
is the `transport` callable of LeaderPipeline.

On the wire each frame (the rtc.js layout: 4 x int32 header + fp32 payload)
is preceded by its byte length as a little-endian uint64. A request gets one
reply on the same connection. A handler that fails closes the connection, so
the leader's hop raises instead of waiting; reads time out after `timeout`
seconds (15 s, the readF32 limit of kernels.js:201-207).
"""
from __future__ import annotations

import socket
import struct
import threading

MAX_FRAME_BYTES = 1 << 31  # 2 GiB: far above n x D x 4 for any prefill chunk


def _recv_exact(sock: socket.socket, n: int) -> bytes:
    buf = bytearray()
    while len(buf) < n:
        chunk = sock.recv(min(n - len(buf), 1 << 20))
        if not chunk:
            raise ConnectionError("peer closed the connection")
        buf += chunk
    return bytes(buf)


def send_frame(sock: socket.socket, data: bytes):
    sock.sendall(struct.pack("<Q", len(data)) + data)


def recv_frame(sock: socket.socket) -> bytes:
    n = struct.unpack("<Q", _recv_exact(sock, 8))[0]
    if n > MAX_FRAME_BYTES:
        raise ValueError(f"frame of {n} bytes exceeds {MAX_FRAME_BYTES}")
    return _recv_exact(sock, n)


class FrameServer:
    """Serves frames on host:port with `handler(bytes) -> bytes`, one request at a
    time (a Stage is not reentrant). `port=0` picks a free port (see `.port`)."""

    def __init__(self, handler, host: str = "127.0.0.1", port: int = 0):
        self.handler = handler
        self.sock = socket.create_server((host, port))
        self.host, self.port = self.sock.getsockname()[:2]
        self._lock = threading.Lock()
        self._thread = None
        self._stop = threading.Event()

    def _serve_conn(self, conn: socket.socket):
        with conn:
            while not self._stop.is_set():
                try:
                    data = recv_frame(conn)
                except (ConnectionError, OSError, ValueError):
                    return  # closed, or an oversized / malformed frame: drop the connection
                try:
                    with self._lock:
                        reply = self.handler(data)
                except Exception:
                    return  # close: the leader's hop raises rather than waits
                send_frame(conn, reply)

    def serve_forever(self):
        self.sock.settimeout(0.2)
        while not self._stop.is_set():
            try:
                conn, _ = self.sock.accept()
            except socket.timeout:
                continue
            except OSError:
                return
            conn.settimeout(None)
            threading.Thread(target=self._serve_conn, args=(conn,), daemon=True).start()

    def start(self) -> "FrameServer":
        self._thread = threading.Thread(target=self.serve_forever, daemon=True)
        self._thread.start()
        return self

    def stop(self):
        self._stop.set()
        try:
            self.sock.close()
        finally:
            if self._thread is not None:
                self._thread.join(timeout=5)


def serve_stage(stage, host: str = "127.0.0.1", port: int = 0) -> FrameServer:
    """A started FrameServer answering hops for `stage` (script.js:163-172)."""
    from .pipeline import handle_stage_frame
    return FrameServer(lambda data: handle_stage_frame(stage, data), host, port).start()


class TcpTransport:
    """LeaderPipeline transport: `transport(peer_id, frame) -> reply frame` over a
    persistent connection per peer. peers: {peer_id: (host, port)}."""

    def __init__(self, peers: dict, timeout: float = 15.0):
        self.peers = dict(peers)
        self.timeout = timeout
        self._socks: dict = {}

    def _sock(self, peer_id) -> socket.socket:
        s = self._socks.get(peer_id)
        if s is None:
            host, port = self.peers[peer_id]
            s = socket.create_connection((host, port), timeout=self.timeout)
            s.settimeout(self.timeout)
            self._socks[peer_id] = s
        return s

    def __call__(self, peer_id, data: bytes) -> bytes:
        s = self._sock(peer_id)
        try:
            send_frame(s, data)
            return recv_frame(s)
        except (OSError, ConnectionError, ValueError):
            self._socks.pop(peer_id, None)
            s.close()
            raise

    def close(self):
        for s in self._socks.values():
            s.close()
        self._socks.clear()
