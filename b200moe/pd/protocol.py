"""Framed JSON control protocol of the PD roles: frame = [u32 little-endian
length][UTF-8 JSON].  The frame format is the reference's
(nanovllm/pd/protocol.py:11-64) so clients of either framework interoperate.
"""
from __future__ import annotations

import json
import socket
import struct
import time

HDR = struct.Struct("<I")


def send_json(sock: socket.socket, obj) -> None:
    data = json.dumps(obj).encode()
    blocking = sock.getblocking()
    sock.setblocking(True)
    try:
        sock.sendall(HDR.pack(len(data)) + data)
    finally:
        sock.setblocking(blocking)


class JsonStream:
    """Incremental parser: ``feed(bytes)`` returns the completed messages."""

    def __init__(self):
        self._buf = bytearray()

    def feed(self, chunk: bytes) -> list:
        self._buf += chunk
        out = []
        while len(self._buf) >= HDR.size:
            (n,) = HDR.unpack_from(self._buf)
            if len(self._buf) < HDR.size + n:
                break
            out.append(json.loads(bytes(self._buf[HDR.size:HDR.size + n])))
            del self._buf[:HDR.size + n]
        return out


def connect_retry(host: str, port: int, tries: int = 120, blocking: bool = False) -> socket.socket:
    for i in range(tries):
        try:
            sock = socket.create_connection((host, port), timeout=5)
            sock.setblocking(blocking)
            return sock
        except OSError:
            time.sleep(0.5 if i < 20 else 2.0)
    raise ConnectionError(f"cannot connect to {host}:{port}")


def recv_exact(sock: socket.socket, n: int) -> bytes:
    chunks = []
    while n > 0:
        chunk = sock.recv(min(n, 1 << 22))
        if not chunk:
            raise ConnectionError("peer closed")
        chunks.append(chunk)
        n -= len(chunk)
    return b"".join(chunks)


def listen(port: int, host: str = "127.0.0.1") -> socket.socket:
    srv = socket.socket(socket.AF_INET, socket.SOCK_STREAM)
    srv.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
    srv.bind((host, port))
    srv.listen(4)
    return srv
