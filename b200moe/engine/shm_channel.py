"""Shared-memory command channel between the driver and one worker rank.

The per-step messages (a step plan out, sampled ids back) travel through a
shared-memory segment with a sequence counter per direction; the receiver spins
on the counter for a bounded window (``B200MOE_SPIN_MS``, default 20 ms) and
then sleeps on a pipe that the sender pokes with a wake byte.  A spinning
receiver sees a message in a few microseconds instead of the ~70 us a pipe
wake-up costs.  The pipe also carries messages larger than the segment and
reports a peer that died (EOF).

Every message is framed as ``<QI`` (sequence number, CRC-32 of the body)
followed by the pickled body.  The receiver checks that the sequence number is
the one it expects next and that the CRC matches before unpickling; a frame
that fails either check raises ``ControlMessageError`` (an ``OSError``, so the
executor reports the rank as failed instead of acting on a torn or stale plan).

``ShmLink`` exposes the ``send`` / ``poll`` / ``recv`` subset of
``multiprocessing.Connection`` that the executor uses, so the failure handling
around it (bounded waits, liveness checks) is unchanged.  It plays the role of
the reference's SharedMemory + Event control plane
(nanovllm/engine/model_runner.py, shm command channel).
"""
from __future__ import annotations

import os
import pickle
import struct
import time
import zlib
from multiprocessing import shared_memory

import numpy as np

CTL = 4096           # control words, then the two data regions
_SEQ, _LEN, _SLEEP, _DONE = 0, 2, 4, 6   # + direction (0: driver -> worker, 1: worker -> driver)
_BIG = -1            # payload travels on the pipe
HEADER = struct.Struct("<QI")   # (sequence number, crc32 of the body)


class ControlMessageError(OSError):
    """A control frame failed its sequence or checksum check."""


def frame(seq: int, body: bytes) -> bytes:
    return HEADER.pack(seq, zlib.crc32(body)) + body


def unframe(data, want_seq: int):
    """Validate one frame and return the unpickled body."""
    if len(data) < HEADER.size:
        raise ControlMessageError(f"control frame of {len(data)} bytes is shorter than its header")
    seq, crc = HEADER.unpack_from(data)
    body = data[HEADER.size:]
    if seq != want_seq:
        raise ControlMessageError(f"control frame carries sequence {seq}, expected {want_seq}")
    if zlib.crc32(body) != crc:
        raise ControlMessageError(f"control frame {seq} failed its checksum")
    return pickle.loads(body)


def _spin_s() -> float:
    return float(os.environ.get("B200MOE_SPIN_MS", "20")) / 1e3


class ShmLink:
    """One end of a bidirectional link. ``side`` 0 = driver, 1 = worker."""

    def __init__(self, name: str, pipe, side: int, capacity: int, create: bool = False):
        self.capacity = capacity
        self.shm = shared_memory.SharedMemory(name=name, create=create, size=CTL + 2 * capacity if create else 0)
        self.ctl = np.ndarray((8,), dtype=np.int64, buffer=self.shm.buf)
        if create:
            self.ctl[:] = 0
        self.pipe, self.side = pipe, side
        self.out_dir, self.in_dir = side, 1 - side
        self.sent = 0
        self.seen = 0
        self.spin_s = _spin_s()

    @classmethod
    def create(cls, pipe, capacity: int = 8 << 20) -> "ShmLink":
        shm = shared_memory.SharedMemory(create=True, size=CTL + 2 * capacity)
        name = shm.name
        shm.close()
        link = cls(name, pipe, 0, capacity)
        link._owner = True
        return link

    def spec(self) -> tuple[str, int]:
        return self.shm.name, self.capacity

    def _region(self, direction: int) -> memoryview:
        off = CTL + direction * self.capacity
        return self.shm.buf[off:off + self.capacity]

    # ---------------------------------------------------------------- send
    def send(self, obj, timeout: float = 60.0) -> None:
        # one message in flight per direction: wait until the peer consumed the last one
        deadline = time.monotonic() + timeout
        while int(self.ctl[_DONE + self.out_dir]) < self.sent:
            if time.monotonic() > deadline:
                raise BrokenPipeError("peer did not consume the previous message")
            time.sleep(0)
        data = frame(self.sent + 1, pickle.dumps(obj, protocol=5))
        if len(data) <= self.capacity:
            with self._region(self.out_dir) as region:
                region[:len(data)] = data
            self.ctl[_LEN + self.out_dir] = len(data)
        else:
            self.ctl[_LEN + self.out_dir] = _BIG
            self.pipe.send_bytes(b"P" + data)
        self.sent += 1
        self.ctl[_SEQ + self.out_dir] = self.sent  # publish after the payload
        if self.ctl[_SLEEP + self.in_dir]:
            self.pipe.send_bytes(b"w")

    # ---------------------------------------------------------------- receive
    def _ready(self) -> bool:
        return int(self.ctl[_SEQ + self.in_dir]) > self.seen

    def poll(self, timeout: float = 0.0) -> bool:
        if self._ready():
            return True
        deadline = time.monotonic() + timeout
        spin_end = time.monotonic() + min(timeout, self.spin_s)
        while time.monotonic() < spin_end:
            if self._ready():
                return True
        while True:
            remaining = deadline - time.monotonic()
            if remaining <= 0:
                return self._ready()
            self.ctl[_SLEEP + self.side] = 1
            try:
                if self._ready():
                    return True
                if self.pipe.poll(remaining):
                    # a wake byte (or a large payload that recv will read)
                    if self._ready():
                        return True
                    msg = self.pipe.recv_bytes()  # EOFError when the peer is gone
                    if msg[:1] == b"P":
                        self._stash = msg[1:]
            finally:
                self.ctl[_SLEEP + self.side] = 0

    def recv(self):
        while not self._ready():
            self.poll(1.0)
        n = int(self.ctl[_LEN + self.in_dir])
        if n == _BIG:
            data = getattr(self, "_stash", None)
            while data is None:
                msg = self.pipe.recv_bytes()
                if msg[:1] == b"P":
                    data = msg[1:]
            self._stash = None
        else:
            with self._region(self.in_dir) as region:
                data = bytes(region[:n])
        obj = unframe(data, self.seen + 1)
        self.seen += 1
        self.ctl[_DONE + self.in_dir] = self.seen
        return obj

    def close(self):
        try:
            del self.ctl
            self.shm.close()
            if getattr(self, "_owner", False):
                self.shm.unlink()
        except (FileNotFoundError, BufferError):
            pass
