"""Whole-block KV transfer between a prefill engine and a decode engine.

The pool layout ``[blocks, layers, k|v, kv_heads, block_size, head_dim]`` makes
one block of one sequence a single contiguous slab across every layer, so a
transfer moves ``n`` slabs (plus the int8 scale slabs when the pool is int8):

* ``LocalKVChannel``   device -> pinned host -> device in one process (the
                       staging cost of a host-routed transfer, no socket).
* ``TcpKVChannel``     pinned staging + one socket; frame header
                       ``<III`` = (n_blocks, data_bytes, scale_bytes), then the
                       data slabs, then the scale slabs.  ``KVFrameAssembler``
                       reassembles frames from a non-blocking socket so the
                       decode side interleaves reception with engine steps.
* ``NvlinkKVChannel``  same-node transfer: the decode engine exports a CUDA IPC
                       handle of its pool once; the prefill engine maps it on
                       its own GPU and copies block slabs with a plain ld/st
                       kernel straight into the decode GPU's memory (no host
                       staging, one NVLink crossing).

Export then import is a bit-exact copy.  Behaviour mirrors the reference's
channels (nanovllm/pd/kv_channel.py:28-220: block-granular export / import,
local and TCP channels, frame assembler); its pool layout differs, so the
frame payload (whole slabs instead of separate K and V planes) differs too.
"""
from __future__ import annotations

import socket
import struct

import torch

FRAME = struct.Struct("<III")


class KVBlockBuffer:
    """Host staging for ``n_blocks`` slabs of ``pool`` (pinned on CUDA hosts)."""

    def __init__(self, pool, n_blocks: int):
        pin = pool.data.is_cuda
        self.data = torch.empty((n_blocks,) + tuple(pool.data.shape[1:]), dtype=pool.data.dtype, pin_memory=pin)
        self.scales = None if pool.scales is None else torch.empty(
            (n_blocks,) + tuple(pool.scales.shape[1:]), dtype=pool.scales.dtype, pin_memory=pin)
        self.n_blocks = n_blocks

    def data_bytes(self, n: int) -> int:
        return self.data[:n].numel() * self.data.element_size()

    def scale_bytes(self, n: int) -> int:
        return 0 if self.scales is None else self.scales[:n].numel() * self.scales.element_size()


def _idx(ids, device) -> torch.Tensor:
    return torch.as_tensor(list(ids), dtype=torch.long, device=device)


def extract_blocks(pool, block_ids, buf: KVBlockBuffer) -> None:
    """pool[block_ids] -> buf[:n] (one gather on the device, one D2H copy)."""
    n = len(block_ids)
    assert n <= buf.n_blocks
    idx = _idx(block_ids, pool.data.device)
    buf.data[:n].copy_(pool.data.index_select(0, idx))
    if buf.scales is not None:
        buf.scales[:n].copy_(pool.scales.index_select(0, idx))


def import_blocks(pool, block_ids, buf: KVBlockBuffer) -> None:
    """buf[:n] -> pool[block_ids] (one H2D copy, one scatter on the device)."""
    n = len(block_ids)
    assert n <= buf.n_blocks
    idx = _idx(block_ids, pool.data.device)
    pool.data.index_copy_(0, idx, buf.data[:n].to(pool.data.device))
    if buf.scales is not None:
        pool.scales.index_copy_(0, idx, buf.scales[:n].to(pool.scales.device))
    if pool.data.is_cuda:
        torch.cuda.synchronize(pool.data.device)


class LocalKVChannel:
    def __init__(self, pool):
        self.pool = pool
        self.bytes_moved = 0

    def send(self, block_ids) -> KVBlockBuffer:
        buf = KVBlockBuffer(self.pool, len(block_ids))
        extract_blocks(self.pool, block_ids, buf)
        self.bytes_moved += buf.data_bytes(len(block_ids)) + buf.scale_bytes(len(block_ids))
        return buf

    def recv(self, block_ids, buf: KVBlockBuffer) -> None:
        import_blocks(self.pool, block_ids, buf)
        self.bytes_moved += buf.data_bytes(len(block_ids)) + buf.scale_bytes(len(block_ids))


class TcpKVChannel:
    def __init__(self, sock: socket.socket, pool, max_blocks: int):
        self.sock, self.pool = sock, pool
        self.buf = KVBlockBuffer(pool, max_blocks)
        self.bytes_moved = 0

    def _grow(self, n: int):
        if n > self.buf.n_blocks:
            self.buf = KVBlockBuffer(self.pool, max(n, 2 * self.buf.n_blocks))

    def send_blocks(self, block_ids) -> None:
        n = len(block_ids)
        self._grow(n)
        extract_blocks(self.pool, block_ids, self.buf)
        data = self.buf.data[:n].contiguous().view(torch.uint8).numpy().tobytes()
        scales = b"" if self.buf.scales is None else \
            self.buf.scales[:n].contiguous().view(torch.uint8).numpy().tobytes()
        blocking = self.sock.getblocking()
        self.sock.setblocking(True)
        try:
            self.sock.sendall(FRAME.pack(n, len(data), len(scales)))
            self.sock.sendall(data)
            if scales:
                self.sock.sendall(scales)
        finally:
            self.sock.setblocking(blocking)
        self.bytes_moved += len(data) + len(scales)

    def import_frame(self, block_ids, frame) -> None:
        """Import an assembled ``(n_blocks, data, scales)`` frame into ``block_ids``."""
        n, data, scales = frame
        if n > len(block_ids):
            raise ValueError(f"frame carries {n} blocks for a table of {len(block_ids)}")
        self._grow(n)
        self.buf.data[:n].view(torch.uint8).view(-1).copy_(torch.frombuffer(bytearray(data), dtype=torch.uint8))
        if scales:
            self.buf.scales[:n].view(torch.uint8).view(-1).copy_(torch.frombuffer(bytearray(scales),
                                                                                  dtype=torch.uint8))
        import_blocks(self.pool, list(block_ids)[:n], self.buf)
        self.bytes_moved += len(data) + len(scales)


class KVFrameAssembler:
    """Incremental reassembly of TcpKVChannel frames from a non-blocking socket."""

    def __init__(self):
        self._buf = bytearray()
        self._hdr = None

    def feed(self, chunk: bytes) -> list[tuple[int, bytes, bytes]]:
        self._buf += chunk
        out = []
        while True:
            if self._hdr is None:
                if len(self._buf) < FRAME.size:
                    break
                self._hdr = FRAME.unpack_from(self._buf)
                del self._buf[:FRAME.size]
            n, dl, sl = self._hdr
            if len(self._buf) < dl + sl:
                break
            out.append((n, bytes(self._buf[:dl]), bytes(self._buf[dl:dl + sl])))
            del self._buf[:dl + sl]
            self._hdr = None
        return out


# ------------------------------------------------------------------ NVLink
def export_pool_handle(pool) -> dict:
    """Decode side: what a same-node prefill engine needs to map this pool."""
    if not pool.data.is_cuda:
        raise RuntimeError("NVLink KV transfer needs a CUDA pool")

    from b200moe import ops
    C = ops.native()

    def one(t: torch.Tensor) -> dict:
        handle, offset = C.ipc_export(t.data_ptr(), t.device.index)
        return {"handle": bytes(handle.numpy()).hex(), "offset": int(offset),
                "block_bytes": t[0].numel() * t.element_size(), "blocks": t.shape[0]}
    out = {"device": pool.data.device.index, "data": one(pool.data)}
    if pool.scales is not None:
        out["scales"] = one(pool.scales)
    return out


class NvlinkKVChannel:
    """Prefill side: writes block slabs into a peer engine's pool over NVLink."""

    def __init__(self, pool, peer: dict):
        from b200moe import ops
        self.C = ops.native()
        self.pool = pool
        self.device = pool.data.device.index
        self._mapped = []
        self.dst = {}
        for key in ("data", "scales"):
            if key not in peer:
                continue
            h = torch.frombuffer(bytearray(bytes.fromhex(peer[key]["handle"])), dtype=torch.uint8)
            base = self.C.ipc_open(h, self.device)
            self._mapped.append(base)
            self.dst[key] = (base + peer[key]["offset"], peer[key]["block_bytes"])
        if (pool.scales is None) != ("scales" not in self.dst):
            raise ValueError("prefill and decode pools disagree on the KV dtype")
        if self.dst["data"][1] != pool.data[0].numel() * pool.data.element_size():
            raise ValueError("prefill and decode pools have different block layouts")
        self.bytes_moved = 0

    def send_blocks(self, src_ids, dst_ids) -> None:
        dev = self.pool.data.device
        s = torch.as_tensor(list(src_ids), dtype=torch.int32, device=dev)
        d = torch.as_tensor(list(dst_ids), dtype=torch.int32, device=dev)
        for key, src in (("data", self.pool.data), ("scales", self.pool.scales)):
            if key in self.dst:
                ptr, bb = self.dst[key]
                self.C.kv_blocks_copy(src, s, ptr, d, bb)
                self.bytes_moved += bb * len(src_ids)
        torch.cuda.synchronize(dev)  # the decode side is told only after the data landed

    def close(self):
        for p in self._mapped:
            self.C.ipc_close(p, self.device)
        self._mapped = []
