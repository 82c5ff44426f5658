"""Paged KV pool.

Layout: ``[num_blocks, num_layers, 2 (k|v), kv_heads, block_size, head_dim]``.
One block of one sequence is a single contiguous slab holding every layer,
so host offload and PD hand-off move one block with one copy, while the
attention kernels see, per layer, contiguous ``block_size x head_dim`` rows per
(block, kv head) at a fixed ``block_stride``.  The last block is a scratch
block the scheduler never hands out: padded CUDA-graph rows write there
(the reference keeps the same extra block, nanovllm/engine/model_runner.py:440-446).

int8 KV keeps one fp32 scale per (block, layer, k|v, head, token) in a
parallel pool (per-token-head absmax quantisation).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class KVLayer:
    k: torch.Tensor            # view [num_blocks, kv_heads, block_size, D] (strided over blocks)
    v: torch.Tensor
    k_scale: torch.Tensor | None
    v_scale: torch.Tensor | None
    block_size: int
    block_stride: int
    scale_block_stride: int
    num_kv_heads: int

    def store(self, slot_mapping: torch.Tensor, k: torch.Tensor, v: torch.Tensor):
        """Reference store (CPU path): k/v [T, kv_heads, D] at flat slots."""
        slots = slot_mapping.long()
        keep = slots >= 0
        slots, k, v = slots[keep], k[keep], v[keep]
        blk, off = slots // self.block_size, slots % self.block_size
        if self.k.dtype == torch.int8:
            for src, dst, sc in ((k, self.k, self.k_scale), (v, self.v, self.v_scale)):
                a = src.float().abs().amax(dim=-1)
                s = torch.where(a > 0, a / 127.0, torch.ones_like(a))
                q = torch.clamp(torch.round(src.float() / s.unsqueeze(-1)), -127, 127).to(torch.int8)
                dst[blk, :, off] = q
                sc[blk, :, off] = s
            return
        self.k[blk, :, off] = k.to(self.k.dtype)
        self.v[blk, :, off] = v.to(self.v.dtype)

    def gather(self, block_table_row: torch.Tensor, length: int):
        """[length, kv_heads, D] keys and values of one sequence (dequantised)."""
        nb = (length + self.block_size - 1) // self.block_size
        blocks = block_table_row[:nb].long()

        def one(pool, scale):
            x = pool[blocks]  # [nb, H, bs, D]
            if scale is not None:
                x = x.float() * scale[blocks].unsqueeze(-1)
            return x.permute(0, 2, 1, 3).reshape(nb * self.block_size, self.num_kv_heads, -1)[:length]

        return one(self.k, self.k_scale), one(self.v, self.v_scale)


class KVPool:

    def __init__(self, num_blocks: int, num_layers: int, num_kv_heads: int, block_size: int, head_dim: int,
                 dtype: torch.dtype, device, int8: bool = False):
        self.num_blocks = num_blocks          # including the scratch block
        self.num_layers = num_layers
        self.num_kv_heads = num_kv_heads
        self.block_size = block_size
        self.head_dim = head_dim
        self.int8 = int8
        store_dtype = torch.int8 if int8 else dtype
        self.data = torch.zeros(num_blocks, num_layers, 2, num_kv_heads, block_size, head_dim,
                                dtype=store_dtype, device=device)
        self.scales = (torch.ones(num_blocks, num_layers, 2, num_kv_heads, block_size, dtype=torch.float32,
                                  device=device) if int8 else None)
        self.block_stride = num_layers * 2 * num_kv_heads * block_size * head_dim
        self.scale_block_stride = num_layers * 2 * num_kv_heads * block_size
        self._layers = [self._make_layer(l) for l in range(num_layers)]

    @staticmethod
    def bytes_per_block(num_layers, num_kv_heads, block_size, head_dim, dtype, int8=False) -> int:
        elem = 1 if int8 else torch.empty(0, dtype=dtype).element_size()
        b = num_layers * 2 * num_kv_heads * block_size * head_dim * elem
        if int8:
            b += num_layers * 2 * num_kv_heads * block_size * 4
        return b

    @property
    def scratch_block(self) -> int:
        return self.num_blocks - 1

    def _make_layer(self, l: int) -> KVLayer:
        return KVLayer(
            k=self.data[:, l, 0], v=self.data[:, l, 1],
            k_scale=None if self.scales is None else self.scales[:, l, 0],
            v_scale=None if self.scales is None else self.scales[:, l, 1],
            block_size=self.block_size, block_stride=self.block_stride,
            scale_block_stride=self.scale_block_stride, num_kv_heads=self.num_kv_heads)

    def layer(self, l: int) -> KVLayer:
        return self._layers[l]

    def block_view(self, block_id: int) -> torch.Tensor:
        """All layers of one block as one contiguous tensor (offload / PD)."""
        return self.data[block_id]
