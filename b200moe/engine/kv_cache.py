"""Paged KV pool.

Layout: ``[num_blocks, num_layers, 2 (k|v), kv_heads, block_size, head_dim]``.
One block of one sequence is a single contiguous slab holding every layer,
so host offload and PD hand-off move one block with one copy, while the
attention kernels see, per layer, contiguous ``block_size x head_dim`` rows per
(block, kv head) at a fixed ``block_stride``.  The last block is a scratch
block the scheduler never hands out: padded CUDA-graph rows write there
(the reference keeps the same extra block, nanovllm/engine/model_runner.py:440-446).

int8 KV has two modes.  "token" keeps one fp32 scale per (block, layer, k|v,
head, token) in a parallel pool (per-token-head absmax quantisation).  "channel"
is the reference's calibrated mixed-precision mode
(nanovllm/kernels/kv_int8.py:1-24): per-channel store scales frozen after a
calibration pass (amax / 127), and up to NOUT_MAX outlier dims per (layer, kv
head) -- dims whose amax / mean|x| exceeds 10 -- kept exactly in bf16 in a side
pool, their int8 payload zero and their read scale 0.  Rounding is
floor(x / scale + 0.5), clamped to [-127, 127].
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


NOUT_MAX = 4               # exact bf16 outlier dims per (layer, kv head) in channel mode
OUTLIER_RATIO = 10.0       # amax / mean|x| above which a dim is an outlier


@dataclass
class ChannelInt8:
    """Per-layer state of the channel-mode int8 KV (views into the pool's tensors)."""
    scale: torch.Tensor        # [2, kv_heads, D] fp32 store scales
    dscale: torch.Tensor       # [2, kv_heads, D] fp32 read scales, 0 at outlier dims
    out_idx: torch.Tensor      # [kv_heads, NOUT_MAX] int32 outlier dims (padded with 0)
    n_out: torch.Tensor        # [kv_heads] int32 outlier dims in use
    side_k: torch.Tensor       # [num_blocks, kv_heads, block_size, NOUT_MAX] bf16 (strided over blocks)
    side_v: torch.Tensor
    side_block_stride: int
    calib_amax: torch.Tensor   # [2, kv_heads, D] running max |x| while calibrating
    calib_sum: torch.Tensor    # [2, kv_heads, D] running sum |x| while calibrating
    calibrating: bool = False


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
    chan: ChannelInt8 | None = None

    def store(self, slot_mapping: torch.Tensor, k: torch.Tensor, v: torch.Tensor):
        """Reference store (CPU path): k/v [T, kv_heads, D] at flat slots."""
        slots = slot_mapping.long()
        keep = slots >= 0
        slots, k, v = slots[keep], k[keep], v[keep]
        blk, off = slots // self.block_size, slots % self.block_size
        if self.chan is not None:
            c = self.chan
            for kv, (src, dst, side) in enumerate(((k, self.k, c.side_k), (v, self.v, c.side_v))):
                x = src.to(torch.bfloat16).float()
                if c.calibrating:
                    c.calib_amax[kv] = torch.maximum(c.calib_amax[kv], x.abs().amax(dim=0))
                    c.calib_sum[kv] += x.abs().sum(dim=0)
                q = torch.clamp(torch.floor(x / c.scale[kv] + 0.5), -127, 127).to(torch.int8)
                for h in range(self.num_kv_heads):
                    n = int(c.n_out[h])
                    if n:
                        dims = c.out_idx[h, :n].long()
                        side[blk, h, off, :n] = x[:, h, dims].to(torch.bfloat16)
                        q[:, h, dims] = 0
                dst[blk, :, off] = q
            return
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

        if self.chan is not None:
            c = self.chan

            def chan(pool, side, kv):
                x = (pool[blocks].float() * c.dscale[kv].unsqueeze(1)).to(torch.bfloat16)  # [nb, H, bs, D]
                sd = side[blocks]                                                         # [nb, H, bs, NOUT]
                for h in range(self.num_kv_heads):
                    n = int(c.n_out[h])
                    if n:
                        x[:, h, :, c.out_idx[h, :n].long()] = sd[:, h, :, :n]
                return x.permute(0, 2, 1, 3).reshape(nb * self.block_size, self.num_kv_heads, -1)[:length]

            return chan(self.k, c.side_k, 0), chan(self.v, c.side_v, 1)
        return one(self.k, self.k_scale), one(self.v, self.v_scale)


class KVPool:

    def __init__(self, num_blocks: int, num_layers: int, num_kv_heads: int, block_size: int, head_dim: int,
                 dtype: torch.dtype, device, int8: bool = False, int8_mode: str = "token"):
        if int8_mode not in ("token", "channel"):
            raise ValueError("int8_mode must be 'token' or 'channel'")
        self.num_blocks = num_blocks          # including the scratch block
        self.num_layers = num_layers
        self.num_kv_heads = num_kv_heads
        self.block_size = block_size
        self.head_dim = head_dim
        self.int8 = int8
        self.int8_mode = int8_mode if int8 else None
        store_dtype = torch.int8 if int8 else dtype
        self.data = torch.zeros(num_blocks, num_layers, 2, num_kv_heads, block_size, head_dim,
                                dtype=store_dtype, device=device)
        token = int8 and int8_mode == "token"
        self.scales = (torch.ones(num_blocks, num_layers, 2, num_kv_heads, block_size, dtype=torch.float32,
                                  device=device) if token else None)
        self.block_stride = num_layers * 2 * num_kv_heads * block_size * head_dim
        self.scale_block_stride = num_layers * 2 * num_kv_heads * block_size
        self.side = None
        if self.int8_mode == "channel":
            L, H, D = num_layers, num_kv_heads, head_dim
            self.side = torch.zeros(num_blocks, L, 2, H, block_size, NOUT_MAX, dtype=torch.bfloat16, device=device)
            # until calibration is frozen: a unit-range grid (values saturate; only statistics matter then)
            self.ch_scale = torch.full((L, 2, H, D), 1.0 / 127.0, dtype=torch.float32, device=device)
            self.ch_dscale = self.ch_scale.clone()
            self.out_idx = torch.zeros(L, H, NOUT_MAX, dtype=torch.int32, device=device)
            self.n_out = torch.zeros(L, H, dtype=torch.int32, device=device)
            self.calib_amax = torch.zeros(L, 2, H, D, dtype=torch.float32, device=device)
            self.calib_sum = torch.zeros(L, 2, H, D, dtype=torch.float32, device=device)
            self.side_block_stride = L * 2 * H * block_size * NOUT_MAX
        self._layers = [self._make_layer(l) for l in range(num_layers)]

    @staticmethod
    def bytes_per_block(num_layers, num_kv_heads, block_size, head_dim, dtype, int8=False,
                        int8_mode: str = "token") -> int:
        elem = 1 if int8 else torch.empty(0, dtype=dtype).element_size()
        b = num_layers * 2 * num_kv_heads * block_size * head_dim * elem
        if int8 and int8_mode == "token":
            b += num_layers * 2 * num_kv_heads * block_size * 4
        elif int8:
            b += num_layers * 2 * num_kv_heads * block_size * NOUT_MAX * 2
        return b

    # ------------------------------------------------- channel-mode calibration
    def calibrate_begin(self):
        """Start collecting per-channel max |x| and sum |x| of every K / V stored."""
        self.calib_amax.zero_()
        self.calib_sum.zero_()
        for ly in self._layers:
            ly.chan.calibrating = True

    def calibrate_freeze(self, tokens_seen: int) -> int:
        """Freeze store scales (amax / 127), outlier dims (the first NOUT_MAX dims, in
        index order, whose K-or-V amax / mean|x| exceeds OUTLIER_RATIO) and read
        scales (0 at outlier dims); returns the number of outlier dims
        (reference: nanovllm/engine/model_runner.py:kv_calibrate_freeze)."""
        for ly in self._layers:
            ly.chan.calibrating = False
        mean = (self.calib_sum / max(tokens_seen, 1)).clamp_min(1e-6)
        self.ch_scale.copy_((self.calib_amax / 127.0).clamp_min(1e-6))
        ratio = torch.maximum(self.calib_amax[:, 0] / mean[:, 0], self.calib_amax[:, 1] / mean[:, 1])  # [L, H, D]
        self.ch_dscale.copy_(self.ch_scale)
        self.out_idx.zero_()
        self.n_out.zero_()
        total = 0
        ratio = ratio.cpu()
        for l in range(self.num_layers):
            for h in range(self.num_kv_heads):
                dims = (ratio[l, h] > OUTLIER_RATIO).nonzero().flatten()[:NOUT_MAX]
                n = int(dims.numel())
                total += n
                if n:
                    self.out_idx[l, h, :n] = dims.to(self.out_idx.device, torch.int32)
                    self.n_out[l, h] = n
                    self.ch_dscale[l, :, h, dims.to(self.ch_dscale.device)] = 0.0
        return total

    @property
    def scratch_block(self) -> int:
        return self.num_blocks - 1

    def _make_layer(self, l: int) -> KVLayer:
        chan = None
        if self.int8_mode == "channel":
            chan = ChannelInt8(scale=self.ch_scale[l], dscale=self.ch_dscale[l], out_idx=self.out_idx[l],
                               n_out=self.n_out[l], side_k=self.side[:, l, 0], side_v=self.side[:, l, 1],
                               side_block_stride=self.side_block_stride, calib_amax=self.calib_amax[l],
                               calib_sum=self.calib_sum[l])
        return KVLayer(
            k=self.data[:, l, 0], v=self.data[:, l, 1],
            k_scale=None if self.scales is None else self.scales[:, l, 0],
            v_scale=None if self.scales is None else self.scales[:, l, 1],
            block_size=self.block_size, block_stride=self.block_stride,
            scale_block_stride=self.scale_block_stride, num_kv_heads=self.num_kv_heads, chan=chan)

    def layer(self, l: int) -> KVLayer:
        return self._layers[l]

    def block_view(self, block_id: int) -> torch.Tensor:
        """All layers of one block as one contiguous tensor (offload / PD)."""
        return self.data[block_id]
