"""The allocation-free decode attention C entry point (``b200moe_decode_attn_noalloc``
exported by the native extension) against the regular ``ops.decode_attention``
and the fp32 reference.  Named to be collected last; it also passes alone."""
import ctypes
import math

import pytest
import torch

from b200moe import ops
from b200moe.engine.kv_cache import KVPool

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _lib():
    mod = ops.native()  # loads the extension (and torch's libraries) into the process
    lib = ctypes.CDLL(mod.__file__)
    f = lib.b200moe_decode_attn_noalloc
    f.restype = ctypes.c_int
    f.argtypes = ([ctypes.c_void_p] * 5 + [ctypes.c_int] + [ctypes.c_void_p] * 2 + [ctypes.c_int] * 3
                  + [ctypes.c_longlong] + [ctypes.c_int] * 3 + [ctypes.c_float] + [ctypes.c_int] * 2
                  + [ctypes.c_void_p] * 2 + [ctypes.c_char_p, ctypes.c_int])
    lib.b200moe_decode_attn_noalloc_max_rows.restype = ctypes.c_int
    return lib


def _setup(seq_lens, nq, nkv, D, bs, int8):
    nb = [math.ceil(L / bs) for L in seq_lens]
    pool = KVPool(sum(nb) + 2, 1, nkv, bs, D, torch.bfloat16, DEV, int8=int8)
    perm = torch.randperm(pool.num_blocks - 1).tolist()
    tables = torch.zeros(len(seq_lens), max(nb), dtype=torch.int32)
    i = 0
    for b, n in enumerate(nb):
        tables[b, :n] = torch.tensor(perm[i:i + n])
        i += n
    layer = pool.layer(0)
    for b, L in enumerate(seq_lens):
        pos = torch.arange(L)
        slots = (tables[b][pos // bs].long() * bs + pos % bs).to(torch.int32).to(DEV)
        layer.store(slots, torch.randn(L, nkv, D, device=DEV).to(torch.bfloat16),
                    torch.randn(L, nkv, D, device=DEV).to(torch.bfloat16))
    q = torch.randn(len(seq_lens), nq, D, device=DEV).to(torch.bfloat16)
    return layer, tables.to(DEV), torch.tensor(seq_lens, dtype=torch.int32, device=DEV), q


def _call(lib, q, layer, tables, lens, scale, out, split_len, nsplit):
    err = ctypes.create_string_buffer(512)
    ptr = lambda t: None if t is None else t.data_ptr()
    rc = lib.b200moe_decode_attn_noalloc(
        ptr(q), ptr(layer.k), ptr(layer.v), ptr(layer.k_scale), ptr(layer.v_scale), int(layer.k.dtype == torch.int8),
        ptr(tables), ptr(lens), q.shape[0], tables.shape[1], layer.block_size, layer.block_stride, q.shape[1],
        layer.num_kv_heads, q.shape[2], scale, nsplit, split_len, ptr(out),
        torch.cuda.current_stream().cuda_stream, err, len(err))
    return rc, err.value.decode()


@pytest.mark.parametrize("int8", [False, True])
def test_noalloc_matches_decode_attention(int8):
    lib = _lib()
    D, nq, nkv, bs = 128, 32, 4, 16
    seq_lens = [1, 17, 255, 256, 257, 700, 1300, 64]
    layer, tables, lens, q = _setup(seq_lens, nq, nkv, D, bs, int8)
    B, scale = len(seq_lens), D ** -0.5
    ref = torch.empty(B, nq, D, device=DEV)
    ops._attention_ref(q, layer, tables, lens, torch.arange(B + 1, dtype=torch.int32), scale, ref)
    for split_len, nsplit in [(256, 6), (64, 21), (2048, 1)]:
        ws = (torch.empty(B * nq * nsplit, D, device=DEV), torch.empty(B * nq * nsplit, device=DEV),
              torch.empty(B * nq * nsplit, device=DEV))
        want = torch.empty(B, nq, D, dtype=torch.bfloat16, device=DEV)
        ops.decode_attention(q, layer, tables, lens, scale, want, split_len, nsplit, ws)
        for _ in range(2):  # two calls in a row reuse the same scratch
            got = torch.full((B, nq, D), float("nan"), dtype=torch.bfloat16, device=DEV)
            rc, msg = _call(lib, q, layer, tables, lens, scale, got, split_len, nsplit)
            assert rc == 0, msg
            torch.cuda.synchronize()
            torch.testing.assert_close(got.float(), want.float(), atol=1e-2, rtol=1e-2)
            torch.testing.assert_close(got.float(), ref, atol=2e-2, rtol=2e-2)


def test_noalloc_rejects_oversize():
    lib = _lib()
    max_rows = lib.b200moe_decode_attn_noalloc_max_rows()
    D, nq, nkv, bs = 128, 32, 4, 16
    layer, tables, lens, q = _setup([64, 64], nq, nkv, D, bs, False)
    out = torch.zeros(2, nq, D, dtype=torch.bfloat16, device=DEV)
    nsplit = max_rows // (2 * nq) + 1  # one split more than the scratch holds
    rc, msg = _call(lib, q, layer, tables, lens, D ** -0.5, out, 64, nsplit)
    assert rc == 2 and "exceeds the scratch limit" in msg
    assert out.abs().sum().item() == 0  # nothing was launched
    rc, msg = _call(lib, q, layer, tables, lens, D ** -0.5, out, 100, 2)
    assert rc == 1 and "split_len" in msg


def test_noalloc_rejects_invalid_arguments():
    """Every malformed shape returns code 1 before anything is launched (a zero head
    count once reached an integer division on the host, a zero split length one on
    the device)."""
    lib = _lib()
    D, nq, nkv, bs = 128, 32, 4, 16
    layer, tables, lens, q = _setup([64, 64], nq, nkv, D, bs, False)
    out = torch.zeros(2, nq, D, dtype=torch.bfloat16, device=DEV)
    good = dict(nq=nq, nkv=nkv, max_blocks=tables.shape[1], block_size=bs, block_stride=layer.block_stride,
                split_len=64, nsplit=2, head_dim=D)
    bad = [dict(nq=0), dict(nkv=0), dict(nq=33), dict(nq=128, nkv=4), dict(nq=12, nkv=4), dict(split_len=0),
           dict(split_len=-64), dict(max_blocks=0), dict(block_stride=0), dict(block_stride=-1), dict(block_size=0),
           dict(nsplit=0), dict(head_dim=96)]
    for case in bad:
        a = {**good, **case}
        err = ctypes.create_string_buffer(512)
        rc = lib.b200moe_decode_attn_noalloc(
            q.data_ptr(), layer.k.data_ptr(), layer.v.data_ptr(), None, None, 0, tables.data_ptr(), lens.data_ptr(),
            2, a["max_blocks"], a["block_size"], a["block_stride"], a["nq"], a["nkv"], a["head_dim"], D ** -0.5,
            a["nsplit"], a["split_len"], out.data_ptr(), torch.cuda.current_stream().cuda_stream, err, len(err))
        assert rc == 1, (case, rc, err.value)
        assert err.value, case
    err = ctypes.create_string_buffer(512)
    rc = lib.b200moe_decode_attn_noalloc(  # int8 KV without scales
        q.data_ptr(), layer.k.data_ptr(), layer.v.data_ptr(), None, None, 1, tables.data_ptr(), lens.data_ptr(), 2,
        good["max_blocks"], bs, good["block_stride"], nq, nkv, D, D ** -0.5, 2, 64, out.data_ptr(),
        torch.cuda.current_stream().cuda_stream, err, len(err))
    assert rc == 1 and b"scale" in err.value
    torch.cuda.synchronize()
    assert out.abs().sum().item() == 0  # nothing was launched
