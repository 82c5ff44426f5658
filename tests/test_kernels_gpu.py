"""Native sm_100a kernels against plain-PyTorch fp32 references of the same op."""
import math

import numpy as np
import pytest
import torch

from b200moe import ops
from b200moe.engine.kv_cache import KVPool
from b200moe.utils.weights import quantize_block_fp8

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _fp8_weight(groups, n, k, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    w = torch.randn(groups, n, k, generator=g, device=DEV) * 0.05
    return quantize_block_fp8(w)


def _ref_w(q, s):
    # the kernel dequantises to bf16 before the MMA
    return ops.dequant_block_fp8(q, s).to(torch.bfloat16).float()


def _close(out, ref, tol=2e-2):
    err = (out.float() - ref).abs().max().item()
    scale = ref.abs().max().item() + 1e-6
    assert err <= tol * scale, f"max err {err:.4g} vs scale {scale:.4g}"


@pytest.mark.parametrize("T", [1, 7, 64, 300])
@pytest.mark.parametrize("n,k", [(512, 256), (5120, 2048)])
def test_gemm_fp8_dense(T, n, k):
    q, s = _fp8_weight(1, n, k, 1)
    x = (torch.randn(T, k, device=DEV) * 0.5).to(torch.bfloat16)
    out = ops.linear(x, q[0], s[0])
    torch.cuda.synchronize()
    ops.check_status(DEV)
    _close(out, x.float() @ _ref_w(q[0], s[0]).t())


@pytest.mark.parametrize("T", [1, 64, 256])
def test_gemm_fp8_split_k(T):
    """o_proj shape at decode token counts: the planner splits K; partials are summed."""
    n, k = 2048, 4096
    bn, splits = ops.plan_dense(T, n // 128, k // 64)
    assert splits > 1
    q, s = _fp8_weight(1, n, k, 5)
    x = (torch.randn(T, k, device=DEV) * 0.5).to(torch.bfloat16)
    out = ops.linear(x, q[0], s[0])
    torch.cuda.synchronize()
    ops.check_status(DEV)
    _close(out, x.float() @ _ref_w(q[0], s[0]).t())


def test_fp8_dequant_bit_exact():
    """One-hot activations read the dequantised weight back: it must equal
    bf16(float(q) * scale) bit for bit (up to the sign of zero), for every
    e4m3 code (subnormals included) and for tiny, ordinary and >= 256 block scales."""
    n = k = 256
    g = torch.Generator().manual_seed(7)
    codes = torch.randint(0, 256, (n, k), generator=g, dtype=torch.int32)
    codes = torch.where((codes & 0x7F) == 0x7F, codes - 1, codes)  # no NaN codes
    q = codes.to(torch.uint8).view(torch.float8_e4m3fn).to(DEV)
    s = torch.tensor([[3.1e-5, 0.0123], [300.0, 1.7]], dtype=torch.float32, device=DEV)
    x = torch.eye(k, dtype=torch.bfloat16, device=DEV)
    out = ops.linear(x, q, s)  # out[t, m] = W[m, t]
    torch.cuda.synchronize()
    sfull = s.repeat_interleave(128, 0).repeat_interleave(128, 1)
    want = (q.float() * sfull).to(torch.bfloat16)
    got = out.t().contiguous()
    # bit-exact except the sign of zero (e4m3 -0 may come out as +0, identical in any product or sum)
    diff = (got.view(torch.int16) != want.view(torch.int16)) & ~((got == 0) & (want == 0))
    bad = diff.nonzero().tolist()
    detail = [(m, t, int(codes[m, t]), float(sfull[m, t]), float(got[m, t]), float(want[m, t]))
              for m, t in bad[:8]]
    assert not bad, f"{len(bad)} mismatches (m, k, code, scale, got, want): {detail}"


@pytest.mark.parametrize("T", [1, 64, 256])
def test_linear_add_rmsnorm_fused_equals_separate(T):
    """o_proj + residual + RMSNorm: split-K partials reduced inside the norm
    kernel give the same bits as the separate reduce + rmsnorm."""
    n, k = 2048, 4096
    q, s = _fp8_weight(1, n, k, 11)
    x = (torch.randn(T, k, device=DEV) * 0.5).to(torch.bfloat16)
    res = (torch.randn(T, n, device=DEV)).to(torch.bfloat16)
    nw = (1 + 0.1 * torch.randn(n, device=DEV)).to(torch.bfloat16)
    r1, r2 = res.clone(), res.clone()
    a = ops.linear_add_rmsnorm(x, q[0], s[0], r1, nw, 1e-6, out=torch.empty_like(res))
    b = ops.rmsnorm(ops.linear(x, q[0], s[0]), nw, 1e-6, residual=r2, out=torch.empty_like(res))
    torch.cuda.synchronize()
    assert torch.equal(a, b) and torch.equal(r1, r2)


@pytest.mark.parametrize("T", [3, 200])
def test_gemm_bf16_f32_out(T):
    w = (torch.randn(256, 2048, device=DEV) * 0.02).to(torch.bfloat16)
    x = torch.randn(T, 2048, device=DEV).to(torch.bfloat16)
    out = ops.linear(x, w, None, out_dtype=torch.float32)
    _close(out, x.float() @ w.float().t(), tol=1e-2)


@pytest.mark.parametrize("bn", [16, 32, 64, 128, 256])
def test_grouped_gate_up_and_down(bn):
    E, I, H = 8, 128, 256
    torch.manual_seed(0)
    counts = torch.tensor([5, 0, 17, 1, 40, 3, 0, 9], dtype=torch.int32, device=DEV)
    rows = int(counts.sum())
    offsets = torch.zeros(E + 1, dtype=torch.int32, device=DEV)
    offsets[1:] = torch.cumsum(counts, 0)
    q13, s13 = _fp8_weight(E, 2 * I, H, 2)
    q2, s2 = _fp8_weight(E, H, I, 3)
    x = (torch.randn(rows, H, device=DEV) * 0.5).to(torch.bfloat16)
    h = torch.empty(rows, I, dtype=torch.bfloat16, device=DEV)
    ops.grouped_gate_up_silu(x, q13, s13, counts, offsets, h, I, bn=min(bn, 128))  # the gate/up pair tile is at most 128 tokens
    slot_of_row = torch.randperm(rows, device=DEV).to(torch.int32)
    wts = torch.rand(rows, device=DEV)
    slots = torch.zeros(rows, H, dtype=torch.bfloat16, device=DEV)
    ops.grouped_down_scatter(h, q2, s2, counts, offsets, slot_of_row, wts, slots, bn=bn)
    torch.cuda.synchronize()
    ops.check_status(DEV)
    cpu_off = offsets.tolist()
    href = torch.empty(rows, I, device=DEV)
    yref = torch.empty(rows, H, device=DEV)
    for e in range(E):
        a, b = cpu_off[e], cpu_off[e + 1]
        if a == b:
            continue
        gu = x[a:b].float() @ _ref_w(q13[e], s13[e]).t()
        he = torch.nn.functional.silu(gu[:, :I]) * gu[:, I:]
        href[a:b] = he
        yref[a:b] = h[a:b].float() @ _ref_w(q2[e], s2[e]).t()
    _close(h, href)
    ref_slots = torch.empty_like(yref)
    ref_slots[slot_of_row.long()] = yref * wts[slot_of_row.long()].unsqueeze(1)
    _close(slots, ref_slots)


@pytest.mark.parametrize("bn", [32, 128, 256])
def test_tile_major_weights_same_bits(bn):
    """e4m3 weights stored tile-major (one contiguous block per pipeline stage)
    give bit-identical GEMM results: dense, split-K, gate/up pair and scatter."""
    for T, n, k in [(300, 5120, 2048), (64, 2048, 4096), (7, 256, 256)]:
        q, s = _fp8_weight(1, n, k, 1)
        x = (torch.randn(T, k, device=DEV) * 0.5).to(torch.bfloat16)
        a = ops.linear(x, q[0], s[0])
        b = ops.linear(x, ops.tile_fp8(q[0]), s[0], tiled=True)
        assert torch.equal(a, b), (T, n, k)
    E, I, H = 8, 256, 512
    counts = torch.tensor([5, 0, 17, 1, 300, 3, 0, 9], dtype=torch.int32, device=DEV)
    rows = int(counts.sum())
    offsets = torch.zeros(E + 1, dtype=torch.int32, device=DEV)
    offsets[1:] = torch.cumsum(counts, 0)
    q13, s13 = _fp8_weight(E, 2 * I, H, 2)
    q2, s2 = _fp8_weight(E, H, I, 3)
    x = (torch.randn(rows, H, device=DEV) * 0.5).to(torch.bfloat16)
    h1, h2 = (torch.empty(rows, I, dtype=torch.bfloat16, device=DEV) for _ in range(2))
    ops.grouped_gate_up_silu(x, q13, s13, counts, offsets, h1, I, bn=min(bn, 128))
    ops.grouped_gate_up_silu(x, ops.tile_fp8(q13), s13, counts, offsets, h2, I, bn=min(bn, 128), tiled=True)
    assert torch.equal(h1, h2)
    sor = torch.randperm(rows, device=DEV).to(torch.int32)
    wts = torch.rand(rows, device=DEV)
    y1, y2 = (torch.zeros(rows, H, dtype=torch.bfloat16, device=DEV) for _ in range(2))
    ops.grouped_down_scatter(h1, q2, s2, counts, offsets, sor, wts, y1, bn=bn)
    ops.grouped_down_scatter(h1, ops.tile_fp8(q2), s2, counts, offsets, sor, wts, y2, bn=bn, tiled=True)
    torch.cuda.synchronize()
    ops.check_status(DEV)
    assert torch.equal(y1, y2)


@pytest.mark.parametrize("tiled", [False, True])
def test_bf16_expert_path_same_bits(tiled):
    """Large prefill steps dequantise the expert weights once (dequant_weights)
    and run the bf16 grouped GEMMs: the weights equal bf16(float(q) * scale) and
    both GEMMs give the e4m3 path's bits."""
    E, I, H = 8, 256, 512
    counts = torch.tensor([5, 0, 17, 1, 300, 3, 0, 129], dtype=torch.int32, device=DEV)
    rows = int(counts.sum())
    offsets = torch.zeros(E + 1, dtype=torch.int32, device=DEV)
    offsets[1:] = torch.cumsum(counts, 0)
    q13, s13 = _fp8_weight(E, 2 * I, H, 2)
    q2, s2 = _fp8_weight(E, H, I, 3)
    w13 = torch.empty(E, 2 * I, H, dtype=torch.bfloat16, device=DEV)
    w2 = torch.empty(E, H, I, dtype=torch.bfloat16, device=DEV)
    ops.dequant_weights(ops.tile_fp8(q13) if tiled else q13, s13, w13, tiled)
    ops.dequant_weights(ops.tile_fp8(q2) if tiled else q2, s2, w2, tiled)
    for e in range(E):
        want = (q13[e].float() * s13[e].repeat_interleave(128, 0).repeat_interleave(128, 1)).to(torch.bfloat16)
        assert torch.equal(w13[e], want), e
    x = (torch.randn(rows, H, device=DEV) * 0.5).to(torch.bfloat16)
    h1, h2 = (torch.empty(rows, I, dtype=torch.bfloat16, device=DEV) for _ in range(2))
    for bn in (64, 128):
        ops.grouped_gate_up_silu(x, q13, s13, counts, offsets, h1, I, bn=bn)
        ops.grouped_gate_up_silu(x, w13, None, counts, offsets, h2, I, bn=bn)
        assert torch.equal(h1, h2), bn
    sor = torch.randperm(rows, device=DEV).to(torch.int32)
    wts = torch.rand(rows, device=DEV)
    for bn in (64, 256):
        y1, y2 = (torch.zeros(rows, H, dtype=torch.bfloat16, device=DEV) for _ in range(2))
        ops.grouped_down_scatter(h1, q2, s2, counts, offsets, sor, wts, y1, bn=bn)
        ops.grouped_down_scatter(h1, w2, None, counts, offsets, sor, wts, y2, bn=bn)
        torch.cuda.synchronize()
        ops.check_status(DEV)
        assert torch.equal(y1, y2), bn


@pytest.mark.parametrize("tiled", [False, True])
def test_dense_bf16_once_same_bits(tiled, monkeypatch):
    """Prefill-size dense GEMMs dequantise the weight once and run in bf16: the
    result equals the e4m3 path's bits."""
    T, n, k = 2100, 1024, 2048
    q, s = _fp8_weight(1, n, k, 6)
    w = ops.tile_fp8(q[0]) if tiled else q[0]
    x = (torch.randn(T, k, device=DEV) * 0.5).to(torch.bfloat16)
    a = ops.linear(x, w, s[0], tiled=tiled)
    monkeypatch.setattr(ops, "BF16_DENSE_ROWS", 0)
    b = ops.linear(x, w, s[0], tiled=tiled)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    _close(a, x.float() @ _ref_w(q[0], s[0]).t())


def test_rmsnorm_and_add():
    T, H = 33, 2048
    x = torch.randn(T, H, device=DEV).to(torch.bfloat16)
    r = torch.randn(T, H, device=DEV).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(H, device=DEV)).to(torch.bfloat16)
    out = ops.rmsnorm(x, w, 1e-6)
    ref = ops.rmsnorm(x.cpu(), w.cpu(), 1e-6)
    torch.testing.assert_close(out.cpu().float(), ref.float(), atol=2e-2, rtol=1e-2)
    r_gpu, r_cpu = r.clone(), r.cpu().clone()
    out = ops.rmsnorm(x, w, 1e-6, residual=r_gpu)
    ref = ops.rmsnorm(x.cpu(), w.cpu(), 1e-6, residual=r_cpu)
    torch.testing.assert_close(r_gpu.cpu().float(), r_cpu.float(), atol=1e-2, rtol=1e-2)
    torch.testing.assert_close(out.cpu().float(), ref.float(), atol=2e-2, rtol=1e-2)


def test_moe_combine():
    T, k, H = 9, 8, 2048
    slots = torch.randn(T * k, H, device=DEV).to(torch.bfloat16)
    r = torch.randn(T, H, device=DEV).to(torch.bfloat16)
    w = torch.ones(H, device=DEV, dtype=torch.bfloat16)
    r_gpu, r_cpu = r.clone(), r.cpu().clone()
    out = ops.moe_combine_add_rmsnorm(slots, k, r_gpu, w, 1e-6)
    ref = ops.moe_combine_add_rmsnorm(slots.cpu(), k, r_cpu, w.cpu(), 1e-6)
    torch.testing.assert_close(r_gpu.cpu().float(), r_cpu.float(), atol=3e-2, rtol=1e-2)
    torch.testing.assert_close(out.cpu().float(), ref.float(), atol=3e-2, rtol=1e-2)


def _pool(num_blocks, bs, nkv, D, int8=False, device=DEV):
    return KVPool(num_blocks, 2, nkv, bs, D, torch.bfloat16, device, int8=int8)


@pytest.mark.parametrize("D,nq,nkv", [(128, 32, 4), (64, 4, 2)])
def test_qknorm_rope_kvstore(D, nq, nkv):
    T, bs = 20, 16
    qkv = torch.randn(T, (nq + 2 * nkv) * D, device=DEV).to(torch.bfloat16)
    pos = torch.randint(0, 4000, (T,), dtype=torch.int32, device=DEV)
    slots = torch.randperm(8 * bs, device=DEV)[:T].to(torch.int32)
    qw = (1 + 0.1 * torch.randn(D, device=DEV)).to(torch.bfloat16)
    kw = (1 + 0.1 * torch.randn(D, device=DEV)).to(torch.bfloat16)
    cs = ops.rope_cos_sin(D, 4096, 1e6, DEV)
    pg, pc = _pool(9, bs, nkv, D), _pool(9, bs, nkv, D, device="cpu")
    qg = ops.qknorm_rope_kvstore(qkv, pos, slots, qw, kw, cs, pg.layer(1), nq, nkv, D, 1e-6)
    qc = ops.qknorm_rope_kvstore(qkv.cpu(), pos.cpu(), slots.cpu(), qw.cpu(), kw.cpu(), cs.cpu(), pc.layer(1),
                                 nq, nkv, D, 1e-6)
    torch.testing.assert_close(qg.cpu().float(), qc.float(), atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(pg.data.cpu().float(), pc.data.float(), atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("T", [1, 32, 256])
def test_qkv_splitk_partials_into_qknorm_same_bits(T):
    """Decode-size QKV: the GEMM's split-K partials summed inside the q/k-norm
    kernel give the same q and KV bits as linear (split-K + reduce) then q/k-norm."""
    D, nq, nkv, bs = 128, 32, 4, 16
    n, k = (nq + 2 * nkv) * D, 2048
    assert ops.plan_dense(T, n // 128, k // 64)[1] > 1 or T >= 256
    q8, s8 = _fp8_weight(1, n, k, 21)
    x = (torch.randn(T, k, device=DEV) * 0.5).to(torch.bfloat16)
    pos = torch.randint(0, 4000, (T,), dtype=torch.int32, device=DEV)
    slots = torch.randperm(40 * bs, device=DEV)[:T].to(torch.int32)
    qw = (1 + 0.1 * torch.randn(D, device=DEV)).to(torch.bfloat16)
    kw = (1 + 0.1 * torch.randn(D, device=DEV)).to(torch.bfloat16)
    cs = ops.rope_cos_sin(D, 4096, 1e6, DEV)
    pa, pb = _pool(41, bs, nkv, D), _pool(41, bs, nkv, D)
    qkv = torch.empty(T, n, dtype=torch.bfloat16, device=DEV)
    qa = ops.qkv_norm_rope_kvstore(x, q8[0], s8[0], pos, slots, qw, kw, cs, pa.layer(0), nq, nkv, D, 1e-6, qkv,
                                   torch.empty(T, nq, D, dtype=torch.bfloat16, device=DEV))
    qb = ops.qknorm_rope_kvstore(ops.linear(x, q8[0], s8[0]), pos, slots, qw, kw, cs, pb.layer(0), nq, nkv, D, 1e-6)
    torch.cuda.synchronize()
    assert torch.equal(qa, qb) and torch.equal(pa.data, pb.data)


def test_router_topk():
    T, E, k = 77, 128, 8
    logits = torch.randn(T, 256, device=DEV)
    ids = torch.empty(T, k, dtype=torch.int32, device=DEV)
    w = torch.empty(T, k, device=DEV)
    counts = torch.zeros(E, dtype=torch.int32, device=DEV)
    ops.router_topk(logits, E, k, True, ids, w, counts)
    ids_c, w_c = torch.empty(T, k, dtype=torch.int32), torch.empty(T, k)
    counts_c = torch.zeros(E, dtype=torch.int32)
    ops.router_topk(logits.cpu(), E, k, True, ids_c, w_c, counts_c)
    # bf16-rounded logits tie exactly; a tie may resolve to either expert, so
    # compare the routing probabilities of the chosen sets, not the ids
    p = torch.softmax(logits.cpu()[:, :E].to(torch.bfloat16).float(), dim=-1)
    pg = p.gather(1, ids.cpu().long()).sort(dim=1).values
    pc = p.gather(1, ids_c.long()).sort(dim=1).values
    torch.testing.assert_close(pg, pc, atol=1e-6, rtol=0)
    assert (ids.cpu().sort(dim=1).values == ids_c.sort(dim=1).values).float().mean() > 0.95
    torch.testing.assert_close(w.cpu().sort(dim=1).values, w_c.sort(dim=1).values, atol=1e-2, rtol=1e-2)
    assert int(counts.sum()) == T * k and int(counts.max()) <= T


@pytest.mark.parametrize("T", [1, 77, 300, 2048])
def test_router_fused_matches_gemm_and_topk(T):
    """One-launch router (GEMM + softmax + top-k) against the fp32 reference of
    the same rounding points: bf16(x . w^T) logits, softmax, top-k, renorm.
    1 / 77 / 300 tokens split K across CTAs (the last CTA of a tile sums the
    partials in K order); 2048 tokens fill the SMs with token tiles alone."""
    E, k, H = 128, 8, 2048
    x = (torch.randn(T, H, device=DEV) * 0.5).to(torch.bfloat16)
    w = (torch.randn(E, H, device=DEV) * 0.05).to(torch.bfloat16)
    ids = torch.empty(T, k, dtype=torch.int32, device=DEV)
    wt = torch.empty(T, k, device=DEV)
    counts = torch.zeros(E, dtype=torch.int32, device=DEV)
    ops.router_fused(x, w, E, k, True, ids, wt, counts)
    torch.cuda.synchronize()
    logits = (x.float() @ w.float().t()).to(torch.bfloat16).float()
    p = torch.softmax(logits, dim=-1)
    pg = p.gather(1, ids.long()).sort(dim=1, descending=True).values
    pr = p.topk(k, dim=-1).values
    # fp32 summation order differs from the reference matmul: compare the chosen
    # probabilities (ties and 1-ulp logit differences may swap equal-valued experts)
    torch.testing.assert_close(pg, pr, atol=2e-3, rtol=2e-2)
    want_w = (pr / pr.sum(-1, keepdim=True)).to(torch.bfloat16).float()
    torch.testing.assert_close(wt.sort(dim=1, descending=True).values, want_w, atol=1e-2, rtol=2e-2)
    assert int(counts.sum()) == T * k
    ids2, wt2 = torch.empty_like(ids), torch.empty_like(wt)
    ops.router_fused(x, w, E, k, True, ids2, wt2, None)
    assert torch.equal(ids, ids2) and torch.equal(wt, wt2), "the split-K sum must be deterministic"


def test_moe_permute():
    T, k, E, H = 50, 8, 128, 2048
    x = torch.randn(T, H, device=DEV).to(torch.bfloat16)
    ids = torch.stack([torch.randperm(E, device=DEV)[:k] for _ in range(T)]).to(torch.int32)
    counts = torch.bincount(ids.flatten().long(), minlength=E).to(torch.int32)
    cursor = torch.zeros(E, dtype=torch.int32, device=DEV)
    xp = torch.empty(T * k, H, dtype=torch.bfloat16, device=DEV)
    sor = torch.empty(T * k, dtype=torch.int32, device=DEV)
    offs = torch.empty(E + 1, dtype=torch.int32, device=DEV)
    ops.moe_permute(x, ids, counts, cursor, xp, sor, offs)
    torch.cuda.synchronize()
    assert torch.equal(xp, x[(sor // k).long()])
    ref_off = torch.zeros(E + 1, dtype=torch.int32)
    ref_off[1:] = torch.cumsum(counts.cpu(), 0)
    assert torch.equal(offs.cpu(), ref_off)
    e_of_row = ids.flatten()[sor.long()].cpu()
    for e in range(E):
        a, b = ref_off[e], ref_off[e + 1]
        assert bool((e_of_row[a:b] == e).all())


def _fill_pool(pool, seq_lens, bs, nkv, D, int8=False):
    """Random K/V for sequences on shuffled blocks; returns block tables."""
    nb = [math.ceil(L / bs) for L in seq_lens]
    perm = torch.randperm(pool.num_blocks - 1).tolist()
    tables = torch.zeros(len(seq_lens), max(nb), dtype=torch.int32)
    i = 0
    for b, n in enumerate(nb):
        tables[b, :n] = torch.tensor(perm[i:i + n])
        i += n
    for b, L in enumerate(seq_lens):
        pos = torch.arange(L)
        slots = (tables[b][pos // bs].long() * bs + pos % bs).to(torch.int32).to(pool.data.device)
        for l in range(pool.num_layers):
            k = torch.randn(L, nkv, D, device=pool.data.device).to(torch.bfloat16)
            v = torch.randn(L, nkv, D, device=pool.data.device).to(torch.bfloat16)
            pool.layer(l).store(slots, k, v)
    return tables.to(pool.data.device)


@pytest.mark.parametrize("int8", [False, True])
@pytest.mark.parametrize("D,nq,nkv,bs", [(128, 32, 4, 256), (128, 32, 4, 16), (64, 4, 2, 16)])
def test_decode_attention(D, nq, nkv, bs, int8):
    seq_lens = [1, 17, 255, 256, 257, 700, 1300]
    B = len(seq_lens)
    nblocks = sum(math.ceil(L / bs) for L in seq_lens) + 2
    pool = _pool(nblocks, bs, nkv, D, int8=int8)
    tables = _fill_pool(pool, seq_lens, bs, nkv, D, int8)
    q = torch.randn(B, nq, D, device=DEV).to(torch.bfloat16)
    lens = torch.tensor(seq_lens, dtype=torch.int32, device=DEV)
    for split_len, nsplit in [(2048, 1), (256, 6), (64, 21)]:
        ws = (torch.empty(B * nq * nsplit, D, device=DEV), torch.empty(B * nq * nsplit, device=DEV),
              torch.empty(B * nq * nsplit, device=DEV))
        out = torch.empty(B, nq, D, dtype=torch.bfloat16, device=DEV)
        ops.decode_attention(q, pool.layer(1), tables, lens, D ** -0.5, out, split_len, nsplit, ws)
        ref = torch.empty(B, nq, D, device=DEV)
        ops._attention_ref(q, pool.layer(1), tables, lens, torch.arange(B + 1, dtype=torch.int32),
                           D ** -0.5, ref)
        torch.testing.assert_close(out.float(), ref, atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("int8", [False, True])
@pytest.mark.parametrize("D,nq,nkv,bs", [(128, 32, 4, 256), (64, 4, 2, 16)])
def test_prefill_attention(D, nq, nkv, bs, int8):
    # (query length, total length): fresh prompts, chunk continuations, prefix hits
    shapes = [(5, 5), (64, 64), (100, 100), (37, 300), (256, 512), (1, 90)]
    seq_lens = [L for _, L in shapes]
    nblocks = sum(math.ceil(L / bs) for L in seq_lens) + 2
    pool = _pool(nblocks, bs, nkv, D, int8=int8)
    tables = _fill_pool(pool, seq_lens, bs, nkv, D, int8)
    cu = [0]
    for qn, _ in shapes:
        cu.append(cu[-1] + qn)
    T = cu[-1]
    q = torch.randn(T, nq, D, device=DEV).to(torch.bfloat16)
    cu_t = torch.tensor(cu, dtype=torch.int32, device=DEV)
    lens = torch.tensor(seq_lens, dtype=torch.int32, device=DEV)
    out = torch.empty(T, nq, D, dtype=torch.bfloat16, device=DEV)
    ops.prefill_attention(q, pool.layer(0), cu_t, lens, tables, max(s for s, _ in shapes), D ** -0.5, out)
    ref = torch.empty(T, nq, D, device=DEV)
    ops._attention_ref(q, pool.layer(0), tables, lens, cu_t, D ** -0.5, ref)
    torch.testing.assert_close(out.float(), ref, atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("bs", [16, 64, 128, 256])
@pytest.mark.parametrize("nq,nkv", [(32, 4), (16, 4), (64, 4), (8, 8)])
def test_prefill_attention_tensor_core(bs, nq, nkv, monkeypatch):
    """tcgen05 prefill kernel (head_dim 128, bf16 KV) against the fp32 reference
    and against the mma.sync kernel: long prompts, prefix hits, ragged tails."""
    D = 128
    shapes = [(700, 700), (300, 1000), (129, 129), (1, 257), (17, 17), (128, 383)]
    seq_lens = [L for _, L in shapes]
    nblocks = sum(math.ceil(L / bs) for L in seq_lens) + 2
    pool = _pool(nblocks, bs, nkv, D)
    tables = _fill_pool(pool, seq_lens, bs, nkv, D)
    cu = [0]
    for qn, _ in shapes:
        cu.append(cu[-1] + qn)
    T = cu[-1]
    q = torch.randn(T, nq, D, device=DEV).to(torch.bfloat16)
    cu_t = torch.tensor(cu, dtype=torch.int32, device=DEV)
    lens = torch.tensor(seq_lens, dtype=torch.int32, device=DEV)
    mq = max(s for s, _ in shapes)
    out_tc = torch.full((T, nq, D), float("nan"), dtype=torch.bfloat16, device=DEV)
    ops.prefill_attention(q, pool.layer(1), cu_t, lens, tables, mq, D ** -0.5, out_tc)
    ops.check_status(DEV)
    monkeypatch.setenv("B200MOE_PREFILL_TC", "0")
    out_mma = torch.empty_like(out_tc)
    ops.prefill_attention(q, pool.layer(1), cu_t, lens, tables, mq, D ** -0.5, out_mma)
    ref = torch.empty(T, nq, D, device=DEV)
    ops._attention_ref(q, pool.layer(1), tables, lens, cu_t, D ** -0.5, ref)
    torch.testing.assert_close(out_tc.float(), ref, atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(out_tc.float(), out_mma.float(), atol=2e-2, rtol=2e-2)


def test_argmax_and_sampler():
    B, V = 6, 151936
    logits = torch.randn(B, V, device=DEV)
    logits[2, 12345] = 50.0
    out = ops.argmax(logits)
    assert torch.equal(out.cpu().long(), logits.argmax(dim=-1).cpu())
    temp = torch.tensor([0.0, 0.7, 1.0, 0.7, 1.0, 0.5], device=DEV)
    top_k = torch.tensor([-1, 5, -1, -1, 1, 50], dtype=torch.int32, device=DEV)
    top_p = torch.tensor([1.0, 1.0, 0.9, 0.5, 1.0, 0.95], device=DEV)
    seeds = torch.arange(B, dtype=torch.int64, device=DEV) + 11
    s = ops.sample(logits, temp, top_k, top_p, None, seeds, None)
    s2 = ops.sample(logits, temp, top_k, top_p, None, seeds, None)
    assert torch.equal(s, s2), "same seed must give the same draw"
    assert int(s[0]) == int(logits[0].argmax())
    assert int(s[4]) == int(logits[4].argmax())  # top_k 1
    assert int(s[2]) == 12345  # dominant logit survives top-p
    top5 = set(torch.topk(logits[1], 5).indices.tolist())
    assert int(s[1]) in top5


def _wide_logits(B, V=151936, seed=0, step=0.25):
    """Wide rows whose values sit on a grid of ``step`` (many exact ties at any threshold)."""
    g = torch.Generator(device=DEV).manual_seed(seed)
    x = torch.randn(B, V, generator=g, device=DEV) * 3.0
    return (x / step).round() * step


def test_penalties_kernel_matches_reference():
    B, V, n = 4, 151936, 3000
    g = torch.Generator().manual_seed(1)
    logits = torch.randn(B, V, generator=g) * 4
    rows = torch.randint(0, B, (n,), generator=g, dtype=torch.int32)
    ids = torch.randint(0, V, (n,), generator=g, dtype=torch.int32)
    key = rows.long() * V + ids.long()  # one entry per (row, id), as the plan packer emits
    keep = torch.ones(n, dtype=torch.bool)
    seen = set()
    for j, k in enumerate(key.tolist()):
        keep[j] = k not in seen
        seen.add(k)
    rows, ids = rows[keep], ids[keep]
    counts = torch.randint(0, 4, (rows.numel(),), generator=g, dtype=torch.int32)
    pres = torch.tensor([0.0, 0.5, -0.3, 1.2])
    freq = torch.tensor([0.0, 0.1, 0.4, -0.2])
    rep = torch.tensor([1.0, 1.3, 0.8, 1.7])
    want = ops.apply_penalties(logits.clone(), rows, ids, counts, pres, freq, rep)
    got = logits.to(DEV)
    ops.apply_penalties(got, rows.to(DEV), ids.to(DEV), counts.to(DEV), pres.to(DEV), freq.to(DEV), rep.to(DEV))
    torch.testing.assert_close(got.cpu(), want, atol=1e-5, rtol=1e-6)
    untouched = torch.ones(B, V, dtype=torch.bool)
    untouched[rows.long(), ids.long()] = False
    assert torch.equal(got.cpu()[untouched], logits[untouched])


@pytest.mark.parametrize("mode", ["top_p", "min_p", "top_k_top_p"])
def test_sampler_filters_on_wide_rows_with_ties(mode):
    """151,936-wide rows on a value grid (ties at every threshold): every draw of
    512 seeds lies in the kept set of the sorted-vocabulary definition (ties kept),
    and the draws follow the renormalised distribution on its most likely tokens."""
    N, V, T = 512, 151936, 0.7
    base = _wide_logits(1, V, seed=3)
    logits = base.expand(N, V).contiguous()
    temp = torch.full((N,), T, device=DEV)
    tk = torch.full((N,), 200 if mode == "top_k_top_p" else -1, dtype=torch.int32, device=DEV)
    tp = torch.full((N,), 0.9 if mode != "min_p" else 1.0, device=DEV)
    mp = torch.full((N,), 0.05 if mode == "min_p" else 0.0, device=DEV)
    seeds = torch.arange(N, dtype=torch.int64, device=DEV) * 7919 + 1
    toks = ops.sample(logits, temp, tk, tp, mp, seeds, None).cpu().long()
    x = base[0].cpu() / T
    keep = ops.sample_keep_reference(x, int(tk[0]), float(tp[0]), float(mp[0]))
    assert keep[toks].all(), "a draw fell outside the kept set"
    p = torch.softmax(torch.where(keep, x, torch.tensor(float("-inf"))), dim=-1)
    top = p.topk(8)
    freq = torch.stack([(toks == int(t)).float().mean() for t in top.indices])
    assert (freq - top.values).abs().max().item() < 0.06, (freq, top.values)


def test_sampler_guided_masks_and_logprobs():
    """Allowed-token masks and the fused log-probs against the CPU sampler: greedy
    rows pick the best allowed token; sampled rows draw inside mask and filters;
    top / chosen log-probs equal a log-softmax over the row's distribution."""
    B, V, k = 6, 151936, 5
    logits = _wide_logits(B, V, seed=5, step=0.001)
    words = (V + 31) // 32
    g = torch.Generator().manual_seed(9)
    masks = torch.randint(-2**31, 2**31 - 1, (3, words), generator=g, dtype=torch.int64).to(torch.int32)
    masks[2] = 0
    masks[2, 100 // 32] = 1 << (100 % 32)          # only token 100 allowed
    allow_row = torch.tensor([0, -1, 1, 2, 0, -1], dtype=torch.int32)
    temp = torch.tensor([0.0, 0.0, 0.8, 0.0, 1.1, 0.9])
    tk = torch.tensor([-1, -1, 100, -1, -1, 50], dtype=torch.int32)
    tp = torch.tensor([1.0, 1.0, 0.95, 1.0, 0.8, 1.0])
    mp = torch.tensor([0.0, 0.0, 0.0, 0.0, 0.0, 0.01])
    seeds = torch.arange(B, dtype=torch.int64) + 11
    top_v = torch.empty(B, k, device=DEV)
    top_i = torch.empty(B, k, dtype=torch.int32, device=DEV)
    chosen = torch.empty(B, device=DEV)
    toks = ops.sample(logits, temp.to(DEV), tk.to(DEV), tp.to(DEV), mp.to(DEV), seeds.to(DEV), None,
                      allow=masks.to(DEV), allow_row=allow_row.to(DEV), logprobs=(k, top_v, top_i, chosen))
    toks, top_v, top_i, chosen = toks.cpu().long(), top_v.cpu(), top_i.cpu(), chosen.cpu()
    bits = torch.arange(V)
    for r in range(B):
        row = logits[r].cpu()
        if allow_row[r] >= 0:
            w = masks[int(allow_row[r])].to(torch.int64) & 0xFFFFFFFF
            ok = ((w[bits // 32] >> (bits % 32)) & 1).bool()
            row = torch.where(ok, row, torch.tensor(float("-inf")))
        if temp[r] < 1e-3:
            x, keep = row, torch.isfinite(row)
            assert toks[r] == int(row.argmax()), r
        else:
            x = row / float(temp[r])
            keep = ops.sample_keep_reference(x, int(tk[r]), float(tp[r]), float(mp[r]))
            assert keep[toks[r]], r
        lp = torch.log_softmax(torch.where(keep, x, torch.tensor(float("-inf"))), dim=-1)
        assert abs(float(chosen[r]) - float(lp[toks[r]])) < 1e-4, r
        n = min(k, int(keep.sum()))
        want = lp.topk(n)
        torch.testing.assert_close(top_v[r, :n], want.values, atol=1e-4, rtol=1e-5)
        torch.testing.assert_close(lp[top_i[r, :n].long()], top_v[r, :n], atol=1e-4, rtol=1e-5)  # ids match values
        assert (top_i[r, n:] == -1).all() and torch.isinf(top_v[r, n:]).all(), r
    assert toks[3] == 100 and abs(float(chosen[3])) < 1e-6  # a single allowed token has log-prob 0


def test_sampler_distribution():
    """Exponential race draws follow softmax(logits / T) over the kept set."""
    V, N = 8, 4000
    base = torch.tensor([2.0, 1.0, 0.5, 0.0, -1.0, -2.0, -3.0, -4.0], device=DEV)
    logits = base.repeat(N, 1).contiguous()
    temp = torch.full((N,), 1.0, device=DEV)
    seeds = torch.arange(N, dtype=torch.int64, device=DEV)
    s = ops.sample(logits, temp, None, None, None, seeds, None)
    freq = torch.bincount(s.long(), minlength=V).float() / N
    p = torch.softmax(base, dim=0)
    assert (freq - p).abs().max().item() < 0.03
    tk = torch.full((N,), 3, dtype=torch.int32, device=DEV)
    s = ops.sample(logits, temp, tk, None, None, seeds, None)
    assert int(s.max()) <= 2


def _ep_wait_args(world, epoch, done, status, wait_ns=None):
    """EpArgs for one GPU whose every per-rank pointer is local memory: the
    wait kernel reads done[rank][r] for r < world and nothing else."""
    i32 = dict(dtype=torch.int32, device=DEV)
    local = [done.data_ptr()] * world
    if wait_ns is None:
        wait_ns = torch.zeros(2 * world, dtype=torch.int64, device=DEV)
    return ([world, 0, 8, 1, 1, 1, 1], torch.zeros(1, **i32), torch.zeros(1, **i32), torch.zeros(1, **i32),
            torch.zeros(world, **i32), torch.zeros(1, **i32), torch.zeros(1, **i32), epoch, status, wait_ns,
            local, local, local, local, [done.data_ptr() + 4 * world * r for r in range(world)])


def test_bounded_flag_wait_returns_status_instead_of_hanging():
    """A flag that nothing sets: the wait gives up after its limit (2 s of
    %globaltimer), records the timeout code and returns, leaving the context
    usable; a flag that is set passes at once with status 0."""
    import time
    C = ops.native()
    i32 = dict(dtype=torch.int32, device=DEV)
    status = torch.zeros(1, **i32)
    done = torch.zeros(16, **i32)
    epoch = torch.ones(1, **i32)
    # world 1: ep_signal releases this rank's own entry, the wait sees it
    C.ep_signal(*_ep_wait_args(1, epoch, done, status))
    C.ep_wait_done(*_ep_wait_args(1, epoch, done, status))
    torch.cuda.synchronize()
    assert int(status.item()) == 0 and int(done[0].item()) == 1
    # world 2: rank 1's entry is never released
    t0 = time.monotonic()
    wait_ns = torch.zeros(4, dtype=torch.int64, device=DEV)
    C.ep_wait_done(*_ep_wait_args(2, epoch, done, status, wait_ns))
    torch.cuda.synchronize()
    waited = time.monotonic() - t0
    assert int(status.item()) == 6, "kStatusTimeoutFlag"
    assert 1.5 < waited < 20.0, waited
    # the device-side wait accounting charges the time to the peer that never answered
    ns = wait_ns.cpu().tolist()
    assert ns[0] == 0 and ns[1] == 0 and ns[2] < 1e8 and 1.5e9 < ns[3] < 2.5e9, ns
    x = torch.randn(4, 1000, device=DEV)  # the context still runs kernels
    assert torch.equal(ops.argmax(x).cpu().long(), x.argmax(dim=-1).cpu())


def _channel_pool(num_blocks, bs, nkv, D, device=DEV, seed=3):
    """An int8 channel-mode pool with frozen scales and 0-2 outlier dims per head, as
    after calibration (identical on every device for the same seed)."""
    pool = KVPool(num_blocks, 2, nkv, bs, D, torch.bfloat16, device, int8=True, int8_mode="channel")
    g = torch.Generator().manual_seed(seed)
    pool.ch_scale.copy_(torch.rand(pool.ch_scale.shape, generator=g) * 0.03 + 0.01)
    pool.ch_dscale.copy_(pool.ch_scale)
    for l in range(2):
        for h in range(nkv):
            n = h % 3
            dims = torch.randperm(D, generator=g)[:n]
            pool.out_idx[l, h, :n] = dims.to(torch.int32)
            pool.n_out[l, h] = n
            pool.ch_dscale[l, :, h, dims] = 0.0
    return pool


@pytest.mark.parametrize("mode", ["token", "channel"])
@pytest.mark.parametrize("bs", [16, 256])
def test_int8_prefill_staged_tensor_core(mode, bs, monkeypatch):
    """int8 prefill through the bf16 staging pool and the tcgen05 kernel.  The stage
    holds exactly the pool's dequantised values (torch dequantisation of the same
    blocks, rounded to bf16 once) with zeros past each sequence, and the attention
    matches the warp-MMA int8 kernel and the fp32 reference."""
    D, nq, nkv = 128, 32, 4
    shapes = [(300, 300), (64, 1000), (1, 257), (17, 17), (129, 400)]
    seq_lens = [L for _, L in shapes]
    nblocks = sum(math.ceil(L / bs) for L in seq_lens) + 2
    pool = _channel_pool(nblocks, bs, nkv, D) if mode == "channel" else _pool(nblocks, bs, nkv, D, int8=True)
    tables = _fill_pool(pool, seq_lens, bs, nkv, D, True)
    layer = pool.layer(1)
    lens = torch.tensor(seq_lens, dtype=torch.int32, device=DEV)
    B, mb = tables.shape
    stage = torch.full((B * mb * 2 * nkv * bs * D,), float("nan"), dtype=torch.bfloat16, device=DEV)
    ops.native().kv_int8_stage(layer.k, layer.v, layer.k_scale, layer.v_scale, tables, lens, stage, bs,
                               layer.block_stride, nkv, ops._chan_read(layer))
    torch.cuda.synchronize()
    st = stage.view(B, mb, 2, nkv, bs, D)
    for b, L in enumerate(seq_lens):
        nb = math.ceil(L / bs)
        k, v = layer.gather(tables[b], L)
        for kv, want in ((0, k), (1, v)):
            got = st[b, :nb, kv].permute(0, 2, 1, 3).reshape(nb * bs, nkv, D)
            assert torch.equal(got[:L], want.to(torch.bfloat16)), (b, kv)
            assert bool((got[L:] == 0).all()), "slots past the sequence are zero"
    cu = [0]
    for qn, _ in shapes:
        cu.append(cu[-1] + qn)
    q = torch.randn(cu[-1], nq, D, device=DEV).to(torch.bfloat16)
    cu_t = torch.tensor(cu, dtype=torch.int32, device=DEV)
    mq = max(s for s, _ in shapes)
    out_tc = torch.full((cu[-1], nq, D), float("nan"), dtype=torch.bfloat16, device=DEV)
    ops.prefill_attention(q, layer, cu_t, lens, tables, mq, D ** -0.5, out_tc)
    monkeypatch.setenv("B200MOE_INT8_STAGE", "0")
    out_mma = torch.empty_like(out_tc)
    ops.prefill_attention(q, layer, cu_t, lens, tables, mq, D ** -0.5, out_mma)
    ref = torch.empty(q.shape, device=DEV)
    ops._attention_ref(q, layer, tables, lens, cu_t.cpu(), D ** -0.5, ref)
    torch.cuda.synchronize()
    ops.check_status(DEV)
    torch.testing.assert_close(out_tc.float(), ref, atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(out_tc.float(), out_mma.float(), atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("D,nq,nkv", [(128, 32, 4), (64, 4, 2)])
def test_int8_channel_store_matches_torch_reference(D, nq, nkv):
    """The reference's int8 channel store on the GPU against the torch store of the same
    values: V (not normalised, so the same bf16 inputs reach both) bit for bit -- int8
    payload, outlier dims zeroed, exact side values, calibration max; K (after the
    kernels' own q/k-norm + RoPE rounding) within one quantum."""
    T, bs = 40, 16
    qkv = (torch.randn(T, (nq + 2 * nkv) * D, device=DEV) * 2).to(torch.bfloat16)
    pos = torch.randint(0, 4000, (T,), dtype=torch.int32, device=DEV)
    slots = torch.randperm(8 * bs, device=DEV)[:T].to(torch.int32)
    qw = (1 + 0.1 * torch.randn(D, device=DEV)).to(torch.bfloat16)
    kw = (1 + 0.1 * torch.randn(D, device=DEV)).to(torch.bfloat16)
    cs = ops.rope_cos_sin(D, 4096, 1e6, DEV)
    pg, pc = _channel_pool(9, bs, nkv, D, DEV), _channel_pool(9, bs, nkv, D, "cpu")
    pg.calibrate_begin()
    pc.calibrate_begin()
    ops.qknorm_rope_kvstore(qkv, pos, slots, qw, kw, cs, pg.layer(1), nq, nkv, D, 1e-6)
    ops.qknorm_rope_kvstore(qkv.cpu(), pos.cpu(), slots.cpu(), qw.cpu(), kw.cpu(), cs.cpu(), pc.layer(1),
                            nq, nkv, D, 1e-6)
    torch.cuda.synchronize()
    g, c = pg.data.cpu(), pc.data
    assert torch.equal(g[:, 1, 1], c[:, 1, 1]), "V int8 payload"
    assert torch.equal(pg.side.cpu()[:, 1, 1], pc.side[:, 1, 1]), "V side values"
    assert torch.equal(pg.calib_amax.cpu()[1, 1], pc.calib_amax[1, 1]), "V calibration max"
    torch.testing.assert_close(pg.calib_sum.cpu()[1, 1], pc.calib_sum[1, 1], rtol=1e-5, atol=1e-4)
    assert (g[:, 1, 0].int() - c[:, 1, 0].int()).abs().max() <= 1, "K within one quantum"
    torch.testing.assert_close(pg.side.cpu()[:, 1, 0].float(), pc.side[:, 1, 0].float(), atol=3e-2, rtol=3e-2)


@pytest.mark.parametrize("D,nq,nkv,bs", [(128, 32, 4, 256), (64, 4, 2, 16)])
def test_int8_channel_attention_decode_and_prefill(D, nq, nkv, bs):
    """Decode (split-KV) and prefill attention over an int8 channel-mode pool against
    the fp32 reference over the same pool's dequantised K/V (per-channel read scales,
    exact outlier dims from the side pool)."""
    seq_lens = [1, 17, 255, 256, 257, 700]
    B = len(seq_lens)
    pool = _channel_pool(sum(math.ceil(L / bs) for L in seq_lens) + 2, bs, nkv, D)
    tables = _fill_pool(pool, seq_lens, bs, nkv, D, True)
    lens = torch.tensor(seq_lens, dtype=torch.int32, device=DEV)
    q = torch.randn(B, nq, D, device=DEV).to(torch.bfloat16)
    for split_len, nsplit in [(2048, 1), (64, 12)]:
        ws = (torch.empty(B * nq * nsplit, D, device=DEV), torch.empty(B * nq * nsplit, device=DEV),
              torch.empty(B * nq * nsplit, device=DEV))
        out = torch.empty(B, nq, D, dtype=torch.bfloat16, device=DEV)
        ops.decode_attention(q, pool.layer(1), tables, lens, D ** -0.5, out, split_len, nsplit, ws)
        ref = torch.empty(B, nq, D, device=DEV)
        ops._attention_ref(q, pool.layer(1), tables, lens, torch.arange(B + 1, dtype=torch.int32), D ** -0.5, ref)
        torch.testing.assert_close(out.float(), ref, atol=2e-2, rtol=2e-2)
    qn = [min(L, 64) for L in seq_lens]
    cu = torch.tensor([0] + list(np.cumsum(qn)), dtype=torch.int32, device=DEV)
    qp = torch.randn(int(sum(qn)), nq, D, device=DEV).to(torch.bfloat16)
    out = torch.empty_like(qp)
    ops.prefill_attention(qp, pool.layer(1), cu, lens, tables, max(qn), D ** -0.5, out)
    ref = torch.empty(qp.shape, device=DEV)
    ops._attention_ref(qp, pool.layer(1), tables, lens, cu.cpu(), D ** -0.5, ref)
    torch.cuda.synchronize()
    ops.check_status(DEV)
    torch.testing.assert_close(out.float(), ref, atol=2e-2, rtol=2e-2)
