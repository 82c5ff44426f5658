"""Full-recompute fp32 oracle: a Qwen3-MoE forward with no KV cache, no paging,
no batching tricks — one sequence, every position, plain torch.

Used to check the engine end to end (the reference's CPU ground truth,
tests/archive/p2_ground_truth.py): the engine's greedy tokens must be the
argmax of this model's logits at every generated position.
"""
from __future__ import annotations

import torch

from b200moe import ops


@torch.no_grad()
def full_forward_logits(model, token_ids: list[int]) -> torch.Tensor:
    """fp32 logits [len(token_ids), vocab] of ``model``'s weights (any device)."""
    a = model.args
    dev = torch.device("cpu")
    ids = torch.tensor(token_ids, dtype=torch.long)
    L = len(token_ids)
    H, D = a.hidden_size, a.head_dim
    nq, nkv = a.num_attention_heads, a.num_key_value_heads
    eps = a.rms_norm_eps

    def W(w, s):
        w = w.detach().to(dev)
        return ops.dequant_block_fp8(w, s.detach().to(dev)) if s is not None else w.float()

    def norm(x, w):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w.detach().to(dev).float()

    cs = ops.rope_cos_sin(D, max(L, 1), a.rope_theta, dev)
    cos, sin = cs[:L, :D // 2].unsqueeze(1), cs[:L, D // 2:].unsqueeze(1)

    def rope(x):
        x1, x2 = x.chunk(2, dim=-1)
        return torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin), dim=-1)

    h = model.embed_tokens.detach().to(dev)[ids].float()
    mask = torch.ones(L, L, dtype=torch.bool).tril()
    for layer in model.layers:
        x = norm(h, layer.input_layernorm)
        qkv = x @ W(layer.qkv_weight, layer.qkv_scale).t()
        q = qkv[:, :nq * D].view(L, nq, D)
        k = qkv[:, nq * D:(nq + nkv) * D].view(L, nkv, D)
        v = qkv[:, (nq + nkv) * D:].view(L, nkv, D)
        q, k = rope(norm(q, layer.q_norm)), rope(norm(k, layer.k_norm))
        G = nq // nkv
        k = k.repeat_interleave(G, dim=1)
        v = v.repeat_interleave(G, dim=1)
        s = torch.einsum("qhd,khd->hqk", q, k) * D ** -0.5
        s = s.masked_fill(~mask, float("-inf"))
        o = torch.einsum("hqk,khd->qhd", torch.softmax(s, -1), v).reshape(L, nq * D)
        h = h + o @ W(layer.o_weight, layer.o_scale).t()
        x = norm(h, layer.post_attention_layernorm)
        I = layer.w2.shape[-1]
        if layer.is_moe:
            logits = x @ layer.router.detach().to(dev).float()[:a.num_experts].t()
            # routing rounds the gate logits and the top-k weights to bf16, as the
            # reference's bf16 gate does (qwen3_moe.py:389-395)
            p = torch.softmax(logits.to(torch.bfloat16).float(), dim=-1)
            w, e = torch.topk(p, a.num_experts_per_tok, dim=-1)
            if a.norm_topk_prob:
                w = w / w.sum(-1, keepdim=True)
            w = w.to(torch.bfloat16).float()
            out = torch.zeros_like(x)
            local = {g: i for i, g in enumerate(model.expert_ids)}
            for t in range(L):
                for j in range(a.num_experts_per_tok):
                    le = local[int(e[t, j])]
                    gu = x[t] @ W(layer.w13[le], None if layer.s13 is None else layer.s13[le]).t()
                    hh = torch.nn.functional.silu(gu[:I]) * gu[I:]
                    out[t] += w[t, j] * (hh @ W(layer.w2[le], None if layer.s2 is None else layer.s2[le]).t())
        else:
            gu = x @ W(layer.w13[0], None if layer.s13 is None else layer.s13[0]).t()
            out = (torch.nn.functional.silu(gu[:, :I]) * gu[:, I:]) @ W(
                layer.w2[0], None if layer.s2 is None else layer.s2[0]).t()
        h = h + out
    h = norm(h, model.norm)
    return h @ model.lm_head.detach().to(dev).float().t()
