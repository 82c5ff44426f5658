"""The fused expert-parallel kernels on ONE GPU: with a world of one rank the rank
is its own owner, so dispatch (rows and per-expert counts into the owner's
buffers), the scatter that places rows from the count matrix, the down GEMM's
done release and the combine's wait all run on local memory -- with the rows sent by
the router's top-k warps and by the stand-alone dispatch kernel.  The result must
equal the single-GPU MoE path bit for bit: the GEMMs see the same rows per
expert, and the combine sums the same slots in the same order."""
import random
from types import SimpleNamespace

import numpy as np
import pytest
import torch
import torch.distributed as dist

from b200moe import ops
from b200moe.config import Config
from b200moe.engine.executor import free_port
from b200moe.engine.kv_cache import KVPool
from b200moe.models.qwen3_moe import Qwen3MoeForCausalLM, StepInputs
from b200moe.utils.weights import random_init_

pytestmark = pytest.mark.gpu


def _inputs(seq_lens, q_lens, bs, vocab, seed):
    rng = random.Random(seed)
    B = len(seq_lens)
    order = sorted(range(B), key=lambda i: (q_lens[i] != 1, i))
    nb = [-(-L // bs) for L in seq_lens]
    ids, pos, slots, tables, base = [], [], [], [], 1
    for i in order:
        L, q = seq_lens[i], q_lens[i]
        blocks = list(range(base, base + nb[i]))
        base += nb[i]
        tables.append(blocks + [0] * (max(nb) - nb[i]))
        p = list(range(L - q, L))
        pos += p
        slots += [blocks[x // bs] * bs + x % bs for x in p]
        ids += [rng.randrange(vocab) for _ in p]
    cu = np.cumsum([0] + [q_lens[i] for i in order]).astype(np.int32)
    nd = sum(1 for q in q_lens if q == 1)
    t = lambda a: torch.tensor(np.asarray(a), dtype=torch.int32, device="cuda")
    return StepInputs(t(ids), t(pos), t(slots), t(cu), t([seq_lens[i] for i in order]), t(tables), t(cu[1:] - 1),
                      nd, max([q_lens[i] for i in order if q_lens[i] != 1] or [0]), max(seq_lens), B,
                      t(cu[nd:] - cu[nd])), base


@pytest.mark.parametrize("bf16_experts", [False, True])
def test_fused_ep_world1_matches_local_moe(monkeypatch, bf16_experts):
    """``bf16_experts``: every step takes the bf16 expert GEMMs on the resident
    dequantised copy (local path and expert-parallel path alike)."""
    from b200moe.parallel.ep import ExpertParallel
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{free_port()}", rank=0, world_size=1,
                            device_id=torch.device("cuda", 0))
    try:
        cfg = Config("tiny-moe-fp8", max_num_batched_tokens=512, max_num_seqs=16, max_model_len=256,
                     kvcache_block_size=16, num_kvcache_blocks=64)
        args = cfg.hf_config
        model = Qwen3MoeForCausalLM(args, "cuda")
        random_init_(model, seed=4)
        model.tile_weights_()
        if bf16_experts:
            monkeypatch.setattr(Qwen3MoeForCausalLM, "BF16_EXPERT_ROWS", 1)
            assert model.cache_bf16_experts_() > 0
        model.reserve_workspace(512, 16, 8)
        runner = SimpleNamespace(world_size=1, rank=0, device=torch.device("cuda", 0), args=args, config=cfg,
                                 model=model)
        ep = ExpertParallel(runner, "fused")
        assert ep.backend == "fused" and ep.p2p is not None
        bs = 16
        steps = [([40, 17, 64, 3], [40, 17, 64, 3]), ([41, 18, 65, 4], [1, 1, 1, 1]), ([42, 19, 66, 5], [1, 1, 1, 1])]
        outs = {}
        # local MoE; EP with the router sending the rows; EP with a separate dispatch launch
        for use_ep, router_dispatch in ((False, False), (True, True), (True, False)):
            model.ep = ep if use_ep else None
            ep.p2p.ROUTER_DISPATCH = router_dispatch
            pool = KVPool(64, args.num_hidden_layers, args.num_key_value_heads, bs, args.head_dim,
                          torch.bfloat16, "cuda")
            got = []
            for i, (lens, q) in enumerate(steps):
                inp, _ = _inputs(lens, q, bs, args.vocab_size, seed=i)
                got.append(model.compute_logits(model(inp, pool)).float().cpu())
            torch.cuda.synchronize()
            ops.check_status(torch.device("cuda", 0))
            outs[(use_ep, router_dispatch)] = got
        for key in ((True, True), (True, False)):
            for a, b in zip(outs[(False, False)], outs[key]):
                assert torch.equal(a, b), key
        waits = ep.p2p.wait_stats()
        assert len(waits["dispatch_ms"]) == 1 and len(waits["combine_ms"]) == 1
        model.ep = None
        ep.p2p.close()
    finally:
        dist.destroy_process_group()
