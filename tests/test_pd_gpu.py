"""PD disaggregation on one B200: prefill and decode roles in two processes,
KV handed over by the NVLink transport (CUDA IPC mapping of the decode pool +
the block copy kernel); tokens must match one collocated engine."""
import os
import subprocess
import sys

import pytest

from b200moe import LLM, SamplingParams
from b200moe.engine.executor import free_port
from b200moe.pd.serve import run_client

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("transport", ["nvlink", "tcp"])
def test_pd_handoff_matches_collocated(tmp_path, transport):
    common = ["--model", "tiny-moe-fp8", "--random-init", "--enforce-eager", "--kvcache-block-size", "16",
              "--num-kvcache-blocks", "128", "--max-model-len", "256", "--max-num-batched-tokens", "512"]
    prompts = [[(11 * i + j) % 1000 + 1 for j in range(24 + 13 * i)] for i in range(4)]
    llm = LLM("tiny-moe-fp8", enforce_eager=True, kvcache_block_size=16, num_kvcache_blocks=128, max_model_len=256,
              max_num_batched_tokens=512, random_init="seeded")
    want = [o["token_ids"] for o in llm.generate(prompts, SamplingParams(temperature=0.0, max_tokens=9,
                                                                          ignore_eos=True), use_tqdm=False)]
    llm.exit()
    d_port, p_port = free_port(), free_port()
    while abs(d_port - p_port) <= 1:
        p_port = free_port()
    env = dict(os.environ, PYTHONPATH=ROOT)
    logs = [open(tmp_path / n, "w") for n in ("decode.log", "prefill.log")]
    dec = subprocess.Popen([sys.executable, "-m", "b200moe.pd.serve", "--role", "decode", "--port", str(d_port),
                            "--kv-transport", transport, *common], env=env, stdout=logs[0], stderr=subprocess.STDOUT)
    pre = subprocess.Popen([sys.executable, "-m", "b200moe.pd.serve", "--role", "prefill", "--port", str(p_port),
                            "--d-port", str(d_port), "--kv-transport", transport, *common], env=env, stdout=logs[1],
                           stderr=subprocess.STDOUT)
    try:
        res = run_client("127.0.0.1", p_port, [{"req_id": i, "prompt": p, "max_tokens": 9}
                                               for i, p in enumerate(prompts)], timeout_s=180)
        if sorted(res) != [0, 1, 2, 3]:
            for f in logs:
                f.flush()
            tails = {n: (tmp_path / n).read_text()[-3000:] for n in ("decode.log", "prefill.log")}
            pytest.fail(f"missing results {sorted(res)}; role logs: {tails}")
        assert [res[i]["tokens"] for i in range(4)] == want
        assert pre.wait(120) == 0 and dec.wait(120) == 0
    finally:
        for p in (pre, dec):
            if p.poll() is None:
                p.kill()
        for f in logs:
            f.close()
