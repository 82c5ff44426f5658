"""Prefill/decode disaggregation on CPU: protocol framing, KV block channels,
and the prefill -> decode TCP handoff producing the same greedy tokens as one
collocated engine."""
import os
import socket
import subprocess
import sys

import pytest
import torch

from b200moe import LLM, SamplingParams
from b200moe.engine.executor import free_port
from b200moe.engine.kv_cache import KVPool
from b200moe.pd.kv_channel import KVBlockBuffer, KVFrameAssembler, LocalKVChannel, TcpKVChannel
from b200moe.pd.protocol import JsonStream, send_json
from b200moe.pd.serve import run_client

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_json_stream_framing():
    a, b = socket.socketpair()
    send_json(a, {"x": 1})
    send_json(a, {"y": [1, 2]})
    data = b.recv(1 << 16)
    js = JsonStream()
    msgs = js.feed(data[:3]) + js.feed(data[3:])  # split inside the header
    assert msgs == [{"x": 1}, {"y": [1, 2]}]
    a.close()
    b.close()


@pytest.mark.parametrize("int8", [False, True])
def test_kv_block_channels_roundtrip(int8):
    src = KVPool(9, 2, 2, 4, 8, torch.bfloat16, "cpu", int8=int8)
    dst = KVPool(9, 2, 2, 4, 8, torch.bfloat16, "cpu", int8=int8)
    if int8:
        src.data.copy_(torch.randint(-127, 127, src.data.shape, dtype=torch.int8))
        src.scales.copy_(torch.rand(src.scales.shape))
    else:
        src.data.copy_(torch.randn(src.data.shape).to(torch.bfloat16))
    ch = LocalKVChannel(dst)
    buf = LocalKVChannel(src).send([3, 1, 7])
    ch.recv([0, 5, 2], buf)
    for s, d in ((3, 0), (1, 5), (7, 2)):
        assert torch.equal(src.data[s], dst.data[d])
        if int8:
            assert torch.equal(src.scales[s], dst.scales[d])
    # TCP frames through a socket pair and the incremental assembler
    a, b = socket.socketpair()
    tx, rx = TcpKVChannel(a, src, max_blocks=1), TcpKVChannel(b, dst, max_blocks=1)
    tx.send_blocks([4, 6])
    asm, frames, got = KVFrameAssembler(), [], 0
    need = 2 * src.data[0].numel() * src.data.element_size() + (2 * src.scales[0].numel() * 4 if int8 else 0)
    while not frames:
        chunk = b.recv(97)  # small chunks split headers and payloads
        got += len(chunk)
        frames += asm.feed(chunk)
    assert frames[0][0] == 2 and len(frames[0][1]) + len(frames[0][2]) == need
    rx.import_frame([8, 3], frames[0])
    assert torch.equal(src.data[4], dst.data[8]) and torch.equal(src.data[6], dst.data[3])
    a.close()
    b.close()


def _role(args, log):
    env = dict(os.environ, PYTHONPATH=ROOT)
    return subprocess.Popen([sys.executable, "-m", "b200moe.pd.serve", *args], env=env, stdout=log,
                            stderr=subprocess.STDOUT, cwd=ROOT)


def test_pd_tcp_handoff_matches_collocated(tmp_path):
    common = ["--model", "tiny-moe", "--device", "cpu", "--random-init", "--enforce-eager", "--kvcache-block-size",
              "16", "--num-kvcache-blocks", "64", "--max-model-len", "256", "--max-num-batched-tokens", "512"]
    prompts = [[(7 * i + j) % 1000 + 1 for j in range(20 + 9 * i)] for i in range(3)]
    llm = LLM("tiny-moe", device="cpu", enforce_eager=True, kvcache_block_size=16, num_kvcache_blocks=64,
              max_model_len=256, max_num_batched_tokens=512, random_init="seeded")
    want = [o["token_ids"] for o in llm.generate(prompts, SamplingParams(temperature=0.0, max_tokens=7,
                                                                          ignore_eos=True), use_tqdm=False)]
    llm.exit()
    d_port, p_port = free_port(), free_port()
    while d_port + 1 == p_port:
        p_port = free_port()
    logs = [open(tmp_path / n, "w") for n in ("decode.log", "prefill.log")]
    dec = _role(["--role", "decode", "--port", str(d_port), *common], logs[0])
    pre = _role(["--role", "prefill", "--port", str(p_port), "--d-port", str(d_port), *common], logs[1])
    try:
        res = run_client("127.0.0.1", p_port, [{"req_id": i, "prompt": p, "max_tokens": 7}
                                               for i, p in enumerate(prompts)], timeout_s=120)
        assert sorted(res) == [0, 1, 2]
        assert [res[i]["tokens"] for i in range(3)] == want
        assert all(res[i]["prefill_s"] is not None for i in range(3))
        assert pre.wait(60) == 0 and dec.wait(60) == 0
    finally:
        for p in (pre, dec):
            if p.poll() is None:
                p.kill()
        for f in logs:
            f.close()
    assert "clean exit" in (tmp_path / "decode.log").read_text()
