"""The OpenAI server under TP on CPU (two gloo ranks): rank 0 serves HTTP and
broadcasts every batch -- with its streaming interval -- to rank 1, which
runs the same ``generate`` calls in ``follower_loop``; replies (plain and
streamed) equal a single-process engine's, and closing the app releases the
follower."""
import json

import torch

from . import _mp
from .test_engine_tp_gpu import HF, _checkpoint

KW = dict(max_num_seqs=4, max_model_len=128, block_size=16, max_num_batched_tokens=64,
          num_kv_blocks=64, dtype=torch.float32, enforce_eager=True)
PROMPT = list(range(3, 40))


def _body(rank, world, path, out_file):
    from pathlib import Path

    from vllm_sm70_b200.engine import LLM
    from vllm_sm70_b200.entrypoints.openai_server import build_app, follower_loop
    from vllm_sm70_b200.parallel import state

    ps = state.init(tp_size=world, backend="gloo", timeout_s=120)
    llm = LLM(path, tensor_parallel_size=world, load_format="safetensors", **KW)
    if rank != 0:
        follower_loop(llm, ps.cpu_group)
    else:
        from fastapi.testclient import TestClient

        app = build_app(llm, None, "tiny", max_batch=4, group=ps.cpu_group)
        with TestClient(app) as c:
            body = {"prompt": PROMPT, "max_tokens": 11, "temperature": 0.0, "ignore_eos": True}
            plain = c.post("/v1/completions", json=body).json()["choices"][0]["token_ids"]
            streamed = []
            with c.stream("POST", "/v1/completions", json={**body, "stream": True}) as r:
                for line in r.iter_lines():
                    if line.startswith("data: {"):
                        streamed += json.loads(line[6:])["choices"][0]["token_ids"]
        Path(out_file).write_text(json.dumps({"plain": plain, "streamed": streamed}))
    llm.shutdown()
    state.shutdown()


def test_tp2_server_with_follower(tmp_path):
    from vllm_sm70_b200.engine import LLM, SamplingParams

    _checkpoint(tmp_path)
    out = tmp_path / "res.json"
    _mp.run(_body, 2, args=(str(tmp_path), str(out)), timeout=300)
    res = json.loads(out.read_text())
    one = LLM(str(tmp_path), tensor_parallel_size=1, load_format="safetensors", **KW)
    want = one.generate([torch.tensor(PROMPT)], SamplingParams(max_tokens=11))[0].output_token_ids
    assert res["plain"] == want and res["streamed"] == want
    assert HF["num_key_value_heads"] % 2 == 0
