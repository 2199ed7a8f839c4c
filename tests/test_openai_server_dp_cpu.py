"""Data-parallel serving on CPU (two gloo ranks, all-to-all expert
parallelism, Qwen3-MoE): rank 0 serves HTTP and assigns requests to both
ranks; rank 1 runs ``dp_follower_loop``; every reply (plain and streamed,
from either rank) equals a single-process engine's greedy tokens, and
closing the app ends both ranks' loops."""
import json

import torch

from . import _mp
from .test_ep_cpu import KW, _greedy, _model, _prompts
from .test_loader_cpu import _write


def _body(rank, world, path, out_file):
    import threading
    from pathlib import Path

    from vllm_sm70_b200.engine import LLM
    from vllm_sm70_b200.entrypoints.openai_server import build_app, dp_follower_loop
    from vllm_sm70_b200.parallel import state

    ps = state.init(tp_size=1, ep_size=world, backend="gloo", timeout_s=120)
    llm = LLM(path, load_format="safetensors", tensor_parallel_size=1,
              data_parallel_size=world, enable_expert_parallel=True, **KW)
    if rank != 0:
        dp_follower_loop(llm, ps.cpu_group)
    else:
        from fastapi.testclient import TestClient

        app = build_app(llm, None, "moe", max_batch=4)
        res = {}
        with TestClient(app) as c:
            def go(i):
                p = _prompts()[i].tolist()
                body = {"prompt": p, "max_tokens": 3 + i % 4, "temperature": 0.0,
                        "ignore_eos": True}
                if i == 4:  # streamed
                    toks = []
                    with c.stream("POST", "/v1/completions", json={**body, "stream": True}) as r:
                        for line in r.iter_lines():
                            if line.startswith("data: {"):
                                toks += json.loads(line[6:])["choices"][0]["token_ids"]
                    res[i] = toks
                else:
                    res[i] = c.post("/v1/completions", json=body).json()["choices"][0]["token_ids"]
            th = [threading.Thread(target=go, args=(i,)) for i in range(len(_prompts()))]
            [t.start() for t in th]
            [t.join() for t in th]
            owners = sorted(set(app.state.batcher.owner.values()))  # all finished: empty
            loads = list(app.state.batcher.load)
            assigned = list(app.state.batcher.assigned)
        Path(out_file).write_text(json.dumps({"res": res, "owners": owners, "loads": loads,
                                              "assigned": assigned}))
    llm.shutdown()
    state.shutdown()


def test_dp_ep_server(tmp_path):
    from vllm_sm70_b200.engine import LLM

    cfg, hf = _model("qwen3_moe")
    single = LLM(cfg, **KW)
    path = _write(tmp_path, hf, single.model.hf_state_dict())
    want = _greedy(single, range(len(_prompts())))
    out = tmp_path / "res.json"
    _mp.run(_body, 2, args=(path, str(out)), timeout=300)
    got = json.loads(out.read_text())
    assert [got["res"][str(i)] for i in range(len(want))] == want
    assert got["owners"] == [] and got["loads"] == [0, 0]
    assert sum(got["assigned"]) == len(want) and min(got["assigned"]) >= 1  # both ranks served
