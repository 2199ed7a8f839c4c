"""Tensor parallelism end to end on CPU (gloo ranks, fp32): the same
safetensors checkpoint at TP = 2 and TP = 4 gives the same greedy tokens as at
TP = 1. Exercises the host-side TP plumbing -- shard cutting, the replicated
embedding, the row-parallel linear + all-reduce + RMSNorm fallback path and
the vocab-parallel greedy merge -- without a GPU. The checkpoint has two KV
heads, so TP = 4 also covers KV-head replication (each rank keeps the one KV
head its query heads read)."""
import json

import pytest
import torch

from . import _mp
from .test_engine_tp_gpu import HF, _checkpoint, _prompts

KW = dict(max_num_seqs=8, max_model_len=256, block_size=16, max_num_batched_tokens=64,
          num_kv_blocks=128, dtype=torch.float32, enforce_eager=True)


def _generate(path, tp):
    from vllm_sm70_b200.engine import LLM, SamplingParams

    llm = LLM(str(path), tensor_parallel_size=tp, load_format="safetensors", **KW)
    outs = llm.generate(_prompts(), SamplingParams(max_tokens=6, ignore_eos=True))
    toks = [o.output_token_ids for o in outs]
    llm.shutdown()
    return toks


def _tp_body(rank, world, path, out_file):
    from pathlib import Path

    from vllm_sm70_b200.parallel import state

    state.init(tp_size=world, backend="gloo", timeout_s=120)
    toks = _generate(Path(path), world)
    if rank == 0:
        Path(out_file).write_text(json.dumps(toks))
    state.shutdown()


@pytest.mark.parametrize("tp", [2, 4])
def test_tp_equals_tp1_cpu(tmp_path, tp):
    _checkpoint(tmp_path)
    out_file = tmp_path / f"tp{tp}.json"
    _mp.run(_tp_body, tp, args=(str(tmp_path), str(out_file)), timeout=300)
    got = json.loads(out_file.read_text())
    tp1 = _generate(tmp_path, 1)
    assert tp1 == got


def _minp():
    from vllm_sm70_b200.engine import SamplingParams

    return SamplingParams(max_tokens=6, temperature=1.0, min_p=0.5, seed=9)


def _biased():
    """logit_bias and allowed_token_ids with ids in both vocab shards (vocab
    1024 at TP2: [0, 512) and [512, 1024))."""
    from vllm_sm70_b200.engine import SamplingParams

    return SamplingParams(max_tokens=6, logit_bias={7: 3.0, 700: 5.0, 1000: -2.0},
                          allowed_token_ids=[3, 7, 100, 511, 512, 700, 1000, 1023])


def _pen_body(rank, world, path, out_file):
    from pathlib import Path

    from vllm_sm70_b200.engine import LLM, SamplingParams
    from vllm_sm70_b200.parallel import state

    state.init(tp_size=world, backend="gloo", timeout_s=120)
    llm = LLM(str(path), tensor_parallel_size=world, load_format="safetensors", **KW)
    sp = SamplingParams(max_tokens=6, repetition_penalty=1.7, frequency_penalty=0.5)
    toks = [o.output_token_ids for o in llm.generate(_prompts(), sp)]
    toks += [o.output_token_ids for o in llm.generate(_prompts(), _minp())]
    toks += [o.output_token_ids for o in llm.generate(_prompts(), _biased())]
    if rank == 0:
        Path(out_file).write_text(json.dumps(toks))
    llm.shutdown()
    state.shutdown()


def test_tp2_penalties_equal_tp1_cpu(tmp_path):
    """Sampling penalties, min_p, logit_bias and allowed_token_ids on
    vocab-parallel logit shards (each rank rewrites its own slice; min_p's row
    maximum is reduced over the shards) give the TP1 tokens."""
    from vllm_sm70_b200.engine import LLM, SamplingParams

    _checkpoint(tmp_path)
    out_file = tmp_path / "pen.json"
    _mp.run(_pen_body, 2, args=(str(tmp_path), str(out_file)), timeout=300)
    one = LLM(str(tmp_path), tensor_parallel_size=1, load_format="safetensors", **KW)
    sp = SamplingParams(max_tokens=6, repetition_penalty=1.7, frequency_penalty=0.5)
    want = [o.output_token_ids for o in one.generate(_prompts(), sp)]
    want += [o.output_token_ids for o in one.generate(_prompts(), _minp())]
    biased = [o.output_token_ids for o in one.generate(_prompts(), _biased())]
    assert all(set(t) <= set(_biased().allowed_token_ids) for t in biased)
    want += biased
    assert json.loads(out_file.read_text()) == want
