"""Teacher-forced scoring and accuracy gates on CPU (fp32).

* ``LLM.score`` equals the log-softmax of an independent dense forward, with
  prompts longer than one prefill chunk.
* The gate passes a legitimately different run (another chunk size) and
  fails planted bugs: RoPE positions off by one in continuation chunks, a KV
  slot off by one, and
  (MoE model) every expert output scaled by 1.01 -- the mutation checks of
  the reference's model tests.
"""
import pytest
import torch

from vllm_sm70_b200 import ops
from vllm_sm70_b200.engine import LLM
from vllm_sm70_b200.eval import teacher_forced as tf
from vllm_sm70_b200.models.config import ModelConfig
from vllm_sm70_b200.ops import moe as moe_ops

from ._llama_ref import llama_logits
from .test_engine_cpu import TINY

MOE = ModelConfig(arch="qwen3_moe", hidden_size=128, num_layers=2, num_heads=4, num_kv_heads=2,
                  head_dim=32, intermediate_size=256, vocab_size=512, rope_theta=10000.0,
                  rms_eps=1e-5, max_position=512, qk_norm=True, num_experts=8, top_k=2,
                  moe_intermediate_size=64)


def _llm(cfg, chunk):
    return LLM(cfg, max_num_seqs=4, max_model_len=160, block_size=16, dtype=torch.float32,
               enforce_eager=True, max_num_batched_tokens=chunk)


def _prompts():
    g = torch.Generator().manual_seed(17)
    return [torch.randint(0, 512, (n,), generator=g) for n in (70, 33, 101)]


def test_score_matches_dense_reference():
    llm = _llm(TINY, 32)
    got = llm.score(_prompts(), logits_rows=16)
    for p, lp in zip(_prompts(), got):
        ref = torch.log_softmax(llama_logits(llm.model, p), -1)
        want = ref[:-1].gather(1, p[1:, None]).squeeze(1)
        assert lp.shape == (p.numel() - 1,)
        assert torch.allclose(lp, want, atol=1e-4), float((lp - want).abs().max())


def _mutate_rope(mp):
    """RoPE positions off by one in continuation chunks (a uniform shift of
    every position would cancel: RoPE scores depend on relative offsets)."""
    real = ops.rope_kv_write

    def rope_pos_plus_one(qkv, positions, *a, **k):
        shift = 1 if int(positions[0]) > 0 else 0
        return real(qkv, positions + shift, *a, **k)
    mp.setattr(ops, "rope_kv_write", rope_pos_plus_one)


def _mutate_kv_slot(mp):
    real = ops.rope_kv_write

    def kv_slot_plus_one(qkv, positions, cos_sin, kc, vc, slots, *a, **k):
        return real(qkv, positions, cos_sin, kc, vc, slots + 1, *a, **k)
    mp.setattr(ops, "rope_kv_write", kv_slot_plus_one)


def _mutate_moe(mp):
    real = moe_ops.experts_forward

    def scaled(*a, **k):
        out = real(*a, **k)
        out.mul_(1.01)
        return out
    mp.setattr(moe_ops, "experts_forward", scaled)


@pytest.mark.parametrize("cfg,mutations", [
    (TINY, [_mutate_rope, _mutate_kv_slot]),
    (MOE, [_mutate_rope, _mutate_kv_slot, _mutate_moe]),
])
def test_gate_passes_legit_runs_and_catches_mutations(cfg, mutations, monkeypatch):
    ref = _llm(cfg, 160).score(_prompts())
    env = tf.delta(ref, _llm(cfg, 16).score(_prompts()))
    ok = tf.gate(ref, _llm(cfg, 48).score(_prompts()), env, floor=1e-4)
    assert ok.passed, ok
    for mutate in mutations:
        with monkeypatch.context() as mp:
            mutate(mp)
            bad = _llm(cfg, 48).score(_prompts())
        res = tf.gate(ref, bad, env, floor=1e-4)
        assert not res.passed, (mutate.__name__, res)


def test_generate_logprobs_match_dense_reference():
    """``SamplingParams(logprobs=N, prompt_logprobs=M)``: each output token
    carries its log-prob and the top-N of the model's distribution, each
    prompt token (after the first) its log-prob and the top-M -- equal to the
    log-softmax of an independent dense forward; greedy tokens are their
    position's top-1; requests without them are unchanged."""
    from vllm_sm70_b200.engine import SamplingParams

    llm = _llm(TINY, 32)
    p = _prompts()[0][:40]
    sp = SamplingParams(max_tokens=5, logprobs=3, prompt_logprobs=2)
    o = llm.generate([p], sp)[0]
    plain = llm.generate([p], SamplingParams(max_tokens=5))[0]
    assert o.output_token_ids == plain.output_token_ids and plain.logprobs is None
    seq = torch.cat([p, torch.tensor(o.output_token_ids)])
    ref = torch.log_softmax(llama_logits(llm.model, seq), -1)       # [L, V]
    Lp = p.numel()
    assert len(o.logprobs) == 5 and len(o.prompt_logprobs) == Lp and o.prompt_logprobs[0] is None
    for k, tok in enumerate(o.output_token_ids):
        d, row = o.logprobs[k], ref[Lp - 1 + k]
        assert abs(d[tok] - float(row[tok])) < 1e-4
        top = row.topk(3).indices.tolist()
        assert top[0] == tok and set(top) <= set(d)
        assert all(abs(d[t] - float(row[t])) < 1e-4 for t in top)
    for i in range(1, Lp):
        d, row = o.prompt_logprobs[i], ref[i - 1]
        assert abs(d[int(p[i])] - float(row[int(p[i])])) < 1e-4
        assert set(row.topk(2).indices.tolist()) <= set(d)
    echo = llm.generate([p], SamplingParams(max_tokens=0, prompt_logprobs=0))[0]
    assert echo.output_token_ids == [] and len(echo.prompt_logprobs) == Lp
    assert all(len(d) == 1 for d in echo.prompt_logprobs[1:])
