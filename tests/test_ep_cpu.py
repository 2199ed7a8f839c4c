"""Data-parallel attention + expert-parallel MoE on CPU (gloo ranks, fp32).

* The all-to-all dispatch / combine gives the same MoE output as computing
  every expert locally, with uneven token counts per rank (one rank has none).
* ``LLM(data_parallel_size=W, enable_expert_parallel=True)``: each rank
  serves its own share of the prompts and the greedy tokens equal a single
  process serving all of them -- including a rank with no prompts (it only
  serves the other ranks' expert traffic until they finish) and ranks that
  finish at different steps.
"""
import json

import pytest
import torch

from . import _mp
from .test_loader_cpu import _hf_config, _write

E, K, H, I = 8, 2, 64, 32


def _experts_full():
    from vllm_sm70_b200.ops import moe

    g = torch.Generator().manual_seed(21)
    w13 = torch.randn(E, 2 * I, H, generator=g) * 0.1
    w2 = torch.randn(E, H, I, generator=g) * 0.1
    return w13, w2, moe


def _tokens(rank):
    g = torch.Generator().manual_seed(100 + rank)
    T = [5, 0, 9, 3][rank]
    x = torch.randn(T, H, generator=g)
    logits = torch.randn(T, E, generator=g)
    return x, logits


def _dispatch_body(rank, world, out_file):
    from pathlib import Path

    from vllm_sm70_b200.parallel import state
    from vllm_sm70_b200.parallel.ep import EPAllToAll

    ps = state.init(tp_size=1, ep_size=world, backend="gloo", timeout_s=60)
    w13, w2, moe = _experts_full()
    El = E // world
    mine = moe.ExpertWeights("bf16", El, H, I, w13[rank * El:(rank + 1) * El].reshape(-1, H),
                             w2[rank * El:(rank + 1) * El].reshape(-1, I))
    full = moe.ExpertWeights("bf16", E, H, I, w13.reshape(-1, H), w2.reshape(-1, I))
    x, logits = _tokens(rank)
    w, ids = moe.topk_ref(logits, K)
    ep = EPAllToAll(ps, E, K)
    xr, wr, idr, plan = ep.dispatch(x, w, ids)
    yr = moe.experts_forward_ref(xr, wr, idr, mine, rank * El)
    got = ep.combine(yr, plan)
    ref = moe.experts_forward_ref(x, w, ids, full, 0)
    err = float((got - ref).abs().max()) if got.numel() else 0.0
    # every (token, owning rank) pair crossed exactly once
    owners = sum(len(set((ids[t] // El).tolist())) for t in range(x.shape[0]))
    Path(f"{out_file}.{rank}").write_text(json.dumps({"err": err, "sent": ep.sent_rows,
                                                      "owners": owners}))
    state.shutdown()


@pytest.mark.parametrize("world", [2, 4])
def test_dispatch_combine_equals_local_experts(tmp_path, world):
    out = tmp_path / "r"
    _mp.run(_dispatch_body, world, args=(str(out),), timeout=120)
    for r in range(world):
        d = json.loads((tmp_path / f"r.{r}").read_text())
        assert d["err"] < 1e-5, d
        assert d["sent"] == d["owners"], d


KW = dict(max_num_seqs=4, max_model_len=128, block_size=16, dtype=torch.float32,
          enforce_eager=True, max_num_batched_tokens=32)


NEXT_HF = {"model_type": "qwen3_next", "hidden_size": 128, "num_hidden_layers": 4,
           "num_attention_heads": 4, "num_key_value_heads": 2, "head_dim": 32,
           "intermediate_size": 256, "vocab_size": 512, "rope_theta": 10000.0,
           "rms_norm_eps": 1e-6, "max_position_embeddings": 512, "tie_word_embeddings": False,
           "num_experts": 8, "num_experts_per_tok": 2, "moe_intermediate_size": 64,
           "shared_expert_intermediate_size": 64, "norm_topk_prob": True,
           "linear_num_key_heads": 2, "linear_num_value_heads": 4, "linear_key_head_dim": 32,
           "linear_value_head_dim": 32, "linear_conv_kernel_dim": 4,
           "full_attention_interval": 2, "partial_rotary_factor": 0.25}


def _model(arch):
    """(config, HF config.json dict) of a tiny MoE model."""
    from vllm_sm70_b200.models.config import ModelConfig

    if arch == "qwen3_next":  # hybrid: gated DeltaNet + gated attention, shared expert
        return ModelConfig.from_hf(NEXT_HF), NEXT_HF
    if arch == "flint":  # sliding / full attention with sinks, dense + sigmoid MoE layers
        from .test_flint_cpu import HF as FLINT_HF

        return ModelConfig.from_hf(FLINT_HF), FLINT_HF
    cfg = ModelConfig(arch="qwen3_moe", hidden_size=128, num_layers=2, num_heads=4,
                      num_kv_heads=2, head_dim=32, intermediate_size=256, vocab_size=512,
                      rope_theta=10000.0, rms_eps=1e-5, max_position=512, qk_norm=True,
                      num_experts=8, top_k=2, moe_intermediate_size=64)
    return cfg, _hf_config(cfg)


def _prompts():
    g = torch.Generator().manual_seed(8)
    return [torch.randint(0, 512, (n,), generator=g) for n in (9, 40, 4, 23, 17)]


def _greedy(llm, idx):
    """Greedy tokens of the prompts ``idx`` (global indices: the budget of
    prompt i is 3 + i % 4 tokens, so ranks finish at different steps)."""
    from vllm_sm70_b200.engine import SamplingParams

    p = _prompts()
    outs = llm.generate([p[i] for i in idx], [SamplingParams(max_tokens=3 + i % 4) for i in idx])
    return [o.output_token_ids for o in outs]


def _dp_body(rank, world, path, out_file):
    from pathlib import Path

    from vllm_sm70_b200.engine import LLM
    from vllm_sm70_b200.parallel import state

    state.init(tp_size=1, ep_size=world, backend="gloo", timeout_s=120)
    llm = LLM(path, load_format="safetensors", tensor_parallel_size=1,
              data_parallel_size=world, enable_expert_parallel=True, **KW)
    assert llm.model.ep_a2a is not None and llm.model.E_local == 8 // world
    mine = list(range(rank, len(_prompts()), world))
    toks = _greedy(llm, mine)
    # a second call on the same engine in which only rank 0 has a prompt: the
    # others only serve its expert traffic
    again = _greedy(llm, mine[:1] if rank == 0 else [])
    Path(f"{out_file}.{rank}").write_text(json.dumps({"ids": mine, "toks": toks,
                                                      "again": again}))
    llm.shutdown()
    state.shutdown()


@pytest.mark.parametrize("arch,world", [("qwen3_moe", 2), ("qwen3_moe", 4), ("qwen3_next", 2),
                                        ("flint", 2)])
def test_dp_ep_engine_equals_single_process(tmp_path, arch, world):
    from vllm_sm70_b200.engine import LLM

    cfg, hf = _model(arch)
    single = LLM(cfg, **KW)
    path = _write(tmp_path, hf, single.model.hf_state_dict())
    ref = _greedy(single, range(len(_prompts())))
    _mp.run(_dp_body, world, args=(path, str(tmp_path / "dp")), timeout=300)
    got = {}
    for r in range(world):
        rec = json.loads((tmp_path / f"dp.{r}").read_text())
        for i, t in zip(rec["ids"], rec["toks"]):
            got[i] = t
        if r == 0:
            assert rec["again"] == [ref[0]]
        else:
            assert rec["again"] == []
    assert [got[i] for i in range(len(ref))] == ref


def _tpxep_body(rank, world, tp, path, out_file):
    from pathlib import Path

    from vllm_sm70_b200.engine import LLM
    from vllm_sm70_b200.parallel import state

    state.init(tp_size=tp, ep_size=world, backend="gloo", timeout_s=120)
    dp = world // tp
    llm = LLM(path, load_format="safetensors", tensor_parallel_size=tp, data_parallel_size=dp,
              enable_expert_parallel=True, **KW)
    assert llm.model.ep_a2a is not None and llm.model.E_local == 8 // world
    d = rank // tp  # contiguous ranks form a replica; its ranks serve the same prompts
    mine = list(range(d, len(_prompts()), dp))
    toks = _greedy(llm, mine)
    Path(f"{out_file}.{rank}").write_text(json.dumps({"ids": mine, "toks": toks}))
    llm.shutdown()
    state.shutdown()


@pytest.mark.parametrize("arch", ["qwen3_moe", "qwen3_next"])
def test_tp_x_ep_engine_equals_single_process(tmp_path, arch):
    """TP x EP (two replicas of TP 2 on four ranks, experts over all four):
    inside a replica the tokens are replicated, each TP rank dispatches a
    disjoint slice through the expert exchange and the TP all-reduce after
    the block sums the slices with the shared-expert partials; the greedy
    tokens equal one process serving every prompt."""
    from vllm_sm70_b200.engine import LLM
    from vllm_sm70_b200.models.config import ModelConfig

    cfg, hf = _model(arch)
    if arch == "qwen3_next":
        # TP 2 shards the shared expert: keep each shard at one 64-row gate/up block
        hf = dict(hf, shared_expert_intermediate_size=128)
        cfg = ModelConfig.from_hf(hf)
    single = LLM(cfg, **KW)
    path = _write(tmp_path, hf, single.model.hf_state_dict())
    ref = _greedy(single, range(len(_prompts())))
    world, tp = 4, 2
    _mp.run(_tpxep_body, world, args=(tp, path, str(tmp_path / "tpep")), timeout=300)
    for r in range(world):
        rec = json.loads((tmp_path / f"tpep.{r}").read_text())
        for i, t in zip(rec["ids"], rec["toks"]):
            assert t == ref[i], (arch, r, i)
