"""Tensor parallelism end to end: the same safetensors checkpoint served at
TP = 2 (spawned ranks over NCCL, the fused all-reduce + RMSNorm kernel, CUDA
graphs for decode) and at TP = 1 must give the same greedy tokens. The LM head
is scaled so greedy choices are far from ties and the bf16 summation-order
difference between the two layouts cannot flip one."""
import json
import os

import pytest
import torch

from . import _mp

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

HF = {"model_type": "llama", "hidden_size": 512, "num_hidden_layers": 2,
      "num_attention_heads": 8, "num_key_value_heads": 2, "head_dim": 64,
      "intermediate_size": 1024, "vocab_size": 1024, "rope_theta": 10000.0,
      "rms_norm_eps": 1e-5, "max_position_embeddings": 1024, "tie_word_embeddings": False}
KW = dict(max_num_seqs=8, max_model_len=256, block_size=16, max_num_batched_tokens=256,
          num_kv_blocks=128, tune_gemm=False)


def _checkpoint(path):
    from safetensors.torch import save_file

    g = torch.Generator().manual_seed(11)
    h, inter, v, L = HF["hidden_size"], HF["intermediate_size"], HF["vocab_size"], 2
    qd, kd = HF["num_attention_heads"] * HF["head_dim"], HF["num_key_value_heads"] * HF["head_dim"]

    def r(*s, std=0.02):
        return (torch.randn(*s, generator=g) * std).to(torch.bfloat16)

    sd = {"model.embed_tokens.weight": r(v, h, std=1.0), "model.norm.weight": torch.ones(h).bfloat16(),
          "lm_head.weight": r(v, h, std=2.0)}
    for i in range(L):
        p = f"model.layers.{i}."
        sd.update({p + "input_layernorm.weight": torch.ones(h).bfloat16(),
                   p + "post_attention_layernorm.weight": torch.ones(h).bfloat16(),
                   p + "self_attn.q_proj.weight": r(qd, h), p + "self_attn.k_proj.weight": r(kd, h),
                   p + "self_attn.v_proj.weight": r(kd, h), p + "self_attn.o_proj.weight": r(h, qd),
                   p + "mlp.gate_proj.weight": r(inter, h), p + "mlp.up_proj.weight": r(inter, h),
                   p + "mlp.down_proj.weight": r(h, inter)})
    (path / "config.json").write_text(json.dumps(HF))
    save_file(sd, str(path / "model.safetensors"))


def _prompts():
    g = torch.Generator().manual_seed(5)
    return [torch.randint(0, HF["vocab_size"], (n,), generator=g) for n in (5, 40, 130, 17, 64, 3)]


def _generate(path, tp):
    from vllm_sm70_b200.engine import LLM, SamplingParams

    llm = LLM(str(path), tensor_parallel_size=tp, load_format="safetensors", **KW)
    outs = llm.generate(_prompts(), SamplingParams(max_tokens=12, ignore_eos=True))
    toks = [o.output_token_ids for o in outs]
    llm.shutdown()
    return toks


def _tp_body(rank, world, path, out_file):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    from pathlib import Path

    from vllm_sm70_b200.parallel import state

    state.init(tp_size=world, timeout_s=120)
    toks = _generate(Path(path), world)
    if rank == 0:
        Path(out_file).write_text(json.dumps(toks))
    state.shutdown()


def test_tp2_equals_tp1(b200_ops, tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    _checkpoint(tmp_path)
    out_file = tmp_path / "tp2.json"
    _mp.run(_tp_body, 2, args=(str(tmp_path), str(out_file)), timeout=600)
    tp2 = json.loads(out_file.read_text())
    tp1 = _generate(tmp_path, 1)
    assert tp1 == tp2
