"""GGUF -> HF safetensors conversion on CPU.

* The NVFP4 repack is lossless and agrees with gguf-py's own NVFP4 decoder:
  ModelOpt tensors -> GGUF blocks decode (gguf-py) to exactly the ModelOpt
  reference weight, and convert back bit for bit.
* A Llama GGUF written the way llama.cpp lays it out (RoPE-interleaved q / k
  rows, F32 norms, F16 embedding, NVFP4 projections with per-tensor
  ``.scale``, one Q8_0 projection) converts into a checkpoint whose loaded
  weights are exactly the encoded ones, with a synthesised config.
* Stacked NVFP4 expert tensors (qwen3moe) split into per-expert projections
  with their own global scales.
"""
import numpy as np
import pytest
import torch

gguf = pytest.importorskip("gguf")

from vllm_sm70_b200.engine import LLM, SamplingParams  # noqa: E402
from vllm_sm70_b200.models import convert_gguf as cg  # noqa: E402
from vllm_sm70_b200.ops import quant  # noqa: E402

KW = dict(max_num_seqs=2, max_model_len=64, block_size=16, dtype=torch.float32,
          enforce_eager=True, max_num_batched_tokens=32)


def test_nvfp4_repack_matches_gguf_decoder():
    g = torch.Generator().manual_seed(0)
    w = torch.randn(24, 192, generator=g)
    packed, bs, gsc = quant.quantize_nvfp4(w)
    blocks = cg.modelopt_to_nvfp4_gguf(packed, bs)
    assert blocks.shape == (24, 192 // 64 * 36)
    dec = gguf.quants.dequantize(blocks, gguf.GGMLQuantizationType.NVFP4)
    ref = quant.Nvfp4Linear(packed, bs, gsc).dequant_ref().float()
    assert torch.equal(torch.from_numpy(dec.astype(np.float32)).to(torch.bfloat16).float(), ref)
    p2, s2 = cg.nvfp4_gguf_to_modelopt(blocks, 192)
    assert torch.equal(p2, packed) and torch.equal(s2.view(torch.uint8), bs.view(torch.uint8))


def _permute(w, n_head):
    """llama.cpp's q / k row interleave (the converter must undo it)."""
    return (w.reshape(n_head, 2, w.shape[0] // n_head // 2, *w.shape[1:]).transpose(1, 2)
            .reshape(w.shape))


def _nv(wr, name, w):
    packed, bs, gsc = quant.quantize_nvfp4(w)
    wr.add_tensor(name, cg.modelopt_to_nvfp4_gguf(packed, bs),
                  raw_dtype=gguf.GGMLQuantizationType.NVFP4)
    wr.add_tensor(name[: -len(".weight")] + ".scale", np.array([gsc], dtype=np.float32))
    return quant.Nvfp4Linear(packed, bs, gsc).reference_weight()


def _header(wr, arch, L, h, nh, nkv, d, inter, extra=None):
    wr.add_block_count(L)
    wr.add_embedding_length(h)
    wr.add_head_count(nh)
    wr.add_head_count_kv(nkv)
    wr.add_key_length(d)
    wr.add_value_length(d)
    wr.add_feed_forward_length(inter)
    wr.add_rope_freq_base(10000.0)
    wr.add_layer_norm_rms_eps(1e-5)
    wr.add_context_length(512)
    for k, v in (extra or {}).items():
        getattr(wr, k)(v)


def _finish(wr):
    wr.write_header_to_file()
    wr.write_kv_data_to_file()
    wr.write_tensors_to_file()
    wr.close()


def test_llama_gguf_converts_and_loads(tmp_path):
    L, h, nh, nkv, d, inter, V = 2, 128, 4, 2, 32, 256, 512
    g = torch.Generator().manual_seed(1)
    r = lambda *s: torch.randn(*s, generator=g) * 0.05  # noqa: E731
    src = tmp_path / "m.gguf"
    wr = gguf.GGUFWriter(str(src), "llama")
    _header(wr, "llama", L, h, nh, nkv, d, inter)
    emb = r(V, h) * 20
    wr.add_tensor("token_embd.weight", emb.numpy().astype(np.float16))
    wr.add_tensor("output_norm.weight", np.ones(h, dtype=np.float32))
    lm = r(V, h) * 40
    wr.add_tensor("output.weight", lm.numpy().astype(np.float32))
    want = {}
    for i in range(L):
        p = f"blk.{i}."
        wr.add_tensor(p + "attn_norm.weight", np.ones(h, dtype=np.float32))
        wr.add_tensor(p + "ffn_norm.weight", np.ones(h, dtype=np.float32))
        q, k = r(nh * d, h), r(nkv * d, h)
        # the GGUF holds the interleaved rows; the HF checkpoint the original order
        wq = _nv(wr, p + "attn_q.weight", _permute(q, nh))
        wk = _nv(wr, p + "attn_k.weight", _permute(k, nkv))
        want[(i, "q")] = cg._unpermute(wq, nh)
        want[(i, "k")] = cg._unpermute(wk, nkv)
        want[(i, "v")] = _nv(wr, p + "attn_v.weight", r(nkv * d, h))
        want[(i, "o")] = _nv(wr, p + "attn_output.weight", r(h, nh * d))
        want[(i, "gate")] = _nv(wr, p + "ffn_gate.weight", r(inter, h))
        want[(i, "up")] = _nv(wr, p + "ffn_up.weight", r(inter, h))
        down = r(h, inter)
        q8 = gguf.quants.quantize(down.numpy(), gguf.GGMLQuantizationType.Q8_0)
        wr.add_tensor(p + "ffn_down.weight", q8, raw_dtype=gguf.GGMLQuantizationType.Q8_0)
        want[(i, "down")] = torch.from_numpy(gguf.quants.dequantize(
            q8, gguf.GGMLQuantizationType.Q8_0)).float().to(torch.bfloat16).float()
    _finish(wr)
    out = tmp_path / "hf"
    s = cg.convert(src, out)
    assert s["nvfp4"] == 6 * L and s["dense"] == 3 + 3 * L
    llm = LLM(str(out), load_format="safetensors", **KW)
    assert llm.cfg.quant == "nvfp4" and llm.cfg.num_kv_heads == nkv and llm.cfg.head_dim == d
    def close(a, b):  # fused parts with different global scales share the largest one
        return ((a - b).abs() / b.abs().clamp_min(1e-3)).max().item() < 0.07

    for i, Ly in enumerate(llm.model.layers):
        assert close(Ly["qkv"].reference_weight(),
                     torch.cat([want[(i, "q")], want[(i, "k")], want[(i, "v")]]))
        assert torch.equal(Ly["o"].reference_weight(), want[(i, "o")])          # exact
        assert close(Ly["gate_up"].lin.reference_weight(),
                     torch.cat([want[(i, "gate")], want[(i, "up")]]))
        assert torch.equal(Ly["down"].w.float(), want[(i, "down")])   # Q8_0 -> dense bf16
    # F16 in the GGUF, bf16 in the checkpoint (the model's dtype: fp32 here)
    assert torch.equal(llm.model.embed_full.float(), emb.half().to(torch.bfloat16).float())
    out_ids = llm.generate([torch.arange(5, 25)], SamplingParams(max_tokens=4))[0]
    assert len(out_ids.output_token_ids) == 4


def test_stacked_nvfp4_experts_split(tmp_path):
    L, h, nh, nkv, d, E, I = 1, 128, 4, 4, 32, 4, 128
    g = torch.Generator().manual_seed(2)
    r = lambda *s: torch.randn(*s, generator=g) * 0.05  # noqa: E731
    src = tmp_path / "moe.gguf"
    wr = gguf.GGUFWriter(str(src), "qwen3moe")
    _header(wr, "qwen3moe", L, h, nh, nkv, d, 256,
            {"add_expert_count": E, "add_expert_used_count": 2,
             "add_expert_feed_forward_length": I})
    wr.add_tensor("token_embd.weight", r(256, h).numpy())
    wr.add_tensor("output_norm.weight", np.ones(h, dtype=np.float32))
    wr.add_tensor("output.weight", r(256, h).numpy())
    p = "blk.0."
    for n in ("attn_norm", "ffn_norm"):
        wr.add_tensor(p + n + ".weight", np.ones(h, dtype=np.float32))
    for n in ("attn_q_norm", "attn_k_norm"):
        wr.add_tensor(p + n + ".weight", np.ones(d, dtype=np.float32))
    for n, rows in (("attn_q", nh * d), ("attn_k", nkv * d), ("attn_v", nkv * d)):
        wr.add_tensor(p + n + ".weight", r(rows, h).numpy())
    wr.add_tensor(p + "attn_output.weight", r(h, nh * d).numpy())
    wr.add_tensor(p + "ffn_gate_inp.weight", r(E, h).numpy())
    want = {}
    for kind, (n_out, n_in) in (("gate", (I, h)), ("up", (I, h)), ("down", (h, I))):
        blocks, scales = [], []
        for e in range(E):
            packed, bs, gsc = quant.quantize_nvfp4(r(n_out, n_in) * (e + 1))
            blocks.append(cg.modelopt_to_nvfp4_gguf(packed, bs))
            scales.append(gsc)
            want[(kind, e)] = quant.Nvfp4Linear(packed, bs, gsc).reference_weight()
        wr.add_tensor(p + f"ffn_{kind}_exps.weight", np.stack(blocks),
                      raw_dtype=gguf.GGMLQuantizationType.NVFP4)
        wr.add_tensor(p + f"ffn_{kind}_exps.scale", np.array(scales, dtype=np.float32))
    _finish(wr)
    out = tmp_path / "hf"
    s = cg.convert(src, out)
    assert s["experts"] == 3 * E
    from safetensors import safe_open

    with safe_open(str(out / "model.safetensors"), "pt") as f:
        for e in range(E):
            for kind in ("gate", "up", "down"):
                base = f"model.layers.0.mlp.experts.{e}.{kind}_proj"
                lin = quant.Nvfp4Linear(f.get_tensor(base + ".weight"),
                                        f.get_tensor(base + ".weight_scale"),
                                        float(f.get_tensor(base + ".weight_scale_2")))
                assert torch.equal(lin.reference_weight(), want[(kind, e)])
    llm = LLM(str(out), load_format="safetensors", **KW)
    assert llm.cfg.arch == "qwen3_moe" and llm.model.layers[0]["experts"].fmt == "nvfp4"
