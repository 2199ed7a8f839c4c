"""Convert a GGUF checkpoint into an HF-layout safetensors directory this
runtime loads (``LLM(path, load_format="safetensors")``).

    python -m vllm_sm70_b200.models.convert_gguf model.gguf OUT_DIR [--hf-config DIR]

* NVFP4 GGUF tensors are repacked LOSSLESSLY into ModelOpt NVFP4
  (``weight`` / ``weight_scale`` / ``weight_scale_2``). A GGUF NVFP4 block is
  36 bytes for 64 values: four unsigned-E4M3 scale bytes (one per 16 values)
  then 32 code bytes, where code byte i of 16-value group g holds value i in
  its low nibble and value i + 8 in its high nibble; ModelOpt stores the same
  E2M1 codes two consecutive values per byte (low nibble first) and the same
  E4M3 scales, so only the nibble order changes. The per-tensor factor is the
  companion ``<name>.scale`` F32 tensor when present (one per expert for
  stacked expert tensors), else 1.
* F32 tensors (norms, sinks) pass through; F16 / BF16 / other GGML types are
  dequantised (gguf-py) and written in bf16.
* Names map from llama.cpp's (``blk.N.attn_q.weight``, ``ffn_gate_exps``,
  ...) to HF's; stacked expert tensors are split per expert. For the
  ``llama`` architecture the q / k rows are un-permuted (llama.cpp
  interleaves the RoPE halves when it converts Llama checkpoints).
* ``config.json`` (and tokenizer files) come from ``--hf-config`` when given,
  else a config is synthesised from the GGUF metadata (llama / qwen2 / qwen3
  / qwen3moe keys); a ``quantization_config`` is added when NVFP4 tensors
  were written.

Tensors stream from the memory-mapped GGUF into safetensors shards, so peak
memory is about one shard.

Reference parity: the reference's GGUF -> ModelOpt NVFP4 converter for its
Flint checkpoint (``sm70/tools/flint/convert_gguf.py``,
``sm70/tools/flint/gguf_nvfp4.py``).
"""
from __future__ import annotations

import argparse
import json
import re
import shutil
from pathlib import Path

import numpy as np
import torch

NVFP4_BLOCK_BYTES = 36   # 4 scale bytes + 32 code bytes per 64 values
NVFP4_BLOCK = 64

_LAYER = {
    "attn_norm.weight": "input_layernorm.weight",
    "ffn_norm.weight": "post_attention_layernorm.weight",
    "post_attention_norm.weight": "post_attention_layernorm.weight",
    "attn_q_norm.weight": "self_attn.q_norm.weight",
    "attn_k_norm.weight": "self_attn.k_norm.weight",
    "attn_sinks.weight": "self_attn.softmax_offset",
    "attn_sinks": "self_attn.softmax_offset",
    "attn_q": "self_attn.q_proj",
    "attn_k": "self_attn.k_proj",
    "attn_v": "self_attn.v_proj",
    "attn_output": "self_attn.o_proj",
    "ffn_gate": "mlp.gate_proj",
    "ffn_up": "mlp.up_proj",
    "ffn_down": "mlp.down_proj",
    "ffn_gate_inp": "mlp.gate",
    "ffn_gate_shexp": "mlp.shared_expert.gate_proj",
    "ffn_up_shexp": "mlp.shared_expert.up_proj",
    "ffn_down_shexp": "mlp.shared_expert.down_proj",
    "ffn_gate_inp_shexp": "mlp.shared_expert_gate",
}
_EXPERTS = {"ffn_gate_exps": "gate_proj", "ffn_up_exps": "up_proj", "ffn_down_exps": "down_proj"}
_GLOBAL = {"token_embd.weight": "model.embed_tokens.weight", "output_norm.weight": "model.norm.weight",
           "output.weight": "lm_head.weight"}


# ----------------------------------------------------------------------------- NVFP4
def nvfp4_gguf_to_modelopt(raw: np.ndarray, K: int) -> tuple[torch.Tensor, torch.Tensor]:
    """GGUF NVFP4 bytes ``[rows, K/64*36]`` -> (ModelOpt codes uint8
    ``[rows, K/2]``, E4M3 block scales ``[rows, K/16]``)."""
    rows = raw.shape[0]
    nb = K // NVFP4_BLOCK
    b = torch.from_numpy(np.array(raw, dtype=np.uint8)).view(rows, nb, NVFP4_BLOCK_BYTES)
    scales = b[:, :, :4].reshape(rows, nb * 4).clone()
    scales[scales == 0x7F] = 0                       # the format's zero encoding
    codes = b[:, :, 4:].reshape(rows, nb, 4, 8)      # [.., group, byte i]
    lo, hi = codes & 0xF, codes >> 4                 # value i, value i + 8
    vals = torch.cat([lo, hi], dim=-1)               # [.., group, 16] in value order
    packed = (vals[..., 0::2] | (vals[..., 1::2] << 4)).reshape(rows, K // 2)
    return packed.contiguous(), scales.view(torch.float8_e4m3fn).contiguous()


def modelopt_to_nvfp4_gguf(packed: torch.Tensor, scales: torch.Tensor) -> np.ndarray:
    """Inverse of :func:`nvfp4_gguf_to_modelopt` (GGUF bytes ``[rows, K/64*36]``)."""
    rows, half = packed.shape
    K = half * 2
    nb = K // NVFP4_BLOCK
    p = packed.view(torch.uint8).reshape(rows, nb, 4, 8)
    vals = torch.stack([p & 0xF, p >> 4], dim=-1).reshape(rows, nb, 4, 16)
    codes = vals[..., :8] | (vals[..., 8:] << 4)                       # [.., 4, 8]
    sc = scales.view(torch.uint8).reshape(rows, nb, 4)
    out = torch.cat([sc, codes.reshape(rows, nb, 32)], dim=-1)
    return out.reshape(rows, nb * NVFP4_BLOCK_BYTES).numpy()


# ----------------------------------------------------------------------------- names
def hf_name(gguf_name: str) -> str | None:
    """HF tensor name of a non-expert GGUF tensor (None: not a model tensor)."""
    if gguf_name in _GLOBAL:
        return _GLOBAL[gguf_name]
    m = re.fullmatch(r"blk\.(\d+)\.(.+)", gguf_name)
    if not m:
        return None
    i, rest = m.group(1), m.group(2)
    if rest in _LAYER:
        return f"model.layers.{i}.{_LAYER[rest]}"
    base, _, suffix = rest.rpartition(".")
    if base in _LAYER and suffix in ("weight", "bias"):
        return f"model.layers.{i}.{_LAYER[base]}.{suffix}"
    return None


def _unpermute(w: torch.Tensor, n_head: int) -> torch.Tensor:
    """Undo llama.cpp's RoPE row interleave of a Llama q / k projection."""
    rows = w.shape[0]
    return (w.reshape(n_head, rows // n_head // 2, 2, *w.shape[1:]).transpose(1, 2)
            .reshape(w.shape))


# ----------------------------------------------------------------------------- metadata
def _field(reader, key):
    f = reader.fields.get(key)
    if f is None:
        return None
    v = f.parts[f.data[0]]
    if f.types and f.types[0].name == "STRING":
        return bytes(v).decode()
    return v.tolist()[0] if hasattr(v, "tolist") else v


def synth_config(reader, vocab: int) -> dict:
    arch = _field(reader, "general.architecture")
    g = lambda k, d=None: (_field(reader, f"{arch}.{k}") if _field(reader, f"{arch}.{k}")  # noqa: E731
                           is not None else d)
    h = int(g("embedding_length"))
    nh = int(g("attention.head_count"))
    cfg = {"architectures": [{"llama": "LlamaForCausalLM", "qwen2": "Qwen2ForCausalLM",
                              "qwen3": "Qwen3ForCausalLM",
                              "qwen3moe": "Qwen3MoeForCausalLM"}.get(arch, arch)],
           "model_type": {"qwen3moe": "qwen3_moe"}.get(arch, arch),
           "hidden_size": h, "num_hidden_layers": int(g("block_count")),
           "num_attention_heads": nh,
           "num_key_value_heads": int(g("attention.head_count_kv", nh)),
           "head_dim": int(g("attention.key_length", h // nh)),
           "intermediate_size": int(g("feed_forward_length", 4 * h)),
           "vocab_size": vocab, "rope_theta": float(g("rope.freq_base", 10000.0)),
           "rms_norm_eps": float(g("attention.layer_norm_rms_epsilon", 1e-6)),
           "max_position_embeddings": int(g("context_length", 8192)),
           "tie_word_embeddings": False}
    if g("expert_count"):
        cfg.update(num_experts=int(g("expert_count")),
                   num_experts_per_tok=int(g("expert_used_count")),
                   moe_intermediate_size=int(g("expert_feed_forward_length")),
                   norm_topk_prob=True)
    return cfg


# ----------------------------------------------------------------------------- convert
class _ShardWriter:
    def __init__(self, out: Path, max_bytes: int):
        self.out, self.max_bytes = out, max_bytes
        self.cur: dict = {}
        self.size = 0
        self.files: list[str] = []
        self.weight_map: dict = {}

    def add(self, name: str, t: torch.Tensor) -> None:
        t = t.contiguous()
        self.cur[name] = t
        self.size += t.numel() * t.element_size()
        if self.size >= self.max_bytes:
            self.flush()

    def flush(self) -> None:
        from safetensors.torch import save_file

        if not self.cur:
            return
        fn = f"model-{len(self.files) + 1:05d}.safetensors"
        save_file(self.cur, str(self.out / fn))
        self.files.append(fn)
        for k in self.cur:
            self.weight_map[k] = fn
        self.cur, self.size = {}, 0

    def finish(self) -> None:
        self.flush()
        if len(self.files) == 1:
            (self.out / self.files[0]).rename(self.out / "model.safetensors")
            return
        (self.out / "model.safetensors.index.json").write_text(
            json.dumps({"metadata": {}, "weight_map": self.weight_map}, indent=1))


def _dense(t) -> torch.Tensor:
    """Full-precision tensor of a non-NVFP4 GGUF tensor (torch, numpy order)."""
    import gguf

    qt = gguf.GGMLQuantizationType(int(t.tensor_type))
    if qt == gguf.GGMLQuantizationType.F32:
        return torch.from_numpy(np.array(t.data, dtype=np.float32))
    if qt == gguf.GGMLQuantizationType.F16:
        return torch.from_numpy(np.array(t.data, dtype=np.float16))
    if qt == gguf.GGMLQuantizationType.BF16:
        raw = np.ascontiguousarray(t.data).view(np.int16)
        return torch.from_numpy(raw.copy()).view(torch.bfloat16)
    return torch.from_numpy(gguf.quants.dequantize(np.asarray(t.data), qt).astype(np.float32))


def convert(src: str | Path, out: str | Path, hf_config: str | Path | None = None,
            max_shard_bytes: int = 4 << 30) -> dict:
    """Convert ``src`` (a .gguf file or a directory holding one) into ``out``.
    Returns a summary (tensor counts per output kind)."""
    import gguf

    src = Path(src)
    if src.is_dir():
        found = sorted(src.glob("*.gguf"))
        if not found:
            raise FileNotFoundError(f"no .gguf file in {src}")
        src = found[0]
    out = Path(out)
    out.mkdir(parents=True, exist_ok=True)
    reader = gguf.GGUFReader(str(src))
    arch = _field(reader, "general.architecture")
    tensors = {t.name: t for t in reader.tensors}
    n_head = _field(reader, f"{arch}.attention.head_count")
    n_head_kv = _field(reader, f"{arch}.attention.head_count_kv") or n_head
    NV = gguf.GGMLQuantizationType.NVFP4
    w = _ShardWriter(out, max_shard_bytes)
    summary = {"nvfp4": 0, "dense": 0, "experts": 0}
    nvfp4_excluded: list[str] = []

    def tensor_scale(name, n_exp=None):
        s = tensors.get(name[: -len(".weight")] + ".scale") if name.endswith(".weight") else None
        if s is None:
            return [1.0] * (n_exp or 1)
        return [float(x) for x in np.asarray(s.data, dtype=np.float32).reshape(-1)]

    def emit(hname: str, t, rows_perm: int | None, exp: int | None = None, dense=None):
        if int(t.tensor_type) == int(NV):
            K = int(t.shape[0])
            raw = np.asarray(t.data)
            raw = raw[exp] if exp is not None else raw
            packed, scales = nvfp4_gguf_to_modelopt(raw.reshape(-1, raw.shape[-1]), K)
            if rows_perm:
                packed, scales = _unpermute(packed, rows_perm), _unpermute(scales, rows_perm)
            g = tensor_scale(t.name, None if exp is None else int(t.shape[-1]))
            base = hname[: -len(".weight")]
            w.add(base + ".weight", packed)
            w.add(base + ".weight_scale", scales)
            w.add(base + ".weight_scale_2", torch.tensor(g[exp or 0], dtype=torch.float32))
            w.add(base + ".input_scale", torch.tensor(1.0, dtype=torch.float32))
            summary["nvfp4"] += 1
            return
        d = dense if dense is not None else _dense(t)
        d = d[exp] if exp is not None else d
        if rows_perm:
            d = _unpermute(d, rows_perm)
        keep_f32 = int(t.tensor_type) == int(gguf.GGMLQuantizationType.F32) and d.dim() == 1
        w.add(hname, d if keep_f32 else d.to(torch.bfloat16))
        summary["dense"] += 1
        if hname.endswith("_proj.weight") or hname.endswith("lm_head.weight"):
            nvfp4_excluded.append(hname[: -len(".weight")])

    for name, t in tensors.items():
        if name.endswith(".scale"):
            continue  # NVFP4 per-tensor factors, consumed with their tensor
        m = re.fullmatch(r"blk\.(\d+)\.(ffn_(?:gate|up|down)_exps)\.weight", name)
        if m:
            i, kind = m.group(1), _EXPERTS[m.group(2)]
            d_all = None if int(t.tensor_type) == int(NV) else _dense(t)  # dequantised once
            for e in range(int(t.shape[-1])):
                emit(f"model.layers.{i}.mlp.experts.{e}.{kind}.weight", t, None, exp=e,
                     dense=d_all)
                summary["experts"] += 1
            continue
        hname = hf_name(name)
        if hname is None:
            continue
        perm = None
        if arch == "llama" and hname.endswith(("q_proj.weight", "k_proj.weight")):
            perm = n_head if "q_proj" in hname else n_head_kv
        emit(hname, t, perm)
    w.finish()

    if hf_config is not None:
        hc = Path(hf_config)
        for f in hc.iterdir():
            if f.suffix in (".json", ".jinja", ".model", ".txt") and "safetensors" not in f.name:
                shutil.copy(f, out / f.name)
        cfg = json.loads((out / "config.json").read_text())
    else:
        vocab = int(tensors["token_embd.weight"].shape[-1])
        cfg = synth_config(reader, vocab)
    if summary["nvfp4"]:
        cfg["quantization_config"] = {"quant_method": "modelopt", "quant_algo": "NVFP4",
                                      "group_size": 16,
                                      "exclude_modules": sorted(set(nvfp4_excluded))}
    (out / "config.json").write_text(json.dumps(cfg, indent=1))
    return summary


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("src", help=".gguf file or a directory holding one")
    ap.add_argument("out", help="output directory (HF layout)")
    ap.add_argument("--hf-config", default=None,
                    help="directory with config.json / tokenizer files to copy")
    ap.add_argument("--max-shard-gb", type=float, default=4.0)
    a = ap.parse_args(argv)
    s = convert(a.src, a.out, a.hf_config, int(a.max_shard_gb * (1 << 30)))
    print(json.dumps(s))


if __name__ == "__main__":
    main()
