"""GEMM plan LUT on CPU (the plan table is host state of the extension, so
it needs no GPU): export -> save -> clear -> load round trip including
library-routed shapes, the manifest check (strict mode refuses a LUT made
for another build / GPU; non-strict imports it with a warning), and the
model's GEMM shape list covering every projection at every batch size."""
import json

import pytest
import torch

from vllm_sm70_b200 import _ext

pytestmark = pytest.mark.skipif(not _ext.load(), reason="extension not built")


def _plans():
    from vllm_sm70_b200.ops import linear as lin

    return [[256, 6144, 4096, 0, 3, 0], [16384, 4096, 4096, 0, 1, 4],
            [256, 28672, 4096, 1, lin.LIBRARY_CFG, 0]]


def _key(p):
    return tuple(p[:4])


def test_lut_roundtrip(tmp_path):
    from vllm_sm70_b200.engine import warmup
    from vllm_sm70_b200.ops import linear as lin

    torch.ops._b200_C.gemm_clear_plans()
    lin.clear_library()
    warmup.install_plans(_plans())
    path = tmp_path / "lut.json"
    warmup.save_lut(path)
    saved = {_key(p): p for p in json.loads(path.read_text())["plans"]}
    assert {_key(p) for p in _plans()} <= set(saved)
    assert saved[(256, 28672, 4096, 1)][4] == lin.LIBRARY_CFG
    torch.ops._b200_C.gemm_clear_plans()
    lin.clear_library()
    assert warmup.load_lut(path, strict=True) == len(saved)
    again = {_key(p): p for p in warmup.export_plans()}
    for k, p in saved.items():
        assert again[k][4:] == p[4:]
    torch.ops._b200_C.gemm_clear_plans()
    lin.clear_library()


def test_lut_manifest_strict(tmp_path):
    from vllm_sm70_b200.engine import warmup
    from vllm_sm70_b200.ops import linear as lin

    path = tmp_path / "other.json"
    man = dict(warmup.manifest(), fingerprint="abi=0;so=deadbeef")
    path.write_text(json.dumps({"manifest": man, "plans": _plans()}))
    with pytest.raises(RuntimeError, match="was made for"):
        warmup.load_lut(path, strict=True)
    assert warmup.load_lut(path, strict=False) == 3  # non-strict: imported anyway
    torch.ops._b200_C.gemm_clear_plans()
    lin.clear_library()


def test_model_gemm_shapes_cover_projections():
    from vllm_sm70_b200.engine import warmup
    from vllm_sm70_b200.models import build_model
    from vllm_sm70_b200.models.config import ModelConfig

    cfg = ModelConfig(arch="llama", hidden_size=256, num_layers=2, num_heads=4, num_kv_heads=2,
                      head_dim=64, intermediate_size=512, vocab_size=1024)
    m = build_model(cfg, torch.device("cpu"), torch.bfloat16)  # bf16 weights are tuned
    m.init_dummy()
    shapes = set(warmup.model_gemm_shapes(m, [1, 64], lm_ms=[1]))
    for M in (1, 64):
        assert (M, (4 + 2 * 2) * 64, 256, warmup.EPI_NONE) in shapes  # qkv
        assert (M, 256, 256, warmup.EPI_NONE) in shapes                # o
        assert (M, 1024, 256, warmup.EPI_SILU) in shapes               # gate|up + SiLU*up
        assert (M, 256, 512, warmup.EPI_NONE) in shapes                # down
    lm = (1024, 256, warmup.EPI_NONE)
    assert (1,) + lm in shapes and (64,) + lm not in shapes           # LM head at lm_ms only
