"""bench.py's online-load mode on CPU with a tiny model: every request is
served, and the JSON line carries TTFT / TPOT percentiles and is marked as
profiling (not the headline)."""
import types

import torch


def test_online_mode_tiny(monkeypatch, capsys):
    import bench
    from vllm_sm70_b200.models.config import ModelConfig

    tiny = ModelConfig(arch="llama", hidden_size=128, num_layers=2, num_heads=4, num_kv_heads=2,
                       head_dim=32, intermediate_size=256, vocab_size=512, max_position=512)
    monkeypatch.setattr(bench, "PRESET", tiny)
    monkeypatch.setattr(bench, "N_REQ", 6)
    monkeypatch.setattr(bench, "PROMPT", 12)
    monkeypatch.setattr(bench, "OUT", 5)
    monkeypatch.setattr(bench, "make_prompts", lambda seed=0: torch.randint(
        0, 512, (6, 12), generator=torch.Generator().manual_seed(seed)))
    args = types.SimpleNamespace(arrival_rate=50.0, warmup=1, block_size=16, chunk=64)
    res = bench.run_online(args)
    assert res["requests"] == 6 and res["profiling"] is True
    assert res["value"] > 0 and res["p50_ttft_ms"] is not None and res["p90_tpot_ms"] is not None
    assert '"metric": "online serving' in capsys.readouterr().out


def test_profiling_flags_mark_the_line(monkeypatch):
    """--requests / --prompt-len / --output-len change the workload and mark
    the JSON line as profiling; the default headline workload does not."""
    import bench

    for name in ("N_REQ", "PROMPT", "OUT", "MODEL", "PRESET", "TEMPERATURE", "SPEC_K",
                 "PROFILING"):  # main() rewrites these module globals: restore them after
        monkeypatch.setattr(bench, name, getattr(bench, name))
    seen = []
    monkeypatch.setattr(bench, "run_ours", lambda args: seen.append(
        (bench.N_REQ, bench.PROMPT, bench.OUT, bench.PROFILING)))
    bench.main(["--steps", "1"])
    bench.main(["--requests", "8", "--output-len", "4"])
    assert seen == [(256, 1024, 256, False), (8, 1024, 4, True)]
