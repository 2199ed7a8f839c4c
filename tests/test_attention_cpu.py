"""CPU correctness of paged decode attention vs a dense torch SDPA reference.

This is the reference's CPU configuration: batch 8, 32 query heads, 8 KV
heads, head_dim 128, KV block size 16, per-sequence context lengths uniform in
[1, 2048], q/k/v fp32 N(0, 1), KV scattered into a random block table, fixed
seed. Unused cache slots hold NaN so any out-of-context read poisons the
result. Reference parity: sm70/tests/attention/_fv100_ref.py:17-60.
"""
import math

import torch

from vllm_sm70_b200.ops import attention as A


def _config1(seed=1234):
    g = torch.Generator().manual_seed(seed)
    B, HQ, HKV, D, BS = 8, 32, 8, 128, 16
    lens = torch.randint(1, 2049, (B,), generator=g).tolist()
    ks = [torch.randn(L, HKV, D, generator=g) for L in lens]
    vs = [torch.randn(L, HKV, D, generator=g) for L in lens]
    q = torch.randn(B, HQ, D, generator=g)
    kc, vc, bt, sl = A.build_paged_kv(ks, vs, BS, generator=g)
    cu = torch.arange(B + 1, dtype=torch.int32)
    return q, ks, vs, kc, vc, bt, sl, cu, D


def test_config1_paged_decode_vs_sdpa():
    q, ks, vs, kc, vc, bt, sl, cu, D = _config1()
    scale = 1 / math.sqrt(D)
    out = torch.empty_like(q)
    A.paged_attention(out, q, kc, vc, bt, sl, cu, 1, scale, decode=True)
    for i in range(q.shape[0]):
        ref = A.sdpa_ref(q[i:i + 1], ks[i], vs[i], scale)
        torch.testing.assert_close(out[i:i + 1], ref, rtol=1e-4, atol=1e-4)
    assert torch.isfinite(out).all()


def test_paged_gather_roundtrip():
    q, ks, vs, kc, vc, bt, sl, cu, D = _config1(7)
    for i in range(len(ks)):
        torch.testing.assert_close(A.gather_paged(kc, bt[i], int(sl[i])), ks[i])
        torch.testing.assert_close(A.gather_paged(vc, bt[i], int(sl[i])), vs[i])


def test_window_and_sinks_oracle_consistency():
    g = torch.Generator().manual_seed(3)
    k = torch.randn(50, 2, 64, generator=g)
    v = torch.randn(50, 2, 64, generator=g)
    q = torch.randn(3, 8, 64, generator=g)
    full = A.attention_ref(q, k, v, 0.125)
    big_window = A.attention_ref(q, k, v, 0.125, window=1000)
    torch.testing.assert_close(full, big_window)
    # A sink of -inf is the same as no sink.
    no_sink = A.attention_ref(q, k, v, 0.125, sinks=torch.full((8,), float("-inf")))
    torch.testing.assert_close(full, no_sink)
    torch.testing.assert_close(full, A.sdpa_ref(q, k, v, 0.125), rtol=1e-5, atol=1e-5)


def test_rope_llama3_scaling_shapes():
    cs = A.rope_cos_sin(128, 64, 5e5, {"rope_type": "llama3", "factor": 8.0,
                                        "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                                        "original_max_position_embeddings": 8192})
    assert cs.shape == (64, 128)
    torch.testing.assert_close(cs[0, :64], torch.ones(64))
    torch.testing.assert_close(cs[0, 64:], torch.zeros(64))
