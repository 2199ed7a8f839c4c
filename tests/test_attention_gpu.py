"""Paged attention kernels (prefill / decode / split-KV / sinks / window) vs
the fp32 dense oracle, plus the fused RoPE + KV-cache writer."""
import math

import pytest
import torch

from vllm_sm70_b200.ops import attention as A

pytestmark = pytest.mark.gpu


def _case(lens_q, lens_ctx, hq, hkv, d, bs, seed=0):
    g = torch.Generator().manual_seed(seed)
    ks = [torch.randn(L, hkv, d, generator=g).to(torch.bfloat16).cuda() for L in lens_ctx]
    vs = [torch.randn(L, hkv, d, generator=g).to(torch.bfloat16).cuda() for L in lens_ctx]
    kc, vc, bt, sl = A.build_paged_kv(ks, vs, bs, generator=g)
    T = sum(lens_q)
    q = torch.randn(T, hq, d, generator=g).to(torch.bfloat16).cuda()
    cu = torch.tensor([0] + list(torch.tensor(lens_q).cumsum(0)), dtype=torch.int32).cuda()
    return q, kc, vc, bt, sl, cu


@pytest.mark.parametrize("d,hq,hkv", [(128, 32, 8), (128, 8, 1), (256, 16, 2), (64, 8, 8)])
@pytest.mark.parametrize("bs", [16, 32, 128])
def test_decode(b200_ops, d, hq, hkv, bs, rel_err):
    lens = [1, 17, 300, 1029, 64]
    q, kc, vc, bt, sl, cu = _case([1] * len(lens), lens, hq, hkv, d, bs)
    out = torch.empty_like(q)
    scale = 1 / math.sqrt(d)
    A.paged_attention(out, q, kc, vc, bt, sl, cu, 1, scale, decode=True)
    ref = A.paged_attention_ref(q, kc, vc, bt, sl, cu, scale)
    assert rel_err(out, ref) < 2e-2


@pytest.mark.parametrize("splits", [2, 5])
@pytest.mark.parametrize("d,hq,hkv", [(128, 32, 8), (256, 16, 2)])
def test_decode_split_kv(b200_ops, splits, d, hq, hkv, rel_err):
    lens = [3, 700, 2100]
    q, kc, vc, bt, sl, cu = _case([1] * 3, lens, hq, hkv, d, 16, seed=1)
    out = torch.empty_like(q)
    T, H, D = q.shape
    po = torch.empty(splits, T, H, D, device="cuda")
    pml = torch.empty(splits, T, H, 2, device="cuda")
    A.paged_attention(out, q, kc, vc, bt, sl, cu, 1, 0.088, decode=True, num_splits=splits,
                      part_o=po, part_ml=pml)
    ref = A.paged_attention_ref(q, kc, vc, bt, sl, cu, 0.088)
    assert rel_err(out, ref) < 2e-2


@pytest.mark.parametrize("d,hq,hkv", [(128, 32, 8), (256, 16, 2)])
def test_prefill_and_chunked(b200_ops, d, hq, hkv, rel_err):
    lens_q = [5, 130, 64, 1]
    lens_ctx = [5, 200, 64, 33]  # seq 1 and 3 have a cached prefix (chunked prefill)
    q, kc, vc, bt, sl, cu = _case(lens_q, lens_ctx, hq, hkv, d, 16, seed=2)
    out = torch.empty_like(q)
    A.paged_attention(out, q, kc, vc, bt, sl, cu, max(lens_q), 1 / math.sqrt(d))
    ref = A.paged_attention_ref(q, kc, vc, bt, sl, cu, 1 / math.sqrt(d))
    assert rel_err(out, ref) < 2e-2


@pytest.mark.parametrize("d,hq,hkv,bs", [(128, 32, 8, 16), (256, 16, 2, 16), (256, 16, 2, 64),
                                         (256, 16, 2, 128)])
def test_prefill_long_tcgen05(b200_ops, d, hq, hkv, bs, rel_err):
    """Multi-tile causal prefill and chunked prefill through the tcgen05
    kernel (head_dim 256: 64-key tiles; block size 128 exceeds its tile and
    takes the mma.sync kernel), against the fp32 oracle."""
    lens_q = [700, 300, 129]
    lens_ctx = [700, 900, 129]
    q, kc, vc, bt, sl, cu = _case(lens_q, lens_ctx, hq, hkv, d, bs, seed=12)
    out = torch.empty_like(q)
    A.paged_attention(out, q, kc, vc, bt, sl, cu, max(lens_q), 1 / math.sqrt(d))
    ref = A.paged_attention_ref(q, kc, vc, bt, sl, cu, 1 / math.sqrt(d))
    assert torch.isfinite(out.float()).all()
    assert rel_err(out, ref) < 2e-2
    assert int(torch.ops._b200_C.read_status(0, True)) == 0


@pytest.mark.parametrize("d,hq,hkv", [(128, 32, 8), (256, 16, 2)])
def test_spec_verify_rows(b200_ops, d, hq, hkv, rel_err):
    # 4 query tokens per request (k=3 draft + 1) through the decode variant
    # (D = 256: the Qwen3-Next gated-attention shape, 8 query heads per KV head).
    q, kc, vc, bt, sl, cu = _case([4, 4], [50, 400], hq, hkv, d, 16, seed=3)
    out = torch.empty_like(q)
    A.paged_attention(out, q, kc, vc, bt, sl, cu, 4, 0.09, decode=True)
    ref = A.paged_attention_ref(q, kc, vc, bt, sl, cu, 0.09)
    assert rel_err(out, ref) < 2e-2


def test_sinks_and_window(b200_ops, rel_err):
    q, kc, vc, bt, sl, cu = _case([1, 1, 9], [600, 40, 300], 16, 2, 128, 16, seed=4)
    sinks = torch.randn(16, device="cuda")
    out = torch.empty_like(q)
    A.paged_attention(out, q, kc, vc, bt, sl, cu, 9, 0.1, window=128, sinks=sinks)
    ref = A.paged_attention_ref(q, kc, vc, bt, sl, cu, 0.1, window=128, sinks=sinks)
    assert rel_err(out, ref) < 2e-2


@pytest.mark.parametrize("d,hq,hkv", [(128, 32, 8), (256, 16, 2)])
def test_decode_sinks_window(b200_ops, d, hq, hkv, rel_err):
    q, kc, vc, bt, sl, cu = _case([1, 1, 1], [600, 40, 1300], hq, hkv, d, 16, seed=6)
    sinks = torch.randn(hq, device="cuda")
    out = torch.empty_like(q)
    A.paged_attention(out, q, kc, vc, bt, sl, cu, 1, 0.1, window=256, sinks=sinks, decode=True)
    ref = A.paged_attention_ref(q, kc, vc, bt, sl, cu, 0.1, window=256, sinks=sinks)
    assert rel_err(out, ref) < 2e-2


@pytest.mark.parametrize("bs", [16, 64])
def test_decode_interleaved_cache(b200_ops, bs, rel_err):
    """K and V of a block interleaved in one allocation ([blocks, 2, Hkv, BS, D],
    the vLLM backend layout): strided cache blocks through the decode path."""
    q, kc, vc, bt, sl, cu = _case([1] * 4, [5, 333, 1024, 77], 32, 8, 128, bs, seed=7)
    both = torch.stack([kc, vc], dim=1).contiguous()
    out = torch.empty_like(q)
    A.paged_attention(out, q, both[:, 0], both[:, 1], bt, sl, cu, 1, 0.09, decode=True)
    ref = A.paged_attention_ref(q, kc, vc, bt, sl, cu, 0.09)
    assert rel_err(out, ref) < 2e-2


@pytest.mark.parametrize("d,hq,hkv,bs", [(128, 32, 8, 16), (128, 32, 8, 128), (256, 16, 2, 16),
                                         (256, 16, 2, 64)])
@pytest.mark.parametrize("decode", [True, False])
def test_stale_cache_rows_nan(b200_ops, d, hq, hkv, bs, decode, rel_err):
    """Cache rows past each sequence end hold NaN (stale contents of a
    recycled block): masking and V-row zeroing keep them out of the output."""
    lens = [1, 17, 300, 129]
    lens_q = [1] * 4 if decode else [1, 17, 44, 129]
    q, kc, vc, bt, sl, cu = _case(lens_q, lens, hq, hkv, d, bs, seed=8)
    for i, L in enumerate(lens):
        if L % bs:
            blk = int(bt[i, (L - 1) // bs])
            kc[blk, :, L % bs:] = float("nan")
            vc[blk, :, L % bs:] = float("nan")
    out = torch.empty_like(q)
    A.paged_attention(out, q, kc, vc, bt, sl, cu, max(lens_q), 0.09, decode=decode)
    ref = A.paged_attention_ref(q, kc, vc, bt, sl, cu, 0.09)
    assert torch.isfinite(out.float()).all()
    assert rel_err(out, ref) < 2e-2


@pytest.mark.parametrize("d,rot,norm", [(128, 128, True), (128, 128, False), (64, 64, True),
                                         (256, 256, True), (256, 64, True)])
def test_rope_kv_write(b200_ops, rel_err, d, rot, norm):
    """Full-width rotation runs the 16-byte-access kernel (D/16 threads per
    head), partial rotation the warp-per-head kernel; both against the fp32
    reference, V copied bit-exactly."""
    torch.manual_seed(5)
    T, hq, hkv, bs = 37, 8, 2, 16
    qkv = torch.randn(T, (hq + 2 * hkv) * d, device="cuda", dtype=torch.bfloat16)
    pos = torch.randint(0, 500, (T,), device="cuda")
    slots = torch.randperm(64 * bs, device="cuda")[:T]
    slots[3] = -1
    cs = A.rope_cos_sin(rot, 1024, 5e5, device="cuda")
    qn = torch.randn(d, device="cuda", dtype=torch.bfloat16) if norm else None
    kn = torch.randn(d, device="cuda", dtype=torch.bfloat16) if norm else None
    kc = torch.zeros(64, hkv, bs, d, device="cuda", dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    qkv2, kc2, vc2 = qkv.clone(), kc.clone(), vc.clone()
    A.rope_kv_write(qkv, pos, cs, kc, vc, slots, hq, hkv, qn, kn, 1e-6)
    A.rope_kv_write_ref(qkv2, pos, cs, kc2, vc2, slots, hq, hkv, qn, kn, 1e-6)
    assert rel_err(qkv, qkv2) < 1e-2
    assert rel_err(kc, kc2) < 1e-2
    assert torch.equal(vc, vc2)
