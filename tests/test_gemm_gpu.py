"""tcgen05 BF16 GEMM vs an fp32 torch reference (all tile configs)."""
import pytest
import torch

from vllm_sm70_b200.ops import linear

pytestmark = pytest.mark.gpu

CFGS = {"n256": 0, "n128": 1, "swap16": 2, "swap32": 3, "swap64": 4, "n192": 5, "n96": 6,
        "n64": 7, "swap128": 8, "m2n256": 9, "m2n224": 10, "m2n128": 11, "m2n112": 12,
        "m2n64": 13, "cl_n256": 14, "cl_n128": 15, "cl_m2n128": 16, "cl_m2n112": 17,
        "cl_m2n64": 18, "p2n256": 19, "p2n128": 20, "p2n192": 21, "p2n64": 22, "p2n96": 23}
# cluster split-K config -> the plain tile of the same shape (same summation order)
CL_PLAIN = {"cl_n256": "n256", "cl_n128": "n128", "cl_m2n128": "m2n128", "cl_m2n112": "m2n112",
            "cl_m2n64": "m2n64"}


def _ref(a, w):
    return a.float() @ w.float().t()


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 4096), (300, 1000, 520),
                                   (1, 4096, 4096), (17, 6144, 4096), (64, 384, 128),
                                   (1024, 1024, 1024)])
@pytest.mark.parametrize("cfg", list(CFGS))
def test_gemm_configs(b200_ops, M, N, K, cfg, rel_err):
    torch.manual_seed(0)
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
    if cfg.startswith("swap") and M > int(cfg[4:]) * 8:
        pytest.skip("swap configs target small M")
    out = linear.gemm(a, w, cfg=CFGS[cfg])
    torch.cuda.synchronize()
    ref = _ref(a, w)
    assert rel_err(out, ref) < 1e-2, (M, N, K, cfg)


def test_gemm_auto_and_strided(b200_ops, rel_err):
    torch.manual_seed(1)
    big = torch.randn(64, 4096 + 64, device="cuda", dtype=torch.bfloat16)
    a = big[:, :4096]  # leading dim 4160
    w = torch.randn(2048, 4096, device="cuda", dtype=torch.bfloat16) * 0.02
    out = linear.gemm(a, w)
    assert rel_err(out, _ref(a, w)) < 1e-2


@pytest.mark.parametrize("M", [1, 40, 256, 777])
def test_gemm_silu_mul(b200_ops, M, rel_err):
    torch.manual_seed(2)
    K, N = 512, 768
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    wg = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
    wu = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
    wi = linear.interleave_gate_up(wg, wu)
    out = linear.gemm_silu_mul(a, wi)
    g = a.float() @ wg.float().t()
    u = a.float() @ wu.float().t()
    ref = g * torch.sigmoid(g) * u
    assert rel_err(out, ref) < 2e-2


@pytest.mark.parametrize("cfg", [0, 1, 9, 11, 19, 20])
@pytest.mark.parametrize("M", [200, 256, 777])
def test_gemm_silu_mul_configs(b200_ops, cfg, M, rel_err):
    torch.manual_seed(6)
    K, N = 1024, 640
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    wg = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
    wu = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
    wi = linear.interleave_gate_up(wg, wu)
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    torch.ops._b200_C.gemm_bf16_silu_mul_out(out, a, wi, cfg)
    g = a.float() @ wg.float().t()
    u = a.float() @ wu.float().t()
    assert rel_err(out, g * torch.sigmoid(g) * u) < 2e-2


def test_gemm_deterministic(b200_ops):
    torch.manual_seed(3)
    a = torch.randn(512, 1024, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(2048, 1024, device="cuda", dtype=torch.bfloat16)
    o1 = linear.gemm(a, w)
    o2 = linear.gemm(a, w)
    assert torch.equal(o1, o2)


@pytest.mark.parametrize("cfg", ["n256", "n128", "swap16", "swap64", "n192", "n96", "swap128",
                                 "m2n256", "m2n224", "m2n128", "m2n112", "m2n64"])
@pytest.mark.parametrize("splits", [2, 3, 5, 8])
def test_gemm_split_k(b200_ops, cfg, splits, rel_err):
    torch.manual_seed(4)
    M = {"n256": 256, "n128": 200, "swap16": 9, "swap64": 50, "n192": 256, "n96": 130,
         "swap128": 100, "m2n256": 256, "m2n224": 300, "m2n128": 200, "m2n112": 512,
         "m2n64": 256}[cfg]
    N, K = 1536, 4096 + 64
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
    ref = _ref(a, w)
    outs = [linear.gemm(a, w, cfg=CFGS[cfg], splits=splits) for _ in range(3)]
    torch.cuda.synchronize()
    assert rel_err(outs[0], ref) < 1e-2
    # Fixed-order reduction: bitwise identical across calls (counters re-arm).
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])


@pytest.mark.parametrize("cfg", ["p2n256", "p2n128", "p2n192", "p2n64", "p2n96"])
@pytest.mark.parametrize("M,N,K", [(256, 1024, 4096), (300, 640, 520), (1024, 2048, 1024),
                                   (128, 256, 64), (777, 1536, 2048)])
def test_gemm_cta_pair(b200_ops, cfg, M, N, K, rel_err):
    torch.manual_seed(9)
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
    out = linear.gemm(a, w, cfg=CFGS[cfg], splits=1)
    torch.cuda.synchronize()
    assert rel_err(out, _ref(a, w)) < 1e-2, (cfg, M, N, K)


@pytest.mark.parametrize("cfg", ["p2n256", "p2n128", "p2n96"])
@pytest.mark.parametrize("splits", [2, 3, 8])
def test_gemm_cta_pair_split_k(b200_ops, cfg, splits, rel_err):
    torch.manual_seed(10)
    M, N, K = 256, 1536, 4096 + 64
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
    outs = [linear.gemm(a, w, cfg=CFGS[cfg], splits=splits) for _ in range(2)]
    torch.cuda.synchronize()
    assert rel_err(outs[0], _ref(a, w)) < 1e-2
    assert torch.equal(outs[0], outs[1])


@pytest.mark.parametrize("cfg", list(CL_PLAIN))
@pytest.mark.parametrize("splits", [2, 3, 5, 8])
@pytest.mark.parametrize("M", [256, 200, 64])
def test_gemm_cluster_split_matches_workspace_split(b200_ops, cfg, splits, M, rel_err):
    torch.manual_seed(7)
    N, K = 1024 + 128, 4096 + 64
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
    outs = [linear.gemm(a, w, cfg=CFGS[cfg], splits=splits) for _ in range(2)]
    plain = linear.gemm(a, w, cfg=CFGS[CL_PLAIN[cfg]], splits=splits)
    torch.cuda.synchronize()
    assert rel_err(outs[0], _ref(a, w)) < 1e-2
    # DSMEM reduction sums the splits in the same fixed order as the workspace path.
    assert torch.equal(outs[0], outs[1])
    assert torch.equal(outs[0], plain)


@pytest.mark.parametrize("cfg", [14, 16])
@pytest.mark.parametrize("splits", [2, 4])
def test_gemm_silu_cluster_split(b200_ops, cfg, splits, rel_err):
    torch.manual_seed(8)
    M, K, N = 256, 4096, 640
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    wg = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.02
    wu = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.02
    wi = linear.interleave_gate_up(wg, wu)
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    torch.ops._b200_C.gemm_set_plan(M, 2 * N, K, 1, cfg, splits)
    try:
        torch.ops._b200_C.gemm_bf16_silu_mul_out(out, a, wi, -1)
    finally:
        torch.ops._b200_C.gemm_set_plan(M, 2 * N, K, 1, -1, 0)
    g = a.float() @ wg.float().t()
    u = a.float() @ wu.float().t()
    assert rel_err(out, g * torch.sigmoid(g) * u) < 2e-2


def test_gemm_silu_split(b200_ops, rel_err):
    torch.manual_seed(5)
    M, K, N = 256, 4096, 512
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    wg = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.02
    wu = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.02
    wi = linear.interleave_gate_up(wg, wu)
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    torch.ops._b200_C.gemm_bf16_silu_mul_out(out, a, wi, -1)
    g = a.float() @ wg.float().t()
    u = a.float() @ wu.float().t()
    assert rel_err(out, g * torch.sigmoid(g) * u) < 2e-2


def test_planner_uses_split_for_decode_shapes(b200_ops):
    cfg, s = linear.plan(256, 6144, 4096, 0, 148)
    assert s > 1
    cfg, s = linear.plan(16384, 6144, 4096, 0, 148)
    assert s == 1


def test_tuner_installs_plans(b200_ops):
    from vllm_sm70_b200.engine import warmup

    torch.ops._b200_C.gemm_clear_plans()
    linear.clear_library()
    plans = warmup.tune_shapes([(256, 1536, 1024, 0), (64, 1024, 512, 0), (128, 1024, 512, 1)],
                               iters=2, library=False)
    assert len(plans) == 3
    exported = warmup.export_plans()
    assert sorted(map(tuple, exported)) == sorted(map(tuple, plans))
    for M, N, K, epi, cfg, sp in plans:
        assert tuple(torch.ops._b200_C.gemm_bf16_plan(M, N, K, epi, 148)) == (cfg, sp)
    torch.ops._b200_C.gemm_clear_plans()


def test_tuner_library_route(b200_ops, rel_err):
    """A shape the tuner routes to the vendor library still computes the GEMM,
    and the route survives an export / import round trip."""
    from vllm_sm70_b200.engine import warmup

    torch.ops._b200_C.gemm_clear_plans()
    linear.clear_library()
    try:
        M, N, K = 256, 2048, 1024
        plans = warmup.tune_shapes([(M, N, K, 0)], iters=2, library=True)
        exported = warmup.export_plans()
        assert sorted(map(tuple, exported)) == sorted(map(tuple, plans))
        linear.set_library(M, N, K)  # force the library route for the check
        a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
        w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
        assert rel_err(linear.gemm(a, w), _ref(a, w)) < 1e-2
        linear.clear_library()
        warmup.install_plans([[M, N, K, 0, linear.LIBRARY_CFG, 0]])
        assert (M, N, K) in linear.library_shapes()
    finally:
        torch.ops._b200_C.gemm_clear_plans()
        linear.clear_library()


def test_silu_mul_interleaved_and_library_route(b200_ops, rel_err):
    torch.manual_seed(11)
    M, K, N = 200, 512, 640
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    wg = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
    wu = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
    wi = linear.interleave_gate_up(wg, wu)
    g = a.float() @ wg.float().t()
    u = a.float() @ wu.float().t()
    ref = g * torch.sigmoid(g) * u
    # interleaved SiLU kernel on a precomputed [M, 2N] interleaved product
    gu = (a.float() @ wi.float().t()).to(torch.bfloat16)
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    torch.ops._b200_C.silu_mul(out, gu, linear.GATE_UP_BLOCK)
    assert rel_err(out, ref) < 2e-2
    # the tuner's library route for gate_up
    linear.clear_library()
    try:
        linear.set_library(M, 2 * N, K, True, 1)
        assert rel_err(linear.gemm_silu_mul(a, wi), ref) < 2e-2
    finally:
        linear.clear_library()


@pytest.mark.parametrize("cfg,M", [("n128", 1024), ("p2n128", 2048), ("swap64", 200)])
@pytest.mark.parametrize("splits", [2, 3])
def test_gemm_split_k_multi_round(b200_ops, cfg, M, splits, rel_err):
    """More split units than resident CTAs: the serial (last-arriving split)
    reduction, not the distributed one-round reduction, runs; results are
    correct and bitwise repeatable."""
    torch.manual_seed(12)
    N, K = 4096, 2048
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
    outs = [linear.gemm(a, w, cfg=CFGS[cfg], splits=splits) for _ in range(2)]
    torch.cuda.synchronize()
    assert rel_err(outs[0], _ref(a, w)) < 1e-2
    assert torch.equal(outs[0], outs[1])


@pytest.mark.parametrize("M,N,K", [(256, 6144, 4096), (256, 4096, 14336), (256, 4096, 4096)])
def test_gemm_decode_shapes_all_plans(b200_ops, M, N, K, rel_err):
    """Every tuner candidate (tile config x split) on the decode shapes of the
    headline model: correct, and repeatable bit for bit."""
    from vllm_sm70_b200.engine import warmup

    torch.manual_seed(13)
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.02
    ref = _ref(a, w)
    for cfg, sp in warmup.candidates(M, N, K, 0):
        o1 = linear.gemm(a, w, cfg=cfg, splits=sp)
        o2 = linear.gemm(a, w, cfg=cfg, splits=sp)
        torch.cuda.synchronize()
        assert rel_err(o1, ref) < 1e-2, (cfg, sp)
        assert torch.equal(o1, o2), (cfg, sp)


@pytest.mark.parametrize("M,cfg,splits", [(256, 0, 1), (256, 0, 3), (1000, 11, 2), (4096, 9, 1),
                                          (7, 0, 2)])
def test_gemm_add_rmsnorm_tp1_bitwise(b200_ops, M, cfg, splits):
    """TP1 row GEMM + residual add + RMSNorm in one kernel (the fused
    all-reduce epilogue with one rank) equals the GEMM with the same plan
    followed by fused_add_rms_norm, bit for bit, across repeated calls."""
    from vllm_sm70_b200.ops import norm
    from vllm_sm70_b200.parallel import symm

    torch.manual_seed(11)
    N, K = 4096, 4096
    f = symm.LocalAddRmsNorm("cuda", 4096, N)
    w = (torch.randn(N, K, device="cuda") * 0.02).to(torch.bfloat16)
    nw = (torch.randn(N, device="cuda") * 0.5 + 1).to(torch.bfloat16)
    for it in range(3):
        x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
        res = torch.randn(M, N, device="cuda", dtype=torch.bfloat16)
        got_x, got_r = f.gemm(x, w, res.clone(), nw, 1e-5, cfg, splits)
        # the fused launcher maps the plan onto its tiles; compare with that plan
        ref_x = linear.gemm(x, w, cfg=cfg, splits=splits)
        ref_r = res.clone()
        norm.fused_add_rms_norm(ref_x, ref_r, nw, 1e-5)
        torch.cuda.synchronize()
        assert torch.equal(got_r, ref_r), (M, cfg, splits, it)
        assert torch.equal(got_x, ref_x), (M, cfg, splits, it)
    assert int(torch.ops._b200_C.read_status(0, True)) == 0
