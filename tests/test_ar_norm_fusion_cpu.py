"""The all-reduce + fused add + RMSNorm graph rewrite on CPU: traced graphs
of vLLM's op pair (``vllm.all_reduce`` -> ``vllm_ir.fused_add_rms_norm``)
are rewritten into one ``vllm_b200`` op per site; an all-reduce with another
user is left alone; the rewritten graph computes the same values (the op
falls back to the unfused pair without an installed fused route, and uses
the route when one is installed); the composite pass carries the pattern."""
import pytest
import torch

vllm_ops = pytest.importorskip("vllm.ir.ops")
pytest.importorskip("vllm.distributed.communication_op")  # registers torch.ops.vllm.all_reduce


@pytest.fixture
def world1(monkeypatch):
    """``vllm.all_reduce`` of a one-rank group (identity), without a vLLM
    distributed environment."""
    from vllm_sm70_b200.integration import ar_norm_fusion as f

    calls = []

    def fake_unfused(x, residual, weight, eps, group):
        calls.append(group)
        return torch.ops.vllm_ir.fused_add_rms_norm(x.clone(), residual, weight, eps)
    monkeypatch.setattr(f, "_unfused", fake_unfused)
    return calls


def _layer_pair(x, r, w1, w2):
    a = torch.ops.vllm.all_reduce(x, "tp:0")
    h, r = torch.ops.vllm_ir.fused_add_rms_norm(a, r, w1, 1e-6)
    b = torch.ops.vllm.all_reduce(h * 2.0, "tp:0")
    h2, r = torch.ops.vllm_ir.fused_add_rms_norm(b, r, w2, 1e-6)
    return h2, r


def _shared_ar(x, r, w):
    a = torch.ops.vllm.all_reduce(x, "tp:0")
    h, r = torch.ops.vllm_ir.fused_add_rms_norm(a, r, w, 1e-6)
    return h + a, r  # the all-reduce output has a second user


def _trace(fn):
    return torch.fx.symbolic_trace(fn)


def _count(gm, target):
    return sum(1 for n in gm.graph.nodes if n.op == "call_function" and n.target is target)


def test_rewrites_every_site(world1):
    from vllm_sm70_b200.integration import ar_norm_fusion as f

    gm = _trace(_layer_pair)
    targets = (torch.ops.vllm.all_reduce, torch.ops.vllm_ir.fused_add_rms_norm)
    n = f.fuse_all_reduce_add_rms_norm(gm, targets)
    assert n == 2
    fused = torch.ops.vllm_b200.all_reduce_fused_add_rms_norm.default
    assert _count(gm, fused) == 2 and _count(gm, targets[0]) == 0 and _count(gm, targets[1]) == 0
    g = torch.Generator().manual_seed(0)
    x, r = torch.randn(5, 16, generator=g), torch.randn(5, 16, generator=g)
    w1, w2 = torch.rand(16, generator=g) + 0.5, torch.rand(16, generator=g) + 0.5
    # reference: all-reduce of one rank is the identity
    a, r0 = torch.ops.vllm_ir.fused_add_rms_norm(x.clone(), r.clone(), w1, 1e-6)
    want = torch.ops.vllm_ir.fused_add_rms_norm(a * 2.0, r0, w2, 1e-6)
    got = gm(x.clone(), r.clone(), w1, w2)
    assert torch.allclose(got[0], want[0]) and torch.allclose(got[1], want[1])
    assert world1 == ["tp:0", "tp:0"]  # the unfused fallback ran with the group name


def test_leaves_shared_all_reduce_alone():
    from vllm_sm70_b200.integration import ar_norm_fusion as f

    gm = _trace(_shared_ar)
    targets = (torch.ops.vllm.all_reduce, torch.ops.vllm_ir.fused_add_rms_norm)
    assert f.fuse_all_reduce_add_rms_norm(gm, targets) == 0


def test_installed_route_is_used(world1, monkeypatch):
    from vllm_sm70_b200.integration import ar_norm_fusion as f

    seen = []

    def route(x, residual, weight, eps):
        seen.append(x.shape)
        return x + 1.0, residual + 2.0
    monkeypatch.setattr(f, "_route", {"fn": route})
    x, r, w = torch.ones(2, 4), torch.zeros(2, 4), torch.ones(4)
    out, res = torch.ops.vllm_b200.all_reduce_fused_add_rms_norm(x, r, w, 1e-6, "tp:0")
    assert seen == [torch.Size([2, 4])] and torch.equal(out, x + 1) and torch.equal(res, r + 2)
    assert world1 == []


def test_composite_pass_carries_pattern():
    from vllm_sm70_b200.integration import ar_norm_fusion as f
    from vllm_sm70_b200.integration import passes

    passes.register()
    assert f.fuse_all_reduce_add_rms_norm in passes.CompositePass().patterns


def test_worker_install_declines_without_tp():
    """Outside a vLLM TP group (here: no distributed state) nothing is
    allocated or installed."""
    from vllm_sm70_b200.integration import ar_norm_fusion as f

    before = f._route["fn"]
    assert f.install_for_worker(object()) is False
    assert f._route["fn"] is before
