"""Multi-process (gloo, CPU) tests of the TP communication layer: the NCCL-
baseline path of all_reduce + add + RMSNorm, vocab-parallel greedy merge,
and the warm-up plan agreement protocol including a failing rank."""
import torch

from . import _mp


def _ar_norm_body(rank, world):
    from vllm_sm70_b200.ops import norm
    from vllm_sm70_b200.parallel import comm, state

    ps = state.init(tp_size=world, backend="gloo")
    g = torch.Generator().manual_seed(0)
    parts = [torch.randn(5, 64, generator=g).to(torch.bfloat16) for _ in range(world)]
    res = torch.randn(5, 64, generator=g).to(torch.bfloat16)
    w = torch.randn(64, generator=g).to(torch.bfloat16)
    x, r = comm.all_reduce_add_rms_norm(parts[rank].clone(), res.clone(), w, 1e-6)
    tot = parts[0].float()
    for p in parts[1:]:
        tot = tot + p.float()
    x_ref, r_ref = tot.to(torch.bfloat16), res.clone()
    norm.fused_add_rms_norm(x_ref, r_ref, w, 1e-6)
    assert torch.allclose(x.float(), x_ref.float(), atol=2e-2), (x - x_ref).abs().max()
    assert torch.allclose(r.float(), r_ref.float(), atol=2e-2)
    state.shutdown()


def test_all_reduce_add_rms_norm_gloo():
    _mp.run(_ar_norm_body, 2, timeout=120)


def _greedy_body(rank, world):
    from vllm_sm70_b200.ops import sampling
    from vllm_sm70_b200.parallel import comm, state

    state.init(tp_size=world, backend="gloo")
    g = torch.Generator().manual_seed(1)
    full = torch.randn(4, 40, generator=g)
    full[1, 3] = full[1, 33] = 50.0  # cross-rank tie -> lower id
    full[2, 25] = float("nan")
    shard = full[:, rank * 20:(rank + 1) * 20]
    ids, vals = sampling.argmax(shard, id_offset=rank * 20)
    merged = comm.greedy_merge(vals, ids)
    ref, _ = sampling.argmax_ref(full)
    assert merged.tolist() == ref.tolist(), (merged, ref)
    state.shutdown()


def test_vocab_parallel_greedy_gloo():
    _mp.run(_greedy_body, 2, timeout=120)


def _agree_body(rank, world, fail_rank):
    import pytest  # noqa: F401
    from vllm_sm70_b200.engine import warmup
    from vllm_sm70_b200.parallel import state

    ps = state.init(tp_size=world, backend="gloo")
    installed = []
    warmup.install_plans = lambda p: installed.extend(p)  # no native table on CPU
    plans = [[256, 6144, 4096, 0, 0, 3]] if rank == 0 else None
    if rank == fail_rank:
        plans = None
    try:
        out = warmup.agree(plans, ps)
        assert fail_rank < 0, "agreement should fail when rank 0 has no plans"
        assert out == [[256, 6144, 4096, 0, 0, 3]]
        if rank != 0:
            assert installed == out
    except RuntimeError as e:
        assert fail_rank == 0 and "failed on ranks [0]" in str(e), e
    state.shutdown()


def test_warmup_plan_agreement_gloo():
    _mp.run(_agree_body, 2, args=(-1,), timeout=120)


def test_warmup_failure_is_shared_gloo():
    # Rank 0's tuning "fails": every rank raises instead of hanging in a collective.
    _mp.run(_agree_body, 2, args=(0,), timeout=120)
