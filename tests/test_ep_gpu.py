"""Expert-parallel exchange over NVLink peer memory (csrc/comm/ep_a2a.cu) on
2+ GPUs: the peer-memory dispatch / combine returns exactly (bit for bit) the
MoE output of the NCCL all-to-all baseline, over several blocks in a row
(epoch flags advance), with uneven token counts and an idle rank, and both
match computing every expert locally."""
import json
import os

import pytest
import torch

from . import _mp

pytestmark = pytest.mark.gpu

E, K, H, I = 16, 4, 512, 256


def _body(rank, world, out_file):
    from pathlib import Path

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    from vllm_sm70_b200.ops import moe
    from vllm_sm70_b200.parallel import state
    from vllm_sm70_b200.parallel.ep import EPAllToAll

    ps = state.init(tp_size=1, ep_size=world, backend="nccl", timeout_s=120)
    dev = ps.device
    g = torch.Generator(device=dev).manual_seed(3)
    w13 = torch.randn(E, 2 * I, H, device=dev, generator=g) * 0.05
    w2 = torch.randn(E, H, I, device=dev, generator=g) * 0.05
    El = E // world
    mine = moe.ExpertWeights.from_dense("bf16", w13[rank * El:(rank + 1) * El],
                                        w2[rank * El:(rank + 1) * El])
    full = moe.ExpertWeights.from_dense("bf16", w13, w2)
    ep = EPAllToAll(ps, E, K)
    ep.reserve(128, H)
    assert ep.peer is not None
    ws = moe.MoEWorkspace(1024, K, El, H, I, dev)
    ws_full = moe.MoEWorkspace(1024, K, E, H, I, dev)
    res = []
    for it, T in enumerate([[37, 0, 64, 5], [1, 9, 0, 128], [100, 100, 3, 0]]):
        T = T[rank % 4]
        gt = torch.Generator(device=dev).manual_seed(1000 * it + rank)
        x = torch.randn(T, H, device=dev, generator=gt).to(torch.bfloat16)
        shared = torch.randn(T, H, device=dev, generator=gt).to(torch.bfloat16)
        w, ids = moe.topk(torch.randn(T, E, device=dev, generator=gt), K)
        outs = []
        for peer in (True, False):
            saved = ep.peer
            if not peer:
                ep.peer = None  # the NCCL all-to-all baseline
            ep.step(True, T)
            xr, wr, idr, plan = ep.dispatch(x, w, ids)
            yr = xr.new_empty(xr.shape[0], H)
            if xr.shape[0]:
                moe.experts_forward(xr, wr, idr, mine, ws, rank * El, None, yr)
            outs.append(ep.combine(yr, plan, shared))
            ep.peer = saved
        torch.cuda.synchronize()
        local = moe.experts_forward(x, w, ids, full, ws_full, 0, shared) if T else outs[1]
        st = int(torch.ops._b200_C.read_status(dev.index, True))
        res.append({"T": T, "equal": bool(torch.equal(outs[0], outs[1])),
                    "err_local": float((outs[0].float() - local.float()).abs().max()) if T else 0.0,
                    "status": st})
    Path(f"{out_file}.{rank}").write_text(json.dumps(res))
    torch.cuda.synchronize()
    state.shutdown()


@pytest.mark.parametrize("world", [2, 4])
def test_peer_ep_equals_nccl_baseline(tmp_path, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    out = tmp_path / "r"
    _mp.run(_body, world, args=(str(out),), timeout=600)
    for r in range(world):
        for d in json.loads((tmp_path / f"r.{r}").read_text()):
            assert d["equal"] and d["status"] == 0, (r, d)
            assert d["err_local"] < 0.05, (r, d)
