"""Every ``_b200_C`` op either traces under FakeTensor mode or is a listed
host-side control / collective op (the reference's NO_FAKE_OPS rule)."""
import pytest
import torch

from vllm_sm70_b200 import _ext


@pytest.fixture(scope="module")
def ext():
    if not _ext.load():
        pytest.skip(f"_b200_C not built: {_ext.error()}")
    from vllm_sm70_b200.ops import _fakes

    _fakes.register_all()
    return _fakes


def test_every_op_has_a_fake_or_a_reason(ext):
    assert ext.missing() == []
    names = {s.name.split("::", 1)[1] for s in ext._schemas()}
    assert set(ext.NO_FAKE) <= names, "stale NO_FAKE entries"


def test_fakes_trace(ext):
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        a = torch.empty(7, 64, dtype=torch.bfloat16)
        w = torch.empty(32, 64, dtype=torch.bfloat16)
        out = torch.ops._b200_C.gemm_bf16(a, w, -1)
        assert out.shape == (7, 32)
        o = torch.empty(7, 16, dtype=torch.bfloat16)
        torch.ops._b200_C.silu_mul(o, torch.empty(7, 32, dtype=torch.bfloat16), 0)
