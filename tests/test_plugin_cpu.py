"""Plugin surface on CPU: platform activation through a fake NVML (indices,
UUIDs, mixed GPUs, no NVML), area registration and strict mode, env kill-
switch semantics, the typed config, graph policy, the composite pass and the
U1 hook wiring. Reference parity: sm70/tests/plugin/conftest.py:20-131
(FakeNvml, fresh_plugin, no_ext) and the plugin test directory."""
import pytest
import torch

import vllm_sm70_b200 as pkg
from vllm_sm70_b200 import config as cfgmod
from vllm_sm70_b200 import envs, platform


class FakeNvml:
    def __init__(self, caps, uuids=None, fail_init=False):
        self.caps = caps
        self.uuids = uuids or [f"GPU-{i:04d}" for i in range(len(caps))]
        self.fail_init = fail_init
        self.shutdowns = 0

    def nvmlInit(self):
        if self.fail_init:
            raise RuntimeError("no NVML")

    def nvmlShutdown(self):
        self.shutdowns += 1

    def nvmlDeviceGetCount(self):
        return len(self.caps)

    def nvmlDeviceGetHandleByIndex(self, i):
        return i

    def nvmlDeviceGetHandleByUUID(self, u):
        return self.uuids.index(u)

    def nvmlDeviceGetCudaComputeCapability(self, h):
        return self.caps[h]


@pytest.fixture
def fake_nvml(monkeypatch):
    def install(caps, **kw):
        nv = FakeNvml(caps, **kw)
        monkeypatch.setattr(platform, "_nvml", lambda: nv)
        return nv
    return install


def test_activate_all_b200(fake_nvml, monkeypatch):
    monkeypatch.delenv("CUDA_VISIBLE_DEVICES", raising=False)
    fake_nvml([(10, 0)] * 8)
    assert platform.activate() == platform.PLATFORM_QUALNAME


def test_activate_rejects_mixed(fake_nvml, monkeypatch):
    monkeypatch.delenv("CUDA_VISIBLE_DEVICES", raising=False)
    fake_nvml([(10, 0), (9, 0)])
    assert platform.activate() is None


def test_visible_devices_indices_and_uuids(fake_nvml, monkeypatch):
    nv = fake_nvml([(9, 0), (10, 0), (10, 0)])
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "1,2")
    assert platform.activate() == platform.PLATFORM_QUALNAME
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "GPU-0002")
    assert platform.activate() == platform.PLATFORM_QUALNAME
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "0")
    assert platform.activate() is None
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "")
    assert platform.activate() is None
    assert nv.shutdowns >= 4


def test_no_nvml_and_kill_switch(fake_nvml, monkeypatch):
    fake_nvml([(10, 0)], fail_init=True)
    assert platform.activate() is None
    fake_nvml([(10, 0)])
    monkeypatch.setenv("VLLM_B200_PLATFORM", "0")
    assert platform.activate() is None


def test_register_is_idempotent_and_records_areas():
    pkg._reset_for_tests()
    pkg.register()
    pkg.register()
    st = pkg.area_status()
    assert set(st) == set(pkg.AREAS)
    assert pkg.failed_areas() == {}


def test_failed_area_recorded_and_retried(monkeypatch):
    pkg._reset_for_tests()
    monkeypatch.setitem(pkg._AREA_MODULES, "passes", "vllm_sm70_b200.does_not_exist")
    pkg.register()
    assert "passes" in pkg.failed_areas()
    monkeypatch.setitem(pkg._AREA_MODULES, "passes", "vllm_sm70_b200.integration.passes")
    assert pkg.retry_failed_areas() == {}
    pkg._reset_for_tests()


def test_kill_switch_semantics(monkeypatch):
    monkeypatch.setenv("VLLM_B200_GEMM", "1")
    assert envs.get("VLLM_B200_GEMM") is True
    monkeypatch.setenv("VLLM_B200_GEMM", "false")  # only "0" acts
    assert envs.get("VLLM_B200_GEMM") is True
    monkeypatch.setenv("VLLM_B200_GEMM", "0")
    assert envs.get("VLLM_B200_GEMM") is False
    monkeypatch.setenv("VLLM_B200_NVLS", "yes")  # opt-in: only "1" acts
    assert envs.get("VLLM_B200_NVLS") is False
    monkeypatch.setenv("VLLM_B200_NVLS", "1")
    assert envs.get("VLLM_B200_NVLS") is True


def test_typed_config_env_can_only_disable(monkeypatch):
    c = cfgmod.B200Config(gemm=False)
    monkeypatch.setenv("VLLM_B200_GEMM", "1")
    assert c.with_env().gemm is False  # env never re-enables
    monkeypatch.setenv("VLLM_B200_ATTN", "0")
    assert cfgmod.B200Config().with_env().attention is False
    with pytest.raises(Exception):
        cfgmod.B200Config(not_a_field=1)
    with pytest.raises(Exception):
        c.gemm = True  # frozen


def test_config_hash_covers_graph_fields_only():
    a = cfgmod.B200Config()
    assert a.compute_hash() == cfgmod.B200Config(gemm_lut_path="/x").compute_hash()
    assert a.compute_hash() != cfgmod.B200Config(attention=False).compute_hash()


def test_config_from_vllm_additional_config():
    class V:
        additional_config = {"sm70": {"block_size": 32}}

    v = V()
    c = cfgmod.b200_config(v)
    assert c.block_size == 32
    assert cfgmod.b200_config(v) is c  # cached per config object


def test_graph_policy_sizes():
    from vllm_sm70_b200.integration import graph_policy

    s = graph_policy.capture_sizes(256)
    assert s[0] == 1 and s[-1] == 256 and s == sorted(set(s))
    sp = graph_policy.capture_sizes(8, spec_tokens=3)
    assert all(x % 4 == 0 for x in sp)


def test_composite_pass_runs_patterns_and_hashes():
    from vllm_sm70_b200.integration import passes

    seen = []

    def pat(graph):
        seen.append(graph)
        return 1

    cp = passes.CompositePass([pat])
    cp("g")
    assert seen == ["g"]
    assert len(cp.uuid()) == 64

    class Comp:
        inductor_compile_config = {}

    class V:
        compilation_config = Comp()

    assert passes.install_composite_pass(V())
    assert isinstance(V.compilation_config.inductor_compile_config["post_grad_custom_post_pass"],
                      passes.CompositePass)


def test_u1_gemm_fallback_matches_linear():
    from vllm_sm70_b200.integration import hooks

    x = torch.randn(3, 5, 16)
    w = torch.randn(8, 16)
    b = torch.randn(8)
    torch.testing.assert_close(hooks.b200_unquantized_gemm(None, x, w, b),
                               torch.nn.functional.linear(x, w, b))


def test_ext_fingerprint_and_ops():
    from vllm_sm70_b200 import _ext

    fp = _ext.fingerprint()
    assert fp.startswith("abi=")
    if _ext.load():
        assert _ext.has_op("gemm_bf16_out") and _ext.has_op("paged_attention")
        assert not _ext.has_op("definitely_not_an_op")


def test_top_level_cli_dispatch(monkeypatch, capsys):
    import importlib

    from vllm_sm70_b200 import __main__ as cli

    seen = []
    mod = importlib.import_module("vllm_sm70_b200.models.convert_gguf")
    monkeypatch.setattr(mod, "main", lambda argv: seen.append(argv))
    assert cli.main(["convert-gguf", "a.gguf", "out"]) == 0 and seen == [["a.gguf", "out"]]
    assert cli.main([]) == 0 and "serve" in capsys.readouterr().out
    assert cli.main(["nope"]) == 2
    from vllm_sm70_b200.integration.models import ENGINE_ARCHS, VLLM_ARCHS

    assert ENGINE_ARCHS["flint"].endswith(":FlintModel")
    assert VLLM_ARCHS["B200LlamaForCausalLM"].endswith(":B200LlamaForCausalLM")
