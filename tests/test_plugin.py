"""vLLM plugin surface: entry points, platform detection, IR providers, OOT custom ops,
env flags, native-arch guard, collect-env (CPU; NVML and devices faked)."""
import importlib
import json
import sys
import types

import pytest
import torch


def test_entry_points_declared():
    src = open("setup.py").read()
    assert "vllm.platform_plugins" in src and "b200 = vllm_musa_b200:b200_platform_plugin" in src
    assert "vllm.general_plugins" in src and "vllm_musa_b200:register_custom_ops" in src


def _fake_nvml(monkeypatch, caps):
    m = types.ModuleType("pynvml")
    m.nvmlInit = lambda: None
    m.nvmlShutdown = lambda: None
    m.nvmlDeviceGetCount = lambda: len(caps)
    m.nvmlDeviceGetHandleByIndex = lambda i: i
    m.nvmlDeviceGetCudaComputeCapability = lambda h: caps[h]
    monkeypatch.setitem(sys.modules, "pynvml", m)


def test_platform_plugin_detection(monkeypatch):
    from vllm_musa_b200 import plugin
    monkeypatch.delenv("B200_FORCE_PLATFORM", raising=False)
    _fake_nvml(monkeypatch, [(9, 0), (10, 0)])
    assert plugin.platform_plugin() == "vllm_musa_b200.platform.B200Platform"
    _fake_nvml(monkeypatch, [(9, 0)])
    assert plugin.platform_plugin() is None
    monkeypatch.setenv("B200_FORCE_PLATFORM", "1")
    assert plugin.platform_plugin() == "vllm_musa_b200.platform.B200Platform"


def test_env_flags_typed(monkeypatch):
    from vllm_musa_b200 import envs
    monkeypatch.setenv("B200_DISABLE_CUSTOM_AR", "yes")
    assert envs.get("B200_DISABLE_CUSTOM_AR") is True
    monkeypatch.setenv("B200_AR_ONE_SHOT_MAX_BYTES", "abc")
    with pytest.raises(ValueError):
        envs.get("B200_AR_ONE_SHOT_MAX_BYTES")
    monkeypatch.delenv("B200_AR_ONE_SHOT_MAX_BYTES")
    assert envs.snapshot()["B200_AR_ONE_SHOT_MAX_BYTES"] == 0  # automatic (world-dependent)


def test_native_arch_guard():
    from vllm_musa_b200.native_arch import check_device_arch
    check_device_arch((10, 0), "B200")
    with pytest.raises(RuntimeError, match="sm_100a"):
        check_device_arch((9, 0), "H100")


def test_ir_providers_register_and_match_native():
    vllm_ir = pytest.importorskip("vllm.ir")
    from vllm_musa_b200 import plugin
    if "b200" not in vllm_ir.ops.rms_norm.impls:
        plugin.register_ir_providers(vllm_ir)
    assert "b200" in vllm_ir.ops.rms_norm.impls
    assert "b200" in vllm_ir.ops.fused_add_rms_norm.impls
    impl = vllm_ir.ops.rms_norm.impls["b200"]
    x = torch.randn(4, 64, dtype=torch.bfloat16)
    assert not impl.supports_args(x, None, 1e-6)  # CPU tensors are not ours


def test_oot_custom_op_classes():
    pytest.importorskip("vllm")
    from vllm_musa_b200 import plugin
    silu, rope = plugin.make_custom_op_classes()
    from vllm.model_executor.layers.activation import SiluAndMul
    from vllm.model_executor.layers.rotary_embedding import RotaryEmbedding
    assert issubclass(silu, SiluAndMul) and issubclass(rope, RotaryEmbedding)


def test_collect_env_runs():
    from vllm_musa_b200.collect_env import get_env_info
    info = get_env_info()
    assert "flags" in info and "built_archs" in info
    json.dumps(info, default=str)


def test_rope_rotate_only_cpu_matches_reference():
    from vllm_musa_b200 import ops
    T, Hq, Hk, D = 5, 4, 2, 64
    qkv = torch.randn(T, (Hq + 2 * Hk) * D)
    pos = torch.arange(T, dtype=torch.int32)
    cs = ops.build_cos_sin_cache(D, 64, 1e4)
    a = qkv.clone()
    ops.rope_kv(a, pos, cs, None, None, torch.full((T,), -1, dtype=torch.int32), Hq, Hk, D,
                write_k=True, head_dim=D)
    from vllm_musa_b200.ops.rope import _rotate_ref
    q = _rotate_ref(qkv[:, :Hq * D].view(T, Hq, D), cs[pos.long()], D, True)
    k = _rotate_ref(qkv[:, Hq * D:(Hq + Hk) * D].view(T, Hk, D), cs[pos.long()], D, True)
    torch.testing.assert_close(a[:, :Hq * D], q.reshape(T, -1))
    torch.testing.assert_close(a[:, Hq * D:(Hq + Hk) * D], k.reshape(T, -1))
    torch.testing.assert_close(a[:, (Hq + Hk) * D:], qkv[:, (Hq + Hk) * D:])


def test_custom_op_preload_list_imports():
    from vllm_musa_b200 import plugin
    assert "vllm_musa_b200.ops" in plugin.CUSTOM_OP_MODULES
    plugin.preload_custom_op_modules()
