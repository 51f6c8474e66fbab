"""TurboQuant KV cache on CPU: level tables, rotation, slot format round trips and the tiny
Llama through the engine with each cache preset (reference behaviour: vllm_musa/v1/attention/
backends/turboquant.py:37-114 and its upstream TurboQuant quantiser)."""
import math
import os
import re

import pytest
import torch

from vllm_musa_b200 import LLM, SamplingParams
from vllm_musa_b200.models.presets import tiny_llama
from vllm_musa_b200.ops import turboquant as tq

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("bits", [3, 4])
def test_levels_are_lloyd_max_and_match_cuda_tables(bits):
    calc = tq.lloyd_max_normal(1 << bits)
    assert max(abs(a - b) for a, b in zip(calc, tq.LEVELS[bits])) < 1e-6
    src = open(os.path.join(ROOT, "csrc", "attention", "turboquant.cu")).read()
    body = re.search(r"c_lv%d\[%d\] = \{([^}]*)\}" % (bits, 1 << bits), src).group(1)
    cuda = [float(x.strip().rstrip("f")) for x in body.split(",") if x.strip()]
    assert cuda == tq.LEVELS[bits]


@pytest.mark.parametrize("D", [64, 128, 256])
def test_rotation_is_orthogonal_and_inverts(D):
    x = torch.randn(32, D)
    y = tq.rotate(x)
    torch.testing.assert_close(y.norm(dim=-1), x.norm(dim=-1), rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(tq.unrotate(y), x, rtol=1e-5, atol=1e-5)


def test_slot_sizes():
    assert tq.tq_format("turboquant_4bit_nc", 128).slot_bytes == 144
    assert tq.tq_format("turboquant_k8v4", 128).slot_bytes == 208
    assert tq.tq_format("turboquant_k3v4_nc", 128).slot_bytes == 128
    assert tq.tq_format("turboquant_3bit_nc", 64).slot_bytes == 64
    # fp8: 128 + 128 code bytes + 6 scale bytes, padded to 16 (vs 512 bytes of bf16 K + V)
    assert tq.tq_format("fp8", 128).slot_bytes == 272
    assert tq.tq_format("fp8_e4m3", 64).slot_bytes == 144
    with pytest.raises(ValueError):
        tq.tq_format("fp4", 128)


@pytest.mark.parametrize("name,kerr,verr", [("fp8", 0.05, 0.05), ("turboquant_k8v4", 0.05, 0.2),
                                            ("turboquant_4bit_nc", 0.15, 0.2),
                                            ("turboquant_k3v4_nc", 0.25, 0.2),
                                            ("turboquant_3bit_nc", 0.25, 0.4)])
@pytest.mark.parametrize("D", [64, 128])
def test_round_trip_error(name, kerr, verr, D):
    g = torch.Generator().manual_seed(1)
    k = torch.randn(256, D, generator=g) * 3
    v = torch.randn(256, D, generator=g)
    fmt = tq.tq_format(name, D)
    slots = tq.quantize_vectors(k, v, fmt)
    assert slots.shape == (256, fmt.slot_bytes)
    kh, vh = tq.dequantize_slots(slots, fmt)
    rel = lambda a, b: ((a - b).norm() / b.norm()).item()  # noqa: E731
    assert rel(kh, k) < kerr
    assert rel(vh, v) < verr
    if fmt.norm_correction:  # dequantised keys keep the vector norm (fp16 scale)
        torch.testing.assert_close(kh.norm(dim=-1), k.norm(dim=-1), rtol=2e-3, atol=1e-3)


def test_scores_in_rotated_space_equal_original_space():
    fmt = tq.tq_format("turboquant_4bit_nc", 128)
    k, v, q = torch.randn(64, 128), torch.randn(64, 128), torch.randn(4, 128)
    slots = tq.quantize_vectors(k, v, fmt)
    k_rot, _ = tq.dequantize_slots(slots, fmt, rotated_keys=True)
    k_org, _ = tq.dequantize_slots(slots, fmt)
    torch.testing.assert_close(tq.rotate(q) @ k_rot.T, q @ k_org.T, rtol=1e-4, atol=1e-4)


def test_store_and_decode_ops_cpu():
    fmt = tq.tq_format("turboquant_k3v4_nc", 64)
    Hq, Hkv, bs, D = 4, 2, 16, 64
    cache = torch.zeros(8, Hkv, bs, fmt.slot_bytes, dtype=torch.uint8)
    T = 40
    k, v = torch.randn(T, Hkv * D), torch.randn(T, Hkv * D)
    tq.tq_store(k, v, cache, torch.arange(T, dtype=torch.int32) + 16, fmt)  # blocks 1..3
    bt = torch.tensor([[1, 2, 3, 0]], dtype=torch.int32)
    q = torch.randn(1, Hq * D)
    out = tq.tq_decode(q, cache, bt, torch.tensor([T], dtype=torch.int32), Hq, 0.125, fmt)
    kh, vh = tq.dequantize_slots(tq.quantize_vectors(k.reshape(-1, D), v.reshape(-1, D), fmt), fmt)
    kh, vh = kh.reshape(T, Hkv, D), vh.reshape(T, Hkv, D)
    qh = q.reshape(Hq, D)
    ref = torch.stack([torch.softmax(qh[h] @ kh[:, h // 2].T * 0.125, -1) @ vh[:, h // 2]
                       for h in range(Hq)]).reshape(1, -1)
    torch.testing.assert_close(out, ref, rtol=1e-4, atol=1e-4)
    kd, vd, bt2 = tq.tq_dequant_pages(cache, bt, torch.tensor([T], dtype=torch.int32), fmt, 3)
    assert bt2.tolist() == [[0, 1, 2]]
    torch.testing.assert_close(kd.float().permute(0, 2, 1, 3).reshape(-1, Hkv, D)[:T], kh,
                               rtol=1e-2, atol=1e-2)


def _generate(kv_cache_dtype):
    cfg = tiny_llama()
    llm = LLM(cfg, device="cpu", block_size=16, seed=0, num_gpu_blocks=64, max_model_len=128,
              max_num_seqs=4, max_num_batched_tokens=48, kv_cache_dtype=kv_cache_dtype)
    llm.engine.runner.record_logits = True
    g = torch.Generator().manual_seed(0)
    prompts = torch.randint(0, 1024, (4, 32), generator=g).tolist()
    outs = llm.generate(prompts, SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True))
    return outs, llm.engine.runner.logits_log


@pytest.mark.parametrize("name", sorted(tq.PRESETS))
def test_tiny_llama_with_turboquant_cache(name):
    base_outs, base_logits = _generate("auto")
    outs, logits = _generate(name)
    assert all(len(o.outputs[0].token_ids) == 8 for o in outs)
    # first sampled step (prefill logits) stays close to the bf16-cache model
    a, b = logits[0].flatten(), base_logits[0].flatten()
    cos = torch.nn.functional.cosine_similarity(a, b, dim=0).item()
    assert cos > (0.99 if name in ("turboquant_k8v4", "fp8", "fp8_e4m3") else 0.95), cos
    assert not math.isnan(cos)


def test_contract_names_turboquant_for_dense_only():
    from vllm_musa_b200.config import EngineConfig
    from vllm_musa_b200.plan import contract as C
    cfg = tiny_llama()
    cfg.kv_cache_dtype = "turboquant_4bit_nc"
    ec = EngineConfig(model=cfg, device="cuda")
    c = C.resolve(ec)
    assert c.supports(C.Feature.TURBOQUANT_KV)
    C.validate(c)
    cfg.kv_cache_dtype = "fp4_magic"
    with pytest.raises(ValueError):
        C.validate(C.resolve(EngineConfig(model=cfg, device="cuda")))
