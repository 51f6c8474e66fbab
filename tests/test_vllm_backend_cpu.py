"""The vLLM attention backend and platform hooks on CPU: vLLM's CommonAttentionMetadata for a
decodes-first batch goes through the builder, the KV-cache update and the forward, and the
output equals plain causal attention over each request's whole sequence; the platform selects
the backend for bf16 decoder attention and keeps vLLM's choice otherwise."""
import math
from types import SimpleNamespace

import pytest
import torch

pytest.importorskip("vllm.v1.attention.backend")

from vllm.v1.attention.backend import CommonAttentionMetadata  # noqa: E402

from vllm_musa_b200 import vllm_backend as vb  # noqa: E402


def _vllm_config(Hq, Hkv, D, max_len=256, max_seqs=8):
    mc = SimpleNamespace(get_num_kv_heads=lambda pc: Hkv, get_num_attention_heads=lambda pc: Hq,
                         get_head_size=lambda: D, max_model_len=max_len)
    return SimpleNamespace(model_config=mc, parallel_config=SimpleNamespace(
        decode_context_parallel_size=1), scheduler_config=SimpleNamespace(max_num_seqs=max_seqs),
        speculative_config=None)


def _ref_attention(q, ks, vs, scale):
    """q [n, Hq, D] of the last n positions of a sequence with keys / values ks, vs [L, Hkv, D]."""
    n, Hq, D = q.shape
    L, Hkv = ks.shape[0], ks.shape[1]
    rep = Hq // Hkv
    k = ks.repeat_interleave(rep, 1)
    v = vs.repeat_interleave(rep, 1)
    s = torch.einsum("nhd,lhd->hnl", q, k) * scale
    pos = torch.arange(L - n, L)
    mask = torch.arange(L)[None, :] > pos[:, None]
    s = s.masked_fill(mask[None], float("-inf"))
    return torch.einsum("hnl,lhd->nhd", s.softmax(-1), v)


def test_backend_builder_kv_update_and_forward_match_reference():
    torch.manual_seed(0)
    Hq, Hkv, D, bs = 4, 2, 64, 16
    ctx = [30, 5, 0]   # tokens already cached per request
    new = [1, 1, 20]   # decodes first, then one prefill chunk
    R = len(ctx)
    total = [c + n for c, n in zip(ctx, new)]
    blocks_per = [(t + bs - 1) // bs for t in total]
    nb = sum(blocks_per) + 2
    perm = torch.randperm(nb)
    bt = torch.zeros(R, max(blocks_per), dtype=torch.int32)
    used = 0
    for r in range(R):
        bt[r, :blocks_per[r]] = perm[used:used + blocks_per[r]].to(torch.int32)
        used += blocks_per[r]
    kv_cache = torch.zeros(vb.B200AttentionBackend.get_kv_cache_shape(nb, bs, Hkv, D))
    # the full sequences' keys / values; the cached part is written up front
    K = [torch.randn(t, Hkv, D) for t in total]
    V = [torch.randn(t, Hkv, D) for t in total]
    impl = vb.B200AttentionImpl(Hq, D, 1 / math.sqrt(D), Hkv)

    def slots(r, a, b):
        return torch.tensor([int(bt[r, p // bs]) * bs + p % bs for p in range(a, b)],
                            dtype=torch.int64)
    for r in range(R):
        if ctx[r]:
            impl.do_kv_cache_update(None, K[r][:ctx[r]], V[r][:ctx[r]], kv_cache,
                                    slots(r, 0, ctx[r]))
    T = sum(new)
    q = torch.randn(T, Hq, D)
    key = torch.cat([K[r][ctx[r]:] for r in range(R)])
    val = torch.cat([V[r][ctx[r]:] for r in range(R)])
    slot_mapping = torch.cat([slots(r, ctx[r], total[r]) for r in range(R)])
    qsl = torch.tensor([0] + list(torch.tensor(new).cumsum(0)), dtype=torch.int32)
    cm = CommonAttentionMetadata(
        query_start_loc=qsl, query_start_loc_cpu=qsl, seq_lens=torch.tensor(total, dtype=torch.int32),
        num_reqs=R, num_actual_tokens=T, max_query_len=max(new), max_seq_len=max(total),
        block_table_tensor=bt, slot_mapping=slot_mapping)
    builder = vb.B200AttentionMetadataBuilder(None, ["l0"], _vllm_config(Hq, Hkv, D),
                                              torch.device("cpu"))
    assert builder.reorder_batch_threshold == 1
    meta = builder.build(0, cm)
    assert (meta.num_decodes, meta.num_prefills) == (2, 1)
    impl.do_kv_cache_update(None, key, val, kv_cache, slot_mapping)
    out = torch.empty(T, Hq, D)
    impl.forward(None, q, key, val, kv_cache, meta, out)
    o0 = 0
    for r in range(R):
        want = _ref_attention(q[o0:o0 + new[r]], K[r], V[r], 1 / math.sqrt(D))
        torch.testing.assert_close(out[o0:o0 + new[r]], want, rtol=1e-4, atol=1e-4)
        o0 += new[r]
    # the memory-profiling run passes no metadata
    assert impl.forward(None, q, key, val, kv_cache, None, out.fill_(1.0)).abs().sum() == 0


def test_platform_selects_backend_and_communicator():
    from vllm.v1.attention.backend import AttentionType
    from vllm.v1.attention.selector import AttentionSelectorConfig
    from vllm_musa_b200.platform import B200Platform
    cfg = AttentionSelectorConfig(head_size=128, dtype=torch.bfloat16, kv_cache_dtype="auto",
                                  block_size=64)
    assert vb.serves(cfg)
    path = B200Platform.get_attn_backend_cls(None, cfg)
    assert path.endswith("vllm_backend.B200AttentionBackend")
    from vllm.v1.attention.backends.registry import AttentionBackendEnum
    assert AttentionBackendEnum.CUSTOM.get_path() == path
    for other in (cfg._replace(use_mla=True), cfg._replace(head_size=96),
                  cfg._replace(kv_cache_dtype="fp8"), cfg._replace(dtype=torch.float16),
                  cfg._replace(attn_type=AttentionType.ENCODER_ONLY)):
        assert not vb.serves(other)
    assert B200Platform.get_device_communicator_cls().endswith("vllm_comm.B200Communicator")
    import importlib
    mod, cls = B200Platform.get_device_communicator_cls().rsplit(".", 1)
    assert issubclass(getattr(importlib.import_module(mod), cls),
                      importlib.import_module(
                          "vllm.distributed.device_communicators.cuda_communicator"
                      ).CudaCommunicator)


def test_quant_fp8_override_matches_vllm_native():
    """The QuantFP8 OOT class quantises 1x128 groups like vLLM's native path and defers every
    other configuration to vLLM."""
    from vllm.config import DeviceConfig, VllmConfig, set_current_vllm_config
    from vllm.model_executor.layers.quantization.utils.quant_utils import GroupShape
    from vllm_musa_b200.plugin import make_quant_fp8_class
    cls = make_quant_fp8_class()
    with set_current_vllm_config(VllmConfig(device_config=DeviceConfig(device="cpu"))):
        op = cls(static=False, group_shape=GroupShape(1, 128))
        per_token = cls(static=False, group_shape=GroupShape.PER_TOKEN)
    op.use_ue8m0 = False
    torch.manual_seed(0)
    x = (torch.randn(5, 512) * 3).to(torch.bfloat16)
    assert op._b200_serves(x, None)
    q, s = op.forward_oot(x)
    qn, sn = op.forward_native(x)
    torch.testing.assert_close(s.float(), sn.float().reshape(s.shape), rtol=1e-3, atol=1e-6)
    deq = q.float().view(5, 4, 128) * s.unsqueeze(-1)
    deqn = qn.float().view(5, 4, 128) * sn.float().reshape(5, 4, 1)
    assert (deq - deqn).abs().max() <= 0.0625 * x.float().abs().max()
    assert not per_token._b200_serves(x, None)


def test_platform_selects_worker_class():
    from vllm_musa_b200.platform import B200Platform
    par = SimpleNamespace(worker_cls="auto")
    cfg = SimpleNamespace(parallel_config=par, cache_config=None, compilation_config=None)
    try:
        B200Platform.check_and_update_config(cfg)
    except Exception:
        pass  # vLLM's own checks need a full config; the worker choice happens first
    assert par.worker_cls == "vllm_musa_b200.vllm_worker.B200Worker"
    from vllm.v1.worker.gpu_worker import Worker
    from vllm_musa_b200.vllm_worker import B200Worker
    assert issubclass(B200Worker, Worker)
