"""Gated DeltaNet kernels on B200 vs the fp32 PyTorch token loops, and a tiny Qwen3-Next
model through the engine on the GPU (eager vs CUDA graphs, and vs the fp32 CPU engine)."""
import pytest
import torch

pytestmark = pytest.mark.gpu

from vllm_musa_b200 import ops
from vllm_musa_b200.ops import _ext
from vllm_musa_b200.ops import gdn


@pytest.fixture(autouse=True)
def _errs():
    yield
    torch.cuda.synchronize()
    _ext.check_device_errors()


def _batch(q_lens, hist, g):
    """cu_q, seq_lens for requests with ``q_lens`` new tokens after ``hist`` earlier ones."""
    cu = torch.tensor([0] + list(torch.tensor(q_lens).cumsum(0)), dtype=torch.int32)
    seq = torch.tensor([q + h for q, h in zip(q_lens, hist)], dtype=torch.int32)
    slots = torch.randperm(8, generator=g)[:len(q_lens)].to(torch.int32)
    return cu, seq, slots


@pytest.mark.parametrize("C", [256, 1024 + 128])
def test_causal_conv1d(C):
    g = torch.Generator().manual_seed(C)
    q_lens, hist = [1, 1, 7, 40, 1], [5, 0, 0, 9, 2]
    cu, seq, slots = _batch(q_lens, hist, g)
    T = int(cu[-1])
    x = torch.randn(T, C + 64, generator=g).to(torch.bfloat16)  # z channels trail
    w = (torch.randn(C, 4, generator=g) * 0.5).to(torch.bfloat16)
    state = torch.randn(8, C, 3, generator=g).to(torch.bfloat16)
    ref_state = state.clone()
    ref = gdn.causal_conv1d(x, w, ref_state, cu, seq, slots)
    st = state.cuda()
    out = gdn.causal_conv1d(x.cuda(), w.cuda(), st, cu.cuda(), seq.cuda(), slots.cuda())
    torch.testing.assert_close(out.cpu().float(), ref.float(), rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(st.cpu().float(), ref_state.float(), rtol=0, atol=0)


@pytest.mark.parametrize("Hk,Hv", [(1, 2), (2, 4), (4, 4)])
def test_gdn_recurrent(Hk, Hv):
    g = torch.Generator().manual_seed(Hk * 10 + Hv)
    q_lens, hist = [1, 3, 1, 37, 20], [4, 0, 0, 2, 0]
    cu, seq, slots = _batch(q_lens, hist, g)
    T = int(cu[-1])
    qkv = torch.randn(T, (2 * Hk + Hv) * 128, generator=g).to(torch.bfloat16)
    ba = torch.randn(T, 2 * Hv, generator=g).to(torch.bfloat16)
    A_log = torch.log(torch.linspace(1, 16, Hv))
    dt_bias = torch.randn(Hv, generator=g) * 0.5
    state = torch.randn(8, Hv, 128, 128, generator=g) * 0.05
    ref_state = state.clone()
    ref = gdn.gdn_recurrent(qkv, ba, A_log, dt_bias, ref_state, cu, seq, slots, Hk, Hv)
    st = state.cuda()
    out = gdn.gdn_recurrent(qkv.cuda(), ba.cuda(), A_log.cuda(), dt_bias.cuda(), st, cu.cuda(),
                            seq.cuda(), slots.cuda(), Hk, Hv)
    torch.testing.assert_close(out.cpu().float(), ref.float(), rtol=3e-2, atol=3e-2)
    torch.testing.assert_close(st.cpu(), ref_state, rtol=2e-3, atol=2e-3)


@pytest.mark.parametrize("Hk,Hv", [(1, 2), (16, 32)])
def test_gdn_decode_single_token(Hk, Hv):
    """Decode rows (one new token each, some without history) through the single-token kernel
    against the fp32 PyTorch recurrence."""
    g = torch.Generator().manual_seed(5 + Hv)
    R = 37
    q_lens, hist = [1] * R, [(r * 7) % 5 for r in range(R)]
    cu, seq, _ = _batch(q_lens, hist, g)
    slots = torch.randperm(64, generator=g)[:R].to(torch.int32)
    T = int(cu[-1])
    qkv = torch.randn(T, (2 * Hk + Hv) * 128, generator=g).to(torch.bfloat16)
    ba = torch.randn(T, 2 * Hv, generator=g).to(torch.bfloat16)
    A_log = torch.log(torch.linspace(1, 16, Hv))
    dt_bias = torch.randn(Hv, generator=g) * 0.5
    nslots = 64
    state = torch.randn(nslots, Hv, 128, 128, generator=g) * 0.05
    ref_state = state.clone()
    ref = gdn.gdn_recurrent(qkv, ba, A_log, dt_bias, ref_state, cu, seq, slots, Hk, Hv)
    st = state.cuda()
    out = gdn.gdn_recurrent(qkv.cuda(), ba.cuda(), A_log.cuda(), dt_bias.cuda(), st, cu.cuda(),
                            seq.cuda(), slots.cuda(), Hk, Hv, single_token=True)
    torch.testing.assert_close(out.cpu().float(), ref.float(), rtol=3e-2, atol=3e-2)
    torch.testing.assert_close(st.cpu(), ref_state, rtol=2e-3, atol=2e-3)


def test_sigmoid_gate_and_gated_norm_strided():
    g = torch.Generator().manual_seed(7)
    T, W = 37, 512
    buf = torch.randn(T, 3 * W, generator=g).to(torch.bfloat16)
    out = torch.randn(T, W, generator=g).to(torch.bfloat16)
    ref = gdn.sigmoid_gate(out.clone(), buf[:, 2 * W:])
    dev = out.cuda()
    gdn.sigmoid_gate(dev, buf.cuda()[:, 2 * W:])
    torch.testing.assert_close(dev.cpu().float(), ref.float(), rtol=1e-2, atol=1e-2)
    x = torch.randn(T, W, generator=g).to(torch.bfloat16)
    w = torch.rand(128, generator=g).to(torch.bfloat16)
    ref = ops.rms_norm_gated(x, buf[:, W:2 * W], w, 128, 1e-6)
    got = ops.rms_norm_gated(x.cuda(), buf.cuda()[:, W:2 * W], w.cuda(), 128, 1e-6)
    torch.testing.assert_close(got.cpu().float(), ref.float(), rtol=2e-2, atol=2e-2)


def _tiny_next(dtype):
    from vllm_musa_b200.config import ModelConfig
    return ModelConfig(arch="qwen3_next", vocab_size=2048, hidden_size=256, num_layers=4,
                       num_heads=4, num_kv_heads=2, head_dim=128, intermediate_size=512,
                       rms_norm_eps=1e-6, rope_theta=1e4, max_position=1024, qk_norm=True,
                       num_experts=16, num_experts_per_tok=2, moe_intermediate_size=128,
                       shared_expert_intermediate_size=128, full_attention_interval=4,
                       linear_num_key_heads=2, linear_num_value_heads=4,
                       linear_key_head_dim=128, linear_value_head_dim=128,
                       partial_rotary_factor=0.25, attn_output_gate=True, dtype=dtype,
                       name="tiny-next-gpu")


def test_tiny_qwen3_next_engine_graph_vs_eager():
    from vllm_musa_b200 import LLM, SamplingParams
    cfg = _tiny_next(torch.bfloat16)
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, 2048, (n,), generator=g).tolist() for n in (5, 77, 200)]
    sp = SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True)
    outs = {}
    for eager in (True, False):
        llm = LLM(cfg, block_size=64, seed=0, num_gpu_blocks=64, max_model_len=512,
                  max_num_seqs=8, max_num_batched_tokens=128, enforce_eager=eager,
                  cuda_graph_sizes=[1, 2, 4, 8])
        outs[eager] = [o.outputs[0].token_ids for o in llm.generate(prompts, sp)]
        llm.shutdown()
    assert outs[True] == outs[False]


@pytest.mark.parametrize("lens,ctx", [([64], [0]), ([200, 1, 77], [0, 9, 130]),
                                      ([1000, 65], [64, 0])])
def test_gdn_chunked_matches_recurrent(lens, ctx):
    """Chunked prefill kernels (parallel chunk prep + tensor-core chunk scan) against the fp32
    PyTorch token recurrence on CPU (the oracle) and against the token-recurrent kernel:
    outputs and the carried state."""
    from vllm_musa_b200.ops import gdn
    Hk, Hv = 2, 4
    T = sum(lens)
    g = torch.Generator().manual_seed(3)
    qkv = torch.randn(T, 2 * Hk * 128 + Hv * 128, generator=g).to(torch.bfloat16).cuda()
    ba = torch.randn(T, 2 * Hv, generator=g).to(torch.bfloat16).cuda()
    A_log = (torch.randn(Hv, generator=g) * 0.5).cuda()
    dt_bias = (torch.randn(Hv, generator=g) * 0.5).cuda()
    cu = torch.tensor([0] + list(torch.cumsum(torch.tensor(lens), 0)), dtype=torch.int32).cuda()
    sl = torch.tensor([c + n for c, n in zip(ctx, lens)], dtype=torch.int32).cuda()
    R = len(lens)
    slots = torch.arange(R, dtype=torch.int32).flip(0).contiguous().cuda()
    st0 = (torch.randn(R, Hv, 128, 128, generator=g) * 0.05).cuda()
    s_ref, s_got = st0.clone(), st0.clone()
    ref = gdn.gdn_recurrent(qkv, ba, A_log, dt_bias, s_ref, cu, sl, slots, Hk, Hv)
    got = gdn.gdn_chunked(qkv, ba, A_log, dt_bias, s_got, cu, sl, slots, Hk, Hv)
    torch.cuda.synchronize()
    from vllm_musa_b200.ops import _ext
    _ext.check_device_errors()
    torch.testing.assert_close(got.float(), ref.float(), rtol=3e-2, atol=3e-2)
    torch.testing.assert_close(s_got, s_ref, rtol=3e-2, atol=3e-2)
    s_cpu = st0.cpu()
    oracle = gdn.gdn_recurrent(qkv.cpu(), ba.cpu(), A_log.cpu(), dt_bias.cpu(), s_cpu, cu.cpu(),
                               sl.cpu(), slots.cpu(), Hk, Hv)
    torch.testing.assert_close(got.cpu().float(), oracle.float(), rtol=3e-2, atol=3e-2)
    torch.testing.assert_close(s_got.cpu(), s_cpu, rtol=3e-2, atol=3e-2)
