"""MoE kernels on B200 vs the PyTorch reference: routers, expert-sorted grouped GEMMs,
combine, and a tiny Qwen3-MoE model through the engine (eager and CUDA graphs)."""
import pytest
import torch

pytestmark = pytest.mark.gpu

from vllm_musa_b200 import ops
from vllm_musa_b200.ops import _ext
from vllm_musa_b200.ops import moe as moe_ops


@pytest.fixture(autouse=True)
def _errs():
    yield
    torch.cuda.synchronize()
    _ext.check_device_errors()


@pytest.mark.parametrize("T,E,k", [(1, 128, 8), (300, 128, 8), (33, 512, 10), (5, 64, 6)])
def test_topk_softmax(T, E, k):
    logits = torch.randn(T, E, generator=torch.Generator().manual_seed(T)) * 2
    ids, w = moe_ops.topk_softmax(logits.cuda(), k, True)
    rids, rw = moe_ops.topk_softmax(logits, k, True)
    assert torch.equal(ids.cpu().long().sort(-1).values, rids.long().sort(-1).values)
    torch.testing.assert_close(w.cpu().sort(-1).values, rw.sort(-1).values, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("T,E,k,ng,tg", [(64, 256, 8, 8, 4), (3, 64, 4, 4, 2)])
def test_grouped_topk(T, E, k, ng, tg):
    g = torch.Generator().manual_seed(9)
    logits = torch.randn(T, E, generator=g)
    bias = torch.randn(E, generator=g) * 0.1
    ids, w = moe_ops.grouped_topk(logits.cuda(), k, ng, tg, bias.cuda(), True, True, 2.5)
    rids, rw = moe_ops.grouped_topk(logits, k, ng, tg, bias, True, True, 2.5)
    assert torch.equal(ids.cpu().long().sort(-1).values, rids.long().sort(-1).values)
    torch.testing.assert_close(w.cpu().sort(-1).values, rw.sort(-1).values, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("E,N,K,tiles", [(8, 256, 128, 3), (4, 512, 256, 5), (16, 128, 512, 16)])
def test_grouped_gemm(mode, E, N, K, tiles):
    """Grouped GEMM alone: tile t (128 rows) multiplies expert tile_expert[t]'s weights."""
    g = torch.Generator().manual_seed(E * N + K + mode)
    max_rows = (tiles + 2) * 128  # trailing tiles beyond num_tiles are never written
    A = (torch.randn(max_rows, K, generator=g) * 0.5).to(torch.bfloat16)
    B = (torch.randn(E * N, K, generator=g) * 0.05).to(torch.bfloat16)
    te = torch.randint(0, E, (max_rows // 128,), generator=g, dtype=torch.int32)
    nt = torch.tensor([tiles], dtype=torch.int32)
    width = N // 2 if mode == 1 else N
    C = torch.zeros(max_rows, width, dtype=torch.bfloat16, device="cuda")
    torch.ops.b200.gemm_grouped_bf16(A.cuda(), B.cuda(), C, te.cuda(), nt.cuda(), E, mode, 0)
    torch.cuda.synchronize()
    for t in range(tiles):
        a = A[t * 128:(t + 1) * 128].float()
        w = B[int(te[t]) * N:(int(te[t]) + 1) * N].float()
        y = a @ w.t()
        if mode == 1:  # interleaved groups of 8 gate rows then 8 up rows
            y = y.view(128, N // 16, 2, 8)
            y = (torch.nn.functional.silu(y[:, :, 0]) * y[:, :, 1]).reshape(128, N // 2)
        torch.testing.assert_close(C[t * 128:(t + 1) * 128].float().cpu(), y, atol=3e-2, rtol=3e-2)


@pytest.mark.parametrize("T,E,k,H,I", [(1, 8, 2, 256, 128), (7, 128, 8, 512, 256),
                                        (300, 128, 8, 256, 128), (64, 16, 4, 1024, 512)])
def test_fused_moe(T, E, k, H, I):
    g = torch.Generator().manual_seed(T + E)
    x = (torch.randn(T, H, generator=g)).to(torch.bfloat16)
    gates = [torch.randn(I, H, generator=g) * 0.05 for _ in range(E)]
    ups = [torch.randn(I, H, generator=g) * 0.05 for _ in range(E)]
    w_gu = torch.cat([ops.interleave_gate_up(gates[e], ups[e]) for e in range(E)]).to(torch.bfloat16)
    w_dn = (torch.randn(E * H, I, generator=g) * 0.05).to(torch.bfloat16)
    ids, w = moe_ops.topk_softmax(torch.randn(T, E, generator=g), k)
    shared = (torch.randn(T, H, generator=g) * 0.1).to(torch.bfloat16)
    # router-GEMM-shaped logits whose column E is the shared expert's gate
    logits = torch.randn(T, E + 8, generator=g)
    gate = logits[:, E:E + 1] if T % 2 else None
    ref = moe_ops.fused_moe(x, w_gu, w_dn, ids, w, E, shared, shared_gate=gate)
    lg = logits.cuda()
    out = moe_ops.fused_moe(x.cuda(), w_gu.cuda(), w_dn.cuda(), ids.cuda(), w.cuda(), E,
                            shared.cuda(), shared_gate=lg[:, E:E + 1] if T % 2 else None)
    torch.testing.assert_close(out.cpu().float(), ref.float(), rtol=3e-2, atol=3e-2)


@pytest.mark.parametrize("T,E,k,H,I,e0", [(1, 128, 8, 2048, 768, 0), (5, 64, 8, 1024, 256, 16),
                                           (16, 32, 4, 512, 512, 0)])
def test_moe_gemv_matches_grouped_and_reference(T, E, k, H, I, e0, monkeypatch):
    """Small-batch dispatch: the per-pair GEMV path and the grouped-GEMM path give the same
    combined output as the fp32 reference, also with expert parallelism (this rank holds
    experts [e0, e0 + E) of 2E; the rest contribute nothing here)."""
    g = torch.Generator().manual_seed(T * 7 + E)
    E_all = 2 * E if e0 else E
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    w_gu = (torch.randn(E * 2 * I, H, generator=g) * 0.05).to(torch.bfloat16)
    w_dn = (torch.randn(E * H, I, generator=g) * 0.05).to(torch.bfloat16)
    ids, w = moe_ops.topk_softmax(torch.randn(T, E_all, generator=g), k)
    shared = (torch.randn(T, H, generator=g) * 0.1).to(torch.bfloat16)
    ref = moe_ops.fused_moe(x, w_gu, w_dn, ids, w, E, shared, expert_offset=e0)
    outs = {}
    for name, limit in (("gemv", 1 << 20), ("grouped", 0)):
        monkeypatch.setenv("B200_MOE_GEMV_MAX_PAIRS", str(limit))
        assert moe_ops.use_gemv(T, k, H, I) == (name == "gemv")
        outs[name] = moe_ops.fused_moe(x.cuda(), w_gu.cuda(), w_dn.cuda(), ids.cuda(), w.cuda(),
                                       E, shared.cuda(), expert_offset=e0).cpu().float()
    torch.cuda.synchronize()
    torch.testing.assert_close(outs["gemv"], ref.float(), rtol=3e-2, atol=3e-2)
    torch.testing.assert_close(outs["gemv"], outs["grouped"], rtol=3e-2, atol=3e-2)


def test_tiny_moe_engine_graph_vs_eager():
    from vllm_musa_b200 import LLM, SamplingParams
    from vllm_musa_b200.config import ModelConfig
    cfg = ModelConfig(arch="qwen3_moe", vocab_size=2048, hidden_size=512, num_layers=2,
                      num_heads=8, num_kv_heads=2, head_dim=64, intermediate_size=1024,
                      rms_norm_eps=1e-6, rope_theta=1e4, max_position=1024, qk_norm=True,
                      num_experts=32, num_experts_per_tok=4, moe_intermediate_size=256,
                      shared_expert_intermediate_size=256, name="tiny-moe-gpu")
    g = torch.Generator().manual_seed(4)
    prompts = [torch.randint(0, 2048, (n,), generator=g).tolist() for n in (5, 77, 200)]
    sp = SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True)
    outs = {}
    for eager in (True, False):
        llm = LLM(cfg, block_size=64, seed=0, num_gpu_blocks=64, max_model_len=512,
                  max_num_seqs=8, max_num_batched_tokens=512, enforce_eager=eager,
                  cuda_graph_sizes=[1, 2, 4, 8])
        outs[eager] = [o.outputs[0].token_ids for o in llm.generate(prompts, sp)]
        llm.shutdown()
    assert outs[True] == outs[False]
