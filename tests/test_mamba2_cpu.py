"""Mamba2 on CPU: the scan op against a direct restatement of the SSD recurrence, and a tiny
random Mamba2 model through the engine (chunked prefill + decode with per-request state
slots) against a whole-sequence reference forward written from the published layer math."""
import math

import pytest
import torch
import torch.nn.functional as F

from vllm_musa_b200 import LLM, SamplingParams
from vllm_musa_b200.config import ModelConfig
from vllm_musa_b200.models.weights import dummy_weights
from vllm_musa_b200.ops import mamba as M


def tiny_mamba2(G=2):
    return ModelConfig.from_hf({"architectures": ["Mamba2ForCausalLM"], "model_type": "mamba2",
                                "vocab_size": 512, "hidden_size": 128, "num_hidden_layers": 3,
                                "state_size": 64, "expand": 2, "head_dim": 32, "n_groups": G,
                                "conv_kernel": 4, "layer_norm_epsilon": 1e-5,
                                "tie_word_embeddings": True})


def test_config_from_hf():
    c = tiny_mamba2()
    assert c.arch == "mamba2" and c.mamba_num_heads == 8 and c.ssm_state_size == 64
    assert c.mamba_dt_max == math.inf


def test_scan_matches_direct_recurrence_and_resumes_state():
    g = torch.Generator().manual_seed(0)
    H, G, P, N, T = 4, 2, 16, 16, 11
    xbc = torch.randn(T, H * P + 2 * G * N, generator=g)
    dt = torch.randn(T, H, generator=g)
    dtb, Alog, D = torch.randn(H, generator=g), torch.rand(H, generator=g), torch.randn(H, generator=g)
    st = torch.zeros(2, H, P, N)
    cu = torch.tensor([0, T], dtype=torch.int32)
    y = M.mamba2_scan(xbc, H * P, H * P + G * N, dt, dtb, Alog, D, st, cu,
                      torch.tensor([T], dtype=torch.int32), torch.tensor([1], dtype=torch.int32),
                      H, G, P, N)
    # direct: one head at a time
    for h in range(H):
        gg = h // (H // G)
        S = torch.zeros(P, N)
        for t in range(T):
            d = F.softplus(dt[t, h] + dtb[h])
            x = xbc[t, h * P:(h + 1) * P]
            B = xbc[t, H * P + gg * N:H * P + (gg + 1) * N]
            C = xbc[t, H * P + G * N + gg * N:H * P + G * N + (gg + 1) * N]
            S = torch.exp(-d * torch.exp(Alog[h])) * S + d * torch.outer(x, B)
            torch.testing.assert_close(y[t, h * P:(h + 1) * P], S @ C + D[h] * x, rtol=1e-4,
                                       atol=1e-4)
    # two chunks with a carried state equal one pass
    st2 = torch.zeros(2, H, P, N)
    y2 = torch.cat([M.mamba2_scan(xbc[a:b], H * P, H * P + G * N, dt[a:b], dtb, Alog, D, st2,
                                  torch.tensor([0, b - a], dtype=torch.int32),
                                  torch.tensor([b], dtype=torch.int32),
                                  torch.tensor([1], dtype=torch.int32), H, G, P, N)
                    for a, b in ((0, 4), (4, T))])
    torch.testing.assert_close(y2, y, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(st2, st)


class Mamba2Reference:
    """Whole-sequence fp32 forward from HF parameter names (no engine code)."""

    def __init__(self, cfg, W):
        self.c, self.W = cfg, {k: v.float() for k, v in W.items()}

    def logits(self, ids):
        c, W = self.c, self.W
        H, P, G, N = c.mamba_num_heads, c.mamba_head_dim, c.mamba_n_groups, c.ssm_state_size
        dI = H * P
        eps = c.rms_norm_eps
        rms = lambda v, w: v * torch.rsqrt(v.pow(2).mean(-1, keepdim=True) + eps) * w
        h = W["backbone.embeddings.weight"][torch.tensor(ids)]
        T = h.shape[0]
        for i in range(c.num_layers):
            p = f"backbone.layers.{i}.mixer."
            zx = rms(h, W[f"backbone.layers.{i}.norm.weight"]) @ W[p + "in_proj.weight"].T
            z, xBC, dt = zx[:, :dI], zx[:, dI:2 * dI + 2 * G * N], zx[:, 2 * dI + 2 * G * N:]
            conv = F.conv1d(F.pad(xBC.T, (3, 0)).unsqueeze(0), W[p + "conv1d.weight"],
                            W[p + "conv1d.bias"], groups=xBC.shape[1])[0].T
            xBC = F.silu(conv)
            x = xBC[:, :dI].view(T, H, P)
            B = xBC[:, dI:dI + G * N].view(T, G, N).repeat_interleave(H // G, 1)
            C = xBC[:, dI + G * N:].view(T, G, N).repeat_interleave(H // G, 1)
            d = F.softplus(dt + W[p + "dt_bias"])
            A = -torch.exp(W[p + "A_log"])
            S = torch.zeros(H, P, N)
            ys = []
            for t in range(T):
                S = torch.exp(d[t] * A).view(H, 1, 1) * S + \
                    (d[t].view(H, 1) * x[t]).unsqueeze(-1) * B[t].unsqueeze(1)
                ys.append((S * C[t].unsqueeze(1)).sum(-1) + W[p + "D"].view(H, 1) * x[t])
            y = torch.stack(ys).reshape(T, dI) * F.silu(z)
            y = y.view(T, G, dI // G)
            y = (y * torch.rsqrt(y.pow(2).mean(-1, keepdim=True) + eps)).reshape(T, dI)
            h = h + (y * W[p + "norm.weight"]) @ W[p + "out_proj.weight"].T
        h = rms(h, W["backbone.norm_f.weight"])
        return h @ W["backbone.embeddings.weight"].T

    def greedy(self, ids, n):
        ids = list(ids)
        out = []
        for _ in range(n):
            t = int(self.logits(ids)[-1].argmax())
            out.append(t)
            ids.append(t)
        return out


@pytest.mark.parametrize("budget", [256, 24])
def test_tiny_mamba2_engine_matches_reference(budget):
    cfg = tiny_mamba2()
    cfg.dtype = torch.float32
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, 512, (n,), generator=g).tolist() for n in (5, 40, 17)]
    llm = LLM(cfg, device="cpu", block_size=16, seed=0, num_gpu_blocks=64, max_model_len=128,
              max_num_seqs=4, max_num_batched_tokens=budget)
    outs = llm.generate(prompts, SamplingParams(temperature=0.0, max_tokens=4, ignore_eos=True))
    ref = Mamba2Reference(cfg, dict(dummy_weights(cfg, seed=0, std=0.02)))
    for i, p in enumerate(prompts):
        assert outs[i].outputs[0].token_ids == ref.greedy(p, 4), f"request {i} diverged"


def _ssd_case(H, G, P, N, lens, seed):
    g = torch.Generator().manual_seed(seed)
    T = sum(n for _, n in lens)
    xbc = (torch.randn(T, H * P + 2 * G * N, generator=g) * 0.5).to(torch.bfloat16)
    dt = torch.randn(T, H, generator=g).to(torch.bfloat16)
    dtb = torch.randn(H, generator=g) * 0.5
    Alog = torch.rand(H, generator=g) * 2
    D = torch.randn(H, generator=g)
    st = torch.randn(6, H, P, N, generator=g) * 0.1
    cu = torch.tensor([0] + list(torch.cumsum(torch.tensor([n for _, n in lens]), 0)),
                      dtype=torch.int32)
    sl = torch.tensor([c + n for c, n in lens], dtype=torch.int32)
    slots = torch.tensor([3, 0, 5, 1, 2][:len(lens)], dtype=torch.int32)
    return xbc, dt, dtb, Alog, D, st, cu, sl, slots


@pytest.mark.parametrize("H,G,P,N", [(4, 2, 32, 64), (2, 1, 64, 128)])
def test_chunked_ssd_matches_token_recurrence(H, G, P, N):
    """The matrix form the chunked kernels implement (intra-chunk decayed C B^T x, the chunk-
    start state through C, chunk states carried across chunk borders) equals the token loop,
    with and without a cached state, over partial and multi-chunk requests."""
    from vllm_musa_b200.ops import mamba as M
    lens = [(0, 1), (0, 150), (20, 64), (7, 65)]
    xbc, dt, dtb, Alog, D, st, cu, sl, slots = _ssd_case(H, G, P, N, lens, H * N)
    st_a, st_b = st.clone(), st.clone()
    ref = M.mamba2_scan(xbc, H * P, H * P + G * N, dt, dtb, Alog, D, st_a, cu, sl, slots,
                        H, G, P, N, 0.0, 10.0)
    got = M.mamba2_chunked(xbc, H * P, H * P + G * N, dt, dtb, Alog, D, st_b, cu, sl, slots,
                           H, G, P, N, 0.0, 10.0)
    torch.testing.assert_close(got.float(), ref.float(), rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(st_b, st_a, rtol=1e-4, atol=1e-4)
    # fp32 check of the algorithm itself (no bf16 output rounding)
    st_c = st.clone()
    y = M.mamba2_chunked_ref(xbc, H * P, H * P + G * N, dt, dtb, Alog, D, st_c, cu, sl, slots,
                             H, G, P, N, 0.0, 10.0)
    st_d = st.clone()
    A = -torch.exp(Alog)
    rep = H // G
    for r in range(len(lens)):
        a0, b0 = int(cu[r]), int(cu[r + 1])
        S = st_d[int(slots[r])].clone() if lens[r][0] > 0 else torch.zeros(H, P, N)
        for t in range(a0, b0):
            x = xbc[t, :H * P].float().view(H, P)
            Bt = xbc[t, H * P:H * P + G * N].float().view(G, N).repeat_interleave(rep, 0)
            Ct = xbc[t, H * P + G * N:].float().view(G, N).repeat_interleave(rep, 0)
            d = torch.nn.functional.softplus(dt[t].float() + dtb).clamp(0.0, 10.0)
            S = S * torch.exp(d * A).view(H, 1, 1) + (d.view(H, 1) * x)[..., None] * Bt[:, None]
            want = (S * Ct[:, None]).sum(-1) + D.view(H, 1) * x
            torch.testing.assert_close(y[t].view(H, P), want, rtol=1e-4, atol=1e-4)
        st_d[int(slots[r])] = S
    torch.testing.assert_close(st_c, st_d, rtol=1e-4, atol=1e-4)
