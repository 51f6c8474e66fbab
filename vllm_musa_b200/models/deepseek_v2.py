"""DeepSeek-V2 / V3 / V3.2 family: multi-head latent attention (optionally with the V3.2
lightning-indexer sparse attention), sigmoid grouped-top-k MoE with shared experts, block-FP8
linears.

Per layer on each tensor-parallel rank (Hl = heads / tp):
    a      = x W_a                 W_a = [q_a | kv_a | idx_k | idx_w] (each padded to 128 rows)
    q      = RMSNorm(q_a) W_qb     (+ the indexer's query rows W_iq in the same GEMM)
    prep   : q_pe RoPE, c_kv RMSNorm + k_pe RoPE -> latent cache [slot] (576 wide)
    q_lat  = q_nope[h] . W_kb[h]   (absorbed key up-projection, 512 wide per head)
    sparse : indexer scores -> top-k positions per token (V3.2)
    o_lat  = MLA(q_lat | q_pe, cache, positions)                      (csrc/attention/mla.cu)
    o      = o_lat[h] . W_vb[h]^T -> o_proj -> fused all-reduce + residual + RMSNorm
    MLP    : dense SwiGLU (first_k_dense layers) or routed experts + shared experts.
FP8 checkpoints (``weight`` e4m3 + ``weight_scale_inv`` per 128 x 128 block) run on the
block-scaled tcgen05 GEMM (ops.fp8); bf16 weights are quantised at load when the config asks
for fp8 (random-init benchmarks).  Routed experts run as grouped FP8 GEMMs with SwiGLU + 1x128
re-quantisation between them (the silu_mul_fp8_quant kernel).

Reference counterparts: vllm_musa/v1/attention/backends/mla/common.py:202-774 (MLA impl:
_v_up_proj :182, forward_mqa :756), flashmla.py / flashmla_sparse.py (backends),
vllm_musa/model_executor/layers/fused_moe/fused_moe.py:824-1051 (DeepGEMM FP8 grouped experts),
fused_moe/router/grouped_topk_router.py:388 (grouped top-k), quantization/fp8.py:27-297.
"""
from __future__ import annotations

import math
import re
from collections import defaultdict
from typing import Iterable, Optional, Tuple

import torch

from .. import ops
from ..ops import fp8 as fp8_ops
from ..ops import mla as mla_ops
from ..ops import moe as moe_ops
from ..parallel.communicator import LocalCommunicator
from ..parallel.state import ParallelState
from .llama import shard_cols, shard_rows

_LAYER_RE = re.compile(r"model\.layers\.(\d+)\.(.+)")


class Lin:
    """One linear layer's weight on this rank: bf16 [N, K], or e4m3 [N, K] + fp32 block
    scales [ceil(N/128), ceil(K/128)]."""
    __slots__ = ("w", "s")

    def __init__(self, w, s=None):
        self.w, self.s = w, s

    @property
    def fp8(self):
        return self.s is not None

    def __call__(self, x, out=None):
        if self.s is not None:
            return fp8_ops.linear_fp8(x, self.w, self.s, out)
        return ops.linear(x, self.w, out=out)

    def quantized(self, q, sq, out=None):
        """fp8 layer on an input already quantised per token (1x128 e4m3 + scales)."""
        return fp8_ops.gemm_fp8(q, sq, self.w, self.s, out)


class _Layer:
    __slots__ = ("ln1", "ln2", "w_a", "q_a_norm", "kv_a_norm", "w_qb", "w_kb", "w_vb", "o", "idx_ln_w",
                 "idx_ln_b", "gu", "down", "router_w", "router_bias", "experts_gu", "experts_gu_s",
                 "experts_down", "experts_down_s", "shared_gu", "shared_down", "w4",
                 # multi-token-prediction layer only
                 "enorm", "hnorm", "eh_proj", "head_norm", "head")

    def __init__(self):
        for s in self.__slots__:
            setattr(self, s, None)


def _pad_rows(w: torch.Tensor, mult: int = 128) -> torch.Tensor:
    pad = (-w.shape[0]) % mult
    return torch.cat([w, w.new_zeros(pad, *w.shape[1:])]) if pad else w


def yarn_mscale(scale: float, mscale: float = 1.0) -> float:
    return 0.1 * mscale * math.log(scale) + 1.0 if scale > 1 else 1.0


class DeepseekV2ForCausalLM:
    def __init__(self, cfg, pstate: Optional[ParallelState] = None, comm=None, device="cuda"):
        self.cfg = cfg
        self.device = torch.device(device)
        self.dtype = cfg.dtype
        self.pstate = pstate or ParallelState()
        self.tp, self.rank = self.pstate.tp_size, self.pstate.tp_rank
        self.comm = comm or LocalCommunicator(self.device)
        if cfg.num_heads % self.tp:
            raise ValueError("num_heads must be divisible by tensor_parallel_size")
        self.hq = cfg.num_heads // self.tp
        self.nope, self.rope = cfg.qk_nope_head_dim, cfg.qk_rope_head_dim
        self.vdim, self.kv_lora, self.q_lora = cfg.v_head_dim, cfg.kv_lora_rank, cfg.q_lora_rank
        if self.kv_lora != 512 or self.rope != 64 or self.nope != 128:
            raise ValueError("MLA kernels are built for kv_lora 512, rope 64, nope 128")
        # block-FP8 GEMMs run on the GPU in bf16 models; other runs (CPU fp32) dequantise
        self.fp8 = cfg.quant in ("fp8_block", "w4afp8") and cfg.dtype == torch.bfloat16
        # W4AFP8: routed experts stay packed int4 (group-128 bf16 scales) on every device
        self.w4 = cfg.quant == "w4afp8"
        self.sparse = cfg.index_topk > 0
        self.idx_heads, self.idx_dim = cfg.index_n_heads, cfg.index_head_dim
        # fused A-projection row layout (every part padded to 128 rows)
        q_rows = self.q_lora if self.q_lora else cfg.num_heads * (self.nope + self.rope)
        self.a_parts = [("q", q_rows), ("kv", self.kv_lora + self.rope)]
        if self.sparse:
            self.a_parts += [("ik", self.idx_dim), ("iw", self.idx_heads)]
        self.a_off, o = {}, 0
        for name, n in self.a_parts:
            self.a_off[name] = o
            o += n + (-n) % 128
        self.E = cfg.num_experts
        self.topk = cfg.num_experts_per_tok
        self.ep = self.pstate.ep_size > 1
        if self.E and self.ep:
            self.E_local = self.E // self.pstate.ep_size
            self.e0 = self.pstate.ep_rank * self.E_local
        else:
            self.E_local, self.e0 = self.E, 0
        self.vocab_local = cfg.vocab_size // self.tp
        self.layers = [_Layer() for _ in range(cfg.num_layers)]
        self.embed = self.final_norm = self.lm_head = None
        if cfg.vocab_size % self.tp:
            raise ValueError("vocab_size must be divisible by tensor_parallel_size")
        # lm_head rows are vocab-sharded: rank r's logits start at token id r * V / tp (the
        # vocab-parallel sampler adds this offset to its candidates)
        self.vocab_start = self.rank * (cfg.vocab_size // self.tp)
        rs = cfg.rope_scaling or {}
        self.cos_sin = ops.build_cos_sin_cache(self.rope, cfg.max_position, cfg.rope_theta,
                                               self.device, scaling=cfg.rope_scaling)
        self.scale = (self.nope + self.rope) ** -0.5
        if rs.get("type", rs.get("rope_type")) == "yarn":
            m = yarn_mscale(rs["factor"], rs.get("mscale_all_dim", 0.0))
            self.scale *= m * m
        self._staging = defaultdict(dict)
        self._mla_ws = None
        self.dcp, self.kv_block_size = 1, 0  # decode context parallelism (enable_dcp)
        self._slots = None
        # DeepSeek multi-token prediction: checkpoint layer index num_layers (loaded if present)
        self.mtp: Optional[_Layer] = None
        self._mtp_staging: dict = {}

    # ------------------------------------------------------------------ weights
    def _to(self, t):
        return t.to(device=self.device, dtype=self.dtype).contiguous()

    def _lin(self, w: torch.Tensor, s: Optional[torch.Tensor] = None, quant: bool = True) -> Lin:
        """Place a (sharded) weight: keep checkpoint fp8, quantise bf16 when the model is fp8,
        else keep the compute dtype."""
        if s is not None and not self.fp8:
            w, s = fp8_ops.dequantize_weight_block(w, s.float()), None
        if s is not None:
            return Lin(w.to(self.device).contiguous(), s.float().to(self.device).contiguous())
        if self.fp8 and quant:
            q, sc = fp8_ops.quantize_weight_block(w.to(self.device))
            return Lin(q, sc)
        return Lin(self._to(w))

    def _dense(self, st, name) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
        """Weight as bf16/fp32 (fp8 dequantised) for layers we reshape or absorb."""
        w = st[name + ".weight"]
        s = st.get(name + ".weight_scale_inv")
        if w.dtype == torch.float8_e4m3fn:
            return fp8_ops.dequantize_weight_block(w, s.float())
        return w.float()

    def _raw(self, st, name):
        w = st[name + ".weight"]
        return w, st.get(name + ".weight_scale_inv")

    @staticmethod
    def _deq(w, s):
        return fp8_ops.dequantize_weight_block(w, s.float()) if s is not None else w.float()

    def _rows(self, w, s, r0, r1):
        """Rows [r0, r1) of a weight (and of its block scales; bounds must be 128-aligned)."""
        if s is None:
            return w[r0:r1], None
        assert r0 % 128 == 0 and (r1 % 128 == 0 or r1 == w.shape[0])
        return w[r0:r1], s[r0 // 128:(r1 + 127) // 128]

    def _cols(self, w, s, c0, c1):
        if s is None:
            return w[:, c0:c1], None
        assert c0 % 128 == 0 and c1 % 128 == 0
        return w[:, c0:c1], s[:, c0 // 128:c1 // 128]

    def _cat_rows(self, parts):
        """Concatenate (w, s) row blocks, each padded to 128 rows (fp8 or bf16 uniformly)."""
        if not self.fp8:
            return torch.cat([_pad_rows(self._deq(w, s)) for w, s in parts]), None
        ws, ss = [], []
        for w, s in parts:
            if s is None:
                w, s = fp8_ops.quantize_weight_block(w.float())
            ws.append(_pad_rows(w.view(torch.uint8)).view(torch.float8_e4m3fn))
            ss.append(s.float())  # ceil(rows / 128) scale rows == padded rows / 128
        return torch.cat(ws), torch.cat(ss)

    def _attn_keys(self):
        k = ["self_attn.kv_a_proj_with_mqa.weight", "self_attn.kv_a_layernorm.weight",
             "self_attn.kv_b_proj.weight", "self_attn.o_proj.weight"]
        k += ["self_attn.q_a_proj.weight", "self_attn.q_a_layernorm.weight",
              "self_attn.q_b_proj.weight"] if self.q_lora else ["self_attn.q_proj.weight"]
        if self.sparse:
            k += ["self_attn.indexer.wq_b.weight", "self_attn.indexer.wk.weight",
                  "self_attn.indexer.k_norm.weight", "self_attn.indexer.k_norm.bias",
                  "self_attn.indexer.weights_proj.weight"]
        return k

    def _is_moe(self, i):
        return self.E > 0 and i >= self.cfg.first_k_dense

    def _mlp_keys(self, i):
        if not self._is_moe(i):
            return ["mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight"]
        k = ["mlp.gate.weight"]
        for e in range(self.e0, self.e0 + self.E_local):
            k += [f"mlp.experts.{e}.{p}.weight" for p in ("gate_proj", "up_proj", "down_proj")]
        if self.cfg.shared_expert_intermediate_size:
            k += [f"mlp.shared_experts.{p}.weight" for p in ("gate_proj", "up_proj", "down_proj")]
        return k

    def _wanted(self, i, key):
        if key.startswith("mlp.experts.") and self._is_moe(i):
            e = int(key.split(".")[2])
            return self.e0 <= e < self.e0 + self.E_local
        return True

    def _needs_scale(self, st, key):
        return key.endswith(".weight") and st[key].dtype in (torch.float8_e4m3fn, torch.int8) \
            and key[:-len("weight")] + "weight_scale_inv" not in st

    def _try_finalize(self, i):
        st = self._staging[i]
        need = ["input_layernorm.weight", "post_attention_layernorm.weight"] + \
            self._attn_keys() + self._mlp_keys(i)
        if not all(k in st for k in need) or any(self._needs_scale(st, k) for k in need):
            return
        L = self.layers[i]
        self._finalize_attention(L, st)
        self._finalize_mlp(i, L, st)
        L.ln1 = self._to(st["input_layernorm.weight"])
        L.ln2 = self._to(st["post_attention_layernorm.weight"])
        del self._staging[i]

    def _finalize_attention(self, L, st):
        r, t, H = self.rank, self.tp, self.cfg.hidden_size
        hq, nope, rope, v = self.hq, self.nope, self.rope, self.vdim
        parts = [self._raw(st, "self_attn.q_a_proj" if self.q_lora else "self_attn.q_proj"),
                 self._raw(st, "self_attn.kv_a_proj_with_mqa")]
        if not self.q_lora:  # V2-Lite style: q rows sharded by heads inside the A GEMM
            w, s = parts[0]
            rows = hq * (nope + rope)
            parts[0] = self._rows(w, s, r * rows, (r + 1) * rows)
        if self.sparse:
            parts += [self._raw(st, "self_attn.indexer.wk"),
                      self._raw(st, "self_attn.indexer.weights_proj")]
        w, s = self._cat_rows(parts)
        L.w_a = self._lin(w, s)
        L.kv_a_norm = self._to(st["self_attn.kv_a_layernorm.weight"])
        if self.q_lora:
            L.q_a_norm = self._to(st["self_attn.q_a_layernorm.weight"])
            w, s = self._raw(st, "self_attn.q_b_proj")
            rows = hq * (nope + rope)
            qb = [self._rows(w, s, r * rows, (r + 1) * rows)]
            if self.sparse:
                qb.append(self._raw(st, "self_attn.indexer.wq_b"))
            w, s = self._cat_rows(qb)
            L.w_qb = self._lin(w, s)
        kvb = self._dense(st, "self_attn.kv_b_proj").view(self.cfg.num_heads, nope + v, self.kv_lora)
        kvb = kvb[r * hq:(r + 1) * hq]
        L.w_kb = self._to(kvb[:, :nope])                                 # [hq, 128, 512]
        L.w_vb = self._to(kvb[:, nope:].transpose(1, 2))                 # [hq, 512, 128]
        w, s = self._raw(st, "self_attn.o_proj")
        L.o = self._lin(*self._cols(w, s, r * hq * v, (r + 1) * hq * v))
        if self.sparse:
            L.idx_ln_w = self._to(st["self_attn.indexer.k_norm.weight"])
            L.idx_ln_b = self._to(st["self_attn.indexer.k_norm.bias"])

    def _finalize_mlp(self, i, L, st):
        r, t = self.rank, self.tp
        if not self._is_moe(i):
            L.gu, L.down = self._swiglu(st, "mlp", r, t)
            return
        L.router_w = self._to(st["mlp.gate.weight"])
        b = st.get("mlp.gate.e_score_correction_bias")
        L.router_bias = b.float().to(self.device).contiguous() if b is not None else None
        if self.w4:
            self._finalize_experts_w4(L, st)
            if self.cfg.shared_expert_intermediate_size:
                L.shared_gu, L.shared_down = self._swiglu(st, "mlp.shared_experts", r, t)
            return
        gus, gss, dws, dss = [], [], [], []
        for e in range(self.e0, self.e0 + self.E_local):
            p = f"mlp.experts.{e}."
            g, gs = self._raw(st, p + "gate_proj")
            u, us = self._raw(st, p + "up_proj")
            d, ds = self._raw(st, p + "down_proj")
            if not self.ep:
                I = g.shape[0] // t
                g, gs = self._rows(g, gs, r * I, (r + 1) * I)
                u, us = self._rows(u, us, r * I, (r + 1) * I)
                d, ds = self._cols(d, ds, r * I, (r + 1) * I)
            if self.fp8:
                w, s = self._cat_rows([(g, gs), (u, us)])  # [gate (I) ; up (I)]
                gus.append(w)
                gss.append(s)
                w, s = self._cat_rows([(d, ds)])
                dws.append(w)
                dss.append(s)
            else:
                gus.append(ops.interleave_gate_up(self._deq(g, gs), self._deq(u, us)))
                dws.append(self._deq(d, ds))
        if self.fp8:
            L.experts_gu = torch.cat(gus).to(self.device)
            L.experts_gu_s = torch.cat(gss).to(self.device)
            L.experts_down = torch.cat(dws).to(self.device)
            L.experts_down_s = torch.cat(dss).to(self.device)
        else:
            L.experts_gu = self._to(torch.cat(gus))
            L.experts_down = self._to(torch.cat(dws))
        if self.cfg.shared_expert_intermediate_size:
            L.shared_gu, L.shared_down = self._swiglu(st, "mlp.shared_experts", r, t)

    def _finalize_experts_w4(self, L, st):
        """Routed experts as packed int4: w13 [E, 2I, H/2] ([gate ; up] rows), w2 [E, H, I/2],
        bf16 scales per (row, 128 columns).  bf16 checkpoint experts (random-init models) are
        quantised here; TP shards the intermediate, which must stay 128-aligned."""
        from ..ops.w4afp8 import quantize_w4
        r, t = self.rank, self.tp

        def w4(st_name):
            w, s = self._raw(st, st_name)
            if w.dtype != torch.int8:
                w, s = quantize_w4(self._deq(w, s))
            return w, s.to(torch.bfloat16)

        w13, s13, w2, s2 = [], [], [], []
        for e in range(self.e0, self.e0 + self.E_local):
            p = f"mlp.experts.{e}."
            (g, gs), (u, us), (d, ds) = w4(p + "gate_proj"), w4(p + "up_proj"), w4(p + "down_proj")
            if not self.ep:
                I = g.shape[0] // t
                if I % 128:
                    raise ValueError("W4AFP8 needs a 128-aligned intermediate size per TP rank; "
                                     "use expert parallelism")
                g, gs, u, us = (g[r * I:(r + 1) * I], gs[r * I:(r + 1) * I],
                                u[r * I:(r + 1) * I], us[r * I:(r + 1) * I])
                d, ds = d[:, r * I // 2:(r + 1) * I // 2], ds[:, r * I // 128:(r + 1) * I // 128]
            w13.append(torch.cat([g, u]))
            s13.append(torch.cat([gs, us]))
            w2.append(d)
            s2.append(ds)
        dev = self.device
        L.w4 = tuple(torch.stack(v).to(dev).contiguous() for v in (w13, s13, w2, s2))

    def _swiglu(self, st, prefix, r, t):
        """Dense SwiGLU (TP-sharded intermediate): fp8 -> [gate ; up] rows for the
        silu_mul_fp8_quant path; bf16 -> interleaved rows for the GEMM's SwiGLU epilogue."""
        g, gs = self._raw(st, prefix + ".gate_proj")
        u, us = self._raw(st, prefix + ".up_proj")
        d, ds = self._raw(st, prefix + ".down_proj")
        I = g.shape[0] // t
        g, gs = self._rows(g, gs, r * I, (r + 1) * I)
        u, us = self._rows(u, us, r * I, (r + 1) * I)
        d, ds = self._cols(d, ds, r * I, (r + 1) * I)
        if self.fp8:
            w, s = self._cat_rows([(g, gs), (u, us)])
            gu = self._lin(w, s)
            return gu, self._lin(d, ds)
        g, u, d = self._deq(g, gs), self._deq(u, us), self._deq(d, ds)
        if self.cfg.swiglu_limit > 0:  # clamped SwiGLU runs after the GEMM: keep [gate ; up]
            return Lin(self._to(torch.cat([g, u]))), Lin(self._to(d))
        return Lin(self._to(ops.interleave_gate_up(g, u))), Lin(self._to(d))

    def load_weights(self, weights: Iterable[Tuple[str, torch.Tensor]]) -> None:
        cfg = self.cfg
        for name, w in weights:
            if name == "model.embed_tokens.weight":
                self.embed = self._to(w)
            elif name == "lm_head.weight":
                self.lm_head = self._to(shard_rows(w, self.rank, self.tp))
            elif name == "model.norm.weight":
                self.final_norm = self._to(w)
            else:
                m = _LAYER_RE.match(name)
                if not m:
                    continue
                i, key = int(m.group(1)), m.group(2)
                if i == cfg.num_layers and cfg.num_nextn_predict_layers > 0:
                    if self._wanted(i, key) and key != "embed_tokens.weight":
                        self._mtp_staging[key] = w
                        self._try_finalize_mtp()
                    continue
                if i >= cfg.num_layers or not self._wanted(i, key):
                    continue
                self._staging[i][key] = w
                self._try_finalize(i)
        if cfg.tie_word_embeddings and self.lm_head is None and self.embed is not None:
            self.lm_head = self._to(shard_rows(self.embed, self.rank, self.tp))
        missing = [i for i in range(cfg.num_layers) if self.layers[i].ln1 is None]
        if missing or self.embed is None or self.final_norm is None or self.lm_head is None:
            raise RuntimeError(f"incomplete checkpoint: layers {missing[:8]}")
        self._staging.clear()
        self._mtp_staging = {}

    def _try_finalize_mtp(self):
        st = self._mtp_staging
        i = self.cfg.num_layers
        need = ["enorm.weight", "hnorm.weight", "eh_proj.weight", "shared_head.norm.weight",
                "shared_head.head.weight", "input_layernorm.weight",
                "post_attention_layernorm.weight"] + self._attn_keys() + self._mlp_keys(i)
        if self.mtp is not None or not all(k in st for k in need) or \
                any(self._needs_scale(st, k) for k in need):
            return
        L = _Layer()
        self._finalize_attention(L, st)
        self._finalize_mlp(i, L, st)
        L.ln1 = self._to(st["input_layernorm.weight"])
        L.ln2 = self._to(st["post_attention_layernorm.weight"])
        L.enorm = self._to(st["enorm.weight"])
        L.hnorm = self._to(st["hnorm.weight"])
        L.eh_proj = self._lin(*self._raw(st, "eh_proj"))
        L.head_norm = self._to(st["shared_head.norm.weight"])
        L.head = self._to(shard_rows(st["shared_head.head.weight"], self.rank, self.tp))
        self.mtp = L
        self._mtp_staging = {}

    def forward_mtp(self, next_ids, prev_hidden, meta, cache):
        """One multi-token-prediction step: position p combines the embedding of token p+1
        with the main model's final hidden state at p, runs the MTP decoder layer (own latent
        cache, same block tables), and returns hidden states whose logits predict token p+2."""
        L, eps = self.mtp, self.cfg.rms_norm_eps
        T = next_ids.shape[0]
        self.comm.begin_forward()
        self._slots = self._dcp_slots(meta.slot_mapping) if self.dcp > 1 else meta.slot_mapping
        e = ops.rms_norm(ops.embedding(next_ids, self.embed), L.enorm, eps)
        hp = ops.rms_norm(prev_hidden, L.hnorm, eps)
        x = L.eh_proj(torch.cat([e, hp], -1).contiguous())
        residual = x
        x = ops.rms_norm(x, L.ln1, eps)
        a = self._attention(L, x, meta, cache, T)
        o = L.o(a, out=self.comm.out_buffer(T))
        x, residual = self.comm.allreduce_add_rmsnorm(o, residual, L.ln2, eps)
        d = self._mlp(self.cfg.num_layers, L, x, T)
        x, residual = self.comm.allreduce_add_rmsnorm(d, residual, L.head_norm, eps)
        return x

    def compute_logits_mtp(self, hidden):
        return ops.linear(hidden, self.mtp.head, out_dtype=torch.float32)

    def linear_shapes(self):
        """(N, K) of the bf16 GEMMs (split-K workspace planning)."""
        out = {tuple(self.lm_head.shape)}
        for L in self.layers + ([self.mtp] if self.mtp is not None else []):
            for lin in (L.w_a, L.w_qb, L.o, L.gu, L.down, L.shared_gu, L.shared_down):
                if lin is not None and not lin.fp8:
                    out.add(tuple(lin.w.shape))
        return sorted(out)

    # ------------------------------------------------------------------ KV cache
    def kv_cache_spec(self) -> dict:
        return {"num_layers": self.cfg.num_layers, "num_kv_heads": 1, "head_dim": 576,
                "dtype": self.dtype}

    def kv_bytes_per_block(self, block_size: int) -> int:
        elt = torch.tensor([], dtype=self.dtype).element_size()
        per = 576 + (self.idx_dim if self.sparse else 0)
        n = self.cfg.num_layers + (1 if self.mtp is not None else 0)
        return n * block_size * per * elt

    def allocate_kv_cache(self, num_blocks: int, block_size: int) -> list:
        """One latent (+ index) cache per layer, plus one for the MTP layer when loaded."""
        n = self.cfg.num_layers + (1 if self.mtp is not None else 0)
        lat = torch.zeros(n, num_blocks, block_size, 576, dtype=self.dtype, device=self.device)
        idx = torch.zeros(n, num_blocks, block_size, self.idx_dim, dtype=self.dtype,
                          device=self.device) if self.sparse else None
        return [(lat[i], idx[i] if idx is not None else None) for i in range(n)]

    def _splits(self, T: int) -> int:
        """KV splits of the MLA kernel for T query tokens (static for a graph size)."""
        if T > 64 or self.device.type != "cuda":
            return 1
        groups = T * ((self.hq * self.dcp + 15) // 16)
        keys = self.cfg.index_topk if self.sparse else self.cfg.max_position // self.dcp
        return mla_ops.choose_splits(groups, keys)

    def _ws(self, T: int, splits: int):
        if splits == 1:
            return None
        heads = self.hq * self.dcp  # decode context parallelism attends every head
        need = splits * T * heads * 512
        if self._mla_ws is None or self._mla_ws[0].numel() < need:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("MLA split workspace must be reserved before graph capture")
            self._mla_ws = (torch.empty(need, device=self.device),
                            torch.empty(splits * T * heads, device=self.device))
        return self._mla_ws

    # ------------------------------------------------------------------ decode context parallel
    def enable_dcp(self, size: int, kv_block_size: int) -> None:
        """Decode context parallelism over the tensor-parallel group (size == TP): the latent
        cache is sharded by token (rank r keeps tokens p % size == r at local index p // size)
        instead of replicated on every rank, so each rank holds 1 / size of every request's
        context.  The scheduler's blocks then span kv_block_size * size tokens, kv_block_size
        of them on each rank.  Dense MLA only (the V3.2 sparse indexer keeps its own cache)."""
        if size > 1 and self.sparse:
            raise ValueError("decode context parallelism supports dense MLA (no sparse indexer)")
        if size > 1 and size != self.tp:
            raise ValueError("decode_context_parallel_size must equal tensor_parallel_size")
        self.dcp, self.kv_block_size = size, kv_block_size

    def _dcp_slots(self, slot_mapping: torch.Tensor) -> torch.Tensor:
        """Scheduler slot (virtual block * bs * dcp + offset) -> this rank's local slot, or -1
        for tokens another rank stores."""
        bs, n = self.kv_block_size, self.dcp
        span = bs * n
        off = torch.remainder(slot_mapping, span)
        local = torch.div(slot_mapping, span, rounding_mode="floor") * bs + off // n
        keep = (slot_mapping >= 0) & (off % n == self.rank)
        return torch.where(keep, local, torch.full_like(local, -1)).to(slot_mapping.dtype)

    def reserve_workspaces(self, max_tokens: int) -> None:
        for T in range(1, min(max_tokens, 64) + 1):
            self._ws(T, self._splits(T))

    # ------------------------------------------------------------------ forward
    def forward(self, input_ids, meta, kv_caches):
        cfg, eps = self.cfg, self.cfg.rms_norm_eps
        T = input_ids.shape[0]
        self.comm.begin_forward()
        self._slots = self._dcp_slots(meta.slot_mapping) if self.dcp > 1 else meta.slot_mapping
        h = ops.embedding(input_ids, self.embed)
        residual = h
        n = len(self.layers)
        # the attention input's only consumer is the fused q_a / kv_a projection: with fp8
        # weights the norm quantises it in the same pass (1x128 e4m3 groups)
        xq = None
        if self.layers[0].w_a.fp8:
            q0, s0, _ = ops.rms_norm_quant_fp8(h, self.layers[0].ln1, eps)
            x, xq = h, (q0, s0)
        else:
            x = ops.rms_norm(h, self.layers[0].ln1, eps)
        for i, L in enumerate(self.layers):
            a = self._attention(L, x, meta, kv_caches[i], T, xq)
            o = L.o(a, out=self.comm.out_buffer(T))
            x, residual = self.comm.allreduce_add_rmsnorm(o, residual, L.ln2, eps)
            d = self._mlp(i, L, x, T)
            if i + 1 < n and self.layers[i + 1].w_a.fp8:
                x, residual, xq = self.comm.allreduce_add_rmsnorm_quant(
                    d, residual, self.layers[i + 1].ln1, eps)
            else:
                nxt = self.layers[i + 1].ln1 if i + 1 < n else self.final_norm
                x, residual = self.comm.allreduce_add_rmsnorm(d, residual, nxt, eps)
                xq = None
        return x

    def _attention(self, L, x, meta, cache, T, xq=None):
        hq, eps = self.hq, self.cfg.rms_norm_eps
        lat_cache, idx_cache = cache
        a = L.w_a(x) if xq is None else L.w_a.quantized(*xq)
        kv = a[:, self.a_off["kv"]:self.a_off["kv"] + 576]
        if self.q_lora:
            q_a = ops.rms_norm(a[:, :self.q_lora], L.q_a_norm, eps)
            q = L.w_qb(q_a)
        else:
            q = a
        qh = q[:, :hq * 192]
        mla_ops.mla_prep(qh, kv, L.kv_a_norm, eps, meta.positions, self.cos_sin, lat_cache,
                         self._slots if self._slots is not None else meta.slot_mapping, hq)
        q3 = qh.view(T, hq, 192)
        q_lat = torch.bmm(q3[:, :, :128].transpose(0, 1), L.w_kb)  # [hq, T, 512]
        indices = None
        if self.sparse:
            indices = self._indexer(L, q, a, meta, idx_cache, T)
        splits = self._splits(T)
        if self.dcp > 1:
            # every rank attends ALL heads over its token shard, then an LSE-weighted
            # reduce-scatter returns each rank its own heads
            ql = self.comm.all_gather(q_lat.transpose(0, 1).contiguous(), dim=1)  # [T, H, 512]
            qp = self.comm.all_gather(q3[:, :, 128:].contiguous(), dim=1)         # [T, H, 64]
            H = ql.shape[1]
            o_all = torch.empty(T, H, 512, dtype=a.dtype, device=a.device)
            lse = torch.empty(T, H, dtype=torch.float32, device=a.device)
            mla_ops.mla_attention(ql, qp, lat_cache, meta.block_tables, meta.cu_q, meta.seq_lens,
                                  None, o_all, self.scale, splits, self._ws(T, splits),
                                  dcp=(self.dcp, self.rank), lse_out=lse)
            o_lat = mla_ops.dcp_combine(o_all, lse, self.comm).transpose(0, 1).contiguous()
        else:
            o_lat = torch.empty(hq, T, 512, dtype=a.dtype, device=a.device)
            mla_ops.mla_attention(q_lat.transpose(0, 1), q3[:, :, 128:], lat_cache,
                                  meta.block_tables, meta.cu_q, meta.seq_lens, indices,
                                  o_lat.transpose(0, 1), self.scale, splits, self._ws(T, splits))
        o = torch.bmm(o_lat, L.w_vb)  # [hq, T, 128]
        return o.transpose(0, 1).reshape(T, hq * self.vdim)

    def _indexer(self, L, q, a, meta, idx_cache, T):
        nh, dh = self.idx_heads, self.idx_dim
        qi = q[:, self.hq * 192:self.hq * 192 + nh * dh]
        ops.rope_kv(qi, meta.positions, self.cos_sin, None, None, meta.slot_mapping, nh, 0,
                    self.rope, True, head_dim=dh)
        k = a[:, self.a_off["ik"]:self.a_off["ik"] + dh]
        mla_ops.indexer_k_prep(k, L.idx_ln_w, L.idx_ln_b, 1e-6, meta.positions, self.cos_sin,
                               idx_cache, meta.slot_mapping)
        w = a[:, self.a_off["iw"]:self.a_off["iw"] + nh].float() * (nh ** -0.5 * dh ** -0.5)
        L_keys = max(64, -(-int(meta.max_seq_len) // 64) * 64)
        topk = self.cfg.index_topk
        out = torch.empty(T, topk, dtype=torch.int32, device=q.device)
        chunk = max(1, (256 << 20) // (4 * L_keys))  # bound the fp32 score buffer to 256 MB
        for t0 in range(0, T, chunk):
            t1 = min(T, t0 + chunk)
            # a chunk of query tokens is a contiguous range of requests' tokens: score it with
            # the full metadata (rows beyond the chunk are not computed)
            scores = torch.empty(t1 - t0, L_keys, dtype=torch.float32, device=q.device)
            if t0 == 0 and t1 == T:
                mla_ops.indexer_scores(qi, w, idx_cache, meta.block_tables, meta.cu_q,
                                       meta.seq_lens, scores)
                out[:] = mla_ops.topk_indices(scores, meta.cu_q, meta.seq_lens, topk)
            else:
                cu, sl, bt = _sub_meta(meta, t0, t1)
                mla_ops.indexer_scores(qi[t0:t1], w[t0:t1], idx_cache, bt, cu, sl, scores)
                out[t0:t1] = mla_ops.topk_indices(scores, cu, sl, topk)
        return out

    def _mlp(self, i, L, x, T):
        if not self._is_moe(i):
            return self._swiglu_fwd(L.gu, L.down, x, out=self.comm.out_buffer(T))
        cfg = self.cfg
        logits = ops.linear(x, L.router_w, out_dtype=torch.float32)
        ids, w = moe_ops.grouped_topk(logits, self.topk, cfg.n_group, cfg.topk_group,
                                      bias=L.router_bias, sigmoid=cfg.scoring_func == "sigmoid",
                                      renorm=cfg.norm_topk_prob, scale=cfg.routed_scaling_factor)
        shared = self._swiglu_fwd(L.shared_gu, L.shared_down, x) if L.shared_gu is not None else None
        out = self.comm.out_buffer(T)
        if self.w4:
            from ..ops.w4afp8 import w4afp8_moe
            w13, s13, w2, s2 = L.w4
            return w4afp8_moe(x, w13, w2, s13, s2, w, ids, out=out, expert_offset=self.e0,
                              shared=shared, swiglu_limit=cfg.swiglu_limit or None)
        if self.fp8:
            return moe_ops.fused_moe_fp8(x, L.experts_gu, L.experts_gu_s, L.experts_down,
                                         L.experts_down_s, ids, w, self.E_local, shared, out=out,
                                         expert_offset=self.e0, swiglu_limit=cfg.swiglu_limit)
        if cfg.swiglu_limit > 0:
            raise NotImplementedError("clamped SwiGLU experts need fp8 or W4AFP8 weights")
        return moe_ops.fused_moe(x, L.experts_gu, L.experts_down, ids, w, self.E_local, shared,
                                 out=out, expert_offset=self.e0)

    def _swiglu_fwd(self, gu: Lin, down: Lin, x, out=None):
        """Row-parallel SwiGLU MLP: gate/up GEMM -> (clamped) SwiGLU + 1x128 e4m3 quant ->
        FP8 down GEMM; the caller's fused all-reduce + residual + RMSNorm completes it
        (reference: vllm_musa/model_executor/layers/linear.py:31-127, forward_swiglu_clamp)."""
        limit = self.cfg.swiglu_limit
        if gu.fp8:
            hq, hs = ops.activation.silu_mul_fp8_quant(gu(x), limit)
            return fp8_ops.gemm_fp8(hq, hs, down.w, down.s, out)
        if limit > 0:
            return down(ops.act_and_mul(gu(x), ops.activation.SILU, limit), out=out)
        return down(ops.linear_silu_mul(x, gu.w), out=out)

    def compute_logits(self, hidden):
        return ops.linear(hidden, self.lm_head, out_dtype=torch.float32)


def _sub_meta(meta, t0: int, t1: int):
    """cu_q / seq_lens / block tables restricted to query tokens [t0, t1) (host-side split of a
    long prefill for the indexer's score buffer; runs outside CUDA graphs)."""
    cu = meta.cu_q.tolist()
    sl = meta.seq_lens.tolist()
    rows, cus, lens = [], [0], []
    for r in range(len(cu) - 1):
        a, b = max(cu[r], t0), min(cu[r + 1], t1)
        if a >= b:
            continue
        # tokens [a, b) of request r end at prefix length seq_len - (cu[r+1] - b)
        rows.append(r)
        lens.append(sl[r] - (cu[r + 1] - b))
        cus.append(cus[-1] + (b - a))
    dev = meta.cu_q.device
    return (torch.tensor(cus, dtype=torch.int32, device=dev),
            torch.tensor(lens, dtype=torch.int32, device=dev),
            meta.block_tables[torch.tensor(rows, device=dev)])
