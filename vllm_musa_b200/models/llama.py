"""Dense decoder family: Llama-2/3, Mistral-style and Qwen2/Qwen3 (QK-RMSNorm) models.

One forward = per layer
    qkv GEMM -> fused [QK-norm] + RoPE + paged KV insert -> paged attention -> o_proj GEMM
    -> all-reduce + residual add + RMSNorm (one fused op) -> gate/up GEMM with SwiGLU epilogue
    -> down GEMM -> all-reduce + residual add + next RMSNorm
so every norm rides on the collective before it and SwiGLU never round-trips HBM.  Weights
are sharded Megatron-style for tensor parallelism (heads / intermediate / vocab); the
embedding is replicated so the first layer needs no collective.

The reference runs upstream vLLM's model files with its custom ops swapped in
(vllm_musa/model_executor/layers/*: RMSNorm, SiluAndMul, RotaryEmbedding, RowParallelLinear)
and compile-time fusions (vllm_musa/_inductor/musa_allreduce_rms_fusion.py:254).  Here the
fused graph is written directly.
"""
from __future__ import annotations

import re
from collections import defaultdict
from typing import Iterable, Optional, Tuple

import torch

from .. import ops
from ..attention import AttnMetadata, PagedAttention
from ..config import ModelConfig
from ..parallel.communicator import LocalCommunicator
from ..parallel.state import ParallelState

_LAYER_RE = re.compile(r"^model\.layers\.(\d+)\.(.+)$")


def shard_rows(w: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    n = w.shape[0]
    assert n % world == 0, f"cannot shard {n} rows over {world} ranks"
    s = n // world
    return w[rank * s:(rank + 1) * s]


def shard_cols(w: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    n = w.shape[1]
    assert n % world == 0, f"cannot shard {n} columns over {world} ranks"
    s = n // world
    return w[:, rank * s:(rank + 1) * s]


def pp_layer_range(num_layers: int, pp_size: int, pp_rank: int) -> Tuple[int, int]:
    """Layers [l0, l1) of pipeline stage ``pp_rank``: an even split, the remainder going to the
    first stages (the last one also runs the final norm and the LM head)."""
    if pp_size > num_layers:
        raise ValueError("pipeline_parallel_size exceeds the number of layers")
    base, extra = divmod(num_layers, pp_size)
    l0 = pp_rank * base + min(pp_rank, extra)
    return l0, l0 + base + (1 if pp_rank < extra else 0)


def kv_head_range(num_kv_heads: int, rank: int, world: int) -> Tuple[int, int]:
    """KV heads owned by ``rank``; heads are replicated when there are fewer than ranks."""
    if num_kv_heads >= world:
        per = num_kv_heads // world
        return rank * per, per
    return (rank * num_kv_heads) // world, 1


class _Layer:
    __slots__ = ("ln1", "ln2", "qkv_w", "o_w", "gu_w", "down_w", "q_norm", "k_norm", "router_w",
                 "router_bias", "experts_gu", "experts_down", "shared_gu", "shared_down",
                 "shared_gate", "extra")

    def __init__(self):
        for s in self.__slots__:
            setattr(self, s, None)


class DenseDecoderForCausalLM:
    """Llama / Qwen2 / Qwen3 dense decoder (see module docstring)."""

    def __init__(self, cfg: ModelConfig, pstate: Optional[ParallelState] = None,
                 comm=None, device: str | torch.device = "cuda"):
        self.cfg = cfg
        self.device = torch.device(device)
        self.dtype = cfg.dtype
        self.pstate = pstate or ParallelState()
        self.tp, self.rank = self.pstate.tp_size, self.pstate.tp_rank
        self.comm = comm or LocalCommunicator(self.device)
        if cfg.num_heads % self.tp:
            raise ValueError("num_heads must be divisible by tensor_parallel_size")
        self.hq = cfg.num_heads // self.tp
        self.kv0, self.hkv = kv_head_range(cfg.num_kv_heads, self.rank, self.tp)
        self.D = cfg.head_dim
        if cfg.intermediate_size % self.tp:
            raise ValueError("intermediate_size must be divisible by tensor_parallel_size")
        self.I = cfg.intermediate_size // self.tp
        self.I_pad = (self.I + 7) // 8 * 8  # gate/up interleave groups of 8
        self.vocab_local = cfg.vocab_size // self.tp
        if cfg.vocab_size % self.tp:
            raise ValueError("vocab_size must be divisible by tensor_parallel_size")
        self.vocab_start = self.rank * self.vocab_local
        self.layers = [_Layer() for _ in range(cfg.num_layers)]
        # pipeline stage: layers [l0, l1); the first stage embeds, the last normalises and
        # projects to the vocabulary; between stages the residual stream is handed on
        self.l0, self.l1 = pp_layer_range(cfg.num_layers, self.pstate.pp_size,
                                          self.pstate.pp_rank)
        self.first_stage = self.pstate.pp_rank == 0
        self.last_stage = self.pstate.pp_rank == self.pstate.pp_size - 1
        self._stage_norm = None  # unit norm weight closing a non-last stage's last layer
        self.embed = None
        self.final_norm = None
        self.lm_head = None
        self.tq = None
        self.draft_head = None  # EAGLE head (speculative decoding): one extra cache layer
        self.aux_buf = None     # EAGLE-3: residual streams entering the aux layers, [T, k*H]
        self._aux_pos = {}      # layer index -> column block of aux_buf
        self.lora = None        # LoRAManager when adapters are enabled
        if cfg.kv_cache_dtype not in ("auto", None, "bf16", "bfloat16"):
            from ..attention import TurboQuantAttention
            self.attn = TurboQuantAttention(self.hq, self.hkv, self.D, cfg.kv_cache_dtype)
            self.tq = self.attn.fmt
            # model-defined cache: one packed uint8 cache per layer (the runner asks for these)
            self.allocate_kv_cache = self._tq_allocate_kv_cache
            self.kv_bytes_per_block = self._tq_kv_bytes_per_block
        else:
            self.attn = PagedAttention(self.hq, self.hkv, self.D)
        self.cos_sin = ops.build_cos_sin_cache(cfg.rot_dim, cfg.max_position, cfg.rope_theta,
                                               device=self.device, scaling=cfg.rope_scaling)
        self._staging = defaultdict(dict)

    # ------------------------------------------------------------------ weights
    @property
    def qkv_width(self) -> int:
        return (self.hq + 2 * self.hkv) * self.D

    def _to(self, t: torch.Tensor) -> torch.Tensor:
        return t.to(device=self.device, dtype=self.dtype).contiguous()

    def load_weights(self, weights: Iterable[Tuple[str, torch.Tensor]]) -> None:
        """Consume HF-named tensors; shard, fuse (qkv, interleaved gate/up) and keep them."""
        cfg = self.cfg
        first, last = self.first_stage, self.last_stage
        for name, w in weights:
            if name == "model.embed_tokens.weight":
                if first:
                    self.embed = self._to(w)
                if cfg.tie_word_embeddings and last:
                    self.lm_head = self._to(shard_rows(w, self.rank, self.tp))
            elif name == "lm_head.weight":
                if last:
                    self.lm_head = self._to(shard_rows(w, self.rank, self.tp))
            elif name == "model.norm.weight":
                if last:
                    self.final_norm = self._to(w)
            else:
                m = _LAYER_RE.match(name)
                if not m:
                    continue
                i, key = int(m.group(1)), m.group(2)
                if not self.l0 <= i < self.l1 or not self._wanted(i, key):
                    continue
                self._staging[i][key] = w
                self._try_finalize(i)
        missing = [i for i in range(self.l0, self.l1) if self.layers[i].qkv_w is None]
        if missing or (first and self.embed is None) or \
                (last and (self.final_norm is None or self.lm_head is None)):
            raise RuntimeError(f"incomplete checkpoint: layers {missing[:8]} ... embed/norm/lm_head "
                               f"present={self.embed is not None},{self.final_norm is not None},"
                               f"{self.lm_head is not None}")
        if not last:
            self._stage_norm = torch.ones(cfg.hidden_size, dtype=self.dtype, device=self.device)
        self._staging.clear()

    def _wanted(self, i: int, key: str) -> bool:
        """Whether this rank keeps layer ``i``'s tensor ``key`` (expert parallelism drops the
        experts other ranks own before they are staged)."""
        return True

    def _mlp_keys(self, i: int) -> list:
        return ["mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight"]

    def _finalize_mlp(self, i: int, L, st: dict) -> None:
        L.gu_w, L.down_w = self._dense_mlp_weights(st["mlp.gate_proj.weight"],
                                                   st["mlp.up_proj.weight"],
                                                   st["mlp.down_proj.weight"])

    def _dense_mlp_weights(self, gate, up, down):
        """TP-shard a SwiGLU MLP: interleaved gate/up rows, down columns padded to I_pad."""
        r, t = self.rank, self.tp
        I = gate.shape[0] // t
        I_pad = (I + 7) // 8 * 8
        gu = ops.interleave_gate_up(shard_rows(gate, r, t), shard_rows(up, r, t))
        dn = shard_cols(down, r, t)
        if I_pad != I:
            dn = torch.cat([dn, torch.zeros(dn.shape[0], I_pad - I, dtype=dn.dtype,
                                            device=dn.device)], 1)
        return self._to(gu), self._to(dn)

    def _try_finalize(self, i: int) -> None:
        need = ["input_layernorm.weight", "post_attention_layernorm.weight",
                "self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight",
                "self_attn.o_proj.weight"] + self._mlp_keys(i)
        if self.cfg.qk_norm:
            need += ["self_attn.q_norm.weight", "self_attn.k_norm.weight"]
        st = self._staging[i]
        if not all(k in st for k in need):
            return
        L, D, r, t = self.layers[i], self.D, self.rank, self.tp
        q = shard_rows(st["self_attn.q_proj.weight"], r, t)
        k = st["self_attn.k_proj.weight"][self.kv0 * D:(self.kv0 + self.hkv) * D]
        v = st["self_attn.v_proj.weight"][self.kv0 * D:(self.kv0 + self.hkv) * D]
        L.qkv_w = self._to(torch.cat([q, k, v], 0))
        L.o_w = self._to(shard_cols(st["self_attn.o_proj.weight"], r, t))
        self._finalize_mlp(i, L, st)
        L.ln1 = self._to(st["input_layernorm.weight"])
        L.ln2 = self._to(st["post_attention_layernorm.weight"])
        if self.cfg.qk_norm:
            L.q_norm = self._to(st["self_attn.q_norm.weight"])
            L.k_norm = self._to(st["self_attn.k_norm.weight"])
        del self._staging[i]

    def linear_shapes(self) -> list:
        """(N, K) of every dense GEMM weight, for workspace planning."""
        out = {tuple(self.lm_head.shape)} if self.lm_head is not None else set()
        for L in self.layers:
            for w in (L.qkv_w, L.o_w, L.gu_w, L.down_w):
                if w is not None:
                    out.add(tuple(w.shape))
        return sorted(out)

    # ------------------------------------------------------------------ forward
    def forward(self, input_ids: torch.Tensor, meta: AttnMetadata, kv_caches: list,
                hidden_in: Optional[torch.Tensor] = None) -> torch.Tensor:
        """input_ids int32 [T] -> final normalised hidden states [T, H].  Under pipeline
        parallelism a stage after the first starts from ``hidden_in`` (the residual stream the
        previous stage returned), and a stage before the last returns its residual stream."""
        cfg, eps = self.cfg, self.cfg.rms_norm_eps
        T = meta.num_tokens
        self.comm.begin_forward()
        h = ops.embedding(input_ids, self.embed) if self.first_stage else hidden_in
        residual = h
        x = ops.rms_norm(h, self.layers[self.l0].ln1, eps)
        n = self.l1
        for i in range(self.l0, self.l1):
            L = self.layers[i]
            for k in self._aux_pos.get(i, ()):  # EAGLE-3: the stream entering layer i
                H = cfg.hidden_size
                self.aux_buf[:T, k * H:(k + 1) * H].copy_(residual[:T])
            kc, vc = kv_caches[i - self.l0]
            qkv = ops.linear(x, L.qkv_w)
            lora = getattr(meta, "lora", None)
            if lora is not None:
                self._lora_qkv(i, x, qkv, lora)
            if self.tq is not None:
                D, hq, hkv = self.D, self.hq, self.hkv
                ops.rope_kv(qkv, meta.positions, self.cos_sin, None, None, meta.slot_mapping,
                            hq, hkv, cfg.rot_dim, cfg.rope_neox, L.q_norm, L.k_norm, eps,
                            write_k=True, head_dim=D)
                self.attn.write_kv(qkv[:, hq * D:(hq + hkv) * D],
                                   qkv[:, (hq + hkv) * D:(hq + 2 * hkv) * D], kc,
                                   meta.slot_mapping)
            else:
                ops.rope_kv(qkv, meta.positions, self.cos_sin, kc, vc, meta.slot_mapping,
                            self.hq, self.hkv, cfg.rot_dim, cfg.rope_neox, L.q_norm, L.k_norm,
                            eps)
            a = self.attn.forward(qkv, kc, vc, meta)
            delta = None
            if lora is not None and self.lora.has(i, "o"):
                delta = lambda inp, out, i=i: self.lora.add_delta(i, "o", inp, out, lora)  # noqa: E731
            x, residual = self.comm.linear_allreduce_add_rmsnorm(a, L.o_w, residual, L.ln2, eps,
                                                                 delta=delta)
            nxt = self.layers[i + 1].ln1 if i + 1 < n else \
                (self.final_norm if self.last_stage else self._stage_norm)
            if lora is not None and self.lora.has(i, "down"):
                x, residual = self._lora_mlp(i, L, x, residual, nxt, eps, lora)
            else:
                x, residual = self._mlp_allreduce(i, L, x, T, residual, nxt, eps)
        return x if self.last_stage else residual

    def enable_aux(self, layers, max_tokens: int) -> None:
        """Record the residual stream entering each of ``layers`` into ``aux_buf`` (one H-wide
        column block per layer, rows = step tokens) on every forward."""
        H = self.cfg.hidden_size
        self._aux_pos = {}
        for k, l in enumerate(layers):
            self._aux_pos.setdefault(int(l), []).append(k)
        self.aux_buf = torch.zeros(max_tokens, len(layers) * H, dtype=self.dtype,
                                   device=self.device)

    # ------------------------------------------------------------------ LoRA
    def _lora_qkv(self, i, x, qkv, batch) -> None:
        D, hq, hkv = self.D, self.hq, self.hkv
        cuts = {"q": (0, hq * D), "k": (hq * D, (hq + hkv) * D),
                "v": ((hq + hkv) * D, (hq + 2 * hkv) * D)}
        for mod, (c0, c1) in cuts.items():
            if self.lora.has(i, mod):
                self.lora.add_delta(i, mod, x, qkv[:, c0:c1], batch)

    def _lora_mlp(self, i, L, x, residual, nxt, eps, batch):
        """Dense MLP with adapters: plain gate/up GEMM, gate and up deltas added before the
        SwiGLU, down projection's delta added to its partial sum before the all-reduce."""
        from ..lora import add_interleaved, silu_mul_interleaved
        T = x.shape[0]
        gu = ops.linear(x, L.gu_w)
        dg = torch.zeros(T, self.I_pad, dtype=gu.dtype, device=gu.device)
        du = torch.zeros_like(dg)
        if self.lora.has(i, "gate"):
            self.lora.add_delta(i, "gate", x, dg[:, :self.I], batch)
        if self.lora.has(i, "up"):
            self.lora.add_delta(i, "up", x, du[:, :self.I], batch)
        add_interleaved(gu, dg, du)
        act = silu_mul_interleaved(gu)
        return self.comm.linear_allreduce_add_rmsnorm(
            act, L.down_w, residual, nxt, eps,
            delta=lambda inp, out: self.lora.add_delta(i, "down", inp, out, batch))

    def _mlp_allreduce(self, i, L, x, T, residual, nxt, eps):
        """MLP + all-reduce + residual + next norm; the dense down projection fuses its
        reduce-scatter into the GEMM epilogue."""
        if L.gu_w is not None and L.down_w is not None:
            act = ops.linear_silu_mul(x, L.gu_w)
            return self.comm.linear_allreduce_add_rmsnorm(act, L.down_w, residual, nxt, eps)
        d = self._mlp(i, L, x, T)
        return self.comm.allreduce_add_rmsnorm(d, residual, nxt, eps)

    def _mlp(self, i: int, L, x: torch.Tensor, T: int) -> torch.Tensor:
        """Dense SwiGLU MLP; returns this rank's partial sum (all-reduced by the caller)."""
        act = ops.linear_silu_mul(x, L.gu_w)
        return ops.linear(act, L.down_w, out=self.comm.out_buffer(T))

    def compute_logits(self, hidden: torch.Tensor) -> torch.Tensor:
        """[S, H] -> this rank's vocab shard of the logits, fp32 [S, V/tp]."""
        return ops.linear(hidden, self.lm_head, out_dtype=torch.float32)

    # ------------------------------------------------------------------ KV cache geometry
    def _tq_kv_bytes_per_block(self, block_size: int) -> int:
        return (self.l1 - self.l0) * self.hkv * block_size * self.tq.slot_bytes

    def _tq_allocate_kv_cache(self, num_blocks: int, block_size: int) -> list:
        """TurboQuant cache per layer: uint8 [num_blocks, Hkv, block_size, slot_bytes]."""
        n = self.l1 - self.l0
        buf = torch.zeros(n, num_blocks, self.hkv, block_size,
                          self.tq.slot_bytes, dtype=torch.uint8, device=self.device)
        return [(buf[i], None) for i in range(n)]

    def kv_cache_spec(self) -> dict:
        """Cache layers of this stage (its decoder layers, plus the EAGLE head's layer)."""
        d = self.draft_head
        n = self.l1 - self.l0 + (1 if d is not None and not d.replicated else 0)
        spec = {"num_layers": n, "num_kv_heads": self.hkv, "head_dim": self.D,
                "dtype": self.dtype}
        if d is not None and d.replicated:  # a whole-head draft layer keeps its own cache
            spec["draft_kv_heads"] = d.hkv
        return spec
