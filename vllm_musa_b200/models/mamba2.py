"""Mamba2 family (state-space language models; transformers' ``Mamba2ForCausalLM``).

Per layer (pre-norm residual block; TP shards heads and groups):
    zxbcdt = x W_in                      rows [z (dI) | x (dI) | B (G*N) | C (G*N) | dt (H)]
    xBC    = silu(causal_conv1d_k4(xBC) + b)     per-request conv state slot
    y      = SSD scan(x, B, C, dt)                per-request [H, P, N] fp32 state slots
    out    = RMSNorm_group(y * silu(z)) * w W_out -> fused all-reduce + residual + next norm
There is no KV cache: the engine's blocks only pace the scheduler, and prefix caching is off
(a recurrent state cannot resume from cached blocks).

Reference: the reference serves Mamba-family models through the vLLM Mamba2 mixer it patches
(vllm-patches 0038, 0117-0119, 0132, 0200); layer math as in transformers' Mamba2 and the
published Mamba2 (Dao & Gu, 2024).
"""
from __future__ import annotations

import re
from collections import defaultdict
from typing import Iterable, Optional, Tuple

import torch

from .. import ops
from ..ops import gdn as gdn_ops
from ..ops import mamba as mamba_ops
from ..parallel.communicator import LocalCommunicator
from ..parallel.state import ParallelState
from .llama import shard_cols, shard_rows

_LAYER_RE = re.compile(r"^backbone\.layers\.(\d+)\.(.+)$")
_KEYS = ("norm.weight", "mixer.in_proj.weight", "mixer.conv1d.weight", "mixer.dt_bias",
         "mixer.A_log", "mixer.D", "mixer.norm.weight", "mixer.out_proj.weight")


class _Layer:
    __slots__ = ("norm", "in_w", "conv_w", "conv_b", "dt_bias", "A_log", "D", "norm_w", "out_w")

    def __init__(self):
        for s in self.__slots__:
            setattr(self, s, None)


class Mamba2ForCausalLM:
    def __init__(self, cfg, pstate: Optional[ParallelState] = None, comm=None,
                 device: str | torch.device = "cuda"):
        self.cfg = cfg
        self.device = torch.device(device)
        self.dtype = cfg.dtype
        self.pstate = pstate or ParallelState()
        self.tp, self.rank = self.pstate.tp_size, self.pstate.tp_rank
        self.comm = comm or LocalCommunicator(self.device)
        nh, G = cfg.mamba_num_heads, cfg.mamba_n_groups
        if nh % self.tp or G % self.tp:
            raise ValueError("Mamba2 heads and n_groups must be divisible by "
                             "tensor_parallel_size")
        if cfg.mamba_conv_kernel != 4:
            raise ValueError("Mamba2: conv kernel width 4 only")
        self.P, self.N = cfg.mamba_head_dim, cfg.ssm_state_size
        self.H_l, self.G_l = nh // self.tp, G // self.tp
        self.dI = nh * self.P
        self.dI_l = self.H_l * self.P
        self.group = self.dI // G  # norm group (channels per group, same on every rank)
        self.conv_dim = self.dI_l + 2 * self.G_l * self.N
        self.dt_off = self.dI_l + self.conv_dim
        from .. import envs
        self.chunked = mamba_ops.mamba2_chunked_supported(self.P, self.N) and \
            envs.get("B200_MAMBA_CHUNKED")
        self.in_width = (self.dt_off + self.H_l + 63) // 64 * 64  # 128-byte aligned rows
        if cfg.vocab_size % self.tp:
            raise ValueError("vocab_size must be divisible by tensor_parallel_size")
        self.vocab_local = cfg.vocab_size // self.tp
        self.vocab_start = self.rank * self.vocab_local
        self.layers = [_Layer() for _ in range(cfg.num_layers)]
        self.embed = self.final_norm = self.lm_head = None
        self.conv_state: Optional[torch.Tensor] = None
        self.ssm_state: Optional[torch.Tensor] = None
        self._staging = defaultdict(dict)

    # ------------------------------------------------------------------ state / "KV"
    def allocate_state(self, slots: int) -> None:
        n = self.cfg.num_layers
        self.conv_state = torch.zeros(n, slots, self.conv_dim, 3, dtype=self.dtype,
                                      device=self.device)
        self.ssm_state = torch.zeros(n, slots, self.H_l, self.P, self.N, dtype=torch.float32,
                                     device=self.device)

    def kv_cache_spec(self) -> dict:
        return {"num_layers": 0, "num_kv_heads": 1, "head_dim": 64, "dtype": self.dtype}

    def kv_bytes_per_block(self, block_size: int) -> int:
        return 1 << 20  # nominal: no KV cache, blocks only bound the scheduler's admission

    def allocate_kv_cache(self, num_blocks: int, block_size: int) -> list:
        return []

    # ------------------------------------------------------------------ weights
    def _to(self, t: torch.Tensor, dtype=None) -> torch.Tensor:
        return t.to(device=self.device, dtype=dtype or self.dtype).contiguous()

    def load_weights(self, weights: Iterable[Tuple[str, torch.Tensor]]) -> None:
        cfg = self.cfg
        for name, w in weights:
            if name == "backbone.embeddings.weight":
                self.embed = self._to(w)
                if cfg.tie_word_embeddings:
                    self.lm_head = self._to(shard_rows(w, self.rank, self.tp))
            elif name == "lm_head.weight":
                self.lm_head = self._to(shard_rows(w, self.rank, self.tp))
            elif name == "backbone.norm_f.weight":
                self.final_norm = self._to(w)
            else:
                m = _LAYER_RE.match(name)
                if not m or int(m.group(1)) >= cfg.num_layers:
                    continue
                i = int(m.group(1))
                self._staging[i][m.group(2)] = w
                self._try_finalize(i)
        missing = [i for i, L in enumerate(self.layers) if L.in_w is None]
        if missing or self.embed is None or self.final_norm is None or self.lm_head is None:
            raise RuntimeError(f"incomplete Mamba2 checkpoint: layers {missing[:8]}")
        self._staging.clear()

    def _try_finalize(self, i: int) -> None:
        st = self._staging[i]
        need = list(_KEYS) + (["mixer.conv1d.bias"] if self.cfg.mamba_conv_bias else [])
        if not all(k in st for k in need):
            return
        L, r = self.layers[i], self.rank
        dI, dIl, GN, GNl, N = self.dI, self.dI_l, self.cfg.mamba_n_groups * self.N, \
            self.G_l * self.N, self.N
        h0, g0 = r * self.H_l, r * self.G_l * N

        def conv_rows(t):  # [x | B | C] channels of this rank
            return torch.cat([t[r * dIl:(r + 1) * dIl], t[dI + g0:dI + g0 + GNl],
                              t[dI + GN + g0:dI + GN + g0 + GNl]])

        w = st["mixer.in_proj.weight"]
        rows = [w[r * dIl:(r + 1) * dIl], conv_rows(w[dI:]),
                w[2 * dI + 2 * GN + h0:2 * dI + 2 * GN + h0 + self.H_l]]
        pad = self.in_width - self.dt_off - self.H_l
        if pad:
            rows.append(torch.zeros(pad, w.shape[1], dtype=w.dtype, device=w.device))
        L.in_w = self._to(torch.cat(rows))
        L.conv_w = self._to(conv_rows(st["mixer.conv1d.weight"].reshape(-1, 4)))
        if self.cfg.mamba_conv_bias:
            L.conv_b = self._to(conv_rows(st["mixer.conv1d.bias"]))
        for k, attr in (("mixer.dt_bias", "dt_bias"), ("mixer.A_log", "A_log"), ("mixer.D", "D")):
            setattr(L, attr, self._to(st[k][h0:h0 + self.H_l], torch.float32))
        L.norm_w = self._to(st["mixer.norm.weight"][r * dIl:(r + 1) * dIl])
        L.out_w = self._to(shard_cols(st["mixer.out_proj.weight"], r, self.tp))
        L.norm = self._to(st["norm.weight"])
        del self._staging[i]

    def linear_shapes(self) -> list:
        out = {tuple(self.lm_head.shape)}
        for L in self.layers:
            out.add(tuple(L.in_w.shape))
            out.add(tuple(L.out_w.shape))
        return sorted(out)

    # ------------------------------------------------------------------ forward
    def forward(self, input_ids: torch.Tensor, meta, kv_caches: list) -> torch.Tensor:
        cfg, eps = self.cfg, self.cfg.rms_norm_eps
        T = input_ids.shape[0]
        self.comm.begin_forward()
        h = ops.embedding(input_ids, self.embed)
        residual = h
        x = ops.rms_norm(h, self.layers[0].norm, eps)
        n = len(self.layers)
        for i, L in enumerate(self.layers):
            zx = ops.linear(x, L.in_w)
            xbc = gdn_ops.causal_conv1d(zx[:, self.dI_l:], L.conv_w, self.conv_state[i],
                                        meta.cu_q, meta.seq_lens, meta.state_slots,
                                        bias=L.conv_b)
            y = self._scan(i, L, xbc, zx, meta, T)
            g = mamba_ops.gated_rmsnorm(y, zx, L.norm_w, self.group, eps)
            o = ops.linear(g, L.out_w, out=self.comm.out_buffer(T))
            nxt = self.layers[i + 1].norm if i + 1 < n else self.final_norm
            x, residual = self.comm.allreduce_add_rmsnorm(o, residual, nxt, eps)
        return x

    def _scan(self, i, L, xbc, zx, meta, T):
        """SSD scan of one layer: decode rows through the token recurrence, a prefill part of
        at least CHUNK_MIN_TOKENS tokens through the chunked kernels."""
        cfg = self.cfg
        nd, npf = meta.num_decodes, meta.num_prefills
        args = (xbc, self.dI_l, self.dI_l + self.G_l * self.N, zx[:, self.dt_off:], L.dt_bias,
                L.A_log, L.D, self.ssm_state[i])
        geo = (self.H_l, self.G_l, self.P, self.N, cfg.mamba_dt_min, cfg.mamba_dt_max)
        sl, slots = meta.seq_lens, meta.state_slots
        if T - nd < mamba_ops.CHUNK_MIN_TOKENS or not self.chunked:
            return mamba_ops.mamba2_scan(*args, meta.cu_q, sl, slots, *geo)
        y = torch.empty(T, self.H_l * self.P, dtype=xbc.dtype, device=xbc.device)
        if nd > 0:
            mamba_ops.mamba2_scan(*args, meta.cu_q[:nd + 1], sl[:nd], slots[:nd], *geo, out=y)
        return mamba_ops.mamba2_chunked(*args, meta.cu_q[nd:nd + npf + 1], sl[nd:nd + npf],
                                        slots[nd:nd + npf], *geo, out=y, num_tokens=T - nd)

    def compute_logits(self, hidden: torch.Tensor) -> torch.Tensor:
        return ops.linear(hidden, self.lm_head, out_dtype=torch.float32)
