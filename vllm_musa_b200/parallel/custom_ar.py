"""NVSwitch peer-memory communicator (CUDA IPC) for tensor-parallel all-reduce + RMSNorm.

Per rank one cudaMalloc'd buffer, exported with cudaIpcGetMemHandle and opened by every peer:

    [staging 0][staging 1][output 0][output 1][flags: 4 x 128 blocks x 8 ranks][epochs]

The row-parallel GEMM (o_proj / down_proj) writes its partial sums straight into this rank's
staging slot (``staging_view``); ``allreduce_add_rmsnorm`` then launches one kernel
(csrc/comm/custom_ar.cu) that reduces over the peers' staging slots with NVLink loads, adds
the residual, normalises and (two-shot) scatters the normalised rows into every rank's output
slot with NVLink stores.  Slots alternate by call parity; each forward pass has an even
number of calls and starts at parity 0, so consecutive calls always alternate.

When the GPUs sit on an NVSwitch with multicast support, a second buffer is allocated from
PyTorch's symmetric memory and bound to one NVLink multicast object (NVLS): the all-reduce of
larger messages then reduces in the switch with multimem loads and broadcasts the normalised
rows with multimem stores (csrc/comm/nvls_ar.cu), so each rank's links carry about one copy of
the message per direction instead of (2 - 2/world) copies.  ``B200_AR_NVLS=0`` disables it.

Set-up is fail-closed like the reference's (vllm_musa/distributed/device_communicators/
musa_jit_custom_all_reduce.py:1762-1938, MIN consensus over a CPU group): if any rank cannot
allocate, export or open a buffer, every rank falls back to NCCL.
"""
from __future__ import annotations

import logging
import os
from typing import Optional

import torch
import torch.distributed as dist

from ..ops import _ext

log = logging.getLogger("vllm_musa_b200")

ONE_SHOT_MAX_BYTES = int(os.environ.get("B200_AR_ONE_SHOT_MAX_BYTES", "0"))
# one-shot (every rank reads every peer's whole message, one barrier) while the peer reads stay
# under this many bytes; two-shot (reduce-scatter + all-gather, two barriers) beyond.  Measured
# at TP=2, H=4096 (CUDA-graph replay): 256 tokens 22.2 us one-shot vs 26.4 us two-shot,
# 64 tokens 16.4 vs 25.2 us; 1024 tokens favour two-shot.
ONE_SHOT_READ_BYTES = 2 << 20
# The epilogue reduce-scatter stores 32-byte row pieces to peers, which NVLink moves less
# efficiently than the two-shot kernel's warp-contiguous loads: measured at TP=2 decode
# (256 tokens, Llama-3-8B) 9.31 ms/step fused vs 8.42 ms unfused, so it is opt-in.
FUSE_GEMM_RS = os.environ.get("B200_FUSE_GEMM_RS", "0") == "1"
NVLS = os.environ.get("B200_AR_NVLS", "1") != "0"
# Per-size choice between the peer-to-peer kernels and the NVLS kernel, by world size: messages
# of more than NVLS_MIN_BYTES[world] bytes take NVLS (None: never) -- two-shot from `world` rows
# up, one-shot below.  Measured (CUDA-graph replays, H=4096, all-reduce + residual + RMSNorm):
#   TP=2: peer-to-peer wins at every size (one-shot 22.0 us vs NVLS 30.3 / 25.1 us at 256 rows;
#         two-shot 127.5 us vs NVLS 204.6 us at 8192 rows): with two ranks NVLS moves twice the
#         bytes per link (the switch reads every copy, the local one included).
#   TP=8: NVLS wins up to 2048 rows (8 rows: one-shot 17.6 us vs peer-to-peer 35.0; 256 rows:
#         two-shot 27.3 vs 49.7; 1024 rows: 41.9 vs 66.9) and ties beyond (4096 rows: 114.8 vs
#         110.9; 8192: 204.5 vs 200.9); the Llama-3-8B serving bench at TP=8 runs 30.0k tok/s
#         with NVLS against 26.5k with the peer-to-peer kernels.
#   TP=4: peer-to-peer wins or ties at every size (8 rows: one-shot 12.0 us vs NVLS 16.4;
#         256 rows: two-shot 26.6 vs 25.6; 1024: 42.2 vs 41.7; 8192: 171.2 vs 210.1).
# B200_AR_NVLS_MIN_BYTES overrides the threshold for every world size.
NVLS_MIN_BYTES = {2: None, 4: None, 8: 0}
# rows each warp of the NVLS kernel walks (0: the kernel's size rule; tuning / benchmarks)
NVLS_ROWS_PER_WARP = int(os.environ.get("B200_AR_NVLS_ROWS_PER_WARP", "0"))
if os.environ.get("B200_AR_NVLS_MIN_BYTES"):
    NVLS_MIN_BYTES = {w: int(os.environ["B200_AR_NVLS_MIN_BYTES"]) for w in (2, 4, 8)}
# the NVLS kernel's fused 1x128 e4m3 output replaces AR + norm + a separate quantisation from
# this many rows up, by world size.  TP=2: never (against the peer-to-peer AR + norm + group
# quantisation it measures 25.9 vs 14.2 us at 8 rows, 34.8 vs 23.7 at 256, 69.0 vs 53.7 at
# 2048); TP=4: from ~1k rows (24.1 vs 14.1 us at 8 rows, 28.4 vs 28.7 at 256, 58.3 vs 76.0 at
# 2048); TP=8: faster at every measured size (26.0 vs 37.5 us at 8 rows, 32.5 vs 52.4 at 256,
# 61.2 vs 81.6 at 2048).
NVLS_QUANT_MIN_ROWS = {2: 1 << 30, 4: 1024, 8: 1}
if os.environ.get("B200_AR_NVLS_QUANT_MIN_ROWS"):
    NVLS_QUANT_MIN_ROWS = {w: int(os.environ["B200_AR_NVLS_QUANT_MIN_ROWS"]) for w in (2, 4, 8)}


def _consensus(ok: bool, group) -> bool:
    t = torch.tensor([1 if ok else 0], dtype=torch.int32)
    dist.all_reduce(t, op=dist.ReduceOp.MIN, group=group)
    return int(t) == 1


class NvlsBuffer:
    """The NVLS half of the communicator: one symmetric-memory buffer per rank, bound to an
    NVLink multicast object, laid out as

        [staging 0][staging 1][out 0][out 1][q 0][q 1][scales 0][scales 1][counters]

    (staging / out: [max_tokens, hidden] bf16; q: e4m3 rows; scales: fp32 [max_tokens,
    hidden / 128]; counters: the kernel's barrier counters).  Every offset has a local address
    (this rank's copy) and a multicast address."""

    def __init__(self, st, device, max_tokens: int, hidden: int, mod):
        import torch.distributed._symmetric_memory as symm
        self.mod = mod
        H, T = hidden, max_tokens
        al = lambda n: (n + 255) // 256 * 256  # noqa: E731
        self.slot = al(T * H * 2)
        self.qslot = al(T * H)
        self.sslot = al(T * max(1, H // 128) * 4)
        self.off_out = 2 * self.slot
        self.off_q = 4 * self.slot
        self.off_s = self.off_q + 2 * self.qslot
        self.off_flags = self.off_s + 2 * self.sslot
        total = self.off_flags + al(int(mod.nvls_flag_bytes()))
        group = st.tp_group
        symm.enable_symm_mem_for_group(group.group_name)
        self.buf = symm.empty(total, dtype=torch.uint8, device=device)
        self.buf.zero_()
        self.handle = symm.rendezvous(self.buf, group)
        from torch._C._autograd import DeviceType
        from torch._C._distributed_c10d import _SymmetricMemory
        self.base = self.buf.data_ptr()
        self.mc = 0
        if _SymmetricMemory.has_multicast_support(DeviceType.CUDA, device.index):
            mc = int(self.handle.multicast_ptr or 0)
            if mc:
                # the multicast mapping covers the whole allocation: same offset as the tensor
                # has from this rank's base of it
                self.mc = mc + (self.base - int(self.handle.buffer_ptrs[st.tp_rank]))
        self.epochs = torch.zeros(2 * int(mod.comm_max_blocks()), dtype=torch.int32, device=device)
        dev = device.index
        self.staging = [mod.tensor_from_ptr(self.base + k * self.slot, [T, H], torch.bfloat16, dev)
                        for k in range(2)]
        self.out = [mod.tensor_from_ptr(self.base + self.off_out + k * self.slot, [T, H],
                                        torch.bfloat16, dev) for k in range(2)]
        self.q = [mod.tensor_from_ptr(self.base + self.off_q + k * self.qslot, [T, H],
                                      torch.float8_e4m3fn, dev) for k in range(2)]
        self.s = [mod.tensor_from_ptr(self.base + self.off_s + k * self.sslot,
                                      [T, max(1, H // 128)], torch.float32, dev) for k in range(2)]

    def ptrs(self, parity: int, two_shot: bool, quant: bool) -> list:
        mc, loc = self.mc, self.base
        st = self.slot * parity
        out = self.off_out + self.slot * parity
        q = self.off_q + self.qslot * parity
        sc = self.off_s + self.sslot * parity
        return [mc + st,
                mc + out if two_shot and not quant else 0,
                loc + out if not two_shot and not quant else 0,
                mc + self.off_flags, loc + self.off_flags, self.epochs.data_ptr(),
                mc + q if two_shot and quant else 0,
                loc + q if not two_shot and quant else 0,
                mc + sc if two_shot and quant else 0,
                loc + sc if not two_shot and quant else 0]

    def close(self):
        self.staging = self.out = self.q = self.s = []
        self.handle = None
        self.buf = None


def self_world_pad(st) -> int:
    return st.tp_size


class CustomAllReduce:
    def __init__(self, st, device: torch.device, max_tokens: int, hidden: int):
        mod = _ext.require()
        self.mod = mod
        self.world, self.rank = st.tp_size, st.tp_rank
        self.device = device
        self.hidden = hidden
        self.max_tokens = max_tokens
        # rows + world: the epilogue reduce-scatter lays out world blocks of ceil(T/world) rows
        self.slot = ((max_tokens + self_world_pad(st)) * hidden * 2 + 255) // 256 * 256
        self.flag_off = 4 * self.slot
        # sampling candidates: [2 parities][world][max_tokens] fp32 scores + int64 ids
        self.cand_rows = max_tokens
        self.cand_off = self.flag_off + (mod.comm_flag_bytes() + 255) // 256 * 256
        n = self.world * max_tokens
        self.cand_ids_off = (n * 4 + 255) // 256 * 256   # int64 ids after the fp32 scores
        self.cand_parity_bytes = self.cand_ids_off + (n * 8 + 255) // 256 * 256
        cand_bytes = 2 * self.cand_parity_bytes
        # top-k / top-p candidate rows: [2 parities][world][topk_rows] rows of cand_row_bytes
        self.topk_rows = min(max_tokens, 1024)
        self.row_bytes = int(mod.cand_row_bytes())
        self.topk_off = self.cand_off + cand_bytes
        self.topk_parity_bytes = (self.world * self.topk_rows * self.row_bytes + 255) // 256 * 256
        total = self.topk_off + 2 * self.topk_parity_bytes
        self.max_blocks = int(mod.comm_max_blocks())
        self.base = mod.ipc_malloc(total)
        self.opened = []
        handles = [None] * self.world
        dist.all_gather_object(handles, mod.ipc_handle(self.base), group=st.tp_cpu_group)
        self.peer_base = []
        for p in range(self.world):
            if p == self.rank:
                self.peer_base.append(self.base)
            else:
                addr = mod.ipc_open(handles[p])
                self.opened.append(addr)
                self.peer_base.append(addr)
        self.epochs = self.base + self.flag_off + (mod.comm_flag_bytes() - 128 * 4)
        dev = device.index
        self._staging = [mod.tensor_from_ptr(self.base + k * self.slot, [max_tokens, hidden],
                                             torch.bfloat16, dev) for k in range(2)]
        self._out = [mod.tensor_from_ptr(self.base + (2 + k) * self.slot, [max_tokens, hidden],
                                         torch.bfloat16, dev) for k in range(2)]
        self._bufs = []
        for k in range(2):
            staging = [b + k * self.slot for b in self.peer_base]
            out = [b + (2 + k) * self.slot for b in self.peer_base]
            flags = [b + self.flag_off for b in self.peer_base]
            self._bufs.append(staging + out + flags)
        self.parity = 0
        self.cand_parity = 0
        # every kernel ends with a barrier (needed when calls are not strictly alternating
        # buffers, e.g. vLLM mixing eager calls and graph replays)
        self.end_barrier = False
        self.nvls: Optional[NvlsBuffer] = None
        if NVLS:
            self._init_nvls(st, device, max_tokens, hidden)

    def _init_nvls(self, st, device, max_tokens, hidden) -> None:
        """Collective: every rank tries; NVLS is used only if every rank got a multicast
        mapping (MIN consensus), otherwise every rank releases its buffer."""
        ok = True
        try:
            import torch.distributed._symmetric_memory  # noqa: F401
            ok = hasattr(self.mod, "nvls_allreduce") and st.tp_group is not None
        except Exception:  # pragma: no cover - torch built without symmetric memory
            ok = False
        if not _consensus(ok, st.tp_cpu_group):
            return
        buf = None
        try:
            buf = NvlsBuffer(st, device, max_tokens, hidden, self.mod)
            ok = buf.mc != 0
        except Exception as e:  # fail closed
            log.warning("NVLS buffer unavailable on rank %d: %s", st.rank, e)
            ok = False
        if _consensus(ok, st.tp_cpu_group):
            torch.cuda.synchronize(device)
            dist.barrier(group=st.tp_cpu_group)  # every rank's counters are zero before use
            self.nvls = buf
            log.info("NVLS all-reduce enabled (multicast buffer %.0f MiB)",
                     buf.buf.numel() / 2**20)
        elif buf is not None:
            buf.close()

    # ------------------------------------------------------------------ interface
    def begin_forward(self) -> None:
        self.parity = 0

    def can_run(self, x: torch.Tensor) -> bool:
        return (x.dtype == torch.bfloat16 and x.dim() == 2 and x.shape[1] == self.hidden and
                x.shape[0] <= self.max_tokens)

    def use_nvls(self, T: int) -> int:
        """NVLS for messages above the threshold of this world size: 2 (two-shot) from `world`
        rows up, 1 (one-shot) below; 0: the peer-to-peer kernels."""
        lim = NVLS_MIN_BYTES.get(self.world)
        if self.nvls is None or lim is None or T * self.hidden * 2 <= lim:
            return 0
        return 2 if T >= self.world else 1

    def staging_view(self, T: int) -> torch.Tensor:
        if self.use_nvls(T):
            return self.nvls.staging[self.parity][:T]
        return self._staging[self.parity][:T]

    def _plan(self, T: int):
        """Peer-to-peer algorithm for T rows: (two_shot, blocks)."""
        limit = ONE_SHOT_MAX_BYTES or ONE_SHOT_READ_BYTES // max(1, self.world - 1)
        two_shot = T * self.hidden * 2 > limit and T >= self.world
        rows = (T + self.world - 1) // self.world if two_shot else T
        return two_shot, max(1, min(rows, self.max_blocks))

    def _run_nvls(self, x, residual, weight, eps, two_shot=True, quant=False):
        T = x.shape[0]
        nv, k = self.nvls, self.parity
        if x.data_ptr() != nv.staging[k].data_ptr():
            nv.staging[k][:T].copy_(x)
        self.mod.nvls_allreduce(x, nv.ptrs(k, two_shot, quant), self.rank, self.world, T,
                                self.hidden, two_shot, residual, weight, eps,
                                NVLS_ROWS_PER_WARP)
        self.parity ^= 1
        if quant:
            return nv.q[k][:T], nv.s[k][:T]
        return nv.out[k][:T]

    def _run(self, x, residual, weight, eps):
        T = x.shape[0]
        mode = self.use_nvls(T)
        if mode:
            return self._run_nvls(x, residual, weight, eps, two_shot=mode == 2)
        if x.data_ptr() != self._staging[self.parity].data_ptr():
            self._staging[self.parity][:T].copy_(x)
        two_shot, blocks = self._plan(T)
        self.mod.fused_allreduce(x, self._bufs[self.parity], self.epochs, self.rank, self.world,
                                 T, self.hidden, blocks, self.parity, two_shot, residual, weight,
                                 eps, 0, self.end_barrier)
        out = self._out[self.parity][:T]
        self.parity ^= 1
        return out

    def all_reduce_out_of_place(self, x: torch.Tensor) -> torch.Tensor:
        """Sum over the ranks into a new tensor (x unchanged)."""
        return self._run(x, None, None, 0.0).clone()

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        out = self._run(x, None, None, 0.0)
        if out.data_ptr() != x.data_ptr():
            x.copy_(out)
        return x

    def allreduce_add_rmsnorm(self, x, residual, weight, eps):
        return self._run(x, residual, weight, eps), residual

    def can_quant(self, x: torch.Tensor) -> bool:
        """The fused all-reduce + norm emits the 1x128 e4m3 rows itself (NVLS kernels), for
        batches where that beats all-reduce + norm followed by the group quantisation."""
        return (self.nvls is not None and self.can_run(x) and self.hidden % 256 == 0 and
                x.shape[0] >= NVLS_QUANT_MIN_ROWS.get(self.world, 1 << 30))

    def allreduce_add_rmsnorm_quant(self, x, residual, weight, eps):
        """residual <- AR(x) + residual; returns (q, scales) of RMSNorm(residual) * weight per
        token in 1x128 e4m3 groups, produced inside the all-reduce kernel (NVLS one-shot for
        small messages, two-shot beyond)."""
        T = x.shape[0]
        return self._run_nvls(x, residual, weight, eps, two_shot=T >= self.world, quant=True)

    def staging_blocks(self, rows: int) -> torch.Tensor:
        """This call's staging slot viewed as world blocks of `rows` rows (epilogue / expert
        return targets of the local-source reduce)."""
        return self._staging[self.parity][:self.world * rows]

    def reduce_blocks_add_rmsnorm(self, T, residual, weight, eps, like):
        """Two-shot reduce of the world blocks already stored in this rank's staging slot
        (+ residual, RMSNorm, all-gather of the normalised rows)."""
        rows = (T + self.world - 1) // self.world
        _, blocks = self._plan(T)
        self.mod.fused_allreduce(like, self._bufs[self.parity], self.epochs, self.rank,
                                 self.world, T, self.hidden, blocks, self.parity, True, residual,
                                 weight, eps, rows)
        out = self._out[self.parity][:T]
        self.parity ^= 1
        return out, residual

    def merge_candidates(self, vals: torch.Tensor, ids: torch.Tensor) -> Optional[torch.Tensor]:
        """Vocab-parallel sampling: each rank's per-row (score, token) goes into every peer's
        candidate region by NVLink stores; one kernel barriers and merges (no NCCL).

        Returns None when the batch does not fit the region (caller falls back to NCCL).
        A rank can only overwrite a peer's region in its next call after a collective of the
        forward pass in between has seen that peer finish this call, and the two parities
        alternate as well, so no end-of-call barrier is needed."""
        R = vals.shape[0]
        if R > self.cand_rows or R > 128 * 256:
            return None
        k = self.cand_parity
        vals_ptrs = [b + self.cand_off + k * self.cand_parity_bytes for b in self.peer_base]
        ids_ptrs = [v + self.cand_ids_off for v in vals_ptrs]
        flags = [b + self.flag_off for b in self.peer_base]
        out = torch.empty_like(ids)
        self.mod.exchange_candidates(vals.contiguous(), ids.contiguous(), out,
                                     vals_ptrs + ids_ptrs + flags, self.epochs, self.rank,
                                     self.world, k)
        self.cand_parity ^= 1
        return out

    def sample_topk(self, logits, temperature, top_k, top_p, min_p, seeds, steps,
                    vocab_offset: int, V_total: int) -> Optional[torch.Tensor]:
        """Vocab-parallel sampling with top-k / top-p / min-p: each rank reduces its logits
        shard to candidate rows (<= 128 per row), one kernel stores them into every peer's
        region over NVLink, barriers and merges (csrc/sampling/topk_exchange.cu).  Returns the
        sampled ids, -1 on rows the candidates cannot decide exactly, or None when the batch
        does not fit the region.  Same parity / ordering argument as ``merge_candidates``."""
        from ..ops.sampling import shard_candidates
        R = logits.shape[0]
        if R > self.topk_rows:
            return None
        mine = shard_candidates(logits, temperature, seeds, steps, vocab_offset)
        k = self.cand_parity
        regions = [b + self.topk_off + k * self.topk_parity_bytes for b in self.peer_base]
        flags = [b + self.flag_off for b in self.peer_base]
        out = torch.empty(R, dtype=torch.int64, device=logits.device)
        self.mod.topk_exchange(mine, regions + flags, self.epochs, self.rank, self.world, k,
                               V_total, temperature, top_k, top_p, min_p, seeds, steps, out)
        self.cand_parity ^= 1
        return out

    def local_source_ok(self, T: int) -> bool:
        """The two-shot kernel's local-source mode (row blocks already scattered into this
        rank's staging slot by a producer: the GEMM epilogue or the EP return) applies."""
        return 0 < T <= self.max_tokens and self._plan(T)[0]

    def can_fuse_gemm(self, T: int) -> bool:
        """Row-parallel GEMM + all-reduce as one reduce-scatter-in-epilogue GEMM and a local
        reduce + norm + all-gather kernel (opt-in: B200_FUSE_GEMM_RS=1)."""
        return FUSE_GEMM_RS and self.local_source_ok(T)

    def linear_allreduce_add_rmsnorm(self, x, w, residual, weight, eps):
        """residual <- sum_ranks(x @ w^T) + residual; returns (RMSNorm(residual) * weight,
        residual).  The GEMM epilogue stores each row block straight into its owner's staging
        slot over NVLink (reduce-scatter fused with the tcgen05 tiles); the all-reduce kernel
        then reduces local memory only and all-gathers the normalised rows."""
        from ..ops import gemm as gemm_ops
        T = x.shape[0]
        rows = (T + self.world - 1) // self.world
        recv = self._bufs[self.parity][:self.world]
        M, N, K = T, w.shape[0], w.shape[1]
        bn, splits, mt, need = gemm_ops.plan_for(M, N, K)
        ws = gemm_ops._workspace(x.device, need) if need > 0 else None
        cnt = gemm_ops._counters(x.device) if need > 0 else None
        self.mod.gemm_bf16_rs(x, w, recv, rows, self.rank, bn, splits, mt, ws, cnt)
        _, blocks = self._plan(T)
        self.mod.fused_allreduce(x, self._bufs[self.parity], self.epochs, self.rank, self.world,
                                 T, self.hidden, blocks, self.parity, True, residual, weight,
                                 eps, rows)
        out = self._out[self.parity][:T]
        self.parity ^= 1
        return out, residual

    def close(self) -> None:
        if self.nvls is not None:
            torch.cuda.synchronize(self.device)
            self.nvls.close()
            self.nvls = None
        for a in self.opened:
            try:
                self.mod.ipc_close(a)
            except Exception:  # pragma: no cover - teardown
                pass
        self.opened = []
        if self.base:
            try:
                torch.cuda.synchronize(self.device)
                self.mod.ipc_free(self.base)
            except Exception:  # pragma: no cover
                pass
            self.base = 0


def maybe_create_custom_allreduce(st, device, max_tokens: int = 8192, hidden: int = 0
                                  ) -> Optional[CustomAllReduce]:
    """Build the communicator on every TP rank, or on none (MIN consensus over Gloo)."""
    if st.tp_size < 2 or st.tp_size > 8 or hidden <= 0:
        return None
    if os.environ.get("B200_DISABLE_CUSTOM_AR", "0") == "1":
        return None
    comm, ok = None, 1
    from .topology import group_nvlink_ok
    if os.environ.get("B200_SKIP_NVLINK_CHECK", "0") != "1" and \
            not group_nvlink_ok(device, st.tp_cpu_group):
        log.warning("rank %d: not every peer GPU is reachable over NVLink; NCCL all-reduce",
                    st.rank)
        ok = 0
    try:
        comm = CustomAllReduce(st, device, max_tokens, hidden) if ok else None
    except Exception as e:  # fail closed
        log.warning("custom all-reduce unavailable on rank %d: %s", st.rank, e)
        ok = 0
    t = torch.tensor([ok], dtype=torch.int32)
    dist.all_reduce(t, op=dist.ReduceOp.MIN, group=st.tp_cpu_group)
    if int(t) == 0:
        if comm is not None:
            comm.close()
        return None
    return comm
