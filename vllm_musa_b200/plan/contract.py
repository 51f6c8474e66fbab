"""Optimisation contract: one frozen decision record per engine, resolved from the model and
execution signatures, naming which of the framework's optimised paths a configuration may use
(``supported``) and which it should use (``preferred``).  Consumers ask the contract instead of
re-deriving model-name and shape predicates; ``B200_*`` environment switches still override.

The preferences encode this pool's measurements: the NVSwitch all-reduce + RMSNorm kernels
beat NCCL at 2-8 ranks; the GEMM epilogue reduce-scatter is measured slower than GEMM + AR and
stays opt-in; the two-head tcgen05 prefill beats the one-head kernel where the GQA group is
even; prefix caching is off for recurrent-state models (a state cannot resume from cached KV).

Reference: vllm_musa/optimization_contract/types.py:1-150 (signatures, features, contract),
vllm_musa/optimization_contract/resolver.py:1-391 (signature extraction + provider dispatch),
vllm_musa/optimization_contract/policy.py:1-317 (consumer queries).
"""
from __future__ import annotations

import logging
from dataclasses import dataclass
from enum import Enum
from typing import Optional

log = logging.getLogger("vllm_musa_b200")


class ModelFamily(str, Enum):
    DENSE = "dense"            # Llama / Qwen2 / Qwen3 decoders
    MOE = "moe"                # Qwen3-MoE
    DEEPSEEK = "deepseek"      # DeepSeek-V2/V3/V3.2 (MLA)
    HYBRID_GDN = "hybrid_gdn"  # Qwen3-Next
    SSM = "ssm"                # Mamba2
    UNKNOWN = "unknown"


class Feature(str, Enum):
    CUDA_GRAPH_DECODE = "engine.cuda_graph_decode"
    PREFIX_CACHING = "engine.prefix_caching"
    FUSED_AR_RMSNORM = "comm.fused_allreduce_rmsnorm"
    GEMM_RS_EPILOGUE = "comm.gemm_reduce_scatter_epilogue"
    VOCAB_PARALLEL_SAMPLING = "sample.vocab_parallel_candidates"
    EP_ALL_TO_ALL = "moe.ep_nvlink_all_to_all"
    PREFILL_TCGEN05 = "attn.prefill_tcgen05"
    PREFILL_TWO_HEADS = "attn.prefill_tcgen05_two_heads"
    GEMM_SPLITK_REDUCE = "gemm.splitk_reduce_grid"
    NORM_QUANT_FP8 = "deepseek.rmsnorm_fp8_quant"
    MLA_DCP = "deepseek.mla_decode_context_parallel"
    SPARSE_INDEXER = "deepseek.sparse_indexer"
    MTP = "spec.mtp"
    EAGLE = "spec.eagle"
    EAGLE3 = "spec.eagle3"
    SPEC_TREE = "spec.token_tree"
    PIPELINE_MICROBATCH = "pp.microbatched_stages"
    GDN_CHUNKED_PREFILL = "gdn.chunked_prefill"
    W4AFP8_EXPERTS = "moe.w4afp8_experts"
    TURBOQUANT_KV = "attn.turboquant_kv_cache"


@dataclass(frozen=True)
class ModelSignature:
    family: ModelFamily
    arch: str
    dtype: str
    quant: Optional[str]
    hidden_size: int
    num_layers: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    num_experts: int
    uses_mla: bool
    sparse_attention: bool
    recurrent_state: bool
    kv_cache_dtype: str = "auto"


@dataclass(frozen=True)
class ExecutionSignature:
    device: str
    tensor_parallel_size: int
    data_parallel_size: int
    pipeline_parallel_size: int
    decode_context_parallel_size: int
    enable_expert_parallel: bool
    use_custom_allreduce: bool
    speculative_method: Optional[str]
    enforce_eager: bool
    block_size: int
    max_num_seqs: int
    speculative_tree: bool = False


@dataclass(frozen=True)
class OptimizationContract:
    model: ModelSignature
    execution: ExecutionSignature
    profile: str
    supported: frozenset
    preferred: frozenset

    def supports(self, f: Feature) -> bool:
        return f in self.supported

    def prefers(self, f: Feature) -> bool:
        return f in self.preferred

    def describe(self) -> str:
        return f"{self.profile}: " + ", ".join(sorted(f.value for f in self.preferred))


def _family(arch: str) -> ModelFamily:
    if arch in ("llama", "qwen3"):
        return ModelFamily.DENSE
    if arch == "qwen3_moe":
        return ModelFamily.MOE
    if arch.startswith("deepseek"):
        return ModelFamily.DEEPSEEK
    if arch == "qwen3_next":
        return ModelFamily.HYBRID_GDN
    if arch == "mamba2":
        return ModelFamily.SSM
    return ModelFamily.UNKNOWN


def model_signature(cfg) -> ModelSignature:
    fam = _family(cfg.arch)
    return ModelSignature(
        family=fam, arch=cfg.arch, dtype=str(cfg.dtype).removeprefix("torch."),
        quant=cfg.quant, hidden_size=cfg.hidden_size, num_layers=cfg.num_layers,
        num_heads=cfg.num_heads, num_kv_heads=cfg.num_kv_heads, head_dim=cfg.head_dim,
        num_experts=cfg.num_experts, uses_mla=cfg.kv_lora_rank > 0,
        sparse_attention=cfg.index_topk > 0,
        recurrent_state=fam in (ModelFamily.HYBRID_GDN, ModelFamily.SSM),
        kv_cache_dtype=getattr(cfg, "kv_cache_dtype", "auto") or "auto")


def execution_signature(config) -> ExecutionSignature:
    p = config.parallel
    return ExecutionSignature(
        device=str(config.device).split(":")[0], tensor_parallel_size=p.tensor_parallel_size,
        data_parallel_size=p.data_parallel_size,
        pipeline_parallel_size=p.pipeline_parallel_size,
        decode_context_parallel_size=p.decode_context_parallel_size,
        enable_expert_parallel=p.enable_expert_parallel,
        use_custom_allreduce=p.use_custom_allreduce,
        speculative_method=config.speculative.method, enforce_eager=config.enforce_eager,
        block_size=config.cache.block_size, max_num_seqs=config.scheduler.max_num_seqs,
        speculative_tree=config.speculative.tree)


def resolve(config) -> OptimizationContract:
    """EngineConfig -> contract (pure: no device or process-group queries)."""
    m, e = model_signature(config.model), execution_signature(config)
    cuda = e.device == "cuda"
    tp = e.tensor_parallel_size
    sup, pref = set(), set()

    def both(f: Feature, prefer: bool = True) -> None:
        sup.add(f)
        if prefer:
            pref.add(f)

    if cuda:
        both(Feature.CUDA_GRAPH_DECODE, not e.enforce_eager)
        both(Feature.GEMM_SPLITK_REDUCE)
    both(Feature.PREFIX_CACHING, not m.recurrent_state)
    if tp > 1:
        both(Feature.VOCAB_PARALLEL_SAMPLING)
        if cuda and e.use_custom_allreduce and tp in (2, 4, 8):
            both(Feature.FUSED_AR_RMSNORM)
            both(Feature.GEMM_RS_EPILOGUE, prefer=False)  # measured below GEMM + all-reduce
    if cuda and m.family in (ModelFamily.DENSE, ModelFamily.MOE, ModelFamily.HYBRID_GDN) \
            and m.head_dim == 128:
        both(Feature.PREFILL_TCGEN05)
        heads = m.num_heads // max(1, tp)
        kv = max(1, m.num_kv_heads // max(1, tp))
        if heads % kv == 0 and (heads // kv) % 2 == 0:
            both(Feature.PREFILL_TWO_HEADS)
    if m.num_experts and e.enable_expert_parallel and tp > 1:
        both(Feature.EP_ALL_TO_ALL, cuda and tp in (2, 4, 8))
    if m.family == ModelFamily.DEEPSEEK:
        if m.quant in ("fp8_block", "w4afp8") and m.dtype == "bfloat16":
            both(Feature.NORM_QUANT_FP8)
        if m.sparse_attention:
            both(Feature.SPARSE_INDEXER)
        if e.decode_context_parallel_size > 1:
            both(Feature.MLA_DCP)
        if e.speculative_method == "mtp":
            both(Feature.MTP)
    if m.family == ModelFamily.DENSE and e.speculative_method == "eagle":
        both(Feature.EAGLE)
    if m.family == ModelFamily.DENSE and e.speculative_method == "eagle3":
        both(Feature.EAGLE3)
    if e.speculative_tree:
        both(Feature.SPEC_TREE)
    if m.quant == "w4afp8" and m.num_experts:
        both(Feature.W4AFP8_EXPERTS)
    if m.family == ModelFamily.HYBRID_GDN and cuda:
        both(Feature.GDN_CHUNKED_PREFILL)
    if _quantized_kv(m.kv_cache_dtype) and m.family == ModelFamily.DENSE:
        both(Feature.TURBOQUANT_KV)
    if e.pipeline_parallel_size > 1:
        both(Feature.PIPELINE_MICROBATCH)
    parts = [m.family.value, m.quant or m.dtype, f"tp{tp}"]
    if e.pipeline_parallel_size > 1:
        parts.append(f"pp{e.pipeline_parallel_size}")
    if e.data_parallel_size > 1:
        parts.append(f"dp{e.data_parallel_size}")
    if e.enable_expert_parallel:
        parts.append("ep")
    if e.decode_context_parallel_size > 1:
        parts.append(f"dcp{e.decode_context_parallel_size}")
    return OptimizationContract(m, e, "-".join(parts), frozenset(sup), frozenset(pref))


def _quantized_kv(kv_cache_dtype: str) -> bool:
    """fp8 (e4m3 keys and values, per-vector scales) or a TurboQuant format."""
    return kv_cache_dtype.startswith("turboquant") or kv_cache_dtype in ("fp8", "fp8_e4m3")


def validate(contract: OptimizationContract) -> None:
    """Fail closed on combinations no path serves."""
    m, e = contract.model, contract.execution
    if e.decode_context_parallel_size > 1 and not m.uses_mla:
        raise ValueError("decode context parallelism is implemented for MLA (DeepSeek) models")
    if m.kv_cache_dtype not in ("auto", "bf16", "bfloat16"):
        if not _quantized_kv(m.kv_cache_dtype):
            raise ValueError(f"kv_cache_dtype {m.kv_cache_dtype!r} is not served")
        if m.family != ModelFamily.DENSE or m.uses_mla:
            raise ValueError("quantised KV caches (fp8, TurboQuant) serve the dense decoders "
                             "(no MLA, recurrent or MoE families)")
    if e.speculative_method == "mtp" and m.family != ModelFamily.DEEPSEEK:
        raise ValueError("MTP speculative decoding needs a DeepSeek multi-token-prediction layer")
    if e.speculative_method == "eagle3":
        if m.family != ModelFamily.DENSE or m.kv_cache_dtype not in ("auto", "bf16", "bfloat16"):
            raise ValueError("EAGLE-3 heads are served over the dense decoders with a bf16 KV "
                             "cache")
        if e.tensor_parallel_size > 1 or e.pipeline_parallel_size > 1:
            raise ValueError("EAGLE-3 is served at tensor / pipeline parallel size 1 (its "
                             "features are the target's full residual streams)")
    if e.speculative_method == "eagle":
        if m.family != ModelFamily.DENSE:
            raise ValueError("EAGLE heads are served over the dense decoders (Llama / Qwen)")
        if m.kv_cache_dtype not in ("auto", "bf16", "bfloat16"):
            raise ValueError("EAGLE drafts need a bf16 KV cache")
    if e.pipeline_parallel_size > 1:
        if m.family not in (ModelFamily.DENSE, ModelFamily.MOE):
            raise ValueError("pipeline parallelism is served for the dense and MoE decoders")
        if e.speculative_method in ("mtp", "eagle", "eagle3") or \
                e.decode_context_parallel_size > 1:
            raise ValueError("pipeline parallelism does not combine with model-based drafters "
                             "or decode context parallelism")
        if m.num_layers < e.pipeline_parallel_size:
            raise ValueError("pipeline_parallel_size exceeds the number of layers")
    if e.speculative_tree:
        if e.speculative_method not in ("ngram", "eagle", "eagle3", "medusa"):
            raise ValueError("token trees are proposed by the ngram, EAGLE and Medusa drafters")
        if m.family != ModelFamily.DENSE or m.kv_cache_dtype not in ("auto", "bf16", "bfloat16"):
            raise ValueError("token-tree verification runs the paged bf16 attention of the "
                             "dense decoders (Llama / Qwen)")
    if e.speculative_method == "medusa":
        if m.family not in (ModelFamily.DENSE, ModelFamily.MOE) or e.pipeline_parallel_size > 1:
            raise ValueError("Medusa heads are served over the dense and MoE decoders without "
                             "pipeline stages")
    if e.speculative_method not in (None, "ngram", "mtp", "eagle", "eagle3", "medusa"):
        raise ValueError(f"speculative method {e.speculative_method!r} is not served")
