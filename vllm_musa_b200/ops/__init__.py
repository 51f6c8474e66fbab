"""Op layer: Python entry points over the sm_100a kernels (``torch.ops.b200.*``).

Every function takes and returns torch tensors.  CUDA tensors go to the hand-written kernels
(the extension must be loaded, otherwise the call raises); CPU tensors go to plain PyTorch
implementations of the same math, which serve the tiny CPU configuration and double as the
numerics oracle of the kernel tests.
"""
from . import _ext  # noqa: F401
from .activation import act_and_mul, silu_and_mul  # noqa: F401
from .attention import paged_decode, paged_prefill, varlen_attention  # noqa: F401
from .gemm import linear, linear_silu_mul, interleave_gate_up  # noqa: F401
from .misc import embedding, gather_rows  # noqa: F401
from .norm import fused_add_rms_norm, rms_norm, rms_norm_gated, rms_norm_quant_fp8  # noqa: F401
from .rope import build_cos_sin_cache, rope_kv  # noqa: F401
from .sampling import apply_penalties, sample_tokens  # noqa: F401
