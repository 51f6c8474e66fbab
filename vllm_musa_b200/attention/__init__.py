"""Attention backends and metadata (paged FlashAttention on the sm_100a kernels)."""
from .metadata import AttnMetadata  # noqa: F401
from .backend import (MMEncoderAttention, PagedAttention, TreeAttention,  # noqa: F401
                      TurboQuantAttention)
