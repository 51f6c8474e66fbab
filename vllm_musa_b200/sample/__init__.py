"""Sampling: parameters and the (vocab-parallel) sampler."""
from .sampling_params import SamplingParams  # noqa: F401
