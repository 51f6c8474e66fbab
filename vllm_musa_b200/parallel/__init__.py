"""Parallelism: process groups, the NVSwitch TP communicator and its fused collectives."""
from .state import (ParallelState, destroy_distributed, get_parallel_state,  # noqa: F401
                    init_distributed, set_parallel_state)
