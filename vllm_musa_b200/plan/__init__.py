"""Execution planning: the optimisation contract resolved once per engine."""
from .contract import (ExecutionSignature, Feature, ModelFamily, ModelSignature,  # noqa: F401
                       OptimizationContract, resolve, validate)
