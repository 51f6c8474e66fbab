"""Graph passes that rewrite traced (torch.fx) models onto the fused sm_100a ops."""
from .passes import (AllReduceRMSNormFusionPass, B200PassManager,  # noqa: F401
                     RMSNormQuantFusionPass, SiluMulQuantFusionPass)
