"""Model-side adapter of the ALUT path: the cached MoE layer forward on the ALUT kernels."""
from .fused_moe import ALUTCachedMoE

__all__ = ["ALUTCachedMoE"]
