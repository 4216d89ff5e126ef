from ferrite.kernels.flash_attention import flash_attention, flash_attention_reference
from ferrite.kernels.matmul import matmul, matmul_reference
from ferrite.kernels.rmsnorm import rmsnorm, rmsnorm_reference

__all__ = [
    "flash_attention",
    "flash_attention_reference",
    "matmul",
    "matmul_reference",
    "rmsnorm",
    "rmsnorm_reference",
]
