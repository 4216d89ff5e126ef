"""ferrite on B200: sm_100a CUDA kernels behind ferrite's kernel API.

The three hot-path operators of anxnd2211/ferrite-tpu (causal flash attention,
fused residual-add + RMSNorm, blocked matmul) run as hand-written sm_100a CUDA
kernels in ``_lib/libferrite_b200.so`` behind a C ABI (``include/ferrite_b200.h``),
called through ctypes with torch providing device memory and streams.
"""

from ferrite import platform
from ferrite.kernels.flash_attention import flash_attention
from ferrite.kernels.matmul import matmul
from ferrite.kernels.rmsnorm import rmsnorm

__all__ = ["flash_attention", "matmul", "rmsnorm", "platform"]
__version__ = "0.1.0"
