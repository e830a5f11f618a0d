"""Public fused-op surface (parity with the reference's ``pluggy/kernels/__init__.py:12-24``).

Every op runs this package's sm_100a kernels on CUDA tensors and the same math
in eager PyTorch on CPU tensors (the oracle the CPU test-suite uses).
"""

from pluggy_b200.ops.attention import flash_attention
from pluggy_b200.ops.ce import fused_linear_cross_entropy
from pluggy_b200.ops.elementwise import apply_rotary, geglu_mul, logit_softcap, rotate_half, swiglu_mul
from pluggy_b200.ops.linear import WeightCache, linear
from pluggy_b200.ops.moe import moe_expert_ffn
from pluggy_b200.ops.norm import rms_norm

__all__ = [
    "apply_rotary",
    "flash_attention",
    "fused_linear_cross_entropy",
    "geglu_mul",
    "linear",
    "logit_softcap",
    "moe_expert_ffn",
    "rms_norm",
    "rotate_half",
    "swiglu_mul",
    "WeightCache",
]
