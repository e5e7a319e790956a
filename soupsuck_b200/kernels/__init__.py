"""sm_100a kernels of the QLoRA hot path, behind the reference's kernel-level API
(solution/kernels/__init__.py): same names, argument meaning and errors, plus the
fused projections this library adds (``nf4_lora_linear``, ``nf4_swiglu_mlp``)."""

from .cross_entropy import fused_linear_cross_entropy
from .rmsnorm import rms_norm
from .add_rmsnorm import add_rms_norm
from .nf4 import dequantize_nf4
from .nf4_gemm import nf4_matmul, nf4_lora_linear
from .lora_epilogue import lora_epilogue
from .mlp import nf4_swiglu_mlp, swiglu_fused_backward, swiglu_fused_forward
from .rope import fused_rope

__all__ = ["fused_linear_cross_entropy", "rms_norm", "add_rms_norm", "dequantize_nf4",
           "nf4_matmul", "nf4_lora_linear", "lora_epilogue", "nf4_swiglu_mlp",
           "swiglu_fused_forward", "swiglu_fused_backward", "fused_rope"]
