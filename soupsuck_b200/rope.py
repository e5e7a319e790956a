"""Qwen2's ``apply_rotary_pos_emb`` on the fused q/k RoPE kernel (reference:
solution/rope.py:55-80 replaces the module global that Qwen2Attention looks up
at call time).

The replacement takes the kernel when RoPE is enabled, ``unsqueeze_dim`` is 1
and (q, k, cos, sin) fit it (``kernels.rope.rope_fault``: CUDA fp16/fp32, q/k
[B, H, S, even D] with unit column stride, detached cos/sin [1|B, S, D]);
everything else calls the function it replaced, kept under the marker
attribute ``_solution_rope_original``.
"""

from functools import wraps

from .utils import enabled

_MARKER = "_solution_rope_original"


def patch_qwen2_rope(module):
    """Install on ``module.apply_rotary_pos_emb`` once; True when installed."""
    original = getattr(module, "apply_rotary_pos_emb", None)
    if not callable(original):
        return False
    if hasattr(original, _MARKER):
        return True

    def apply_rotary_pos_emb(q, k, cos, sin, unsqueeze_dim=1, **kwargs):
        if enabled() and not kwargs and unsqueeze_dim == 1 and type(unsqueeze_dim) is int:
            from .kernels.rope import fused_rope, rope_fault
            if rope_fault(q, k, cos, sin) is None:
                return fused_rope(q, k, cos, sin)
        return original(q, k, cos, sin, unsqueeze_dim=unsqueeze_dim, **kwargs)

    replacement = wraps(original)(apply_rotary_pos_emb)
    setattr(replacement, _MARKER, original)
    module.apply_rotary_pos_emb = replacement
    return True
