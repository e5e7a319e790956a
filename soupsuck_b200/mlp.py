"""Qwen2MLP.forward as the fused NF4 MLP (reference: the frozen MLP boundary
``patch_qwen2_mlp_fused`` / ``fused_qwen2_mlp``, solution/mlp.py:500-638).

The replacement runs ``kernels.nf4_swiglu_mlp`` -- gate/up in one launch with
the SwiGLU epilogue, down, and in the backward the down dX with the SwiGLU
derivatives in its epilogue and one two-weight gate/up dX -- when every
projection is either a frozen bitsandbytes ``Linear4bit`` (nested fp16 NF4, no
bias, no hooks) or PEFT's LoRA wrapper of one whose adapter the fused GEMM can
carry (one active adapter, no active dropout, gate and up adapted together
with one scaling), the activation is SiLU and x is fp16 on an sm_100 device.
Any other call runs the forward it replaced (marker ``_solution_fused_original``).
"""

from functools import wraps
import math
import numbers

from .utils import enabled, no_hooks, supported_tensor

_MARKER = "_solution_fused_original"


def _bnb_base(module):
    """(packed, quant_state) of a frozen bitsandbytes Linear4bit, or None."""
    import torch

    if (type(module).__module__ != "bitsandbytes.nn.modules" or type(module).__name__ != "Linear4bit"
            or not no_hooks(module) or getattr(module, "bias", None) is not None):
        return None
    weight = getattr(module, "weight", None)
    state = getattr(weight, "quant_state", None)
    if state is None or weight.requires_grad or not weight.is_contiguous():
        return None
    if getattr(module, "compute_dtype", torch.float16) not in (None, torch.float16):
        return None
    from .kernels.nf4 import nested_shape
    packed = weight.data.reshape(-1, 1)
    try:
        nested_shape(packed, state, entry="Qwen2MLP")
    except ValueError:
        return None
    return packed, state


def _projection(module):
    """(packed, state, lora_a, lora_b, scaling) of one MLP projection, or None."""
    import torch

    base = _bnb_base(module)
    if base is not None:
        return (*base, None, None, None)
    if (type(module).__module__ != "peft.tuners.lora.bnb" or type(module).__name__ != "Linear4bit"
            or not no_hooks(module) or module.disable_adapters or module.merged
            or len(module.active_adapters) != 1):
        return None
    name = module.active_adapters[0]
    if (name not in module.lora_A or name not in module.lora_B
            or name in getattr(module, "lora_variant", {}) or getattr(module, "use_dora", {}).get(name, False)):
        return None
    a, b, dropout = module.lora_A[name], module.lora_B[name], module.lora_dropout[name]
    scaling = module.scaling[name]
    active_dropout = type(dropout) is torch.nn.Dropout and dropout.p > 0 and dropout.training
    if (type(a) is not torch.nn.Linear or type(b) is not torch.nn.Linear or a.bias is not None
            or b.bias is not None or active_dropout
            or type(dropout) not in (torch.nn.Dropout, torch.nn.Identity)
            or not all(no_hooks(m) for m in (a, b, dropout))
            or not isinstance(scaling, numbers.Real) or not math.isfinite(scaling)):
        return None
    base = _bnb_base(module.base_layer)
    if base is None:
        return None
    return (*base, a.weight, b.weight, float(scaling))


def _fused_plan(mlp, x):
    """The arguments of nf4_swiglu_mlp for this call, or None."""
    import torch

    if not enabled() or not supported_tensor(x) or x.dtype != torch.float16 or x.ndim < 2:
        return None
    if torch.is_autocast_enabled("cuda") and torch.get_autocast_dtype("cuda") != torch.float16:
        return None
    act = getattr(mlp, "act_fn", None)
    if type(act) is not torch.nn.SiLU and type(act).__name__ != "SiLUActivation":
        return None
    projections = [_projection(getattr(mlp, key, None)) for key in ("gate_proj", "up_proj", "down_proj")]
    if any(p is None for p in projections):
        return None
    (gp, gs, ag, bg, sg), (up, us, au, bu, su), (dp, ds, ad, bd, sd) = projections
    if (ag is None) != (au is None):
        return None
    scales = {s for s in (sg, su, sd) if s is not None}
    if len(scales) > 1:
        return None
    if any(t is not None and t.device != x.device for t in (gp, up, dp)):
        return None
    n, h = gs.shape
    if tuple(us.shape) != (n, h) or tuple(ds.shape) != (h, n) or x.shape[-1] != h or n % 128 or h % 64:
        return None
    for a in (ag, au, ad):
        if a is not None and (a.shape[0] > 32 or a.device != x.device):
            return None
    if ag is not None and ag.shape[0] != au.shape[0]:
        return None
    scaling = scales.pop() if scales else 1.0
    return (gp, gs, ag, bg), (up, us, au, bu), (dp, ds, ad, bd), scaling


def patch_qwen2_mlp(module):
    """Install the fused forward on ``module.Qwen2MLP`` once; True when installed."""
    import torch

    cls = getattr(module, "Qwen2MLP", None)
    if not (isinstance(cls, type) and issubclass(cls, torch.nn.Module) and cls.__module__ == module.__name__):
        return False
    original = cls.forward
    if hasattr(original, _MARKER):
        return True

    def forward(self, x):
        plan = _fused_plan(self, x) if type(self) is cls else None
        if plan is None:
            return original(self, x)
        from .kernels.mlp import nf4_swiglu_mlp
        gate, up, down, scaling = plan
        return nf4_swiglu_mlp(x, gate, up, down, scaling)

    replacement = wraps(original)(forward)
    setattr(replacement, _MARKER, original)
    cls.forward = replacement
    return True
