"""Run-time eligibility of the drop-in patches; importing this module imports no torch.

Each check returns None when the sm_100a path can serve a call, or one line
saying why not; the patches then run the library's own code.  The on/off
switch is the reference's ``SOUP_FUSED_DISABLE`` (1/true/yes turns every patch
off).  Only compute-capability 10.x devices qualify: the library is built for
sm_100a alone.
"""

import os

_DISABLE_VALUES = ("1", "true", "yes")


def enabled():
    return os.environ.get("SOUP_FUSED_DISABLE", "0").strip().lower() not in _DISABLE_VALUES


def tensor_fault(x, name):
    """Why ``x`` cannot enter the kernels (not a contiguous fp16/fp32 CUDA tensor on
    an sm_100 device), or None."""
    import torch

    if not isinstance(x, torch.Tensor):
        return f"{name}: {type(x).__name__} is not a tensor"
    if x.device.type != "cuda":
        return f"{name}: on {x.device}, not on a CUDA device"
    if x.dtype not in (torch.float16, torch.float32):
        return f"{name}: dtype {x.dtype} is neither fp16 nor fp32"
    if not x.is_contiguous():
        return f"{name}: strided {tuple(x.stride())}, not contiguous"
    major, minor = torch.cuda.get_device_capability(x.device)
    if major != 10:
        return f"{name}: device is sm_{major}{minor}; the library runs on sm_100 devices"
    return None


def supported_tensor(x):
    return tensor_fault(x, "tensor") is None


def no_hooks(module):
    """No forward/backward hooks and no per-instance forward override."""
    return not (module._forward_hooks or module._forward_pre_hooks or module._backward_hooks
                or module._backward_pre_hooks or "forward" in vars(module))


# Forward options of Qwen2ForCausalLM the fused head does not implement.
_UNSUPPORTED_OPTIONS = ("shift_labels", "softcap", "logit_softcap", "num_logits_to_keep")
_UNSUPPORTED_CONFIG = ("final_logit_softcapping", "logit_softcap", "num_virtual_tokens")


def head_fault(model, labels=None, logits_to_keep=0, **kwargs):
    """Why the fused causal-LM head cannot serve this forward call, or None.

    The conditions are the reference's (solution/utils.py:64-131): training mode,
    non-empty contiguous int64 CUDA labels [batch, seq], no logit slicing,
    soft-capping or custom shifting, ignore_index -100, a qwen2 config without
    tensor-parallel pretraining, a frozen bias-free plain Linear head of
    [vocab, hidden] on the labels' device, and fp16 arithmetic (fp16 autocast,
    or an fp16 head without autocast)."""
    import torch

    def label_fault():
        if not isinstance(labels, torch.Tensor):
            return "no label tensor was passed"
        if labels.device.type != "cuda" or labels.dtype != torch.int64 or not labels.is_contiguous():
            return f"labels must be contiguous int64 on CUDA (got {labels.dtype} on {labels.device})"
        if labels.ndim != 2 or labels.numel() == 0:
            return f"labels of shape {tuple(labels.shape)} are not a non-empty [batch, seq] matrix"
        return None

    def option_fault():
        if isinstance(logits_to_keep, bool) or logits_to_keep != 0:
            return f"logits_to_keep={logits_to_keep!r} asks for logits"
        given = [key for key in _UNSUPPORTED_OPTIONS if key in kwargs]
        if given:
            return f"forward option {given[0]} is not implemented by the fused head"
        if kwargs.get("return_dict") is False:
            return "return_dict=False asks for a tuple output"
        if kwargs.get("ignore_index", -100) != -100:
            return f"ignore_index {kwargs['ignore_index']!r} differs from -100"
        return None

    def config_fault():
        config = model.config
        if getattr(config, "model_type", None) != "qwen2":
            return f"model_type {getattr(config, 'model_type', None)!r} is not qwen2"
        if getattr(config, "pretraining_tp", 1) != 1:
            return f"pretraining_tp {config.pretraining_tp} splits the head"
        for key in _UNSUPPORTED_CONFIG:
            if getattr(config, key, None):
                return f"config.{key} is set"
        if getattr(config, "return_dict", True) is False:
            return "config.return_dict is False"
        return None

    def weight_fault():
        head = model.lm_head
        if type(head) is not torch.nn.Linear or head.bias is not None:
            return f"lm_head is a {type(head).__name__}{' with a bias' if head.bias is not None else ''}"
        weight = head.weight
        if weight.requires_grad:
            return "lm_head.weight is trainable"
        reason = tensor_fault(weight, "lm_head.weight")
        if reason is not None:
            return reason
        if weight.device != labels.device:
            return f"lm_head.weight is on {weight.device}, the labels on {labels.device}"
        config = model.config
        if tuple(weight.shape) != (config.vocab_size, config.hidden_size):
            return f"lm_head.weight {tuple(weight.shape)} does not match the config's vocabulary/hidden sizes"
        if torch.is_autocast_enabled("cuda"):
            dtype = torch.get_autocast_dtype("cuda")
            return None if dtype == torch.float16 else f"autocast runs in {dtype}, not fp16"
        if weight.dtype != torch.float16:
            return f"lm_head.weight is {weight.dtype} and no fp16 autocast is active"
        return None

    if not enabled():
        return "SOUP_FUSED_DISABLE is set"
    if not model.training:
        return "the model is in eval mode"
    for check in (label_fault, option_fault, config_fault, weight_fault):
        reason = check()
        if reason is not None:
            return reason
    return None
