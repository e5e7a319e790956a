"""Runtime eligibility checks for the patches; nothing here imports CUDA code.

Mirror of the reference's solution/utils.py:1-40 (``enabled``,
``tensor_ineligibility``, ``supported_tensor``) with one difference: the
kernels behind these patches are compiled for sm_100a only, so a tensor is
supported only on a compute-capability 10.x device.
"""

import os


def enabled():
    """Developer switch shared with the reference (SOUP_FUSED_DISABLE=1 turns every patch off)."""
    return os.environ.get("SOUP_FUSED_DISABLE", "0").lower() not in {"1", "true", "yes"}


def tensor_ineligibility(x, name):
    """None when ``x`` can enter the sm_100a kernels, else a one-line reason."""
    import torch

    if not isinstance(x, torch.Tensor):
        return f"{name} is not a torch.Tensor"
    if not x.is_cuda:
        return f"{name}.device={x.device} (requires CUDA)"
    if x.dtype not in (torch.float16, torch.float32):
        return f"{name}.dtype={x.dtype} (requires fp16/fp32)"
    if not x.is_contiguous():
        return f"{name} is noncontiguous, stride={x.stride()}"
    capability = torch.cuda.get_device_capability(x.device)
    if capability[0] != 10:
        return f"{name} device capability={capability} (requires sm_100)"
    return None


def supported_tensor(x):
    return tensor_ineligibility(x, "tensor") is None


def no_hooks(module):
    """True when no forward/backward hook or instance-level forward override is set."""
    return not (module._forward_hooks or module._forward_pre_hooks or module._backward_hooks
                or module._backward_pre_hooks or "forward" in module.__dict__)


def head_ineligibility(model, labels=None, logits_to_keep=0, **kwargs):
    """First reason the fused causal-LM head cannot serve this call, or None.

    Same conditions as the reference's head check (solution/utils.py:64-124):
    training mode, int64 CUDA labels [B, S], no logit slicing or soft-capping,
    ignore_index -100, a plain bias-free frozen lm_head of [vocab, hidden] and
    fp16 arithmetic (fp16 autocast, or an fp16 weight without autocast).
    """
    import torch

    if not enabled():
        return "SOUP_FUSED_DISABLE is enabled"
    if not model.training:
        return "model.training=False"
    if not isinstance(labels, torch.Tensor) or not labels.is_cuda:
        return "labels are absent or not on CUDA"
    if not labels.is_contiguous() or labels.dtype != torch.int64:
        return "labels must be contiguous int64"
    if labels.ndim != 2 or labels.numel() == 0:
        return f"labels.shape={tuple(labels.shape)} (requires nonempty [B,S])"
    if not isinstance(logits_to_keep, int) or logits_to_keep != 0:
        return f"unsupported logits_to_keep={logits_to_keep!r}"
    for key in ("shift_labels", "softcap", "logit_softcap", "num_logits_to_keep"):
        if key in kwargs:
            return f"unsupported forward option {key}"
    if kwargs.get("return_dict") is False or kwargs.get("ignore_index", -100) != -100:
        return "return_dict=False or ignore_index != -100"
    config = model.config
    if getattr(config, "model_type", None) != "qwen2" or getattr(config, "pretraining_tp", 1) != 1:
        return "not a plain qwen2 config"
    if getattr(config, "final_logit_softcapping", None) or getattr(config, "return_dict", True) is False:
        return "logit soft-capping or return_dict=False in config"
    head = model.lm_head
    if type(head) is not torch.nn.Linear or head.bias is not None or head.weight.requires_grad:
        return "lm_head must be a frozen bias-free nn.Linear"
    reason = tensor_ineligibility(head.weight, "lm_head.weight")
    if reason is not None:
        return reason
    if head.weight.device != labels.device:
        return "lm_head.weight and labels are on different devices"
    if torch.is_autocast_enabled("cuda"):
        dtype = torch.get_autocast_dtype("cuda")
        return None if dtype == torch.float16 else f"CUDA autocast dtype={dtype} (requires fp16)"
    if head.weight.dtype != torch.float16:
        return f"lm_head.weight.dtype={head.weight.dtype} without fp16 autocast"
    return None
