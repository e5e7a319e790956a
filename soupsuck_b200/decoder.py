"""Qwen2 decoder layer with the attention residual add fused into the post-attention RMSNorm.

Reference: solution/decoder.py:54-89 replaces ``Qwen2DecoderLayer.forward``
(transformers modeling_qwen2.py) keeping its signature; the residual add after
attention and ``post_attention_layernorm`` become one ``add_rms_norm`` call
(``sb_add_rmsnorm_fwd`` / ``sb_add_rmsnorm_bwd``), everything else (input norm,
attention with its cache kwargs, MLP, final residual add) runs unchanged.  The
layer returns one tensor, as the pinned transformers version does.
"""

from functools import wraps
import importlib
from types import ModuleType

from .utils import enabled, supported_tensor

_MARKER = "_solution_fused_original"


def _norm_ok(norm, norm_cls, residual, hidden):
    return (type(norm) is norm_cls and supported_tensor(hidden) and supported_tensor(norm.weight)
            and hidden.shape == residual.shape and hidden.device == residual.device == norm.weight.device
            and norm.weight.ndim == 1 and norm.weight.numel() == residual.shape[-1]
            and not norm._forward_hooks and not norm._forward_pre_hooks
            and not norm._backward_hooks and not norm._backward_pre_hooks)


def patch_qwen2_decoder(module=None):
    """Install the Qwen2DecoderLayer patch once; return whether it is active."""
    try:
        import torch

        if module is None:
            module = importlib.import_module("transformers.models.qwen2.modeling_qwen2")
    except (ImportError, AttributeError):
        return False
    if not isinstance(module, ModuleType):
        return False
    cls = getattr(module, "Qwen2DecoderLayer", None)
    norm_cls = getattr(module, "Qwen2RMSNorm", None)
    if (not isinstance(cls, type) or not issubclass(cls, torch.nn.Module)
            or cls.__module__ != module.__name__ or not isinstance(norm_cls, type)):
        return False
    original = cls.forward
    if hasattr(original, _MARKER):
        return True

    @wraps(original)
    def forward(self, hidden_states, attention_mask=None, position_ids=None,
                past_key_values=None, use_cache=False, position_embeddings=None, **kwargs):
        if not enabled() or type(self) is not cls or not supported_tensor(hidden_states):
            return original(self, hidden_states, attention_mask=attention_mask,
                            position_ids=position_ids, past_key_values=past_key_values,
                            use_cache=use_cache, position_embeddings=position_embeddings, **kwargs)
        residual = hidden_states
        hidden_states = self.input_layernorm(hidden_states)
        hidden_states, _ = self.self_attn(
            hidden_states=hidden_states, attention_mask=attention_mask,
            position_ids=position_ids, past_key_values=past_key_values,
            use_cache=use_cache, position_embeddings=position_embeddings, **kwargs)
        norm = self.post_attention_layernorm
        if _norm_ok(norm, norm_cls, residual, hidden_states):
            from .kernels.add_rmsnorm import add_rms_norm

            residual, hidden_states = add_rms_norm(residual, hidden_states, norm.weight,
                                                   norm.variance_epsilon)
        else:
            residual = residual + hidden_states
            hidden_states = norm(residual)
        hidden_states = self.mlp(hidden_states)
        return residual + hidden_states

    setattr(forward, _MARKER, original)
    cls.forward = forward
    return True
