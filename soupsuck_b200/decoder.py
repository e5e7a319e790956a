"""Qwen2 decoder layer whose attention residual add runs inside the next RMSNorm.

The reference patches ``Qwen2DecoderLayer.forward`` (solution/decoder.py:54-89)
so that ``residual + attention_output`` and ``post_attention_layernorm`` become
one fused call.  The layer computes, as transformers' implementation does,

    attended      = self_attn(input_layernorm(x), ...)
    stream, normed = add_rms_norm(x, attended, post_attention_layernorm.weight, eps)
    return stream + mlp(normed)

where the middle line is the single ``sb_add_rmsnorm_fwd`` / ``_bwd`` row kernel
pair.  The replacement keeps the original's signature (the reference's tests
assert it) and calls the original whenever the patch is disabled, the layer is a
subclass, or the hidden states cannot enter the kernels; a post-attention norm
that cannot be fused (another class, hooks, a shape or device mismatch) runs
unfused inside the patched forward.
"""

from functools import wraps

from .utils import enabled, no_hooks, supported_tensor

_MARKER = "_solution_fused_original"


def _norm_fault(norm, norm_cls, stream, update):
    """Why ``norm`` cannot take the fused residual add, or None."""
    if type(norm) is not norm_cls:
        return "post-attention norm is not a plain Qwen2RMSNorm"
    if not no_hooks(norm):
        return "post-attention norm has hooks"
    weight = norm.weight
    if not (supported_tensor(update) and supported_tensor(weight)):
        return "attention output or norm weight is not a kernel operand"
    if update.shape != stream.shape or weight.shape != (stream.shape[-1],):
        return "shapes of the residual stream, attention output and norm weight disagree"
    if not (update.device == stream.device == weight.device):
        return "operands on different devices"
    return None


def _add_then_norm(norm, norm_cls, stream, update):
    if _norm_fault(norm, norm_cls, stream, update) is None:
        from .kernels.add_rmsnorm import add_rms_norm
        return add_rms_norm(stream, update, norm.weight, norm.variance_epsilon)
    total = stream + update
    return total, norm(total)


def _layer_forward(original, layer_cls, norm_cls):
    def forward(self, hidden_states, attention_mask=None, position_ids=None,
                past_key_values=None, use_cache=False, position_embeddings=None, **kwargs):
        attention_args = dict(attention_mask=attention_mask, position_ids=position_ids,
                              past_key_values=past_key_values, use_cache=use_cache,
                              position_embeddings=position_embeddings, **kwargs)
        if not enabled() or type(self) is not layer_cls or not supported_tensor(hidden_states):
            return original(self, hidden_states, **attention_args)
        attended, _weights = self.self_attn(hidden_states=self.input_layernorm(hidden_states),
                                            **attention_args)
        stream, normed = _add_then_norm(self.post_attention_layernorm, norm_cls, hidden_states, attended)
        return stream + self.mlp(normed)

    return forward


def patch_qwen2_decoder(module):
    """Install the fused forward on ``module.Qwen2DecoderLayer`` once (True when active)."""
    import torch

    layer_cls = getattr(module, "Qwen2DecoderLayer", None)
    norm_cls = getattr(module, "Qwen2RMSNorm", None)
    if not (isinstance(layer_cls, type) and issubclass(layer_cls, torch.nn.Module)
            and layer_cls.__module__ == module.__name__ and isinstance(norm_cls, type)):
        return False
    original = layer_cls.forward
    if not hasattr(original, _MARKER):
        replacement = wraps(original)(_layer_forward(original, layer_cls, norm_cls))
        setattr(replacement, _MARKER, original)
        layer_cls.forward = replacement
    return True
