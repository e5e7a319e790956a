"""``apply()``: lazy, idempotent installation of the hot-path patches.

The contract (solution/patch.py:425-487, solution/tests/test_integration.py:21-60):
``apply()`` may run before torch, transformers, PEFT or bitsandbytes are
imported and imports none of them; a target module imported later is patched
before its import statement returns; one imported earlier is patched at once;
repeating either route changes nothing (every replaced function carries the
marker attribute ``_solution_fused_original`` naming what it replaced).

Targets:

  transformers.models.qwen2.modeling_qwen2   Qwen2RMSNorm.forward -> rms_norm;
                                              Qwen2DecoderLayer.forward (decoder.py);
                                              Qwen2MLP.forward -> fused NF4 MLP (mlp.py);
                                              apply_rotary_pos_emb -> fused q/k RoPE (rope.py);
                                              Qwen2ForCausalLM.forward -> fused head, no logits
  peft.tuners.lora.bnb                        Linear4bit.forward -> fused NF4 + LoRA (lora.py)
  bitsandbytes(.functional, .backends.cuda.ops)  NF4 decode and matmul_4bit (nf4_patch.py)

Mechanism: a ``sys.meta_path`` finder that only answers for the watched names.
It resolves the spec through the finders behind it and swaps in a loader that
runs the real loader and then this module's patch function for that name.
"""

from functools import wraps
import importlib.abc
import sys
from types import ModuleType

from .utils import enabled, head_fault, supported_tensor

_MARKER = "_solution_fused_original"
_MODEL_STEP = "_solution_fused_step"

_QWEN_MODULE = "transformers.models.qwen2.modeling_qwen2"
_PEFT_BNB_MODULE = "peft.tuners.lora.bnb"
_NF4_MODULES = ("bitsandbytes", "bitsandbytes.functional", "bitsandbytes.backends.cuda.ops")
_TARGET_MODULES = {_QWEN_MODULE, _PEFT_BNB_MODULE, *_NF4_MODULES}

_reported = set()


def _say_once(key, text):
    if key not in _reported:
        _reported.add(key)
        print(f"[soupsuck_b200] {text}", file=sys.stderr, flush=True)


def _replace(cls, make):
    """cls.forward = make(original) once; the replacement remembers the original."""
    original = cls.forward
    if hasattr(original, _MARKER):
        return
    replacement = wraps(original)(make(original))
    setattr(replacement, _MARKER, original)
    cls.forward = replacement


# ------------------------------------------------------------------ Qwen2 patches
def _norm_forward(original):
    """Qwen2RMSNorm.forward(hidden_states) on the RMSNorm kernels
    (reference: solution/patch.py:232-250)."""
    def forward(self, hidden_states):
        weight = self.weight
        if (enabled() and supported_tensor(hidden_states) and supported_tensor(weight)
                and weight.device == hidden_states.device
                and weight.shape == (hidden_states.shape[-1],)):
            from .kernels.rmsnorm import rms_norm
            return rms_norm(hidden_states, weight, self.variance_epsilon)
        return original(self, hidden_states)

    return forward


def _causal_lm_forward(original, lm_cls):
    """Qwen2ForCausalLM.forward whose loss comes from the fused head and whose
    logits are never formed (reference: solution/patch.py:157-229); a call the
    head cannot serve runs the original.  The step's detached statistics are left
    on the model under ``_solution_fused_step``."""
    def forward(self, input_ids=None, attention_mask=None, position_ids=None, past_key_values=None,
                inputs_embeds=None, labels=None, use_cache=None, logits_to_keep=0, **kwargs):
        from transformers.modeling_outputs import CausalLMOutputWithPast

        from .head import fused_head

        setattr(self, _MODEL_STEP, None)
        body = dict(input_ids=input_ids, attention_mask=attention_mask, position_ids=position_ids,
                    past_key_values=past_key_values, inputs_embeds=inputs_embeds, use_cache=use_cache)
        reason = (f"{type(self).__name__} is not exactly Qwen2ForCausalLM" if type(self) is not lm_cls
                  else head_fault(self, labels, logits_to_keep, **kwargs))
        if reason is not None:
            if self.training:
                _say_once("head-off", f"fused head disabled: {reason}")
            return original(self, labels=labels, logits_to_keep=logits_to_keep, **body, **kwargs)
        decoded = self.model(**body, **{k: v for k, v in kwargs.items() if k != "num_items_in_batch"})
        hidden = decoded.last_hidden_state
        weight = self.lm_head.weight
        if (supported_tensor(hidden) and tuple(hidden.shape[:2]) == tuple(labels.shape)
                and hidden.device == weight.device and hidden.shape[-1] == weight.shape[1]):
            loss, step = fused_head(hidden, weight, labels, kwargs.get("num_items_in_batch"))
            setattr(self, _MODEL_STEP, step)
            logits = None
            _say_once("head-on", "fused head active")
        else:
            _say_once("head-off", "fused head disabled: decoder output does not fit the head")
            logits = self.lm_head(hidden)
            loss = self.loss_function(logits=logits, labels=labels, vocab_size=self.config.vocab_size,
                                      **kwargs)
        return CausalLMOutputWithPast(loss=loss, logits=logits, past_key_values=decoded.past_key_values,
                                      hidden_states=decoded.hidden_states, attentions=decoded.attentions)

    return forward


def _patch_qwen2(module):
    classes = [getattr(module, name, None) for name in ("Qwen2ForCausalLM", "Qwen2RMSNorm",
                                                        "Qwen2DecoderLayer")]
    if not all(isinstance(c, type) and c.__module__ == module.__name__ for c in classes):
        return
    lm_cls, norm_cls, _ = classes
    _replace(lm_cls, lambda original: _causal_lm_forward(original, lm_cls))
    _replace(norm_cls, _norm_forward)
    from .decoder import patch_qwen2_decoder
    from .mlp import patch_qwen2_mlp
    from .rope import patch_qwen2_rope
    patch_qwen2_decoder(module)
    patch_qwen2_mlp(module)
    patch_qwen2_rope(module)


def _patch_peft(module):
    cls = getattr(module, "Linear4bit", None)
    if isinstance(cls, type) and cls.__module__ == module.__name__:
        from .lora import _patch_class
        _patch_class(cls, tuple(getattr(module, "VARIANT_KWARG_KEYS", ())))


def _patch_bitsandbytes(module):
    # The three bitsandbytes modules import one another; patch once all of them
    # have finished executing (a module still initialising has _initializing set).
    loaded = [sys.modules.get(name) for name in _NF4_MODULES]
    if not all(isinstance(m, ModuleType) for m in loaded):
        return
    if any(m is not module and getattr(getattr(m, "__spec__", None), "_initializing", False)
           for m in loaded):
        return
    from .nf4_patch import patch_bnb_dequant
    patch_bnb_dequant()


_PATCHERS = {_QWEN_MODULE: _patch_qwen2, _PEFT_BNB_MODULE: _patch_peft,
             **{name: _patch_bitsandbytes for name in _NF4_MODULES}}


def _register_module(name, module):
    """Run the patch function for ``name`` on a module that finished executing.
    Stand-in modules outside a real package (no ``__path__`` on the root) are skipped."""
    root = sys.modules.get(name.split(".")[0])
    if not isinstance(module, ModuleType) or not isinstance(root, ModuleType) \
            or not hasattr(root, "__path__"):
        return
    patcher = _PATCHERS.get(name)
    if patcher is not None:
        patcher(module)


# ------------------------------------------------------------------ import hook
class _AfterExec(importlib.abc.Loader):
    """Loader that runs ``inner`` and then the post-import action for ``name``."""

    def __init__(self, inner, name):
        self._inner, self._name = inner, name

    def create_module(self, spec):
        make = getattr(self._inner, "create_module", None)
        return None if make is None else make(spec)

    def exec_module(self, module):
        self._inner.exec_module(module)
        _register_module(self._name, module)

    def __getattr__(self, attr):  # get_code, get_source, is_package, ... of the real loader
        return getattr(self._inner, attr)


class _ImportWatch(importlib.abc.MetaPathFinder):
    """Answers only for the watched module names, with the spec the finders behind
    it produce and a loader that patches after executing."""

    def __init__(self):
        self._resolving = set()

    def find_spec(self, fullname, path=None, target=None):
        if fullname not in _TARGET_MODULES or fullname in self._resolving:
            return None
        self._resolving.add(fullname)
        try:
            spec = None
            for finder in sys.meta_path:
                if finder is self or not hasattr(finder, "find_spec"):
                    continue
                spec = finder.find_spec(fullname, path, target)
                if spec is not None:
                    break
        finally:
            self._resolving.discard(fullname)
        if spec is not None and spec.loader is not None and hasattr(spec.loader, "exec_module"):
            spec.loader = _AfterExec(spec.loader, fullname)
        return spec


_watch = None


def install():
    """Put the import watch first on sys.meta_path (once) and patch the targets
    that are already imported."""
    global _watch
    if _watch is None:
        _watch = _ImportWatch()
        sys.meta_path.insert(0, _watch)
    for name in sorted(_TARGET_MODULES):
        if name in sys.modules:
            _register_module(name, sys.modules[name])
