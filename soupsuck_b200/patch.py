"""Import-hook installation of the hot-path patches (the drop-in for ``solution.apply()``).

Mirror of the reference's solution/patch.py:425-487: a ``sys.meta_path`` finder
wraps the loaders of a fixed set of target modules so that each is patched
right after it executes and before the importer sees it; modules imported
before ``install()`` are patched immediately.  Marker attributes on every
replaced function keep both routes idempotent.  The targets and what they get:

* ``transformers.models.qwen2.modeling_qwen2`` - ``Qwen2RMSNorm.forward``
  (``rms_norm``), ``Qwen2DecoderLayer.forward`` (residual add fused into the
  post-attention norm) and ``Qwen2ForCausalLM.forward`` (fused linear CE head);
* ``peft.tuners.lora.bnb`` - ``Linear4bit.forward`` (fused NF4 + LoRA GEMM);
* ``bitsandbytes``, ``bitsandbytes.functional``,
  ``bitsandbytes.backends.cuda.ops`` - NF4 dequantize and ``matmul_4bit``.

Only the hot path is patched: the reference's trainer-metrics bridge, Soup's
setup hooks, unpadding, RoPE and MLP fusions are not part of it.  Nothing here
imports torch, transformers, peft or bitsandbytes at ``install()`` time.
"""

from functools import wraps
from importlib.machinery import PathFinder
import sys
from types import ModuleType

from .utils import enabled, head_ineligibility, supported_tensor

_MARKER = "_solution_fused_original"
_MODEL_STEP = "_solution_fused_step"
_DIAGNOSTICS = set()

_QWEN_MODULE = "transformers.models.qwen2.modeling_qwen2"
_PEFT_BNB_MODULE = "peft.tuners.lora.bnb"
_NF4_MODULES = {"bitsandbytes", "bitsandbytes.functional", "bitsandbytes.backends.cuda.ops"}
_TARGET_MODULES = {_QWEN_MODULE, _PEFT_BNB_MODULE, *_NF4_MODULES}
_IMPORT_FINDER = None


def _mark(wrapper, original):
    setattr(wrapper, _MARKER, original)
    return wrapper


def _report_head(reason=None):
    """One line per process for the first refusal and the first activation of the fused head."""
    key = "disabled" if reason is not None else "active"
    if key not in _DIAGNOSTICS:
        _DIAGNOSTICS.add(key)
        message = f"disabled: {reason}" if reason is not None else "active"
        print(f"[soupsuck_b200] fused head {message}", file=sys.stderr, flush=True)


def _patch_norm(cls):
    """Qwen2RMSNorm.forward(hidden_states) -> rms_norm (reference patch.py:232-250)."""
    original = cls.forward
    if hasattr(original, _MARKER):
        return

    @wraps(original)
    def forward(self, hidden_states):
        if (enabled() and supported_tensor(hidden_states) and supported_tensor(self.weight)
                and hidden_states.device == self.weight.device
                and hidden_states.shape[-1] == self.weight.numel()):
            from .kernels.rmsnorm import rms_norm

            return rms_norm(hidden_states, self.weight, self.variance_epsilon)
        return original(self, hidden_states)

    cls.forward = _mark(forward, original)


def _patch_head(cls):
    """Qwen2ForCausalLM.forward with the loss from the fused head and no logits
    (reference patch.py:157-229); any ineligible call runs the original."""
    original = cls.forward
    if hasattr(original, _MARKER):
        return

    @wraps(original)
    def forward(self, input_ids=None, attention_mask=None, position_ids=None,
                past_key_values=None, inputs_embeds=None, labels=None,
                use_cache=None, logits_to_keep=0, **kwargs):
        from transformers.modeling_outputs import CausalLMOutputWithPast

        from .head import fused_head

        setattr(self, _MODEL_STEP, None)
        arguments = dict(input_ids=input_ids, attention_mask=attention_mask,
                         position_ids=position_ids, past_key_values=past_key_values,
                         inputs_embeds=inputs_embeds, use_cache=use_cache, **kwargs)
        if type(self) is not cls:
            reason = f"model type is {type(self).__name__} (requires exact Qwen2ForCausalLM)"
        else:
            reason = head_ineligibility(self, labels, logits_to_keep, **kwargs)
        if reason is not None:
            if self.training:
                _report_head(reason)
            return original(self, labels=labels, logits_to_keep=logits_to_keep, **arguments)
        model_kwargs = {k: v for k, v in arguments.items() if k != "num_items_in_batch"}
        outputs = self.model(**model_kwargs)
        hidden = outputs.last_hidden_state
        if (not supported_tensor(hidden) or hidden.shape[:2] != labels.shape
                or hidden.device != self.lm_head.weight.device
                or hidden.shape[-1] != self.lm_head.weight.shape[1]):
            _report_head("decoder output does not fit the fused head")
            logits = self.lm_head(hidden)
            loss = self.loss_function(logits=logits, labels=labels,
                                      vocab_size=self.config.vocab_size, **kwargs)
        else:
            loss, step = fused_head(hidden, self.lm_head.weight, labels,
                                    kwargs.get("num_items_in_batch"))
            setattr(self, _MODEL_STEP, step)
            logits = None
            _report_head()
        return CausalLMOutputWithPast(loss=loss, logits=logits,
                                      past_key_values=outputs.past_key_values,
                                      hidden_states=outputs.hidden_states,
                                      attentions=outputs.attentions)

    cls.forward = _mark(forward, original)


def _register_module(name, module):
    """Patch one freshly executed target module (fakes that do not look real are ignored)."""
    root = sys.modules.get(name.split(".")[0])
    if (not isinstance(module, ModuleType) or not isinstance(root, ModuleType)
            or not hasattr(root, "__path__")):
        return
    if name == _QWEN_MODULE:
        names = ("Qwen2ForCausalLM", "Qwen2RMSNorm", "Qwen2DecoderLayer")
        if not all(isinstance(getattr(module, key, None), type)
                   and getattr(module, key).__module__ == name for key in names):
            return
        _patch_head(module.Qwen2ForCausalLM)
        _patch_norm(module.Qwen2RMSNorm)
        from .decoder import patch_qwen2_decoder

        patch_qwen2_decoder(module)
    elif name == _PEFT_BNB_MODULE:
        cls = getattr(module, "Linear4bit", None)
        if isinstance(cls, type) and cls.__module__ == name:
            from .lora import _patch_class

            _patch_class(cls, tuple(getattr(module, "VARIANT_KWARG_KEYS", ())))
    elif name in _NF4_MODULES:
        loaded = {key: sys.modules.get(key) for key in _NF4_MODULES}
        if not all(isinstance(value, ModuleType) for value in loaded.values()):
            return
        # bitsandbytes' submodules import each other; patch only once all three
        # have finished executing.
        if any(key != name and getattr(getattr(value, "__spec__", None), "_initializing", False)
               for key, value in loaded.items()):
            return
        from .nf4_patch import patch_bnb_dequant

        patch_bnb_dequant()


class _PatchLoader:
    def __init__(self, loader, name):
        self.loader, self.name = loader, name

    def create_module(self, spec):
        create = getattr(self.loader, "create_module", None)
        return create(spec) if create is not None else None

    def exec_module(self, module):
        self.loader.exec_module(module)
        _register_module(self.name, module)

    def __getattr__(self, name):
        return getattr(self.loader, name)


class _PatchFinder:
    def find_spec(self, fullname, path=None, target=None):
        if fullname not in _TARGET_MODULES:
            return None
        spec = PathFinder.find_spec(fullname, path, target)
        if spec is not None and hasattr(spec.loader, "exec_module"):
            spec.loader = _PatchLoader(spec.loader, fullname)
        return spec


def install():
    """Register the import hook once and patch target modules that are already imported."""
    global _IMPORT_FINDER
    if _IMPORT_FINDER is None:
        _IMPORT_FINDER = _PatchFinder()
        sys.meta_path.insert(0, _IMPORT_FINDER)
    for name in sorted(_TARGET_MODULES):
        module = sys.modules.get(name)
        if module is not None:
            _register_module(name, module)

