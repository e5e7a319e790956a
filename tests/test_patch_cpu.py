"""Host logic of the drop-in: ``apply()`` registration, import hooks, markers and
fallbacks, checked with fake bitsandbytes / PEFT modules on the CPU.

Follows the reference's CPU-side contracts (solution/tests/test_integration.py:21-60):
a cold ``apply()`` imports no training dependency, a hooked module is patched
before its import returns, every patch is idempotent through its marker, and
anything the kernels cannot take (here: CPU tensors) runs the saved original.
"""

import importlib
import subprocess
import sys
from pathlib import Path
from types import ModuleType, SimpleNamespace

import pytest

ROOT = Path(__file__).resolve().parents[1]


def test_cold_apply_imports_no_training_dependency():
    code = """
import sys
import soupsuck_b200
soupsuck_b200.apply()
soupsuck_b200.apply()
heavy = ('torch', 'triton', 'transformers', 'peft', 'bitsandbytes')
assert not any(name in sys.modules for name in heavy), [n for n in heavy if n in sys.modules]
"""
    subprocess.run([sys.executable, "-c", code], cwd=ROOT, check=True)


def test_import_hook_patches_before_import_returns(monkeypatch, tmp_path):
    import soupsuck_b200.patch as patch

    name = "soupsuck_lazy_fixture"
    (tmp_path / f"{name}.py").write_text("class Example:\n    value = 1\n")
    monkeypatch.syspath_prepend(str(tmp_path))
    monkeypatch.setattr(patch, "_TARGET_MODULES", {name})
    seen = []

    def register(fullname, module):
        if not getattr(module.Example, "patched", False):
            module.Example.value = 2
            module.Example.patched = True
            seen.append(fullname)

    monkeypatch.setattr(patch, "_register_module", register)
    patch.install()
    module = importlib.import_module(name)
    try:
        assert module.Example.value == 2 and seen == [name]
        patch.install()
        assert seen == [name]
        importlib.reload(module)
        assert module.Example.value == 2 and seen == [name, name]
    finally:
        sys.modules.pop(name, None)


def _fake_package(monkeypatch, name):
    module = ModuleType(name)
    module.__path__ = []
    monkeypatch.setitem(sys.modules, name, module)
    return module


def _fake_bnb(monkeypatch, version="0.50.2"):
    calls = []
    bnb = _fake_package(monkeypatch, "bitsandbytes")
    bnb.__version__ = version
    functional = ModuleType("bitsandbytes.functional")
    backend = ModuleType("bitsandbytes.backends.cuda.ops")

    def dequantize_4bit(A, quant_state=None, absmax=None, out=None, blocksize=None, quant_type="fp4"):
        calls.append("functional")
        return "functional-original"

    def _dequantize_4bit_impl(A, absmax, blocksize, quant_type, dtype, out):
        calls.append("backend")

    def _dequant_linear_fallback(A, B, shapeB, absmax, blocksize, quant_type, bias=None,
                                 absmax_8bit=None, absmax_code=None, absmax_offset=None):
        import soupsuck_b200.nf4_patch as nf4_patch
        calls.append(("linear", nf4_patch._NESTED_BACKEND.get()))
        return backend._dequantize_4bit_impl(B, absmax, blocksize, quant_type, "fp16", None)

    def matmul_4bit(A, B, quant_state, out=None, bias=None):
        calls.append("matmul")
        return "matmul-original"

    functional.dequantize_4bit = dequantize_4bit
    backend._dequantize_4bit_impl = _dequantize_4bit_impl
    backend._dequant_linear_fallback = _dequant_linear_fallback
    bnb.matmul_4bit = matmul_4bit
    monkeypatch.setitem(sys.modules, "bitsandbytes.functional", functional)
    monkeypatch.setitem(sys.modules, "bitsandbytes.backends.cuda.ops", backend)
    return bnb, functional, backend, calls


def test_bnb_patch_is_idempotent_and_falls_back_on_cpu(monkeypatch):
    import torch

    import soupsuck_b200.nf4_patch as nf4_patch
    import soupsuck_b200.patch as patch

    bnb, functional, backend, calls = _fake_bnb(monkeypatch)
    originals = (functional.dequantize_4bit, backend._dequantize_4bit_impl,
                 backend._dequant_linear_fallback, bnb.matmul_4bit)
    patch._register_module("bitsandbytes.functional", functional)
    patched = (functional.dequantize_4bit, backend._dequantize_4bit_impl,
               backend._dequant_linear_fallback, bnb.matmul_4bit)
    for before, after in zip(originals, patched):
        assert after is not before and getattr(after, nf4_patch._MARKER) is before
    patch._register_module("bitsandbytes", bnb)
    assert (functional.dequantize_4bit, backend._dequantize_4bit_impl,
            backend._dequant_linear_fallback, bnb.matmul_4bit) == patched

    packed = torch.zeros((8, 1), dtype=torch.uint8)
    assert functional.dequantize_4bit(packed, quant_state=None) == "functional-original"
    x = torch.zeros((2, 16), dtype=torch.float16)
    assert bnb.matmul_4bit(x, packed.t(), SimpleNamespace(shape=(1, 16))) == "matmul-original"
    # The nested scope is visible only inside _dequant_linear_fallback, and a CPU
    # buffer is refused by the flat decoder's validation, so the original runs.
    backend._dequant_linear_fallback(x, packed, (1, 16), torch.ones(1), 64, "nf4",
                                     absmax_8bit=torch.ones(1, dtype=torch.uint8))
    assert calls == ["functional", "matmul", ("linear", True), "backend"]
    assert nf4_patch._NESTED_BACKEND.get() is False


def test_bnb_other_versions_are_left_alone(monkeypatch):
    import soupsuck_b200.nf4_patch as nf4_patch

    bnb, functional, backend, _ = _fake_bnb(monkeypatch, version="0.49.0")
    original = functional.dequantize_4bit
    assert nf4_patch.patch_bnb_dequant() is False
    assert functional.dequantize_4bit is original


def test_disable_switch_routes_to_original(monkeypatch):
    import torch

    import soupsuck_b200.nf4_patch as nf4_patch

    bnb, functional, _, calls = _fake_bnb(monkeypatch)
    assert nf4_patch.patch_bnb_dequant()
    monkeypatch.setenv("SOUP_FUSED_DISABLE", "1")
    assert functional.dequantize_4bit(torch.zeros(4, dtype=torch.uint8)) == "functional-original"
    assert calls == ["functional"]


def _fake_peft_linear4bit(monkeypatch):
    import torch

    _fake_package(monkeypatch, "peft")
    module = ModuleType("peft.tuners.lora.bnb")
    module.VARIANT_KWARG_KEYS = ["alora_offsets"]

    class Linear4bit(torch.nn.Module):
        def forward(self, x, *args, **kwargs):
            return "peft-original"

    Linear4bit.__module__ = module.__name__
    module.Linear4bit = Linear4bit
    monkeypatch.setitem(sys.modules, module.__name__, module)
    return module, Linear4bit


def test_peft_linear4bit_patch_marks_and_falls_back(monkeypatch):
    import torch

    import soupsuck_b200.lora as lora
    import soupsuck_b200.patch as patch

    module, cls = _fake_peft_linear4bit(monkeypatch)
    original = cls.forward
    patch._register_module(module.__name__, module)
    assert getattr(cls.forward, lora._MARKER) is original
    patched = cls.forward
    patch._register_module(module.__name__, module)
    assert cls.forward is patched
    layer = cls()
    assert layer(torch.zeros(2, 8)) == "peft-original"  # CPU input: the original runs


def test_qwen2_patches_install_once_and_keep_cpu_results(monkeypatch):
    torch = pytest.importorskip("torch")
    transformers = pytest.importorskip("transformers")
    from transformers.models.qwen2 import modeling_qwen2 as q

    import soupsuck_b200.patch as patch

    # The import hook of an earlier install() may already have patched the module:
    # start from the unpatched methods and restore whatever was there afterwards.
    for cls in (q.Qwen2ForCausalLM, q.Qwen2RMSNorm, q.Qwen2DecoderLayer):
        current = cls.forward
        monkeypatch.setattr(cls, "forward", getattr(current, patch._MARKER, current))
    originals = {cls: cls.forward for cls in (q.Qwen2ForCausalLM, q.Qwen2RMSNorm, q.Qwen2DecoderLayer)}
    patch._register_module(patch._QWEN_MODULE, q)
    for cls, before in originals.items():
        assert getattr(cls.forward, patch._MARKER) is before
    again = {cls: cls.forward for cls in originals}
    patch._register_module(patch._QWEN_MODULE, q)
    assert {cls: cls.forward for cls in originals} == again

    config = transformers.Qwen2Config(vocab_size=64, hidden_size=32, intermediate_size=64,
                                      num_hidden_layers=1, num_attention_heads=4,
                                      num_key_value_heads=2, max_position_embeddings=32)
    torch.manual_seed(0)
    model = q.Qwen2ForCausalLM(config).train()
    ids = torch.randint(64, (2, 8))
    patched = model(input_ids=ids, labels=ids).loss
    for cls, before in originals.items():
        monkeypatch.setattr(cls, "forward", before)
    reference = model(input_ids=ids, labels=ids).loss
    assert torch.equal(patched, reference)  # CPU tensors take the original path
