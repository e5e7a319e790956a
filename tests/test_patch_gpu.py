"""The drop-in on a B200: patched bitsandbytes / PEFT / Qwen2 methods against their originals.

bitsandbytes and PEFT are not installed here, so their two classes on the path
are stood in by minimal modules with the same names, module paths and
attributes the patches inspect (bnb ``Linear4bit`` with a packed NF4 weight
carrying ``quant_state``; PEFT ``Linear4bit`` with ``base_layer``, ``lora_A``,
``lora_B``, ``lora_dropout``, ``scaling``).  Their "original" forwards compute
the reference's math with plain torch ops on the exactly decoded weight
(``dequantize_nf4`` is bit-exact with the reference decoder), so the patched
results are held to the GEMM gate (2e-3 abs + 2e-3 rel, relative L2 1e-3).
Qwen2 is the real transformers implementation on a tiny random config.
"""

import math
import sys
from types import ModuleType

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as O
from tests.helpers import np_of

pytestmark = pytest.mark.gpu


def _gate(actual, expected):
    ok, max_abs, rel = O.gemm_gate(np_of(actual).astype(np.float64), np_of(expected).astype(np.float64))
    assert ok, f"max abs err {max_abs:.3e}, rel-L2 {rel:.3e}"


def _package(monkeypatch, name):
    module = ModuleType(name)
    module.__path__ = []
    monkeypatch.setitem(sys.modules, name, module)
    return module


@pytest.fixture
def fake_bnb_linear(monkeypatch):
    """bitsandbytes.nn.modules.Linear4bit stand-in: frozen NF4 weight, fp16 compute."""
    from soupsuck_b200.kernels import dequantize_nf4

    _package(monkeypatch, "bitsandbytes")
    modules = ModuleType("bitsandbytes.nn.modules")
    monkeypatch.setitem(sys.modules, modules.__name__, modules)

    class Linear4bit(torch.nn.Module):
        def __init__(self, weight16):
            super().__init__()
            from soupsuck_b200.quantize import quantize_nf4
            packed, state = quantize_nf4(weight16)
            self.weight = torch.nn.Parameter(packed, requires_grad=False)
            self.weight.quant_state = state
            self.bias = None
            self.compute_dtype = torch.float16
            self.compute_type_is_set = True

        def forward(self, x):
            w = dequantize_nf4(self.weight, self.weight.quant_state)
            return torch.nn.functional.linear(x.to(torch.float16), w).to(x.dtype)

    Linear4bit.__module__ = modules.__name__
    return Linear4bit


@pytest.fixture
def fake_peft(monkeypatch):
    _package(monkeypatch, "peft")
    module = ModuleType("peft.tuners.lora.bnb")
    module.VARIANT_KWARG_KEYS = ["alora_offsets"]

    class Linear4bit(torch.nn.Module):
        """PEFT LoRA wrapper stand-in; forward is PEFT's math (peft/tuners/lora/bnb.py)."""

        def __init__(self, base, r, scaling, dropout=0.0):
            super().__init__()
            n, k = base.weight.quant_state.shape
            self.base_layer = base
            self.lora_A = torch.nn.ModuleDict({"default": torch.nn.Linear(k, r, bias=False)})
            self.lora_B = torch.nn.ModuleDict({"default": torch.nn.Linear(r, n, bias=False)})
            self.lora_dropout = torch.nn.ModuleDict(
                {"default": torch.nn.Dropout(dropout) if dropout else torch.nn.Identity()})
            self.scaling = {"default": scaling}
            self.active_adapters = ["default"]
            self.disable_adapters = False
            self.merged = False
            self.lora_variant = {}
            self.use_dora = {}

        def _check_forward_args(self, x, *args, **kwargs):
            pass

        def forward(self, x, *args, **kwargs):
            result = self.base_layer(x)
            a, b = self.lora_A["default"], self.lora_B["default"]
            lora_in = self.lora_dropout["default"](x.to(a.weight.dtype))
            lora = torch.nn.functional.linear(
                torch.nn.functional.linear(lora_in.half(), a.weight.half()), b.weight.half())
            return (result.float() + lora.float() * self.scaling["default"]).to(x.dtype)

    Linear4bit.__module__ = module.__name__
    module.Linear4bit = Linear4bit
    monkeypatch.setitem(sys.modules, module.__name__, module)
    return module, Linear4bit


@pytest.mark.parametrize("m,n,k", [(827, 8960, 1536), (300, 256, 1536), (64, 1536, 1536)])
def test_peft_linear4bit_forward_backward(fake_bnb_linear, fake_peft, m, n, k):
    import soupsuck_b200.lora as lora
    import soupsuck_b200.patch as patch

    module, cls = fake_peft
    torch.manual_seed(m)
    w = (torch.randn((n, k), device="cuda") * 0.02).half()
    layer = cls(fake_bnb_linear(w), 16, 2.0).cuda()
    with torch.no_grad():
        layer.lora_A["default"].weight.uniform_(-1 / math.sqrt(k), 1 / math.sqrt(k))
        layer.lora_B["default"].weight.normal_(0, 0.01)
    original = cls.forward
    patch._register_module(module.__name__, module)
    assert getattr(cls.forward, lora._MARKER) is original

    x = torch.randn((m, k), device="cuda", dtype=torch.float16, requires_grad=True)
    dy = torch.randn((m, n), device="cuda", dtype=torch.float16)
    from soupsuck_b200 import _lib
    before = _lib.launch_count()
    y = layer(x)
    assert _lib.launch_count() > before  # the fused path ran
    y.backward(dy)
    got = (y.detach(), x.grad, layer.lora_A["default"].weight.grad, layer.lora_B["default"].weight.grad)
    x.grad = None
    layer.zero_grad()
    y_ref = original(layer, x)
    y_ref.backward(dy)
    ref = (y_ref.detach(), x.grad, layer.lora_A["default"].weight.grad, layer.lora_B["default"].weight.grad)
    assert got[0].dtype == ref[0].dtype == torch.float16
    _gate(got[0], ref[0])
    _gate(got[1], ref[1])
    for g, r in zip(got[2:], ref[2:]):
        rel = (g.double() - r.double()).norm() / r.double().norm()
        assert rel < 2e-3, rel


@pytest.mark.parametrize("x_dtype", [torch.float32, torch.float16])
def test_peft_linear4bit_with_active_dropout_runs_fused_gemm(fake_bnb_linear, fake_peft, x_dtype):
    """Training-mode LoRA dropout: same mask as the reference branch (same RNG
    draw), the fused GEMM on the dropped LoRA input, gradients through the mask."""
    import soupsuck_b200.patch as patch
    from soupsuck_b200 import _lib

    module, cls = fake_peft
    torch.manual_seed(5)
    m, n, k = 300, 1536, 512
    w = (torch.randn((n, k), device="cuda") * 0.02).half()
    layer = cls(fake_bnb_linear(w), 16, 2.0, dropout=0.1).cuda().train()
    with torch.no_grad():
        layer.lora_A["default"].weight.uniform_(-1 / math.sqrt(k), 1 / math.sqrt(k))
        layer.lora_B["default"].weight.normal_(0, 0.05)
    original = cls.forward
    patch._register_module(module.__name__, module)
    x = torch.randn((m, k), device="cuda", dtype=x_dtype, requires_grad=True)
    dy = torch.randn((m, n), device="cuda", dtype=x_dtype)
    torch.manual_seed(7)
    before = _lib.launch_count()
    y = layer(x)
    assert _lib.launch_count() > before
    y.backward(dy)
    got = (y.detach(), x.grad, layer.lora_A["default"].weight.grad, layer.lora_B["default"].weight.grad)
    x.grad = None
    layer.zero_grad()
    torch.manual_seed(7)
    y_ref = original(layer, x)
    y_ref.backward(dy)
    ref = (y_ref.detach(), x.grad, layer.lora_A["default"].weight.grad, layer.lora_B["default"].weight.grad)
    assert got[0].dtype == ref[0].dtype == x_dtype
    _gate(got[0], ref[0])
    _gate(got[1], ref[1])
    for g, r in zip(got[2:], ref[2:]):
        rel = (g.double() - r.double()).norm() / r.double().norm()
        assert rel < 2e-3, rel


def test_matmul_4bit_patch_runs_fused_gemm(monkeypatch, fake_bnb_linear):
    import soupsuck_b200.nf4_patch as nf4_patch
    from soupsuck_b200.kernels import dequantize_nf4

    bnb = sys.modules["bitsandbytes"]

    def original(A, B, quant_state, out=None, bias=None):
        w = dequantize_nf4(B.t().contiguous().view(-1, 1), quant_state)
        return torch.nn.functional.linear(A, w, bias)

    patched = nf4_patch.make_matmul_4bit(original)
    base = fake_bnb_linear((torch.randn((1536, 512), device="cuda") * 0.02).half())
    x = torch.randn((333, 512), device="cuda", dtype=torch.float16, requires_grad=True)
    y = patched(x, base.weight.t(), base.weight.quant_state)
    dy = torch.randn_like(y)
    y.backward(dy)
    dx = x.grad
    x.grad = None
    y_ref = original(x, base.weight.t(), base.weight.quant_state)
    y_ref.backward(dy)
    _gate(y, y_ref)
    _gate(dx, x.grad)
    del bnb


def _tiny_qwen(seed=0):
    import transformers
    from transformers.models.qwen2 import modeling_qwen2 as q

    config = transformers.Qwen2Config(vocab_size=1000, hidden_size=256, intermediate_size=512,
                                      num_hidden_layers=2, num_attention_heads=4,
                                      num_key_value_heads=2, max_position_embeddings=128,
                                      rms_norm_eps=1e-6)
    torch.manual_seed(seed)
    model = q.Qwen2ForCausalLM(config).cuda().half().train()
    model.lm_head.weight.requires_grad_(False)
    return q, model


def test_qwen2_patched_loss_and_gradients_match_original(monkeypatch):
    pytest.importorskip("transformers")
    import soupsuck_b200.patch as patch

    q, model = _tiny_qwen()
    originals = {}
    for cls in (q.Qwen2ForCausalLM, q.Qwen2RMSNorm, q.Qwen2DecoderLayer):
        current = cls.forward
        originals[cls] = getattr(current, patch._MARKER, current)
        monkeypatch.setattr(cls, "forward", originals[cls])
    ids = torch.randint(1000, (3, 40), device="cuda")
    labels = ids.clone()
    labels[0, :5] = -100

    def run():
        model.zero_grad()
        out = model(input_ids=ids, labels=labels)
        out.loss.backward()
        norm_grad = model.model.layers[1].post_attention_layernorm.weight.grad.float().clone()
        q_grad = model.model.layers[0].self_attn.q_proj.weight.grad.float().clone()
        return out, norm_grad, q_grad

    ref_out, ref_norm, ref_q = run()
    patch._register_module(patch._QWEN_MODULE, q)
    for cls, before in originals.items():
        assert getattr(cls.forward, patch._MARKER) is before
    from soupsuck_b200 import _lib
    launches = _lib.launch_count()
    out, norm_grad, q_grad = run()
    assert _lib.launch_count() > launches
    assert out.logits is None and ref_out.logits is not None
    torch.testing.assert_close(out.loss.float(), ref_out.loss.float(), rtol=2e-3, atol=2e-3)
    for got, ref in ((norm_grad, ref_norm), (q_grad, ref_q)):
        rel = (got - ref).norm() / ref.norm()
        assert rel < 2e-2, rel
    step = getattr(model, patch._MODEL_STEP)
    assert step is not None and int(step.labelled) == int((labels[:, 1:] != -100).sum())


def test_qwen2_mlp_patch_runs_fused_mlp_on_nf4_projections(monkeypatch, fake_bnb_linear):
    """Qwen2MLP with frozen bitsandbytes NF4 projections (the reference task's MLP:
    LoRA only on q/v) runs the fused MLP; output and input gradient match the
    original forward on the same decoded weights."""
    import transformers
    from transformers.models.qwen2 import modeling_qwen2 as q

    from soupsuck_b200 import _lib
    from soupsuck_b200.mlp import _MARKER, patch_qwen2_mlp

    current = q.Qwen2MLP.forward
    original = getattr(current, _MARKER, current)
    monkeypatch.setattr(q.Qwen2MLP, "forward", original)
    config = transformers.Qwen2Config(hidden_size=512, intermediate_size=1280, hidden_act="silu")
    torch.manual_seed(11)
    mlp = q.Qwen2MLP(config).cuda()
    for key in ("gate_proj", "up_proj", "down_proj"):
        lin = getattr(mlp, key)
        setattr(mlp, key, fake_bnb_linear((lin.weight.detach() * 0.5).half()).cuda())
    x = torch.randn((3, 100, 512), device="cuda", dtype=torch.float16, requires_grad=True)
    dy = torch.randn((3, 100, 512), device="cuda", dtype=torch.float16)
    ref = original(mlp, x)
    ref.backward(dy)
    ref_dx, x.grad = x.grad, None
    assert patch_qwen2_mlp(q) and getattr(q.Qwen2MLP.forward, _MARKER) is original
    before = _lib.launch_count()
    out = mlp(x)
    assert _lib.launch_count() > before
    out.backward(dy)
    _gate(out.float(), ref.float())
    rel = (x.grad.double() - ref_dx.double()).norm() / ref_dx.double().norm()
    assert rel < 5e-3, rel


def test_qwen2_rope_patch_is_bit_exact_with_eager(monkeypatch):
    from transformers.models.qwen2 import modeling_qwen2 as q

    from soupsuck_b200.rope import _MARKER, patch_qwen2_rope

    current = q.apply_rotary_pos_emb
    original = getattr(current, _MARKER, current)
    monkeypatch.setattr(q, "apply_rotary_pos_emb", original)
    assert patch_qwen2_rope(q) and getattr(q.apply_rotary_pos_emb, _MARKER) is original
    qs = torch.randn(2, 40, 12, 128, device="cuda", dtype=torch.float16).transpose(1, 2)
    ks = torch.randn(2, 40, 2, 128, device="cuda", dtype=torch.float16).transpose(1, 2)
    cos, sin = torch.randn(2, 40, 128, device="cuda"), torch.randn(2, 40, 128, device="cuda")
    got = q.apply_rotary_pos_emb(qs, ks, cos, sin)
    ref = original(qs, ks, cos, sin)
    for a, b in zip(got, ref):
        assert a.dtype == b.dtype and torch.equal(a.contiguous(), b.contiguous())
