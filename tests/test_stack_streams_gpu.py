"""The benchmark's 28-layer stack step with k/v and up on a side
stream gives the gradients of the one-stream step.

bench.stack_step runs k/v beside q and up beside gate; tensors that cross
streams are recorded on the reading stream.  Every kernel is deterministic, so
the only difference allowed is the order in which autograd adds the input
gradients of projections that share an input (q/k/v, gate/up), which then
propagates down the layers: compared at 1e-2 relative L2 for the input and the
LoRA weight gradients.
"""

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _grads(bench, layers, tokens, side):
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(11)
    x = torch.randn((tokens, bench.HIDDEN), device=dev, dtype=torch.float16, generator=g).requires_grad_()
    d = torch.randn((tokens, bench.HIDDEN), device=dev, dtype=torch.float16, generator=g).requires_grad_()
    go = torch.randn((tokens, bench.HIDDEN), device=dev, dtype=torch.float16, generator=g)
    gkv = torch.randn((tokens, bench.KV), device=dev, dtype=torch.float16, generator=g)
    params = [p for layer in layers for p in bench.lora_params(layer)]
    for p in params:
        p.grad = None
    bench.stack_step(torch, layers, x, d, go, gkv, side=side)
    torch.cuda.synchronize()
    return [x.grad.clone(), d.grad.clone()] + [p.grad.clone() for p in params]


@pytest.mark.parametrize("tokens", [256, 1152])
def test_streamed_stack_step_matches_one_stream(tokens):
    import bench
    dev = torch.device("cuda", 0)
    layers = [bench.build_layer(torch, dev, seed=40 + i) for i in range(3)]
    ref = _grads(bench, layers, tokens, None)
    side = torch.cuda.Stream(dev)
    for _ in range(2):
        got = _grads(bench, layers, tokens, side)
        for i, (a, b) in enumerate(zip(got, ref)):
            assert torch.isfinite(a).all(), i
            rel = (a.float() - b.float()).norm() / b.float().norm()
            assert rel < 1e-2, f"gradient {i}: relative L2 {rel:.3e}"
    from soupsuck_b200 import _lib
    assert _lib.take_device_error(dev) == 0
