"""The benchmark's decoder-layer step with its independent projections on side
streams gives the gradients of the one-stream step.

bench.layer_step overlaps o and k/v with the main stream; autograd runs each
backward node on its forward's stream.  Every kernel is deterministic, so the
only difference allowed is the order in which autograd adds the input
gradients of projections that share an input (q/k/v): fp16 sums in a
different order, compared at 1e-2 relative L2 of the fp16 gradients (a fraction
of one fp16 ulp per add) and exactly for the LoRA weight gradients, whose
reductions do not depend on the order of other streams.
"""

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _run(bench, layer, inp, streams):
    for name in bench.DIFF_INPUTS:
        inp[name].grad = None
    params = bench.lora_params(layer)
    for p in params:
        p.grad = None
    bench.layer_step(torch, layer, inp, streams)
    torch.cuda.synchronize()
    return ({name: inp[name].grad.clone() for name in bench.DIFF_INPUTS},
            [p.grad.clone() for p in params])


@pytest.mark.parametrize("tokens", [300, 3300])
def test_streamed_layer_step_matches_one_stream(tokens):
    import bench
    dev = torch.device("cuda", 0)
    layer = bench.build_layer(torch, dev, seed=5)
    g = torch.Generator(device=dev).manual_seed(6)
    inp = {name: torch.randn(shp, device=dev, dtype=torch.float16, generator=g)
           for name, shp in bench.input_shapes(tokens).items()}
    for name in bench.DIFF_INPUTS:
        inp[name].requires_grad_()
    ref_in, ref_p = _run(bench, layer, inp, None)
    streams = (torch.cuda.Stream(dev), torch.cuda.Stream(dev))
    for _ in range(2):
        got_in, got_p = _run(bench, layer, inp, streams)
        for name, ref in ref_in.items():
            got = got_in[name]
            assert torch.isfinite(got).all(), name
            rel = (got.float() - ref.float()).norm() / ref.float().norm()
            assert rel < 1e-2, f"{name}: relative L2 {rel:.3e}"
        for ref, got in zip(ref_p, got_p):
            assert torch.equal(ref, got)
    from soupsuck_b200 import _lib
    assert _lib.take_device_error(dev) == 0
