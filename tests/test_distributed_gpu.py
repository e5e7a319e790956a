"""Multi-GPU paths on real GPUs (needs >= 2 visible B200s; skipped otherwise).

Two NCCL ranks, one per GPU, compare against the single-GPU kernels:
* N-split fused NF4 + LoRA projection (all-gather of Y, all-reduce of dX and dA);
* vocabulary-sharded fused cross-entropy (merged statistics, all-reduced dHidden).
Tolerances are the single-GPU gates (GEMM 2e-3 abs + 2e-3 rel; CE metric 2e-3,
gradient 1e-2 of the ideal norm).
"""

import functools
import math
import os
import socket

import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

WORLD = 2
needs_two = pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < WORLD,
                               reason="needs two GPUs")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _entry(rank, fn, port):
    import datetime
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=WORLD,
                            timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", rank))
    try:
        fn(rank)
    finally:
        dist.destroy_process_group()


def _run(fn):
    mp.spawn(_entry, args=(fn, _free_port()), nprocs=WORLD, join=True)


def _nsplit(rank, m=300):
    import numpy as np

    from oracle import oracle as O
    from soupsuck_b200.distributed import allreduce_sum, nf4_row_shard, nsplit_nf4_lora_linear
    from soupsuck_b200.kernels import nf4_lora_linear
    from soupsuck_b200.quantize import quantize_nf4

    dev = torch.device("cuda", rank)
    n, k, r, s = 1536, 1536, 16, 2.0
    g = torch.Generator(device=dev).manual_seed(0)
    w = (torch.randn((n, k), device=dev, generator=g) * 0.02).half()
    packed, st = quantize_nf4(w)
    a = ((torch.rand((r, k), device=dev, generator=g) * 2 - 1) / math.sqrt(k))
    b = torch.randn((n, r), device=dev, generator=g) * 0.01
    x = torch.randn((m, k), device=dev, dtype=torch.float16, generator=g)
    dy = torch.randn((m, n), device=dev, dtype=torch.float16, generator=g)
    # single-GPU reference
    xr, ar, br = x.clone().requires_grad_(), a.clone().requires_grad_(), b.clone().requires_grad_()
    yr = nf4_lora_linear(xr, packed, st, ar, br, s)
    yr.backward(dy)
    # N-split
    sh = nf4_row_shard(packed, st, rank, WORLD)
    xs, as_ = x.clone().requires_grad_(), a.clone().requires_grad_()
    bs = b[sh.row0:sh.row1].clone().requires_grad_()
    ys = nsplit_nf4_lora_linear(xs, sh, as_, bs, s, n)
    ys.backward(dy)
    allreduce_sum(as_.grad)
    gate = lambda got, ref: O.gemm_gate(got.detach().float().cpu().double().numpy(),
                                        ref.detach().float().cpu().double().numpy())
    for got, ref in ((ys, yr), (xs.grad, xr.grad)):
        ok, err, rel = gate(got, ref)
        assert ok, (rank, err, rel)
    for got, ref in ((as_.grad, ar.grad), (bs.grad, br.grad[sh.row0:sh.row1])):
        rel = ((got.double() - ref.double()).norm() / ref.double().norm()).item()
        assert rel < 2e-3, (rank, rel)


@needs_two
@pytest.mark.parametrize("m", [300, 4])
def test_nsplit_projection_matches_single_gpu(m):
    """m = 300 runs the tcgen05 GEMMs on each rank's shard, m = 4 the small-M kernels."""
    _run(functools.partial(_nsplit, m=m))


def _vocab(rank):
    import numpy as np

    from soupsuck_b200.distributed import even_split, vocab_sharded_cross_entropy
    from soupsuck_b200.kernels import fused_linear_cross_entropy

    dev = torch.device("cuda", rank)
    n, h, v = 777, 256, 20011
    g = torch.Generator(device=dev).manual_seed(3)
    hidden = torch.randn((n, h), device=dev, dtype=torch.float16, generator=g)
    weight = (torch.randn((v, h), device=dev, generator=g) / math.sqrt(h)).half()
    targets = torch.randint(v, (n,), device=dev, generator=g)
    targets[::3] = -100
    up = torch.randn(n, device=dev, generator=g)
    hr = hidden.clone().requires_grad_()
    ref = fused_linear_cross_entropy(hr, weight, targets)
    ref[0].backward(up)
    v0, v1 = even_split(v, WORLD, rank, 256)
    hs = hidden.clone().requires_grad_()
    got = vocab_sharded_cross_entropy(hs, weight[v0:v1], targets, v0, v1)
    got[0].backward(up)
    for a, b_ in ((got[0], ref[0]), (got[1], ref[1]), (got[3], ref[3])):
        torch.testing.assert_close(a, b_, rtol=2e-3, atol=2e-3)
    assert (got[2] == ref[2]).float().mean().item() >= 0.999
    err = (hs.grad.double() - hr.grad.double()).norm().item()
    assert err <= 1e-2 * hr.grad.double().norm().item() + 1e-7


@needs_two
def test_vocab_sharded_cross_entropy_matches_single_gpu():
    _run(_vocab)
