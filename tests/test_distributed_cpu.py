"""Host logic of the multi-GPU paths on CPU: two gloo ranks (spawned processes).

Checks, against single-process references:
* NF4 row shards: slices whose decode (oracle) equals the matching rows of the
  full decode, for Qwen2.5-1.5B and -7B widths, with whole absmax2 groups;
* column-parallel projection: all-gathered Y and summed dX equal the unsharded
  product and its gradient;
* vocabulary-shard cross-entropy merge: per-shard statistics merged with the
  collectives equal loss / entropy / first argmax / lse over the full vocabulary;
* data-parallel LoRA gradient averaging.
The per-shard compute here is a float64 torch restatement; on GPUs it is the
sm_100a kernels (tests/test_distributed_gpu.py).
"""

import math
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(fn, *args):
    port = _free_port()
    mp.spawn(_entry, args=(fn, port, args), nprocs=WORLD, join=True)


def _entry(rank, fn, port, args):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=WORLD)
    try:
        fn(rank, *args)
    finally:
        dist.destroy_process_group()


# ------------------------------------------------------------------ NF4 row shards
def _check_row_shards(rank, n, k):
    from oracle import oracle as O
    from soupsuck_b200.distributed import nf4_row_shard, shard_align_rows
    from soupsuck_b200.quantize import quantize_nf4

    torch.manual_seed(n + k)
    w = (torch.randn((n, k)) * 0.02).to(torch.float16)
    packed, st = quantize_nf4(w)
    npf = lambda t: t.numpy()
    full = O.nf4_dequant_nested(npf(packed).reshape(-1), npf(st.absmax), npf(st.state2.absmax),
                                npf(st.state2.code), npf(st.offset), n * k).reshape(n, k)
    sh = nf4_row_shard(packed, st, rank, WORLD)
    assert sh.row0 % shard_align_rows(k) == 0 and (sh.row0 * k // 64) % 256 == 0
    rows = sh.row1 - sh.row0
    part = O.nf4_dequant_nested(npf(sh.packed).reshape(-1), npf(sh.state.absmax), npf(sh.state.state2.absmax),
                                npf(sh.state.state2.code), npf(sh.state.offset), rows * k).reshape(rows, k)
    assert np.array_equal(part.view(np.uint16), full[sh.row0:sh.row1].view(np.uint16))
    covered = torch.tensor([rows])
    dist.all_reduce(covered)
    assert covered.item() == n


@pytest.mark.parametrize("n,k", [(256, 1536), (1536, 8960), (512, 3584), (300, 128)])
def test_nf4_row_shards_are_exact_slices(n, k):
    _run(_check_row_shards, n, k)


# ------------------------------------------------------------------ column-parallel projection
def _check_column_parallel(rank, m, n, k, known):
    from soupsuck_b200.distributed import column_parallel, even_split

    torch.manual_seed(0)
    x_full = torch.randn(m, k, dtype=torch.float64)
    w = torch.randn(n, k, dtype=torch.float64)
    dy = torch.randn(m, n, dtype=torch.float64)
    r0, r1 = even_split(n, WORLD, rank, 64)
    sizes = [b - a for a, b in (even_split(n, WORLD, r, 64) for r in range(WORLD))] if known else None
    x = x_full.clone().requires_grad_()
    y = column_parallel(x, lambda xi: xi @ w[r0:r1].t(), n, sizes=sizes)
    y.backward(dy)
    assert y.shape == (m, n)
    assert torch.allclose(y, x_full @ w.t())
    assert torch.allclose(x.grad, dy @ w)


# Unequal blocks (300 = 128 + 172: padded gather), equal blocks at one and at
# several rows (gathered as they are), widths passed by the caller.
@pytest.mark.parametrize("m,n,known", [(37, 300, False), (37, 256, False), (1, 256, False), (5, 256, True)])
def test_column_parallel_gathers_y_and_sums_dx(m, n, known):
    _run(_check_column_parallel, m, n, 64, known)


# ------------------------------------------------------------------ vocabulary-shard CE merge
def _shard_stats(hidden, weight, targets, v0, v1, ignore):
    """float64 per-shard statistics, as the kernel reports them."""
    from soupsuck_b200.distributed import CEShardStats, local_targets

    z = (hidden @ weight[v0:v1].t()).to(torch.float16).to(torch.float64)
    tloc, inside = local_targets(targets, v0, v1, ignore)
    m = z.max(1).values
    lse = m + torch.log(torch.exp(z - m[:, None]).sum(1))
    p = torch.exp(z - lse[:, None])
    entropy = lse - (p * z).sum(1)
    zt = torch.where(tloc >= 0, z.gather(1, tloc.clamp_min(0)[:, None])[:, 0], torch.zeros_like(lse))
    loss = lse - zt
    arg = z.argmax(1) + v0  # torch returns the first maximum
    return CEShardStats(lse, entropy, loss, m, arg, inside)


def _check_ce_merge(rank, n, h, v):
    from soupsuck_b200.distributed import even_split, merge_ce_shards

    torch.manual_seed(5)
    hidden = torch.randn(n, h, dtype=torch.float64)
    weight = torch.randn(v, h, dtype=torch.float64) / math.sqrt(h)
    weight[7] = weight[3]            # exact tie across the shard boundary below
    targets = torch.randint(v, (n,))
    targets[::3] = -100
    v0, v1 = even_split(v, WORLD, rank, 1) if v > 7 else (0, v)
    st = _shard_stats(hidden, weight, targets, v0, v1, -100)
    loss, entropy, arg, lse = merge_ce_shards(st, targets, -100)
    ref = _shard_stats(hidden, weight, targets, 0, v, -100)
    assert torch.allclose(lse, ref.lse, atol=1e-9, rtol=1e-9)
    assert torch.allclose(entropy, ref.entropy, atol=1e-9, rtol=1e-9)
    ref_loss = torch.where(targets != -100, ref.loss, torch.zeros_like(ref.loss))
    assert torch.allclose(loss, ref_loss, atol=1e-9, rtol=1e-9)
    assert torch.equal(arg, ref.argmax)


@pytest.mark.parametrize("n,h,v", [(40, 16, 1000), (9, 8, 17)])
def test_vocab_shard_statistics_merge(n, h, v):
    _run(_check_ce_merge, n, h, v)


# ------------------------------------------------------------------ data-parallel gradients
def _check_allreduce_mean(rank):
    from soupsuck_b200.distributed import allreduce_mean

    a = torch.full((3, 4), float(rank + 1))
    b = torch.full((5,), float(10 * (rank + 1)))
    allreduce_mean([a, b, None])
    assert torch.allclose(a, torch.full((3, 4), 1.5)) and torch.allclose(b, torch.full((5,), 15.0))


def test_allreduce_mean_averages_lora_grads():
    _run(_check_allreduce_mean)


def test_even_split_alignment():
    from soupsuck_b200.distributed import even_split, shard_align_rows
    assert shard_align_rows(1536) == 32 and shard_align_rows(8960) == 64 and shard_align_rows(3584) == 32
    for n, w, a in [(8960, 8, 32), (18944, 8, 32), (1536, 8, 64), (257, 4, 32)]:
        parts = [even_split(n, w, r, a) for r in range(w)]
        assert parts[0][0] == 0 and parts[-1][1] == n
        assert all(p[1] == q[0] for p, q in zip(parts, parts[1:]))
        assert all(p[0] % a == 0 for p in parts)
