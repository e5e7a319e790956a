"""Multi-GPU use of the hot path: where it shards, and the collectives that join the shards.

The reference trains on one GPU; these are the natural splits of its hot path
(one process per GPU, ``torch.distributed`` over NCCL for the collectives):

* **Data parallel** (independent micro-batches, weights replicated):
  ``allreduce_mean`` averages the LoRA gradients of all ranks in one flat
  all-reduce per step.
* **N-split NF4 projection**: rank r owns rows [n0_r, n1_r) of the packed weight
  (``nf4_row_shard``) and the matching rows of the LoRA factor B; A is
  replicated.  Forward: the local fused GEMM gives Y[:, n0_r:n1_r] and an
  all-gather assembles Y.  Backward: dX = sum_r dY_r . deq(W_r) + s (dY_r . B_r) . A
  is linear in the column blocks, so every rank runs the fused dX GEMM on its own
  block and one all-reduce sums them; dA is summed the same way
  (``allreduce_sum``); dB_r stays local.
* **Vocabulary-sharded cross-entropy**: rank r owns rows [v0_r, v1_r) of the frozen
  head.  Each rank runs the fused CE over its shard; the per-row statistics are
  merged with three all-reduces (``merge_ce_shards``): lse = logsumexp_r(lse_r),
  entropy = lse - sum_r w_r (lse_r - entropy_r) with w_r = exp(lse_r - lse), the
  target logit from the owning shard, and the first argmax (largest logit, then
  smallest global index).  Backward: every rank forms its dZ against the global
  lse and one all-reduce sums the partial dHidden.

The merge and sharding logic is plain torch and collectives, so it also runs on
CPU tensors with the gloo backend (that is how it is tested without GPUs); the
per-shard compute goes through the sm_100a kernels.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.distributed as dist


# ----------------------------------------------------------------------------- helpers
def _world(group):
    return dist.get_world_size(group), dist.get_rank(group)


def allreduce_sum(t, group=None):
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
    return t


def allreduce_mean(tensors, group=None):
    """Average the given gradient tensors over the ranks with one flat all-reduce."""
    tensors = [t for t in tensors if t is not None]
    if not tensors or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return
    flat = torch.cat([t.reshape(-1).to(torch.float32) for t in tensors])
    dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
    flat.div_(dist.get_world_size(group))
    off = 0
    for t in tensors:
        n = t.numel()
        t.copy_(flat[off:off + n].view_as(t))
        off += n


def even_split(n, world, rank, align=1):
    """[start, stop) of rank's share of n items, boundaries on multiples of `align`."""
    units = -(-n // align)
    u0 = units * rank // world
    u1 = units * (rank + 1) // world
    return min(n, u0 * align), min(n, u1 * align)


# ----------------------------------------------------------------------------- NF4 row shards
@dataclass
class NF4Shard:
    """Rows [row0, row1) of an NF4 weight as a self-contained nested state."""
    packed: torch.Tensor
    state: object
    row0: int
    row1: int


def shard_align_rows(k_in):
    """Smallest row count r such that r * k_in / 64 is a multiple of 256: shards that
    start on such rows keep whole absmax2 groups, so the shard's second-level scales
    are a plain slice of the full array."""
    blocks_per_row = k_in // 64
    return 256 // math.gcd(256, blocks_per_row)


def nf4_row_shard(packed, state, rank, world):
    """Shard of the nested NF4 weight W[N, K] (bitsandbytes layout, K % 64 == 0) for
    `rank`: contiguous rows whose first block index is a multiple of 256, so packed
    bytes, absmax and absmax2 are slices and no scale is recomputed."""
    import copy

    n, k = state.shape
    if k % 64:
        raise ValueError("row sharding needs k_in % 64 == 0")
    align = shard_align_rows(k)
    r0, r1 = even_split(n, world, rank, align)
    flat = packed.reshape(-1)
    b0, b1 = r0 * k // 64, r1 * k // 64
    shard_state = copy.copy(state)
    shard_state.shape = (r1 - r0, k)
    shard_state.absmax = state.absmax[b0:b1]
    shard_state.state2 = copy.copy(state.state2)
    shard_state.state2.absmax = state.state2.absmax[b0 // 256:(b1 + 255) // 256]
    return NF4Shard(flat[r0 * k // 2:r1 * k // 2].reshape(-1, 1), shard_state, r0, r1)


class _GatherColumns(torch.autograd.Function):
    """Forward: all-gather the ranks' column blocks [M, n_r] into [M, N] (blocks in rank
    order).  Backward: each rank keeps the gradient of its own block."""

    @staticmethod
    def forward(ctx, local, sizes, group):
        world, rank = _world(group)
        ctx.sizes, ctx.rank = sizes, rank
        m = local.shape[0]
        width = max(sizes)
        if all(w == width for w in sizes):
            # Equal blocks: gathered as they are into [world, m, width], which is Y
            # for one row and Y after one interleave of the column blocks otherwise.
            buf = local.new_empty((world * m, width))
            dist.all_gather_into_tensor(buf, local.contiguous(), group=group)
            if m == 1:
                return buf.view(1, world * width)
            return buf.view(world, m, width).permute(1, 0, 2).reshape(m, world * width)
        buf = local.new_zeros((world * m, width))
        mine = local.new_zeros((m, width))
        mine[:, :local.shape[1]] = local
        dist.all_gather_into_tensor(buf, mine, group=group)
        buf = buf.view(world, m, width)
        return torch.cat([buf[r, :, :sizes[r]] for r in range(world)], dim=1)

    @staticmethod
    def backward(ctx, grad):
        start = sum(ctx.sizes[:ctx.rank])
        return grad[:, start:start + ctx.sizes[ctx.rank]].contiguous(), None, None


class _SumGradient(torch.autograd.Function):
    """Identity forward; the backward all-reduces (sums) the incoming gradient, which
    turns each rank's partial dX of its column block into the full dX."""

    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return x.view_as(x)

    @staticmethod
    def backward(ctx, grad):
        grad = grad.contiguous()
        allreduce_sum(grad, ctx.group)
        return grad, None


def column_parallel(x, local_fn, n_total, group=None, sizes=None):
    """Y[M, N] = gather_r(local_fn(x)) with dX summed over ranks in the backward.
    `local_fn` maps x to this rank's column block (a differentiable function).
    `sizes` lists every rank's block width when the caller knows them; otherwise
    they are exchanged (one small all-gather and a host read)."""
    world, rank = _world(group)
    x_in = _SumGradient.apply(x, group)
    local = local_fn(x_in)
    lead = local.shape[:-1]
    local2d = local.reshape(-1, local.shape[-1])
    if sizes is None:
        sizes_t = torch.tensor([local2d.shape[1]], device=local.device)
        gathered = [torch.zeros_like(sizes_t) for _ in range(world)]
        dist.all_gather(gathered, sizes_t, group=group)
        sizes = [int(s.item()) for s in gathered]
    sizes = list(sizes)
    if len(sizes) != world or sizes[rank] != local2d.shape[1]:
        raise ValueError(f"column block widths {sizes} do not match this rank's {local2d.shape[1]}")
    if sum(sizes) != n_total:
        raise ValueError(f"column blocks {sizes} do not add up to {n_total}")
    y = _GatherColumns.apply(local2d, sizes, group)
    return y.reshape(*lead, n_total)


def nsplit_nf4_lora_linear(x, shard, lora_a, lora_b_rows, scaling, n_total, bias_rows=None, group=None):
    """N-split fused projection: Y = X . deq(W)^T + s (X . A^T) . B^T with this rank
    holding `shard` (rows of W) and the same rows of B.  After backward, lora_a.grad
    holds this rank's partial dA: sum it over ranks with ``allreduce_sum``."""
    from .kernels.nf4_gemm import nf4_lora_linear

    def local(xi):
        return nf4_lora_linear(xi, shard.packed, shard.state, lora_a, lora_b_rows, scaling, bias_rows)

    world, rank = _world(group)
    k_in = shard.state.shape[1]
    sizes = None
    if k_in % 64 == 0:
        # Shards made by nf4_row_shard: every rank's rows follow from the shape.
        bounds = [even_split(n_total, world, r, shard_align_rows(k_in)) for r in range(world)]
        if bounds[rank] == (shard.row0, shard.row1):
            sizes = [b1 - b0 for b0, b1 in bounds]
    return column_parallel(x, local, n_total, group, sizes=sizes)


# ----------------------------------------------------------------------------- vocabulary shards
@dataclass
class CEShardStats:
    """Per-row statistics of one vocabulary shard (the kernel outputs)."""
    lse: torch.Tensor        # log sum exp over the shard
    entropy: torch.Tensor    # lse - E_softmax[z] over the shard
    loss: torch.Tensor       # lse - z_target, meaningful where has_target
    row_max: torch.Tensor    # largest logit of the shard
    argmax: torch.Tensor     # global index of its first occurrence
    has_target: torch.Tensor  # bool: the row's target lies in this shard


def merge_ce_shards(st: CEShardStats, targets, ignore_index=-100, group=None):
    """Global (loss, entropy, argmax, lse) from every rank's shard statistics."""
    lse_max = st.lse.clone()
    dist.all_reduce(lse_max, op=dist.ReduceOp.MAX, group=group)
    finite = torch.isfinite(lse_max)
    shift = torch.where(finite, lse_max, torch.zeros_like(lse_max))
    w = torch.exp(st.lse - shift)                       # S_r / exp(shift)
    mean_z = st.lse - st.entropy                        # E_r[z] = T_r / S_r
    z_t = torch.where(st.has_target, st.lse - st.loss, torch.zeros_like(st.lse))
    sums = torch.stack([w, w * mean_z, z_t])
    dist.all_reduce(sums, op=dist.ReduceOp.SUM, group=group)
    lse = shift + torch.log(sums[0])
    entropy = lse - sums[1] / sums[0]
    labelled = targets != ignore_index
    loss = torch.where(labelled, lse - sums[2], torch.zeros_like(lse))
    # First argmax: the largest row maximum wins, then the smallest global index.
    best = st.row_max.clone()
    dist.all_reduce(best, op=dist.ReduceOp.MAX, group=group)
    big = torch.iinfo(torch.int64).max
    cand = torch.where(st.row_max == best, st.argmax, torch.full_like(st.argmax, big))
    dist.all_reduce(cand, op=dist.ReduceOp.MIN, group=group)
    return loss, entropy, cand, lse


def local_targets(targets, v0, v1, ignore_index=-100):
    """Targets of this shard: local index inside [v0, v1), -1 for another shard's
    vocabulary (matches no column), ignore_index kept."""
    inside = (targets >= v0) & (targets < v1)
    loc = torch.where(inside, targets - v0, torch.full_like(targets, -1))
    return torch.where(targets == ignore_index, targets, loc), inside


class _VocabShardCE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, hidden, weight_rows, targets, v0, v1, ignore_index, group):
        from . import _lib
        from .kernels.cross_entropy import _half_padded

        n, h = hidden.shape
        v = weight_rows.shape[0]
        h8 = (h + 7) // 8 * 8
        hidden16 = _half_padded(hidden, h8)
        weight16 = _half_padded(weight_rows, h8)
        tloc, inside = local_targets(targets, v0, v1, ignore_index)
        tloc = tloc.contiguous()
        f32 = dict(device=hidden.device, dtype=torch.float32)
        loss, entropy, lse, row_max = (torch.empty(n, **f32) for _ in range(4))
        arg = torch.empty(n, device=hidden.device, dtype=torch.int64)
        if n:
            nbytes = _lib.query("sb_ce_forward_workspace_bytes", n, h8, v)
            ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=hidden.device)
            _lib.call("sb_ce_forward_shard", hidden16.data_ptr(), n, h8, weight16.data_ptr(), v,
                      tloc.data_ptr(), int(ignore_index), loss.data_ptr(), entropy.data_ptr(),
                      arg.data_ptr(), lse.data_ptr(), row_max.data_ptr(), ws.data_ptr(), nbytes,
                      _lib.stream_of(hidden.device))
        stats = CEShardStats(lse, entropy, loss, row_max, arg + v0, inside)
        g_loss, g_ent, g_arg, g_lse = merge_ce_shards(stats, targets, ignore_index, group)
        ctx.save_for_backward(hidden16, weight16, tloc, g_lse)
        ctx.meta = (hidden.dtype, h, ignore_index, group)
        ctx.mark_non_differentiable(g_ent, g_arg, g_lse)
        ctx.set_materialize_grads(False)
        return g_loss, g_ent, g_arg, g_lse

    @staticmethod
    def backward(ctx, grad_loss, _ge, _ga, _gl):
        from . import _lib

        hidden16, weight16, tloc, lse = ctx.saved_tensors
        dtype, h, ignore_index, group = ctx.meta
        if grad_loss is None:
            return None, None, None, None, None, None, None
        n, h8 = hidden16.shape
        v = weight16.shape[0]
        dx = torch.zeros((n, h8), device=hidden16.device, dtype=torch.float32)
        if n:
            grad = grad_loss.to(torch.float32).contiguous()
            nbytes = _lib.query("sb_ce_backward_workspace_bytes", n, h8, v)
            ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=hidden16.device)
            _lib.call("sb_ce_backward", hidden16.data_ptr(), n, h8, weight16.data_ptr(), v,
                      tloc.data_ptr(), int(ignore_index), lse.data_ptr(), grad.data_ptr(),
                      dx.data_ptr(), _lib.SB_F32, ws.data_ptr(), nbytes, _lib.stream_of(hidden16.device))
        allreduce_sum(dx, group)
        dx = dx[:, :h]
        return dx.to(dtype), None, None, None, None, None, None


def vocab_sharded_cross_entropy(hidden, weight_rows, targets, v0, v1, ignore_index=-100, group=None):
    """Fused linear CE with the head's rows [v0, v1) on this rank; returns the global
    (loss, entropy, argmax, lse) on every rank.  Only loss is differentiable."""
    if weight_rows.requires_grad:
        raise ValueError("the head must be frozen")
    if weight_rows.shape[0] != v1 - v0:
        raise ValueError("weight_rows must hold rows [v0, v1) of the head")
    return _VocabShardCE.apply(hidden, weight_rows, targets.contiguous(), v0, v1, ignore_index, group)
