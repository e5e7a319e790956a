"""Causal-LM head: shifted targets, fused linear cross-entropy, mean over labelled tokens.

Reference: ``fused_head`` / ``_shift_targets`` (solution/autograd.py:11-82).
Targets are the labels shifted left by one with -100 in the last column, the
loss is sum(token_loss) / (num_items_in_batch or the labelled count), and the
detached per-token statistics (entropy, loss, correct, labelled) come back in a
``HeadStep`` so trainers can log them without a second head pass.  The logits
never exist in memory: ``fused_linear_cross_entropy`` (sb_ce_forward /
sb_ce_backward) keeps only per-row statistics.
"""

from collections import namedtuple

HeadStep = namedtuple("HeadStep", "token_entropy token_loss correct labelled")


def shift_targets(labels):
    import torch

    targets = torch.empty(labels.shape, device=labels.device, dtype=labels.dtype)
    if labels.shape[-1]:
        targets[..., :-1].copy_(labels[..., 1:])
        targets[..., -1].fill_(-100)
    return targets


def fused_head(hidden, weight, labels, num_items_in_batch=None):
    """Loss over hidden [B, S, H] against frozen lm_head weight [V, H] and labels [B, S]."""
    import torch

    from .kernels.cross_entropy import fused_linear_cross_entropy

    targets = shift_targets(labels)
    flat_hidden = hidden.reshape(-1, hidden.shape[-1])
    if not flat_hidden.is_contiguous():
        flat_hidden = flat_hidden.contiguous()
    flat_targets = targets.reshape(-1)
    token_loss, entropy, argmax, _ = fused_linear_cross_entropy(flat_hidden, weight, flat_targets,
                                                                ignore_index=-100)
    denominator = (flat_targets != -100).sum() if num_items_in_batch is None else num_items_in_batch
    if isinstance(denominator, torch.Tensor):
        denominator = denominator.to(token_loss.device)
    loss = token_loss.sum() / denominator
    with torch.no_grad():
        valid = flat_targets != -100
        step = HeadStep(token_entropy=entropy.reshape(labels.shape).detach(),
                        token_loss=token_loss.reshape(labels.shape).detach(),
                        correct=((argmax == flat_targets) & valid).sum(), labelled=valid.sum())
    return loss, step
