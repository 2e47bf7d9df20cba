"""Sequence-partitioned MTP loss and backward (the drafter training step).

Same functions and semantics as the reference ``pe.partition``
(``src/pe/partition.py:25-131``): a sequence is split into ``S`` anchor
segments; each segment runs the real prefix ``0..a1-1`` plus the ``K-1``
prediction slots of its own anchors, and only slots whose anchor lies in the
segment contribute loss, so the accumulated gradient is exactly the
full-sequence gradient.  Gradients are *added* into ``p.grad`` of the drafter's
trainable parameters; the caller zeroes them and steps the optimizer.

The computation runs in :class:`parallel_eagle_b200.engine.StepEngine` (fused
kernels, no dense mask, no full-vocabulary logits).
"""

from __future__ import annotations

import torch

from . import _lib as L
from . import ops
from .drafter import ParallelDrafter
from .engine import count_loss_slots, engine_for, segment_bounds


def _segment_bounds(n: int, num_segments: int) -> list[tuple[int, int]]:
    return segment_bounds(n, num_segments)


def _total_valid(n: int, k: int) -> int:
    return count_loss_slots(n, k, 0)


def _total_valid_after(n: int, k: int, prompt_len: int = 0) -> int:
    return count_loss_slots(n, k, prompt_len)


def _segment_slots(a0: int, a1: int, k: int, device):
    """Anchors/depths of one segment: real prefix ``0..a1-1`` then anchors
    ``a0..a1-1`` x depths ``1..k-1`` (reference ``partition.py:41-55``)."""
    anchor_real = torch.arange(a1, device=device)
    depth_real = torch.zeros(a1, dtype=torch.long, device=device)
    if k > 1:
        anchor_mtp = torch.arange(a0, a1, device=device).repeat_interleave(k - 1)
        depth_mtp = torch.arange(1, k, device=device).repeat(a1 - a0)
    else:
        anchor_mtp = torch.empty(0, dtype=torch.long, device=device)
        depth_mtp = torch.empty(0, dtype=torch.long, device=device)
    return torch.cat([anchor_real, anchor_mtp]), torch.cat([depth_real, depth_mtp]), a1


def mtp_backward(
    drafter: ParallelDrafter,
    input_ids: torch.Tensor,
    features: torch.Tensor,
    num_segments: int = 1,
    loss_scale: float = 1.0,
    prompt_len: int = 0,
    teacher_labels: torch.Tensor | None = None,
    teacher_hidden: torch.Tensor | None = None,
) -> float:
    """Per-depth cross-entropy of one sequence with gradient accumulation
    (reference ``partition.py:58-118``).  Returns the mean loss.

    ``teacher_labels[p]`` supervises the slot predicting position ``p + 1``.
    ``teacher_hidden`` (an extension with no reference counterpart) switches to
    the soft-target distillation loss: the slot predicting position ``t`` is
    trained towards ``softmax(teacher_hidden[t-1] @ W_head^T)``.
    """
    if drafter.device.type != "cuda":
        raise L.PeError("mtp_backward runs on CUDA only; move the drafter to a CUDA device")
    eng = engine_for(drafter)
    loss = eng.run(input_ids, features, num_segments, loss_scale, prompt_len, teacher_labels,
                   teacher_hidden)
    ops.check_status(drafter.device)
    return loss


@torch.no_grad()
def mtp_eval_loss(drafter: ParallelDrafter, input_ids: torch.Tensor, features: torch.Tensor) -> float:
    """Full-sequence anchor-major mean loss without gradients (reference
    ``partition.py:121-131``); the mask is re-derived from per-slot
    (anchor, depth) instead of read from a dense bias."""
    dev = drafter.device
    ids = input_ids.to(dev)
    x, pos, _bias, labels = drafter.build_training_packed(ids, features.to(dev))
    k = drafter.max_depth
    n = ids.shape[0]
    slot = torch.arange(n * k, device=dev)
    layout = ops.AttnLayout(L.LAYOUT_INDEXED, anchor=(slot // k).to(torch.int32),
                            depth=(slot % k).to(torch.int32))
    hidden = drafter(x, pos, layout)[0]
    valid = labels != -100
    rows = hidden[valid].contiguous()
    lab = labels[valid].to(dev)
    loss = torch.zeros(1, dtype=torch.float32, device=dev)
    _, head, _ = drafter.frozen_heads()
    ops.lmhead_ce(rows, head, lab, 0.0, loss)
    return float(loss.item()) / max(1, rows.shape[0])
