"""Gradient-based one-side sampling (GOSS) of the rows a tree grows on,
yabt/adaptive_features.py:61-110 as called from yabt/boosting.py:371-374,393-396.

The draw has to be the reference's own: the rows with the largest |g| (the
reference's unstable device argsort) and a uniform sample of the rest from a
device generator seeded once per fit (``torch.randperm`` on that generator).
Only torch's own sort and generator reproduce those rows, so the draw is made
with the same calls; everything downstream (weighted gradients, the tree on the
sampled rows, routing every row, leaf models) runs in the library's kernels.
"""

from __future__ import annotations

import torch


def goss_sample(grad: torch.Tensor, ratio: float, gen: torch.Generator):
    """(rows, weights): the kept rows -- the top (1 - ratio) share by |grad|,
    then a uniform draw filling the ``ratio`` budget -- and their per-row
    multipliers of grad / hess (1 for the top rows, (n - top) / drawn for the
    drawn rows), or None when nothing is drawn."""
    n = grad.shape[0]
    ratio = min(max(ratio, 0.0), 1.0)
    keep = max(1, round(n * ratio))
    top = max(1, min(keep, round(n * (1.0 - ratio))))
    drawn = keep - top
    by_mag = torch.argsort(grad.abs(), descending=True)
    head, tail = by_mag[:top], by_mag[top:]
    if drawn <= 0 or tail.numel() == 0:
        return head, None
    pick = tail[torch.randperm(tail.numel(), generator=gen, device=grad.device)[:drawn]]
    weights = torch.ones(top + pick.numel(), device=grad.device)
    weights[top:] = (n - top) / pick.numel()
    return torch.cat([head, pick]), weights
