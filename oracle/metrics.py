"""Error metrics for the parity bar (TEST INFRASTRUCTURE ONLY).

The bar is ``max|o - r| / max|r| <= 2e-2`` and ``mean|o - r| / mean|r| <= 1e-3``, computed globally and
per (batch row, query head) row, so that long-context rows (output std ~0.02) are not hidden behind
short-context rows (std ~1) the way a flattened PCC hides them.
"""
from __future__ import annotations

import torch

MAX_REL = 2e-2
MEAN_REL = 1e-3


def rel_errors(out: torch.Tensor, ref: torch.Tensor):
    """(max-abs relative, mean-abs relative) over the whole tensor, in float64."""
    o, r = out.double().cpu(), ref.double().cpu()
    d = (o - r).abs()
    return (d.max() / r.abs().max().clamp_min(1e-30)).item(), (d.mean() / r.abs().mean().clamp_min(1e-30)).item()


def rowwise_rel_errors(out: torch.Tensor, ref: torch.Tensor):
    """Worst (max-abs relative, mean-abs relative) over rows; a row is the last dimension."""
    o = out.double().cpu().reshape(-1, out.shape[-1])
    r = ref.double().cpu().reshape(-1, ref.shape[-1])
    d = (o - r).abs()
    mx = d.max(-1).values / r.abs().max(-1).values.clamp_min(1e-30)
    mn = d.mean(-1) / r.abs().mean(-1).clamp_min(1e-30)
    return mx.max().item(), mn.max().item()


def round_like(ref: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """The oracle's fp32 output rounded to the dtype the op returns."""
    return ref.to(dtype).float()
