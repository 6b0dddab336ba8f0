"""CPU restatements of the two isolated-op workloads — test infrastructure.

Only tests/ and bench.py's CPU legs use this module; the product path never
does. Neither workload is an op of the reference, so these restatements are
the definition (parity unpinned by reference tests): each follows the
workload text and the reference arithmetic it names.

- ``hex_message_pass``: y = x + W mean_{present}(x[nbr]) + b with a
  six-slot neighbour table, -1 for an absent neighbour and a zero mean when
  none is present (the reference's empty-run-reads-zero convention,
  cell_latents.py:282-283; gather + index_add_ as message_passing.py:102-118).
- ``axial_attention``: scaled dot-product attention with an additive bias
  gathered from a (33, 33, heads) table by the clamped relative axial offset
  (key minus query), added to the fp32 scores the way the reference adds its
  class bias (cell_latents.py:552-555); keys past the valid length are masked
  and query rows past it read zero (attention.py:540-555 pads queries to 0).
"""

from __future__ import annotations

import math

import torch


def hex_message_pass(x: torch.Tensor, nbr: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None) -> torch.Tensor:
    """x (N, F), nbr (N, 6) int, w (F, F) [out, in], b (F,) -> (N, F), in x's float dtype (use fp32/fp64)."""
    present = nbr >= 0
    rows = x[nbr.clamp(min=0).long()] * present[..., None].to(x.dtype)  # (N, 6, F)
    count = present.sum(1, keepdim=True).to(x.dtype)
    agg = rows.sum(1) / count.clamp(min=1)
    y = x + agg @ w.t().to(x.dtype)
    if b is not None:
        y = y + b.to(x.dtype)
    return y


def axial_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, coords: torch.Tensor, valid: torch.Tensor,
                    bias: torch.Tensor) -> torch.Tensor:
    """q, k, v (P, H, L, d); coords (P, L, 2) int; valid (P,) int; bias (33, 33, H) -> (P, H, L, d)."""
    p, h, length, d = q.shape
    s = q @ k.transpose(-1, -2) / math.sqrt(d)  # (P, H, L, L): query i, key j
    c = coords.long()
    dq = (c[:, None, :, 0] - c[:, :, None, 0]).clamp(-16, 16) + 16  # (P, Lq, Lk) key minus query
    dr = (c[:, None, :, 1] - c[:, :, None, 1]).clamp(-16, 16) + 16
    s = s + bias.to(s.dtype)[dq, dr].permute(0, 3, 1, 2)
    pos = torch.arange(length)
    live = pos[None, :] < valid.long()[:, None]  # (P, L)
    s = s.masked_fill(~live[:, None, None, :], float("-inf"))
    attn = torch.softmax(s, dim=-1)
    out = attn @ v
    out = torch.where(live[:, None, :, None], out, torch.zeros((), dtype=out.dtype))
    return torch.nan_to_num(out, nan=0.0)
