"""Batched torch-CPU port of the reference sampling path, for timing.

TEST / BASELINE INFRASTRUCTURE ONLY: used by tests/, the CPU-baseline leg of
bench.py and ``bench.py --impl reference``.  The reference's own sampling
arithmetic is torch on a [B, V] tensor (ecahlang/utils.py:3-18, with the
divides of ecahlang/main.py:169-170); FlashInfer's top-p stage has no CPU
build, so this port completes the op order with torch ops:

  y = D(x / m)                    (penalty divide in the model dtype)
  z = float32(y) / T              (temperature divide)
  top-k: keep z >= k-th largest   (ecahlang/utils.py:12-15, via a descending sort)
  softmax over the kept set
  top-p: keep tokens whose strictly-larger mass is < p * S  (FlashInfer top_k_first)
  draw: inverse CDF in vocab order against u

It uses every host thread torch is given.  Results agree with
oracle/sampler_oracle.py except in CDF / top-p boundary cases (float32 sums
here versus float64 there).
"""
from __future__ import annotations

from typing import Optional

import torch


@torch.no_grad()
def sample_batch_torch(logits: torch.Tensor, temperature: torch.Tensor, top_k: torch.Tensor,
                       top_p: torch.Tensor, uniforms: torch.Tensor,
                       mask: Optional[torch.Tensor] = None) -> torch.Tensor:
    B, V = logits.shape
    x = logits
    if mask is not None:
        x = x / mask
    z = x.float() / temperature.reshape(B, 1).float()
    greedy = ~(temperature.reshape(B) > 0)
    zs, order = torch.sort(z, dim=1, descending=True)
    k = top_k.reshape(B).long()
    k = torch.where((k <= 0) | (k >= V), torch.full_like(k, V), k)
    tau_k = zs.gather(1, (k - 1).clamp(min=0).unsqueeze(1))                # k-th largest
    M = zs[:, :1]
    e_sorted = torch.where(zs >= tau_k, torch.exp(zs - M), torch.zeros_like(zs))
    S = e_sorted.sum(dim=1, keepdim=True)
    p = top_p.reshape(B, 1).float()
    topp_on = (p > 0) & (p < 1)
    # mass strictly above each sorted position, tie groups handled by the value
    csum = torch.cumsum(e_sorted, dim=1)
    excl = csum - e_sorted
    # for tie groups, the strictly-larger mass is the exclusive sum at the
    # first member of the group: take the minimum over equal values
    first_of_group = torch.ones_like(zs, dtype=torch.bool)
    first_of_group[:, 1:] = zs[:, 1:] != zs[:, :-1]
    grp = torch.cumsum(first_of_group.long(), dim=1) - 1
    grp_excl = torch.zeros_like(excl).scatter_reduce(1, grp, excl, reduce="amin", include_self=False)
    strictly_above = grp_excl.gather(1, grp)
    keep_sorted = (zs >= tau_k) & (~topp_on | (strictly_above < p * S))
    keep = torch.zeros_like(keep_sorted).scatter(1, order, keep_sorted)
    e = torch.where(keep, torch.exp(z - M), torch.zeros_like(z))
    C = torch.cumsum(e.double(), dim=1)
    Z = C[:, -1:]
    t = uniforms.reshape(B, 1).double() * Z
    idx = torch.searchsorted(C, t, right=True).clamp(max=V - 1).reshape(B)
    return torch.where(greedy, torch.argmax(x.float(), dim=1), idx).to(torch.int32)
