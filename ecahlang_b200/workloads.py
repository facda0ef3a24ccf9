"""Seeded synthetic inputs for the sampler configurations.

There is no dataset behind the sampler's benchmarks; each configuration is a
distribution of logits plus per-row parameters, generated here on the CPU
with fixed ``torch.Generator`` seeds so every run (and the oracle) sees the
same tensors.  Request parameters go through the reference's normalisation
(ecahlang/main.py:642-645): temperature 0 becomes 1e-5, top_k 0 becomes V,
top_p 0 becomes 1.0.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional, Tuple

import numpy as np
import torch

V_QWEN = 151936     # Qwen2.5 vocabulary
V_LLAMA3 = 128256   # config 4 vocabulary


def normalize(temperature: float, top_k: int, top_p: float, rep: float, vocab: int):
    """ecahlang/main.py:642-645."""
    return (max(1e-5, temperature), vocab if top_k == 0 else top_k,
            1.0 if top_p == 0 else top_p, max(1e-5, rep))


@dataclass
class Workload:
    name: str
    logits: torch.Tensor                 # [B, V] model dtype, CPU
    temperature: torch.Tensor            # [B] float32
    top_k: torch.Tensor                  # [B] int32
    top_p: torch.Tensor                  # [B] float32
    uniforms: torch.Tensor               # [B] float32
    rep_pen: Optional[torch.Tensor] = None
    freq_pen: Optional[torch.Tensor] = None
    pres_pen: Optional[torch.Tensor] = None
    history: Optional[List[Tuple[np.ndarray, np.ndarray]]] = None   # per row (toks, cnts)
    freq_pres: bool = False
    meta: dict = field(default_factory=dict)

    @property
    def batch(self):
        return self.logits.shape[0]

    @property
    def vocab(self):
        return self.logits.shape[1]

    def algorithmic_bytes(self) -> int:
        """One read of the logits plus the sparse history (tok, cnt) pairs."""
        b = self.logits.numel() * self.logits.element_size()
        if self.history is not None:
            b += sum(len(t) for t, _ in self.history) * 8
        return b


def _params(rows, V):
    T, K, P, R = zip(*[normalize(t, k, p, r, V) for (t, k, p, r) in rows])
    return (torch.tensor(T, dtype=torch.float32), torch.tensor(K, dtype=torch.int32),
            torch.tensor(P, dtype=torch.float32), torch.tensor(R, dtype=torch.float32))


def _spiked(g, B, V, sigma, n_spike, spike, mode, dtype):
    x = torch.randn(B, V, generator=g) * sigma
    idx = torch.argsort(torch.rand(B, V, generator=g), dim=1)[:, :n_spike] if n_spike > V // 64 else \
        torch.stack([torch.randperm(V, generator=g)[:n_spike] for _ in range(B)])
    if mode == "set":
        x.scatter_(1, idx, spike)
    else:
        x.scatter_add_(1, idx, torch.full(idx.shape, float(spike)))
    return x.to(dtype)


def config1(seed: int = 0, B: int = 8, V: int = V_QWEN) -> Workload:
    """C1: fp32 N(0,3^2), 5 spikes per row set to +12; T=0.7, k=50, p=0.9."""
    g = torch.Generator().manual_seed(1000 + seed)
    x = _spiked(g, B, V, 3.0, 5, 12.0, "set", torch.float32)
    T, K, P, R = _params([(0.7, 50, 0.9, 1.0)] * B, V)
    u = torch.rand(B, generator=g)
    return Workload("c1_cpu_step", x, T, K, P, u, meta={"seed": seed})


def config2(seed: int = 0, B: int = 128, V: int = V_QWEN, dtype=torch.float16) -> Workload:
    """C2: fp16 N(0,2.5^2), 3% of ids per row shifted +6; four row groups:
    greedy (T=0), top-k only k in {20,40,100}, top-p only p in {0.8,0.95},
    and T~U[0.5,1.2] with k=50, p=0.9."""
    g = torch.Generator().manual_seed(2000 + seed)
    x = _spiked(g, B, V, 2.5, int(round(0.03 * V)), 6.0, "add", dtype)
    tu = torch.rand(B, generator=g)
    rows = []
    q = max(B // 4, 1)
    for r in range(B):
        grp = min(r // q, 3)
        if grp == 0:
            rows.append((0.0, 0, 0.0, 1.0))
        elif grp == 1:
            rows.append((1.0, (20, 40, 100)[r % 3], 0.0, 1.0))
        elif grp == 2:
            rows.append((1.0, 0, (0.8, 0.95)[r % 2], 1.0))
        else:
            rows.append((0.5 + 0.7 * float(tu[r]), 50, 0.9, 1.0))
    T, K, P, R = _params(rows, V)
    u = torch.rand(B, generator=g)
    return Workload("c2_mixed", x, T, K, P, u, meta={"seed": seed})


def zipf_history(g: np.random.Generator, V: int, n_tokens: int, s: float, perm: np.ndarray):
    ranks = np.arange(1, V + 1, dtype=np.float64)
    w = ranks ** (-s)
    cdf = np.cumsum(w)
    cdf /= cdf[-1]
    draws = np.searchsorted(cdf, g.random(n_tokens), side="right")
    ids = perm[np.minimum(draws, V - 1)]
    toks, cnts = np.unique(ids, return_counts=True)
    return toks.astype(np.int32), cnts.astype(np.int32)


def config3(seed: int = 0, B: int = 128, V: int = V_QWEN, dtype=torch.float16,
            hist_len: int = 384) -> Workload:
    """C3: fp16 N(0,2.5^2); per row a 384-token history drawn Zipf(1.1) over
    ranks mapped to ids by a seeded permutation; rp=1.1, f=0.5, pi=0.3,
    T=0.8, p=0.95, k=V."""
    g = torch.Generator().manual_seed(3000 + seed)
    x = (torch.randn(B, V, generator=g) * 2.5).to(dtype)
    ng = np.random.default_rng(3000 + seed)
    perm = ng.permutation(V)
    history = [zipf_history(ng, V, hist_len, 1.1, perm) for _ in range(B)]
    T, K, P, R = _params([(0.8, 0, 0.95, 1.1)] * B, V)
    u = torch.rand(B, generator=g)
    return Workload("c3_penalised", x, T, K, P, u, rep_pen=R,
                    freq_pen=torch.full((B,), 0.5), pres_pen=torch.full((B,), 0.3),
                    history=history, freq_pres=True, meta={"seed": seed, "hist_len": hist_len})


def config4(seed: int = 0, B: int = 512, V: int = V_LLAMA3, dtype=torch.bfloat16) -> Workload:
    """C4: bf16 N(0,3^2), 8 spikes per row at +10; k=64, p=0.9, T=1."""
    g = torch.Generator().manual_seed(4000 + seed)
    x = _spiked(g, B, V, 3.0, 8, 10.0, "set", dtype)
    T, K, P, R = _params([(1.0, 64, 0.9, 1.0)] * B, V)
    u = torch.rand(B, generator=g)
    return Workload("c4_vocab_parallel", x, T, K, P, u, meta={"seed": seed})


CONFIGS = {"c1": config1, "c2": config2, "c3": config3, "c4": config4}
