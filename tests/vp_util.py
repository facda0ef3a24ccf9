"""Shared pieces of the vocab-parallel tests: the per-slice candidate lists
restated in numpy (the contract of ecah_vp_local), and the check that a row
keeps its oracle result when everything outside the gathered lists is
removed (the merge's exactness argument)."""
from __future__ import annotations

import numpy as np

from oracle import sampler_oracle as so


def local_lists(xf: np.ndarray, top_k: np.ndarray, T: np.ndarray, offset: int, cap: int):
    """Per row of the slice xf [B, local]: every entry at or above the slice's
    k-th largest value (ties included; k = 1 for greedy rows), in vocab order,
    as global ids; also the untruncated counts.  Values compare as floats
    (-0.0 == +0.0); ecah_vp_local compares 16-bit keys, where -0.0 sorts
    below +0.0, so its lists can be shorter by the zeros of the other sign."""
    B, n = xf.shape
    ids = np.full((B, cap), -1, np.int64)
    cnt = np.zeros(B, np.int32)
    for r in range(B):
        V_hint = 1 << 30
        k = 1 if not T[r] > 0 else (V_hint if (top_k[r] <= 0) else int(top_k[r]))
        k = min(k, n)
        kth = np.sort(xf[r])[::-1][k - 1]
        sel = np.nonzero(xf[r] >= kth)[0]
        cnt[r] = len(sel)
        m = min(len(sel), cap)
        ids[r, :m] = offset + sel[:m]
    return ids, cnt


def merged_rows(x_full: np.ndarray, all_ids: np.ndarray, all_cnt: np.ndarray, cap: int) -> np.ndarray:
    """x_full with every entry missing from the gathered lists set to -inf."""
    B, V = x_full.shape
    masked = np.full_like(x_full, -np.inf)
    for r in range(B):
        for g in range(all_ids.shape[0]):
            m = min(int(all_cnt[g, r]), cap)
            sel = all_ids[g, r, :m]
            masked[r, sel] = x_full[r, sel]
    return masked


def vp_case(seed: int, B: int, V: int):
    """bf16-valued rows (quantised, many ties) with 8 spikes, mixed parameters."""
    rng = np.random.default_rng(seed)
    x = np.round(rng.normal(0.0, 3.0, (B, V)) * 4) / 4
    for r in range(B):
        x[r, rng.choice(V, 8, replace=False)] = 10.0
    x = x.astype(np.float32)
    T = rng.choice([0.0, 0.7, 1.0, 1.3], B).astype(np.float32)
    K = rng.choice([1, 5, 20, 64], B).astype(np.int32)
    P = rng.choice([1.0, 0.9, 0.5], B).astype(np.float32)
    U = rng.random(B).astype(np.float32)
    return x, T, K, P, U


def oracle_ids(x, T, K, P, U, dtype="bf16"):
    res = so.sample_batch(x, dtype=dtype, temperature=T, top_k=K, top_p=P, uniforms=U)
    return np.array([rr.token for rr in res.rows]), res
