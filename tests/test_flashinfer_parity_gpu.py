"""Top-p, and the top-k-then-top-p order, pinned against the reference's own
GPU sampler.

The reference samples with ``flashinfer.sampling.top_k_top_p_sampling_from_logits(
logits, top_k=..., top_p=..., deterministic=True)`` on ``logits / mask_penalty /
temperature`` (ecahlang/main.py:169-170, :377-379).  FlashInfer
(flashinfer-python, pinned at 0.6.5 in the reference's uv.lock; the installed
0.6.11.post2 runs here) lives outside the reference tree, so the oracle restates
its ``top_k_first`` semantics (oracle/sampler_oracle.py rules 5-8).  These
tests run FlashInfer itself on the same divided logits and check, per row kind
of configs[1] and configs[2]:

- the kept set of FlashInfer's own filters (``top_k_mask_logits``, softmax,
  ``top_p_renorm_probs``) equals the oracle's final set and the CUDA
  sampler's, except where the top-p tail lies within 1e-6 of p * S;
- 10^6 draws of FlashInfer's sampling op (the three steps of
  ``top_k_top_p_sampling_from_logits``, with ``indices`` so the draws share one
  row) never leave the oracle's set and pass a chi-square test against the
  oracle's probabilities;
- the one-call form the reference uses never draws outside the set either.

FlashInfer draws by rejection sampling from its own Philox stream, so its ids
are compared by distribution, not one by one.
"""
from __future__ import annotations

import functools

import numpy as np
import pytest
import torch

from gpu_util import BOUNDARY, run_gpu
from ecahlang_b200 import workloads as W
from oracle import sampler_oracle as so

pytestmark = pytest.mark.gpu

NAMES = ["c2 top-p 0.8", "c2 top-p 0.95", "c2 top-k 40", "c2 T + k 50 + p 0.9",
         "c2 T + k 50 + p 0.9 (b)", "c3 wide", "c3 repetition 1.1"]


@functools.lru_cache(maxsize=1)
def _row_kinds():
    """(name, fp16 logits row [V], T, k, p, history or None, rp)."""
    w2 = W.config2(seed=0)
    w3 = W.config3(seed=0)
    V = w2.vocab
    kinds = []
    for name, r in zip(NAMES[:5], (64, 65, 34, 96, 101)):
        kinds.append((name, w2.logits[r], float(w2.temperature[r]), int(w2.top_k[r]),
                      float(w2.top_p[r]), None, 1.0))
    # the wide nucleus (T 0.8, p 0.95, about 10^4 tokens), and the
    # same row with the repetition penalty, the only penalty the reference has
    # (it multiplies a positive logit by rp^count, so the Zipf head token takes
    # nearly all the mass)
    kinds.append((NAMES[5], w3.logits[0], float(w3.temperature[0]), int(w3.top_k[0]),
                  float(w3.top_p[0]), None, 1.0))
    kinds.append((NAMES[6], w3.logits[0], float(w3.temperature[0]), int(w3.top_k[0]),
                  float(w3.top_p[0]), w3.history[0], float(w3.rep_pen[0])))
    assert all(k[1].shape[0] == V for k in kinds)
    return {k[0]: k for k in kinds}


def _fi():
    return pytest.importorskip("flashinfer")


def _oracle(x, T, k, p, hist, rp):
    toks, cnts = (hist if hist is not None else (None, None))
    return so.sample_row(x.float().numpy(), dtype="f16", temperature=T, top_k=k, top_p=p, u=0.5,
                         toks=toks, cnts=cnts, rp=rp)


def _divided(x, T, hist, rp):
    """The reference's FlashInfer input: fp16 logits / mask_penalty (fp16), then
    / temperature (promotes to float32), computed by torch on the GPU."""
    toks, cnts = (hist if hist is not None else (None, None))
    y = so.penalised_logits(x.float().numpy(), "f16", toks, cnts, rp=rp)
    y16 = torch.from_numpy(y).to(torch.float16).cuda()
    return (y16[None, :] / torch.tensor([[T]], dtype=torch.float32, device="cuda")).contiguous()


def _flashinfer_kept(z, k, p):
    flashinfer = _fi()
    masked = flashinfer.sampling.top_k_mask_logits(z, k)
    probs = torch.softmax(masked, dim=-1)
    if 0.0 < p < 1.0:
        probs = flashinfer.sampling.top_p_renorm_probs(probs, p)
    return (probs[0] > 0).cpu().numpy()


def _chi_square_p(counts, expected):
    from scipy.stats import chi2
    order = np.argsort(expected)[::-1]
    e, o = expected[order], counts[order]
    big = e >= 5.0
    ee = np.append(e[big], e[~big].sum())
    oo = np.append(o[big], o[~big].sum())
    keep = ee > 0
    ee, oo = ee[keep], oo[keep]
    stat = float(((oo - ee) ** 2 / ee).sum())
    return float(chi2.sf(stat, len(ee) - 1)), len(ee)


@pytest.mark.parametrize("kind", NAMES)
def test_flashinfer_kept_set_matches_oracle_and_kernel(kind):
    name, x, T, k, p, hist, rp = _row_kinds()[kind]
    rr = _oracle(x, T, k, p, hist, rp)
    z = _divided(x, T, hist, rp)
    fi = _flashinfer_kept(z, k, p)
    # the CUDA sampler's final set, from its y' threshold
    toks, cnts = (hist if hist is not None else (None, None))
    y = so.penalised_logits(x.float().numpy(), "f16", toks, cnts, rp=rp)
    h = None if hist is None else [hist]
    ids, stats, _ = run_gpu(x[None, :], [T], [k], [p], [0.5], history=h,
                            rp=None if hist is None else [rp], use_mval=False)
    ours = y >= stats[0, 1]
    if rr.p_margin < BOUNDARY:
        pytest.skip(f"{name}: top-p tail within {rr.p_margin:.2g} of p*S")
    assert np.array_equal(fi, rr.kept), \
        f"{name}: FlashInfer keeps {int(fi.sum())}, the oracle {int(rr.kept.sum())} " \
        f"({int((fi & ~rr.kept).sum())} only in FlashInfer, {int((rr.kept & ~fi).sum())} only in the oracle)"
    assert np.array_equal(ours, fi), f"{name}: the CUDA sampler keeps {int(ours.sum())}, FlashInfer {int(fi.sum())}"


@pytest.mark.parametrize("kind", NAMES)
def test_flashinfer_draws_follow_oracle_distribution(kind):
    flashinfer = _fi()
    name, x, T, k, p, hist, rp = _row_kinds()[kind]
    rr = _oracle(x, T, k, p, hist, rp)
    z = _divided(x, T, hist, rp)
    V = z.shape[1]
    masked = flashinfer.sampling.top_k_mask_logits(z, k)
    probs = torch.softmax(masked, dim=-1)
    n_call, calls = 250_000, 4
    idx = torch.zeros(n_call, dtype=torch.int32, device="cuda")
    counts = np.zeros(V, dtype=np.int64)
    for s in range(calls):
        d = flashinfer.sampling.top_p_sampling_from_probs(probs, p, indices=idx, deterministic=True,
                                                          seed=1000 + s, offset=0)
        counts += np.bincount(d.cpu().numpy().astype(np.int64), minlength=V)
    n = n_call * calls
    outside = counts[~rr.kept].sum()
    if rr.p_margin >= BOUNDARY:
        assert outside == 0, f"{name}: {outside} of {n} FlashInfer draws outside the oracle's set"
    kept = np.nonzero(rr.kept)[0]
    if len(kept) == 1:
        assert counts[kept[0]] == n
        return
    pval, bins = _chi_square_p(counts[kept].astype(np.float64), n * rr.probs[kept])
    assert pval > 1e-4, f"{name}: chi-square p = {pval:.3g} over {bins} bins"


def test_reference_one_call_draws_stay_in_the_oracle_set():
    """top_k_top_p_sampling_from_logits as ecahlang/main.py:377-379 calls it,
    on 64 copies of every row kind in one batch."""
    flashinfer = _fi()
    reps = 64
    zs, ks, ps, sets = [], [], [], []
    for name, x, T, k, p, hist, rp in _row_kinds().values():
        rr = _oracle(x, T, k, p, hist, rp)
        if rr.p_margin < BOUNDARY:
            continue
        zs.append(_divided(x, T, hist, rp).repeat(reps, 1))
        ks += [k] * reps
        ps += [p] * reps
        sets += [rr.kept] * reps
    z = torch.cat(zs)
    K = torch.tensor(ks, dtype=torch.int32, device="cuda")
    P = torch.tensor(ps, dtype=torch.float32, device="cuda")
    for s in range(4):
        torch.manual_seed(s)
        ids = flashinfer.sampling.top_k_top_p_sampling_from_logits(z, top_k=K, top_p=P,
                                                                   deterministic=True).cpu().numpy()
        bad = [i for i, (t, m) in enumerate(zip(ids, sets)) if not m[t]]
        assert not bad, f"rows {bad[:8]} drew ids outside the oracle's set"
