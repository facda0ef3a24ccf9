"""Pin the CPU oracle against the reference's own sampler.

The fixtures in tests/golden/ hold outputs of ``ecahlang.utils.logits_to_probs``
(ecahlang/utils.py:3-18) run on seeded inputs, together with the exponential
variates q it drew.  The reference draws ``argmax(probs / q)``; feeding the
oracle's probabilities (rules 1-6 of oracle/sampler_oracle.py) through the
same q must reproduce the reference's ids.
"""
import numpy as np
import pytest
import torch

from conftest import GOLDEN_CASES, golden_history, load_golden
from oracle import sampler_oracle as so


def _q_for(d):
    if "q" in d:
        return d["q"]
    B, V = d["logits_f32"].shape
    torch.manual_seed(int(d["qseed"]))
    return torch.empty(B, V, dtype=torch.float32).exponential_(1).numpy()


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_oracle_reproduces_reference_ids(name):
    d = load_golden(name)
    x = d["logits_f32"]
    B, V = x.shape
    hist = golden_history(d)
    q = _q_for(d)
    mismatches = []
    for r in range(B):
        toks, cnts, mv = hist[r]
        res = so.sample_row(x[r], dtype=d["dtype"], temperature=float(d["temperature"][r]),
                            top_k=int(d["top_k"][r]), top_p=1.0, u=0.5,
                            toks=toks, cnts=cnts, mvals=mv)
        ratio = res.probs / q[r].astype(np.float64)
        mine = int(np.argmax(ratio))
        ref = int(d["ref_ids"][r])
        if mine != ref:
            # only tolerated when the two ratios agree to float32 resolution
            rel = abs(ratio[mine] - ratio[ref]) / ratio[mine]
            mismatches.append((r, mine, ref, rel))
        assert res.kept[ref], f"row {r}: reference id {ref} outside the oracle's kept set"
    hard = [m for m in mismatches if m[3] > 1e-6]
    assert not hard, f"{name}: oracle disagrees with reference: {hard}"


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_penalty_table_matches_reference_rule(name):
    """The fixture's mask values were made by the reference's update statement
    on a torch tensor; the oracle's iterated rule must give the same values."""
    d = load_golden(name)
    ptr = d["hist_ptr"]
    for r in range(len(ptr) - 1):
        s, e = ptr[r], ptr[r + 1]
        rp = float(d["rep_pen"][r])
        for c, m in zip(d["hist_cnt"][s:e], d["hist_mval"][s:e]):
            # CPU torch divides by the scalar itself; the CUDA reciprocal rule can
            # differ in the last place, so compare both against the CPU value.
            exact = so.round_to(np.float32(1.0), d["dtype"])[()]
            for _ in range(int(c)):
                exact = so.round_to(np.float32(exact / np.float32(rp)) if rp > 1
                                    else np.float32(exact * np.float32(rp)), d["dtype"])[()]
            assert exact == m, (name, r, c, exact, m)
            recip = so.penalty_divisor(int(c), rp, d["dtype"])
            assert abs(float(recip) - float(m)) <= abs(float(m)) * 2 ** -7, (name, r, c, recip, m)


def test_topk_ties_inclusive():
    x = np.array([1, 3, 3, 3, 2, 0], dtype=np.float32)
    r = so.sample_row(x, temperature=1.0, top_k=2, u=0.0)
    assert r.topk_kept.tolist() == [False, True, True, True, False, False]


def test_topp_keeps_tie_group_and_minimal_prefix():
    x = np.log(np.array([0.5, 0.2, 0.2, 0.1], dtype=np.float64)).astype(np.float32)
    r = so.sample_row(x, temperature=1.0, top_p=0.6, u=0.0)
    # 0.5 alone < 0.6, the tie group {0.2, 0.2} is kept whole
    assert r.kept.tolist() == [True, True, True, False]
    r = so.sample_row(x, temperature=1.0, top_p=0.5, u=0.0)
    assert r.kept.tolist() == [True, False, False, False]


def test_draw_is_inverse_cdf_in_vocab_order():
    x = np.zeros(4, dtype=np.float32)      # uniform over 4
    for u, want in [(0.0, 0), (0.2499, 0), (0.25, 1), (0.74, 2), (0.9999, 3)]:
        assert so.sample_row(x, temperature=1.0, u=u).token == want


def test_greedy_lowest_index():
    x = np.array([0, 5, 5, 1], dtype=np.float32)
    assert so.sample_row(x, temperature=0.0).token == 1


def test_normalize_request_matches_reference():
    assert so.normalize_request(0.0, 0, 0.0, 0.0, 100) == (1e-5, 100, 1.0, 1e-5)
    assert so.normalize_request(0.7, 50, 0.9, 1.1, 100) == (0.7, 50, 0.9, 1.1)


def test_chi_square_inverse_cdf():
    """1e6 inverse-CDF draws from Philox uniforms follow the oracle's probs."""
    from oracle.philox import row_uniforms
    rng = np.random.default_rng(0)
    x = (rng.standard_normal(64) * 1.5).astype(np.float32)
    res = so.sample_row(x, temperature=0.8, top_k=40, top_p=0.9, u=0.5)
    n = 1_000_000
    u = row_uniforms(seed=7, offset=0, batch=n)
    C = np.cumsum(res.probs)
    ids = np.minimum(np.searchsorted(C, u.astype(np.float64) * C[-1], side="right"), 63)
    counts = np.bincount(ids, minlength=64)
    keep = res.probs > 0
    exp = res.probs[keep] * n
    chi2 = ((counts[keep] - exp) ** 2 / exp).sum()
    dof = keep.sum() - 1
    assert counts[~keep].sum() == 0
    assert chi2 < dof + 6 * np.sqrt(2 * dof), (chi2, dof)
