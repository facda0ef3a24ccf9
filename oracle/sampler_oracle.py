"""CPU oracle for the per-step token sampler.

TEST INFRASTRUCTURE ONLY.  Only tests/, ``__graft_entry__.smoke()`` and the
CPU-baseline / reference legs of bench.py may import this module; the product
path (``ecahlang_b200``) never does and fails loudly without its CUDA library.

What it restates (per row r, token i, logits x in the model dtype D):

 1. Repetition-penalty divisor.  The reference keeps a dense table
    ``mask_penalty[slot, V]`` of ones (ecahlang/manager.py:36, reset at
    :109-111) and after every sampled token does ``m /= rp`` if rp > 1 else
    ``m *= rp`` (ecahlang/main.py:691-694, also :519-522, :596-597).  On a CUDA
    tensor, torch evaluates ``m /= rp`` (rp a Python float) as a float32
    multiply by float32(1/rp) with the reciprocal taken in double, so one
    update is ``m <- D(f32(m) * factor)`` with factor = f32(1/rp) (rp > 1) or
    f32(rp) (rp <= 1); measured against torch on the B200
    (tests/test_sampler_gpu.py::test_hist_update_matches_reference_rule).
    ``penalty_divisor`` iterates that rule ``count`` times.
 2. ``y = D(f32(x) / f32(m))`` -- ``logits / mask_penalty`` in the model dtype
    (ecahlang/main.py:169, :398, :486, :579).
 3. Frequency / presence penalties (additive, OpenAI style).  NOT in the
    reference (ecahlang/parameters.py:4-12 exposes only repetition_penalty);
    applied only when the caller enables them:
    ``y' = D(y - f32(f32(f * c) + pi))`` for c > 0: the penalised logit stays
    in the model dtype D, as rule 2's divide leaves it (and as vLLM applies
    these penalties to the logits tensor in its dtype).  Parity unpinned.
 4. ``z = f32(y') / T`` in float32 -- ``logits / temperature`` promotes to
    float32 (ecahlang/main.py:170, :399, :487, :580).  T <= 0 (only reachable
    by bypassing the request normalisation of ecahlang/main.py:642) is a pure
    argmax with the lowest index winning.
 5. Top-k: keep ``z >= tau_k`` with tau_k the k-th largest z counted with
    multiplicity (ties kept), as ``logits < pivot -> -inf`` in
    ecahlang/utils.py:13-15 and FlashInfer ``top_k_mask_logits`` (``>= pivot``).
    k <= 0 or k >= V keeps everything (the request layer maps 0 to V,
    ecahlang/main.py:643).
 6. Softmax over the kept set: ``e = exp(z - M)``, M = max z.
 7. Top-p after top-k (FlashInfer ``top_k_first`` order): keep token i iff the
    mass of tokens with strictly larger z is < p * S, i.e. keep
    ``z >= tau_p`` where tau_p is the largest z value whose tail mass
    ``sum_{z_j >= tau_p} e_j >= p * S``.  p <= 0 or p >= 1 disables it
    (ecahlang/main.py:644 maps 0 to 1.0).
 8. Draw: the smallest vocab index i in the final set whose inclusive
    cumulative mass (vocab order) exceeds ``u * Z``.  The reference draws with
    FlashInfer's rejection sampler and its own Philox stream, which cannot be
    replayed with caller uniforms; the inverse-CDF draw samples the same
    distribution and is what the CUDA path implements.

Masses are accumulated in float64 here.  Each result carries the margins the
parity tests use to exempt boundary cases: the distance of u from the nearest
CDF boundary and of the top-p tail mass from p*S, both relative.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional, Sequence

import numpy as np

DTYPES = ("f16", "bf16", "f32")


# ---------------------------------------------------------------- dtype helpers
def round_to(x, dtype: str) -> np.ndarray:
    """Round float32 values to the model dtype and return them as float32."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "f32":
        return x.copy()
    if dtype == "f16":
        with np.errstate(over="ignore"):
            return x.astype(np.float16).astype(np.float32)
    if dtype == "bf16":
        bits = x.view(np.uint32).astype(np.uint64)
        nan = np.isnan(x)
        rounded = (bits + np.uint64(0x7FFF) + ((bits >> np.uint64(16)) & np.uint64(1))) >> np.uint64(16)
        out = (rounded.astype(np.uint32) << np.uint32(16)).view(np.float32)
        out = np.where(nan, np.float32(np.nan), out)
        return out.astype(np.float32)
    raise ValueError(f"unknown dtype {dtype}")


def repetition_factor(rp: float) -> np.float32:
    """Per-update multiplier of rule 1 for a request's (double) rp."""
    return np.float32(1.0 / rp) if rp > 1.0 else np.float32(rp)


def penalty_divisor(count: int, rp: float, dtype: str) -> np.float32:
    """Value of one ``mask_penalty`` entry after ``count`` updates (rule 1)."""
    m = np.float32(1.0)
    f = repetition_factor(rp)
    for _ in range(int(count)):
        nxt = round_to(np.float32(m * f), dtype)[()]
        if nxt == m or nxt != nxt:
            m = nxt
            break
        m = nxt
    return np.float32(m)


def normalize_request(temperature: float, top_k: int, top_p: float,
                      repetition_penalty: float, vocab: int):
    """Request-parameter normalisation of ecahlang/main.py:642-645."""
    return (max(1e-5, temperature), vocab if top_k == 0 else top_k,
            1.0 if top_p == 0 else top_p, max(1e-5, repetition_penalty))


# ------------------------------------------------------------------- results
@dataclass
class RowResult:
    token: int
    greedy: bool
    kept: Optional[np.ndarray] = None      # bool [V]: final (top-k then top-p) set
    probs: Optional[np.ndarray] = None     # float64 [V]: renormalised over kept
    topk_kept: Optional[np.ndarray] = None  # bool [V]: top-k set only
    u_margin: float = float("inf")         # |u - nearest CDF boundary|
    p_margin: float = float("inf")         # |tail mass - p*S| / S at the cut
    z: Optional[np.ndarray] = None


@dataclass
class BatchResult:
    tokens: np.ndarray
    rows: List[RowResult] = field(default_factory=list)


# --------------------------------------------------------------------- oracle
def penalised_logits(x, dtype, toks=None, cnts=None, mvals=None, rp=1.0,
                     freq=0.0, pres=0.0, freq_pres=False) -> np.ndarray:
    """Rules 1-3 for one row: returns y' as float32."""
    y = np.asarray(x, dtype=np.float32).copy()
    if toks is None or len(toks) == 0:
        return y
    toks = np.asarray(toks, dtype=np.int64)
    cnts = np.asarray(cnts, dtype=np.int64)
    live = cnts > 0
    toks, cnts = toks[live], cnts[live]
    if mvals is None:
        cache = {}
        m = np.empty(len(toks), dtype=np.float32)
        for j, c in enumerate(cnts):
            if c not in cache:
                cache[c] = penalty_divisor(int(c), rp, dtype)
            m[j] = cache[c]
    else:
        m = np.asarray(mvals, dtype=np.float32)[live]
    yv = round_to(y[toks] / m, dtype)
    if freq_pres:
        pen = (np.float32(freq) * cnts.astype(np.float32)).astype(np.float32)
        pen = (pen + np.float32(pres)).astype(np.float32)
        yv = round_to((yv - pen).astype(np.float32), dtype)
    y[toks] = yv
    return y


def sample_row(x, *, dtype="f32", temperature=1.0, top_k=0, top_p=1.0, u=0.5,
               toks=None, cnts=None, mvals=None, rp=1.0, freq=0.0, pres=0.0,
               freq_pres=False, keep_arrays=True) -> RowResult:
    """Rules 1-8 for one row."""
    y = penalised_logits(x, dtype, toks, cnts, mvals, rp, freq, pres, freq_pres)
    V = y.shape[0]
    T = np.float32(temperature)
    if not (T > 0):
        return RowResult(token=int(np.argmax(y)), greedy=True)
    z = (y / T).astype(np.float32)
    k = int(top_k)
    k_eff = V if (k <= 0 or k >= V) else k
    if k_eff < V:
        tau_k = np.partition(z, V - k_eff)[V - k_eff]
        K = z >= tau_k
    else:
        K = np.ones(V, dtype=bool)
    M = z.max()
    d = (z - M).astype(np.float32).astype(np.float64)
    e = np.where(K, np.exp(d), 0.0)
    S = e.sum()
    p = float(top_p)
    p_margin = float("inf")
    if 0.0 < p < 1.0:
        target = np.float64(np.float32(p)) * S
        zk = z[K]
        ek = e[K]
        vals, inv = np.unique(zk, return_inverse=True)        # ascending
        mass = np.bincount(inv, weights=ek, minlength=len(vals))
        tail = np.cumsum(mass[::-1])                           # mass of z >= vals[::-1][j]
        j = int(np.searchsorted(tail, target, side="left"))   # first tail >= target
        j = min(j, len(vals) - 1)
        tau_p = vals[::-1][j]
        F = K & (z >= tau_p)
        above = tail[j - 1] if j > 0 else 0.0
        p_margin = min(abs(tail[j] - target), abs(target - above)) / S
    else:
        F = K
    eF = np.where(F, e, 0.0)
    C = np.cumsum(eF)
    Z = C[-1]
    uu = float(np.float32(u))
    t = uu * Z
    i = int(np.searchsorted(C, t, side="right"))
    if i >= V:
        i = int(np.nonzero(eF > 0)[0][-1])
    lo = C[i - 1] if i > 0 else 0.0
    u_margin = min(t - lo, C[i] - t) / Z
    res = RowResult(token=i, greedy=False, u_margin=float(u_margin), p_margin=float(p_margin))
    if keep_arrays:
        res.kept = F
        res.topk_kept = K
        res.probs = eF / Z
        res.z = z
    return res


def sample_batch(logits, *, dtype="f32", temperature, top_k, top_p, uniforms,
                 history=None, rep_pen=None, freq_pen=None, pres_pen=None,
                 freq_pres=False, keep_arrays=False) -> BatchResult:
    """Rows of ``sample_row``.  ``history`` is a list (per row) of
    (toks, cnts) or (toks, cnts, mvals) tuples, or None."""
    logits = np.asarray(logits, dtype=np.float32)
    B = logits.shape[0]
    out = np.empty(B, dtype=np.int32)
    rows = []
    for r in range(B):
        h = history[r] if history is not None else None
        toks = cnts = mv = None
        if h is not None:
            toks, cnts = h[0], h[1]
            mv = h[2] if len(h) > 2 else None
        rr = sample_row(
            logits[r], dtype=dtype, temperature=float(temperature[r]),
            top_k=int(top_k[r]), top_p=float(top_p[r]), u=float(uniforms[r]),
            toks=toks, cnts=cnts, mvals=mv,
            rp=1.0 if rep_pen is None else float(rep_pen[r]),
            freq=0.0 if freq_pen is None else float(freq_pen[r]),
            pres=0.0 if pres_pen is None else float(pres_pen[r]),
            freq_pres=freq_pres, keep_arrays=keep_arrays)
        out[r] = rr.token
        rows.append(rr)
    return BatchResult(tokens=out, rows=rows)


def exponential_race_ids(probs_rows: Sequence[np.ndarray], q) -> np.ndarray:
    """argmax(probs / q) per row: the draw of ecahlang/utils.py:17-18 given the
    reference's own exponential variates q, used to pin rules 1-6 against
    ``logits_to_probs`` bit for bit."""
    q = np.asarray(q, dtype=np.float64)
    return np.array([int(np.argmax(p / q[i])) for i, p in enumerate(probs_rows)], dtype=np.int64)
