"""Vocab-parallel rows without top-k (top_k <= 0 or >= vocab: the reference's
default request, ecahlang/main.py:643) through the distributed passes of
ecah_vp_dist_pass.  The ranks are emulated on one GPU: every rank runs each
pass over its own slice, the test combines the outputs as the collective
would (gather in rank order, sum, max) and hands the result to every rank's
combine step.  Every rank must return the same ids, equal to the CPU oracle on
the full rows, for the rows of both paths in one batch."""
import numpy as np
import pytest
import torch

from ecahlang_b200 import sampler as S
from ecahlang_b200.vocab_parallel import VocabParallelSampler, split_vocab
from gpu_util import BOUNDARY
from oracle import sampler_oracle as so
from oracle.philox import row_uniforms
from vp_util import vp_case

pytestmark = pytest.mark.gpu

SEED = 5


def _combine(outs, p):
    st = torch.stack(outs)
    if p in (1, 4):
        return st.contiguous()            # the all-gather, rank order
    if p in (2, 3):
        return st.sum(0).contiguous()     # the all-reduce (sum)
    return st.max(0).values.contiguous()  # the all-reduce (max) of the ids


def _emulated_step(xd, T, K, P, U, world, cap, dtype, pen=None, rows=None):
    """One step on `world` emulated ranks: the candidate path (local lists,
    stacked, merged) and the distributed passes; returns the ids."""
    B, V = xd.shape
    dev = xd.device
    smps = [VocabParallelSampler(B, V, world, g, dtype, dev, seed=SEED, cand_cap=cap, exchange=lambda *a: None)
            for g in range(world)]
    slices = []
    for g in range(world):
        off, loc = split_vocab(V, world, g)
        slices.append(xd[:, off:off + loc].contiguous())
    if rows is None:
        rows, _ = smps[0].find_full_rows(T, K, P)
    kw = {}
    if pen is not None:
        kw = dict(penalty=pen, row_slot=torch.arange(B, dtype=torch.int32, device=dev))
    steps = [smp.full_rows_begin(sl, T, K, P, rows, U, **kw) for smp, sl in zip(smps, slices)]
    lists = [smp.local(sl, T, K, P, **kw) for smp, sl in zip(smps, slices)]
    all_cand = torch.stack([c for c, _ in lists]).contiguous()
    all_count = torch.stack([n for _, n in lists]).contiguous()
    for smp in smps:
        smp.merge(all_cand, all_count, T, K, P, uniforms=U)
    for p in (1, 2, 3, 4, 5):
        outs = [smp.full_rows_pass(st, p).clone() for smp, st in zip(smps, steps)]
        G = _combine(outs, p)
        for smp, st in zip(smps, steps):
            smp.full_rows_combine(st, p, G)
    outs = [smp.out[:B].clone() for smp in smps]
    torch.cuda.synchronize()
    for o in outs[1:]:
        assert torch.equal(o, outs[0]), "ranks disagree"
    return outs[0].cpu().numpy()


def _case(seed, B, V):
    x, T, K, P, U = vp_case(seed, B, V)
    K[0::3] = 0                  # top-k off
    K[1::6] = V                  # top_k = vocab
    P[0::4] = 0.0                # top_p = 0: no top-p (the reference's default)
    return x, T, K, P, U


def _check(got, x, T, K, P, U, dtype="bf16", history=None, rep=None, max_near=2):
    res = so.sample_batch(x, dtype=dtype, temperature=T, top_k=K, top_p=P, uniforms=U, history=history,
                          rep_pen=rep, keep_arrays=False)
    want = np.array([rr.token for rr in res.rows])
    near = np.array([rr.u_margin < BOUNDARY or rr.p_margin < BOUNDARY for rr in res.rows])
    assert (got >= 0).all(), f"rows {np.nonzero(got < 0)[0].tolist()} came back -1"
    bad = np.nonzero((got != want) & ~near)[0]
    assert bad.size == 0, f"rows {bad.tolist()}: got {got[bad].tolist()}, oracle {want[bad].tolist()}"
    assert near.sum() <= max_near


@pytest.mark.parametrize("world", [2, 4, 8])
def test_rows_without_top_k_match_oracle(world):
    dev = torch.device("cuda")
    B, V = 64, 20000
    x, T, K, P, U = _case(51, B, V)
    xd = torch.from_numpy(x).to(torch.bfloat16).to(dev)
    Td, Kd, Pd, Ud = (torch.from_numpy(a).to(dev) for a in (T, K, P, U))
    got = _emulated_step(xd, Td, Kd, Pd, Ud, world, 2048 // world, torch.bfloat16)
    _check(got, x, T, K, P, U)
    # the rows the distributed passes served
    full = (T > 0) & ((K <= 0) | (K >= V))
    assert full.sum() >= 20


def test_rows_without_top_k_philox_fp16():
    """No uniforms given: the step's Philox uniforms are written before the
    merge advances the state, so both paths draw with the same uniforms;
    fp16 slices of an odd-sized vocabulary."""
    dev = torch.device("cuda")
    B, V, world = 40, 20011, 4
    x, T, K, P, _ = _case(53, B, V)
    xd = torch.from_numpy(x).to(torch.float16).to(dev)
    Td, Kd, Pd = (torch.from_numpy(a).to(dev) for a in (T, K, P))
    got = _emulated_step(xd, Td, Kd, Pd, None, world, 512, torch.float16)
    U = row_uniforms(SEED, 0, B)
    _check(got, x, T, K, P, U, dtype="f16")


def test_rows_without_top_k_with_penalties():
    """Repetition-penalty histories whose ids fall in every rank's slice."""
    dev = torch.device("cuda")
    B, V, world = 32, 20000, 4
    x, T, K, P, U = _case(55, B, V)
    rng = np.random.default_rng(56)
    pen = S.PenaltyState(B, 400, torch.bfloat16, dev)
    history = []
    for r in range(B):
        n = int(rng.integers(0, 400))
        toks = np.sort(rng.choice(V, n, replace=False)).astype(np.int32)
        toks[: min(n, 4)] = np.sort(rng.choice(64, min(n, 4), replace=False))   # some near the spikes
        toks = np.unique(toks)
        n = len(toks)
        cnt = rng.integers(1, 4, n).astype(np.int32)
        mv = np.array([so.penalty_divisor(int(c), 1.3, "bf16") for c in cnt], np.float32)
        pen.slot_len[r] = n
        pen.tok[r, :n] = torch.from_numpy(toks)
        pen.cnt[r, :n] = torch.from_numpy(cnt)
        pen.mval[r, :n] = torch.from_numpy(mv)
        history.append((toks, cnt, mv))
    xd = torch.from_numpy(x).to(torch.bfloat16).to(dev)
    Td, Kd, Pd, Ud = (torch.from_numpy(a).to(dev) for a in (T, K, P, U))
    got = _emulated_step(xd, Td, Kd, Pd, Ud, world, 512, torch.bfloat16, pen=pen)
    _check(got, x, T, K, P, U, history=history)


def test_rows_without_top_k_llama3_vocab():
    """The configs[3] shape (V = 128256, bf16 N(0, 3^2) with 8 spikes), every
    row without top-k, top_p 0.9 and 1.0, over 2 and 8 ranks."""
    from ecahlang_b200 import workloads as W
    dev = torch.device("cuda")
    w = W.config4(seed=1, B=24)
    B, V = w.batch, w.vocab
    K = torch.zeros(B, dtype=torch.int32)
    P = w.top_p.clone()
    P[::2] = 1.0
    xd = w.logits.to(dev)
    x = w.logits.float().numpy()
    for world in (2, 8):
        got = _emulated_step(xd, w.temperature.to(dev), K.to(dev), P.to(dev), w.uniforms.to(dev), world, 256,
                             torch.bfloat16)
        _check(got, x, w.temperature.numpy(), K.numpy(), P.numpy(), w.uniforms.numpy())


def test_nan_row_and_listed_top_k_rows():
    """A row without top-k holding a NaN logit comes back -1; rows with a
    top-k listed anyway keep the candidate path's ids."""
    dev = torch.device("cuda")
    B, V, world = 8, 4000, 2
    x, T, K, P, U = vp_case(57, B, V)
    T[:] = 1.0
    K[:] = [0, 0, 5, 20, V, 0, 1, 64]
    x[1, 3000] = np.nan
    xd = torch.from_numpy(x).to(torch.bfloat16).to(dev)
    Td, Kd, Pd, Ud = (torch.from_numpy(a).to(dev) for a in (T, K, P, U))
    rows = torch.arange(B, dtype=torch.int32, device=dev)        # every row listed
    got = _emulated_step(xd, Td, Kd, Pd, Ud, world, 512, torch.bfloat16, rows=rows)
    assert got[1] == -1
    ok = np.array([0, 2, 3, 4, 5, 6, 7])
    xs = x[ok]
    res = so.sample_batch(xs, dtype="bf16", temperature=T[ok], top_k=K[ok], top_p=P[ok], uniforms=U[ok])
    for j, r in enumerate(ok):
        rr = res.rows[j]
        if not (rr.u_margin < BOUNDARY or rr.p_margin < BOUNDARY):
            assert got[r] == rr.token, f"row {r}"


def test_single_rank_call_serves_rows_without_top_k():
    """world = 1 through __call__: the rows are found on the host, the
    collectives are copies, and the ids equal the single-GPU oracle."""
    dev = torch.device("cuda")
    B, V = 32, 20000
    x, T, K, P, U = _case(59, B, V)
    xd = torch.from_numpy(x).to(torch.bfloat16).to(dev)
    Td, Kd, Pd, Ud = (torch.from_numpy(a).to(dev) for a in (T, K, P, U))
    smp = VocabParallelSampler(B, V, 1, 0, torch.bfloat16, dev, seed=SEED, cand_cap=256,
                               exchange=lambda c, n, ac, an: (ac[0].copy_(c), an[0].copy_(n)))
    got = smp(xd, Td, Kd, Pd, uniforms=Ud).cpu().numpy()
    _check(got, x, T, K, P, U)
    # listed explicitly as a device tensor (the graph-capture form)
    got2 = smp(xd, Td, Kd, Pd, uniforms=Ud, full_rows=torch.arange(B, dtype=torch.int32, device=dev))
    assert np.array_equal(got2.cpu().numpy(), got)
