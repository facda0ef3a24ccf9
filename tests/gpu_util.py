"""Shared helpers of the GPU parity tests: run the CUDA sampler through the
C ABI and compare it with the CPU oracle on the same inputs."""
from __future__ import annotations

import numpy as np
import torch

from ecahlang_b200 import sampler as S
from oracle import sampler_oracle as so

DT = {torch.float16: "f16", torch.bfloat16: "bf16", torch.float32: "f32"}
BOUNDARY = 1e-6     # u / top-p margins below this are reported, not asserted


ROW_KERNEL_BATCH = 40   # batches from this size on run one unsplit CTA per row (148 SMs)


def tiled(B):
    """Copies of a B-row batch that reach the row-per-CTA kernel's batch size."""
    return -(-ROW_KERNEL_BATCH // B)


def run_gpu(x, T, K, P, U, *, history=None, rp=None, f=None, pi=None, freq_pres=False,
            use_mval=True, probs=False, row_stride=None, tile=1):
    """x: CPU [B,V] model dtype.  history: per row (toks, cnts[, mvals]) or None.
    tile > 1 samples `tile` stacked copies of the batch in one launch (so a
    small case also runs through the kernel for large batches); every copy
    must give the same results, and the first copy's are returned."""
    if tile > 1:
        B0 = x.shape[0]
        rep = lambda a: None if a is None else np.tile(np.asarray(a), tile)
        out = run_gpu(x.repeat(tile, 1), rep(T), rep(K), rep(P), rep(U),
                      history=None if history is None else list(history) * tile,
                      rp=rep(rp), f=rep(f), pi=rep(pi), freq_pres=freq_pres, use_mval=use_mval,
                      probs=probs, row_stride=row_stride)
        ids, stats, po = out
        for t in range(1, tile):
            sl = slice(t * B0, (t + 1) * B0)
            assert np.array_equal(ids[sl], ids[:B0]), f"copy {t}: ids differ"
            assert np.array_equal(stats[sl], stats[:B0], equal_nan=True), f"copy {t}: row stats differ"
            if po is not None:
                assert np.array_equal(po[sl], po[:B0]), f"copy {t}: probabilities differ"
        return ids[:B0], stats[:B0], (po[:B0] if po is not None else None)
    dev = torch.device("cuda")
    B, V = x.shape
    if row_stride is not None and row_stride != V:
        buf = torch.zeros(B, row_stride, dtype=x.dtype)
        buf[:, :V] = x
        xd = buf.to(dev)[:, :V]
    else:
        xd = x.to(dev)
    out = torch.full((B,), -1, dtype=torch.int32, device=dev)
    stats = torch.zeros(B, 4, dtype=torch.float32, device=dev)
    po = torch.zeros(B, V, dtype=torch.float32, device=dev) if probs else None
    ws = S.new_workspace(B, V, x.dtype, dev)
    pen = row_slot = None
    if history is not None:
        cap = max(1, max(len(h[0]) for h in history))
        pen = S.PenaltyState(B, cap, x.dtype, dev)
        for r, h in enumerate(history):
            pen.load(r, h[0], h[1], h[2] if len(h) > 2 else None)
        row_slot = torch.arange(B, dtype=torch.int32, device=dev)
    f32 = lambda t: None if t is None else torch.as_tensor(t, dtype=torch.float32).to(dev)
    S.launch(xd, f32(T), torch.as_tensor(K, dtype=torch.int32).to(dev), f32(P), out, ws,
             uniforms=f32(U), rep_factor=None if rp is None else f32(S.repetition_factor(rp)),
             freq_pen=f32(f), pres_pen=f32(pi), penalty=pen,
             row_slot=row_slot, freq_pres=freq_pres, use_mval=use_mval, row_stats=stats, probs_out=po)
    torch.cuda.synchronize()
    return out.cpu().numpy(), stats.cpu().numpy(), (po.cpu().numpy() if probs else None)


def run_oracle(x, T, K, P, U, *, history=None, rp=None, f=None, pi=None, freq_pres=False):
    xf = x.float().numpy()
    return so.sample_batch(xf, dtype=DT[x.dtype], temperature=np.asarray(T), top_k=np.asarray(K),
                           top_p=np.asarray(P), uniforms=np.asarray(U, dtype=np.float32),
                           history=history, rep_pen=rp, freq_pen=f, pres_pen=pi,
                           freq_pres=freq_pres, keep_arrays=True)


def compare(x, T, K, P, U, gpu, orc, *, history=None, rp=None, f=None, pi=None, freq_pres=False,
            prob_rtol=1e-5, probs=None):
    """Assert parity; returns the number of rows exempted as CDF/top-p boundary cases."""
    ids, stats, _ = gpu
    xf = x.float().numpy()
    B, V = xf.shape
    boundary = 0
    for r in range(B):
        rr = orc.rows[r]
        if rr.greedy:
            assert ids[r] == rr.token, f"row {r}: greedy id {ids[r]} != {rr.token}"
            continue
        h = history[r] if history is not None else None
        y = so.penalised_logits(xf[r], DT[x.dtype], *(h[:2] if h else (None, None)),
                                mvals=(h[2] if h is not None and len(h) > 2 else None),
                                rp=1.0 if rp is None else float(rp[r]),
                                freq=0.0 if f is None else float(f[r]),
                                pres=0.0 if pi is None else float(pi[r]), freq_pres=freq_pres)
        kk = int(K[r])
        if 0 < kk < V:
            got_k = y >= stats[r, 0]
            assert np.array_equal(got_k, rr.topk_kept), \
                f"row {r}: top-k set differs ({got_k.sum()} vs {rr.topk_kept.sum()})"
        near = rr.u_margin < BOUNDARY or rr.p_margin < BOUNDARY
        if rr.p_margin >= BOUNDARY:
            got_f = y >= stats[r, 1]
            assert np.array_equal(got_f, rr.kept), \
                f"row {r}: final set differs ({got_f.sum()} vs {rr.kept.sum()})"
        if near:
            boundary += 1
        else:
            assert ids[r] == rr.token, (f"row {r}: id {ids[r]} != oracle {rr.token} "
                                        f"(u_margin {rr.u_margin:.3g}, p_margin {rr.p_margin:.3g})")
        if probs is not None and rr.p_margin >= BOUNDARY:
            want = rr.probs
            got = probs[r].astype(np.float64)
            err = np.abs(got - want)
            bad = err > prob_rtol * want + 1e-12
            assert not bad.any(), (f"row {r}: {bad.sum()} probabilities off, max rel "
                                   f"{(err / np.maximum(want, 1e-30))[bad].max():.3g}")
    return boundary
