"""Generate the golden fixtures in this folder from the reference itself.

Run once in a container where the reference checkout is importable:

    python tests/golden/make_golden.py --reference /path/to/ecahLang

It imports ``ecahlang.utils.logits_to_probs`` (ecahlang/utils.py:3-18), the
reference's own torch sampling path, and runs it on CPU for seeded inputs.
For every case it stores the inputs, the reference's sampled ids, and the
exponential variates ``q`` the reference drew inside the call
(ecahlang/utils.py:17: ``torch.empty_like(probs).exponential_(1)``), obtained by
re-seeding torch's CPU generator identically; nothing before that line in
``logits_to_probs`` consumes random numbers.

The repetition-penalty table handed to the reference is built with the
reference's own update statement (``mask[slot, tok] /= rp`` for rp > 1, else
``*= rp``; ecahlang/main.py:691-694) applied ``count`` times on a torch tensor,
so the fixture pins the penalty division, the temperature division, the top-k
pivot with ties and the softmax.  The update rounding on CUDA tensors is
pinned separately on the GPU (tests/test_sampler_gpu.py).
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
TORCH_DT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


def make_case(name, *, seed, B, V, dtype, sigma=3.0, spikes=3, spike_val=8.0,
              quantum=None, with_history=True, store_q=True):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, V, generator=g) * sigma
    if quantum is not None:
        x = torch.round(x / quantum) * quantum
    for r in range(B):
        idx = torch.randperm(V, generator=g)[:spikes]
        x[r, idx] = spike_val
    x = x.to(TORCH_DT[dtype])

    temps = [1e-5, 0.3, 0.7, 1.0, 1.5, 2.0, 0.9, 1.2]
    ks = [1, 3, 5, 20, 50, V, 100, 7]
    T = torch.tensor([temps[r % len(temps)] for r in range(B)], dtype=torch.float32)[:, None]
    K = torch.tensor([min(ks[(r * 3) % len(ks)], V) for r in range(B)], dtype=torch.int64)

    mask = torch.ones(B, V, dtype=TORCH_DT[dtype])
    hist_toks, hist_cnts, hist_rp = [], [], []
    rps = [1.1, 1.3, 0.9, 1.0, 2.0]
    for r in range(B):
        if not with_history or r % 4 == 3:
            hist_toks.append(np.zeros(0, np.int32)); hist_cnts.append(np.zeros(0, np.int32))
            hist_rp.append(1.0)
            continue
        rp = rps[r % len(rps)]
        n = 12
        toks = torch.randperm(V, generator=g)[:n]
        # make the top spike a history token on some rows so penalties move the max
        cnts = torch.randint(1, 7, (n,), generator=g)
        for t, c in zip(toks.tolist(), cnts.tolist()):
            for _ in range(c):
                if rp > 1:
                    mask[r, t] /= rp
                else:
                    mask[r, t] *= rp
        hist_toks.append(toks.numpy().astype(np.int32))
        hist_cnts.append(cnts.numpy().astype(np.int32))
        hist_rp.append(rp)

    from ecahlang.utils import logits_to_probs

    qseed = seed + 1000
    torch.manual_seed(qseed)
    ids = logits_to_probs(x, mask, T, K, None)
    torch.manual_seed(qseed)
    probs_shape = torch.empty(B, V, dtype=torch.float32)
    q = torch.empty_like(probs_shape).exponential_(1)

    ht = np.concatenate(hist_toks)
    hc = np.concatenate(hist_cnts)
    hptr = np.cumsum([0] + [len(a) for a in hist_toks]).astype(np.int32)
    hm = np.concatenate([mask[r, torch.from_numpy(hist_toks[r]).long()].float().numpy()
                         for r in range(B)]).astype(np.float32)
    if dtype == "f16":
        xs = x.numpy()                                   # float16
    elif dtype == "bf16":
        xs = x.view(torch.int16).numpy().view(np.uint16)  # raw bf16 bits
    else:
        xs = x.numpy()
    out = dict(
        name=name, dtype=dtype, logits=xs, temperature=T[:, 0].numpy(),
        top_k=K.numpy().astype(np.int32), hist_ptr=hptr, hist_tok=ht, hist_cnt=hc,
        hist_mval=hm, rep_pen=np.array(hist_rp, np.float32),
        ref_ids=ids[:, 0].numpy().astype(np.int64), qseed=np.int64(qseed),
    )
    if store_q:
        out["q"] = q.numpy()
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **out)
    print(name, "ids", out["ref_ids"][:8])


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("ECAH_REFERENCE", ""))
    a = ap.parse_args()
    if not a.reference:
        sys.exit("pass --reference <path to the ecahLang checkout>")
    sys.path.insert(0, a.reference)
    make_case("ref_f32_basic", seed=1, B=16, V=2048, dtype="f32")
    make_case("ref_f16_basic", seed=2, B=16, V=2048, dtype="f16", sigma=2.5)
    make_case("ref_bf16_basic", seed=3, B=16, V=2048, dtype="bf16")
    make_case("ref_f32_ties", seed=4, B=16, V=1024, dtype="f32", quantum=0.5, spikes=6)
    make_case("ref_f16_ties", seed=5, B=16, V=1024, dtype="f16", quantum=0.25, spikes=6)
    make_case("ref_f16_vocab", seed=6, B=4, V=151936, dtype="f16", sigma=2.5,
              spikes=5, spike_val=12.0, store_q=False)


if __name__ == "__main__":
    main()
