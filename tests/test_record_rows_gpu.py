"""GPU parity of top-p rows without top-k that the row kernel finishes from
per-chunk records (the two largest keys of every 16 entries) instead of a
candidate buffer.  Batches of 40 rows and more run one unsplit CTA per row on
148 SMs, which is where those rows take the record path; the cases cover the
re-read list within and beyond its shared-memory cache, chunks whose two largest
keys tie, penalised rows, odd vocabulary sizes around the record capacity
(12 rounds of 16384 entries) and rows whose nucleus the records cannot place
(they fall back to the re-streaming paths)."""
import numpy as np
import pytest
import torch

from gpu_util import compare, run_gpu, run_oracle
from ecahlang_b200 import workloads as W
from oracle import sampler_oracle as so
from oracle.philox import row_uniforms

pytestmark = pytest.mark.gpu

B_UNSPLIT = 40   # unsplit rows from 38 on (148 SMs / 4 parts)


def _c2_like(seed, B, V, dtype, sigma=2.5, shift=6.0, frac=0.03):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, V, generator=g) * sigma
    n = int(round(frac * V))
    idx = torch.argsort(torch.rand(B, V, generator=g), dim=1)[:, :n]
    x.scatter_add_(1, idx, torch.full(idx.shape, shift))
    return x.to(dtype)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_record_top_p_rows(dtype):
    """C2's top-p distribution over a spread of p and T."""
    B, V = 64, W.V_QWEN
    x = _c2_like(71, B, V, dtype)
    ps = [0.3, 0.5, 0.8, 0.9, 0.95, 0.99, 0.999, 0.8]
    ts = [0.5, 0.8, 1.0, 1.3]
    P = np.array([ps[r % len(ps)] for r in range(B)], np.float32)
    T = np.array([ts[(r // len(ps)) % len(ts)] for r in range(B)], np.float32)
    K = np.full(B, V, np.int32)
    U = row_uniforms(71, 1, B)
    gpu = run_gpu(x, T, K, P, U, probs=True)
    orc = run_oracle(x, T, K, P, U)
    nb = compare(x, T, K, P, U, gpu, orc, probs=gpu[2])
    # p = 0.99 / 0.999 at T = 1.3 leave thousands of entries in the nucleus:
    # CDF steps close to 1e-6 apart, so several ids are boundary cases
    assert nb <= B // 4


def test_record_top_p_ties_in_chunks():
    """Logits on a coarse grid, so most chunks' two largest keys tie and many
    chunks are re-read; plus rows with runs of equal maxima."""
    B, V = 48, W.V_QWEN
    g = torch.Generator().manual_seed(72)
    x = torch.round(torch.randn(B, V, generator=g) * 2.0) * 0.5
    for r in range(0, B, 3):
        x[r, r * 97: r * 97 + 40] = 9.0     # 40 ties at the max in consecutive chunks
    x = x.half()
    P = np.array([(0.5, 0.9, 0.95, 0.99)[r % 4] for r in range(B)], np.float32)
    T = np.array([(1.0, 0.7, 1.2)[r % 3] for r in range(B)], np.float32)
    K = np.full(B, V, np.int32)
    U = row_uniforms(72, 0, B)
    gpu = run_gpu(x, T, K, P, U, probs=True)
    orc = run_oracle(x, T, K, P, U)
    nb = compare(x, T, K, P, U, gpu, orc, probs=gpu[2])
    assert nb <= B // 4


def test_record_top_p_wide_nucleus():
    """C3's wide Gaussian (no shifted group): at T = 0.8 and p = 0.95 some
    thousand chunks hold a second nucleus entry, more than the shared-memory
    cache holds, so those rows leave the record path for the re-streaming
    paths; narrower nuclei (lower p or T) stay on it."""
    B, V = 48, W.V_QWEN
    g = torch.Generator().manual_seed(73)
    x = (torch.randn(B, V, generator=g) * 2.5).half()
    T = np.array([(0.8, 1.0, 0.6)[r % 3] for r in range(B)], np.float32)
    P = np.array([(0.95, 0.9, 0.8, 0.99)[r % 4] for r in range(B)], np.float32)
    K = np.full(B, V, np.int32)
    U = row_uniforms(73, 0, B)
    gpu = run_gpu(x, T, K, P, U, probs=True)
    orc = run_oracle(x, T, K, P, U)
    nb = compare(x, T, K, P, U, gpu, orc, probs=gpu[2])
    assert nb <= B // 8


@pytest.mark.parametrize("freq_pres", [False, True])
def test_record_top_p_penalised(freq_pres):
    """C3 unsplit (B = 40): Zipf histories with the repetition penalty, with
    and without frequency and presence penalties; re-read chunks carry the
    penalty patch."""
    w = W.config3(seed=1, B=B_UNSPLIT)
    rp = w.rep_pen.numpy()
    hist = [(t, c, np.array([so.penalty_divisor(int(ci), float(rp[r]), "f16") for ci in c], np.float32))
            for r, (t, c) in enumerate(w.history)]
    args = dict(history=hist, rp=rp)
    if freq_pres:
        args.update(f=w.freq_pen.numpy(), pi=w.pres_pen.numpy(), freq_pres=True)
    gpu = run_gpu(w.logits, w.temperature, w.top_k, w.top_p, w.uniforms, probs=True, **args)
    orc = run_oracle(w.logits, w.temperature, w.top_k, w.top_p, w.uniforms, **args)
    nb = compare(w.logits, w.temperature, w.top_k, w.top_p, w.uniforms, gpu, orc, probs=gpu[2], **args)
    assert nb <= B_UNSPLIT // 8


@pytest.mark.parametrize("V", [16400, 151935, 196607, 196608, 196609, 200000])
def test_record_top_p_vocab_sizes(V):
    """Ragged last chunks and rounds, and the record capacity: up to 12
    rounds (196608 entries) the records fit, past it the rows keep
    candidates."""
    B = B_UNSPLIT
    x = _c2_like(74 + V, B, V, torch.float16)
    P = np.array([(0.8, 0.95, 0.5, 0.99)[r % 4] for r in range(B)], np.float32)
    T = np.array([(1.0, 0.7)[r % 2] for r in range(B)], np.float32)
    K = np.full(B, V, np.int32)
    U = row_uniforms(74, V, B)
    gpu = run_gpu(x, T, K, P, U)
    orc = run_oracle(x, T, K, P, U)
    nb = compare(x, T, K, P, U, gpu, orc)
    assert nb <= B // 8


def test_record_top_p_nucleus_beyond_window():
    """Nearly flat rows: the records' bound does not reach p S within the
    4096 keys under the row max, so the row takes the dense top-p passes."""
    B, V = B_UNSPLIT, W.V_QWEN
    g = torch.Generator().manual_seed(75)
    x = (torch.randn(B, V, generator=g) * 0.5).half()
    T = np.array([(0.7, 1.0)[r % 2] for r in range(B)], np.float32)
    P = np.array([(0.9, 0.5)[r % 2] for r in range(B)], np.float32)
    K = np.full(B, V, np.int32)
    U = row_uniforms(75, 0, B)
    gpu = run_gpu(x, T, K, P, U)
    orc = run_oracle(x, T, K, P, U)
    nb = compare(x, T, K, P, U, gpu, orc)
    assert nb <= B // 2


def test_record_top_p_max_beyond_round_zero():
    """A dominant token (and a few runners-up) placed after the first 16384
    entries, far above the first round's max: the records' histogram, kept
    from round 0's max upward, does not reach the row max, so the finish
    counts the records again; also rows whose nucleus is that one token."""
    B, V = B_UNSPLIT, W.V_QWEN
    x = _c2_like(76, B, V, torch.float32, sigma=1.0, shift=2.0)
    g = torch.Generator().manual_seed(76)
    for r in range(B):
        pos = 20000 + int(torch.randint(0, V - 20000, (1,), generator=g))
        x[r, pos] = 30.0 + (r % 5)                  # dominant
        if r % 2:
            x[r, (pos + 777) % V] = 28.0 + (r % 3)  # a runner-up two units below
    x = x.half()
    P = np.array([(0.5, 0.9, 0.99, 0.999)[r % 4] for r in range(B)], np.float32)
    T = np.array([(1.0, 3.0, 6.0)[r % 3] for r in range(B)], np.float32)
    K = np.full(B, V, np.int32)
    U = row_uniforms(76, 0, B)
    gpu = run_gpu(x, T, K, P, U, probs=True)
    orc = run_oracle(x, T, K, P, U)
    nb = compare(x, T, K, P, U, gpu, orc, probs=gpu[2])
    # at T = 3 and 6 with p = 0.99 / 0.999 the nucleus spans most of the
    # bulk, so ids within 1e-6 of a CDF step are common (sets and
    # probabilities are still checked on those rows)
    assert nb <= B // 4
