"""GPU parity of the CUDA sampler against the CPU oracle (oracle/), through the
C ABI.  Greedy ids and top-k sets must be bit-exact; final (top-p) sets,
probabilities (1e-5 relative) and sampled ids must match except for rows
whose u or top-p tail mass lies within 1e-6 of a boundary, which are counted
and must stay rare."""
import numpy as np
import pytest
import torch

from conftest import GOLDEN_CASES, golden_history, load_golden
from gpu_util import BOUNDARY, compare, run_gpu, run_oracle, tiled
from ecahlang_b200 import sampler as S
from ecahlang_b200 import workloads as W
from oracle import sampler_oracle as so
from oracle.philox import row_uniforms

pytestmark = pytest.mark.gpu

TDT = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}


def _golden_tensor(d):
    x = torch.from_numpy(d["logits_f32"].copy())
    return x.to(TDT[d["dtype"]])


@pytest.mark.parametrize("name", GOLDEN_CASES)
@pytest.mark.parametrize("top_p", [1.0, 0.9, 0.5])
@pytest.mark.parametrize("big_batch", [False, True])
def test_golden_fixtures(name, top_p, big_batch):
    """The reference-pinned fixtures (penalty table, temperatures, top-k with
    ties) through the CUDA path, with and without top-p; big_batch stacks
    copies of the rows so they also run through the large-batch kernel."""
    d = load_golden(name)
    x = _golden_tensor(d)
    B, V = x.shape
    hist = golden_history(d)
    T, K = d["temperature"], d["top_k"]
    P = np.full(B, top_p, np.float32)
    U = row_uniforms(11, 3, B)
    gpu = run_gpu(x, T, K, P, U, history=hist, probs=V <= 4096, tile=tiled(B) if big_batch else 1)
    orc = run_oracle(x, T, K, P, U, history=hist)
    nb = compare(x, T, K, P, U, gpu, orc, history=hist, probs=gpu[2])
    assert nb <= max(1, B // 8)


def test_config2_mixed_full_size():
    w = W.config2(seed=0)
    gpu = run_gpu(w.logits, w.temperature, w.top_k, w.top_p, w.uniforms)
    orc = run_oracle(w.logits, w.temperature, w.top_k, w.top_p, w.uniforms)
    nb = compare(w.logits, w.temperature, w.top_k, w.top_p, w.uniforms, gpu, orc)
    assert nb <= 2


def _warp_slices(V, w, rounds_of=16384, slice_len=512):
    """Row positions one warp of the one-CTA-per-row kernel streams: entries
    [r * 16384 + 512 w, + 512) of every 16384-entry round r."""
    idx = np.concatenate([np.arange(r + slice_len * w, r + slice_len * (w + 1)) for r in range(0, V, rounds_of)])
    return idx[idx < V]


def test_row_kernel_warp_regions_and_overflow():
    """Rows whose high logits all sit in one warp's slices, so that warp's
    candidate region fills and is compacted, and rows whose ties at the max
    exceed a region, so the row falls back to the radix re-stream; plus
    top-k rows with k above a region's share.  B = 128 (row kernel)."""
    g = torch.Generator().manual_seed(41)
    B, V = 128, W.V_QWEN
    x = torch.randn(B, V, generator=g) * 2.5
    T = np.ones(B, np.float32)
    K = np.zeros(B, np.int32)
    P = np.ones(B, np.float32)
    for r in range(B):
        w = r % 32
        sl = torch.from_numpy(_warp_slices(V, w))
        if r < 32:              # top-p, nucleus concentrated in one warp's slices
            x[r, sl] += 8.0
            P[r] = (0.95, 0.6)[r % 2]
        elif r < 64:            # top-k 200 concentrated in one warp's slices
            x[r, sl] += 6.0
            K[r] = 200
            T[r] = 0.8
        elif r < 80:            # 600 ties at the max inside one warp's slices
            x[r, sl[:600]] = 20.0
            K[r] = (10, 0)[r % 2]
            P[r] = (1.0, 0.9)[r % 2]
        elif r < 96:            # large k, spread: every warp compacts
            K[r] = (2000, 1000)[r % 2]
            P[r] = (1.0, 0.8)[r % 2]
        else:                   # spread top-p / top-k + top-p
            K[r] = (0, 50)[r % 2]
            P[r] = (0.95, 0.9)[r % 2]
            T[r] = (1.0, 0.7)[r % 2]
    x = x.half()
    U = row_uniforms(17, 2, B)
    gpu = run_gpu(x, T, K, P, U)
    orc = run_oracle(x, T, K, P, U)
    nb = compare(x, T, K, P, U, gpu, orc)
    assert nb <= 3


@pytest.mark.parametrize("use_mval", [True, False])
def test_config3_penalised(use_mval):
    """Zipf histories with repetition + frequency + presence penalties (the
    row kernel; the penalised logits stay fp16).  use_mval=False derives m(c)
    from the counts in the kernel."""
    w = W.config3(seed=0, B=32)
    rp = w.rep_pen.numpy()
    hist = []
    for r, (t, c) in enumerate(w.history):
        if use_mval:
            mv = np.array([so.penalty_divisor(int(ci), float(rp[r]), "f16") for ci in c], np.float32)
            hist.append((t, c, mv))
        else:
            hist.append((t, c))
    args = dict(history=hist, rp=rp, f=w.freq_pen.numpy(), pi=w.pres_pen.numpy(), freq_pres=True)
    gpu = run_gpu(w.logits, w.temperature, w.top_k, w.top_p, w.uniforms, use_mval=use_mval, probs=True, **args)
    orc = run_oracle(w.logits, w.temperature, w.top_k, w.top_p, w.uniforms, **args)
    nb = compare(w.logits, w.temperature, w.top_k, w.top_p, w.uniforms, gpu, orc, probs=gpu[2], **args)
    assert nb <= 1


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("big_batch", [False, True])
def test_dense_top_p_rows(dtype, big_batch):
    """Rows without top-k whose nucleus is most of the row: nearly flat
    logits (what a random-init model gives) and C3's wide Gaussian at T = 0.8.
    The nucleus reaches below the candidates, so the threshold comes from the
    bracket passes (or, where the bracket is too wide, the radix passes)."""
    g = torch.Generator().manual_seed(13)
    B, V = 24, 151936
    x = torch.randn(B, V, generator=g) * 0.9
    x[12:] *= 2.5 / 0.9
    x = x.to(dtype)
    T = np.array([0.7, 1.3, 0.7, 0.5, 0.9, 0.6] * 2 + [0.8, 0.8, 1.0, 0.6, 0.8, 1.2] * 2, np.float32)
    K = np.zeros(B, np.int32)
    P = np.array([0.9, 0.9, 0.5, 0.99, 0.95, 0.3] * 2 + [0.95, 0.8, 0.999, 0.3, 0.9, 0.95] * 2, np.float32)
    U = row_uniforms(13, 0, B)
    gpu = run_gpu(x, T, K, P, U, probs=True, tile=tiled(B) if big_batch else 1)
    orc = run_oracle(x, T, K, P, U)
    nb = compare(x, T, K, P, U, gpu, orc, probs=gpu[2])
    # with ~1e5 entries in a flat nucleus the CDF steps are ~1e-5 apart, so
    # many rows have u or p within 1e-6 of a step; those rows still have their
    # kept sets and probabilities checked, only their ids are exempt
    assert nb <= B // 2


def test_config3_repetition_only():
    """C3's Zipf histories and parameters with the repetition penalty alone
    (the row kernel's path; a wide nucleus at T = 0.8, p = 0.95)."""
    w = W.config3(seed=0, B=32)
    rp = w.rep_pen.numpy()
    hist = [(t, c, np.array([so.penalty_divisor(int(ci), float(rp[r]), "f16") for ci in c], np.float32))
            for r, (t, c) in enumerate(w.history)]
    gpu = run_gpu(w.logits, w.temperature, w.top_k, w.top_p, w.uniforms, history=hist, rp=rp, probs=True)
    orc = run_oracle(w.logits, w.temperature, w.top_k, w.top_p, w.uniforms, history=hist, rp=rp)
    nb = compare(w.logits, w.temperature, w.top_k, w.top_p, w.uniforms, gpu, orc, history=hist, rp=rp,
                 probs=gpu[2])
    assert nb <= 1


def test_config1_fp32():
    w = W.config1(seed=0)
    gpu = run_gpu(w.logits, w.temperature, w.top_k, w.top_p, w.uniforms, probs=True)
    orc = run_oracle(w.logits, w.temperature, w.top_k, w.top_p, w.uniforms)
    compare(w.logits, w.temperature, w.top_k, w.top_p, w.uniforms, gpu, orc, probs=gpu[2])


@pytest.mark.parametrize("B", [16, 128])
def test_config4_bf16_subset(B):
    w = W.config4(seed=0, B=B)
    gpu = run_gpu(w.logits, w.temperature, w.top_k, w.top_p, w.uniforms, probs=True)
    orc = run_oracle(w.logits, w.temperature, w.top_k, w.top_p, w.uniforms)
    compare(w.logits, w.temperature, w.top_k, w.top_p, w.uniforms, gpu, orc, probs=gpu[2])


@pytest.mark.parametrize("V", [1, 2, 7, 33, 1000, 4097, 16385, 20481, 65537])
@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
@pytest.mark.parametrize("big_batch", [False, True])
def test_odd_vocab_sizes(V, dtype, big_batch):
    g = torch.Generator().manual_seed(V)
    B = 12
    x = (torch.randn(B, V, generator=g) * 2).to(dtype)
    T = np.array([1e-5, 0.5, 1.0, 2.0, 0.0, 1.0] * 2, np.float32)
    K = np.array([0, 1, 3, V, 5, V - 1, 2, V + 5, -1, 10, 1, 0], np.int32)
    P = np.array([1.0, 0.9, 0.5, 0.99, 1.0, 0.3, 1.0, 0.0, 0.7, 1e-6, 0.999999, 0.95], np.float32)
    U = row_uniforms(V, 0, B)
    gpu = run_gpu(x, T, K, P, U, probs=True, tile=tiled(B) if big_batch else 1)
    orc = run_oracle(x, T, K, P, U)
    compare(x, T, K, P, U, gpu, orc, probs=gpu[2])


@pytest.mark.parametrize("big_batch", [False, True])
def test_unaligned_rows_use_scalar_loads(big_batch):
    g = torch.Generator().manual_seed(5)
    B, V = 6, 3001
    x = (torch.randn(B, V, generator=g) * 3).half()
    T = np.ones(B, np.float32)
    K = np.array([0, 10, 100, 0, 1, 50], np.int32)
    P = np.array([0.9, 1.0, 0.8, 1.0, 1.0, 0.5], np.float32)
    U = row_uniforms(1, 1, B)
    gpu = run_gpu(x, T, K, P, U, row_stride=V + 3, tile=tiled(B) if big_batch else 1)
    orc = run_oracle(x, T, K, P, U)
    compare(x, T, K, P, U, gpu, orc)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("big_batch", [False, True])
def test_ties_and_flat_rows(dtype, big_batch):
    g = torch.Generator().manual_seed(9)
    B, V = 16, 30000
    x = torch.round(torch.randn(B, V, generator=g) * 4) / 2   # many exact ties
    x[0] = 0.0                                               # all equal
    x[1, :] = -float("inf")
    x[1, 123] = 1.0                                          # one finite logit
    x = x.to(dtype)
    T = np.array([1.0, 1.0, 1e-5, 0.7, 1.0, 3.0, 1.0, 0.5] * 2, np.float32)
    K = np.array([7, 0, 0, 5, 1, 40, 2, 100, 0, 3, 17, 0, 1000, 2, 9, 0], np.int32)
    P = np.array([1.0, 0.5, 1.0, 0.9, 1.0, 0.6, 0.95, 1.0, 0.5, 1.0, 0.25, 0.75, 0.9, 1.0, 0.3, 0.999], np.float32)
    U = row_uniforms(3, 0, B)
    gpu = run_gpu(x, T, K, P, U, probs=True, tile=tiled(B) if big_batch else 1)
    orc = run_oracle(x, T, K, P, U)
    nb = compare(x, T, K, P, U, gpu, orc, probs=gpu[2])
    assert nb <= 2


@pytest.mark.parametrize("big_batch", [False, True])
def test_rows_without_finite_mass(big_batch):
    """Sampled rows whose every logit is -inf have no finite z = y / T max
    and take the greedy rule: the lowest index of the max, 0.  (The
    reference's softmax would give NaN probabilities there; the oracle does
    not cover such rows.)  A row with a single finite logit draws it."""
    B, V = 6, 5000
    x = torch.full((B, V), -float("inf")).half()
    x[5, 17] = 2.0
    T = np.array([1.0, 0.7, 1.0, 2.0, 1.0, 1.0], np.float32)
    K = np.array([0, 0, 5, 0, 1, 0], np.int32)
    P = np.array([1.0, 0.9, 1.0, 0.5, 1.0, 0.9], np.float32)
    U = row_uniforms(8, 0, B)
    ids, _, _ = run_gpu(x, T, K, P, U, tile=tiled(B) if big_batch else 1)
    assert ids.tolist() == [0, 0, 0, 0, 0, 17]


def test_many_rows_small_vocab():
    g = torch.Generator().manual_seed(21)
    B, V = 2000, 300
    x = (torch.randn(B, V, generator=g) * 2).half()
    rng = np.random.default_rng(0)
    T = rng.uniform(0.3, 1.5, B).astype(np.float32)
    K = rng.integers(0, 60, B).astype(np.int32)
    P = rng.choice([1.0, 0.9, 0.6], B).astype(np.float32)
    U = row_uniforms(4, 0, B)
    gpu = run_gpu(x, T, K, P, U)
    orc = run_oracle(x, T, K, P, U)
    nb = compare(x, T, K, P, U, gpu, orc)
    assert nb <= 4


def test_philox_device_matches_cpu_twin_and_advances():
    dev = torch.device("cuda")
    st = S.new_philox_state(0xDEADBEEF12345, 77, dev)
    out = torch.empty(1000, dtype=torch.float32, device=dev)
    from ecahlang_b200._abi import lib
    assert lib().ecah_philox_uniforms(st.data_ptr(), 1000, out.data_ptr(), 1,
                                      torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    want = row_uniforms(0xDEADBEEF12345, 77, 1000)
    assert np.array_equal(out.cpu().numpy(), want)
    assert st.cpu().tolist() == [0xDEADBEEF12345, 78]


@pytest.mark.parametrize("B", [16, 128])
def test_sampler_philox_path_and_offset_bump(B):
    dev = torch.device("cuda")
    w = W.config2(seed=1, B=B, V=5000)
    smp = S.Sampler(B, 5000, torch.float16, dev, seed=1234)
    xd = w.logits.to(dev)
    T, K, P = w.temperature.to(dev), w.top_k.to(dev), w.top_p.to(dev)
    got = []
    for _ in range(3):
        got.append(smp(xd, T, K, P).clone())
    torch.cuda.synchronize()
    assert smp.philox_state.cpu().tolist() == [1234, 3]
    for off in range(3):
        U = row_uniforms(1234, off, B)
        ids = S.launch(xd, T, K, P, torch.empty(B, dtype=torch.int32, device=dev),
                       S.new_workspace(B, 5000, torch.float16, dev), uniforms=torch.from_numpy(U).to(dev))
        assert torch.equal(ids, got[off])


@pytest.mark.parametrize("B", [16, 128])
def test_cuda_graph_capture_and_replay(B):
    dev = torch.device("cuda")
    w = W.config2(seed=2, B=B, V=151936)
    smp = S.Sampler(B, w.vocab, torch.float16, dev, seed=99)
    xd = w.logits.to(dev)
    T, K, P = w.temperature.to(dev), w.top_k.to(dev), w.top_p.to(dev)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        smp(xd, T, K, P)      # warm-up (offset 0 -> 1)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = smp(xd, T, K, P)
    outs = []
    for _ in range(3):
        g.replay()
        outs.append(out.clone())
    torch.cuda.synchronize()
    assert smp.philox_state.cpu().tolist() == [99, 4]
    for i, o in enumerate(outs):
        U = torch.from_numpy(row_uniforms(99, 1 + i, B)).to(dev)
        ref = S.launch(xd, T, K, P, torch.empty(B, dtype=torch.int32, device=dev),
                       S.new_workspace(B, w.vocab, torch.float16, dev), uniforms=U)
        assert torch.equal(ref, o)
    del g


def test_custom_op_matches_launch():
    dev = torch.device("cuda")
    w = W.config2(seed=3, B=16, V=20000)
    xd = w.logits.to(dev)
    T, K, P, U = (t.to(dev) for t in (w.temperature, w.top_k, w.top_p, w.uniforms))
    out = torch.empty(16, dtype=torch.int32, device=dev)
    ws = S.new_workspace(16, 20000, torch.float16, dev)
    torch.ops.ecah.sample(xd, T, K, P, U, None, None, None, None, None, None, None, None, None, 0, 0, out, ws)
    ref = S.launch(xd, T, K, P, torch.empty_like(out), ws, uniforms=U)
    assert torch.equal(out, ref)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_penalty_rule_matches_torch_cuda_divide(dtype):
    """The oracle's per-update rule against the reference's update statement
    run by torch on the GPU, over many rp values and up to 60 repeats."""
    dev = torch.device("cuda")
    rps = [1.01, 1.05, 1.1, 1.17, 1.2, 1.3, 1.5, 1.7, 2.0, 3.3, 0.5, 0.8, 0.9, 0.95, 0.99, 1.0]
    mask = torch.ones(len(rps), dtype=dtype, device=dev)
    dts = {torch.float16: "f16", torch.bfloat16: "bf16", torch.float32: "f32"}[dtype]
    for c in range(1, 61):
        for i, rp in enumerate(rps):
            if rp > 1:
                mask[i] /= rp
            else:
                mask[i] *= rp
        got = mask.float().cpu().numpy()
        for i, rp in enumerate(rps):
            assert got[i] == so.penalty_divisor(c, rp, dts), (dts, rp, c, got[i])


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_hist_update_matches_reference_rule(dtype):
    """Device-side history update vs the oracle's iterated mask rule, and that
    rule vs torch's own CUDA in-place divide (the reference's update statement,
    ecahlang/main.py:691-694, run on the GPU)."""
    dev = torch.device("cuda")
    S_, cap = 4, 64
    pen = S.PenaltyState(S_, cap, dtype, dev)
    rng = np.random.default_rng(1)
    rps = [1.1, 1.3, 0.9, 2.0]
    seq = rng.integers(0, 20, (30, S_))
    row_slot = torch.arange(S_, dtype=torch.int32, device=dev)
    rp_t = torch.from_numpy(S.repetition_factor(rps)).to(dev)
    mask = torch.ones(S_, 32, dtype=dtype, device=dev)
    for step in range(seq.shape[0]):
        ids = torch.from_numpy(seq[step].astype(np.int32)).to(dev)
        pen.update(ids, row_slot, rp_t)
        for s in range(S_):
            t = int(seq[step, s])
            if rps[s] > 1:
                mask[s, t] /= rps[s]
            else:
                mask[s, t] *= rps[s]
    torch.cuda.synchronize()
    dts = {torch.float16: "f16", torch.bfloat16: "bf16", torch.float32: "f32"}[dtype]
    for s in range(S_):
        n = int(pen.slot_len[s])
        toks = pen.tok[s, :n].cpu().numpy()
        cnts = pen.cnt[s, :n].cpu().numpy()
        mv = pen.mval[s, :n].cpu().numpy()
        u, c = np.unique(seq[:, s], return_counts=True)
        assert sorted(toks.tolist()) == u.tolist()
        assert dict(zip(toks.tolist(), cnts.tolist())) == dict(zip(u.tolist(), c.tolist()))
        for t, cnt, m in zip(toks, cnts, mv):
            assert m == so.penalty_divisor(int(cnt), rps[s], dts)
            assert m == mask[s, t].float().item(), (s, t, cnt, m, mask[s, t].item())


def test_chi_square_one_million_draws():
    """1e6 draws of one distribution (Philox offsets 0..999 x 1000 rows)
    against the oracle's post-filter probabilities."""
    dev = torch.device("cuda")
    V, B, steps = 256, 1000, 1000
    g = torch.Generator().manual_seed(77)
    row = (torch.randn(V, generator=g) * 1.5).half()
    x = row.repeat(B, 1).to(dev)
    T = torch.full((B,), 0.8, device=dev)
    K = torch.full((B,), 120, dtype=torch.int32, device=dev)
    P = torch.full((B,), 0.9, device=dev)
    smp = S.Sampler(B, V, torch.float16, dev, seed=5)
    counts = torch.zeros(V, dtype=torch.int64, device=dev)
    for _ in range(steps):
        ids = smp(x, T, K, P)
        counts += torch.bincount(ids.long(), minlength=V)
    res = so.sample_row(row.float().numpy(), dtype="f16", temperature=0.8, top_k=120, top_p=0.9)
    c = counts.cpu().numpy()
    keep = res.probs > 0
    assert c[~keep].sum() == 0
    exp = res.probs[keep] * B * steps
    chi2 = float(((c[keep] - exp) ** 2 / exp).sum())
    dof = int(keep.sum()) - 1
    assert chi2 < dof + 6 * np.sqrt(2 * dof), (chi2, dof)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("B", [7, 64])
def test_row_index_gathers_rows(dtype, B):
    """The prefill gather (ecahlang/main.py:476, logits[0, append_indptr[1:]-1]):
    sampling rows row_index[r] of a larger buffer in place gives the same ids,
    thresholds and masses as sampling the gathered copy, and matches the
    oracle on those rows; indices past the buffer are clamped, not read."""
    g = torch.Generator().manual_seed(11 + B)
    L, V = 150, 32000
    dev = torch.device("cuda")
    x = (torch.randn(L, V, generator=g) * 3).to(dtype)
    idx = torch.randint(0, L, (B,), generator=g, dtype=torch.int32)
    idx[0], idx[-1] = L - 1, 0
    T = torch.tensor(np.resize([0.0, 0.7, 1.0, 1.3], B), dtype=torch.float32)
    K = torch.tensor(np.resize([0, 40, L + V, 5], B), dtype=torch.int32)
    P = torch.tensor(np.resize([1.0, 0.9, 0.8, 1.0], B), dtype=torch.float32)
    U = torch.as_tensor(row_uniforms(3, 1, B))

    def run(logits, row_index=None):
        out = torch.empty(B, dtype=torch.int32, device=dev)
        stats = torch.zeros(B, 4, dtype=torch.float32, device=dev)
        ws = S.new_workspace(B, V, dtype, dev)
        S.launch(logits, T.to(dev), K.to(dev), P.to(dev), out, ws, uniforms=U.to(dev),
                 row_stats=stats, row_index=row_index)
        torch.cuda.synchronize()
        return out.cpu().numpy(), stats.cpu().numpy()

    xd = x.to(dev)
    got, st = run(xd, idx.to(dev))
    want, sw = run(x[idx.long()].contiguous().to(dev))
    assert np.array_equal(got, want)
    assert np.array_equal(st, sw)
    xr = x[idx.long()]
    orc = run_oracle(xr, T.numpy(), K.numpy(), P.numpy(), U.numpy())
    compare(xr, T.numpy(), K.numpy(), P.numpy(), U.numpy(), (got, st, None), orc)
    # out-of-range indices are clamped into [0, L)
    bad = idx.clone()
    bad[1], bad[2] = -5, L + 9
    clamped = bad.clamp(0, L - 1)
    g1, _ = run(xd, bad.to(dev))
    g2, _ = run(xd, clamped.to(dev))
    assert np.array_equal(g1, g2)
