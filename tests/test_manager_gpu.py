"""Decode steps through the sampling manager on the GPU: parameters through
the pinned buffers, penalties from the requests' slot histories, the
batched history update after each step; every step's ids must equal the CPU
oracle given the same histories (the reference's dense mask semantics)."""
from collections import Counter

import numpy as np
import pytest
import torch

from ecahlang_b200.manager import SamplingManager
from gpu_util import BOUNDARY
from oracle import sampler_oracle as so

pytestmark = pytest.mark.gpu

V = 5000
RP = [1.1, 1.3, 0.9, 1.0]
T = [0.7, 1.0, 1e-5, 1.2]
K = [50, V, 20, V]
P = [0.9, 1.0, 0.8, 1.0]


@pytest.mark.parametrize("bucket", [None, 8])
def test_manager_decode_steps_match_oracle(bucket):
    dev = torch.device("cuda")
    n = 4
    m = SamplingManager(V, seq_lens=16, dtype=torch.float16, device=dev, history_capacity=64, seed=1)
    m.init_sampling_buffers(8)
    if bucket:
        m.init_cuda_graph_buffers([bucket])
    ids_req = ["r0", "r1", "r2", "r3"]
    for r in ids_req:
        m.allocate(r)
    hist = [Counter() for _ in range(n)]
    rng = np.random.default_rng(0)
    boundary = 0
    for step in range(6):
        B = bucket or n
        x = (rng.normal(0, 2.0, (B, V))).astype(np.float16)
        x[:, :40] += 3.0                                  # a band of likely tokens: repeats happen
        U = rng.random(B).astype(np.float32)
        if bucket:
            m.fill_cuda_graph_sampling_params(bucket, n, T, K, P, rep_pens=RP, batch_ids=ids_req)
        else:
            m.fill_sampling_params(n, T, K, P, rep_pens=RP, batch_ids=ids_req)
        got = m.sample(torch.from_numpy(x).to(dev), bucket_size=bucket, uniforms=torch.from_numpy(U).to(dev))
        got = got[:n].clone()
        m.update_penalties(got if not bucket else torch.cat([got, torch.zeros(bucket - n, dtype=torch.int32, device=dev)]),
                           bucket_size=bucket)
        got = got.cpu().numpy()
        history = [(np.array(sorted(h), np.int32), np.array([h[t] for t in sorted(h)], np.int32)) for h in hist]
        res = so.sample_batch(x[:n].astype(np.float32), dtype="f16", temperature=np.array(T, np.float32),
                              top_k=np.array(K, np.int32), top_p=np.array(P, np.float32), uniforms=U[:n],
                              history=history, rep_pen=np.array(RP), keep_arrays=False)
        for r in range(n):
            rr = res.rows[r]
            if rr.u_margin < BOUNDARY or rr.p_margin < BOUNDARY:
                boundary += 1
            else:
                assert got[r] == rr.token, f"step {step} row {r}: {got[r]} != oracle {rr.token}"
            hist[r][int(got[r])] += 1
    assert boundary <= 1
    # the slot histories hold exactly the sampled tokens and counts
    for r, name in enumerate(ids_req):
        s = m.batch_to_seq_len[name]
        L = int(m.penalty.slot_len[s])
        toks = m.penalty.tok[s, :L].cpu().tolist()
        cnts = m.penalty.cnt[s, :L].cpu().tolist()
        assert dict(zip(toks, cnts)) == dict(hist[r])


def test_manager_prefill_row_index():
    """SamplingManager.sample over the prefill's [tokens, V] logits with the
    last token of each request (append_indptr[1:] - 1, ecahlang/main.py:476):
    host indices are range-checked and give the ids of the gathered rows."""
    from ecahlang_b200.manager import SamplingManager
    dev = torch.device("cuda")
    V, n = 32000, 5
    g = torch.Generator().manual_seed(4)
    lens = [3, 1, 7, 2, 5]
    indptr = np.concatenate([[0], np.cumsum(lens)])
    tokens = (torch.randn(int(indptr[-1]), V, generator=g) * 3).half().to(dev)
    last = indptr[1:] - 1
    mgr = SamplingManager(V, seq_lens=8, dtype=torch.float16, device=dev, seed=3)
    mgr.init_sampling_buffers(8)
    mgr.fill_sampling_params(n, [0.7, 1.0, 0.0, 1.2, 0.9], [50, 0, 0, 20, 0], [0.9, 0.95, 1.0, 1.0, 0.8])
    u = torch.rand(n, generator=g).to(dev)
    ids = mgr.sample(tokens, row_index=last.tolist(), uniforms=u).cpu().numpy()
    ref = mgr.sample(tokens[torch.as_tensor(last, device=dev)].contiguous(), uniforms=u).cpu().numpy()
    assert np.array_equal(ids, ref)
    with pytest.raises(IndexError):
        mgr.sample(tokens, row_index=[0, int(indptr[-1])], uniforms=u[:2])


def test_sample_async_hands_ids_to_host():
    """sample_async: the ids of several pending steps reach pinned host
    memory behind per-step events and equal the synchronous sample's."""
    dev = torch.device("cuda")
    n, Vs = 6, 20000
    m = SamplingManager(Vs, seq_lens=8, dtype=torch.float16, device=dev, seed=5)
    m.init_sampling_buffers(8)
    m.fill_sampling_params(n, [0.8] * n, [40, 0, 10, 0, 5, 0], [0.9, 0.95, 1.0, 0.8, 1.0, 1.0])
    g = torch.Generator().manual_seed(9)
    xs = [(torch.randn(n, Vs, generator=g) * 3).half().to(dev) for _ in range(6)]
    us = [torch.rand(n, generator=g).to(dev) for _ in range(6)]
    pend = [m.sample_async(x, uniforms=u) for x, u in zip(xs, us)]   # more steps than ring slots
    got = [p.wait() for p in pend]
    assert all(p.ready() for p in pend)
    for x, u, gi in zip(xs, us, got):
        assert np.array_equal(gi, m.sample(x, uniforms=u).cpu().numpy())


@pytest.mark.parametrize("bucket", [8])
def test_decode_graph_with_sampler_and_penalty_update(bucket):
    """In-graph decode integration: one CUDA graph holds the LM head (fp16
    GEMM, as decode_forward's last layer, ecahlang/main.py:159-171), the
    sampler (Philox uniforms advanced on the device) and the penalty-history
    update (main.py:691-694).  Each replay's ids equal the oracle's on the
    logits the graph computed, with the histories the earlier replays built."""
    from oracle.philox import row_uniforms
    dev = torch.device("cuda")
    n, H, Vd = 5, 256, 6000
    g = torch.Generator().manual_seed(21)
    W = (torch.randn(Vd, H, generator=g) * 0.2).half().to(dev)
    W[:30] *= 1.5                                          # a band of likely tokens: repeats happen
    hidden = torch.zeros(bucket, H, dtype=torch.float16, device=dev)
    logits = torch.zeros(bucket, Vd, dtype=torch.float16, device=dev)
    m = SamplingManager(Vd, seq_lens=16, dtype=torch.float16, device=dev, history_capacity=64, seed=77)
    m.init_sampling_buffers(bucket)
    m.init_cuda_graph_buffers([bucket])
    names = [f"q{i}" for i in range(n)]
    for r in names:
        m.allocate(r)
    Tn, Kn, Pn, Rn = [0.8, 1.0, 0.6, 1.1, 0.9], [40, Vd, 15, Vd, 100], [0.9, 0.95, 1.0, 0.85, 1.0], [1.2, 1.1, 1.3, 1.0, 1.05]
    m.fill_cuda_graph_sampling_params(bucket, n, Tn, Kn, Pn, rep_pens=Rn, batch_ids=names)
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):                             # warm-up outside the graph
        torch.matmul(hidden, W.t(), out=logits)
        m.sample(logits, bucket_size=bucket)               # the sampler's workspace, allocated once
    torch.cuda.current_stream(dev).wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        torch.matmul(hidden, W.t(), out=logits)
        ids = m.sample(logits, bucket_size=bucket)
        m.update_penalties(ids, bucket_size=bucket)
    torch.cuda.synchronize()
    # the offset every replay starts from (the capture itself launches nothing)
    seed, off0 = [int(v) for v in m.philox_state.cpu().tolist()]
    hist = [Counter() for _ in range(n)]
    boundary = 0
    for step in range(5):
        hidden.copy_((torch.randn(bucket, H, generator=g) * 1.0).half())
        m.fill_cuda_graph_sampling_params(bucket, n, Tn, Kn, Pn, rep_pens=Rn, batch_ids=names)
        graph.replay()
        torch.cuda.synchronize()
        got = ids[:n].cpu().numpy()
        x = logits[:n].float().cpu().numpy()
        U = row_uniforms(seed, off0 + step, bucket)[:n]
        history = [(np.array(sorted(h), np.int32), np.array([h[t] for t in sorted(h)], np.int32)) for h in hist]
        res = so.sample_batch(x, dtype="f16", temperature=np.array(Tn, np.float32), top_k=np.array(Kn, np.int32),
                              top_p=np.array(Pn, np.float32), uniforms=U, history=history,
                              rep_pen=np.array(Rn), keep_arrays=False)
        for r in range(n):
            rr = res.rows[r]
            if rr.u_margin < BOUNDARY or rr.p_margin < BOUNDARY:
                boundary += 1
            else:
                assert got[r] == rr.token, f"replay {step} row {r}: {got[r]} != oracle {rr.token}"
            hist[r][int(got[r])] += 1
    assert boundary <= 1
    assert int(m.philox_state[1].item()) == off0 + 5
    for r, name in enumerate(names):
        sl = m.batch_to_seq_len[name]
        L = int(m.penalty.slot_len[sl])
        assert dict(zip(m.penalty.tok[sl, :L].cpu().tolist(), m.penalty.cnt[sl, :L].cpu().tolist())) == dict(hist[r])
    del graph
