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
