"""The torch-CPU port used for timing agrees with the numpy oracle."""
import numpy as np
import torch

from ecahlang_b200 import workloads as W
from oracle import sampler_oracle as so
from oracle.torch_port import sample_batch_torch


def _check(w, rows=None, max_boundary=1):
    sl = slice(None) if rows is None else slice(0, rows)
    x, T, K, P, U = w.logits[sl], w.temperature[sl], w.top_k[sl], w.top_p[sl], w.uniforms[sl]
    got = sample_batch_torch(x, T, K, P, U).numpy()
    orc = so.sample_batch(x.float().numpy(), dtype={torch.float16: "f16", torch.bfloat16: "bf16",
                                                    torch.float32: "f32"}[x.dtype],
                          temperature=T.numpy(), top_k=K.numpy(), top_p=P.numpy(),
                          uniforms=U.numpy())
    bad = [r for r in range(len(got)) if got[r] != orc.tokens[r]
           and not (orc.rows[r].u_margin < 1e-5 or orc.rows[r].p_margin < 1e-5)]
    assert not bad, bad


def test_port_matches_oracle_c2_subset():
    w = W.config2(seed=0, B=32, V=20000)
    _check(w)


def test_port_matches_oracle_c1():
    _check(W.config1(seed=0, B=4, V=30000))
