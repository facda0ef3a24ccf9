"""Vocab-parallel kernels on the GPU.  With one GPU the ranks are emulated:
every rank's slice goes through ecah_vp_local, the lists are stacked in rank
order as the all-gather would, and ecah_vp_merge runs once per rank; every
rank must return the same ids, equal to the CPU oracle on the full rows.
With two GPUs the same runs as two NCCL ranks."""
import os
import socket

import numpy as np
import pytest
import torch

from ecahlang_b200 import workloads as W
from ecahlang_b200.vocab_parallel import VocabParallelSampler, split_vocab
from gpu_util import BOUNDARY
from vp_util import oracle_ids, vp_case

pytestmark = pytest.mark.gpu


def _emulated(x_dev, T, K, P, U, world, cap, dtype):
    B, V = x_dev.shape
    dev = x_dev.device
    smps = [VocabParallelSampler(B, V, world, g, dtype, dev, seed=5, cand_cap=cap, exchange=lambda *a: None)
            for g in range(world)]
    lists = []
    for g, smp in enumerate(smps):
        off, loc = split_vocab(V, world, g)
        c, n = smp.local(x_dev[:, off:off + loc].contiguous(), T, K, P)
        lists.append((c.clone(), n.clone()))
    all_cand = torch.stack([c for c, _ in lists]).contiguous()
    all_count = torch.stack([n for _, n in lists]).contiguous()
    outs = [smp.merge(all_cand, all_count, T, K, P, uniforms=U).clone() for smp in smps]
    torch.cuda.synchronize()
    for o in outs[1:]:
        assert torch.equal(o, outs[0]), "ranks disagree"
    return outs[0].cpu().numpy(), all_count.cpu().numpy()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_vp_mixed_rows_match_oracle(world):
    dev = torch.device("cuda")
    B, V = 64, 20000
    x, T, K, P, U = vp_case(11, B, V)
    xd = torch.from_numpy(x).to(torch.bfloat16).to(dev)
    Td, Kd, Pd, Ud = (torch.from_numpy(a).to(dev) for a in (T, K, P, U))
    got, counts = _emulated(xd, Td, Kd, Pd, Ud, world, 2048 // world, torch.bfloat16)
    want, res = oracle_ids(x, T, K, P, U)
    near = np.array([rr.u_margin < BOUNDARY or rr.p_margin < BOUNDARY for rr in res.rows])
    assert (got >= 0).all()
    assert np.array_equal(got[~near], want[~near])
    assert near.sum() <= 2


@pytest.mark.parametrize("world", [2, 8])
def test_vp_config4_rows_match_oracle(world):
    dev = torch.device("cuda")
    w = W.config4(seed=0, B=48)
    xd = w.logits.to(dev)
    Td, Kd, Pd, Ud = (t.to(dev) for t in (w.temperature, w.top_k, w.top_p, w.uniforms))
    got, _ = _emulated(xd, Td, Kd, Pd, Ud, world, 2048 // world, torch.bfloat16)
    x = w.logits.float().numpy()
    want, res = oracle_ids(x, w.temperature.numpy(), w.top_k.numpy(), w.top_p.numpy(), w.uniforms.numpy())
    near = np.array([rr.u_margin < BOUNDARY or rr.p_margin < BOUNDARY for rr in res.rows])
    assert np.array_equal(got[~near], want[~near])


def test_vp_rows_without_top_k_are_refused():
    dev = torch.device("cuda")
    B, V = 8, 4000
    x, T, K, P, U = vp_case(2, B, V)
    K[:] = 0                                      # top-k off: the lists cannot hold the row
    T[:] = 1.0
    xd = torch.from_numpy(x).to(torch.bfloat16).to(dev)
    Td, Kd, Pd, Ud = (torch.from_numpy(a).to(dev) for a in (T, K, P, U))
    got, _ = _emulated(xd, Td, Kd, Pd, Ud, 2, 64, torch.bfloat16)
    assert (got == -1).all()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_rank(rank, world, port, outdir):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        dev = torch.device("cuda", rank)
        B, V = 32, 20000
        x, T, K, P, U = vp_case(17, B, V)
        off, loc = split_vocab(V, world, rank)
        xd = torch.from_numpy(x[:, off:off + loc]).to(torch.bfloat16).to(dev).contiguous()
        smp = VocabParallelSampler(B, V, world, rank, torch.bfloat16, dev, seed=5, cand_cap=2048 // world)
        Td, Kd, Pd, Ud = (torch.from_numpy(a).to(dev) for a in (T, K, P, U))
        ids = smp(xd, Td, Kd, Pd, uniforms=Ud)
        np.save(os.path.join(outdir, f"nccl{rank}.npy"), ids.cpu().numpy())
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_vp_two_nccl_ranks(tmp_path):
    import torch.multiprocessing as mp
    mp.spawn(_nccl_rank, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    x, T, K, P, U = vp_case(17, 32, 20000)
    want, res = oracle_ids(x, T, K, P, U)
    near = np.array([rr.u_margin < BOUNDARY or rr.p_margin < BOUNDARY for rr in res.rows])
    a, b = np.load(tmp_path / "nccl0.npy"), np.load(tmp_path / "nccl1.npy")
    assert np.array_equal(a, b)
    assert np.array_equal(a[~near], want[~near])
