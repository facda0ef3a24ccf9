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

from ecahlang_b200 import sampler as S
from ecahlang_b200 import workloads as W
from ecahlang_b200.vocab_parallel import VocabParallelSampler, split_vocab
from gpu_util import BOUNDARY
from oracle import sampler_oracle as so
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


def _keys16(xb: torch.Tensor) -> np.ndarray:
    """Order-preserving 16-bit keys of bf16 values (sign-flipped raw bits)."""
    r = xb.view(torch.int16).numpy().astype(np.int64) & 0xFFFF
    return np.where(r & 0x8000, r ^ 0xFFFF, r ^ 0x8000)


@pytest.mark.parametrize("V,world,cap,view", [(151936, 2, 1024, False), (20011, 4, 512, True),
                                              (4000, 8, 256, True), (70000, 2, 1024, True)])
def test_vp_local_lists_match_restatement(V, world, cap, view):
    """ecah_vp_local against a numpy restatement of its contract, per rank:
    slices wider than one round and up to 75968 columns, odd offsets (unaligned
    rows through a strided view), repetition-penalty histories whose ids fall
    in other ranks' slices, k from 1 to cand_cap (the candidate path and its
    radix fallback) and k above cand_cap (count = k, no list)."""
    dev = torch.device("cuda")
    B = 40
    x, T, K, P, U = vp_case(23, B, V)
    T[:12] = 1.0
    K[:12] = [1, 5, 64, 200, cap // 2, cap, cap + 1, 0, V, 3, 64, 128]
    # penalty histories: ids over the whole vocabulary; row 1 has 1100 ids
    # below 3000, more than the shared-memory buckets hold for one slice
    rng = np.random.default_rng(5)
    cap_h = 1200
    pen = S.PenaltyState(B, cap_h, torch.bfloat16, dev)
    toks = [rng.choice(min(V, 3000), 1100, replace=False) if r == 1 else
            rng.choice(V, int(rng.integers(0, 300)), replace=False) for r in range(B)]
    xp = np.empty_like(x)
    for r in range(B):
        n = len(toks[r])
        cnt = rng.integers(1, 4, n)
        mv = np.array([so.penalty_divisor(int(c), 1.3, "bf16") for c in cnt], np.float32)
        pen.slot_len[r] = n
        pen.tok[r, :n] = torch.from_numpy(toks[r].astype(np.int32))
        pen.cnt[r, :n] = torch.from_numpy(cnt.astype(np.int32))
        pen.mval[r, :n] = torch.from_numpy(mv)
        xp[r] = so.penalised_logits(so.round_to(x[r], "bf16"), "bf16", toks[r], cnt, mv)
    row_slot = torch.arange(B, dtype=torch.int32, device=dev)
    xb = torch.from_numpy(x).to(torch.bfloat16)
    xd = xb.to(dev)
    keys_full = _keys16(torch.from_numpy(xp).to(torch.bfloat16))
    Td, Kd, Pd = (torch.from_numpy(a).to(dev) for a in (T, K, P))
    for g in range(world):
        off, loc = split_vocab(V, world, g)
        sl = xd[:, off:off + loc]
        if not view:
            sl = sl.contiguous()
        smp = VocabParallelSampler(B, V, world, g, torch.bfloat16, dev, seed=5, cand_cap=cap, exchange=lambda *a: None)
        c, n = smp.local(sl, Td, Kd, Pd, penalty=pen, row_slot=row_slot)
        c, n = c.cpu().numpy(), n.cpu().numpy()
        for r in range(B):
            k = 1 if not T[r] > 0 else (loc if (K[r] <= 0 or K[r] >= V) else min(int(K[r]), loc))
            if k > cap:
                assert n[r] == k, (g, r, n[r], k)
                continue
            # the contract compares keys: -0.0 sorts below +0.0
            keys = keys_full[r, off:off + loc]
            sel = np.nonzero(keys >= np.sort(keys)[::-1][k - 1])[0]
            assert n[r] == len(sel), (g, r, n[r], len(sel), k)
            m = min(len(sel), cap)
            got_ids = (c[r, :m] & 0xFFFFFFFF).astype(np.int64)
            assert np.array_equal(got_ids, off + sel[:m]), (g, r, k)
            assert np.array_equal(c[r, :m] >> 32, keys_full[r, got_ids]), (g, r, k)


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
