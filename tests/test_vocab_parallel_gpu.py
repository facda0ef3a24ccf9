"""Vocab-parallel kernels on the GPU.  With one GPU the ranks are emulated:
every rank's slice goes through ecah_vp_local, the lists are stacked in rank
order as the all-gather would, and ecah_vp_merge runs once per rank; every
rank must return the same ids, equal to the CPU oracle on the full rows.
With two GPUs the same runs as two NCCL ranks."""
import ctypes
import os
import socket

import numpy as np
import pytest
import torch

from ecahlang_b200 import _abi
from ecahlang_b200 import sampler as S
from ecahlang_b200 import workloads as W
from ecahlang_b200.vocab_parallel import VocabParallelError, VocabParallelSampler, split_vocab
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
    """The candidate path alone refuses rows without top-k (their kept set
    exceeds any list); the distributed passes serve them
    (test_vp_full_rows_gpu.py)."""
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
        # rows without top-k: the distributed passes over NCCL
        K2 = K.copy()
        K2[0::3] = 0
        ids = smp(xd, Td, torch.from_numpy(K2).to(dev), Pd, uniforms=Ud)
        np.save(os.path.join(outdir, f"full{rank}.npy"), ids.cpu().numpy())
        dist.barrier()
    finally:
        dist.destroy_process_group()


class _Raw:
    """__cuda_array_interface__ over n words of a raw device address."""

    def __init__(self, ptr, n, typestr):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


def _al(x):
    return (x + 255) & ~255


def test_vp_step_wait_runs_out_and_reports():
    """The fused step on one GPU with world = 2 and no second rank: the
    stand-in for rank 1's buffer is never flagged, so every wait runs out
    after timeout_us.  The step returns -1 for every row, sets the error word
    and still advances the epoch; the rows' lists and counts sit in rank 0's
    slot of both buffers, as ecah_vp_local writes them, with the rows' flags
    at epoch 1.  A second step finds the error word set and waits no more."""
    dev = torch.device("cuda")
    B, V, world, cap = 8, 4000, 2, 64
    x, T, K, P, U = vp_case(31, B, V)
    T[:] = 1.0
    K[:] = [1, 5, 20, 64, 65, 0, 3, 10]          # rows 4 and 5: k > cap, count only
    off, loc = split_vocab(V, world, 0)
    xd = torch.from_numpy(x[:, off:off + loc]).to(torch.bfloat16).to(dev).contiguous()
    Td, Kd, Pd, Ud = (torch.from_numpy(a).to(dev) for a in (T, K, P, U))
    smp = VocabParallelSampler(B, V, world, 0, torch.bfloat16, dev, seed=5, cand_cap=cap,
                               exchange=lambda *a: None)
    c_ref, n_ref = (t.clone() for t in smp.local(xd, Td, Kd, Pd))
    L = _abi.lib()
    nbytes = L.ecah_vp_exchange_bytes(B, world, cap)
    bufs = []
    for _ in range(2):
        p = ctypes.c_void_p()
        _abi.check(L.ecah_vp_ipc_alloc(nbytes, ctypes.byref(p), (ctypes.c_ubyte * 64)()), "alloc")
        bufs.append(p.value)
    try:
        base = torch.tensor(bufs, dtype=torch.int64, device=dev)
        peers = _abi.VPPeers(0, B, base.data_ptr(), 20000)
        stream = torch.cuda.current_stream(dev).cuda_stream
        a = smp._args(xd, Td, Kd, Pd, Ud, None, None, None, None)
        _abi.check(L.ecah_vp_step(ctypes.byref(a), ctypes.byref(peers), stream), "ecah_vp_step")
        torch.cuda.synchronize()
        assert (smp.out[:B].cpu() == -1).all()
        hdr = torch.as_tensor(_Raw(bufs[0], 64, "<i4"), device=dev).cpu()
        assert hdr[0] == 1 and hdr[1] == 0 and hdr[2] == 1       # epoch, finished rows, error
        lflag = 256
        lcount = lflag + _al(4 * world * B)
        lcand = lcount + _al(4 * 2 * world * B)
        for buf in bufs:
            flags = torch.as_tensor(_Raw(buf + lflag, world * B, "<i4"), device=dev).cpu().view(world, B)
            assert (flags[0] == 1).all() and (flags[1] == 0).all()
            cnt = torch.as_tensor(_Raw(buf + lcount, 2 * world * B, "<i4"), device=dev).cpu().view(2, world, B)
            lists = torch.as_tensor(_Raw(buf + lcand, 2 * world * B * cap, "<i8"), device=dev).cpu()
            lists = lists.view(2, world, B, cap)
            assert torch.equal(cnt[1, 0], n_ref.cpu())                # epoch 1: parity 1, rank 0's slot
            for r in range(B):
                m = min(int(n_ref[r]), cap) if n_ref[r] <= cap else 0
                assert torch.equal(lists[1, 0, r, :m], c_ref[r, :m].cpu()), r
        _abi.check(L.ecah_vp_step(ctypes.byref(a), ctypes.byref(peers), stream), "ecah_vp_step")
        torch.cuda.synchronize()
        assert (smp.out[:B].cpu() == -1).all()
        hdr = torch.as_tensor(_Raw(bufs[0], 64, "<i4"), device=dev).cpu()
        assert hdr[0] == 2 and hdr[2] == 1
    finally:
        torch.cuda.synchronize()
        for p in bufs:
            _abi.check(L.ecah_vp_ipc_free(p), "free")


def test_vp_step_reset_then_resume():
    """After a step whose waits ran out (sticky error word, every row -1),
    ecah_vp_reset clears the error and sets the step counter; with the
    stand-in rank 1 now flagging the next step (empty lists), the step
    completes and draws exactly what ecah_vp_merge draws from rank 0's lists
    and an empty rank 1."""
    dev = torch.device("cuda")
    B, V, world, cap = 8, 4000, 2, 64
    x, T, K, P, U = vp_case(37, B, V)
    T[:] = 1.0
    K[:] = [1, 5, 20, 64, 65, 0, 3, 10]          # rows 4 and 5: refused (k > cap, no top-k)
    off, loc = split_vocab(V, world, 0)
    xd = torch.from_numpy(x[:, off:off + loc]).to(torch.bfloat16).to(dev).contiguous()
    Td, Kd, Pd, Ud = (torch.from_numpy(a).to(dev) for a in (T, K, P, U))
    smp = VocabParallelSampler(B, V, world, 0, torch.bfloat16, dev, seed=5, cand_cap=cap,
                               exchange=lambda *a: None)
    c_ref, n_ref = (t.clone() for t in smp.local(xd, Td, Kd, Pd))
    L = _abi.lib()
    nbytes = L.ecah_vp_exchange_bytes(B, world, cap)
    bufs = []
    for _ in range(2):
        p = ctypes.c_void_p()
        _abi.check(L.ecah_vp_ipc_alloc(nbytes, ctypes.byref(p), (ctypes.c_ubyte * 64)()), "alloc")
        bufs.append(p.value)
    lflag = 256
    lcount = lflag + _al(4 * world * B)
    try:
        base = torch.tensor(bufs, dtype=torch.int64, device=dev)
        peers = _abi.VPPeers(0, B, base.data_ptr(), 20000)
        stream = torch.cuda.current_stream(dev).cuda_stream
        a = smp._args(xd, Td, Kd, Pd, Ud, None, None, None, None)
        _abi.check(L.ecah_vp_step(ctypes.byref(a), ctypes.byref(peers), stream), "ecah_vp_step")
        torch.cuda.synchronize()
        assert (smp.out[:B].cpu() == -1).all()
        with pytest.raises(VocabParallelError):
            smp.raise_on_failed(smp.out[:B])
        hdr = torch.as_tensor(_Raw(bufs[0], 3, "<i4"), device=dev)
        assert hdr.cpu().tolist() == [1, 0, 1]
        _abi.check(L.ecah_vp_reset(bufs[0], 1, stream), "ecah_vp_reset")
        torch.cuda.synchronize()
        assert hdr.cpu().tolist() == [1, 0, 0]
        # the stand-in rank 1 flags step 2 (parity 0) with empty lists
        flags = torch.as_tensor(_Raw(bufs[0] + lflag, world * B, "<i4"), device=dev).view(world, B)
        cnt = torch.as_tensor(_Raw(bufs[0] + lcount, 2 * world * B, "<i4"), device=dev).view(2, world, B)
        cnt[0, 1].zero_()
        flags[1].fill_(2)
        torch.cuda.synchronize()
        _abi.check(L.ecah_vp_step(ctypes.byref(a), ctypes.byref(peers), stream), "ecah_vp_step")
        torch.cuda.synchronize()
        got = smp.out[:B].cpu().clone()
        assert hdr.cpu().tolist() == [2, 0, 0]
        all_cand = torch.zeros(world, B, cap, dtype=torch.int64, device=dev)
        all_count = torch.zeros(world, B, dtype=torch.int32, device=dev)
        all_cand[0] = c_ref
        all_count[0] = n_ref
        want = smp.merge(all_cand, all_count, Td, Kd, Pd, uniforms=Ud).cpu()
        assert torch.equal(got, want)
        assert (got[[4, 5]] == -1).all() and int((got >= 0).sum()) >= 4   # the step resumed
    finally:
        torch.cuda.synchronize()
        for p in bufs:
            _abi.check(L.ecah_vp_ipc_free(p), "free")


def _peer_rank(rank, world, port, outdir):
    """One rank of the fused step over NVLink peer memory; gloo carries only
    the IPC handles."""
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        dev = torch.device("cuda", rank)
        B, V = 48, 20011
        x, T, K, P, U = vp_case(41, B, V)
        off, loc = split_vocab(V, world, rank)
        xd = torch.from_numpy(x[:, off:off + loc]).to(torch.bfloat16).to(dev).contiguous()
        Td, Kd, Pd, Ud = (torch.from_numpy(a).to(dev) for a in (T, K, P, U))
        smp = VocabParallelSampler(B, V, world, rank, torch.bfloat16, dev, seed=9, cand_cap=2048 // world,
                                   exchange="peer", timeout_us=5_000_000)
        res = {}
        for step, b in enumerate((B, 20, B)):     # both parities, a smaller batch
            res[f"s{step}"] = smp(xd[:b], Td[:b], Kd[:b], Pd[:b], uniforms=Ud[:b]).cpu().numpy().copy()
        res["philox"] = smp(xd, Td, Kd, Pd).cpu().numpy().copy()
        # two steps captured in a CUDA graph, replayed twice (the epoch lives on the device)
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            smp(xd, Td, Kd, Pd, uniforms=Ud)
            smp(xd, Td, Kd, Pd, uniforms=Ud)
        for i in range(2):
            g.replay()
            torch.cuda.synchronize(dev)
            res[f"graph{i}"] = smp.out[:B].cpu().numpy().copy()
        del g
        res["error"] = np.array([smp.peer.error()])
        res["epoch"] = np.array([int(smp.peer.header[0].item())])
        np.savez(os.path.join(outdir, f"peer{rank}.npz"), **res)
        smp.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_vp_fused_step_two_ranks(tmp_path):
    import torch.multiprocessing as mp
    world = 2
    mp.spawn(_peer_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    r0, r1 = (np.load(tmp_path / f"peer{r}.npz") for r in range(world))
    for k in r0.files:
        assert np.array_equal(r0[k], r1[k]), k
    assert r0["error"][0] == 0 and r0["epoch"][0] == 8    # 4 eager steps + 2 replays of 2
    x, T, K, P, U = vp_case(41, 48, 20011)
    want, res = oracle_ids(x, T, K, P, U)
    near = np.array([rr.u_margin < BOUNDARY or rr.p_margin < BOUNDARY for rr in res.rows])
    for k in ("s0", "s2", "graph0", "graph1"):
        assert np.array_equal(r0[k][~near], want[~near]), k
    assert np.array_equal(r0["s1"][~near[:20]], want[:20][~near[:20]])
    assert (r0["philox"] >= 0).all()


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
    K[0::3] = 0
    want, res = oracle_ids(x, T, K, P, U)
    near = np.array([rr.u_margin < BOUNDARY or rr.p_margin < BOUNDARY for rr in res.rows])
    a, b = np.load(tmp_path / "full0.npy"), np.load(tmp_path / "full1.npy")
    assert np.array_equal(a, b) and (a >= 0).all()
    assert np.array_equal(a[~near], want[~near])
