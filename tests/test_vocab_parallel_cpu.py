"""Vocab-parallel sampling across two gloo ranks on the CPU: the vocabulary
split (split_vocab), the candidate exchange (the same all-gather the GPU path
runs over NCCL) and the exactness of drawing from the gathered lists, checked
against the CPU oracle on the full rows."""
import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ecahlang_b200.vocab_parallel import nccl_exchange, split_vocab
from vp_util import local_lists, merged_rows, oracle_ids, vp_case

B, V, CAP = 24, 1000, 512


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, outdir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x, T, K, P, U = vp_case(3, B, V)
        off, loc = split_vocab(V, world, rank)
        ids, cnt = local_lists(x[:, off:off + loc], K, T, off, CAP)
        all_ids = torch.empty(world, B, CAP, dtype=torch.int64)
        all_cnt = torch.empty(world, B, dtype=torch.int32)
        nccl_exchange()(torch.from_numpy(ids), torch.from_numpy(cnt), all_ids, all_cnt)
        masked = merged_rows(x, all_ids.numpy(), all_cnt.numpy(), CAP)
        got, _ = oracle_ids(masked, T, K, P, U)
        np.save(os.path.join(outdir, f"ids{rank}.npy"), got)
    finally:
        dist.destroy_process_group()


def test_split_vocab_covers_the_row():
    for world in (1, 2, 3, 8):
        spans = [split_vocab(1001, world, r) for r in range(world)]
        assert spans[0][0] == 0
        assert all(spans[i][0] + spans[i][1] == spans[i + 1][0] for i in range(world - 1))
        assert spans[-1][0] + spans[-1][1] == 1001


def test_two_gloo_ranks_draw_the_oracle_token(tmp_path):
    world = 2
    mp.spawn(_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    x, T, K, P, U = vp_case(3, B, V)
    want, res = oracle_ids(x, T, K, P, U)
    for r in range(world):
        got = np.load(tmp_path / f"ids{r}.npy")
        # rows whose u sits on a CDF boundary of the full row may differ by one entry
        near = np.array([rr.u_margin < 1e-6 for rr in res.rows])
        assert np.array_equal(got[~near], want[~near])


# ---------------------------------------------------------------- failures
# Failures are made on the host (a rank that raises, or leaves between
# steps); the survivors learn of them from the store before their next step,
# or from a short process-group timeout in their next collective.

def _fail_rank(rank, world, port, outdir, mode):
    import datetime

    from ecahlang_b200.vocab_parallel import RankFailure, RankHealth, agree_epoch
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=4))
    store = dist.distributed_c10d._get_default_store()
    health = RankHealth(store, world, rank, timeout_s=2.0, prefix=f"t_{mode}")
    result = "no error"
    try:
        if mode == "epoch":
            # ranks whose step counters drifted apart agree on the largest
            def gather(obj):
                out = [None] * world
                dist.all_gather_object(out, obj)
                return out
            result = f"epoch {agree_epoch(10 + 3 * rank, gather)}"
            return
        for step in range(3):
            if rank == 1 and step == 1 and mode == "raise_between":
                raise RuntimeError("rank 1 fails between steps")
            if rank == 1 and step == 1 and mode == "leave":
                return                                             # leaves between steps
            health.before_step(step)
            if rank == 1 and step == 1 and mode == "raise_in_step":
                raise RuntimeError("rank 1 fails inside step 1, before its exchange")
            x = torch.full((4,), float(rank + step))
            out = torch.empty(world * 4)
            dist.all_gather_into_tensor(out, x)                    # the step's exchange
    except RankFailure as e:
        result = f"RankFailure step={e.step} missing={e.missing}"
    except RuntimeError as e:
        result = f"raised: {e}"
    finally:
        with open(os.path.join(outdir, f"{mode}{rank}.txt"), "w") as f:
            f.write(result)
        if not (mode.startswith("raise") and rank == 1):
            try:
                dist.destroy_process_group()
            except Exception:
                pass


def _run_fail(mode, tmp_path):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_fail_rank, args=(r, 2, port, str(tmp_path), mode)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(60)
        if p.is_alive():
            p.kill()
            p.join()
    return [open(os.path.join(tmp_path, f"{mode}{r}.txt")).read() if os.path.exists(os.path.join(tmp_path, f"{mode}{r}.txt"))
            else None for r in range(2)]


def test_rank_that_raises_between_steps_is_reported_before_the_next_step(tmp_path):
    r0, r1 = _run_fail("raise_between", tmp_path)
    assert r0 == "RankFailure step=1 missing=[1]", r0
    assert r1 == "raised: rank 1 fails between steps"


def test_rank_that_leaves_between_steps_is_reported_before_the_next_step(tmp_path):
    r0, r1 = _run_fail("leave", tmp_path)
    assert r0 == "RankFailure step=1 missing=[1]", r0
    assert r1 == "no error"


def test_rank_that_raises_inside_a_step_ends_the_collective_with_an_error(tmp_path):
    r0, r1 = _run_fail("raise_in_step", tmp_path)
    assert r0 is not None and r0.startswith("raised:"), r0        # not a hang: the collective errs
    assert r1 == "raised: rank 1 fails inside step 1, before its exchange"


def test_ranks_agree_on_the_epoch_to_resume_from(tmp_path):
    r0, r1 = _run_fail("epoch", tmp_path)
    assert r0 == r1 == "epoch 13"
