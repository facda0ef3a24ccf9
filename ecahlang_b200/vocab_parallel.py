"""Vocab-parallel sampling: the LM-head logits of a row are split by vocabulary
over `world` ranks (one process per GPU), each rank samples from its slice's
candidates, and one all-gather of those candidates lets every rank draw the
same token.

ecahLang runs on a single GPU (ecahlang/env.py:112, main.py:201-204); this is
the multi-GPU form of its sampling call (ecahlang/main.py:377-379) for a
vocabulary-split LM head.  Per row, rank g writes every entry of its slice
whose key is at or above the slice's k-th largest key (ties included), in
vocab order with global ids (``ecah_vp_local``); since the row's k-th largest
key is at least every slice's, the union holds the row's whole top-k set, and
``ecah_vp_merge`` finishes the row exactly as the single-GPU sampler does.

Rows without top-k (top_k <= 0 or >= vocab with T > 0: the reference's
default request) keep more than any list holds; they take the exact
distributed path (``ecah_vp_dist_pass``): five passes over the slices with a
collective between each (the row max; the top-p threshold from two summed
256-bin mass histograms, high key byte then low; each rank's kept mass, which
names the rank that owns the draw; that rank's inverse CDF), every step
decided on the device.  Rows with cand_cap < top_k < vocab come back -1.

Two exchanges: ``exchange="peer"`` runs the whole step as one kernel per rank
(``ecah_vp_step``) that stores each row's list straight into every rank's
exchange buffer over NVLink (CUDA IPC mappings, see ``PeerExchange``);
otherwise a callable all-gathers the lists between ``ecah_vp_local`` and
``ecah_vp_merge`` (``nccl_exchange``: NCCL over NVLink).
"""
from __future__ import annotations

import ctypes
import time
from typing import Callable, List, Optional

import torch

from . import _abi
from ._abi import VPArgs, VPPeers, check, lib
from .sampler import PenaltyState, new_philox_state, resolve_device

_DTYPES = {torch.float16: _abi.DTYPE_F16, torch.bfloat16: _abi.DTYPE_BF16}


def split_vocab(vocab: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous slices: rank r holds [offset, offset + local); the first
    vocab % world ranks hold one column more."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} not in [0, {world})")
    base, extra = divmod(vocab, world)
    offset = rank * base + min(rank, extra)
    return offset, base + (1 if rank < extra else 0)


def nccl_exchange(group=None) -> Callable[[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor], None]:
    """All-gather of the candidate lists and counts over a torch.distributed
    group (NCCL over NVLink on GPUs), rank order."""
    import torch.distributed as dist

    def run(cand, count, all_cand, all_count):
        dist.all_gather_into_tensor(all_cand.view(-1), cand.view(-1), group=group)
        dist.all_gather_into_tensor(all_count.view(-1), count.view(-1), group=group)
    return run


class TorchCollectives:
    """The collectives of the rows without top-k over a torch.distributed
    group (NCCL over NVLink on GPUs): an all-gather in rank order into a flat
    output, and an in-place all-reduce ("sum" or "max")."""

    def __init__(self, group=None):
        self.group = group

    def all_gather(self, out: torch.Tensor, inp: torch.Tensor) -> None:
        import torch.distributed as dist
        dist.all_gather_into_tensor(out, inp, group=self.group)

    def all_reduce(self, t: torch.Tensor, op: str) -> None:
        import torch.distributed as dist
        dist.all_reduce(t, op=dist.ReduceOp.SUM if op == "sum" else dist.ReduceOp.MAX, group=self.group)


class _SingleRank:
    """world == 1: the gathers are copies and the reductions are no-ops."""

    def all_gather(self, out, inp):
        out.copy_(inp)

    def all_reduce(self, t, op):
        pass


class FullRowsStep:
    """One step of the rows without top-k on one rank: the launch arguments
    and the listed rows (built by ``VocabParallelSampler.full_rows_begin``)."""

    def __init__(self, args, rows: torch.Tensor, n: int, keep):
        self.args, self.rows, self.n = args, rows, n
        self._keep = keep          # the tensors the arguments point at


class VocabParallelError(RuntimeError):
    """Rows of a vocab-parallel step came back -1: refused rows (top_k above
    cand_cap, rows without top-k) or a wait on another rank that ran out."""


class RankFailure(RuntimeError):
    """Another rank did not reach a step within the health check's timeout."""

    def __init__(self, step: int, missing: List[int]):
        super().__init__(f"ranks {missing} did not reach step {step}")
        self.step, self.missing = step, missing


def agree_epoch(local_epoch: int, all_gather: Callable) -> int:
    """The step counter every rank resumes from after a failure: the largest
    over the ranks (a rank that skipped a step lags; flags only grow, so no
    flag of an earlier step reaches the next step's epoch)."""
    return max(int(e) for e in all_gather(int(local_epoch)))


class RankHealth:
    """Host-side detection of a rank that raised, hung or left between steps.

    Every rank calls ``before_step(s)`` before launching step s: it records
    the rank's arrival at s in the store and waits up to ``timeout_s`` for
    every other rank's, raising ``RankFailure`` with the ranks that did not
    arrive -- before any kernel or collective of step s is launched, so no
    rank waits on the device for a peer that is gone.  A rank that fails
    inside a step (after its arrival) ends the others' collective of that
    step with an error instead (the process group's timeout bounds it).
    ``store`` is any torch.distributed Store (TCPStore, FileStore, the
    default group's store).
    """

    def __init__(self, store, world: int, rank: int, timeout_s: float = 5.0, prefix: str = "ecah_vp"):
        self.store, self.world, self.rank, self.timeout_s, self.prefix = store, world, rank, timeout_s, prefix

    def _key(self, rank: int, step: int) -> str:
        return f"{self.prefix}/step/{rank}/{step}"

    def before_step(self, step: int) -> None:
        self.store.set(self._key(self.rank, step), "1")
        deadline = time.monotonic() + self.timeout_s
        pending = [g for g in range(self.world) if g != self.rank]
        while pending:
            pending = [g for g in pending if not self.store.check([self._key(g, step)])]
            if not pending:
                return
            if time.monotonic() > deadline:
                raise RankFailure(step, pending)
            time.sleep(0.005)


class _DeviceWords:
    """__cuda_array_interface__ of n int32 words at a raw device address."""

    def __init__(self, ptr: int, n: int):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<i4", "data": (ptr, False),
                                         "version": 3, "strides": None}


class PeerExchange:
    """Exchange buffers of the fused step: this rank's buffer
    (``ecah_vp_ipc_alloc``: zero-filled, with a CUDA IPC handle) and every
    other rank's, mapped into this process (``ecah_vp_ipc_open``).

    ``all_gather(obj)`` returns every rank's object in rank order and
    ``barrier()`` waits for every rank; both default to torch.distributed on
    ``group`` (any backend: only the 64-byte handles travel).  The buffers stay
    mapped until ``close``, which every rank calls once its last step is done.
    """

    def __init__(self, max_batch: int, world: int, rank: int, cand_cap: int, device,
                 timeout_us: int = 1_000_000, group=None,
                 all_gather: Optional[Callable] = None, barrier: Optional[Callable] = None):
        if all_gather is None or barrier is None:
            import torch.distributed as dist

            def _all_gather(obj):
                out = [None] * world
                dist.all_gather_object(out, obj, group=group)
                return out
            all_gather = all_gather or _all_gather
            barrier = barrier or (lambda: dist.barrier(group=group))
        L = lib()
        self.device = resolve_device(device)
        self.world, self.rank, self.max_batch = world, rank, max_batch
        self.nbytes = L.ecah_vp_exchange_bytes(max_batch, world, cand_cap)
        if self.nbytes == 0:
            raise ValueError("vocab-parallel exchange: bad max_batch / world / cand_cap")
        own = ctypes.c_void_p()
        handle = (ctypes.c_ubyte * _abi.IPC_HANDLE_BYTES)()
        with torch.cuda.device(self.device):
            check(L.ecah_vp_ipc_alloc(self.nbytes, ctypes.byref(own), handle), "ecah_vp_ipc_alloc")
        self.own = own.value
        self._mapped = []
        self._barrier = barrier
        self._all_gather = all_gather
        handles = all_gather(bytes(handle))
        bases = []
        with torch.cuda.device(self.device):
            for g, h in enumerate(handles):
                if g == rank:
                    bases.append(self.own)
                    continue
                p = ctypes.c_void_p()
                check(L.ecah_vp_ipc_open((ctypes.c_ubyte * _abi.IPC_HANDLE_BYTES).from_buffer_copy(h),
                                         ctypes.byref(p)), "ecah_vp_ipc_open")
                self._mapped.append(p.value)
                bases.append(p.value)
        self.base = torch.tensor(bases, dtype=torch.int64, device=self.device)
        # header words: [0] step epoch, [1] finished rows, [2] error (a wait ran out)
        self.header = torch.as_tensor(_DeviceWords(self.own, 64), device=self.device)
        self.peers = VPPeers(rank, max_batch, self.base.data_ptr(), timeout_us)
        barrier()   # every rank has mapped every buffer before any step stores into them

    def error(self) -> int:
        """Nonzero once a wait on another rank's row ran out (synchronises)."""
        return int(self.header[2].item())

    def epoch(self) -> int:
        """This rank's step counter (synchronises)."""
        return int(self.header[0].item()) & 0xFFFFFFFF

    def reset(self) -> int:
        """Clears the sticky error word and re-syncs the step counter on every
        rank (collective: every rank calls it, with no step in flight), so
        the next step waits only for flags of that step.  Returns the epoch
        the ranks resume from."""
        torch.cuda.synchronize(self.device)
        self._barrier()
        epoch = agree_epoch(self.epoch(), self._all_gather)
        with torch.cuda.device(self.device):
            check(lib().ecah_vp_reset(self.own, epoch, torch.cuda.current_stream(self.device).cuda_stream),
                  "ecah_vp_reset")
        torch.cuda.synchronize(self.device)
        self._barrier()
        return epoch

    def close(self) -> None:
        if self.own is None:
            return
        torch.cuda.synchronize(self.device)
        self._barrier()   # no rank stores into another's buffer any more
        L = lib()
        with torch.cuda.device(self.device):
            for p in self._mapped:
                check(L.ecah_vp_ipc_close(p), "ecah_vp_ipc_close")
            self._mapped = []
            self.header = None
            check(L.ecah_vp_ipc_free(self.own), "ecah_vp_ipc_free")
        self.own = None


class VocabParallelSampler:
    """Per-rank state of the vocab-parallel sampler (buffers sized for
    max_batch, Philox state seeded identically on every rank)."""

    def __init__(self, max_batch: int, vocab: int, world: int, rank: int, dtype: torch.dtype,
                 device="cuda", seed: int = 0, cand_cap: int = 256,
                 exchange=None, timeout_us: int = 1_000_000, collectives=None):
        if dtype not in _DTYPES:
            raise RuntimeError(f"vocab-parallel sampling takes fp16/bf16 logits, not {dtype}")
        if world * cand_cap > 2048:
            raise ValueError("world * cand_cap must stay <= 2048")
        self.vocab, self.world, self.rank, self.dtype = vocab, world, rank, dtype
        self.offset, self.nlocal = split_vocab(vocab, world, rank)
        self.cap = cand_cap
        dev = resolve_device(device)
        self.device = dev
        self.cand = torch.zeros(max_batch, cand_cap, dtype=torch.int64, device=dev)
        self.count = torch.zeros(max_batch, dtype=torch.int32, device=dev)
        self.all_cand = torch.zeros(world, max_batch, cand_cap, dtype=torch.int64, device=dev)
        self.all_count = torch.zeros(world, max_batch, dtype=torch.int32, device=dev)
        self.workspace = torch.zeros(256, dtype=torch.uint8, device=dev)
        self.philox_state = new_philox_state(seed, 0, dev)
        self.out = torch.zeros(max_batch, dtype=torch.int32, device=dev)
        self.peer = None
        if exchange == "peer":
            self.peer = PeerExchange(max_batch, world, rank, cand_cap, dev, timeout_us=timeout_us)
            self.exchange = None
        else:
            self.exchange = exchange if exchange is not None else nccl_exchange()
        # rows without top-k: the exchanges between the distributed passes
        self.collectives = collectives if collectives is not None else (
            _SingleRank() if world == 1 else TorchCollectives())
        self._fr = None

    def _args(self, logits, temperature, top_k, top_p, uniforms, penalty, row_slot, rep_factor, row_stats):
        B = logits.shape[0]
        a = VPArgs()
        a.abi_version = _abi.ABI_VERSION
        a.dtype = _DTYPES[logits.dtype]
        a.batch, a.vocab = B, self.vocab
        a.vocab_offset, a.vocab_local = self.offset, self.nlocal
        a.row_stride = logits.stride(0)
        a.logits = logits.data_ptr()
        a.temperature, a.top_k, a.top_p = temperature.data_ptr(), top_k.data_ptr(), top_p.data_ptr()
        if penalty is not None:
            a.rep_factor = None if rep_factor is None else rep_factor.data_ptr()
            a.row_slot = row_slot.data_ptr()
            a.slot_len, a.hist_tok, a.hist_cnt = (penalty.slot_len.data_ptr(), penalty.tok.data_ptr(),
                                                  penalty.cnt.data_ptr())
            a.hist_mval = penalty.mval.data_ptr()
            a.hist_cap, a.num_slots = penalty.capacity, penalty.num_slots
        a.cand_cap = self.cap
        a.cand, a.cand_count = self.cand.data_ptr(), self.count.data_ptr()
        a.world = self.world
        a.all_cand, a.all_count = self.all_cand.data_ptr(), self.all_count.data_ptr()
        a.uniforms = None if uniforms is None else uniforms.data_ptr()
        a.philox_state = self.philox_state.data_ptr()
        a.out = self.out.data_ptr()
        a.row_stats = None if row_stats is None else row_stats.data_ptr()
        a.workspace, a.workspace_bytes = self.workspace.data_ptr(), self.workspace.numel()
        return a

    def _check(self, logits, temperature, top_k, top_p, uniforms):
        B = logits.shape[0]
        if logits.shape[1] != self.nlocal:
            raise RuntimeError(f"logits slice has {logits.shape[1]} columns, rank {self.rank} holds {self.nlocal}")
        if logits.dtype not in _DTYPES:
            raise RuntimeError(f"logits: fp16/bf16 expected, got {logits.dtype}")
        if logits.device != self.device or logits.stride(1) != 1:
            raise RuntimeError("logits slice must be on the sampler's device with unit column stride")
        if B > self.cand.shape[0]:
            raise RuntimeError(f"batch {B} exceeds max_batch {self.cand.shape[0]}")
        for t, name, dt in ((temperature, "temperature", torch.float32), (top_k, "top_k", torch.int32),
                            (top_p, "top_p", torch.float32)):
            if t.dtype != dt or t.device != self.device or t.numel() != B or not t.is_contiguous():
                raise RuntimeError(f"{name}: expected contiguous {dt} [{B}] on {self.device}")
        if uniforms is not None and (uniforms.dtype != torch.float32 or uniforms.numel() != B
                                     or uniforms.device != self.device):
            raise RuntimeError("uniforms: expected float32 [B] on the sampler's device")

    def local(self, logits: torch.Tensor, temperature: torch.Tensor, top_k: torch.Tensor, top_p: torch.Tensor,
              penalty: Optional[PenaltyState] = None, row_slot: Optional[torch.Tensor] = None,
              rep_factor: Optional[torch.Tensor] = None):
        """This rank's candidate lists for the rows of `logits` ([B, vocab_local]):
        returns views (cand [B, cap] int64, count [B] int32)."""
        self._check(logits, temperature, top_k, top_p, None)
        B = logits.shape[0]
        a = self._args(logits, temperature.reshape(-1), top_k, top_p, None, penalty, row_slot, rep_factor, None)
        check(lib().ecah_vp_local(ctypes.byref(a), torch.cuda.current_stream(self.device).cuda_stream),
              "ecah_vp_local")
        return self.cand[:B], self.count[:B]

    def merge(self, all_cand: torch.Tensor, all_count: torch.Tensor, temperature: torch.Tensor,
              top_k: torch.Tensor, top_p: torch.Tensor, uniforms: Optional[torch.Tensor] = None,
              row_stats: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Draw from the gathered lists (all_cand [world, B, cap], all_count
        [world, B], rank order).  Every rank gets the same [B] ids."""
        B = all_count.shape[1]
        if all_cand.shape != (self.world, B, self.cap) or all_cand.dtype != torch.int64 or not all_cand.is_contiguous():
            raise RuntimeError(f"all_cand: expected contiguous int64 [{self.world}, {B}, {self.cap}]")
        if all_count.shape != (self.world, B) or all_count.dtype != torch.int32 or not all_count.is_contiguous():
            raise RuntimeError(f"all_count: expected contiguous int32 [{self.world}, {B}]")
        a = VPArgs()
        a.abi_version = _abi.ABI_VERSION
        a.dtype = _DTYPES[self.dtype]
        a.batch, a.vocab = B, self.vocab
        a.vocab_offset, a.vocab_local, a.row_stride = self.offset, self.nlocal, self.nlocal
        a.temperature, a.top_k, a.top_p = temperature.reshape(-1).data_ptr(), top_k.data_ptr(), top_p.data_ptr()
        a.cand_cap, a.world = self.cap, self.world
        a.all_cand, a.all_count = all_cand.data_ptr(), all_count.data_ptr()
        a.uniforms = None if uniforms is None else uniforms.data_ptr()
        a.philox_state = self.philox_state.data_ptr()
        a.out = self.out.data_ptr()
        a.row_stats = None if row_stats is None else row_stats.data_ptr()
        a.workspace, a.workspace_bytes = self.workspace.data_ptr(), self.workspace.numel()
        check(lib().ecah_vp_merge(ctypes.byref(a), torch.cuda.current_stream(self.device).cuda_stream),
              "ecah_vp_merge")
        return self.out[:B]

    # ------------------------------------------------ rows without top-k
    def _fr_buffers(self):
        if self._fr is None:
            mb, w, dev = self.cand.shape[0], self.world, self.device
            f = dict(dtype=torch.float32, device=dev)
            self._fr = {
                "state": torch.zeros(mb, 8, **f), "rows": torch.zeros(mb, dtype=torch.int32, device=dev),
                "u": torch.zeros(mb, **f),
                1: torch.zeros(mb, 3, **f), "g1": torch.zeros(w * mb * 3, **f),
                2: torch.zeros(mb, 256, **f), 3: torch.zeros(mb, 257, **f),
                4: torch.zeros(mb, **f), "g4": torch.zeros(w * mb, **f),
                5: torch.zeros(mb, dtype=torch.int32, device=dev),
            }
        return self._fr

    def full_rows_begin(self, logits, temperature, top_k, top_p, rows, uniforms=None, penalty=None,
                        row_slot=None, rep_factor=None) -> FullRowsStep:
        """Sets up the distributed passes of one step for the listed rows
        (host ints, or a device int32 tensor; rows with a top-k or T <= 0
        are skipped on the device).  Without ``uniforms`` it writes this
        step's Philox uniforms first, so call it before the candidate merge,
        which advances the Philox state."""
        self._check(logits, temperature, top_k, top_p, uniforms)
        B = logits.shape[0]
        fr = self._fr_buffers()
        if torch.is_tensor(rows):
            if rows.dtype != torch.int32 or rows.device != self.device or rows.dim() != 1:
                raise RuntimeError("rows: expected a 1-d int32 tensor on the sampler's device")
            rows_t = rows.contiguous()
        else:
            rows = list(rows)
            if any(not 0 <= r < B for r in rows):
                raise IndexError(f"rows must lie in [0, {B})")
            rows_t = fr["rows"][: len(rows)]
            rows_t.copy_(torch.tensor(rows, dtype=torch.int32))
        n = rows_t.numel()
        if n > self.cand.shape[0]:
            raise RuntimeError(f"{n} rows exceed max_batch {self.cand.shape[0]}")
        stream = torch.cuda.current_stream(self.device).cuda_stream
        if uniforms is None:
            uniforms = fr["u"][:B]
            check(lib().ecah_philox_uniforms(self.philox_state.data_ptr(), B, uniforms.data_ptr(), 0, stream),
                  "ecah_philox_uniforms")
        a = self._args(logits, temperature.reshape(-1), top_k, top_p, uniforms, penalty, row_slot, rep_factor,
                       None)
        return FullRowsStep(a, rows_t, n, (logits, temperature, top_k, top_p, uniforms, penalty, row_slot,
                                           rep_factor))

    def full_rows_pass(self, st: FullRowsStep, p: int) -> torch.Tensor:
        """Slice pass p (1..5) of the listed rows; returns this rank's
        outputs ([n, 3], [n, 256], [n, 257], [n], [n] int32) for the
        collective that follows."""
        fr = self._fr_buffers()
        out = fr[p][: st.n]
        check(lib().ecah_vp_dist_pass(ctypes.byref(st.args), self.rank, p, st.rows.data_ptr(), st.n,
                                      fr["state"].data_ptr(), out.data_ptr(),
                                      torch.cuda.current_stream(self.device).cuda_stream), "ecah_vp_dist_pass")
        return out

    def full_rows_combine(self, st: FullRowsStep, p: int, combined: torch.Tensor) -> None:
        """Folds the combined outputs of pass p into the row state (pass 1
        and 4: gathered [world, n, ...] in rank order; 2 and 3: summed over
        the ranks; 5: the max over the ranks, whose ids go to ``out``)."""
        fr = self._fr_buffers()
        if not combined.is_contiguous() or combined.device != self.device:
            raise RuntimeError("combined outputs: expected a contiguous tensor on the sampler's device")
        check(lib().ecah_vp_dist_pass(ctypes.byref(st.args), self.rank, 10 + p, st.rows.data_ptr(), st.n,
                                      combined.data_ptr(), fr["state"].data_ptr(),
                                      torch.cuda.current_stream(self.device).cuda_stream), "ecah_vp_dist_pass")

    def full_rows_run(self, st: FullRowsStep, top_p_rows: bool = True) -> None:
        """The passes with their collectives (``self.collectives``).  A row
        without top-p has its draw's owner chosen from the pass-1 masses, so
        passes 2-4 run only when a listed row may have 0 < top_p < 1."""
        fr = self._fr_buffers()
        n, w = st.n, self.world
        for p in (1, 2, 3, 4, 5):
            if p in (2, 3, 4) and not top_p_rows:
                continue
            o = self.full_rows_pass(st, p)
            if p in (1, 4):
                g = fr["g1" if p == 1 else "g4"][: w * o.numel()]
                self.collectives.all_gather(g, o.reshape(-1))
                combined = g
            else:
                self.collectives.all_reduce(o, "sum" if p in (2, 3) else "max")
                combined = o
            self.full_rows_combine(st, p, combined)

    def find_full_rows(self, temperature, top_k, top_p):
        """Host scan of the step's parameters (a device read): the rows
        without top-k, and whether any of them has 0 < top_p < 1."""
        T = temperature.reshape(-1).cpu()
        K = top_k.cpu()
        P = top_p.cpu()
        sel = (T > 0) & ((K <= 0) | (K >= self.vocab))
        rows = torch.nonzero(sel).view(-1).tolist()
        return rows, bool(((P[sel] > 0) & (P[sel] < 1)).any()) if rows else False

    def __call__(self, logits: torch.Tensor, temperature: torch.Tensor, top_k: torch.Tensor,
                 top_p: torch.Tensor, uniforms: Optional[torch.Tensor] = None,
                 penalty: Optional[PenaltyState] = None, row_slot: Optional[torch.Tensor] = None,
                 rep_factor: Optional[torch.Tensor] = None, row_stats: Optional[torch.Tensor] = None,
                 check_rows: bool = True, full_rows=None) -> torch.Tensor:
        """logits: this rank's [B, vocab_local] slice.  Local candidates, the
        exchange, then the merge (with ``exchange="peer"``: one fused kernel);
        returns the [B] ids (identical on every rank).

        Rows without top-k go through the distributed passes: ``full_rows``
        lists them (host ints or a device int32 tensor; listing every row
        is allowed, the others are skipped on the device).  Left as None, the
        rows are found by reading the parameters back, outside CUDA-graph
        capture; during capture they then come back -1.

        With ``check_rows`` (outside CUDA-graph capture) the call waits for
        the ids and raises ``VocabParallelError`` when a row came back -1;
        a graph-replaying caller passes False and calls ``raise_on_failed``
        on the ids it reads back."""
        ids = self._step(logits, temperature, top_k, top_p, uniforms, penalty, row_slot, rep_factor, row_stats,
                         full_rows)
        if check_rows and not torch.cuda.is_current_stream_capturing():
            self.raise_on_failed(ids)
        return ids

    def raise_on_failed(self, ids) -> None:
        """Raises ``VocabParallelError`` if any of the step's ids is -1 (reads
        them back, and the exchange's error word)."""
        got = ids.cpu() if torch.is_tensor(ids) else torch.as_tensor(ids)
        bad = torch.nonzero(got.view(-1) < 0).view(-1).tolist()
        if bad:
            err = self.peer.error() if self.peer is not None else 0
            why = ("a wait on another rank ran out (call reset() on every rank before the next step)" if err
                   else "rows refused: cand_cap < top_k < vocab, a NaN logit, or a row without top-k "
                        "that was not listed")
            raise VocabParallelError(f"rows {bad[:16]}{'...' if len(bad) > 16 else ''} came back -1: {why}")

    def reset(self) -> int:
        """After a VocabParallelError from a wait that ran out: clears the
        error word and re-syncs the step counter on every rank (collective)."""
        return self.peer.reset() if self.peer is not None else 0

    def _step(self, logits, temperature, top_k, top_p, uniforms, penalty, row_slot, rep_factor, row_stats,
              full_rows=None):
        self._check(logits, temperature, top_k, top_p, uniforms)
        B = logits.shape[0]
        top_p_rows = True
        if full_rows is None and not torch.cuda.is_current_stream_capturing():
            full_rows, top_p_rows = self.find_full_rows(temperature, top_k, top_p)
        fr = None
        if full_rows is not None and len(full_rows) > 0:
            fr = self.full_rows_begin(logits, temperature, top_k, top_p, full_rows, uniforms, penalty, row_slot,
                                      rep_factor)
        if self.peer is not None:
            a = self._args(logits, temperature.reshape(-1), top_k, top_p, uniforms, penalty, row_slot,
                           rep_factor, row_stats)
            check(lib().ecah_vp_step(ctypes.byref(a), ctypes.byref(self.peer.peers),
                                     torch.cuda.current_stream(self.device).cuda_stream), "ecah_vp_step")
        else:
            cand, count = self.local(logits, temperature, top_k, top_p, penalty, row_slot, rep_factor)
            if B == self.cand.shape[0]:
                all_cand, all_count = self.all_cand, self.all_count
            else:
                all_cand = self.all_cand.view(-1)[: self.world * B * self.cap].view(self.world, B, self.cap)
                all_count = self.all_count.view(-1)[: self.world * B].view(self.world, B)
            self.exchange(cand, count, all_cand, all_count)
            self.merge(all_cand, all_count, temperature, top_k, top_p, uniforms, row_stats)
        if fr is not None:
            self.full_rows_run(fr, top_p_rows)
        return self.out[:B]

    def close(self) -> None:
        """Unmaps the peer exchange buffers (every rank, after its last step)."""
        if self.peer is not None:
            self.peer.close()
