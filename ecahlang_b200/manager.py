"""The sampling side of ecahLang's AutoKVCacheManager, on the B200 sampler.

ecahLang keeps three sampling pieces on its KV-cache manager
(ecahlang/manager.py): the dense repetition-penalty table
``mask_penalty[seq_lens, V]`` (:31, :36) with a slot per live request
(:57-61, :99-120), pinned host + device sampling-parameter buffers filled
every step (:74-97), and per-bucket copies of those buffers for CUDA-graph
decode (:207-226, :255-268).  ``SamplingManager`` keeps the same method names
and signatures -- the new penalty arguments are optional keywords -- and
replaces the dense table with per-slot token histories (``PenaltyState``),
so a step reads only the tokens a request has produced instead of a [B, V]
mask gather (ecahlang/main.py:356-358, :481-484, :566-569), and the
per-request ``mask /= rp`` launches (main.py:691-694, :519-522, :596-597)
become one batched ``update_penalties``.

``sample()`` is the replacement for ``logits / mask_penalty``,
``logits / temperature`` and ``flashinfer.sampling.top_k_top_p_sampling_from_logits``
(main.py:169-170, :377-379, :486-491, :579-584).
"""
from __future__ import annotations

from typing import Dict, Iterable, Optional, Sequence

import numpy as np
import torch

from .sampler import PenaltyState, launch, new_philox_state, new_workspace, repetition_factor, resolve_device


def _pinned(t: torch.Tensor) -> torch.Tensor:
    return t.pin_memory() if torch.cuda.is_available() else t


class SamplingManager:
    """Slot-indexed penalty histories plus the step's sampling buffers."""

    def __init__(self, vocab_size: int, seq_lens: int = 128, dtype: torch.dtype = torch.float16,
                 device="cuda", history_capacity: int = 1024, seed: int = 0,
                 freq_pres_in_graphs: bool = False):
        self.vocab_size = vocab_size
        self.seq_lens = max(seq_lens, 128)                      # manager.py:31
        self.dtype = dtype
        self.device = resolve_device(device)
        # replaces mask_penalty = ones(seq_lens, V) (manager.py:36)
        self.penalty = PenaltyState(self.seq_lens, history_capacity, dtype, self.device)
        self.free_seq_lens = list(range(self.seq_lens))         # manager.py:57
        self.batch_to_seq_len: Dict[object, int] = {}           # manager.py:61
        self.philox_state = new_philox_state(seed, 0, self.device)
        self._fp_eager = False                                  # any frequency/presence penalty filled
        self._fp_cg: Dict[int, bool] = {}
        # Whether a bucket's sampler was captured into a CUDA graph with the
        # frequency/presence penalties on: a graph replays the launch it
        # captured, so a bucket captured without them cannot take them later.
        # freq_pres_in_graphs=True captures every bucket with them.
        self.freq_pres_in_graphs = freq_pres_in_graphs
        self._cg_captured_fp: Dict[int, bool] = {}
        # overflow flags of the slot histories, copied to the host after every
        # update and checked when the next step's parameters are filled (the
        # host has read the previous step's ids by then)
        self._overflow_host = _pinned(torch.zeros(self.seq_lens, dtype=torch.int32))

    # ------------------------------------------------------------------ slots
    def allocate(self, batch_id) -> int:
        """The penalty slot of a new request, reset to an empty history
        (manager.py:109-111)."""
        if not self.free_seq_lens:
            raise RuntimeError("no free sequence slot")
        seq_len = self.free_seq_lens.pop()
        self.batch_to_seq_len[batch_id] = seq_len
        self.penalty.reset(seq_len)
        self._overflow_host[seq_len] = 0
        return seq_len

    def free(self, batch_id) -> None:
        """manager.py:114-120 (the slot part)."""
        seq_len = self.batch_to_seq_len.pop(batch_id, None)
        if seq_len is not None:
            self.free_seq_lens.append(seq_len)

    def _slots(self, batch_ids: Optional[Sequence]) -> Optional[np.ndarray]:
        if batch_ids is None:
            return None
        slots = np.array([self.batch_to_seq_len[b] for b in batch_ids], dtype=np.int32)
        full = [int(s) for s in slots if self._overflow_host[int(s)]]
        if full:
            raise RuntimeError(
                f"penalty history of slot(s) {full} is full ({self.penalty.capacity} distinct tokens): "
                "later tokens would go unpenalised; raise history_capacity")
        return slots

    # ------------------------------------------------------- eager buffers
    def init_sampling_buffers(self, max_batch_size: int) -> None:
        """Pinned host buffers with numpy views and persistent device buffers
        (manager.py:74-88), plus the penalty columns and the sampler's own
        workspace and output."""
        B, V, dev = max_batch_size, self.vocab_size, self.device
        self.max_batch_size = B
        self.sampling_temperature_cpu = _pinned(torch.ones(B, 1, dtype=torch.float32))
        self.sampling_top_k_cpu = _pinned(torch.full((B,), V, dtype=torch.int32))
        self.sampling_top_p_cpu = _pinned(torch.ones(B, dtype=torch.float32))
        self.sampling_rep_cpu = _pinned(torch.ones(B, dtype=torch.float32))
        self.sampling_freq_cpu = _pinned(torch.zeros(B, dtype=torch.float32))
        self.sampling_pres_cpu = _pinned(torch.zeros(B, dtype=torch.float32))
        self.sampling_slot_cpu = _pinned(torch.full((B,), -1, dtype=torch.int32))
        self.sampling_temperature_np = self.sampling_temperature_cpu.numpy()
        self.sampling_top_k_np = self.sampling_top_k_cpu.numpy()
        self.sampling_top_p_np = self.sampling_top_p_cpu.numpy()
        self.sampling_rep_np = self.sampling_rep_cpu.numpy()
        self.sampling_freq_np = self.sampling_freq_cpu.numpy()
        self.sampling_pres_np = self.sampling_pres_cpu.numpy()
        self.sampling_slot_np = self.sampling_slot_cpu.numpy()
        self.sampling_temperature_gpu = torch.ones(B, 1, dtype=torch.float32, device=dev)
        self.sampling_top_k_gpu = torch.full((B,), V, dtype=torch.int32, device=dev)
        self.sampling_top_p_gpu = torch.ones(B, dtype=torch.float32, device=dev)
        self.sampling_rep_gpu = torch.ones(B, dtype=torch.float32, device=dev)
        self.sampling_freq_gpu = torch.zeros(B, dtype=torch.float32, device=dev)
        self.sampling_pres_gpu = torch.zeros(B, dtype=torch.float32, device=dev)
        self.sampling_slot_gpu = torch.full((B,), -1, dtype=torch.int32, device=dev)
        self.sampling_out = torch.zeros(B, dtype=torch.int32, device=dev)
        self._workspace = None

    def _write_host(self, n, temperatures, top_ks, top_ps, rep_pens, freq_pens, pres_pens, batch_ids) -> bool:
        self.sampling_temperature_np[:n, 0] = temperatures
        self.sampling_top_k_np[:n] = top_ks
        self.sampling_top_p_np[:n] = top_ps
        self.sampling_rep_np[:n] = 1.0 if rep_pens is None else repetition_factor(rep_pens)
        self.sampling_freq_np[:n] = 0.0 if freq_pens is None else freq_pens
        self.sampling_pres_np[:n] = 0.0 if pres_pens is None else pres_pens
        slots = self._slots(batch_ids)
        self.sampling_slot_np[:n] = -1 if slots is None else slots
        return bool(np.any(self.sampling_freq_np[:n] != 0) or np.any(self.sampling_pres_np[:n] != 0))

    def fill_sampling_params(self, n: int, temperatures, top_ks, top_ps, rep_pens=None, freq_pens=None,
                             pres_pens=None, batch_ids: Optional[Sequence] = None) -> None:
        """Writes the first n rows' parameters through the pinned buffers
        (manager.py:90-97).  rep_pens are the requests' repetition penalties
        (stored as the per-update factor), batch_ids select their slots."""
        self._fp_eager = self._write_host(n, temperatures, top_ks, top_ps, rep_pens, freq_pens, pres_pens, batch_ids)
        for g, c in ((self.sampling_temperature_gpu, self.sampling_temperature_cpu),
                     (self.sampling_top_k_gpu, self.sampling_top_k_cpu),
                     (self.sampling_top_p_gpu, self.sampling_top_p_cpu),
                     (self.sampling_rep_gpu, self.sampling_rep_cpu),
                     (self.sampling_freq_gpu, self.sampling_freq_cpu),
                     (self.sampling_pres_gpu, self.sampling_pres_cpu),
                     (self.sampling_slot_gpu, self.sampling_slot_cpu)):
            g[:n].copy_(c[:n], non_blocking=True)

    # ---------------------------------------------------- CUDA-graph buffers
    def init_cuda_graph_buffers(self, bucket_sizes: Iterable[int]) -> None:
        """Per-bucket device copies of the sampling buffers (the sampling part
        of manager.py:207-226) and a sampler output per bucket."""
        V, dev = self.vocab_size, self.device
        self._cg_temperature, self._cg_top_k, self._cg_top_p = {}, {}, {}
        self._cg_rep, self._cg_freq, self._cg_pres, self._cg_slot, self._cg_out = {}, {}, {}, {}, {}
        for bs in bucket_sizes:
            self._cg_temperature[bs] = torch.ones(bs, 1, dtype=torch.float32, device=dev)
            self._cg_top_k[bs] = torch.full((bs,), V, dtype=torch.int32, device=dev)
            self._cg_top_p[bs] = torch.ones(bs, dtype=torch.float32, device=dev)
            self._cg_rep[bs] = torch.ones(bs, dtype=torch.float32, device=dev)
            self._cg_freq[bs] = torch.zeros(bs, dtype=torch.float32, device=dev)
            self._cg_pres[bs] = torch.zeros(bs, dtype=torch.float32, device=dev)
            self._cg_slot[bs] = torch.full((bs,), -1, dtype=torch.int32, device=dev)
            self._cg_out[bs] = torch.zeros(bs, dtype=torch.int32, device=dev)
            self._fp_cg[bs] = False

    def fill_cuda_graph_sampling_params(self, bucket_size: int, n: int, temperatures, top_ks, top_ps,
                                        rep_pens=None, freq_pens=None, pres_pens=None,
                                        batch_ids: Optional[Sequence] = None) -> None:
        """Padding rows reset to (T=1, k=V, p=1, no penalty); the first n rows
        written through the pinned buffers (manager.py:255-268)."""
        bs = bucket_size
        self._cg_temperature[bs].fill_(1.0)
        self._cg_top_k[bs].fill_(self.vocab_size)
        self._cg_top_p[bs].fill_(1.0)
        self._cg_rep[bs].fill_(1.0)
        self._cg_freq[bs].fill_(0.0)
        self._cg_pres[bs].fill_(0.0)
        self._cg_slot[bs].fill_(-1)
        fp = self._write_host(n, temperatures, top_ks, top_ps, rep_pens, freq_pens, pres_pens, batch_ids)
        if fp and self._cg_captured_fp.get(bs) is False:
            raise RuntimeError(
                f"bucket {bs} was captured into a CUDA graph without frequency/presence penalties; "
                "a replay cannot apply them (construct the manager with freq_pres_in_graphs=True)")
        self._fp_cg[bs] = fp
        for g, c in ((self._cg_temperature[bs], self.sampling_temperature_cpu),
                     (self._cg_top_k[bs], self.sampling_top_k_cpu),
                     (self._cg_top_p[bs], self.sampling_top_p_cpu),
                     (self._cg_rep[bs], self.sampling_rep_cpu),
                     (self._cg_freq[bs], self.sampling_freq_cpu),
                     (self._cg_pres[bs], self.sampling_pres_cpu),
                     (self._cg_slot[bs], self.sampling_slot_cpu)):
            g[:n].copy_(c[:n], non_blocking=True)

    # ---------------------------------------------------------------- steps
    def _buffers(self, B: int, bucket_size: Optional[int]):
        if bucket_size is not None:
            bs = bucket_size
            return (self._cg_temperature[bs], self._cg_top_k[bs], self._cg_top_p[bs], self._cg_rep[bs],
                    self._cg_freq[bs], self._cg_pres[bs], self._cg_slot[bs], self._cg_out[bs], self._fp_cg[bs])
        return (self.sampling_temperature_gpu[:B], self.sampling_top_k_gpu[:B], self.sampling_top_p_gpu[:B],
                self.sampling_rep_gpu[:B], self.sampling_freq_gpu[:B], self.sampling_pres_gpu[:B],
                self.sampling_slot_gpu[:B], self.sampling_out[:B], self._fp_eager)

    def sample(self, logits: torch.Tensor, bucket_size: Optional[int] = None,
               uniforms: Optional[torch.Tensor] = None, row_index=None) -> torch.Tensor:
        """One token per row of ``logits`` [B, V] (B = bucket_size for the
        CUDA-graph buffers, else the filled rows), penalties from the rows'
        slots.  Enqueued on the current stream; capturable into a CUDA graph
        (the Philox offset advances on the device).

        ``row_index`` samples rows of a larger [L, V] buffer instead: the
        prefill's ``output.logits[0]`` with the last token of each request,
        ``append_indptr[1:] - 1`` (ecahlang/main.py:476), read in place.  A
        host sequence is range-checked here and copied to the device; a
        device int32 tensor is used as it is."""
        if row_index is not None:
            if not torch.is_tensor(row_index) or not row_index.is_cuda:
                idx = np.asarray(torch.as_tensor(row_index).cpu() if torch.is_tensor(row_index) else row_index,
                                 dtype=np.int64).reshape(-1)
                if idx.size and (idx.min() < 0 or idx.max() >= logits.shape[0]):
                    raise IndexError(f"row_index outside [0, {logits.shape[0]})")
                row_index = torch.as_tensor(idx.astype(np.int32)).to(self.device, non_blocking=True)
            B = row_index.numel()
        else:
            B = logits.shape[0]
        if bucket_size is not None and B != bucket_size:
            raise RuntimeError(f"bucket {bucket_size} needs {bucket_size} logits rows, got {B}")
        T, K, P, rep, freq, pres, slot, out, fp = self._buffers(B, bucket_size)
        if bucket_size is not None:
            fp = fp or self.freq_pres_in_graphs
            if torch.cuda.is_current_stream_capturing():
                self._cg_captured_fp[bucket_size] = fp
        if self._workspace is None:
            self._workspace = new_workspace(self.max_batch_size, self.vocab_size, self.dtype, self.device)
        return launch(logits, T.view(-1), K, P, out, self._workspace,
                      uniforms=uniforms, philox_state=None if uniforms is not None else self.philox_state,
                      rep_factor=rep, freq_pen=freq if fp else None, pres_pen=pres if fp else None,
                      penalty=self.penalty, row_slot=slot, freq_pres=fp, row_index=row_index)

    def sample_async(self, logits: torch.Tensor, bucket_size: Optional[int] = None,
                     uniforms: Optional[torch.Tensor] = None, row_index=None) -> "PendingIds":
        """``sample`` plus the device-to-host copy of the ids, without a
        host sync: the ids go to a pinned host buffer on the current stream
        and an event marks their arrival.  Replaces ``idx_next.cpu()`` after
        ``fwd_stream.synchronize()`` (ecahlang/main.py:415-419, :610-615):
        the host waits on that event only when it needs the ids, and keeps
        scheduling meanwhile.  Each pending step holds its own pinned buffer,
        taken from a pool that ``PendingIds.wait`` refills."""
        ids = self.sample(logits, bucket_size=bucket_size, uniforms=uniforms, row_index=row_index)
        if not hasattr(self, "_id_pool"):
            self._id_pool = []
        n = ids.numel()
        buf = None
        for i, b in enumerate(self._id_pool):
            if b.numel() >= n:
                buf = self._id_pool.pop(i)
                break
        if buf is None:
            buf = _pinned(torch.empty(max(n, getattr(self, "max_batch_size", n)), dtype=torch.int32))
        buf[:n].copy_(ids, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        return PendingIds(buf, n, ev, self._id_pool)

    def update_penalties(self, ids: torch.Tensor, bucket_size: Optional[int] = None) -> None:
        """Records each row's sampled id in its slot history (rows without a
        slot are skipped): one launch for the batch instead of the per-request
        ``mask_penalty[slot, idx] /= rp`` of main.py:691-694."""
        B = ids.numel()
        _, _, _, rep, _, _, slot, _, _ = self._buffers(B, bucket_size)
        self.penalty.update(ids.view(-1)[:B], slot[:B], rep[:B])
        self._overflow_host.copy_(self.penalty.overflow, non_blocking=True)


class PendingIds:
    """A step's sampled ids on their way to pinned host memory."""

    def __init__(self, host: torch.Tensor, n: int, event: "torch.cuda.Event", pool: list):
        self._host, self._n, self._event, self._pool = host, n, event, pool
        self._ids: Optional[np.ndarray] = None

    def ready(self) -> bool:
        """True once the ids are on the host (never blocks)."""
        return self._ids is not None or self._event.query()

    def wait(self) -> np.ndarray:
        """Blocks on this step's event only, then returns the ids; the pinned
        buffer goes back to the pool."""
        if self._ids is None:
            self._event.synchronize()
            self._ids = self._host[:self._n].numpy().copy()
            self._pool.append(self._host)
            self._host = None
        return self._ids
