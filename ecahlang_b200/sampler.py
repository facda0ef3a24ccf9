"""Python entry points of the sampler: ``sample()`` / ``Sampler`` and the torch
custom op ``torch.ops.ecah.sample``.

The arithmetic lives in ``libecah_sampler.so`` (sm_100a CUDA).  This module
only checks tensors, builds the C-ABI argument struct and launches on the
current torch stream, so it can be captured in the CUDA graph of the decode
step (the reference captures ``decode_forward`` at ecahlang/main.py:130-157
and runs FlashInfer's sampler eagerly after ``replay()`` at :369-379; this
op can sit inside the graph instead).
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _abi
from ._abi import SamplerArgs, check, lib

_DTYPES = {torch.float16: _abi.DTYPE_F16, torch.bfloat16: _abi.DTYPE_BF16, torch.float32: _abi.DTYPE_F32}


def resolve_device(device) -> torch.device:
    """torch.device with an explicit index ("cuda" -> the current CUDA
    device), so it compares equal to the device of the tensors made on it."""
    dev = torch.device(device)
    if dev.type == "cuda" and dev.index is None and torch.cuda.is_available():
        dev = torch.device("cuda", torch.cuda.current_device())
    return dev


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _need(t: torch.Tensor, name: str, dtype: torch.dtype, numel: int, device: torch.device):
    if t.dtype != dtype:
        raise RuntimeError(f"{name}: expected {dtype}, got {t.dtype}")
    if t.device != device:
        raise RuntimeError(f"{name}: expected device {device}, got {t.device}")
    if not t.is_contiguous():
        raise RuntimeError(f"{name}: must be contiguous")
    if t.numel() != numel:
        raise RuntimeError(f"{name}: expected {numel} elements, got {t.numel()}")


class PenaltyState:
    """Per-slot token histories on the device.

    The sparse equivalent of the reference's dense ``mask_penalty[slot, V]``
    table (ecahlang/manager.py:36): slot s holds up to ``capacity`` distinct
    token ids with their counts and their current mask value m (the value the
    dense table would hold for that token, in the model dtype).  ``reset``
    mirrors the row reset at allocation (manager.py:109-111) and ``update``
    the per-token ``m /= rp`` / ``m *= rp`` of ecahlang/main.py:691-694.
    """

    def __init__(self, num_slots: int, capacity: int, dtype: torch.dtype, device="cuda"):
        if dtype not in _DTYPES:
            raise RuntimeError(f"unsupported model dtype {dtype}")
        self.num_slots, self.capacity, self.dtype = num_slots, capacity, dtype
        dev = torch.device(device)
        self.slot_len = torch.zeros(num_slots, dtype=torch.int32, device=dev)
        self.tok = torch.zeros(num_slots, capacity, dtype=torch.int32, device=dev)
        self.cnt = torch.zeros(num_slots, capacity, dtype=torch.int32, device=dev)
        self.mval = torch.ones(num_slots, capacity, dtype=torch.float32, device=dev)
        self.overflow = torch.zeros(num_slots, dtype=torch.int32, device=dev)

    @property
    def device(self):
        return self.slot_len.device

    def reset(self, slot: int) -> None:
        self.slot_len[slot] = 0
        self.overflow[slot] = 0

    def update(self, ids: torch.Tensor, row_slot: torch.Tensor, rep_factor: Optional[torch.Tensor]) -> None:
        """Record ids[r] in slot row_slot[r] (rows with slot -1 are skipped).
        ``rep_factor`` comes from ``repetition_factor`` (None: no penalty)."""
        B = ids.numel()
        if B == 0:
            return
        dev = self.device
        _need(ids, "ids", torch.int32, B, dev)
        _need(row_slot, "row_slot", torch.int32, B, dev)
        if rep_factor is not None:
            _need(rep_factor, "rep_factor", torch.float32, B, dev)
        stream = torch.cuda.current_stream(dev).cuda_stream
        st = lib().ecah_hist_update(_ptr(ids), B, _ptr(row_slot), _ptr(rep_factor), _ptr(self.slot_len),
                                    _ptr(self.tok), _ptr(self.cnt), _ptr(self.mval), self.capacity,
                                    self.num_slots, _DTYPES[self.dtype], _ptr(self.overflow), stream)
        check(st, "ecah_hist_update")

    def load(self, slot: int, toks, cnts, mvals=None) -> None:
        """Host-side fill of one slot from (token, count[, m]) lists."""
        n = len(toks)
        if n > self.capacity:
            raise RuntimeError("history longer than the slot capacity")
        self.slot_len[slot] = n
        if n:
            self.tok[slot, :n] = torch.as_tensor(toks, dtype=torch.int32)
            self.cnt[slot, :n] = torch.as_tensor(cnts, dtype=torch.int32)
            if mvals is not None:
                self.mval[slot, :n] = torch.as_tensor(mvals, dtype=torch.float32)


def repetition_factor(rp) -> "np.ndarray":
    """Per-update mask multiplier for repetition penalties ``rp`` (floats).

    The reference updates its table with ``mask /= rp`` if rp > 1 else
    ``mask *= rp`` (ecahlang/main.py:691-694) on a CUDA tensor, which torch
    evaluates as one float32 multiply by float32(1/rp) -- the reciprocal taken
    in double -- or by float32(rp).  Computed here on the host from the
    request's double-precision rp, exactly as torch does."""
    import numpy as np
    rp = np.asarray(rp, dtype=np.float64)
    with np.errstate(divide="ignore"):
        return np.where(rp > 1.0, (1.0 / rp), rp).astype(np.float32)


def workspace_bytes(batch: int, vocab: int, dtype: torch.dtype) -> int:
    return int(lib().ecah_sampler_workspace_bytes(batch, vocab, _DTYPES[dtype]))


def new_workspace(batch: int, vocab: int, dtype: torch.dtype, device="cuda") -> torch.Tensor:
    """Zero-filled workspace for launches of up to `batch` rows on `device`
    (its size depends on the device's SM count); every launch leaves its
    counters at zero again.  One workspace per stream that may run a sampler
    launch concurrently."""
    dev = torch.device(device)
    if dev.type == "cuda" and torch.cuda.is_available():
        with torch.cuda.device(dev):
            n = workspace_bytes(batch, vocab, dtype)
    else:
        n = workspace_bytes(batch, vocab, dtype)
    return torch.zeros(n, dtype=torch.uint8, device=dev)


def new_philox_state(seed: int, offset: int = 0, device="cuda") -> torch.Tensor:
    """Device-resident (seed, offset) pair; the sampler bumps the offset."""
    return torch.tensor([seed, offset], dtype=torch.int64, device=device)


def launch(logits: torch.Tensor, temperature: torch.Tensor, top_k: torch.Tensor, top_p: torch.Tensor,
           out: torch.Tensor, workspace: torch.Tensor, *, uniforms: Optional[torch.Tensor] = None,
           philox_state: Optional[torch.Tensor] = None, rep_factor: Optional[torch.Tensor] = None,
           freq_pen: Optional[torch.Tensor] = None, pres_pen: Optional[torch.Tensor] = None,
           penalty: Optional[PenaltyState] = None, row_slot: Optional[torch.Tensor] = None,
           freq_pres: bool = False, use_mval: bool = True, row_stats: Optional[torch.Tensor] = None,
           probs_out: Optional[torch.Tensor] = None, stream: Optional[int] = None,
           row_index: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Enqueue one sampler launch writing ``out[B]`` (int32).

    Optional outputs: ``row_stats`` [B,4] float32 (top-k and final y'
    thresholds, M, Z) and ``probs_out`` [B,V] float32 (the renormalised
    distribution the draw used).

    ``row_index`` (int32 [B] on the device) gathers rows: row r samples
    ``logits[row_index[r]]`` of an [L, V] buffer (the prefill's last token of
    each request, ``append_indptr[1:] - 1`` in ecahlang/main.py:476) without
    copying the rows out; parameters, penalty slots and outputs stay indexed
    by r.  Indices outside [0, L) are clamped on the device, so callers keep
    them in range (``SamplingManager.sample`` checks host-side indices)."""
    if logits.dim() != 2:
        raise RuntimeError("logits must be [B, V]")
    if logits.dtype not in _DTYPES:
        raise RuntimeError(f"unsupported logits dtype {logits.dtype}")
    if not logits.is_cuda:
        raise RuntimeError("logits must be a CUDA tensor (the sampler has no CPU path)")
    if logits.stride(1) != 1:
        raise RuntimeError("logits rows must be contiguous")
    L, V = logits.shape
    dev = logits.device
    B = L
    if row_index is not None:
        B = row_index.numel()
        _need(row_index, "row_index", torch.int32, B, dev)
    _need(temperature, "temperature", torch.float32, B, dev)
    _need(top_k, "top_k", torch.int32, B, dev)
    _need(top_p, "top_p", torch.float32, B, dev)
    _need(out, "out", torch.int32, B, dev)
    for name, t in (("uniforms", uniforms), ("rep_factor", rep_factor), ("freq_pen", freq_pen),
                    ("pres_pen", pres_pen)):
        if t is not None:
            _need(t, name, torch.float32, B, dev)
    if uniforms is None:
        if philox_state is None:
            raise RuntimeError("pass uniforms or a philox_state")
        _need(philox_state, "philox_state", torch.int64, 2, dev)
    if workspace.device != dev or workspace.dtype != torch.uint8:
        raise RuntimeError("workspace must be a uint8 tensor on the logits' device")
    a = SamplerArgs()
    a.abi_version = _abi.ABI_VERSION
    a.dtype = _DTYPES[logits.dtype]
    a.batch, a.vocab = B, V
    a.row_stride = logits.stride(0) if L > 1 else V
    if row_index is not None:
        a.row_index, a.logit_rows = row_index.data_ptr(), L
    a.logits = logits.data_ptr()
    a.temperature, a.top_k, a.top_p = temperature.data_ptr(), top_k.data_ptr(), top_p.data_ptr()
    a.rep_factor, a.freq_pen, a.pres_pen = _ptr(rep_factor), _ptr(freq_pen), _ptr(pres_pen)
    if penalty is not None:
        if row_slot is None:
            raise RuntimeError("penalty state needs row_slot")
        _need(row_slot, "row_slot", torch.int32, B, dev)
        if penalty.dtype != logits.dtype:
            raise RuntimeError("penalty state dtype differs from the logits dtype")
        a.row_slot, a.slot_len = row_slot.data_ptr(), penalty.slot_len.data_ptr()
        a.hist_tok, a.hist_cnt = penalty.tok.data_ptr(), penalty.cnt.data_ptr()
        a.hist_mval = penalty.mval.data_ptr() if use_mval else None
        a.hist_cap = penalty.capacity
        a.num_slots = penalty.slot_len.numel()
    a.flags = _abi.FLAG_FREQ_PRES if freq_pres else 0
    a.uniforms = _ptr(uniforms)
    a.philox_state = _ptr(philox_state)
    a.out = out.data_ptr()
    if row_stats is not None:
        _need(row_stats, "row_stats", torch.float32, 4 * B, dev)
        a.row_stats = row_stats.data_ptr()
    if probs_out is not None:
        _need(probs_out, "probs_out", torch.float32, B * V, dev)
        a.probs_out = probs_out.data_ptr()
    a.workspace, a.workspace_bytes = workspace.data_ptr(), workspace.numel()
    if stream is None:
        stream = torch.cuda.current_stream(dev).cuda_stream
    check(lib().ecah_sampler_launch(a, stream), "ecah_sampler_launch")
    return out


class Sampler:
    """Owns the workspace, the Philox state and the output buffer for one
    stream, so repeated calls (and CUDA-graph replays) allocate nothing."""

    def __init__(self, max_batch: int, vocab: int, dtype: torch.dtype, device="cuda", seed: int = 0):
        self.vocab, self.dtype = vocab, dtype
        self.device = resolve_device(device)
        self.workspace = new_workspace(max_batch, vocab, dtype, self.device)
        self.philox_state = new_philox_state(seed, 0, self.device)
        self.out = torch.zeros(max_batch, dtype=torch.int32, device=self.device)

    def __call__(self, logits, temperature, top_k, top_p, **kw) -> torch.Tensor:
        B = logits.shape[0]
        kw.setdefault("philox_state", None if kw.get("uniforms") is not None else self.philox_state)
        return launch(logits, temperature.reshape(-1), top_k, top_p, self.out[:B], self.workspace, **kw)


# ------------------------------------------------------------ torch custom op
_LIB = torch.library.Library("ecah", "DEF")
_LIB.define(
    "sample(Tensor logits, Tensor temperature, Tensor top_k, Tensor top_p, Tensor? uniforms, "
    "Tensor(a!)? philox_state, Tensor? rep_factor, Tensor? freq_pen, Tensor? pres_pen, "
    "Tensor? row_slot, Tensor? slot_len, Tensor? hist_tok, Tensor? hist_cnt, Tensor? hist_mval, "
    "int hist_cap, int flags, Tensor(b!) out, Tensor(c!) workspace) -> ()")


class _View:
    """PenaltyState-shaped view over raw tensors for the custom op."""

    def __init__(self, slot_len, tok, cnt, mval, cap, dtype):
        self.slot_len, self.tok, self.cnt, self.capacity, self.dtype = slot_len, tok, cnt, cap, dtype
        self.mval = mval if mval is not None else cnt


def _sample_op_cuda(logits, temperature, top_k, top_p, uniforms, philox_state, rep_factor, freq_pen, pres_pen,
                    row_slot, slot_len, hist_tok, hist_cnt, hist_mval, hist_cap, flags, out, workspace):
    pen = None
    if row_slot is not None:
        pen = _View(slot_len, hist_tok, hist_cnt, hist_mval, hist_cap, logits.dtype)
    launch(logits, temperature.reshape(-1), top_k, top_p, out, workspace, uniforms=uniforms,
           philox_state=philox_state, rep_factor=rep_factor, freq_pen=freq_pen, pres_pen=pres_pen, penalty=pen,
           row_slot=row_slot, freq_pres=bool(flags & _abi.FLAG_FREQ_PRES), use_mval=hist_mval is not None)


_LIB.impl("sample", _sample_op_cuda, "CUDA")


@torch.library.register_fake("ecah::sample")
def _sample_op_fake(logits, temperature, top_k, top_p, uniforms, philox_state, rep_factor, freq_pen, pres_pen,
                    row_slot, slot_len, hist_tok, hist_cnt, hist_mval, hist_cap, flags, out, workspace):
    # writes only into `out` (and the Philox offset / workspace); no new tensors
    return None
