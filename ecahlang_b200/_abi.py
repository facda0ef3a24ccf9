"""ctypes binding of the C ABI in include/ecah_sampler.h.

This is the reference-side binding a maintainer would add to ecahLang: plain
pointers and sizes into ``libecah_sampler.so``.  Loading fails loudly when the
library is missing -- there is no CPU or torch fallback for the sampler.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import c_int32, c_int64, c_size_t, c_uint32, c_void_p

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libecah_sampler.so")

ABI_VERSION = 2
DTYPE_F16, DTYPE_BF16, DTYPE_F32 = 0, 1, 2
FLAG_FREQ_PRES = 0x1

STATUS = {0: "ok", 1: "null pointer", 2: "dtype", 3: "shape", 4: "workspace", 5: "launch", 6: "abi"}

# exported symbols declared in include/ecah_sampler.h
EXPORTS = ("ecah_sampler_abi_version", "ecah_status_string", "ecah_sampler_workspace_bytes",
           "ecah_sampler_launch", "ecah_hist_update", "ecah_philox_uniforms",
           "ecah_sampler_launch_noalloc", "ecah_sampler_noalloc_scratch_bytes",
           "ecah_vp_local", "ecah_vp_merge", "ecah_vp_exchange_bytes", "ecah_vp_step",
           "ecah_vp_ipc_alloc", "ecah_vp_ipc_open", "ecah_vp_ipc_close", "ecah_vp_ipc_free",
           "ecah_quotient_mismatches", "ecah_vp_reset", "ecah_vp_dist_pass")
IPC_HANDLE_BYTES = 64


class SamplerArgs(ctypes.Structure):
    """Mirror of ``struct ecah_sampler_args``."""
    _fields_ = [
        ("abi_version", c_int32), ("dtype", c_int32), ("batch", c_int32), ("vocab", c_int32),
        ("row_stride", c_int64), ("logits", c_void_p), ("temperature", c_void_p),
        ("top_k", c_void_p), ("top_p", c_void_p), ("rep_factor", c_void_p),
        ("freq_pen", c_void_p), ("pres_pen", c_void_p), ("row_slot", c_void_p),
        ("slot_len", c_void_p), ("hist_tok", c_void_p), ("hist_cnt", c_void_p),
        ("hist_mval", c_void_p), ("hist_cap", c_int32), ("num_slots", c_int32),
        ("flags", c_uint32),
        ("uniforms", c_void_p), ("philox_state", c_void_p), ("out", c_void_p), ("row_stats", c_void_p), ("probs_out", c_void_p),
        ("workspace", c_void_p), ("workspace_bytes", c_size_t),
        ("row_index", c_void_p), ("logit_rows", c_int32),
    ]


class VPArgs(ctypes.Structure):
    """Mirror of ``struct ecah_vp_args``."""
    _fields_ = [
        ("abi_version", c_int32), ("dtype", c_int32), ("batch", c_int32), ("vocab", c_int32),
        ("vocab_offset", c_int32), ("vocab_local", c_int32), ("row_stride", c_int64),
        ("logits", c_void_p), ("temperature", c_void_p), ("top_k", c_void_p), ("top_p", c_void_p),
        ("rep_factor", c_void_p), ("row_slot", c_void_p), ("slot_len", c_void_p),
        ("hist_tok", c_void_p), ("hist_cnt", c_void_p), ("hist_mval", c_void_p),
        ("hist_cap", c_int32), ("num_slots", c_int32), ("cand_cap", c_int32),
        ("cand", c_void_p), ("cand_count", c_void_p), ("world", c_int32),
        ("all_cand", c_void_p), ("all_count", c_void_p), ("uniforms", c_void_p),
        ("philox_state", c_void_p), ("out", c_void_p), ("row_stats", c_void_p),
        ("workspace", c_void_p), ("workspace_bytes", c_size_t),
    ]


class VPPeers(ctypes.Structure):
    """Mirror of ``struct ecah_vp_peers``."""
    _fields_ = [("rank", c_int32), ("max_batch", c_int32), ("base", c_void_p), ("timeout_us", c_uint32)]


class EcahError(RuntimeError):
    pass


_lib = None


def lib():
    """Load libecah_sampler.so once; raise if it is absent."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise EcahError(f"{LIB_PATH} is missing: build it with `python -m ecahlang_b200.build` "
                            "(the sampler has no fallback path)")
        L = ctypes.CDLL(LIB_PATH)
        L.ecah_sampler_abi_version.restype = c_int32
        L.ecah_status_string.restype = ctypes.c_char_p
        L.ecah_status_string.argtypes = [c_int32]
        L.ecah_sampler_workspace_bytes.restype = c_size_t
        L.ecah_sampler_workspace_bytes.argtypes = [c_int32, c_int32, c_int32]
        L.ecah_sampler_launch.restype = c_int32
        L.ecah_sampler_launch.argtypes = [ctypes.POINTER(SamplerArgs), c_void_p]
        L.ecah_sampler_launch_noalloc.restype = c_int32
        L.ecah_sampler_launch_noalloc.argtypes = [ctypes.POINTER(SamplerArgs), c_void_p]
        L.ecah_sampler_noalloc_scratch_bytes.restype = c_size_t
        L.ecah_sampler_noalloc_scratch_bytes.argtypes = []
        L.ecah_hist_update.restype = c_int32
        L.ecah_hist_update.argtypes = [c_void_p, c_int32, c_void_p, c_void_p, c_void_p, c_void_p,
                                       c_void_p, c_void_p, c_int32, c_int32, c_int32, c_void_p,
                                       c_void_p]
        L.ecah_vp_local.restype = c_int32
        L.ecah_vp_local.argtypes = [ctypes.POINTER(VPArgs), c_void_p]
        L.ecah_vp_merge.restype = c_int32
        L.ecah_vp_merge.argtypes = [ctypes.POINTER(VPArgs), c_void_p]
        L.ecah_philox_uniforms.restype = c_int32
        L.ecah_philox_uniforms.argtypes = [c_void_p, c_int32, c_void_p, c_int32, c_void_p]
        L.ecah_vp_exchange_bytes.restype = c_size_t
        L.ecah_vp_exchange_bytes.argtypes = [c_int32, c_int32, c_int32]
        L.ecah_vp_step.restype = c_int32
        L.ecah_vp_step.argtypes = [ctypes.POINTER(VPArgs), ctypes.POINTER(VPPeers), c_void_p]
        L.ecah_vp_ipc_alloc.restype = c_int32
        L.ecah_vp_ipc_alloc.argtypes = [c_size_t, ctypes.POINTER(c_void_p), c_void_p]
        L.ecah_vp_ipc_open.restype = c_int32
        L.ecah_vp_ipc_open.argtypes = [c_void_p, ctypes.POINTER(c_void_p)]
        L.ecah_vp_ipc_close.restype = c_int32
        L.ecah_vp_ipc_close.argtypes = [c_void_p]
        L.ecah_vp_reset.restype = c_int32
        L.ecah_vp_dist_pass.restype = c_int32
        L.ecah_vp_dist_pass.argtypes = [ctypes.POINTER(VPArgs), c_int32, c_int32, c_void_p, c_int32, c_void_p,
                                        c_void_p, c_void_p]
        L.ecah_vp_reset.argtypes = [c_void_p, c_uint32, c_void_p]
        L.ecah_vp_ipc_free.restype = c_int32
        L.ecah_vp_ipc_free.argtypes = [c_void_p]
        L.ecah_quotient_mismatches.restype = c_int32
        L.ecah_quotient_mismatches.argtypes = [c_int32, c_void_p, c_int32, c_void_p, c_void_p]
        if L.ecah_sampler_abi_version() != ABI_VERSION:
            raise EcahError("libecah_sampler.so ABI version mismatch")
        _lib = L
    return _lib


def check(status: int, what: str) -> None:
    if status != 0:
        msg = lib().ecah_status_string(status).decode()
        raise EcahError(f"{what} failed: {msg} (status {status})")
