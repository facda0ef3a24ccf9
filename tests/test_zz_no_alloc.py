"""The sampler entry point for callers that cannot allocate device memory.

``ecah_sampler_launch_noalloc`` serves hosts that may not call cudaMalloc at
sampling time (a runtime that owns all device memory through its own pool, an
FFI caller without a CUDA allocator): it runs the same sampler with scratch
kept in the library's own device memory instead of a caller workspace.  Here
it is called through the C ABI twice in a row and must return exactly the ids
of ``ecah_sampler_launch`` with a caller workspace, advancing the Philox
offset the same way (the Philox path is the one that uses the scratch).
"""
import ctypes

import pytest
import torch

from ecahlang_b200 import _abi
from ecahlang_b200 import workloads as W
from ecahlang_b200._abi import SamplerArgs, lib

pytestmark = pytest.mark.gpu


def _args(x, T, K, P, philox, out, workspace=None):
    a = SamplerArgs()
    a.abi_version = _abi.ABI_VERSION
    a.dtype = _abi.DTYPE_F16
    a.batch, a.vocab = x.shape
    a.row_stride = x.stride(0)
    a.logits = x.data_ptr()
    a.temperature, a.top_k, a.top_p = T.data_ptr(), K.data_ptr(), P.data_ptr()
    a.philox_state = philox.data_ptr()
    a.out = out.data_ptr()
    if workspace is not None:
        a.workspace, a.workspace_bytes = workspace.data_ptr(), workspace.numel()
    return a


def test_noalloc_matches_workspace_entry_point_on_two_calls():
    dev = torch.device("cuda")
    w = W.config2(seed=5, B=64, V=151936)
    x = w.logits.to(dev)
    T, K, P = w.temperature.to(dev), w.top_k.to(dev), w.top_p.to(dev)
    seed = 20261201
    st_ws = torch.tensor([seed, 0], dtype=torch.int64, device=dev)
    st_na = torch.tensor([seed, 0], dtype=torch.int64, device=dev)
    L = lib()
    ws = torch.zeros(L.ecah_sampler_workspace_bytes(64, 151936, _abi.DTYPE_F16), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    # the library's scratch holds the smallest workspace a launch accepts
    assert L.ecah_sampler_noalloc_scratch_bytes() >= 256
    for call in range(2):
        out_ws = torch.full((64,), -1, dtype=torch.int32, device=dev)
        out_na = torch.full((64,), -2, dtype=torch.int32, device=dev)
        a = _args(x, T, K, P, st_ws, out_ws, ws)
        b = _args(x, T, K, P, st_na, out_na)
        assert L.ecah_sampler_launch(ctypes.byref(a), stream) == 0
        assert L.ecah_sampler_launch_noalloc(ctypes.byref(b), stream) == 0
        torch.cuda.synchronize()
        assert torch.equal(out_ws, out_na), f"call {call}: ids differ"
        assert ((out_na >= 0) & (out_na < 151936)).all()
    assert st_ws.cpu().tolist() == st_na.cpu().tolist() == [seed, 2]


def test_noalloc_rejects_bad_arguments():
    L = lib()
    assert L.ecah_sampler_launch_noalloc(None, None) == 1
    a = SamplerArgs()
    a.abi_version = _abi.ABI_VERSION
    a.dtype, a.batch, a.vocab, a.row_stride = 0, 0, 10, 10
    assert L.ecah_sampler_launch_noalloc(ctypes.byref(a), None) == 0   # empty batch
    a.dtype = 9
    assert L.ecah_sampler_launch_noalloc(ctypes.byref(a), None) == 2
