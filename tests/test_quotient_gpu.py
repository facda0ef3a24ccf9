"""The quotient behind every softmax mass, checked exhaustively on the GPU.

The reference divides the penalised logits by the temperature with torch
(``logits / temperature``, ecahlang/main.py:170), an IEEE float32 divide.  The
kernels compute masses from ``quot_rn`` (the reciprocal of T and one
correction step) instead of a divide per entry.  These tests run every input
of each dtype through both on the device, over a spread of temperatures, and
require equal values wherever the IEEE quotient is a normal float32.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from ecahlang_b200 import _abi

pytestmark = pytest.mark.gpu


def _temperatures():
    rng = np.random.default_rng(7)
    fixed = [1e-5, 1e-4, 0.01, 0.1, 0.3, 0.5, 0.7, 0.8, 0.9, 1.0, 1.1, 1.2, 1.5, 2.0, 3.0, 7.0, 100.0]
    spread = rng.uniform(0.5, 1.2, 48).tolist() + (10.0 ** rng.uniform(-5, 2, 32)).tolist()
    return np.asarray(fixed + spread, dtype=np.float32)


def _mismatches(dtype, temps):
    dev = torch.device("cuda")
    T = torch.as_tensor(temps, dtype=torch.float32, device=dev)
    counts = torch.zeros(2 * len(temps), dtype=torch.int64, device=dev)
    st = _abi.lib().ecah_quotient_mismatches(dtype, ctypes.c_void_p(T.data_ptr()), len(temps),
                                             ctypes.c_void_p(counts.data_ptr()),
                                             ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _abi.check(st, "ecah_quotient_mismatches")
    torch.cuda.synchronize()
    return counts.cpu().numpy().reshape(-1, 2)


@pytest.mark.parametrize("dtype", [_abi.DTYPE_F16, _abi.DTYPE_BF16])
def test_sixteen_bit_inputs_divide_exactly(dtype):
    temps = _temperatures()
    c = _mismatches(dtype, temps)
    bad = {float(t): int(n) for t, n in zip(temps, c[:, 0]) if n}
    assert not bad, f"quotients differ from the IEEE divide at T: {bad}"


def test_float32_inputs_divide_exactly():
    # every float32 bit pattern, at a smaller set of temperatures (each sweep
    # is 2^32 quotients)
    temps = np.asarray([1e-5, 0.5, 0.7, 0.8, 1.0, 1.1, 1.2, 3.0, 0.6180339887, 0.9134], dtype=np.float32)
    c = _mismatches(_abi.DTYPE_F32, temps)
    bad = {float(t): int(n) for t, n in zip(temps, c[:, 0]) if n}
    assert not bad, f"quotients differ from the IEEE divide at T: {bad}"
