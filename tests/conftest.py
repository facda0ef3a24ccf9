import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running CPU test")


def bits_to_f32(arr, dtype):
    """Fixture logits (float16, raw bf16 bits as uint16, or float32) -> float32."""
    arr = np.asarray(arr)
    if dtype == "bf16":
        return (arr.astype(np.uint32) << np.uint32(16)).view(np.float32)
    return arr.astype(np.float32)


def load_golden(name):
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    d = {k: z[k] for k in z.files}
    d["dtype"] = str(d["dtype"])
    d["logits_f32"] = bits_to_f32(d["logits"], d["dtype"])
    return d


def golden_history(d):
    ptr = d["hist_ptr"]
    out = []
    for r in range(len(ptr) - 1):
        s, e = ptr[r], ptr[r + 1]
        out.append((d["hist_tok"][s:e], d["hist_cnt"][s:e], d["hist_mval"][s:e]))
    return out


GOLDEN_CASES = ["ref_f32_basic", "ref_f16_basic", "ref_bf16_basic",
                "ref_f32_ties", "ref_f16_ties", "ref_f16_vocab"]
