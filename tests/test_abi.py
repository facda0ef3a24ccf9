"""CPU checks of the C-ABI library: it loads without a GPU, exports every
symbol include/ecah_sampler.h declares, and rejects bad arguments with status
codes before touching the device."""
import ctypes
import os
import re
import subprocess

import pytest

from ecahlang_b200 import _abi
from ecahlang_b200.build import ROOT, build


@pytest.fixture(scope="module")
def L():
    build()
    return _abi.lib()


def _declared():
    hdr = open(os.path.join(ROOT, "include", "ecah_sampler.h")).read()
    return sorted(set(re.findall(r"ECAH_API\s+[\w\s\*]*?\b(ecah_\w+)\s*\(", hdr)))


def test_header_and_binding_agree():
    assert sorted(_abi.EXPORTS) == _declared()


def test_library_exports_every_declared_symbol(L):
    for name in _declared():
        assert hasattr(L, name), name


def test_abi_version_and_status_strings(L):
    assert L.ecah_sampler_abi_version() == _abi.ABI_VERSION
    for s in range(7):
        assert L.ecah_status_string(s)
    assert L.ecah_sampler_workspace_bytes(128, 151936, 0) >= 4


@pytest.mark.parametrize("mirror,cname", [(_abi.SamplerArgs, "ecah_sampler_args"), (_abi.VPArgs, "ecah_vp_args")])
def test_struct_layout_matches_header(tmp_path, mirror, cname):
    """ctypes mirror vs offsetof() of the C struct, compiled with gcc."""
    fields = [n for n, _ in mirror._fields_]
    src = tmp_path / "off.c"
    src.write_text("#include <stdio.h>\n#include <stddef.h>\n#include \"ecah_sampler.h\"\nint main(){"
                   + "".join(f'printf("%zu\\n", offsetof({cname}, {f}));' for f in fields)
                   + f'printf("%zu\\n", sizeof({cname}));return 0;}}')
    exe = tmp_path / "off"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    got = [int(v) for v in subprocess.run([str(exe)], check=True, capture_output=True,
                                          text=True).stdout.split()]
    want = [getattr(mirror, f).offset for f in fields] + [ctypes.sizeof(mirror)]
    assert got == want


def _args(**kw):
    a = _abi.SamplerArgs()
    a.abi_version = _abi.ABI_VERSION
    a.dtype, a.batch, a.vocab, a.row_stride = 0, 4, 100, 100
    for k, v in kw.items():
        setattr(a, k, v)
    return a


def test_launch_rejects_bad_arguments_without_a_device(L):
    assert L.ecah_sampler_launch(None, None) == 1
    assert L.ecah_sampler_launch(_args(abi_version=99), None) == 6
    assert L.ecah_sampler_launch(_args(dtype=7), None) == 2
    assert L.ecah_sampler_launch(_args(row_stride=50), None) == 3
    assert L.ecah_sampler_launch(_args(vocab=0), None) == 3
    assert L.ecah_sampler_launch(_args(), None) == 1            # no logits
    assert L.ecah_sampler_launch(_args(batch=0), None) == 0     # empty batch is a no-op
    fake = 0x1000
    a = _args(logits=fake, temperature=fake, top_k=fake, top_p=fake, out=fake, uniforms=fake)
    assert L.ecah_sampler_launch(a, None) == 4                  # no workspace
    a = _args(logits=fake, temperature=fake, top_k=fake, top_p=fake, out=fake, uniforms=fake,
              workspace=fake, workspace_bytes=1 << 20, vocab=1 << 30, row_stride=1 << 30)
    assert L.ecah_sampler_launch(a, None) == 3                  # vocab too large for the plan
    assert L.ecah_hist_update(None, 4, None, None, None, None, None, None, 8, 4, 0, None, None) == 1
    assert L.ecah_hist_update(None, 0, None, None, None, None, None, None, 8, 4, 0, None, None) == 0
    assert L.ecah_philox_uniforms(None, 4, None, 0, None) == 1


def test_vocab_parallel_rejects_bad_arguments_without_a_device(L):
    def vp(**kw):
        a = _abi.VPArgs()
        a.abi_version = _abi.ABI_VERSION
        a.dtype, a.batch, a.vocab, a.vocab_offset, a.vocab_local, a.row_stride = 1, 4, 1000, 500, 500, 500
        a.cand_cap, a.world = 64, 2
        for k, v in kw.items():
            setattr(a, k, v)
        return ctypes.byref(a)
    assert L.ecah_vp_local(None, None) == 1
    assert L.ecah_vp_local(vp(abi_version=3), None) == 6
    assert L.ecah_vp_local(vp(dtype=2), None) == 2                  # fp32 logits: not supported
    assert L.ecah_vp_local(vp(vocab_offset=600), None) == 3         # slice past the row end
    assert L.ecah_vp_local(vp(vocab_local=524289, vocab=600000, row_stride=524289), None) == 3  # > 32 rounds
    assert L.ecah_vp_local(vp(vocab_local=70000, vocab=200000, row_stride=69999), None) == 3  # stride < slice
    assert L.ecah_vp_local(vp(world=16, cand_cap=256), None) == 3   # world * cap > 2048
    assert L.ecah_vp_local(vp(), None) == 1                         # parameter arrays missing
    assert L.ecah_vp_merge(vp(batch=0), None) == 0
    # parameter arrays present (never dereferenced: every call below returns before a launch)
    par = dict(temperature=16, top_k=16, top_p=16)
    peers = _abi.VPPeers(0, 4, None, 1000)
    assert L.ecah_vp_step(vp(**par), None, None) == 1                 # no peers
    assert L.ecah_vp_step(vp(**par), ctypes.byref(_abi.VPPeers(2, 4, None, 1000)), None) == 3  # rank >= world
    assert L.ecah_vp_step(vp(**par), ctypes.byref(_abi.VPPeers(0, 3, None, 1000)), None) == 3  # max_batch < batch
    assert L.ecah_vp_step(vp(**par), ctypes.byref(peers), None) == 1  # logits, out and buffers missing
    assert L.ecah_vp_step(vp(batch=0), ctypes.byref(peers), None) == 0
    assert L.ecah_vp_exchange_bytes(0, 2, 64) == 0
    # header, flags [2][4] u32, counts [2][2][4] i32, lists [2][2][4][64] u64, each 256-aligned
    assert L.ecah_vp_exchange_bytes(4, 2, 64) == 256 + 256 + 256 + 2 * 2 * 4 * 64 * 8
    assert L.ecah_vp_ipc_open(None, None) == 1
    assert L.ecah_vp_ipc_close(None) == 1
    assert L.ecah_vp_ipc_free(None) == 1


def test_product_path_fails_loudly_without_library(monkeypatch):
    monkeypatch.setattr(_abi, "_lib", None)
    monkeypatch.setattr(_abi, "LIB_PATH", "/nonexistent/libecah_sampler.so")
    with pytest.raises(_abi.EcahError):
        _abi.lib()


def test_cpu_tensors_are_rejected():
    import torch
    from ecahlang_b200.sampler import launch
    x = torch.zeros(2, 8, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="CUDA"):
        launch(x, torch.ones(2), torch.ones(2, dtype=torch.int32), torch.ones(2),
               torch.zeros(2, dtype=torch.int32), torch.zeros(256, dtype=torch.uint8),
               uniforms=torch.rand(2))
