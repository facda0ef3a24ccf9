"""Philox4x32-10 known-answer vectors (Salmon et al., SC'11; Random123 KAT)."""
import numpy as np

from oracle.philox import philox4x32_10, row_uniforms

KAT = [
    ((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
    ((0xFFFFFFFF,) * 4, (0xFFFFFFFF,) * 2, (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
    ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
     (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)),
]


def test_philox_kat():
    for ctr, key, want in KAT:
        got = philox4x32_10(np.array(ctr, np.uint32), np.array(key, np.uint32))
        assert tuple(int(v) for v in got) == want


def test_row_uniforms_range_and_offset():
    u0 = row_uniforms(123, 0, 4096)
    u1 = row_uniforms(123, 1, 4096)
    assert u0.dtype == np.float32 and (u0 >= 0).all() and (u0 < 1).all()
    assert not np.array_equal(u0, u1)
    assert abs(float(u0.mean()) - 0.5) < 0.02
