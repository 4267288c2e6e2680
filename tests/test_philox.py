"""Philox4x32-10 known-answer vectors (Salmon et al., SC'11; the Random123 KAT set)."""
import numpy as np

from oracle.oracle import Oracle

KAT = [
    ((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
    ((0xFFFFFFFF,) * 4, (0xFFFFFFFF,) * 2, (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
    ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
     (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)),
]


def test_philox_kat():
    o = Oracle("f32")
    for ctr, key, want in KAT:
        assert tuple(int(x) for x in o.philox(ctr, key)) == want
