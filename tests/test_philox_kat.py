"""CPU: the Philox4x32-10 generator behind tensor_randn / malus_rand_int /
malus_rand_uniform (metal.rs:1692-1711), in the oracle and in the runtime
library (host code, no GPU needed), against the published known-answer
vectors of the algorithm (Salmon, Moraes, Dror and Shaw, "Parallel random
numbers: as easy as 1, 2, 3", SC'11; the Random123 known-answer set for
philox4x32 with 10 rounds).  Seeded weights agree with the reference only if
this block function is exact, so it is pinned here independently of both
implementations."""
import ctypes as C
import math

import numpy as np
import pytest

# (counter[4], key[2]) -> output[4]
KAT = [
    ((0x00000000, 0x00000000, 0x00000000, 0x00000000), (0x00000000, 0x00000000),
     (0x6627e8d5, 0xe169c58d, 0xbc57ac4c, 0x9b00dbd8)),
    ((0xffffffff, 0xffffffff, 0xffffffff, 0xffffffff), (0xffffffff, 0xffffffff),
     (0x408f276d, 0x41c83b0e, 0xa20bc7c6, 0x6d5451fd)),
    ((0x243f6a88, 0x85a308d3, 0x13198a2e, 0x03707344), (0xa4093822, 0x299f31d0),
     (0xd16cfe09, 0x94fdcceb, 0x5001e420, 0x24126ea1)),
]


@pytest.mark.parametrize("ctr,key,want", KAT)
def test_oracle_philox_kat(orc, ctr, key, want):
    assert tuple(int(x) for x in orc.philox4x32_10(ctr, key)) == want


@pytest.mark.parametrize("ctr,key,want", KAT)
def test_runtime_philox_kat(rt, ctr, key, want):
    c = (C.c_uint32 * 4)(*ctr)
    k = (C.c_uint32 * 2)(*key)
    rt.malus_philox4x32_10(c, k)
    assert tuple(c) == want


def test_rand_int_uses_the_block_function(orc):
    """rand_int(n) of call i = philox(ctr [1,0,0,0], key = i)[0] % n."""
    for i in (0, 1, 12345, 2 ** 33 + 7):
        r = orc.philox4x32_10((1, 0, 0, 0), (i & 0xffffffff, i >> 32))
        assert orc.rand_int(1000003, i) == int(r[0]) % 1000003


def test_randn_box_muller_of_the_block_function(orc):
    """randn element pair k of call i: Box-Muller (f64) of philox(ctr [k,0,0,0], key = i)."""
    i = 77
    out = orc.randn((6,), i)
    for k in range(3):
        r = orc.philox4x32_10((k, 0, 0, 0), (i, 0))
        u1 = (float(r[0]) + 0.5) / 4294967296.0
        u2 = (float(r[1]) + 0.5) / 4294967296.0
        mag = math.sqrt(-2.0 * math.log(u1))
        assert out[2 * k] == np.float32(mag * math.cos(2.0 * math.pi * u2))
        assert out[2 * k + 1] == np.float32(mag * math.sin(2.0 * math.pi * u2))
