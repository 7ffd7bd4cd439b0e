"""Ciphertext byte containers (pnb_lwe_serialize / pnb_lwe_deserialize) on the CPU: round trips
of [count][dim+1] u64 rows, the header, and the refusals of foreign or truncated bytes."""
from __future__ import annotations

import struct

import numpy as np
import pytest


@pytest.mark.parametrize("count,dim", [(0, 834), (1, 2048), (7, 834), (3, 8192)])
def test_lwe_container_round_trip(pnb, count, dim):
    rng = np.random.default_rng(count + dim)
    ct = rng.integers(0, 1 << 64, (count, dim + 1), dtype=np.uint64)
    data = pnb.serialize_lwe(ct)
    assert data[:4] == b"PNBC" and struct.unpack("<III", data[4:16]) == (1, count, dim)
    assert len(data) == 16 + 8 * count * (dim + 1)
    assert np.array_equal(pnb.deserialize_lwe(data), ct)


def test_lwe_container_refusals(pnb):
    ct = np.arange(3 * 11, dtype=np.uint64).reshape(3, 11)
    data = pnb.serialize_lwe(ct)
    with pytest.raises(pnb.LibraryError, match="bytes given"):
        pnb.deserialize_lwe(data[:-8])
    with pytest.raises(pnb.LibraryError, match="not a version-1 ciphertext container"):
        pnb.deserialize_lwe(b"XXXX" + data[4:])
    with pytest.raises(pnb.LibraryError, match="not a version-1 key-set container"):
        pnb.deserialize_keys(b"PNBC" + bytes(100))
