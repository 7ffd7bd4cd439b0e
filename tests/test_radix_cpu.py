"""Radix split / merge programs (pnb_radix_plan_create) executed noise-free on the CPU: wide
integers to the reference's signed radix blocks (runtime/src/encrypt.rs:20-22, two's complement
digits of 2 bits, block 0 least significant) and back, for every width up to 12 blocks."""
from __future__ import annotations

import numpy as np
import pytest


def _digits(v, nb):
    u = np.asarray(v, dtype=np.int64) & ((1 << (2 * nb)) - 1)
    return np.stack([(u >> (2 * i)) & 3 for i in range(nb)], axis=-1)


@pytest.mark.parametrize("nb", [1, 2, 4, 8, 11, 12])
def test_split_then_merge_round_trip(pnb, nb):
    lo, hi = -(1 << (2 * nb - 1)), (1 << (2 * nb - 1)) - 1
    scale = 62 - 2 * nb
    rng = np.random.default_rng(nb)
    v = rng.integers(lo, hi + 1, (3, 5))
    v[0, :4] = [lo, hi, 0, -1][:4]
    split = pnb.radix_plan(nb, pnb.TensorDesc.make(5, lo, hi, scale), to_blocks=True)
    blocks, _ = split.simulate(v)
    assert np.array_equal(blocks, _digits(v, nb).reshape(3, -1))
    d = split.desc(True)
    assert (d.elems, d.scale_log2, d.lo, d.hi) == (5 * nb, 59, 0, 3)
    merge = pnb.radix_plan(nb, pnb.TensorDesc.make(5, 0, 0), to_blocks=False)
    back, margin = merge.simulate(blocks)
    assert np.array_equal(back, v) and margin >= 63.5
    assert merge.desc(True).scale_log2 == 63 - 2 * nb


def test_merge_of_carry_blocks_and_unsigned(pnb):
    # blocks still holding carries (digits up to 15) merge to sum(d_i 4^i), top digit signed
    nb = 3
    merge = pnb.radix_plan(nb, pnb.TensorDesc.make(2, 0, 0), to_blocks=False, block_max=15)
    d = np.array([[[5, 9, 1], [15, 0, 3]]]).reshape(1, -1)
    back, _ = merge.simulate(d)
    assert back[0].tolist() == [5 + 36 + 16, 15 + 0 - 16]
    merge = pnb.radix_plan(nb, pnb.TensorDesc.make(1, 0, 0), to_blocks=False, signed=False)
    back, _ = merge.simulate(np.array([[3, 2, 3]]))
    assert back[0].tolist() == [3 + 8 + 48]


def test_radix_refusals(pnb):
    with pytest.raises(pnb.LibraryError, match="do not fit"):
        pnb.radix_plan(2, pnb.TensorDesc.make(1, -9, 7, 40), to_blocks=True)
    with pytest.raises(pnb.LibraryError, match="too large to read"):
        pnb.radix_plan(4, pnb.TensorDesc.make(1, -128, 127, 40, 39.0), to_blocks=True)
    with pytest.raises(pnb.LibraryError, match="no key set"):
        pnb.radix_plan(16, pnb.TensorDesc.make(1, 0, 0), to_blocks=False)
