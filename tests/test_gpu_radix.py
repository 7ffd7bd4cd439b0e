"""Radix merge through the C ABI: integers encrypted the way the reference encrypts a signed
radix integer (one 2-bit digit per block, runtime/src/encrypt.rs:20-22) become wide
ciphertexts that decrypt to the same integers (decrypt-exact, like every bootstrap output)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

SEED = 2031


@pytest.fixture(scope="module")
def rkeys(pnb):
    return pnb.keygen(seed=SEED, device=0)


def _encrypt_blocks(pnb, keys, digits: np.ndarray, seed: int) -> torch.Tensor:
    """digits [count][nb] -> block ciphertexts [count][nb][kN+1] at the block delta 2^59."""
    count, nb = digits.shape
    ct = pnb.encrypt(keys, torch.tensor(digits.reshape(-1)), seed=seed)
    return ct.reshape(count, nb, -1)


def _decode(pnb, keys, ct: torch.Tensor, log_delta: int):
    ph = pnb.phase(keys, ct).cpu().numpy().astype(np.int64)
    v = ((ph >> (log_delta - 1)) + 1) >> 1  # round to the nearest multiple of delta
    err = ph - (v << log_delta)
    return v, err


def test_merge_signed_8bit_every_value(pnb, rkeys):
    v = np.arange(-128, 128, dtype=np.int64)
    nb = 4
    u = v & 0xFF
    digits = np.stack([(u >> (2 * i)) & 3 for i in range(nb)], axis=1)
    blocks = _encrypt_blocks(pnb, rkeys, digits, SEED + 1)
    out = pnb.radix_merge(rkeys, blocks, 1 << 55, signed=True)
    got, err = _decode(pnb, rkeys, out, 55)
    assert np.array_equal(got, v)
    assert np.abs(err).max() < (1 << 53)


def test_merge_unsigned_with_carries(pnb, rkeys):
    rng = np.random.default_rng(SEED + 2)
    nb, count = 3, 256
    digits = rng.integers(0, 16, (count, nb))  # digit plus carry room, as before propagation
    want = sum(digits[:, i] << (2 * i) for i in range(nb))
    blocks = _encrypt_blocks(pnb, rkeys, digits, SEED + 3)
    out = pnb.radix_merge(rkeys, blocks, 1 << 53, signed=False)
    got, _ = _decode(pnb, rkeys, out, 53)
    assert np.array_equal(got, want)


def test_merge_signed_top_carry_dropped(pnb, rkeys):
    # carries above the top digit of a signed integer lie beyond its width
    nb = 2
    digits = np.array([[1, 2], [3, 2 + 4], [0, 1 + 8], [2, 3 + 12]])
    want = np.array([1 + 4 * -2, 3 + 4 * -2, 0 + 4 * 1, 2 + 4 * -1])
    blocks = _encrypt_blocks(pnb, rkeys, digits, SEED + 4)
    out = pnb.radix_merge(rkeys, blocks, 1 << 56, signed=True)
    got, _ = _decode(pnb, rkeys, out, 56)
    assert np.array_equal(got, want)


def test_merge_rejects_bad_shapes(pnb, rkeys):
    L = rkeys.big_dim + 1
    with pytest.raises(ValueError):
        pnb.radix_merge(rkeys, torch.zeros((2, 2, L - 1), dtype=torch.int64, device="cuda:0"),
                        1 << 56)
    with pytest.raises(pnb.LibraryError, match="63-bit"):
        pnb.radix_merge(rkeys, torch.zeros((1, 32, L), dtype=torch.int64, device="cuda:0"),
                        1 << 56)
