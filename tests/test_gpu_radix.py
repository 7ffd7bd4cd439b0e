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


def test_merge_signed_lower_carries_within_width(pnb, rkeys):
    # lower blocks that still hold carries: the merge equals decrypt_signed's reading (the
    # blocks' sum reduced to the 6-bit width, sign-extended) while the lower blocks' weighted
    # sum stays below the top block's weight (16)
    digits = np.array([[5, 1, 1], [7, 2, 3], [13, 0, 2], [4, 2, 2], [9, 1, 0]])
    width = 6

    def decrypt_signed(d):
        u = sum(int(x) << (2 * i) for i, x in enumerate(d)) % (1 << width)
        return u - (1 << width) if u >= 1 << (width - 1) else u

    want = np.array([decrypt_signed(d) for d in digits])
    blocks = _encrypt_blocks(pnb, rkeys, digits, SEED + 5)
    out = pnb.radix_merge(rkeys, blocks, 1 << 56, signed=True)
    got, _ = _decode(pnb, rkeys, out, 56)
    assert np.array_equal(got, want)


def test_merge_22bit_integers_with_a_multilevel_key_set(pnb):
    # The merged noise is the sum of one bootstrap output per block: 11 blocks through the
    # (2^7, 6) key set (output noise 2^33.8 each) decrypt exactly at delta 2^39, where the
    # single-level set (2^49 each) is limited to about 8-bit integers.
    p = pnb.default_params()
    p.pbs_base_log, p.pbs_level = 7, 6
    keys = pnb.keygen(p, seed=SEED, device=0)
    rng = np.random.default_rng(SEED + 6)
    nb, count = 11, 512
    v = rng.integers(-(1 << 21), 1 << 21, count)
    v[:4] = [-(1 << 21), (1 << 21) - 1, 0, -1]
    u = v & ((1 << (2 * nb)) - 1)
    digits = np.stack([(u >> (2 * i)) & 3 for i in range(nb)], axis=1)
    blocks = _encrypt_blocks(pnb, keys, digits, SEED + 7)
    out = pnb.radix_merge(keys, blocks, 1 << 39, signed=True)
    got, err = _decode(pnb, keys, out, 39)
    assert np.array_equal(got, v)
    assert np.log2(err.astype(np.float64).std()) < 36.5
    assert pnb.device_status(0) == 0


@pytest.fixture(scope="module")
def ring(pnb):
    return pnb.KeyRing(seed=SEED, device=0)


@pytest.mark.parametrize("nb", [4, 12])
def test_split_merge_round_trip_encrypted(pnb, ring, nb):
    # wide signed integers -> the reference's 2-bit radix blocks -> wide again, exactly; 12
    # blocks (24-bit integers) is the widest merge whose summed block noise the lowest-noise
    # key set keeps 7 sigma inside a cell
    lo, hi = -(1 << (2 * nb - 1)), (1 << (2 * nb - 1)) - 1
    scale = 62 - 2 * nb
    rng = np.random.default_rng(SEED + nb)
    count = 64
    v = rng.integers(lo, hi + 1, count)
    v[:4] = [lo, hi, 0, -1]
    split = pnb.radix_plan(nb, pnb.TensorDesc.make(count, lo, hi, scale), to_blocks=True)
    merge = pnb.radix_plan(nb, pnb.TensorDesc.make(count, 0, 0), to_blocks=False)
    ev_s = pnb.Evaluator(split, ring=ring)
    ev_m = pnb.Evaluator(merge, ring=ring)
    wide = ring.encrypt(v.reshape(1, count), scale, seed=SEED + 40 + nb)
    blocks = ev_s.evaluate(wide)                       # [1][count * nb][kN+1]
    digits = ring.decrypt(blocks, 59).cpu().numpy().reshape(count, nb)
    u = v & ((1 << (2 * nb)) - 1)
    assert np.array_equal(digits, np.stack([(u >> (2 * i)) & 3 for i in range(nb)], axis=1))
    back = ev_m.evaluate(blocks)
    got = ring.decrypt(back, merge.desc(True).scale_log2).cpu().numpy().reshape(-1)
    assert np.array_equal(got, v)
    assert pnb.device_status(0) == 0
