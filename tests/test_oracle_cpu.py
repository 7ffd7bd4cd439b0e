"""CPU checks of the oracle itself (no GPU): known-answer vectors, the Gaussian sampler, the
exact negacyclic product, keyswitch and bootstrapping decrypt to the reference's golden values.

Golden values come from the reference's own tests:
  * runtime/tests/hello_fhe.rs:50-67 -- LUT f(v) = (v + 1) mod 4 over the 2-bit message space,
    applied by programmable bootstrapping under PARAM_MESSAGE_2_CARRY_2_KS_PBS;
  * runtime/tests/hello_fhe.rs:25-44 -- x*w + b with x=1, w=2, b=1 decrypts to 3 (the Linear core).
"""
from __future__ import annotations

import ctypes as C
import math
import struct

import numpy as np
import pytest


def test_chacha20_zero_key_known_answer(oracle):
    # All-zero 256-bit key, zero nonce, block 0: the published ChaCha20 (20 rounds) keystream.
    L = oracle.lib()
    L.orc_chacha20_block_key.argtypes = [C.POINTER(C.c_uint32), C.c_uint64, C.c_uint64,
                                         C.POINTER(C.c_uint32)]
    key = (C.c_uint32 * 8)()
    out = (C.c_uint32 * 16)()
    L.orc_chacha20_block_key(key, 0, 0, out)
    ks = struct.pack("<16I", *out).hex()
    assert ks == ("76b8e0ada0f13d90405d6ae55386bd28bdd219b8a08ded1aa836efcc8b770dc7"
                  "da41597c5157488d7724e03fb8d84a376a43b8f41518a11cc387b669b2ee6586")


def test_series_ln_cos_accuracy(oracle):
    L = oracle.lib()
    rng = np.random.default_rng(1)
    for u in list(rng.random(2000)) + [2.0 ** -53, 0.5, 1.0, 0.7071, 0.9999999]:
        if u <= 0:
            continue
        assert abs(L.orc_ln(u) - math.log(u)) <= 4e-16 * max(1.0, abs(math.log(u)))
    for u in list(rng.random(2000)) + [0.0, 0.25, 0.5, 0.75, 0.125]:
        assert abs(L.orc_cos2pi(u) - math.cos(2 * math.pi * u)) <= 1e-15


def test_gaussian_moments(oracle):
    L = oracle.lib()
    sig = 2.0 ** 40
    z = np.array([L.orc_gaussian(7, 99, i, sig) for i in range(40000)], dtype=np.float64) / sig
    assert abs(z.mean()) < 0.02
    assert abs(z.std() - 1.0) < 0.02
    # fourth moment of a standard normal is 3
    assert abs((z ** 4).mean() - 3.0) < 0.15


def _schoolbook_negacyclic(a, b, N):
    out = [0] * N
    for i in range(N):
        for j in range(N):
            k = i + j
            v = int(a[i]) * int(b[j])
            if k < N:
                out[k] += v
            else:
                out[k - N] -= v
    return np.array([x % (1 << 64) for x in out], dtype=np.uint64)


@pytest.mark.parametrize("N", [64, 128])
def test_exact_negacyclic_mul(oracle, N):
    L = oracle.lib()
    rng = np.random.default_rng(N)
    a = rng.integers(0, 2 ** 63, N, dtype=np.uint64) * np.uint64(2) + rng.integers(0, 2, N,
                                                                                   dtype=np.uint64)
    b = rng.integers(0, 2 ** 63, N, dtype=np.uint64)
    out = np.zeros(N, dtype=np.uint64)
    u64p = C.POINTER(C.c_uint64)
    L.orc_negacyclic_mul(N, a.ctypes.data_as(u64p), b.ctypes.data_as(u64p),
                         out.ctypes.data_as(u64p))
    assert np.array_equal(out, _schoolbook_negacyclic(a, b, N))


@pytest.fixture(scope="module")
def okeys(oracle):
    return oracle.OracleKeys(oracle.default_params(), seed=2024)


def test_encrypt_decrypt_and_linear_core(okeys):
    msgs = np.arange(16)
    ct = okeys.encrypt_big(msgs, seed=5)
    assert np.array_equal(okeys.decode(okeys.phase_big(ct)), msgs)
    # hello_fhe.rs:25-44: x*w + b with plaintext w=2, b=1 on an encryption of x=1 gives 3.
    x = okeys.encrypt_big([1], seed=6)[0]
    y = x * np.uint64(2)
    y[-1] += np.uint64(okeys.delta())
    assert okeys.decode(okeys.phase_big(y[None]))[0] == 3


def test_keyswitch_preserves_message(okeys):
    msgs = np.array([0, 1, 5, 9, 15, 3, 7, 12])
    ct = okeys.encrypt_big(msgs, seed=11)
    ks = okeys.keyswitch(ct)
    assert np.array_equal(okeys.decode(okeys.phase_small(ks)), msgs)


def test_hello_fhe_lut_golden_fft(okeys):
    # runtime/tests/hello_fhe.rs:50-67: f(v) = (v + 1) % 4 over the 2-bit message space.
    lut = [(v + 1) % 4 for v in range(4)] + [0] * 12
    tv = okeys.test_vector(lut)
    ct = okeys.encrypt_big(range(4), seed=21)
    out = okeys.pbs_fft(ct, tv)
    assert list(okeys.decode(okeys.phase_big(out))) == [1, 2, 3, 0]


def test_exact_and_fft_bootstrap_agree_on_values(okeys):
    rng = np.random.default_rng(3)
    msgs = rng.integers(0, 16, 2)
    lut = rng.integers(0, 16, 16)
    tv = okeys.test_vector(lut)
    ct = okeys.encrypt_big(msgs, seed=31)
    ex = okeys.pbs_exact(ct, tv)
    ff = okeys.pbs_fft(ct, tv)
    want = lut[msgs]
    assert np.array_equal(okeys.decode(okeys.phase_big(ex)), want)
    assert np.array_equal(okeys.decode(okeys.phase_big(ff)), want)
    # both outputs carry noise far below delta / 2 = 2^58
    d = okeys.delta()
    for out in (ex, ff):
        err = (okeys.phase_big(out) - (want.astype(np.uint64) * np.uint64(d))).view(np.int64)
        assert np.all(np.abs(err.astype(np.float64)) < 2.0 ** 54)


def test_contraction_matches_integer_sum(oracle, okeys):
    rng = np.random.default_rng(4)
    M, K, B = 3, 5, 2
    W = rng.integers(-8, 8, (M, K))
    bias = rng.integers(-50, 50, M)
    x = rng.integers(0, 4, (B, K))
    delta = 1 << 40  # a wide plaintext space for the accumulator
    X = np.stack([okeys.encrypt_big(x[b], seed=40 + b, delta=delta) for b in range(B)])
    Y = oracle.contract(W, bias, delta, X)
    want = x @ W.T + bias
    ph = okeys.phase_big(Y.reshape(B * M, -1)).view(np.int64)
    dec = np.round(ph.astype(np.float64) / delta).astype(np.int64)
    assert np.array_equal(dec.reshape(B, M), want)
