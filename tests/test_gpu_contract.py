"""Bit-exact parity of the ciphertext x cleartext-weight contraction against the oracle.

The contraction replaces the scalar_mul / add / scalar_add loops of Linear::eval
(runtime/src/ops/linear.rs:52-75); mod 2^64 it is integer arithmetic, so every output word
must equal the oracle's for any input words.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,K,B,L,with_bias", [
    (10, 36, 3, 2049, True),     # tiny-CNN head (36 -> 10) at N = 2048
    (128, 784, 2, 2049, True),   # 784 -> 128 layer
    (33, 65, 1, 300, False),     # ragged tiles, no bias
    (1, 1, 1, 1, True),          # degenerate
])
def test_contract_bit_exact(pnb, oracle, M, K, B, L, with_bias):
    rng = np.random.default_rng(M * 1000 + K)
    W = rng.integers(-128, 128, (M, K), dtype=np.int64)
    X = rng.integers(0, 1 << 63, (B, K, L), dtype=np.uint64) * np.uint64(2) + \
        rng.integers(0, 2, (B, K, L), dtype=np.uint64)
    bias = rng.integers(-1000, 1000, M) if with_bias else None
    delta = 1 << 45
    Wt = torch.tensor(W.astype(np.int8), device="cuda")
    Xt = torch.tensor(X.view(np.int64), device="cuda")
    bt = None if bias is None else torch.tensor(bias, device="cuda")
    got = pnb.lwe_contract(Wt, bt, delta, Xt).cpu().numpy().view(np.uint64)
    want = oracle.contract(W, bias, delta, X)
    assert np.array_equal(got, want)


def test_contract_decrypts_to_integer_linear_layer(pnb):
    keys = pnb.keygen(seed=5, device=0)
    rng = np.random.default_rng(6)
    M, K, B = 10, 36, 4
    x = rng.integers(0, 4, (B, K))
    W = rng.integers(-8, 8, (M, K))
    bias = rng.integers(-100, 100, M)
    delta = 1 << 40
    X = pnb.encrypt(keys, torch.tensor(x.reshape(-1)), seed=9, delta=delta)
    X = X.reshape(B, K, -1)
    Y = pnb.lwe_contract(torch.tensor(W.astype(np.int8), device="cuda"),
                         torch.tensor(bias, device="cuda"), delta, X)
    ph = pnb.phase(keys, Y.reshape(B * M, -1)).cpu().numpy()
    dec = np.round(ph.astype(np.float64) / delta).astype(np.int64).reshape(B, M)
    assert np.array_equal(dec, x @ W.T + bias)
