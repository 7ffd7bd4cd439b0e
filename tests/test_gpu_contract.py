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
    (128, 784, 2, 2049, True),   # 784 -> 128 layer (7 K blocks through 4 pipeline stages)
    (33, 65, 1, 300, False),     # ragged tiles, no bias
    (1, 1, 1, 1, True),          # degenerate
    (200, 130, 3, 2049, True),   # two M tiles; 390 tiles over the persistent CTAs
    (16, 72, 9, 2049, False),    # 585 tiles: several per CTA, both TMEM buffers reused
    (64, 1000, 2, 2049, True),   # one M tile but K > 896: weights streamed per stage
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


def test_contract_gather_matches_im2col(pnb, oracle):
    # A 2x2 / stride-1 "convolution" over a 1 x 5 x 5 map of ciphertexts with zero padding 1:
    # the gather table holds, per output position, the input ciphertext under each tap.
    rng = np.random.default_rng(77)
    H = W_ = 5
    L = 2049
    X = rng.integers(0, 1 << 63, (H * W_, L), dtype=np.uint64) * np.uint64(2)
    kh = kw = 2
    pad = 1
    oh, ow = H + 2 * pad - kh + 1, W_ + 2 * pad - kw + 1
    idx = np.full((oh * ow, kh * kw), -1, dtype=np.int32)
    for oy in range(oh):
        for ox in range(ow):
            for ky in range(kh):
                for kx in range(kw):
                    iy, ix = oy + ky - pad, ox + kx - pad
                    if 0 <= iy < H and 0 <= ix < W_:
                        idx[oy * ow + ox, ky * kw + kx] = iy * W_ + ix
    Wt = rng.integers(-8, 8, (3, kh * kw), dtype=np.int64)
    bias = rng.integers(-20, 20, 3)
    delta = 1 << 50
    got = pnb.lwe_contract_gather(torch.tensor(Wt.astype(np.int8), device="cuda"),
                                  torch.tensor(bias, device="cuda"), delta,
                                  torch.tensor(X.view(np.int64), device="cuda"),
                                  torch.tensor(idx, device="cuda"))
    got = got.cpu().numpy().view(np.uint64)
    Xg = np.zeros((oh * ow, kh * kw, L), dtype=np.uint64)
    for g in range(oh * ow):
        for k in range(kh * kw):
            if idx[g, k] >= 0:
                Xg[g, k] = X[idx[g, k]]
    want = oracle.contract(Wt, bias, delta, Xg)
    assert np.array_equal(got, want)
    assert pnb.device_status(0) == 0


@pytest.mark.parametrize("M,K,B,L,ld", [
    (128, 784, 2, 2049, 2050),   # the evaluator's pitch: TMA tiles
    (10, 36, 3, 2049, 2050),     # rows of one group end inside a stage: the next group's
                                 # rows meet zero weights, the last group's read past the end
    (200, 130, 5, 2049, 2052),   # two M tiles, a wider pitch
    (33, 65, 2, 301, 302),       # ragged tiles
    (16, 72, 3, 2049, 2049),     # odd pitch: 8-byte gathers
    (128, 256, 2, 8193, 8194),   # N = 8192 ciphertexts at their even pitch
])
def test_contract_pitched_bit_exact(pnb, oracle, M, K, B, L, ld):
    rng = np.random.default_rng(M * 7 + K + ld)
    W = rng.integers(-128, 128, (M, K), dtype=np.int64)
    X = rng.integers(0, 1 << 63, (B, K, ld), dtype=np.uint64) * np.uint64(2) + \
        rng.integers(0, 2, (B, K, ld), dtype=np.uint64)
    bias = rng.integers(-1000, 1000, M)
    delta = 1 << 45
    out = torch.full((B, M, ld), 7, dtype=torch.int64, device="cuda")
    got = pnb.lwe_contract_ld(torch.tensor(W.astype(np.int8), device="cuda"),
                              torch.tensor(bias, device="cuda"), delta,
                              torch.tensor(X.view(np.int64), device="cuda"), L, out=out)
    got = got.cpu().numpy().view(np.uint64)
    want = oracle.contract(W, bias, delta, np.ascontiguousarray(X[:, :, :L]))
    assert np.array_equal(got[:, :, :L], want)
    assert np.all(got[:, :, L:] == 7)  # the pad words are left alone
    assert pnb.device_status(0) == 0


@pytest.mark.parametrize("ld", [2050, 2049])
def test_contract_gather_pitched_bit_exact(pnb, oracle, ld):
    # 16-byte gathers (even pitch) and 8-byte gathers (odd pitch) of a padded 3x3 convolution
    rng = np.random.default_rng(ld)
    L, C, H = 2049, 2, 6
    n_in = C * H * H
    X = rng.integers(0, 1 << 63, (n_in, ld), dtype=np.uint64) * np.uint64(2)
    W = rng.integers(-128, 128, (3, C * 9), dtype=np.int64)
    idx = np.full((H * H, C * 9), -1, dtype=np.int32)
    for oy in range(H):
        for ox in range(H):
            for c in range(C):
                for ky in range(3):
                    for kx in range(3):
                        iy, ix = oy + ky - 1, ox + kx - 1
                        if 0 <= iy < H and 0 <= ix < H:
                            idx[oy * H + ox, c * 9 + ky * 3 + kx] = c * H * H + iy * H + ix
    got = pnb.lwe_contract_gather_ld(torch.tensor(W.astype(np.int8), device="cuda"), None, 0,
                                     torch.tensor(X.view(np.int64), device="cuda"),
                                     torch.tensor(idx, device="cuda"), L)
    got = got.cpu().numpy().view(np.uint64)[:, :, :L]
    Xz = np.concatenate([X[:, :L], np.zeros((1, L), np.uint64)])
    gathered = Xz[np.where(idx < 0, n_in, idx)]          # [G][K][L]
    want = oracle.contract(W, None, 0, np.ascontiguousarray(gathered))
    assert np.array_equal(got, want)
    assert pnb.device_status(0) == 0
