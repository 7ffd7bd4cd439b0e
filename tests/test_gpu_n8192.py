"""The 6-bit parameter set at N = 8192 (pnb_params_n8192) on the GPU, through the C ABI: the
4096-point transform's products against exact negacyclic products, keys bit for bit against the
oracle, decrypt-exact bootstraps with every compiled gadget, the noise against its analytic
model, and the Linear 784 -> 128 + Requant configuration evaluated exactly."""
from __future__ import annotations

import json
import os

import numpy as np
import pytest
import torch

import ir_eval

pytestmark = pytest.mark.gpu

SEED = 8192


def _u64(t):
    return t.cpu().numpy().view(np.uint64)


def _oracle_params(oracle, p):
    return oracle.Params(p.n, p.k, p.N, p.pbs_base_log, p.pbs_level, p.ks_base_log, p.ks_level,
                         p.msg_bits, p.carry_bits, 0, p.lwe_std, p.glwe_std)


def test_fft8k_product_precision(pnb, oracle):
    rng = np.random.default_rng(3)
    N, count = 8192, 3
    a = rng.integers(-(1 << 22), 1 << 22, (count, N), dtype=np.int64)
    b = rng.integers(0, 1 << 64, (count, N), dtype=np.uint64)
    got = _u64(pnb.fft_negacyclic_mul(torch.tensor(a, device="cuda"),
                                      torch.tensor(b.view(np.int64), device="cuda")))
    worst = 0.0
    for c in range(count):
        d = (got[c] - oracle.negacyclic_mul(a[c].view(np.uint64), b[c])).view(np.int64)
        worst = max(worst, float(np.abs(d.astype(np.float64)).max()))
    # products of magnitude ~2^92 keep ~53 bits
    assert worst < 2.0 ** 47, f"worst FFT error 2^{np.log2(worst):.1f}"


def test_keygen_8k_bit_exact(pnb, oracle):
    # a reduced small dimension keeps the oracle's bootstrapping-key generation short; every
    # other field is the 6-bit set's
    p = pnb.params_n8192()
    p.n = 24
    g = pnb.keygen(p, seed=SEED, device=0)
    ok = oracle.OracleKeys(_oracle_params(oracle, p), SEED)
    ex = g.export(lwe_sk=True, glwe_sk=True, bsk=True, ksk=True)
    for name in ("lwe_sk", "glwe_sk", "bsk", "ksk"):
        assert np.array_equal(ex[name], getattr(ok, name)), name
    msgs = np.arange(64)
    ct = pnb.encrypt(g, torch.tensor(msgs), seed=5)
    assert np.array_equal(_u64(ct), ok.encrypt_big(msgs, seed=5))


def _analytic_log2_sigma(p):
    # key noise through the digits, gadget rounding, and the f64 product error (relative
    # 2^-51.1 of the product's spread), the last two amplified by the secret key
    s = p.glwe_std * 2.0 ** 64
    ed2 = (2.0 ** p.pbs_base_log) ** 2 / 12
    v1 = p.n * (p.k + 1) * p.pbs_level * p.N * ed2 * s * s
    eps = 2.0 ** (64 - p.pbs_base_log * p.pbs_level)
    v2 = (p.n / 2) * (1 + p.k * p.N / 2) * eps * eps / 12
    sp2 = 2.0 ** (-102.2) * p.N * ed2 * 2.0 ** 126 / 3
    v3 = p.n * (1 + p.k * p.N / 2) * (p.k + 1) * p.pbs_level * sp2
    return 0.5 * np.log2(v1 + v2 + v3)


@pytest.mark.parametrize("base_log,level", [(23, 1), (15, 2), (11, 4)])
def test_pbs_8k_decrypts_to_the_lut(pnb, base_log, level):
    p = pnb.params_n8192()
    p.pbs_base_log, p.pbs_level = base_log, level
    keys = pnb.keygen(p, seed=SEED, device=0)
    rng = np.random.default_rng(base_log)
    count = 512
    msgs = rng.integers(0, 64, count)
    msgs[:64] = np.arange(64)
    lut = rng.integers(0, 64, 64)
    tv = pnb.test_vector(keys, lut)
    ct = pnb.encrypt(keys, torch.tensor(msgs), seed=SEED + 1)
    out = pnb.pbs_batch(keys, tv, ct)
    got = pnb.decrypt_vec(keys, out).cpu().numpy()
    assert np.array_equal(got, lut[msgs])
    ph = pnb.phase(keys, out).cpu().numpy().view(np.uint64)
    err = (ph - lut[msgs].astype(np.uint64) * np.uint64(p.delta())).view(np.int64)
    log2_std = float(np.log2(err.astype(np.float64).std()))
    assert abs(log2_std - _analytic_log2_sigma(p)) < 1.0, (log2_std, _analytic_log2_sigma(p))
    assert pnb.device_status(0) == 0


def test_linear_requant_at_8k_exact(pnb):
    # the Linear 784 -> 128 (int4 weights) + ReLU-Requant configuration on the 6-bit N = 8192
    # set: contraction over 8193-word ciphertexts, then the exact requant programs
    import importlib.util
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    spec = importlib.util.spec_from_file_location("bench", os.path.join(root, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    g = bench.linear_requant_graph()
    plan = pnb.Plan(pnb.Graph(g), params=pnb.params_n8192())
    ev = pnb.Evaluator(plan, device=0, seed=SEED)
    rng = np.random.default_rng(11)
    x = rng.integers(0, 64, (3, 784))
    got = ev.decrypt(ev.evaluate(ev.encrypt(x, seed=4))).cpu().numpy()
    for xi, row in zip(x, got):
        assert row.tolist() == ir_eval.evaluate(g, {"x": xi.tolist()})["y"]
    assert pnb.device_status(0) == 0
