"""One op at a time on the GPU, through the C ABI: the per-op entry points an FFI shell keeping
the reference's node walk (runtime/src/eval.rs:104-153) routes each node to -- the contraction
for Linear, pnb_requant_batch / pnb_argmax_batch / pnb_add_batch on a key ring for the rest --
checked by decryption against the reference's integer semantics."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import ir_eval
from test_ops_cpu import SWEEPS, _expect

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ring(pnb):
    return pnb.KeyRing(seed=4242, device=0)


@pytest.mark.parametrize("name", sorted(SWEEPS))
def test_requant_batch_golden_sweep(pnb, ring, name):
    op, xs = SWEEPS[name]
    batch = 3
    x = np.array([xs] * batch, dtype=np.int64)
    scale = 44
    ct = ring.encrypt(x, scale, seed=11)
    desc = pnb.TensorDesc.make(len(xs), -1024, 1023, scale, 0.0)  # fresh encryptions
    kw = {}
    if "mults" in op:
        kw = dict(shift=op["shifts"], mult=op["mults"], round_bias=op["round_biases"],
                  channel_size=op["channel_size"])
    else:
        kw = dict(shift=op["shift"], mult=op["mult"], round_bias=op["round_bias"])
    out, od = pnb.requant_batch(ring, ct, desc, out_bits=2, **kw)
    got = ring.decrypt(out, od.scale_log2).cpu().numpy()
    want = _expect(op, xs)
    for row in got:
        assert row.tolist() == want
    assert (od.lo, od.hi) == (0, 3)
    assert pnb.device_status(0) == 0


def test_node_walk_linear_requant_add_argmax(pnb, ring):
    # Linear (tensor cores) -> Requant -> Add(requant, requant) -> Linear to one logit -> Argmax,
    # each node one call, each output descriptor the next node's input descriptor.  The Requant
    # is asked for a scale and a noise bound its consumers can read exactly.
    rng = np.random.default_rng(5)
    B, K, M = 4, 36, 10
    x = rng.integers(0, 16, (B, K))
    W1 = rng.integers(-8, 8, (M, K))
    b1 = rng.integers(-20, 20, M)
    W2 = rng.integers(-3, 4, (1, M))
    graph = {"inputs": ["x"], "outputs": ["o"], "nodes": [
        {"inputs": ["x"], "outputs": ["a"],
         "op": {"op_type": "Linear", "weights": W1.tolist(), "bias": b1.tolist()}},
        {"inputs": ["a"], "outputs": ["r"],
         "op": {"op_type": "Requant", "shift": 6, "mult": 5, "round_bias": 32, "out_bits": 2,
                "clamp_lut": [0, 1, 2, 3]}},
        {"inputs": ["r", "r"], "outputs": ["s"], "op": {"op_type": "Add"}},
        {"inputs": ["s"], "outputs": ["l"],
         "op": {"op_type": "Linear", "weights": W2.tolist(), "bias": [1]}},
        {"inputs": ["l"], "outputs": ["o"], "op": {"op_type": "Argmax", "threshold": 2}}]}
    s_in = 48
    ct = ring.encrypt(x, s_in, seed=21)
    fresh = float(np.log2(ring.params.glwe_std) + 64)
    # Linear: exact contraction at the input's scale; range and noise follow the weights
    acc = pnb.lwe_contract(torch.tensor(W1.astype(np.int8), device="cuda"),
                           torch.tensor(b1), 1 << s_in, ct)
    lo = int((np.minimum(0, W1) * 15).sum(1).min() + b1.min())
    hi = int((np.maximum(0, W1) * 15).sum(1).max() + b1.max())
    d_acc = pnb.TensorDesc.make(M, lo, hi, s_in, fresh + 0.5 * np.log2((W1 ** 2).sum(1).max()))
    r, d_r = pnb.requant_batch(ring, acc, d_acc, shift=6, mult=5, round_bias=32,
                               out_scale=54, out_sigma=45.0)
    assert d_r.scale_log2 == 54 and d_r.log2_sigma <= 45.0
    s, d_s = pnb.add_batch(ring, r, d_r, r, d_r)
    logit = pnb.lwe_contract(torch.tensor(W2.astype(np.int8), device="cuda"),
                             torch.tensor([1]), 1 << d_s.scale_log2, s)
    d_l = pnb.TensorDesc.make(1, int(np.minimum(0, W2).sum() * 6 + 1),
                              int(np.maximum(0, W2).sum() * 6 + 1), d_s.scale_log2,
                              d_s.log2_sigma + 0.5 * np.log2(float((W2 ** 2).sum())))
    o, d_o = pnb.argmax_batch(ring, logit, d_l, threshold=2)
    got = {"r": ring.decrypt(r, d_r.scale_log2), "s": ring.decrypt(s, d_s.scale_log2),
           "o": ring.decrypt(o, d_o.scale_log2)}
    for b in range(B):
        want = ir_eval.evaluate_all(graph, {"x": x[b].tolist()})
        for t in ("r", "s", "o"):
            assert got[t][b].cpu().tolist() == want[t], (b, t)
    assert pnb.device_status(0) == 0
