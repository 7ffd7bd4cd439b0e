"""The reference runtime's own golden tests, restated: same graphs, parameters and inputs.

Each case follows one test of the reference (file cited per case): the graph it builds, its
`num_blocks` / `input_bits`, its (signed) inputs and its cleartext expectation, which here is
the cleartext oracle `ir_eval` (pinned to the reference's integer evaluator elsewhere).  Every
case is checked twice: the compiled program executed noise-free on the CPU, and the encrypted
evaluation on the GPU through the C ABI.
"""
from __future__ import annotations

import numpy as np
import pytest

import ir_eval


def _g(nodes, inputs, outputs, num_blocks, input_bits):
    return {"schema_version": "0.6.0", "num_blocks": num_blocks, "input_bits": input_bits,
            "inputs": inputs, "outputs": outputs, "nodes": nodes}


def _conv(weights, bias, in_h, in_w, cin, k, stride, pad):
    return {"op_type": "Conv2d", "weights": weights, "bias": bias, "weight_bits": 4,
            "in_h": in_h, "in_w": in_w, "in_channels": cin, "kernel_h": k, "kernel_w": k,
            "stride": stride, "padding": pad}


def _requant(shift, mult=1, rb=0, **extra):
    op = {"op_type": "Requant", "shift": shift, "mult": mult, "round_bias": rb, "out_bits": 2,
          "clamp_lut": [0, 1, 2, 3]}
    op.update(extra)
    return op


def _cases():
    cases = {}
    # runtime/tests/golden_conv2d.rs: 2 -> 2 channels, 3x3, stride 1, no padding, 4x4 map;
    # inputs (i % 9) - 4, weights (i % 5) - 2 and 1 - (i % 3), bias [1, -3]
    x = [(i % 9) - 4 for i in range(32)]
    w = [[(i % 5) - 2 for i in range(18)], [1 - (i % 3) for i in range(18)]]
    cases["conv2d_no_padding"] = (
        _g([{"name": "conv", "inputs": ["x"], "outputs": ["y"],
             "op": _conv(w, [1, -3], 4, 4, 2, 3, 1, 0)}], ["x"], ["y"], 8, 4), [x], None)
    # golden_conv2d.rs: 1 channel, 3x3, stride 1, padding 1; weights (i % 3) - 1, bias [2]
    x = [(i % 9) - 4 for i in range(16)]
    cases["conv2d_padding"] = (
        _g([{"name": "conv", "inputs": ["x"], "outputs": ["y"],
             "op": _conv([[(i % 3) - 1 for i in range(9)]], [2], 4, 4, 1, 3, 1, 1)}],
           ["x"], ["y"], 8, 4), [x], None)
    # runtime/tests/golden_pool.rs (avg): 2 channels 4x4, 2x2 window, stride 2; inputs i - 5
    x = [i - 5 for i in range(32)]
    cases["pool_avg"] = (
        _g([{"name": "pool", "inputs": ["x"], "outputs": ["y"],
             "op": {"op_type": "Pool", "mode": "avg", "in_h": 4, "in_w": 4, "channels": 2,
                    "pool_h": 2, "pool_w": 2, "stride": 2}}], ["x"], ["y"], 6, 5), [x], None)
    # golden_pool.rs (max): the same map and window, the window maximum of wide values
    cases["pool_max"] = (
        _g([{"name": "pool", "inputs": ["x"], "outputs": ["y"],
             "op": {"op_type": "Pool", "mode": "max", "in_h": 4, "in_w": 4, "channels": 2,
                    "pool_h": 2, "pool_w": 2, "stride": 2}}], ["x"], ["y"], 6, 5), [x], None)
    # runtime/tests/golden_add.rs: a = [3, -5], b = [4, 6]
    cases["add"] = (
        _g([{"name": "add", "inputs": ["a", "b"], "outputs": ["sum"],
             "op": {"op_type": "Add"}}], ["a", "b"], ["sum"], 4, 4), [[3, -5, 4, 6]], [2, 2])
    # runtime/tests/golden_requant.rs: shift 4, out_bits 2, inputs up to +-1000
    xs = [-100, 0, 16, 47, 64, 1000, -1, 31, 48]
    cases["requant_shift"] = (
        _g([{"name": "rq", "inputs": ["x"], "outputs": ["y"], "op": _requant(4)}],
           ["x"], ["y"], 6, 10), [xs], [len(xs)])
    # runtime/tests/golden_requant_mult.rs: mult 3, round_bias 16, shift 5
    xs = [-100, -1, 0, 1, 7, 16, 31, 47, 63, 64, 200, 511]
    cases["requant_mult"] = (
        _g([{"name": "rq", "inputs": ["x"], "outputs": ["y"],
             "op": _requant(5, mult=3, rb=16)}], ["x"], ["y"], 7, 10), [xs], [len(xs)])
    # runtime/tests/golden_requant_per_channel.rs: mults [1, 3], shifts [4, 5],
    # round_biases [0, 16], channel_size 3
    xs = [-100, 63, 511, -1, 47, 200]
    cases["requant_per_channel"] = (
        _g([{"name": "rq", "inputs": ["x"], "outputs": ["y"],
             "op": _requant(0, mults=[1, 3], shifts=[4, 5], round_biases=[0, 16],
                            channel_size=3)}], ["x"], ["y"], 7, 10), [xs], [len(xs)])
    # runtime/tests/hello_fhe.rs:50-67: LUT (v + 1) mod 4 over 0..3
    cases["activation_lut"] = (
        _g([{"name": "act", "inputs": ["x"], "outputs": ["y"],
             "op": {"op_type": "Activation", "lut": [1, 2, 3, 0], "output_bits": 2}}],
           ["x"], ["y"], 2, 2), [[0, 1, 2, 3]], [4])
    return cases


CASES = _cases()


def _expect(g, x, lens):
    lens = lens or [len(x)]
    env, off = {}, 0
    for name, n in zip(g["inputs"], lens):
        env[name] = x[off:off + n]
        off += n
    out = []
    for v in ir_eval.evaluate(g, env).values():
        out += v
    return out


def _plan(pnb, g, lens):
    bits = g["input_bits"]
    return pnb.Plan(pnb.Graph(g), input_range=(-(1 << bits) + 1, (1 << bits) - 1),
                    input_lens=lens)


@pytest.mark.parametrize("name", sorted(CASES))
def test_reference_golden_program(pnb, name):
    g, xs, lens = CASES[name]
    pnb.Graph(g).check_budget()
    plan = _plan(pnb, g, lens)
    y, margin = plan.simulate(np.array(xs, dtype=np.int64))
    for x, got in zip(xs, y):
        assert got.tolist() == _expect(g, x, lens)
    assert margin >= 63.5


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(CASES))
def test_reference_golden_encrypted(pnb, name):
    g, xs, lens = CASES[name]
    plan = _plan(pnb, g, lens)
    ev = pnb.Evaluator(plan, device=0, seed=31)
    got = ev.decrypt(ev.evaluate(ev.encrypt(np.array(xs, dtype=np.int64), seed=8)))
    for x, row in zip(xs, got.cpu().numpy()):
        assert row.tolist() == _expect(g, x, lens)
    assert pnb.device_status(0) == 0


def test_max_pool_of_wide_values_random_inputs(pnb):
    # golden_pool.rs's max mode over inputs spanning 63 values: the digit-wise program equals
    # the window maximum on random inputs too
    g, _, lens = CASES["pool_max"]
    plan = _plan(pnb, g, lens)
    xs = np.random.default_rng(7).integers(-31, 32, (32, 32))
    y, margin = plan.simulate(xs)
    for x, got in zip(xs, y):
        assert got.tolist() == _expect(g, x.tolist(), lens)
    assert margin >= 63.5


def _linear_requant_graph():
    # Encrypted Linear 784 -> 128 with int4 weights U[-8, 7] and 6-bit inputs, followed by a
    # ReLU-fused requantization to 2 bits (the synthetic Linear + Requant configuration)
    rng = np.random.default_rng(3)
    W = rng.integers(-8, 8, (128, 784)).tolist()
    nodes = [{"name": "fc", "inputs": ["x"], "outputs": ["acc"],
              "op": {"op_type": "Linear", "weights": W, "bias": [0] * 128, "weight_bits": 4}},
             {"name": "rq", "inputs": ["acc"], "outputs": ["y"],
              "op": _requant(11, mult=1, rb=1024)}]
    return _g(nodes, ["x"], ["y"], 12, 6)


def test_linear_requant_program(pnb):
    g = _linear_requant_graph()
    plan = pnb.Plan(pnb.Graph(g))
    xs = np.random.default_rng(4).integers(0, 64, (6, 784))
    y, margin = plan.simulate(xs)
    for x, got in zip(xs, y):
        assert got.tolist() == ir_eval.evaluate(g, {"x": x.tolist()})["y"]
    assert margin >= 63.5


@pytest.mark.gpu
def test_linear_requant_encrypted(pnb):
    g = _linear_requant_graph()
    plan = pnb.Plan(pnb.Graph(g))
    ev = pnb.Evaluator(plan, device=0, seed=17)
    xs = np.random.default_rng(5).integers(0, 64, (4, 784))
    got = ev.decrypt(ev.evaluate(ev.encrypt(xs, seed=6))).cpu().numpy()
    for x, row in zip(xs, got):
        assert row.tolist() == ir_eval.evaluate(g, {"x": x.tolist()})["y"]
    assert pnb.device_status(0) == 0


def _maxpool_graph():
    # Conv2d -> ReLU-Requant -> 2x2 max pool (stride 2) -> Linear head
    rng = np.random.default_rng(8)
    conv = _conv(rng.integers(-7, 8, (3, 9)).tolist(), [4, -6, 0], 6, 6, 1, 3, 1, 1)
    nodes = [{"name": "conv", "inputs": ["x"], "outputs": ["c"], "op": conv},
             {"name": "rq", "inputs": ["c"], "outputs": ["r"], "op": _requant(6, mult=3, rb=32)},
             {"name": "mp", "inputs": ["r"], "outputs": ["m"],
              "op": {"op_type": "Pool", "mode": "max", "in_h": 6, "in_w": 6, "channels": 3,
                     "pool_h": 2, "pool_w": 2, "stride": 2}},
             {"name": "fc", "inputs": ["m"], "outputs": ["y"],
              "op": {"op_type": "Linear", "weights": rng.integers(-7, 8, (4, 27)).tolist(),
                     "bias": [1, 2, 3, 4], "weight_bits": 4}}]
    return _g(nodes, ["x"], ["m", "y"], 10, 4)


def test_max_pool_program(pnb):
    g = _maxpool_graph()
    plan = pnb.Plan(pnb.Graph(g))
    xs = np.random.default_rng(9).integers(0, 16, (8, 36))
    y, margin = plan.simulate(xs)
    for x, got in zip(xs, y):
        r = ir_eval.evaluate(g, {"x": x.tolist()})
        assert got.tolist() == r["m"] + r["y"]
    assert margin >= 63.5


@pytest.mark.gpu
def test_max_pool_encrypted(pnb):
    g = _maxpool_graph()
    plan = pnb.Plan(pnb.Graph(g))
    ev = pnb.Evaluator(plan, device=0, seed=23)
    xs = np.random.default_rng(10).integers(0, 16, (5, 36))
    got = ev.decrypt(ev.evaluate(ev.encrypt(xs, seed=2))).cpu().numpy()
    for x, row in zip(xs, got):
        r = ir_eval.evaluate(g, {"x": x.tolist()})
        assert row.tolist() == r["m"] + r["y"]
    assert pnb.device_status(0) == 0
