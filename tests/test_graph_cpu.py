"""Graph reader, bit-width budget and the compiled ciphertext program, checked on the CPU.

* The cleartext oracle (``oracle/ir_eval.py``) is pinned against every tensor of the golden
  fixtures, which the reference's own quantizer and integer evaluator produced.
* The library's program for each graph is executed noise-free (``pnb_plan_simulate``): its
  decoded outputs must equal the reference's integers exactly, and every bootstrap input must
  sit half a cell (64 units of 2^52 for five-bit windows) from its decision boundary -- the
  margin the noise model is sized against.
* Graph-loading errors carry the reference's diagnoses (``runtime/src/ir.rs:169-452``,
  ``runtime/src/eval.rs:237-276``).
"""
from __future__ import annotations

import glob
import json
import os
import random

import numpy as np
import pytest

import ir_eval
from conftest import GOLDEN_DIR

FIXTURES = sorted(glob.glob(os.path.join(GOLDEN_DIR, "*.json")))


def _doc(path):
    with open(path) as f:
        return json.load(f)


def _flat(o):
    return o if isinstance(o, list) else [o]


@pytest.mark.parametrize("path", FIXTURES, ids=os.path.basename)
def test_oracle_pinned_to_reference_tensors(path):
    d = _doc(path)
    g = d["graph"]
    for x, tensors in zip(d["inputs"], d["tensors"]):
        env = ir_eval.evaluate_all(g, {g["inputs"][0]: x})
        for name, want in tensors.items():
            assert env[name] == _flat(want), name


@pytest.mark.parametrize("path", FIXTURES, ids=os.path.basename)
def test_program_reproduces_reference_outputs(pnb, path):
    d = _doc(path)
    graph = pnb.Graph(d["graph"])
    plan = pnb.Plan(graph)
    y, margin = plan.simulate(np.array(d["inputs"], dtype=np.int64))
    want = np.array([_flat(o) for o in d["outputs"]], dtype=np.int64)
    assert np.array_equal(y, want)
    assert margin >= 63.5
    assert plan.pbs_per_sample > 0 or "Requant" not in json.dumps(d["graph"])


def _graph(nodes, inputs=("x",), outputs=None, num_blocks=16, input_bits=10):
    return {"schema_version": "0.6.0", "num_blocks": num_blocks, "input_bits": input_bits,
            "inputs": list(inputs), "outputs": outputs or [nodes[-1]["outputs"][0]],
            "nodes": nodes}


def _node(name, op, inputs, out=None):
    return {"name": name, "inputs": inputs, "outputs": [out or name + "_out"], "op": op}


def _requant(shift, mult=1, rb=0, out_bits=2, lut=(0, 1, 2, 3), **extra):
    op = {"op_type": "Requant", "shift": shift, "mult": mult, "round_bias": rb,
          "out_bits": out_bits, "clamp_lut": list(lut)}
    op.update(extra)
    return op


def _check_program(pnb, g, xs, input_range, input_lens=None):
    plan = pnb.Plan(pnb.Graph(g), input_range=input_range, input_lens=input_lens)
    y, margin = plan.simulate(np.array(xs, dtype=np.int64))
    for x, got in zip(xs, y):
        want = []
        for v in ir_eval.evaluate(g, {g["inputs"][0]: list(x)}).values():
            want += v
        assert got.tolist() == want, (x, got.tolist(), want)
    assert margin >= 63.5
    return plan


def test_requant_sweep_matches_reference_golden_inputs(pnb):
    # the inputs and rescale of the reference's golden_requant_mult sweep, every value at once
    xs = [-100, -1, 0, 1, 7, 16, 31, 47, 63, 64, 200, 511]
    g = _graph([_node("rq", _requant(5, mult=3, rb=16), ["x"])], num_blocks=7)
    _check_program(pnb, g, [xs], (-512, 511), input_lens=[len(xs)])


@pytest.mark.parametrize("mult,shift,rb,lut", [
    (1, 6, 0, (0, 1, 2, 3)), (3, 5, 16, (0, 1, 2, 3)), (21, 10, 512, (0, 1, 2, 3)),
    (7, 4, 3, (3, 0, 2, 1)), (1, 3, 100, (0, 1, 2, 3)), (5, 9, 0, (2, 2, 2, 2)),
])
def test_requant_exhaustive_over_range(pnb, mult, shift, rb, lut):
    lo, hi = -700, 900
    xs = list(range(lo, hi + 1))
    g = _graph([_node("rq", _requant(shift, mult=mult, rb=rb, lut=lut), ["x"])])
    _check_program(pnb, g, [[v] for v in xs], (lo, hi), input_lens=[1])


def test_per_channel_requant_conv_padding_pool_add_activation_argmax(pnb):
    rnd = random.Random(3)
    C_in, H, W, C_out, kh, kw = 2, 6, 5, 3, 3, 3
    conv = {"op_type": "Conv2d", "weights": [[rnd.randint(-20, 20) for _ in range(C_in * kh * kw)]
                                             for _ in range(C_out)],
            "bias": [rnd.randint(-50, 50) for _ in range(C_out)], "weight_bits": 6,
            "in_h": H, "in_w": W, "in_channels": C_in, "kernel_h": kh, "kernel_w": kw,
            "stride": 1, "padding": 1}
    positions = H * W
    rq = _requant(0, mults=[7, 11, 3], shifts=[8, 9, 7], round_biases=[128, 3, 64],
                  channel_size=positions, lut=(0, 2, 1, 3))
    act = {"op_type": "Activation", "lut": [1, 3, 0, 2], "output_bits": 2}
    pool = {"op_type": "Pool", "mode": "avg", "in_h": H, "in_w": W, "channels": C_out,
            "pool_h": 2, "pool_w": 2, "stride": 2}
    n_pool = C_out * ((H - 2) // 2 + 1) * ((W - 2) // 2 + 1)
    lin = {"op_type": "Linear", "weights": [[rnd.randint(-9, 9) for _ in range(n_pool)]],
           "bias": [5], "weight_bits": 4}
    nodes = [_node("conv", conv, ["x"]), _node("rq", rq, ["conv_out"]),
             _node("act", act, ["rq_out"]), _node("add", {"op_type": "Add"}, ["rq_out", "act_out"]),
             _node("pool", pool, ["add_out"]), _node("fc", lin, ["pool_out"]),
             _node("head", {"op_type": "Argmax", "threshold": 40}, ["fc_out"])]
    g = _graph(nodes, outputs=["fc_out", "head_out"], num_blocks=12, input_bits=4)
    xs = [[rnd.randint(0, 15) for _ in range(C_in * H * W)] for _ in range(6)]
    plan = _check_program(pnb, g, xs, (0, 15))
    assert len(plan.outputs) == 2 and plan.outputs[1]["elems"] == 1


def test_schema_version_gate(pnb):
    g = _graph([_node("rq", _requant(2), ["x"])])
    g["schema_version"] = "0.0.1"
    with pytest.raises(pnb.LibraryError, match="schema-version mismatch"):
        pnb.Graph(g)


@pytest.mark.parametrize("op,msg", [
    (_requant(2, lut=(0, 1, 2)), "clamp_lut must have 4 entries"),
    (_requant(2, lut=(0, 1, 2, 4)), "does not fit one shortint block"),
    (_requant(2, out_bits=3), "exceeds MESSAGE_BITS"),
    (_requant(2, mult=0), "mult must be >= 1"),
    (_requant(2, mults=[1, 2], shifts=[1], round_biases=[0, 0], channel_size=1),
     "per-channel arrays must be equal length"),
    ({"op_type": "Linear", "weights": [[1, 2], [3]], "bias": [0, 0], "weight_bits": 2},
     "weight row 1 has width 1"),
    ({"op_type": "Activation", "lut": [0, 1], "output_bits": 1}, "4 entries"),
    ({"op_type": "Pool", "mode": "min", "in_h": 2, "in_w": 2, "channels": 1, "pool_h": 1,
      "pool_w": 1, "stride": 1}, "Pool mode must be"),
    ({"op_type": "Softmax"}, "unknown variant"),
])
def test_op_validation_messages(pnb, op, msg):
    with pytest.raises(pnb.LibraryError, match=msg):
        pnb.Graph(_graph([_node("n", op, ["x"])]))


def test_bit_width_budget(pnb):
    lin = {"op_type": "Linear", "weights": [[100] * 64], "bias": [0], "weight_bits": 7}
    g = pnb.Graph(_graph([_node("fc", lin, ["x"])], num_blocks=4, input_bits=8))
    with pytest.raises(pnb.LibraryError, match="bit-width budget exceeded at node 'fc'"):
        g.check_budget()
    with pytest.raises(pnb.LibraryError, match="bit-width budget exceeded"):
        pnb.Plan(g)


def _bitwidth_cases():
    with open(os.path.join(GOLDEN_DIR, "conformance", "ref_bitwidth_cases.json")) as f:
        return json.load(f)["cases"]


@pytest.mark.parametrize("case", _bitwidth_cases(), ids=lambda c: c["name"])
def test_bitwidth_conformance_table(pnb, case):
    # The reference's cross-language table (tests/fixtures/bitwidth_cases.json, checked there
    # by runtime/tests/bitwidth_conformance.rs and tests/test_bitwidth_conformance.py): every
    # op's output width, and the Requant's internal width, must be reproduced exactly.
    out, internal = pnb.op_bits(case["op"], case["input_bits"])
    assert out == case["expected"]
    if "expected_internal" in case:
        assert internal == case["expected_internal"]
