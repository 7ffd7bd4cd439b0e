"""One-op programs (pnb_op_plan_create) on the CPU: the reference's golden Requant sweeps
compiled for inputs that arrive from an earlier op (a pinned scale and noise), executed
noise-free, and the planner's refusals when a pinned encoding cannot hold an op exactly."""
from __future__ import annotations

import numpy as np
import pytest

import ir_eval

# (op payload, inputs) of runtime/tests/golden_requant.rs, golden_requant_mult.rs and
# golden_requant_per_channel.rs
SWEEPS = {
    "requant_shift": ({"op_type": "Requant", "shift": 4, "mult": 1, "round_bias": 0,
                       "out_bits": 2, "clamp_lut": [0, 1, 2, 3]},
                      [-100, 0, 16, 47, 64, 1000, -1, 31, 48]),
    "requant_mult": ({"op_type": "Requant", "shift": 5, "mult": 3, "round_bias": 16,
                      "out_bits": 2, "clamp_lut": [0, 1, 2, 3]},
                     [-100, -1, 0, 1, 7, 16, 31, 47, 63, 64, 200, 511]),
    "requant_per_channel": ({"op_type": "Requant", "shift": 0, "mults": [1, 3],
                             "shifts": [4, 5], "round_biases": [0, 16], "channel_size": 3,
                             "out_bits": 2, "clamp_lut": [0, 1, 2, 3]},
                            [-100, 63, 511, -1, 47, 200]),
}


def _expect(op, xs):
    g = {"inputs": ["x"], "outputs": ["y"], "nodes": [{"inputs": ["x"], "outputs": ["y"], "op": op}]}
    return ir_eval.evaluate(g, {"x": list(xs)})["y"]


@pytest.mark.parametrize("name", sorted(SWEEPS))
@pytest.mark.parametrize("scale,sigma", [(0, 0.0), (44, 30.0), (40, 24.0)])
def test_one_op_requant_sweep(pnb, name, scale, sigma):
    op, xs = SWEEPS[name]
    d = pnb.TensorDesc.make(len(xs), -1024, 1023, scale, sigma)
    pl = pnb.op_plan(op, [d])
    y, margin = pl.simulate(np.array([xs], dtype=np.int64))
    assert y[0].tolist() == _expect(op, xs)
    assert margin >= 63.5
    din = pl.desc(False)
    assert din.scale_log2 == (scale or din.scale_log2) and din.elems == len(xs)
    dout = pl.desc(True)
    assert (dout.lo, dout.hi) == (0, 3)


def test_one_op_output_scale_is_pinned(pnb):
    op, xs = SWEEPS["requant_mult"]
    pl = pnb.op_plan(op, [pnb.TensorDesc.make(len(xs), -1024, 1023, 44, 30.0)], out_scale=55)
    assert pl.desc(True).scale_log2 == 55
    y, _ = pl.simulate(np.array([xs], dtype=np.int64))
    assert y[0].tolist() == _expect(op, xs)


def test_one_op_add_and_argmax(pnb):
    # runtime/tests/golden_add.rs: a = [3, -5], b = [4, 6]
    d = pnb.TensorDesc.make(2, -8, 8, 50, 30.0)
    pl = pnb.op_plan({"op_type": "Add"}, [d, d])
    y, _ = pl.simulate(np.array([[3, -5, 4, 6]], dtype=np.int64))
    assert y[0].tolist() == [7, 1]
    pl = pnb.op_plan({"op_type": "Argmax", "threshold": 5},
                     [pnb.TensorDesc.make(1, -300, 300, 45, 28.0)])
    y, margin = pl.simulate(np.array([[-300], [4], [5], [300]], dtype=np.int64))
    assert y[:, 0].tolist() == [0, 0, 1, 1] and margin >= 63.5


def test_one_op_refusals(pnb):
    op, xs = SWEEPS["requant_mult"]
    # a 2^60 scale leaves no room for values up to 1023
    with pytest.raises(pnb.LibraryError, match="leaves no room"):
        pnb.op_plan(op, [pnb.TensorDesc.make(len(xs), -1024, 1023, 60, 30.0)])
    # noise as large as the scale: no exact threshold decision exists
    with pytest.raises(pnb.LibraryError):
        pnb.op_plan(op, [pnb.TensorDesc.make(len(xs), -1024, 1023, 40, 41.0)])
    # Add operands pinned at different scales
    with pytest.raises(pnb.LibraryError, match="meet where one encoding"):
        pnb.op_plan({"op_type": "Add"}, [pnb.TensorDesc.make(2, -8, 8, 50, 30.0),
                                         pnb.TensorDesc.make(2, -8, 8, 49, 30.0)])
    # the reference's own validation message
    with pytest.raises(pnb.LibraryError, match="clamp_lut must have 4 entries"):
        pnb.op_plan(dict(op, out_bits=3, clamp_lut=list(range(8))),
                    [pnb.TensorDesc.make(len(xs), -1024, 1023)])
