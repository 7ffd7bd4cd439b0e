"""Encrypted graph evaluation on the GPU: decrypted outputs equal the reference's integers.

Every golden fixture (graph, inputs and outputs produced by the reference quantizer and integer
evaluator) is encrypted, evaluated through ``pnb_evaluate`` and decrypted; the result must be
bit-exact.  This is the golden invariant of ``runtime/src/lib.rs:12-16`` checked on the
configurations' own graphs.
"""
from __future__ import annotations

import json
import os
import random

import numpy as np
import pytest
import torch

import ir_eval
from conftest import GOLDEN_DIR

pytestmark = pytest.mark.gpu


def _flat(o):
    return o if isinstance(o, list) else [o]


@pytest.mark.parametrize("name", ["ref_phase2_fixture", "ref_phase4_cnn_fixture",
                                  "cfg1_tiny_cnn", "cfg4_mlp", "cfg5_cnn",
                                  # the models the reference's golden tests skip as too slow
                                  "ref_phase5_digits_fixture", "ref_phase5_qat_fixture",
                                  "ref_phase6_onnx_fixture", "ref_phase6_sklearn_fixture",
                                  "ref_phase7_faces_fixture"])
def test_golden_graph_decrypts_exactly(pnb, name):
    with open(os.path.join(GOLDEN_DIR, name + ".json")) as f:
        d = json.load(f)
    plan = pnb.Plan(pnb.Graph(d["graph"]))
    ev = pnb.Evaluator(plan, device=0, seed=21)
    x = np.array(d["inputs"], dtype=np.int64)
    ct = ev.encrypt(x, seed=5)
    out = ev.evaluate(ct)
    got = ev.decrypt(out).cpu().numpy()
    want = np.array([_flat(o) for o in d["outputs"]], dtype=np.int64)
    assert np.array_equal(got, want), (got, want)
    assert pnb.device_status(0) == 0


def test_mixed_graph_and_chunking(pnb):
    rnd = random.Random(9)
    C_in, H, W, C_out = 1, 5, 5, 2
    conv = {"op_type": "Conv2d", "weights": [[rnd.randint(-20, 20) for _ in range(9)]
                                             for _ in range(C_out)],
            "bias": [3, -7], "weight_bits": 6, "in_h": H, "in_w": W, "in_channels": C_in,
            "kernel_h": 3, "kernel_w": 3, "stride": 1, "padding": 1}
    rq = {"op_type": "Requant", "shift": 0, "mult": 1, "round_bias": 0, "out_bits": 2,
          "clamp_lut": [0, 2, 1, 3], "mults": [7, 3], "shifts": [7, 6],
          "round_biases": [64, 0], "channel_size": H * W}
    act = {"op_type": "Activation", "lut": [1, 3, 0, 2], "output_bits": 2}
    lin = {"op_type": "Linear", "weights": [[rnd.randint(-9, 9) for _ in range(C_out * H * W)]],
           "bias": [5], "weight_bits": 4}
    g = {"schema_version": "0.6.0", "num_blocks": 12, "input_bits": 4, "inputs": ["x"],
         "outputs": ["fc_out", "head_out"], "nodes": [
             {"name": "conv", "inputs": ["x"], "outputs": ["conv_out"], "op": conv},
             {"name": "rq", "inputs": ["conv_out"], "outputs": ["rq_out"], "op": rq},
             {"name": "act", "inputs": ["rq_out"], "outputs": ["act_out"], "op": act},
             {"name": "add", "inputs": ["rq_out", "act_out"], "outputs": ["add_out"],
              "op": {"op_type": "Add"}},
             {"name": "fc", "inputs": ["add_out"], "outputs": ["fc_out"], "op": lin},
             {"name": "head", "inputs": ["fc_out"], "outputs": ["head_out"],
              "op": {"op_type": "Argmax", "threshold": 10}}]}
    plan = pnb.Plan(pnb.Graph(g), input_range=(0, 15))
    # a small memory budget forces several chunks per call
    per_sample = 0
    ev = pnb.Evaluator(plan, device=0, seed=4, max_bytes=64 << 20)
    xs = [[rnd.randint(0, 15) for _ in range(H * W)] for _ in range(7)]
    got = ev.decrypt(ev.evaluate(ev.encrypt(xs, seed=3))).cpu().numpy()
    for x, row in zip(xs, got):
        r = ir_eval.evaluate(g, {"x": x})
        assert row.tolist() == r["fc_out"] + r["head_out"]
    assert pnb.device_status(0) == 0
    del per_sample
