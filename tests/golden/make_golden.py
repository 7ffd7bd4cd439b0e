"""Generate the committed golden fixtures from the reference's own Python code.

Run with the path of a reference checkout (Harikeshav-R/Penumbra-FHE) as the argument:

    python tests/golden/make_golden.py REF

For every benchmark configuration it builds the model with the reference quantizer
(``python/penumbra/model.py`` ``Model.quantize``) on seeded synthetic data, quantizes seeded
inputs with the reference input spec, runs the reference integer oracle
(``python/penumbra/reference.py`` ``evaluate_graph_int``) and writes the IR graph, the
quantized inputs and every intermediate tensor to ``tests/golden/<name>.json``.  It also
re-evaluates the reference's committed fixtures (``examples/mnist/phase2_fixture.json``,
``phase4_cnn_fixture.json``, and the heavy models its golden tests skip: ``phase5_digits``,
``phase5_qat``, ``phase6_onnx``, ``phase6_sklearn``, ``examples/faces/phase7_faces``) and checks
the oracle against their ``expected_*`` values.

Only this script reads the reference; tests and the GPU box read the JSON it writes.

The MLP and CNN graphs need a quantizer workaround: the reference's ``insert_requants``
(``python/penumbra/compile.py:184``) sizes requantized accumulators from the un-requantized
graph and rejects them at the final radix; requants are inserted at the 64-block probe width
and the graph is then given the minimal width computed on the requantized graph (the
reference's own ``Model._minimal_num_blocks``, ``python/penumbra/model.py:354-369``).
"""
from __future__ import annotations

import dataclasses
import json
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
if len(sys.argv) != 2:
    sys.exit("usage: python tests/golden/make_golden.py <path of a reference checkout>")
REF = sys.argv[1]


def _import_reference():
    # The reference package imports its ONNX loader at import time; onnx is not installed here
    # and not needed for these graphs, so register an empty stand-in module.
    if "onnx" not in sys.modules:
        onnx = types.ModuleType("onnx")
        onnx.numpy_helper = types.ModuleType("onnx.numpy_helper")
        sys.modules["onnx"] = onnx
        sys.modules["onnx.numpy_helper"] = onnx.numpy_helper
    sys.path.insert(0, os.path.join(REF, "python"))
    import penumbra
    import penumbra.model as model_mod

    orig = model_mod.insert_requants

    def insert_requants_probe_width(graph, **kw):
        if graph.num_blocks == 64:
            return orig(graph, **kw)
        wide = orig(dataclasses.replace(graph, num_blocks=64), **kw)
        return dataclasses.replace(wide, num_blocks=graph.num_blocks)

    model_mod.insert_requants = insert_requants_probe_width
    return penumbra


def _relu(v):
    return max(v, 0.0)


def _run(P, name, layers, input_bits, calib, n_bits, samples, note):
    from penumbra.quantization.spec import symmetric_spec
    m = P.Model(layers, input_bits=input_bits)
    g = m.quantize(calib, n_bits=n_bits)
    spec = symmetric_spec(calib, input_bits, signed=False)
    xs = [spec.quantize(row).astype(int).tolist() for row in samples]
    # every intermediate tensor: make each node's output a graph output
    tensors = []
    for x in xs:
        env = {}
        for node in g.nodes:
            sub = dataclasses.replace(g, outputs=[node.outputs[0]])
            env[node.outputs[0]] = P.evaluate_graph_int(sub, {"x": x})[node.outputs[0]]
        out = P.evaluate_graph_int(g, {"x": x})
        assert out[g.outputs[0]] == env[g.outputs[0]]
        tensors.append(env)
    doc = {
        "_comment": note,
        "graph": json.loads(g.to_json()),
        "inputs": xs,
        "tensors": tensors,
        "outputs": [t[g.outputs[0]] for t in tensors],
    }
    path = os.path.join(HERE, f"{name}.json")
    with open(path, "w") as f:
        json.dump(doc, f, separators=(",", ":"))
    print(f"{name}: num_blocks={g.num_blocks} nodes={[n.op.op_type for n in g.nodes]} "
          f"-> {os.path.relpath(path)} ({os.path.getsize(path)} bytes)")
    return g


def main():
    P = _import_reference()
    from penumbra.layers import Activation, Conv2d, Linear, Pool

    # Config 1: tiny CNN (the reference README model), PTQ n_bits=4, 1 sample.
    rng = np.random.default_rng(0)
    w1 = rng.normal(0, 0.5, (4, 1, 3, 3))
    w2 = rng.normal(0, 0.5, (10, 36))
    b2 = rng.normal(0, 0.5, 10)
    calib = rng.random((64, 64))
    _run(P, "cfg1_tiny_cnn",
         [Conv2d(weight=w1, in_h=8, in_w=8, in_channels=1, stride=2), Activation(_relu),
          Linear(weight=w2, bias=b2)],
         4, calib, 4, rng.random((4, 64)),
         "Tiny CNN: Conv2d 1->4 3x3 s2 on 8x8, fused ReLU+Requant, Linear 36->10. Weights "
         "N(0,0.5) seed 0, PTQ n_bits=4 on 64 U[0,1) samples; reference quantizer + oracle.")

    # Config 4: MLP 784-128-128-10, PTQ n_bits=6 on 256 U[0,1) samples.
    rng = np.random.default_rng(4)
    ws = [rng.normal(0, np.sqrt(1 / 784), (128, 784)), rng.normal(0, np.sqrt(1 / 128), (128, 128)),
          rng.normal(0, np.sqrt(1 / 128), (10, 128))]
    calib = rng.random((256, 784))
    _run(P, "cfg4_mlp",
         [Linear(weight=ws[0], bias=np.zeros(128)), Activation(_relu),
          Linear(weight=ws[1], bias=np.zeros(128)), Activation(_relu),
          Linear(weight=ws[2], bias=np.zeros(10))],
         6, calib, 6, rng.random((4, 784)),
         "MLP 784-128-128-10 with ReLU, weights N(0,1/fan_in) seed 4, PTQ n_bits=6 on 256 "
         "U[0,1) samples (requants inserted at the probe width, then the minimal width).")

    # Config 5: small CNN on 1x28x28, PTQ n_bits=6.
    rng = np.random.default_rng(5)
    c1 = rng.normal(0, np.sqrt(1 / 9), (8, 1, 3, 3))
    c2 = rng.normal(0, np.sqrt(1 / 72), (16, 8, 3, 3))
    fc = rng.normal(0, np.sqrt(1 / 576), (10, 576))
    calib = rng.random((64, 784))
    _run(P, "cfg5_cnn",
         [Conv2d(weight=c1, in_h=28, in_w=28, in_channels=1, stride=1), Activation(_relu),
          Pool(mode="avg", in_h=26, in_w=26, channels=8, pool_h=2, pool_w=2, stride=2),
          Conv2d(weight=c2, in_h=13, in_w=13, in_channels=8, stride=2), Activation(_relu),
          Linear(weight=fc, bias=np.zeros(10))],
         6, calib, 6, rng.random((2, 784)),
         "CNN 1x28x28: Conv 8ch 3x3 s1, ReLU, avg-pool 2x2, Conv 16ch 3x3 s2, ReLU, Linear "
         "576->10; weights N(0,1/fan_in) seed 5, PTQ n_bits=6 (probe-width requant workaround).")

    # The reference's committed fixtures: re-evaluate and check their expected values.
    for fx, key in (("examples/mnist/phase4_cnn_fixture.json", "expected_logits"),
                    ("examples/mnist/phase2_fixture.json", "expected_labels"),
                    # the models the reference's own golden tests skip as minutes per sample
                    ("examples/mnist/phase5_digits_fixture.json", "expected_logits"),
                    ("examples/mnist/phase5_qat_fixture.json", "expected_logits"),
                    ("examples/mnist/phase6_onnx_fixture.json", "expected_logits"),
                    ("examples/mnist/phase6_sklearn_fixture.json", "expected_logits"),
                    ("examples/faces/phase7_faces_fixture.json", "expected_logits")):
        d = json.load(open(os.path.join(REF, fx)))
        g = P.ir.Graph.from_json(json.dumps(d["graph"]))
        outs = [P.evaluate_graph_int(g, {"x": x})[g.outputs[0]] for x in d["test_inputs"]]
        exp = d[key]
        flat = [o if len(o) > 1 else o[0] for o in outs]
        assert flat == exp, f"{fx}: oracle {flat} != fixture {exp}"
        name = os.path.splitext(os.path.basename(fx))[0]
        # the logistic-regression head: keep the pre-Argmax logit as a tensor for the GPU path
        tensors = []
        for x in d["test_inputs"]:
            env = {}
            for node in g.nodes:
                sub = dataclasses.replace(g, outputs=[node.outputs[0]])
                env[node.outputs[0]] = P.evaluate_graph_int(sub, {"x": x})[node.outputs[0]]
            tensors.append(env)
        doc = {"_comment": f"Reference fixture {fx}: graph and test inputs as committed there, "
                           f"every tensor re-evaluated by the reference oracle; {key} checked.",
               "graph": d["graph"], "inputs": d["test_inputs"], "tensors": tensors,
               "outputs": outs}
        path = os.path.join(HERE, f"ref_{name}.json")
        with open(path, "w") as f:
            json.dump(doc, f, separators=(",", ":"))
        print(f"ref_{name}: {len(outs)} samples, {key} reproduced -> {os.path.relpath(path)}")


def copy_bitwidth_cases():
    """The reference's cross-language bit-width conformance table (tests/fixtures/
    bitwidth_cases.json), copied unchanged for tests/test_graph_cpu.py."""
    src = os.path.join(REF, "tests", "fixtures", "bitwidth_cases.json")
    dst_dir = os.path.join(HERE, "conformance")
    os.makedirs(dst_dir, exist_ok=True)
    with open(src) as f:
        doc = json.load(f)
    with open(os.path.join(dst_dir, "ref_bitwidth_cases.json"), "w") as f:
        json.dump(doc, f, indent=1)
    print(f"ref_bitwidth_cases: {len(doc['cases'])} cases")


if __name__ == "__main__":
    main()
    copy_bitwidth_cases()
