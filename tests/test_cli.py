"""The command-line evaluator (penumbra-fhe_b200/pnb_eval): model + inputs files in, decrypted
outputs out, through the C ABI only."""
from __future__ import annotations

import json
import os
import subprocess

import pytest

from conftest import GOLDEN_DIR, PKG_DIR

CLI = os.path.join(PKG_DIR, "pnb_eval")


def _run(args):
    if not os.path.exists(CLI):
        pytest.fail(f"{CLI} is not built (make -C {PKG_DIR})")
    out = subprocess.run([CLI] + args, capture_output=True, text=True, timeout=600)
    return out


@pytest.mark.parametrize("name", ["cfg1_tiny_cnn", "ref_phase4_cnn_fixture", "cfg4_mlp"])
def test_cli_simulate_matches_golden(name):
    path = os.path.join(GOLDEN_DIR, name + ".json")
    r = _run([path, path, "--simulate"])
    assert r.returncode == 0, r.stderr
    want = [o if isinstance(o, list) else [o] for o in json.load(open(path))["outputs"]]
    assert json.loads(r.stdout)["outputs"] == want


def test_cli_reports_graph_errors(tmp_path):
    bad = tmp_path / "bad.fhe"
    bad.write_text(json.dumps({"schema_version": "0.0.1", "num_blocks": 4, "input_bits": 4,
                               "inputs": ["x"], "outputs": ["y"], "nodes": []}))
    r = _run([str(bad), str(bad), "--simulate"])
    assert r.returncode != 0 and "schema-version mismatch" in r.stderr


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["cfg1_tiny_cnn", "ref_phase2_fixture"])
def test_cli_encrypted_matches_golden(name):
    path = os.path.join(GOLDEN_DIR, name + ".json")
    r = _run([path, path, "--seed", "9"])
    assert r.returncode == 0, r.stderr
    want = [o if isinstance(o, list) else [o] for o in json.load(open(path))["outputs"]]
    assert json.loads(r.stdout)["outputs"] == want
