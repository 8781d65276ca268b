"""Drop-in check: the reference's own DecisionModel::forward (CPU fp32) against
snapjudge::FastSnapjudge::forward built from snapjudge_b200/integration/fast.cpp
(encoder on the GPU through the C ABI), inside one binary linked from the
reference sources (oracle/_ref/adapter_check, built by oracle/Makefile).
Bar: logits within 2e-2 max-abs, act probabilities within 5e-3 (bf16 mode)."""
import json
import os
import subprocess

import pytest

from snapjudge_b200 import synth
from snapjudge_b200.checkpoint import save_checkpoint

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "oracle", "_ref", "adapter_check")


@pytest.mark.skipif(not os.path.exists(BIN), reason="oracle/_ref/adapter_check not built")
@pytest.mark.parametrize("name", ["tiny", "c1"])
def test_fast_snapjudge_matches_decision_model(name, tmp_path):
    spec = synth.SPECS[name]
    save_checkpoint(str(tmp_path), spec.cfg, synth.make_weights(spec))
    r = subprocess.run([BIN, str(tmp_path)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    d = json.loads(r.stdout.strip().splitlines()[-1])
    assert d["logits_max_abs"] <= 2e-2 and d["act_max_abs"] <= 5e-3, d
