"""The reference's own tiny checkpoint and runtime through the GPU path.

The reference pins its runtime with a tiny fp16 checkpoint fixture
(tests/fixtures/tiny-ckpt: D=16, 2 heads of 8, a sliding layer, one head
layer) and the golden answer of Agent::system_one on it
(tests/golden/model_tiny.json, checked by tests/test_model.cpp:29-45).
oracle/Makefile copies both into oracle/_ref/ and builds, from the
reference's sources, oracle/_ref/agent_check: the reference Agent and C API
with the fast-path dispatch a maintainer adds (a FastSnapjudge built once the
device resolves to "cuda", called in place of DecisionModel::forward), linked
with this repository's FastSnapjudge adapter.  Checked here:

* Agent(ckpt, "cuda").system_one — the whole DecisionModel::forward of every
  question on the GPU — equals the golden in fp32 mode (numbers to the
  golden's 4 decimals) and matches it within the bf16 probability bar (5e-3)
  in bf16 mode; sj_predict with {"device": "cuda"} (tests/capi/test_capi.c's
  call) answers like the CPU engine;
* FastSnapjudge::forward against DecisionModel::forward on the fixture
  (oracle/_ref/adapter_check, ragged padded batch);
* the Python loader on the fp16 safetensors: fp32-mode encoder states within
  1e-4 relative of the reference's compiled DecisionModel::encode.
"""
import json
import os
import subprocess

import numpy as np
import pytest

pytest.importorskip("torch")

from oracle import oracle  # noqa: E402
from snapjudge_b200.fast import FastSnapjudge  # noqa: E402

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "oracle", "_ref")
CKPT = os.path.join(REF, "tiny-ckpt")
AGENT = os.path.join(REF, "agent_check")
ADAPTER = os.path.join(REF, "adapter_check")
need = pytest.mark.skipif(not (os.path.exists(AGENT) and os.path.isdir(CKPT)),
                          reason="oracle/_ref/agent_check or the tiny fixture not built")


def _run(precision, tol):
    env = dict(os.environ, SNAPJUDGE_FAST_PRECISION=precision, AGENT_CHECK_TOL=str(tol))
    r = subprocess.run([AGENT, CKPT, os.path.join(REF, "model_tiny.json")], capture_output=True,
                       text=True, timeout=300, env=env)
    d = json.loads(r.stdout.strip().splitlines()[-1])
    return r.returncode, d, r.stderr


@need
def test_agent_system_one_fp32_equals_golden():
    rc, d, err = _run("fp32", 0.0)
    assert d["cpu_equals_golden"], d
    assert d["accelerated"], err
    assert d["agent_mismatch"] == "" and d["ties_accepted"] == 0, d
    assert d["capi_ok"], d
    assert rc == 0, (d, err)


@need
def test_agent_system_one_bf16_within_bars():
    rc, d, err = _run("bf16", 5e-3)
    assert d["accelerated"], err
    assert d["agent_mismatch"] == "" and d["agent_max_diff"] <= 5e-3, d
    assert d["capi_ok"] and d["capi_max_diff"] <= 5e-3, d
    assert rc == 0, (d, err)


@pytest.mark.skipif(not (os.path.exists(ADAPTER) and os.path.isdir(CKPT)),
                    reason="oracle/_ref/adapter_check or the tiny fixture not built")
def test_adapter_on_reference_fixture():
    r = subprocess.run([ADAPTER, CKPT], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    d = json.loads(r.stdout.strip().splitlines()[-1])
    assert d["logits_max_abs"] <= 2e-2 and d["act_max_abs"] <= 5e-3, d


@pytest.mark.skipif(not (os.path.isdir(CKPT) and oracle.ref_available()),
                    reason="the tiny fixture or oracle/_ref/libsjref.so not built")
def test_python_loader_on_fp16_fixture():
    eng = FastSnapjudge.from_checkpoint(CKPT, precision="fp32")
    ref = oracle.RefModel(CKPT)
    D = eng.D
    rng = np.random.default_rng(5)
    V = eng.cfg.vocab_size
    lengths = [37, 5, 1, 20]
    L = max(lengths)
    ids = np.zeros((len(lengths), L), np.int64)
    mask = np.zeros((len(lengths), L), np.int64)
    for b, n in enumerate(lengths):
        ids[b, :n] = rng.integers(0, V, n)
        mask[b, :n] = 1
    want = ref.encode(ids, mask, D)
    got = eng.encode(ids, mask)
    assert np.abs(got - want).max() <= 1e-4 * np.abs(want).max()
