"""The whole DecisionModel::forward on the GPU (sj_fast_forward) against the reference.

DecisionModel::forward (src/model.cpp:309-536) adds the decision-model tail to
the encoder: type embedding, the head TransformerEncoderLayers, the scorer on
the marker rows and the act head.  Bars (written here, from the north-star
tolerances):
* fp32 mode: logits within 1e-4 of the reference (relative to max(1, |logit|)),
  act probabilities within 1e-5;
* bf16 mode: logits within 2e-2 max-abs, act probabilities within 5e-3
  max-abs, masked markers exactly -1e4.

References: the committed outputs of the reference's own forward
(tests/golden/encoder_ref.npz, tiny and C1, ragged padded batches) and, for the
C3 architecture, the C restatement's forward (oracle/).
"""
import os

import numpy as np
import pytest

pytest.importorskip("torch")

from oracle import oracle  # noqa: E402
from snapjudge_b200 import synth  # noqa: E402
from snapjudge_b200.fast import FastSnapjudge, SnapjudgeError  # noqa: E402

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "encoder_ref.npz")


@pytest.fixture(scope="module", autouse=True)
def _blas():
    oracle.set_blas()


def cases(E, name):
    ci = 0
    while f"{name}.{ci}.lengths" in E:
        yield {k.split(".", 2)[2]: E[k] for k in E.files if k.startswith(f"{name}.{ci}.")}
        ci += 1


def markers(rng, lengths, K):
    B = len(lengths)
    pos = np.zeros((B, K), np.int64)
    mm = np.zeros((B, K), np.uint8)
    for b in range(B):
        k = int(rng.integers(1, K + 1))
        pos[b, :k] = rng.integers(0, lengths[b], size=k)
        pos[b, k:] = rng.integers(-3, lengths[b] + 3, size=K - k)  # masked, some out of range
        mm[b, :k] = 1
    return pos, mm


@pytest.mark.parametrize("precision", ["fp32", "bf16"])
@pytest.mark.parametrize("name", ["tiny", "c1"])
def test_forward_matches_reference_goldens(name, precision):
    E = np.load(GOLD)
    spec = synth.SPECS[name]
    eng = FastSnapjudge(spec.cfg, synth.make_weights(spec), precision=precision)
    assert eng.n_act == spec.cfg.n_act
    for c in cases(E, name):
        pid, mask = synth.pad_batch(c["ids"], c["lengths"])
        logits, act = eng.forward(pid, mask, c["marker_pos"], c["marker_mask"], c["qtype"])
        want_l, want_a = c["logits"], c["act"]
        masked = c["marker_mask"] == 0
        assert (logits[masked] == -1e4).all()
        d = np.abs(logits - want_l)[~masked]
        if precision == "fp32":
            assert (d <= 1e-4 * np.maximum(1.0, np.abs(want_l[~masked]))).all(), d.max()
            assert np.abs(act - want_a).max() <= 1e-5
        else:
            assert d.max() <= 2e-2, d.max()
            assert np.abs(act - want_a).max() <= 5e-3


def test_forward_c3_architecture_vs_oracle():
    """C3 architecture (12 x 768, one head layer), 8 requests padded to 300 rows:
    2400 rows, so the head layers run on the CTA-pair tensor-core GEMMs."""
    spec = synth.SPECS["c3"]
    t = synth.make_weights(spec)
    rng = np.random.default_rng(11)
    lengths = np.minimum(synth.make_lengths(spec, batch=8, seed=31), 300)
    lengths[0] = 300
    ids = synth.make_ids(spec, lengths, seed=32)
    pid, mask = synth.pad_batch(ids, lengths)
    pos, mm = markers(rng, lengths, 6)
    qt = rng.integers(0, 3, size=len(lengths)).astype(np.int64)
    eng = FastSnapjudge(spec.cfg, t, precision="bf16")
    logits, act = eng.forward(pid, mask, pos, mm, qt)
    want_l, want_a = oracle.Oracle(spec.cfg, t).forward_padded(pid, mask, pos, mm, qt)
    live = mm == 1
    assert np.isfinite(logits).all() and np.isfinite(act).all()
    assert (logits[~live] == -1e4).all()
    assert np.abs(logits - want_l)[live].max() <= 2e-2
    assert np.abs(act - want_a).max() <= 5e-3
    # the same batch through two passes (max_tokens below the batch): identical
    eng2 = FastSnapjudge(spec.cfg, t, precision="bf16", max_tokens=1200)
    l2, a2 = eng2.forward(pid, mask, pos, mm, qt)
    assert np.abs(l2 - logits).max() <= 2e-2 and np.abs(a2 - act).max() <= 5e-3


@pytest.mark.parametrize("precision", ["fp32", "bf16"])
def test_forward_packed_equals_padded(precision):
    """Packing a padded batch to its valid rows (markers on valid rows) gives the
    outputs of computing the padding; a live marker on a padded row makes the
    padded computation necessary (and pack=None picks it)."""
    spec = synth.SPECS["c1"]
    t = synth.make_weights(spec)
    eng = FastSnapjudge(spec.cfg, t, precision=precision)
    lengths = np.array([32, 17, 1, 9])
    pid, mask = synth.pad_batch(synth.make_ids(spec, lengths, seed=5), lengths)
    rng = np.random.default_rng(6)
    pos, mm = markers(rng, lengths, 4)
    pos[mm == 0] = 0
    qt = rng.integers(0, 3, size=4).astype(np.int64)
    lp, ap = eng.forward(pid, mask, pos, mm, qt, pack=True)
    lf, af = eng.forward(pid, mask, pos, mm, qt, pack=False)
    assert np.abs(lp - lf).max() <= 1e-5 and np.abs(ap - af).max() <= 1e-5
    # a live marker on a padded row: only the padded computation matches the reference
    E = np.load(GOLD)
    c = next(c for c in cases(E, "c1") if len(c["lengths"]) == 4 and c["lengths"][1] == 17)
    pid, mask = synth.pad_batch(c["ids"], c["lengths"])
    pos, mm = c["marker_pos"].copy(), c["marker_mask"].copy()
    la, aa = eng.forward(pid, mask, pos, mm, c["qtype"])
    lb, ab = eng.forward(pid, mask, pos, mm, c["qtype"], pack=False)
    assert np.abs(la - lb).max() <= 1e-5 and np.abs(aa - ab).max() <= 1e-5
    pos[3, 0], mm[3, 0] = 20, 1  # row 3 has 9 valid rows
    lc, _ = eng.forward(pid, mask, pos, mm, c["qtype"])
    ld, _ = eng.forward(pid, mask, pos, mm, c["qtype"], pack=False)
    assert np.abs(lc - ld).max() <= 1e-5


def test_forward_errors():
    spec = synth.SPECS["c1"]
    t = synth.make_weights(spec)
    eng = FastSnapjudge(spec.cfg, t, precision="bf16")
    lengths = np.array([5, 3])
    pid, mask = synth.pad_batch(synth.make_ids(spec, lengths, seed=1), lengths)
    pos = np.zeros((2, 2), np.int64)
    mm = np.ones((2, 2), np.uint8)
    with pytest.raises(SnapjudgeError, match="qtype"):
        eng.forward(pid, mask, pos, mm, np.array([0, 3]))
    # an engine without the decision-model tensors cannot run forward
    enc_only = {k: v for k, v in t.items()
                if not k.startswith(("type_emb", "head.", "scorer.", "act_head."))}
    eng2 = FastSnapjudge(spec.cfg, enc_only, precision="bf16")
    assert eng2.n_act == 0
    with pytest.raises(SnapjudgeError, match="decision-model head"):
        eng2.forward(pid, mask, pos, mm, np.array([0, 1]))
