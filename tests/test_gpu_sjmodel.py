"""SjModel (reference src/sj_model.cpp) on the GPU engine (SJ_ARCH_SJMODEL).

SjModel is the reference's second encoder family: a BERT-style pre-LN encoder
with learned positions, separate biased q/k/v/o projections, biased LNs and a
GELU FFN (sj_model.cpp:206-255), plus its forward tail (type embedding, head
layers, scorer, act = [top1, 1 - top1], :277-368).  Bars, as for the
DecisionModel encoder:
* fp32 mode: hidden states within 1e-4 relative, logits within 1e-4 of
  max(1, |logit|), act within 1e-5;
* bf16 mode: hidden states within 6e-2 max-abs, logits 2e-2, act 5e-3.

References: the committed outputs of the reference's own SjModel
(tests/golden/sjmodel_ref.npz, sj_tiny) and, at the C3 width, the reference
compiled from its sources (oracle/_ref, OpenBLAS).
"""
import os
import tempfile

import numpy as np
import pytest

pytest.importorskip("torch")

from oracle import oracle  # noqa: E402
from snapjudge_b200 import synth  # noqa: E402
from snapjudge_b200.checkpoint import save_sj_checkpoint  # noqa: E402
from snapjudge_b200.fast import FastSnapjudge, SnapjudgeError  # noqa: E402

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "sjmodel_ref.npz")


@pytest.fixture(scope="module", autouse=True)
def _blas():
    oracle.set_blas()


def cases(E):
    ci = 0
    while f"sj_tiny.{ci}.lengths" in E:
        yield {k.split(".", 2)[2]: E[k] for k in E.files if k.startswith(f"sj_tiny.{ci}.")}
        ci += 1


@pytest.mark.parametrize("precision", ["fp32", "bf16"])
def test_sjmodel_matches_reference_goldens(precision):
    E = np.load(GOLD)
    cfg, seed = synth.SJ_SPECS["sj_tiny"]
    eng = FastSnapjudge(cfg, synth.make_sj_weights(cfg, seed), precision=precision)
    assert eng.n_act == 2
    n = 0
    for c in cases(E):
        pid, mask = synth.pad_batch(c["ids"], c["lengths"])
        h = eng.encode(pid, mask)
        want = c["hidden"]
        if precision == "fp32":
            assert np.abs(h - want).max() <= 1e-4 * np.abs(want).max()
        else:
            assert np.abs(h - want).max() <= 6e-2
        lg, act = eng.forward(pid, mask, c["marker_pos"], c["marker_mask"], c["qtype"])
        live = c["marker_mask"] != 0
        assert (lg[~live] == -1e4).all()
        d = np.abs(lg - c["logits"])[live]
        if precision == "fp32":
            assert (d <= 1e-4 * np.maximum(1.0, np.abs(c["logits"][live]))).all()
            assert np.abs(act - c["act"]).max() <= 1e-5
        else:
            assert d.max() <= 2e-2 and np.abs(act - c["act"]).max() <= 5e-3
        n += 1
    assert n == 3


def test_sjmodel_base_width_vs_reference():
    """12 x 768 SjModel, 8 requests padded to 300 rows (2400 rows): the biased
    QKV, GELU-FFN and residual epilogues on the tensor cores, against the
    reference compiled from its sources."""
    cfg, seed = synth.SJ_SPECS["sj_base"]
    t = synth.make_sj_weights(cfg, seed)
    rng = np.random.default_rng(41)
    lengths = np.array([300, 251, 177, 128, 96, 64, 17, 1])
    ids = rng.integers(0, cfg.vocab_size, size=int(lengths.sum())).astype(np.int64)
    pid, mask = synth.pad_batch(ids, lengths)
    K = 5
    pos = np.zeros((8, K), np.int64)
    mm = np.zeros((8, K), np.uint8)
    for b, n in enumerate(lengths):
        k = int(rng.integers(1, K + 1))
        pos[b, :k] = rng.integers(0, n, size=k)
        mm[b, :k] = 1
    qt = rng.integers(0, cfg.n_types, size=8).astype(np.int64)
    eng = FastSnapjudge(cfg, t, precision="bf16")
    h = eng.encode(pid, mask)
    lg, act = eng.forward(pid, mask, pos, mm, qt)
    with tempfile.TemporaryDirectory() as d:
        save_sj_checkpoint(d, cfg, t)
        ref = oracle.RefSjModel(d, cfg.hidden_size)
        want_h = ref.encode(pid, mask)
        want_l, want_a = ref.forward(pid, mask, pos, mm, qt)
    valid = mask.astype(bool)
    assert np.isfinite(h).all()
    assert np.abs(h - want_h)[valid].max() <= 6e-2
    assert np.abs(lg - want_l)[mm == 1].max() <= 2e-2
    assert np.abs(act - want_a).max() <= 5e-3


def test_sjmodel_positions_clamp_past_the_table():
    """Rows past max_positions take the table's last row (sj_model.cpp:228-230)."""
    cfg, seed = synth.SJ_SPECS["sj_tiny"]
    t = synth.make_sj_weights(cfg, seed)
    lengths = np.array([cfg.max_positions + 9, 5])
    ids = np.random.default_rng(3).integers(0, cfg.vocab_size, size=int(lengths.sum()))
    pid, mask = synth.pad_batch(ids, lengths)
    eng = FastSnapjudge(cfg, t, precision="fp32")
    got = eng.encode(pid, mask)
    want = oracle.SjOracle(cfg, t).encode_padded(pid, mask)
    assert np.abs(got - want).max() <= 1e-4 * np.abs(want).max()


def test_sjmodel_errors():
    cfg, seed = synth.SJ_SPECS["sj_tiny"]
    t = synth.make_sj_weights(cfg, seed)
    bad = dict(t)
    bad["sj.encoder.layers.1.attn.k.weight"] = bad["sj.encoder.layers.1.attn.k.weight"][:, :-1]
    with pytest.raises(SnapjudgeError, match="attn.k.weight"):
        FastSnapjudge(cfg, bad, precision="fp32")
    eng = FastSnapjudge(cfg, t, precision="fp32")
    pid, mask = synth.pad_batch(np.arange(6), np.array([4, 2]))
    with pytest.raises(SnapjudgeError, match="qtype"):
        eng.forward(pid, mask, np.zeros((2, 1), np.int64), np.ones((2, 1), np.uint8),
                    np.array([0, cfg.n_types]))
