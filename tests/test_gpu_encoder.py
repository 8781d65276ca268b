"""Encoder-level parity on the GPU through the C ABI (FastSnapjudge).

Bars (written here):
* fp32 mode: hidden states within 1e-4 relative of the reference CPU forward
  (max |d| <= 1e-4 * max |want|); decision-head probabilities within 1e-5.
* bf16 mode: [CLS] decision logits within 2e-2 max-abs, probabilities within
  5e-3 max-abs, argmax labels identical; hidden states within 6e-2 max-abs.

The reference outputs are the committed goldens of the reference's own
DecisionModel::encode (tests/golden/encoder_ref.npz); larger configs use the
C restatement (oracle/) on a subset of the requests, GEMMs through OpenBLAS.
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


def logits_of(cls_hidden, tensors, heads):
    out = []
    x = np.asarray(cls_hidden, np.float64)
    for i, _ in enumerate(heads):
        out.append(x @ tensors[f"task_heads.{i}.weight"].astype(np.float64).T
                   + tensors[f"task_heads.{i}.bias"])
    return out


@pytest.mark.parametrize("name", ["tiny", "c1"])
def test_fp32_matches_reference_goldens(name):
    E = np.load(GOLD)
    spec = synth.SPECS[name]
    t = synth.make_weights(spec)
    eng = FastSnapjudge(spec.cfg, t, precision="fp32", heads=spec.heads)
    for c in cases(E, name):
        lengths, ids, want = c["lengths"], c["ids"], c["hidden"]
        pid, mask = synth.pad_batch(ids, lengths)
        got = eng.encode(pid, mask)  # reference padded semantics, padded rows included
        rel = np.abs(got - want).max() / np.abs(want).max()
        assert rel <= 1e-4, rel
        hp = eng.encode_packed(ids, lengths)
        cu = synth.cu_seqlens(lengths)
        for b in range(len(lengths)):
            d = np.abs(hp[cu[b]:cu[b + 1]] - want[b, :lengths[b]]).max()
            assert d <= 1e-4 * np.abs(want).max(), d
        probs = eng.decide(ids, lengths)
        wantp = oracle.task_heads(want[:, 0, :], t, spec.heads)
        np.testing.assert_allclose(probs, np.concatenate(wantp, axis=1), atol=1e-5, rtol=0)


@pytest.mark.parametrize("name", ["tiny", "c1"])
def test_bf16_small_configs(name):
    E = np.load(GOLD)
    spec = synth.SPECS[name]
    t = synth.make_weights(spec)
    eng = FastSnapjudge(spec.cfg, t, precision="bf16", heads=spec.heads)
    for c in cases(E, name):
        lengths, ids, want = c["lengths"], c["ids"], c["hidden"]
        hp = eng.encode_packed(ids, lengths)
        cu = synth.cu_seqlens(lengths)
        for b in range(len(lengths)):
            assert np.abs(hp[cu[b]:cu[b + 1]] - want[b, :lengths[b]]).max() <= 6e-2
        probs = eng.decide(ids, lengths)
        lg = logits_of(hp[cu[:-1]], t, spec.heads)
        lw = logits_of(want[:, 0, :], t, spec.heads)
        for a, b in zip(lg, lw):
            assert np.abs(a - b).max() <= 2e-2
        wantp = np.concatenate(oracle.task_heads(want[:, 0, :], t, spec.heads), axis=1)
        assert np.abs(probs - wantp).max() <= 5e-3
        assert (probs.argmax(1) == wantp.argmax(1)).all()


def _subset_check(spec, n_req, seed, max_len=None):
    t = synth.make_weights(spec)
    lengths = synth.make_lengths(spec, batch=n_req, seed=seed)
    if max_len:
        lengths = np.minimum(lengths, max_len)
    ids = synth.make_ids(spec, lengths, seed=seed + 1)
    eng = FastSnapjudge(spec.cfg, t, precision="bf16", heads=spec.heads)
    hp = eng.encode_packed(ids, lengths)
    probs = eng.decide(ids, lengths)
    orc = oracle.Oracle(spec.cfg, t)
    want = orc.encode_packed(ids, lengths)
    cu = synth.cu_seqlens(lengths)
    assert np.isfinite(hp).all()
    assert np.abs(hp - want).max() <= 6e-2
    lg = logits_of(hp[cu[:-1]], t, spec.heads)
    lw = logits_of(want[cu[:-1]], t, spec.heads)
    for a, b in zip(lg, lw):
        assert np.abs(a - b).max() <= 2e-2
    wantp = np.concatenate(oracle.task_heads(want[cu[:-1]], t, spec.heads), axis=1)
    assert np.abs(probs - wantp).max() <= 5e-3
    off = 0
    for h in spec.heads:
        if h.n_out > 1:
            assert (probs[:, off:off + h.n_out].argmax(1) == wantp[:, off:off + h.n_out].argmax(1)).all()
        off += h.n_out
    return eng, t, lengths, ids, hp


def test_c3_subset_vs_oracle():
    _subset_check(synth.SPECS["c3"], 6, 77)


def test_sliding_window_layers_at_scale():
    """ModernBERT's layer pattern on the C3 architecture: every third layer
    global, the others sliding (local_attention 128 -> |i - j| <= 64, RoPE
    theta of the sliding layers), on sequences up to 512 tokens (model.cpp:103-111)."""
    import dataclasses
    base = synth.SPECS["c3"]
    cfg = dataclasses.replace(
        base.cfg, local_attention=128,
        layer_types=["full_attention" if i % 3 == 0 else "sliding_attention"
                     for i in range(base.cfg.num_hidden_layers)])
    spec = dataclasses.replace(base, cfg=cfg)
    assert cfg.layer_window(1) == 64 and cfg.layer_window(0) == 0
    t = synth.make_weights(spec)
    lengths = np.array([512, 300, 129, 64, 1])
    ids = synth.make_ids(spec, lengths, seed=91)
    eng = FastSnapjudge(cfg, t, precision="bf16")
    got = eng.encode_packed(ids, lengths)
    want = oracle.Oracle(cfg, t).encode_packed(ids, lengths)
    assert np.isfinite(got).all()
    assert np.abs(got - want).max() <= 6e-2
    # the window changes the result (the oracle's windowed and full forwards
    # differ by 0.47 here): the same weights without sliding layers differ
    full = FastSnapjudge(base.cfg, t, precision="bf16").encode_packed(ids, lengths)
    assert np.abs(full - got)[:512].max() > 3 * 6e-2


def test_c5_subset_vs_oracle():
    _subset_check(synth.SPECS["c5"], 24, 78)


def test_c5_256_requests_vs_oracle():
    """Config 5's four heads (choice-3, choice-8, score-5, noul) on 256
    requests of its length distribution (lognormal(48, 0.8) in [4, 512]):
    hidden states, logits, probabilities and labels at the bf16 bars."""
    spec = synth.SPECS["c5"]
    _subset_check(spec, 256, spec.seed + 2000)


def test_c4_full_length_vs_oracle():
    """C4 at its full size per sequence: 24 layers x 1024, 16 heads, two
    sequences of 2048 tokens (the config's fixed length) against the C
    restatement, hidden states / logits / probabilities at the bf16 bars."""
    spec = synth.SPECS["c4"]
    eng, t, lengths, ids, hp = _subset_check(spec, 2, 79)
    assert (lengths == 2048).all()


def test_c3_full_batch_vs_oracle():
    """C3 at its full size: all 256 requests of the config's length
    distribution (lognormal(128, 0.6) in [8, 512]) in one packed batch against
    the C restatement, hidden states / logits / probabilities / labels at the
    bf16 bars."""
    spec = synth.SPECS["c3"]
    _subset_check(spec, spec.batch, spec.seed + 1000)


def test_c3_full_batch_properties():
    """Full C3 batch: finite, batch-invariant (packed batch == per-sequence), LN-shaped."""
    spec = synth.SPECS["c3"]
    t = synth.make_weights(spec)
    lengths = synth.make_lengths(spec)
    ids = synth.make_ids(spec, lengths)
    eng = FastSnapjudge(spec.cfg, t, precision="bf16", heads=spec.heads)
    hp = eng.encode_packed(ids, lengths)
    assert np.isfinite(hp).all()
    m = hp.mean(1)
    v = hp.var(1)
    assert np.abs(m).max() < 1e-3 and np.abs(v - 1).max() < 2e-3
    cu = synth.cu_seqlens(lengths)
    for b in (0, 100, 255):
        one = eng.encode_packed(ids[cu[b]:cu[b + 1]], lengths[b:b + 1])
        np.testing.assert_array_equal(one, hp[cu[b]:cu[b + 1]])
    # a run through several passes (small max_tokens) gives the same answer
    eng2 = FastSnapjudge(spec.cfg, t, precision="bf16", heads=spec.heads, max_tokens=4096)
    np.testing.assert_array_equal(eng2.decide(ids, lengths), eng.decide(ids, lengths))


def test_errors_are_reported():
    spec = synth.SPECS["c1"]
    t = synth.make_weights(spec)
    eng = FastSnapjudge(spec.cfg, t, precision="bf16", heads=spec.heads)
    with pytest.raises(SnapjudgeError, match="vocabulary"):
        eng.encode_packed(np.array([1, 2, 5000]), [3])
    with pytest.raises(SnapjudgeError, match="max_position_embeddings"):
        eng.encode_packed(np.zeros(9000, np.int64), [9000])
    with pytest.raises(SnapjudgeError, match="empty"):
        eng.decide(np.array([1, 2]), [2, 0])
    bad = dict(t)
    bad["encoder.layers.1.attn.Wo.weight"] = np.zeros((3, 3), np.float32)
    with pytest.raises(SnapjudgeError, match="architecture mismatch"):
        FastSnapjudge(spec.cfg, bad)
    del bad["encoder.layers.1.attn.Wo.weight"]
    with pytest.raises(SnapjudgeError, match="missing tensor"):
        FastSnapjudge(spec.cfg, bad)
    # the engine stays usable after errors
    assert np.isfinite(eng.encode_packed(np.array([1, 2, 3]), [3])).all()


def test_lora_adapter():
    spec = synth.SPECS["c1"]
    t = dict(synth.make_weights(spec))
    rng = np.random.default_rng(3)
    t["lora_A.weight"] = rng.standard_normal((4, 64), dtype=np.float32) * 0.1
    t["lora_B.weight"] = rng.standard_normal((64, 4), dtype=np.float32) * 0.1
    lengths = np.array([32, 17])
    ids = synth.make_ids(spec, lengths, seed=9)
    eng = FastSnapjudge(spec.cfg, t, precision="fp32", heads=spec.heads)
    got = eng.encode_packed(ids, lengths)
    want = oracle.Oracle(spec.cfg, t).encode_packed(ids, lengths)
    assert np.abs(got - want).max() <= 1e-4 * np.abs(want).max()
