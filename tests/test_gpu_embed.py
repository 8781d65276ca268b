"""Mean-pooled embeddings on the GPU (sj_fast_embed) against the reference.

Agent::embed (src/agent.cpp:315-357) encodes a right-padded batch and averages
each row's final hidden states over its valid positions (fp32, position
order).  Bars:
* against the GPU's own final hidden states: bit-exact (same values, same
  summation order and the same IEEE division);
* against the reference's hidden states (tests/golden/encoder_ref.npz):
  fp32 mode within 1e-4 relative, bf16 mode within 6e-2 max-abs (the hidden
  states' bar; a mean of rows does not widen it).
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


def cases(E, name):
    ci = 0
    while f"{name}.{ci}.lengths" in E:
        yield {k.split(".", 2)[2]: E[k] for k in E.files if k.startswith(f"{name}.{ci}.")}
        ci += 1


@pytest.mark.parametrize("precision", ["fp32", "bf16"])
@pytest.mark.parametrize("name", ["tiny", "c1"])
def test_embed_matches_reference_hidden_states(name, precision):
    E = np.load(GOLD)
    spec = synth.SPECS[name]
    eng = FastSnapjudge(spec.cfg, synth.make_weights(spec), precision=precision)
    n = 0
    for c in cases(E, name):
        pid, mask = synth.pad_batch(c["ids"], c["lengths"])
        got = eng.embed(pid, mask)
        want = oracle.embed_mean(c["hidden"], mask)
        assert got.shape == (len(c["lengths"]), spec.cfg.hidden_size)
        if precision == "fp32":
            assert np.abs(got - want).max() <= 1e-4 * np.abs(want).max()
        else:
            assert np.abs(got - want).max() <= 6e-2
        n += 1
    assert n >= 1


@pytest.mark.parametrize("precision", ["bf16", "fp8_tensor"])
def test_embed_is_the_mean_of_the_encoder_rows(precision):
    """C3 architecture, ragged lengths with empty segments: bit-exact against the
    fp32 row-order mean of the engine's own packed hidden states; empty
    segments give zeros.  In the per-tensor FP8 variant the embed call is the
    engine's first and calibrates it, so the encode after it runs at the same
    scales."""
    spec = synth.SPECS["c3"]
    eng = FastSnapjudge(spec.cfg, synth.make_weights(spec), precision=precision)
    rng = np.random.default_rng(5)
    lengths = np.array([0, 300, 1, 77, 0, 128, 129, 512, 5])
    ids = rng.integers(0, spec.cfg.vocab_size, size=int(lengths.sum())).astype(np.int64)
    got = eng.embed_packed(ids, lengths)
    h = eng.encode_packed(ids, lengths)
    cu = np.concatenate([[0], np.cumsum(lengths)])
    for b, n in enumerate(lengths):
        acc = np.zeros(h.shape[1], np.float32)
        for i in range(cu[b], cu[b + 1]):
            acc += h[i]
        want = acc / np.float32(max(1, int(n)))
        assert np.array_equal(got[b], want), b
    assert (got[lengths == 0] == 0).all()


def test_embed_passes_and_many_empty_segments():
    """More sequences than max_tokens (most of them empty) split into passes
    of at most max_tokens sequences; results match a single pass."""
    spec = synth.SPECS["tiny"]
    t = synth.make_weights(spec)
    small = FastSnapjudge(spec.cfg, t, precision="fp32", max_tokens=128)
    big = FastSnapjudge(spec.cfg, t, precision="fp32", max_tokens=4096)
    rng = np.random.default_rng(9)
    lengths = np.zeros(400, np.int64)
    lengths[rng.choice(400, size=12, replace=False)] = rng.integers(1, 40, size=12)
    ids = rng.integers(0, spec.cfg.vocab_size, size=int(lengths.sum())).astype(np.int64)
    a = small.embed_packed(ids, lengths)
    b = big.embed_packed(ids, lengths)
    assert np.array_equal(a, b)
    assert (a[lengths == 0] == 0).all()


def test_embed_errors():
    spec = synth.SPECS["tiny"]
    eng = FastSnapjudge(spec.cfg, synth.make_weights(spec), precision="fp32")
    with pytest.raises(SnapjudgeError, match="vocabulary"):
        eng.embed_packed(np.array([0, spec.cfg.vocab_size]), np.array([2]))
    with pytest.raises(SnapjudgeError, match="max_tokens"):
        FastSnapjudge(spec.cfg, synth.make_weights(spec), precision="fp32",
                      max_tokens=128).embed_packed(np.zeros(200, np.int64), np.array([200]))
