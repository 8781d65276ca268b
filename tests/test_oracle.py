"""The CPU oracle (C restatement) pinned against the reference.

* the reference's own op-level golden vectors (``tensor_ops_ref.npz``, from the
  reference's ``tests/golden/tensor_ops.json``) at the reference's tolerances
  (``tests/test_tensor.cpp:67-100``: 1e-5, layer norm 1e-4);
* the reference's compiled ``DecisionModel::encode``/``forward`` outputs on
  seeded synthetic checkpoints (``encoder_ref.npz``);
* live against ``oracle/_ref`` (the reference sources compiled unchanged) on
  random inputs, when that library has been built.
"""
import os

import numpy as np
import pytest

from oracle import oracle
from snapjudge_b200 import synth


@pytest.fixture(scope="module")
def G(golden_dir):
    return dict(np.load(os.path.join(golden_dir, "tensor_ops_ref.npz")))


def close(got, want, tol):
    err = float(np.max(np.abs(np.asarray(got, np.float64) - np.asarray(want, np.float64))))
    assert err <= tol, err
    return err


def test_gemm_goldens(G):
    a, w, b = G["gemm.a"], G["gemm.w"], G["gemm.bias"]
    close(oracle.gemm_nt(a, w, b, 0), G["gemm.out"], 1e-5)
    close(oracle.gemm_nt(a, w, b, 1), G["gemm_gelu.out"], 1e-5)
    close(oracle.gemm_nt(a, w, b, 2), G["gemm_relu.out"], 1e-5)
    close(oracle.geglu(a, G["geglu.wi"]), G["geglu.out"], 1e-5)


def test_layer_norm_goldens(G):
    x, w, b = G["layer_norm.x"], G["layer_norm.w"], G["layer_norm.b"]
    close(oracle.layer_norm(x, w, b), G["layer_norm.out"], 1e-4)
    close(oracle.layer_norm(x, w, None), G["layer_norm.out_nobias"], 1e-4)


def test_attention_goldens(G):
    q, k, v = G["attn_full.q"], G["attn_full.k"], G["attn_full.v"]
    lens = G["attn_full.lens"]
    close(oracle.attention(q, k, v, lens, 0), G["attn_full.out"], 1e-5)
    close(oracle.attention(q, k, v, lens, 2), G["attn_window.out"], 1e-5)


def test_rope_goldens(G):
    L, H, Dh = int(G["rope.L"]), int(G["rope.H"]), int(G["rope.Dh"])
    out = oracle.rope(G["rope.qkv"], G["rope.cos"], G["rope.sin"], L, H, Dh)
    close(out, G["rope.out"], 1e-5)
    # the oracle's own table (fp64 angles -> fp32, src/model.cpp:173-190) matches
    c, s = oracle.rope_table(float(G["rope.theta"]), Dh, L)
    close(c, G["rope.cos"], 1e-7)
    close(s, G["rope.sin"], 1e-7)


@pytest.mark.parametrize("name", ["tiny", "c1"])
def test_encoder_matches_reference_goldens(golden_dir, name):
    E = np.load(os.path.join(golden_dir, "encoder_ref.npz"))
    spec = synth.SPECS[name]
    orc = oracle.Oracle(spec.cfg, synth.make_weights(spec))
    ci = 0
    while f"{name}.{ci}.lengths" in E:
        p = f"{name}.{ci}."
        lengths, ids = E[p + "lengths"], E[p + "ids"]
        pid, mask = synth.pad_batch(ids, lengths)
        h = orc.encode_padded(pid, mask)
        # padded rows included: same padded semantics as DecisionModel::encode
        close(h, E[p + "hidden"], 2e-5)
        # packed varlen gives the same valid rows
        hp = orc.encode_packed(ids, lengths)
        cu = synth.cu_seqlens(lengths)
        for b in range(len(lengths)):
            close(hp[cu[b]:cu[b + 1]], E[p + "hidden"][b, :lengths[b]], 2e-5)
        lg, act = orc.forward_padded(pid, mask, E[p + "marker_pos"], E[p + "marker_mask"],
                                     E[p + "qtype"])
        close(lg, E[p + "logits"], 1e-4)
        close(act, E[p + "act"], 1e-5)
        ci += 1
    assert ci >= 3


ref = pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built")


@ref
def test_ops_match_compiled_reference():
    rng = np.random.default_rng(5)
    a = rng.standard_normal((33, 40), dtype=np.float32)
    w = rng.standard_normal((24, 40), dtype=np.float32) * 0.1
    b = rng.standard_normal(24, dtype=np.float32)
    for act in (0, 1, 2):
        close(oracle.gemm_nt(a, w, b, act), oracle.ref_gemm_nt(a, w, b, act), 1e-5)
    wi = rng.standard_normal((2 * 12, 40), dtype=np.float32) * 0.1
    close(oracle.geglu(a, wi), oracle.ref_geglu(a, wi), 1e-5)
    x = rng.standard_normal((9, 70), dtype=np.float32) * 3 + 1
    lw = rng.standard_normal(70, dtype=np.float32)
    close(oracle.layer_norm(x, lw, None), oracle.ref_layer_norm(x, lw, None), 0)
    q, k, v = (rng.standard_normal((2, 3, 37, 16), dtype=np.float32) for _ in range(3))
    lens = np.array([37, 20])
    for win in (0, 3):
        close(oracle.attention(q, k, v, lens, win), oracle.ref_attention(q, k, v, lens, win), 0)
    c, s = oracle.rope_table(10000.0, 16, 64)
    qkv = rng.standard_normal((50, 3 * 2 * 16), dtype=np.float32)
    close(oracle.rope(qkv, c, s, 25, 2, 16), oracle.ref_rope(qkv, c, s, 25, 2, 16), 0)


def test_sjmodel_restatement_matches_reference_goldens(golden_dir):
    """The NumPy SjModel restatement against the reference's own SjModel::encode /
    forward outputs (tests/golden/sjmodel_ref.npz, ragged padded batches)."""
    E = np.load(os.path.join(golden_dir, "sjmodel_ref.npz"))
    cfg, seed = synth.SJ_SPECS["sj_tiny"]
    orc = oracle.SjOracle(cfg, synth.make_sj_weights(cfg, seed))
    ci = 0
    while f"sj_tiny.{ci}.lengths" in E:
        g = {k.split(".", 2)[2]: E[k] for k in E.files if k.startswith(f"sj_tiny.{ci}.")}
        pid, mask = synth.pad_batch(g["ids"], g["lengths"])
        h = orc.encode_padded(pid, mask)
        assert np.abs(h - g["hidden"]).max() <= 1e-5 * max(1.0, np.abs(g["hidden"]).max())
        lg, act = orc.forward_padded(pid, mask, g["marker_pos"], g["marker_mask"], g["qtype"])
        assert np.abs(lg - g["logits"]).max() <= 1e-5
        assert np.abs(act - g["act"]).max() <= 1e-6
        ci += 1
    assert ci == 3


def test_embed_mean_known_answer():
    """Agent::embed's pooling (agent.cpp:347-354): valid positions only, in fp32,
    divided by max(1, n) — an empty row gives zeros."""
    h = np.arange(2 * 3 * 2, dtype=np.float32).reshape(2, 3, 2)
    mask = np.array([[1, 1, 0], [0, 0, 0]])
    got = oracle.embed_mean(h, mask)
    assert np.array_equal(got, np.array([[1.0, 2.0], [0.0, 0.0]], np.float32))
    # rows past the mask do not enter the sum, whatever they hold
    h2 = h.copy()
    h2[0, 2] = np.nan
    assert np.array_equal(oracle.embed_mean(h2, mask), got)


@pytest.mark.parametrize("H,Dh,lens,window,kv_lens", [
    (2, 8, [6, 4], 0, None), (2, 8, [6, 4], 2, None), (3, 16, [40, 1, 0, 17], 0, [30, 1, 0, 3]),
    (2, 64, [300, 129], 0, None), (2, 64, [200, 50], 7, None), (1, 16, [5, 9], 0, [0, 9])])
def test_numpy_attention_matches_c_restatement(H, Dh, lens, window, kv_lens):
    """The matrix-product restatement (used for long segments in the GPU
    parity tests) agrees with the scalar C restatement of
    src/tensor.cpp:156-228, including kv_lens (padded-batch semantics), windows,
    empty segments and segments with no visible key."""
    rng = np.random.default_rng(21)
    T = int(np.sum(lens))
    q, k, v = (rng.standard_normal((T, H, Dh), dtype=np.float32) for _ in range(3))
    want = oracle.attention_packed(q, k, v, lens, window, kv_lens)
    close(oracle.attention_packed_np(q, k, v, lens, window, kv_lens), want, 2e-6)
    close(oracle.attention_packed_np(q, k, v, lens, window, kv_lens, dtype=np.float32), want, 2e-5)
