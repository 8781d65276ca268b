"""The FP8 variants: e4m3 quantisation, the e4m3 tcgen05 GEMM, and the encoder
with its QKV and Wi projections on e4m3 operands (SJ_PREC_FP8: per-token and
per-channel scales) or its QKV, Wi and Wo2 projections (SJ_PREC_FP8_TENSOR:
one scale per tensor, activation scales calibrated on the first pass).

The reference has no FP8 path, so the kernels are checked against what they
define, and the encoder against the fp32 CPU forward with a bar of its own:
* quantisation: bit-exact against torch's float32 -> float8_e4m3fn conversion
  (round to nearest even) of x * (448 / amax), with scale = amax / 448, both
  divisions correctly rounded in fp32;
* GEMM: against a float64 product of the dequantised codes (code value x row
  scale x channel scale), within bf16 output rounding: |got - want| <=
  2^-7 |want| + 1e-5 rms(want);
* encoder (C3 architecture, 12 x 768, ragged batch of 8): final hidden states
  against the fp32 forward within a relative (Frobenius) error of 0.06 and a
  row cosine of at least 0.998.  Measured on a B200: relative error 0.031
  (bf16 mode 0.0024), smallest row cosine 0.9991, max-abs 0.15 (bf16 0.011).
"""
import numpy as np
import pytest
from scipy.special import erf

torch = pytest.importorskip("torch")

from oracle import oracle  # noqa: E402
from snapjudge_b200 import ops, synth  # noqa: E402
from snapjudge_b200.fast import FastSnapjudge, SnapjudgeError  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture(scope="module", autouse=True)
def _blas():
    oracle.set_blas()


def ref_quant(x):
    """CPU reference of sj_quant_e4m3: (codes uint8, scales fp32)."""
    x = np.asarray(x, np.float32)
    amax = np.abs(x).max(axis=1)
    scale = np.where(amax > 0, amax / np.float32(448), np.float32(1)).astype(np.float32)
    inv = np.where(amax > 0, np.float32(448) / np.where(amax > 0, amax, 1), 0).astype(np.float32)
    y = (x * inv[:, None]).astype(np.float32)
    codes = torch.from_numpy(y).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    return codes, scale


def dequant(codes, scale):
    v = torch.from_numpy(np.ascontiguousarray(codes)).view(torch.float8_e4m3fn).double().numpy()
    return v * np.asarray(scale, np.float64)[:, None]


def quant_dev(x):
    q, s = ops.quant_e4m3(torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(DEV))
    return q, s


@pytest.mark.parametrize("rows,cols", [(1, 4), (7, 64), (300, 768), (2049, 2048)])
def test_quant_e4m3_bit_exact(rows, cols):
    rng = np.random.default_rng(rows + cols)
    x = rng.standard_normal((rows, cols), dtype=np.float32)
    x *= np.exp(rng.uniform(-6, 6, size=(rows, 1))).astype(np.float32)  # row magnitudes
    x[0, : cols // 2] *= 1e-4  # tiny values (e4m3 subnormals) next to the row's maximum
    if rows > 2:
        x[1] = 0.0  # an all-zero row: scale 1, codes 0
    q, s = quant_dev(x)
    torch.cuda.synchronize()
    want_q, want_s = ref_quant(x)
    assert np.array_equal(s.cpu().numpy(), want_s)
    assert np.array_equal(q.cpu().numpy(), want_q)


def gelu(x):
    return 0.5 * x * (1.0 + erf(x / np.sqrt(2.0)))


def _close(got, want):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    tol = 2.0 ** -7 * np.abs(want) + 1e-5 * np.sqrt(np.mean(want ** 2))
    bad = np.abs(got - want) > tol
    assert not bad.any(), f"{bad.sum()} mismatches, max err {np.abs(got - want).max():.3g}"


@pytest.mark.parametrize("M,N,K", [(37, 64, 128), (300, 384, 256), (129, 768, 768),
                                   (2100, 2304, 768), (4096, 768, 768)])
@pytest.mark.parametrize("act,bias", [(0, False), (1, True)])
def test_gemm_e4m3(M, N, K, act, bias):
    rng = np.random.default_rng(M + N + K)
    A = rng.standard_normal((M, K), dtype=np.float32)
    W = rng.standard_normal((N, K), dtype=np.float32) * 0.05
    qa, sa = quant_dev(A)
    qw, sw = quant_dev(W)
    b = torch.from_numpy(rng.standard_normal(N, dtype=np.float32) * 0.1).to(DEV) if bias else None
    got = ops.gemm_e4m3(qa, sa, qw, sw, b, act).float().cpu().numpy()
    want = dequant(qa.cpu().numpy(), sa.cpu().numpy()) @ dequant(qw.cpu().numpy(),
                                                                  sw.cpu().numpy()).T
    if bias:
        want = want + b.cpu().numpy().astype(np.float64)
    if act == 1:
        want = gelu(want)
    _close(got, want)


@pytest.mark.parametrize("M,F,K", [(200, 256, 128), (513, 2048, 768), (3000, 2048, 768),
                                   (300, 192, 128)])
def test_gemm_e4m3_geglu(M, F, K):
    rng = np.random.default_rng(M + F)
    A = rng.standard_normal((M, K), dtype=np.float32)
    Wi = rng.standard_normal((2 * F, K), dtype=np.float32) * 0.05
    qa, sa = quant_dev(A)
    qw, sw = quant_dev(Wi)
    got = ops.gemm_e4m3(qa, sa, qw, sw, geglu=True).float().cpu().numpy()
    h = dequant(qa.cpu().numpy(), sa.cpu().numpy()) @ dequant(qw.cpu().numpy(), sw.cpu().numpy()).T
    _close(got, gelu(h[:, :F]) * h[:, F:])


def test_gemm_e4m3_rejects_bad_shapes():
    qa = torch.zeros(8, 96, dtype=torch.uint8, device=DEV)
    s = torch.ones(8, dtype=torch.float32, device=DEV)
    with pytest.raises(SnapjudgeError, match="K % 128"):
        ops.gemm_e4m3(qa, s, torch.zeros(64, 96, dtype=torch.uint8, device=DEV),
                      torch.ones(64, dtype=torch.float32, device=DEV))


def _rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def test_fp8_encoder_against_fp32_forward():
    """C3 architecture, ragged batch: the FP8 variant's final hidden states
    against the fp32 CPU forward, beside the bf16 mode's error."""
    spec = synth.SPECS["c3"]
    t = synth.make_weights(spec)
    rng = np.random.default_rng(12)
    lengths = np.array([300, 251, 177, 128, 96, 64, 17, 1])
    ids = rng.integers(0, spec.cfg.vocab_size, size=int(lengths.sum())).astype(np.int64)
    want = oracle.Oracle(spec.cfg, t).encode_packed(ids, lengths)
    h8 = FastSnapjudge(spec.cfg, t, precision="fp8").encode_packed(ids, lengths)
    h16 = FastSnapjudge(spec.cfg, t, precision="bf16").encode_packed(ids, lengths)
    assert np.isfinite(h8).all()
    e8, e16 = _rel(h8, want), _rel(h16, want)
    cos = np.sum(h8 * want, axis=1) / (np.linalg.norm(h8, axis=1) * np.linalg.norm(want, axis=1))
    print(f"relative error: fp8 {e8:.4f}, bf16 {e16:.4f}; min row cosine fp8 {cos.min():.5f}; "
          f"max abs fp8 {np.abs(h8 - want).max():.4f}, bf16 {np.abs(h16 - want).max():.4f}")
    assert e8 <= 0.06 and cos.min() >= 0.998


def test_fp8_is_decisionmodel_only():
    cfg, seed = synth.SJ_SPECS["sj_tiny"]
    with pytest.raises(SnapjudgeError):
        FastSnapjudge(cfg, synth.make_sj_weights(cfg, seed), precision="fp8")


@pytest.mark.parametrize("precision", ["fp8", "fp8_tensor"])
def test_fp8_forward_against_fp32_forward(precision):
    """The whole DecisionModel::forward with the encoder in the FP8 variant (the
    head layers, scorer and act head unchanged): C3 architecture, 8 requests
    padded to 300 rows, against the fp32 CPU forward.  Bars for the FP8
    variant: logits within 0.04 max-abs, act probabilities within 5e-3.
    Measured on a B200: logits 0.014 per-token, 0.018 per-tensor (inside even
    the bf16 bar of 2e-2), act below 1e-4."""
    spec = synth.SPECS["c3"]
    t = synth.make_weights(spec)
    rng = np.random.default_rng(11)
    lengths = np.minimum(synth.make_lengths(spec, batch=8, seed=31), 300)
    lengths[0] = 300
    ids = synth.make_ids(spec, lengths, seed=32)
    pid, mask = synth.pad_batch(ids, lengths)
    K = 6
    pos = np.zeros((8, K), np.int64)
    mm = np.zeros((8, K), np.uint8)
    for b, n in enumerate(lengths):
        k = int(rng.integers(1, K + 1))
        pos[b, :k] = rng.integers(0, n, size=k)
        mm[b, :k] = 1
    qt = rng.integers(0, 3, size=8).astype(np.int64)
    logits, act = FastSnapjudge(spec.cfg, t, precision=precision).forward(pid, mask, pos, mm, qt)
    want_l, want_a = oracle.Oracle(spec.cfg, t).forward_padded(pid, mask, pos, mm, qt)
    live = mm == 1
    dl, da = np.abs(logits - want_l)[live].max(), np.abs(act - want_a).max()
    print(f"{precision} forward: logits max-abs {dl:.4f}, act max-abs {da:.4f}")
    assert np.isfinite(logits).all() and (logits[~live] == -1e4).all()
    assert dl <= 0.04 and da <= 5e-3


def _fp8_vs_oracle(cfg, t, lengths, seed, rel_bar=0.06, cos_bar=0.998, precision="fp8"):
    ids = np.random.default_rng(seed).integers(0, cfg.vocab_size, size=int(lengths.sum()))
    ids = ids.astype(np.int64)
    want = oracle.Oracle(cfg, t).encode_packed(ids, lengths)
    got = FastSnapjudge(cfg, t, precision=precision).encode_packed(ids, lengths)
    assert np.isfinite(got).all()
    cos = np.sum(got * want, axis=1) / (np.linalg.norm(got, axis=1) * np.linalg.norm(want, axis=1))
    e = _rel(got, want)
    print(f"{precision}: relative error {e:.4f}, min row cosine {cos.min():.5f}")
    assert e <= rel_bar and cos.min() >= cos_bar
    return got, ids


@pytest.mark.parametrize("precision", ["fp8", "fp8_tensor"])
def test_fp8_sliding_window_layers(precision):
    """ModernBERT's layer pattern (sliding layers with their own RoPE theta) in
    the FP8 variant, C3 architecture, against the fp32 forward."""
    import dataclasses
    base = synth.SPECS["c3"]
    cfg = dataclasses.replace(
        base.cfg, local_attention=128,
        layer_types=["full_attention" if i % 3 == 0 else "sliding_attention"
                     for i in range(base.cfg.num_hidden_layers)])
    _fp8_vs_oracle(cfg, synth.make_weights(dataclasses.replace(base, cfg=cfg)),
                   np.array([512, 300, 129, 64, 1]), 93, precision=precision)


def test_fp8_c4_architecture_and_passes():
    """C4 architecture (24 x 1024, F = 2816) in the FP8 variant, and the same
    batch split into several passes (max_tokens below the batch): identical.
    Twice the layers of C3 accumulate about twice the error: measured on a
    B200, relative error 0.069 and smallest row cosine 0.9967; bars 0.12 and
    0.994."""
    spec = synth.SPECS["c4"]
    t = synth.make_weights(spec)
    lengths = np.array([300, 77, 129])
    got, ids = _fp8_vs_oracle(spec.cfg, t, lengths, 94, rel_bar=0.12, cos_bar=0.994)
    again = FastSnapjudge(spec.cfg, t, precision="fp8", max_tokens=320).encode_packed(ids, lengths)
    assert np.array_equal(got, again)


# ---- SJ_PREC_FP8_TENSOR: per-tensor scales, calibrated activation scales ----

def _vs(got, want):
    cos = np.sum(got * want, axis=1) / (np.linalg.norm(got, axis=1) * np.linalg.norm(want, axis=1))
    return _rel(got, want), float(cos.min())


def test_fp8_tensor_encoder_against_fp32_forward():
    """The per-tensor variant (QKV, Wi and Wo2 on e4m3, one scale per weight
    tensor, static activation scales from a calibration pass over this same
    batch), C3 architecture, ragged batch of 8, against the fp32 forward with
    the per-token variant's bars.  Measured on a B200: relative error 0.0386
    (per-token 0.0309), smallest row cosine 0.9991."""
    spec = synth.SPECS["c3"]
    t = synth.make_weights(spec)
    rng = np.random.default_rng(12)
    lengths = np.array([300, 251, 177, 128, 96, 64, 17, 1])
    ids = rng.integers(0, spec.cfg.vocab_size, size=int(lengths.sum())).astype(np.int64)
    want = oracle.Oracle(spec.cfg, t).encode_packed(ids, lengths)
    ht = FastSnapjudge(spec.cfg, t, precision="fp8_tensor").encode_packed(ids, lengths)
    h8 = FastSnapjudge(spec.cfg, t, precision="fp8").encode_packed(ids, lengths)
    assert np.isfinite(ht).all()
    et, ct = _vs(ht, want)
    e8, c8 = _vs(h8, want)
    print(f"relative error: fp8_tensor {et:.4f} (min row cosine {ct:.5f}), "
          f"fp8 {e8:.4f} ({c8:.5f})")
    assert et <= 0.06 and ct >= 0.998


def test_fp8_tensor_scales_fixed_after_first_pass():
    """Calibration runs once, on the engine's first pass: the same batch again
    gives identical states, and a later batch of other lengths and ids, run at
    the first batch's scales, stays within the bars against the fp32 forward."""
    spec = synth.SPECS["c3"]
    t = synth.make_weights(spec)
    rng = np.random.default_rng(21)
    la = np.array([200, 150, 33, 9])
    lb = np.array([511, 64, 2, 300, 120])
    ia = rng.integers(0, spec.cfg.vocab_size, size=int(la.sum())).astype(np.int64)
    ib = rng.integers(0, spec.cfg.vocab_size, size=int(lb.sum())).astype(np.int64)
    eng = FastSnapjudge(spec.cfg, t, precision="fp8_tensor")
    a1 = eng.encode_packed(ia, la)
    hb = eng.encode_packed(ib, lb)
    a2 = eng.encode_packed(ia, la)
    assert np.array_equal(a1, a2)
    e, c = _vs(hb, oracle.Oracle(spec.cfg, t).encode_packed(ib, lb))
    print(f"second batch at the first batch's scales: relative error {e:.4f}, min cosine {c:.5f}")
    assert e <= 0.06 and c >= 0.998


def test_fp8_tensor_reset_calibration():
    """After sj_fast_reset_calibration the next call calibrates on its own
    batch: the engine then gives what a fresh engine gives on that batch.
    Other precisions refuse the call."""
    spec = synth.SPECS["c3"]
    t = synth.make_weights(spec)
    rng = np.random.default_rng(23)
    la, lb = np.array([64, 9, 200]), np.array([300, 5, 77, 128])
    ia = rng.integers(0, spec.cfg.vocab_size, size=int(la.sum())).astype(np.int64)
    ib = rng.integers(0, spec.cfg.vocab_size, size=int(lb.sum())).astype(np.int64)
    eng = FastSnapjudge(spec.cfg, t, precision="fp8_tensor")
    eng.encode_packed(ia, la)
    at_a = eng.encode_packed(ib, lb)  # b at a's scales
    eng.reset_calibration()
    own = eng.encode_packed(ib, lb)   # b calibrated on b
    fresh = FastSnapjudge(spec.cfg, t, precision="fp8_tensor").encode_packed(ib, lb)
    assert np.array_equal(own, fresh)
    assert not np.array_equal(own, at_a)
    with pytest.raises(SnapjudgeError):
        FastSnapjudge(spec.cfg, t, precision="fp8").reset_calibration()


def test_fp8_tensor_passes():
    """A batch larger than max_tokens runs in several passes; the activation
    scales come from the first pass alone and the later passes run at them:
    within the bars against the fp32 forward."""
    spec = synth.SPECS["c3"]
    t = synth.make_weights(spec)
    lengths = np.array([300, 77, 129, 250, 64, 9])
    ids = np.random.default_rng(95).integers(0, spec.cfg.vocab_size, size=int(lengths.sum()))
    ids = ids.astype(np.int64)
    want = oracle.Oracle(spec.cfg, t).encode_packed(ids, lengths)
    got = FastSnapjudge(spec.cfg, t, precision="fp8_tensor", max_tokens=320).encode_packed(
        ids, lengths)
    e, c = _vs(got, want)
    print(f"fp8_tensor in passes of <= 320 tokens: relative error {e:.4f}, min cosine {c:.5f}")
    assert np.isfinite(got).all() and e <= 0.06 and c >= 0.998


def test_fp8_tensor_c4_architecture():
    """C4 architecture (24 x 1024, F = 2816, a multiple of 128) in the
    per-tensor variant, with the per-token variant's C4 bars.  Measured on a
    B200: relative error 0.085 (per-token 0.069), smallest row cosine 0.9950."""
    spec = synth.SPECS["c4"]
    t = synth.make_weights(spec)
    lengths = np.array([300, 77, 129])
    ids = np.random.default_rng(94).integers(0, spec.cfg.vocab_size, size=int(lengths.sum()))
    ids = ids.astype(np.int64)
    want = oracle.Oracle(spec.cfg, t).encode_packed(ids, lengths)
    got = FastSnapjudge(spec.cfg, t, precision="fp8_tensor").encode_packed(ids, lengths)
    e, c = _vs(got, want)
    print(f"fp8_tensor c4: relative error {e:.4f}, min row cosine {c:.5f}")
    assert np.isfinite(got).all() and e <= 0.12 and c >= 0.994


def test_fp8_tensor_needs_intermediate_multiple_of_128():
    import dataclasses
    spec = synth.SPECS["c3"]
    cfg = dataclasses.replace(spec.cfg, intermediate_size=2048 - 64)
    t = synth.make_weights(dataclasses.replace(spec, cfg=cfg))
    with pytest.raises(SnapjudgeError):
        FastSnapjudge(cfg, t, precision="fp8_tensor")
    FastSnapjudge(cfg, t, precision="fp8").close()  # the per-token variant takes F % 64


def test_fp8_variants_on_c5_heads():
    """Config 5's four decision heads (choice3, choice8, score5, noul) on 64
    requests of its length distribution: decision probabilities of the bf16
    mode and both FP8 variants against the fp32 CPU forward and fp64 heads.
    Bars: bf16 5e-3 (the bf16 probability bar), both FP8 variants 5e-2; the
    [CLS] states within 0.06 relative.  Measured on a B200: probabilities
    bf16 1.9e-3, fp8 2.4e-2, fp8_tensor 3.0e-2; [CLS] relative error 0.0025,
    0.032, 0.039."""
    spec = synth.SPECS["c5"]
    t = synth.make_weights(spec)
    lengths = synth.make_lengths(spec, batch=64, seed=515)
    ids = synth.make_ids(spec, lengths, seed=516)
    want_h = oracle.Oracle(spec.cfg, t).encode_packed(ids, lengths)
    cls = synth.cu_seqlens(lengths)[:-1]
    want = np.concatenate(oracle.task_heads(want_h[cls], t, spec.heads), axis=1)
    res = {}
    for prec in ("bf16", "fp8", "fp8_tensor"):
        eng = FastSnapjudge(spec.cfg, t, precision=prec, heads=spec.heads)
        p = eng.decide(ids, lengths)
        h = eng.encode_packed(ids, lengths)[cls]
        res[prec] = (float(np.abs(p - want).max()), _rel(h, want_h[cls]))
        eng.close()
    print("c5 heads, probability max-abs / [CLS] relative error: " +
          ", ".join(f"{k} {v[0]:.2e} / {v[1]:.4f}" for k, v in res.items()))
    assert res["bf16"][0] <= 5e-3
    for k in ("fp8", "fp8_tensor"):
        assert res[k][0] <= 5e-2 and res[k][1] <= 0.06, (k, res[k])
