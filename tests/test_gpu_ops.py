"""Kernel-level parity on the GPU: each C-ABI launcher against the CPU oracle.

bf16 in / bf16 out with fp32 accumulation, so the bar is bf16 output rounding:
max |got - want| <= 2^-7 * max(1, |want|) elementwise (about 2 bf16 ulps),
except the LayerNorm residual stream X, which is fp32 and must match to 1e-6.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle  # noqa: E402
from snapjudge_b200 import ops  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def bf(x):
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(DEV).to(torch.bfloat16)


def f32(t):
    return t.float().cpu().numpy()


def assert_bf16_close(got, want, k=2.0):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    tol = k * 2.0 ** -8 * np.maximum(1.0, np.abs(want))
    bad = np.abs(got - want) > tol
    assert not bad.any(), f"{bad.sum()} mismatches, max err {np.abs(got - want).max():.3g}"


def rnd(shape, seed, scale=1.0):
    return np.random.default_rng(seed).standard_normal(shape, dtype=np.float32) * scale


@pytest.mark.parametrize("M,N,K", [(1, 64, 64), (37, 96, 48), (300, 256, 128), (129, 768, 768),
                                   (1000, 2304, 768), (77, 768, 2048),
                                   # CTA-pair tiles (M >= 2048): full and partial 256-row tiles
                                   (4096, 768, 768), (2100, 2304, 768), (2311, 768, 2048)])
@pytest.mark.parametrize("act,bias", [(0, False), (1, True), (2, True)])
def test_gemm(M, N, K, act, bias):
    A = bf(rnd((M, K), 1))
    W = bf(rnd((N, K), 2, 0.05))
    b = torch.from_numpy(rnd(N, 3, 0.1)).to(DEV) if bias else None
    got = f32(ops.gemm(A, W, b, act))
    want = oracle.gemm_nt(f32(A), f32(W), None if b is None else b.cpu().numpy(), act)
    assert_bf16_close(got, want)


@pytest.mark.parametrize("M,F,K", [(5, 8, 16), (200, 256, 64), (513, 2048, 768), (64, 2816, 1024),
                                   (3000, 2048, 768), (2048, 2816, 1024),
                                   # F an odd multiple of 64: 128-column tiles, direct stores
                                   (300, 192, 128), (2200, 320, 256)])
def test_gemm_geglu(M, F, K):
    A = bf(rnd((M, K), 4))
    Wi = bf(rnd((2 * F, K), 5, 0.05))
    got = f32(ops.gemm_geglu(A, Wi))
    want = oracle.geglu(f32(A), f32(Wi))
    assert_bf16_close(got, want)


@pytest.mark.parametrize("M,D", [(1, 16), (33, 64), (1000, 768), (257, 1024), (9, 100)])
@pytest.mark.parametrize("residual,bias", [(False, False), (True, False), (True, True)])
def test_add_ln(M, D, residual, bias):
    x = rnd((M, D), 6, 3.0) + 1.0
    X = torch.from_numpy(x).to(DEV)
    R = bf(rnd((M, D), 7)) if residual else None
    w = torch.from_numpy(rnd(D, 8)).to(DEV)
    b = torch.from_numpy(rnd(D, 9)).to(DEV) if bias else None
    Y = ops.add_ln(X, R, w, b, eps=1e-5)
    xs = x + (f32(R) if residual else 0)
    np.testing.assert_allclose(X.cpu().numpy(), xs, rtol=0, atol=1e-6)
    want = oracle.layer_norm(xs, w.cpu().numpy(), None if b is None else b.cpu().numpy(), 1e-5)
    assert_bf16_close(f32(Y), want)


@pytest.mark.parametrize("H,Dh,lens", [(2, 8, [5, 17, 1]), (12, 64, [128, 1, 77, 300]),
                                       (16, 64, [2048])])
def test_rope(H, Dh, lens):
    lens = np.asarray(lens)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    T = int(cu[-1])
    qkv0 = rnd((T, 3 * H * Dh), 10)
    qkv = bf(qkv0)
    c, s = oracle.rope_table(10000.0, Dh, int(lens.max()))
    ops.rope_(qkv, torch.from_numpy(c).to(DEV), torch.from_numpy(s).to(DEV), cu, H, Dh)
    ref = f32(bf(qkv0))
    want = np.empty_like(ref)
    for b in range(len(lens)):
        seg = ref[cu[b]:cu[b + 1]]
        want[cu[b]:cu[b + 1]] = oracle.rope(seg, c, s, max(1, int(lens[b])), H, Dh)
    assert_bf16_close(f32(qkv), want)


ATTN_CASES = [
    # (H, Dh, lens, window, kv_lens)
    (3, 8, [6, 4], 0, None),
    (3, 8, [6, 4], 2, None),
    (2, 16, [32, 32, 17, 1], 0, None),
    (2, 16, [40, 23, 1], 4, None),
    (12, 64, [1, 7, 33, 127, 128, 129, 255, 256, 257, 512], 0, None),
    (12, 64, [300, 200], 64, None),
    (4, 64, [100, 100], 0, [100, 37]),  # padded-batch semantics: keys < kv_len
    (16, 64, [2048], 0, None),
    (16, 64, [2048, 1000], 128, None),  # sliding window at scale: out-of-window tiles skipped
    # long segments (>= 512 tokens, full attention) on attn_long beside short ones on
    # attn_tc: partial last key tiles (<= 64 and > 64 visible keys), items with one Q
    # tile or a second tile of one row, kv_lens down to one key and to none
    (12, 64, [300, 512, 1000, 777, 511, 64, 2], 0, [300, 100, 999, 1, 511, 64, 2]),
    (2, 64, [511, 512, 513, 639, 640, 641, 767], 0, None),
    (2, 64, [700, 600, 40], 0, [0, 37, 40]),
    # empty segments among short ones (sj_attn's host-sorted tile list skips them)
    (4, 64, [0, 130, 0, 5, 300, 0], 0, None),
    (4, 64, [0, 130, 0, 5, 300, 0], 32, [0, 100, 0, 5, 299, 0]),
]


@pytest.mark.parametrize("H,Dh,lens,window,kv_lens", ATTN_CASES)
def test_attention(H, Dh, lens, window, kv_lens):
    lens = np.asarray(lens)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    T = int(cu[-1])
    qkv0 = rnd((T, 3 * H * Dh), 11)
    qkv = bf(qkv0)
    O = ops.attn(qkv, cu, H, Dh, window, kv_lens)
    x = f32(qkv).reshape(T, 3, H, Dh)
    want = oracle.attention_packed(x[:, 0], x[:, 1], x[:, 2], lens, window, kv_lens)
    assert_bf16_close(f32(O).reshape(T, H, Dh), want, k=4.0)


def test_attention_c2_shapes():
    """C2 in full: 64 sequences, 12 heads x 64, lengths U[32, 512], Q/K/V N(0,1)
    (seed 1) — segments of 256 tokens or more on attn_long, the rest on attn_tc."""
    from snapjudge_b200 import synth
    lens, q, k, v = synth.attention_inputs()
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    T, H, Dh = q.shape
    qkv = bf(np.concatenate([q, k, v], axis=1).reshape(T, 3 * H * Dh))
    O = f32(ops.attn(qkv, cu, H, Dh)).reshape(T, H, Dh)
    x = f32(qkv).reshape(T, 3, H, Dh)
    want = oracle.attention_packed_np(x[:, 0], x[:, 1], x[:, 2], lens)
    assert_bf16_close(O, want, k=4.0)


@pytest.mark.parametrize("B,n,H", [(64, 512, 12), (32, 2048, 16)])
def test_attention_long_shapes(B, n, H):
    """The bench's fixed-length attention shapes in full against the oracle:
    64 x 512 tokens (12 heads) and C4's 32 x 2048 tokens (16 heads)."""
    lens = np.full(B, n)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    T = int(cu[-1])
    qkv = torch.randn(T, 3 * H * 64, generator=torch.Generator().manual_seed(B + n)).to(DEV).to(
        torch.bfloat16)
    O = f32(ops.attn(qkv, cu, H, 64)).reshape(T, H, 64)
    x = f32(qkv).reshape(T, 3, H, 64)
    want = oracle.attention_packed_np(x[:, 0], x[:, 1], x[:, 2], lens, dtype=np.float32)
    assert_bf16_close(O, want, k=4.0)


def test_attention_many_short_segments():
    """More short-segment query tiles than sj_attn's parameter-block tile list
    holds (2,048): the call falls back to the kernel's own grid order.  2,100
    segments of 1-128 tokens, 2 heads, against the oracle."""
    lens = np.random.default_rng(21).integers(1, 129, 2100)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    T, H = int(cu[-1]), 2
    qkv = torch.randn(T, 3 * H * 64, generator=torch.Generator().manual_seed(21)).to(DEV).to(
        torch.bfloat16)
    O = f32(ops.attn(qkv, cu, H, 64)).reshape(T, H, 64)
    x = f32(qkv).reshape(T, 3, H, 64)
    want = oracle.attention_packed_np(x[:, 0], x[:, 1], x[:, 2], lens, dtype=np.float32)
    assert_bf16_close(O, want, k=4.0)


def test_attention_output_alignment():
    """The tensor-core attention writes each output row with 32-byte stores when
    O is 32-byte aligned and falls back to 16-byte stores otherwise: an O
    buffer at a 16-byte offset gives the same bits as an aligned one."""
    import ctypes as C
    from snapjudge_b200 import _lib
    H, Dh = 4, 64
    lens = np.array([200, 77, 1, 128])
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    T = int(cu[-1])
    qkv = bf(rnd((T, 3 * H * Dh), 13))
    want = ops.attn(qkv, cu, H, Dh)
    big = torch.zeros(T * H * Dh + 8, dtype=torch.bfloat16, device=DEV)
    O = big[8:]  # 16 bytes past a 256-byte-aligned allocation
    assert O.data_ptr() % 32 == 16
    cu_d = torch.from_numpy(cu).to(DEV)
    rc = _lib.lib().sj_attn(C.c_void_p(qkv.data_ptr()), C.c_void_p(cu_d.data_ptr()),
                            C.c_void_p(cu.ctypes.data), None, C.c_void_p(O.data_ptr()),
                            len(lens), H, Dh, 0, C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    torch.cuda.synchronize()
    assert torch.equal(O.view(T, H * Dh), want)
    assert (big[:8] == 0).all()
