"""sj_attn_noalloc: attention for callers that cannot allocate device memory.

Some hosts cannot call cudaMalloc on their inference path (their device memory
is owned by their own pool allocator, or allocation is not allowed there).
sj_attn_noalloc keeps the query-tile schedule the engine would allocate in a
static device array of the library instead.  Checked here through the C ABI:

* against the CPU oracle (and against sj_attn) on two calls in a row with
  different batches, in both orders: a larger schedule followed by a smaller
  one, and a smaller one followed by a larger one (the second call must write
  every entry it reads; the shared array keeps the previous call's contents);
* a segment long enough for the capped bucket of the schedule (>= 255 tiles),
  against sj_attn on the same inputs;
* a batch above the array's capacity is rejected with a message;
* sj_check_device_errors reports nothing after these calls.

The file is named to be collected last: a failure here comes after every other
test has run.
"""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle  # noqa: E402
from snapjudge_b200 import _lib  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _run(fn_name, qkv, cu_h, H, Dh, window, kv_lens=None):
    L = _lib.lib()
    cu_d = torch.from_numpy(cu_h).to(DEV)
    kv = None if kv_lens is None else torch.from_numpy(np.asarray(kv_lens, np.int32)).to(DEV)
    O = torch.zeros(int(cu_h[-1]), H * Dh, dtype=torch.bfloat16, device=DEV)
    rc = getattr(L, fn_name)(C.c_void_p(qkv.data_ptr()), C.c_void_p(cu_d.data_ptr()),
                             C.c_void_p(cu_h.ctypes.data),
                             None if kv is None else C.c_void_p(kv.data_ptr()),
                             C.c_void_p(O.data_ptr()), len(cu_h) - 1, H, Dh, window, _stream())
    assert rc == 0, L.sj_last_error()
    assert L.sj_check_device_errors(_stream()) == 0, L.sj_last_error()
    return O.float().cpu().numpy()


def _case(lens, H, Dh, seed):
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    g = torch.Generator(device="cpu").manual_seed(seed)
    qkv = torch.randn(int(cu[-1]), 3 * H * Dh, generator=g).to(DEV).to(torch.bfloat16)
    return qkv, cu


def _close(got, want):
    tol = 4.0 * 2.0 ** -8 * np.maximum(1.0, np.abs(want))
    assert (np.abs(got - want) <= tol).all(), np.abs(got - want).max()


LARGE = [300, 1, 129, 512, 77, 256, 700]  # 16 tiles of 128 rows
SMALL = [33, 5, 128, 128]                 # 4 tiles


@pytest.mark.parametrize("order", ["large_first", "small_first"])
@pytest.mark.parametrize("H,Dh,window", [(12, 64, 0), (12, 64, 48), (2, 16, 0)])
def test_noalloc_matches_oracle_twice(H, Dh, window, order):
    batches = [LARGE, SMALL] if order == "large_first" else [SMALL, LARGE]
    for i, lens in enumerate(batches):  # two calls in a row, different batches
        qkv, cu = _case(lens, H, Dh, 100 + i)
        kv = [max(1, n - 3) for n in lens] if i == 1 else None
        got = _run("sj_attn_noalloc", qkv, cu, H, Dh, window, kv)
        T = int(cu[-1])
        x = qkv.float().cpu().numpy().reshape(T, 3, H, Dh)
        want = oracle.attention_packed(x[:, 0], x[:, 1], x[:, 2], lens, window, kv)
        _close(got.reshape(T, H, Dh), want)
        _close(got, _run("sj_attn", qkv, cu, H, Dh, window, kv))


@pytest.mark.parametrize("Dh,qt", [(64, 128), (16, 64)])
def test_noalloc_long_segment_capped_bucket(Dh, qt):
    # two segments of >= 255 query tiles share the schedule's last (capped)
    # bucket, beside short ones in other buckets
    lens = [255 * qt + 17, 3, 300 * qt, qt + 1]
    qkv, cu = _case(lens, 1, Dh, 7)
    got = _run("sj_attn_noalloc", qkv, cu, 1, Dh, 0)
    want = _run("sj_attn", qkv, cu, 1, Dh, 0)
    _close(got, want)


def test_noalloc_rejects_batches_over_capacity():
    L = _lib.lib()
    cu = np.arange(0, 65537 * 2, 2, dtype=np.int32)  # 65536 one-tile sequences + 1
    cu = np.concatenate([cu, [cu[-1] + 2]]).astype(np.int32)
    rc = L.sj_attn_noalloc(None, None, C.c_void_p(cu.ctypes.data), None, None, len(cu) - 1, 12,
                           64, 0, None)
    assert rc == _lib.SJ_ERR_INVALID
    assert b"capacity" in L.sj_last_error()
