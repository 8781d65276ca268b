"""sj_attn_noalloc: attention for callers that cannot allocate device memory.

Some hosts cannot call cudaMalloc on their inference path (their device memory
is owned by their own pool allocator, or allocation is not allowed there).
sj_attn_noalloc keeps the query-tile schedule the engine would allocate in a
static device array of the library instead.  This checks it through the C ABI
against sj_attn on the same inputs, within the bf16 bar of the other attention
tests, on two calls in a row with different batches (the shared array keeps the
previous call's schedule, which must not leak into the next result), and that a
batch above the array's capacity is rejected with a message.

The file is named to be collected last: a failure here comes after every other
test has run.
"""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from snapjudge_b200 import _lib  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _run(fn_name, qkv, cu_h, H, Dh, window, kv_lens=None):
    L = _lib.lib()
    cu_d = torch.from_numpy(cu_h).to(DEV)
    kv = None if kv_lens is None else torch.from_numpy(np.asarray(kv_lens, np.int32)).to(DEV)
    O = torch.zeros(int(cu_h[-1]), H * Dh, dtype=torch.bfloat16, device=DEV)
    st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = getattr(L, fn_name)(C.c_void_p(qkv.data_ptr()), C.c_void_p(cu_d.data_ptr()),
                             C.c_void_p(cu_h.ctypes.data),
                             None if kv is None else C.c_void_p(kv.data_ptr()),
                             C.c_void_p(O.data_ptr()), len(cu_h) - 1, H, Dh, window, st)
    torch.cuda.synchronize()
    assert rc == 0, L.sj_last_error()
    return O.float().cpu().numpy()


def _case(lens, H, Dh, seed):
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    g = torch.Generator(device="cpu").manual_seed(seed)
    qkv = torch.randn(int(cu[-1]), 3 * H * Dh, generator=g).to(DEV).to(torch.bfloat16)
    return qkv, cu


@pytest.mark.parametrize("H,Dh,window", [(12, 64, 0), (12, 64, 48), (2, 16, 0)])
def test_noalloc_matches_sj_attn_twice(H, Dh, window):
    batches = [[300, 1, 129, 512, 77, 256], [33, 700, 5, 128, 128]]
    for i, lens in enumerate(batches):  # two calls in a row, different batches
        qkv, cu = _case(lens, H, Dh, 100 + i)
        kv = [max(1, n - 3) for n in lens] if i == 1 else None
        want = _run("sj_attn", qkv, cu, H, Dh, window, kv)
        got = _run("sj_attn_noalloc", qkv, cu, H, Dh, window, kv)
        tol = 4.0 * 2.0 ** -8 * np.maximum(1.0, np.abs(want))
        assert (np.abs(got - want) <= tol).all(), np.abs(got - want).max()


def test_noalloc_rejects_batches_over_capacity():
    L = _lib.lib()
    cu = np.arange(0, 65537 * 2, 2, dtype=np.int32)  # 65536 one-tile sequences + 1
    cu = np.concatenate([cu, [cu[-1] + 2]]).astype(np.int32)
    rc = L.sj_attn_noalloc(None, None, C.c_void_p(cu.ctypes.data), None, None, len(cu) - 1, 12,
                           64, 0, None)
    assert rc == _lib.SJ_ERR_INVALID
    assert b"capacity" in L.sj_last_error()
