"""Failure detection on the GPU: a bounded device-side wait that runs out.

Every mbarrier wait in the tensor-core kernels gives up after about 2 s; the
kernel then records a code, stops issuing, waits for its own copies, frees its
tensor memory and returns.  These tests make one wait run out without any
fault: the test hook ``sj_test_attn_wait_timeout`` makes the attention kernel
issue no TMA load, so the first wait on the Q tile waits for a barrier that
nothing completes.  Nothing is in flight when the kernel leaves, and the
context stays usable; the tests check that

* the kernel-level entry points (``sj_attn``, ``sj_attn_noalloc``) report the
  failure through ``sj_check_device_errors`` (SJ_ERR_TIMEOUT, message), the
  way the reference's C API reports failures as a status plus a message
  (src/capi.cpp:89-93);
* the engine (``sj_fast_encode``) returns SJ_ERR_TIMEOUT from the call;
* with the hook off again, the same calls give the correct results.
"""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle  # noqa: E402
from snapjudge_b200 import _lib, ops, synth  # noqa: E402
from snapjudge_b200.fast import FastSnapjudge, SnapjudgeError  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _inputs(H=4, lens=(100, 37, 200)):
    lens = np.asarray(lens)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    T = int(cu[-1])
    x = np.random.default_rng(5).standard_normal((T, 3 * H * 64), dtype=np.float32)
    qkv = torch.from_numpy(x).to(DEV).to(torch.bfloat16)
    return qkv, cu, lens, H


def _oracle(qkv, lens, H):
    T = qkv.shape[0]
    x = qkv.float().cpu().numpy().reshape(T, 3, H, 64)
    return oracle.attention_packed(x[:, 0], x[:, 1], x[:, 2], lens)


class _Hook:
    def __enter__(self):
        _lib.lib().sj_test_attn_wait_timeout(1)

    def __exit__(self, *exc):
        _lib.lib().sj_test_attn_wait_timeout(0)
        return False


def test_kernel_entry_points_report_a_wait_that_ran_out():
    L = _lib.lib()
    qkv, cu, lens, H = _inputs()
    assert L.sj_check_device_errors(_stream()) == _lib.SJ_OK  # nothing recorded so far
    cu_d = torch.from_numpy(cu).to(DEV)
    for name in ("sj_attn", "sj_attn_noalloc"):
        O = torch.zeros(qkv.shape[0], H * 64, dtype=torch.bfloat16, device=DEV)
        with _Hook():
            rc = getattr(L, name)(C.c_void_p(qkv.data_ptr()), C.c_void_p(cu_d.data_ptr()),
                                  C.c_void_p(cu.ctypes.data), None, C.c_void_p(O.data_ptr()),
                                  len(lens), H, 64, 0, _stream())
            assert rc == _lib.SJ_OK  # queued: the failure happens later, on the device
            rc = L.sj_check_device_errors(_stream())
        assert rc == _lib.SJ_ERR_TIMEOUT, name
        assert b"attention" in L.sj_last_error()
        # the word was cleared by the check; the context still works
        assert L.sj_check_device_errors(_stream()) == _lib.SJ_OK
    O = ops.attn(qkv, cu, H, 64)
    assert L.sj_check_device_errors(_stream()) == _lib.SJ_OK
    want = _oracle(qkv, lens, H)
    got = O.float().cpu().numpy().reshape(want.shape)
    tol = 4.0 * 2.0 ** -8 * np.maximum(1.0, np.abs(want))
    assert (np.abs(got - want) <= tol).all()


def test_engine_call_returns_timeout_and_recovers():
    cfg = synth._enc(128, 2, 256, 1000, 2)  # head_dim 64: the tensor-core attention
    spec = synth.SynthSpec("timeout", cfg, 11, [synth.TaskHead("choice3", 3, synth.SOFTMAX)], 3,
                           "uniform:5:40", "bf16")
    t = synth.make_weights(spec)
    lengths = np.array([130, 7, 64])
    ids = synth.make_ids(spec, lengths, seed=12)
    eng = FastSnapjudge(cfg, t, precision="bf16", heads=spec.heads)
    good = eng.encode_packed(ids, lengths)
    with _Hook():
        with pytest.raises(SnapjudgeError) as ei:
            eng.encode_packed(ids, lengths)
    assert ei.value.code == _lib.SJ_ERR_TIMEOUT
    assert "attention" in str(ei.value)
    # the next call on the same engine runs normally and gives the same bits
    np.testing.assert_array_equal(eng.encode_packed(ids, lengths), good)
    want = oracle.Oracle(cfg, t).encode_packed(ids, lengths)
    assert np.abs(good - want).max() <= 6e-2
