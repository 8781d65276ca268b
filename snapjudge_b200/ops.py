"""Kernel-level entry points on torch device tensors.

Thin wrappers over the C ABI launchers (``sj_gemm``, ``sj_gemm_geglu``,
``sj_add_ln``, ``sj_rope``, ``sj_attn``), the varlen forms of the reference's
``cuda/kernels.cu`` entry points.  Tensors must be contiguous CUDA tensors of
the documented dtypes; the launch is asynchronous on torch's current stream.
torch is used only to own device memory and streams.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _lib
from ._lib import check


def _p(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _need(t, dtype, name):
    if not (t.is_cuda and t.dtype == dtype and t.is_contiguous()):
        raise ValueError(f"{name} must be a contiguous CUDA {dtype} tensor")


def gemm(A, W, bias=None, act=0):
    """bf16 C[M,N] = act(A[M,K] W[N,K]^T + bias)."""
    _need(A, torch.bfloat16, "A")
    _need(W, torch.bfloat16, "W")
    M, K = A.shape
    N = W.shape[0]
    C_ = torch.empty(M, N, dtype=torch.bfloat16, device=A.device)
    if bias is not None:
        _need(bias, torch.float32, "bias")
    check(_lib.lib().sj_gemm(_p(A), _p(W), _p(bias), _p(C_), M, N, K, int(bias is not None), act,
                             _stream()))
    return C_


def gemm_geglu(A, Wi):
    """bf16 C[M,F] = gelu(A Wi[:F]^T) * (A Wi[F:]^T)."""
    _need(A, torch.bfloat16, "A")
    _need(Wi, torch.bfloat16, "Wi")
    M, K = A.shape
    F = Wi.shape[0] // 2
    C_ = torch.empty(M, F, dtype=torch.bfloat16, device=A.device)
    check(_lib.lib().sj_gemm_geglu(_p(A), _p(Wi), _p(C_), M, F, K, _stream()))
    return C_


def add_ln(X, R, w, b=None, eps=1e-5):
    """X (fp32, in place) += R (bf16, optional); returns Y = LN(X) * w (+ b), bf16."""
    _need(X, torch.float32, "X")
    M, D = X.shape
    Y = torch.empty(M, D, dtype=torch.bfloat16, device=X.device)
    if R is not None:
        _need(R, torch.bfloat16, "R")
    check(_lib.lib().sj_add_ln(_p(X), _p(R), _p(w), _p(b), _p(Y), M, D, eps, int(R is not None),
                               int(b is not None), _stream()))
    return Y


def rope_(qkv, cos_t, sin_t, cu, H, Dh):
    """In-place RoPE on packed bf16 qkv [T, 3*H*Dh]; cu int32 cumulative lengths (host array)."""
    _need(qkv, torch.bfloat16, "qkv")
    cu_h = np.ascontiguousarray(cu, np.int32)
    cu_d = torch.from_numpy(cu_h).to(qkv.device)
    check(_lib.lib().sj_rope(_p(qkv), _p(cos_t), _p(sin_t), _p(cu_d),
                             C.c_void_p(cu_h.ctypes.data), len(cu_h) - 1, H, Dh, _stream()))
    return qkv


def attn(qkv, cu, H, Dh, window=0, kv_lens=None):
    """Packed varlen attention: bf16 qkv [T, 3*H*Dh] -> O [T, H*Dh]."""
    _need(qkv, torch.bfloat16, "qkv")
    cu_h = np.ascontiguousarray(cu, np.int32)
    cu_d = torch.from_numpy(cu_h).to(qkv.device)
    kv = None
    if kv_lens is not None:
        kv = torch.from_numpy(np.ascontiguousarray(kv_lens, np.int32)).to(qkv.device)
    T = int(cu_h[-1])
    O = torch.empty(T, H * Dh, dtype=torch.bfloat16, device=qkv.device)
    check(_lib.lib().sj_attn(_p(qkv), _p(cu_d), C.c_void_p(cu_h.ctypes.data), _p(kv), _p(O),
                             len(cu_h) - 1, H, Dh, window, _stream()))
    return O


def quant_e4m3(x):
    """fp32 x[rows, cols] -> (e4m3 codes uint8 [rows, cols], fp32 row scales [rows])."""
    _need(x, torch.float32, "x")
    rows, cols = x.shape
    q = torch.empty(rows, cols, dtype=torch.uint8, device=x.device)
    s = torch.empty(rows, dtype=torch.float32, device=x.device)
    check(_lib.lib().sj_quant_e4m3(_p(x), rows, cols, _p(q), _p(s), _stream()))
    return q, s


def gemm_e4m3(A, sa, W, sw, bias=None, act=0, geglu=False):
    """bf16 C[M,N] = act(sa sw (A W^T) + bias) on e4m3 codes A [M,K], W [N,K]
    (geglu: W = [Wg; Wu] [2N, K], C = gelu(g) * u)."""
    _need(A, torch.uint8, "A")
    _need(W, torch.uint8, "W")
    _need(sa, torch.float32, "sa")
    _need(sw, torch.float32, "sw")
    M, K = A.shape
    N = W.shape[0] // 2 if geglu else W.shape[0]
    C_ = torch.empty(M, N, dtype=torch.bfloat16, device=A.device)
    if bias is not None:
        _need(bias, torch.float32, "bias")
    check(_lib.lib().sj_gemm_e4m3(_p(A), _p(W), _p(sa), _p(sw), _p(bias), _p(C_), M, N, K,
                                  int(bias is not None), act, int(geglu), _stream()))
    return C_
