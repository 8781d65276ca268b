"""FastSnapjudge — host-side mirror of the reference's CUDA fast path.

Mirrors ``snapjudge::FastSnapjudge`` (include/snapjudge/fast.hpp:15-31) and the
encoder entry point it accelerates, ``DecisionModel::encode``
(src/model.cpp:222-307), over the C ABI of ``libsnapjudge_b200.so``:

* ``encode(input_ids, attention_mask)`` — the reference signature: a
  right-padded ``[B, L]`` batch in, ``[B, L, D]`` final-norm hidden states out,
  padded rows included (they attend the valid keys, as in the reference).
* ``encode_packed(ids, lengths)`` — packed variable-length form: only valid
  rows are computed.
* ``decide(ids, lengths)`` — encoder + decision heads on the [CLS] rows.
* ``encode_device(...)`` — the same on caller-owned device buffers (torch
  tensors), asynchronous on a CUDA stream.

Errors raise :class:`SnapjudgeError` carrying the library's message, the way
the reference throws ``std::runtime_error("snapjudge CUDA: ...")``.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib
from ._lib import SnapjudgeError, check  # noqa: F401  (re-exported)
from .checkpoint import EncoderConfig, SjConfig, load_checkpoint, load_sj_checkpoint

_I64P = C.POINTER(C.c_int64)


def _ptr(a: np.ndarray):
    return C.c_void_p(a.ctypes.data) if a is not None else None


class FastSnapjudge:
    """One encoder engine resident on one GPU."""

    def __init__(self, cfg: EncoderConfig | SjConfig, tensors: dict[str, np.ndarray], *,
                 precision: str = "bf16", heads=None, device: int = 0, max_tokens: int = 0):
        """`cfg` is a DecisionModel encoder config (``EncoderConfig``, tensors
        "encoder.*" ...) or an SjModel config (``SjConfig``, tensors "sj.*")."""
        L = _lib.lib()
        self.cfg = cfg
        self.precision = precision
        self.D = cfg.hidden_size
        prec = {"bf16": _lib.SJ_PREC_BF16, "fp32": _lib.SJ_PREC_FP32,
                "fp8": _lib.SJ_PREC_FP8,
                "fp8_tensor": _lib.SJ_PREC_FP8_TENSOR}.get(precision, -1)
        if isinstance(cfg, SjConfig):
            sl = None
            c = _lib.FastConfig(cfg.hidden_size, cfg.num_layers, cfg.num_heads,
                                cfg.intermediate_size, cfg.vocab_size, cfg.max_positions,
                                cfg.norm_eps, 0, sl, 10000.0, 10000.0, prec, device, max_tokens,
                                _lib.SJ_ARCH_SJMODEL)
        else:
            sl = (C.c_int * max(1, cfg.num_hidden_layers))(
                *[int(cfg.layer_sliding(i)) for i in range(cfg.num_hidden_layers)])
            c = _lib.FastConfig(cfg.hidden_size, cfg.num_hidden_layers, cfg.num_attention_heads,
                                cfg.intermediate_size, cfg.vocab_size, cfg.max_position_embeddings,
                                cfg.norm_eps, cfg.local_attention, sl, cfg.rope_theta_full,
                                cfg.rope_theta_sliding, prec, device, max_tokens,
                                _lib.SJ_ARCH_MODERNBERT)
        if prec < 0:
            raise ValueError("precision must be 'bf16', 'fp32', 'fp8' or 'fp8_tensor', "
                             f"got {precision!r}")
        h = C.c_void_p()
        rc = L.sj_fast_create(C.byref(c), C.byref(h))
        if rc != 0:
            raise SnapjudgeError(rc, "sj_fast_create failed (invalid config or CUDA error)")
        self._h = h
        self.heads = list(heads or [])
        self.n_out = sum(hd.n_out for hd in self.heads)
        try:
            for name, t in tensors.items():
                a = np.ascontiguousarray(t, dtype=np.float32)
                shape = (C.c_int64 * max(1, a.ndim))(*a.shape)
                check(L.sj_fast_set_tensor(h, name.encode(), _ptr(a), shape, a.ndim), h)
            if self.heads:
                n = (C.c_int * len(self.heads))(*[hd.n_out for hd in self.heads])
                k = (C.c_int * len(self.heads))(*[hd.kind for hd in self.heads])
                check(L.sj_fast_set_heads(h, len(self.heads), n, k), h)
            check(L.sj_fast_commit(h), h)
        except Exception:
            self.close()
            raise

    @classmethod
    def from_checkpoint(cls, path: str, **kw) -> "FastSnapjudge":
        cfg, tensors = load_checkpoint(path)
        return cls(cfg, tensors, **kw)

    @classmethod
    def from_sj_checkpoint(cls, path: str, **kw) -> "FastSnapjudge":
        """An SjModel directory (sj_config.json + model.safetensors)."""
        cfg, tensors = load_sj_checkpoint(path)
        return cls(cfg, tensors, **kw)

    def close(self) -> None:
        if getattr(self, "_h", None):
            try:
                _lib.lib().sj_fast_destroy(self._h)
            except TypeError:  # interpreter shutdown: the bindings are gone already
                pass
            self._h = None

    def __del__(self):
        self.close()

    # -- host buffers ------------------------------------------------------
    def encode_packed(self, ids, lengths, kv_lens=None) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int64)
        lengths = np.asarray(lengths, dtype=np.int64)
        cu = np.zeros(len(lengths) + 1, np.int32)
        np.cumsum(lengths, out=cu[1:])
        out = np.empty((int(cu[-1]), self.D), np.float32)
        kvl = None if kv_lens is None else np.ascontiguousarray(kv_lens, np.int32)
        check(_lib.lib().sj_fast_encode(self._h, _ptr(ids), _ptr(cu), _ptr(kvl), len(lengths),
                                        _ptr(out)), self._h)
        return out

    def encode(self, input_ids, attention_mask) -> np.ndarray:
        """DecisionModel::encode: padded [B, L] ids + mask -> [B, L, D]."""
        ids = np.ascontiguousarray(input_ids, dtype=np.int64)
        mask = np.asarray(attention_mask, dtype=np.int64)
        B, L = ids.shape
        lens = mask.sum(axis=1).astype(np.int32)
        out = self.encode_packed(ids.reshape(-1), np.full(B, L, np.int64), kv_lens=lens)
        return out.reshape(B, L, self.D)

    def embed_packed(self, ids, lengths) -> np.ndarray:
        """Mean-pooled final hidden states per segment, [B, D] (zeros for an
        empty segment); pooled on the device."""
        ids = np.ascontiguousarray(ids, dtype=np.int64)
        lengths = np.asarray(lengths, dtype=np.int64)
        cu = np.zeros(len(lengths) + 1, np.int32)
        np.cumsum(lengths, out=cu[1:])
        out = np.empty((len(lengths), self.D), np.float32)
        check(_lib.lib().sj_fast_embed(self._h, _ptr(ids), _ptr(cu), len(lengths), _ptr(out)),
              self._h)
        return out

    def embed(self, input_ids, attention_mask) -> np.ndarray:
        """Agent::embed's pooling (src/agent.cpp:315-357) on a tokenised,
        right-padded batch: the mean of each row's final hidden states over its
        valid positions, [B, D].  Valid rows do not see the padding, so the
        batch is packed to them first."""
        ids = np.ascontiguousarray(input_ids, dtype=np.int64)
        lens = np.asarray(attention_mask, dtype=np.int64).sum(axis=1)
        rows = np.arange(ids.shape[1])[None, :] < lens[:, None]
        return self.embed_packed(ids[rows], lens)

    @property
    def n_act(self) -> int:
        """Outputs of the act head (0 without a decision-model head)."""
        return int(_lib.lib().sj_fast_n_act(self._h))

    def forward(self, input_ids, attention_mask, marker_pos, marker_mask, qtype, pack=None):
        """DecisionModel::forward (src/model.cpp:309-536) on the GPU: padded
        [B, L] ids + mask, marker_pos / marker_mask [B, K], qtype [B] ->
        (logits [B, K], act [B, n_act]).

        The outputs depend on the padded rows only through a live marker that
        points past its row's length (the reference gathers that padded row).
        Without one, the batch is packed to its valid rows (``pack=None``:
        decided per batch; True / False force it), which gives the same
        outputs without computing the padding."""
        ids = np.ascontiguousarray(input_ids, dtype=np.int64)
        mask = np.asarray(attention_mask, dtype=np.int64)
        B, L = ids.shape
        pos = np.ascontiguousarray(marker_pos, dtype=np.int64)
        mm = np.ascontiguousarray(marker_mask, dtype=np.uint8)
        qt = np.ascontiguousarray(qtype, dtype=np.int64)
        K = pos.shape[1] if pos.ndim == 2 else 0
        if pos.shape != (B, K) or mm.shape != (B, K) or qt.shape != (B,):
            raise ValueError("marker_pos / marker_mask must be [B, K] and qtype [B]")
        lens = mask.sum(axis=1)
        if pack is None:
            gathered = np.clip(pos, 0, L - 1)
            pack = bool((lens >= 1).all() and not ((mm != 0) & (gathered >= lens[:, None])).any())
        if pack:
            rows = np.arange(L)[None, :] < lens[:, None]
            flat = np.ascontiguousarray(ids[rows])
            cu = np.zeros(B + 1, np.int32)
            np.cumsum(lens, out=cu[1:])
            kvl = None
        else:
            flat = ids
            cu = (np.arange(B + 1, dtype=np.int64) * L).astype(np.int32)
            kvl = np.ascontiguousarray(lens, dtype=np.int32)
        logits = np.empty((B, K), np.float32)
        act = np.empty((B, max(1, self.n_act)), np.float32)
        check(_lib.lib().sj_fast_forward(self._h, _ptr(flat), _ptr(cu), _ptr(kvl), B, _ptr(pos),
                                         _ptr(mm), K, _ptr(qt), _ptr(logits), _ptr(act)), self._h)
        return logits, act[:, :self.n_act]

    def decide(self, ids, lengths, out: np.ndarray | None = None, cu=None) -> np.ndarray:
        """Encoder + heads; probs [B, sum n_out].  `out` / `cu` may be preallocated
        (e.g. pinned) host arrays: float32 [B, n_out] and int32 [B + 1]."""
        ids = np.ascontiguousarray(ids, dtype=np.int64)
        lengths = np.asarray(lengths, dtype=np.int64)
        if cu is None:
            cu = np.zeros(len(lengths) + 1, np.int32)
            np.cumsum(lengths, out=cu[1:])
        if out is None:
            out = np.empty((len(lengths), max(1, self.n_out)), np.float32)
        check(_lib.lib().sj_fast_decide(self._h, _ptr(ids), _ptr(cu), len(lengths), _ptr(out)),
              self._h)
        return out

    def split_heads(self, probs: np.ndarray) -> list[np.ndarray]:
        out, off = [], 0
        for hd in self.heads:
            out.append(probs[:, off:off + hd.n_out])
            off += hd.n_out
        return out

    # -- device buffers (torch tensors) --------------------------------------
    def encode_device(self, ids, cu, cu_host: np.ndarray, *, kv_lens=None, hidden=None,
                      probs=None, stream=None) -> None:
        """Asynchronous forward on device tensors (int64 ids, int32 cu/kv_lens)."""
        cu_host = np.ascontiguousarray(cu_host, np.int32)
        self._cu_host = cu_host  # must outlive the launch (the schedule reads it now)
        dp = lambda t: None if t is None else C.c_void_p(t.data_ptr())  # noqa: E731
        st = None if stream is None else C.c_void_p(stream.cuda_stream)
        check(_lib.lib().sj_fast_encode_device(self._h, dp(ids), dp(cu), _ptr(cu_host),
                                               dp(kv_lens), len(cu_host) - 1, dp(hidden),
                                               dp(probs), st), self._h)

    def sync(self, stream=None) -> None:
        st = None if stream is None else C.c_void_p(stream.cuda_stream)
        check(_lib.lib().sj_fast_sync(self._h, st), self._h)

    def launch_count(self) -> int:
        return _lib.lib().sj_fast_launch_count(self._h)

    def reset_calibration(self) -> None:
        """fp8_tensor: the next call calibrates the activation scales again, on
        its own batch."""
        check(_lib.lib().sj_fast_reset_calibration(self._h), self._h)

    def set_profiling(self, enable: bool) -> None:
        check(_lib.lib().sj_fast_set_profiling(self._h, int(enable)), self._h)

    def profile(self, reset: bool = True) -> dict[str, tuple[float, int]]:
        """{kernel class: (total ms, launches)} accumulated since the last reset."""
        n = len(_lib.KERNEL_CLASSES)
        ms = (C.c_double * n)()
        cnt = (C.c_int64 * n)()
        check(_lib.lib().sj_fast_profile(self._h, ms, cnt, int(reset)), self._h)
        return {k: (ms[i], cnt[i]) for i, k in enumerate(_lib.KERNEL_CLASSES)}
