"""Python bindings for the parity checkers.  TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline / reference
legs of ``bench.py`` import this module.  The product path
(``snapjudge_b200``) never does.

Two checkers:

* :class:`Oracle` — ``lib/liboracle.so``, the C restatement of the reference
  fp32 forward (``sj_oracle.c``; each C function cites the reference lines it
  follows).
* :class:`RefModel` — ``_ref/libsjref.so``, the reference's own
  ``src/model.cpp``/``src/tensor.cpp``/``src/safetensors.cpp`` compiled
  unchanged (``Makefile``), used to pin the restatement and as the timed
  reference CPU baseline.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_F = C.POINTER(C.c_float)
_I64 = C.POINTER(C.c_int64)
_U8 = C.POINTER(C.c_uint8)


def reference_tree() -> str | None:
    """The snapjudge reference checkout the _ref checkers compile from:
    $SNAPJUDGE_REFERENCE, else a directory named "reference" beside this
    repository; None when neither holds src/model.cpp."""
    cands = [os.environ.get("SNAPJUDGE_REFERENCE"),
             os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")]
    for c in cands:
        if c and os.path.exists(os.path.join(c, "src", "model.cpp")):
            return c
    return None


def build() -> None:
    """Build the checkers (make; the _ref part only where the reference tree exists)."""
    args = ["make", "-s", "-C", HERE, "all"]
    ref = reference_tree()
    if ref:
        args.append(f"REF={ref}")
    blas = find_openblas()
    if blas:
        args.append(f"OPENBLAS={blas}")
    subprocess.run(args, check=True)


def _fp(a):
    return None if a is None else a.ctypes.data_as(_F)


def _ip(a):
    return None if a is None else a.ctypes.data_as(_I64)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


# ------------------------------------------------------------------ restatement
class _Layer(C.Structure):
    _fields_ = [("attn_norm", _F), ("wqkv", _F), ("wo", _F), ("mlp_norm", _F), ("wi", _F),
                ("wo2", _F), ("window", C.c_int), ("sliding", C.c_int)]


class _Model(C.Structure):
    _fields_ = [("D", C.c_int), ("H", C.c_int), ("F", C.c_int), ("V", C.c_int),
                ("n_layers", C.c_int), ("max_pos", C.c_int64), ("eps", C.c_float),
                ("emb", _F), ("emb_norm", _F), ("final_norm", _F),
                ("layers", C.POINTER(_Layer)),
                ("cos_full", _F), ("sin_full", _F), ("cos_slide", _F), ("sin_slide", _F),
                ("lora_r", C.c_int), ("lora_a", _F), ("lora_b", _F)]


class _HeadLayer(C.Structure):
    _fields_ = [(n, _F) for n in ("n1w", "n1b", "n2w", "n2b", "in_w", "in_b", "out_w",
                                  "out_b", "l1w", "l1b", "l2w", "l2b")]


class _Head(C.Structure):
    _fields_ = [("type_emb", _F), ("n_head_layers", C.c_int),
                ("head", C.POINTER(_HeadLayer)),
                ("sc_ln_w", _F), ("sc_ln_b", _F), ("sc_w1", _F), ("sc_b1", _F),
                ("sc_w2", _F), ("sc_b2", _F),
                ("act_w1", _F), ("act_b1", _F), ("act_w2", _F), ("act_b2", _F),
                ("n_act", C.c_int)]


_LIB = None


def _lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(HERE, "lib", "liboracle.so")
        if not os.path.exists(path):
            build()
        lib = C.CDLL(path)
        lib.orc_layer_norm.argtypes = [_F, C.c_int64, C.c_int64, _F, _F, C.c_float, _F]
        lib.orc_gemm_nt.argtypes = [_F, C.c_int64, C.c_int64, _F, C.c_int64, _F, C.c_int, _F]
        lib.orc_geglu.argtypes = [_F, C.c_int64, C.c_int64, _F, C.c_int64, _F]
        lib.orc_rope_table.argtypes = [C.c_double, C.c_int, C.c_int64, _F, _F]
        lib.orc_rope.argtypes = [_F, C.c_int64, _F, _F, C.c_int64, C.c_int64, C.c_int64]
        lib.orc_attention.argtypes = [_F, _F, _F, C.c_int64, C.c_int64, C.c_int64, C.c_int64,
                                      _I64, C.c_int, _F]
        lib.orc_encode.argtypes = [C.POINTER(_Model), _I64, _I64, C.c_int64, C.c_int64, _F]
        lib.orc_encode.restype = C.c_int
        lib.orc_forward_head.argtypes = [C.POINTER(_Model), C.POINTER(_Head), _F, _I64,
                                         C.c_int64, C.c_int64, _I64, _U8, C.c_int64, _I64,
                                         _F, _F]
        lib.orc_set_blas.argtypes = [C.c_char_p]
        lib.orc_set_threads.argtypes = [C.c_int]
        _LIB = lib
    return _LIB


def set_blas(path: str | None = None) -> bool:
    """Route the oracle's GEMMs through a shared BLAS (the reference's OpenBLAS)."""
    if path is None:
        path = find_openblas()
    if not path:
        return False
    return _lib().orc_set_blas(path.encode()) == 0


def find_openblas() -> str | None:
    """The OpenBLAS the reference is timed with: $SNAPJUDGE_OPENBLAS, else the
    copy bundled with opencv-python-headless in this interpreter's
    site-packages (OpenBLAS 0.3.15, which exports cblas_sgemm)."""
    import glob
    import site
    env = os.environ.get("SNAPJUDGE_OPENBLAS")
    if env and os.path.exists(env):
        return env
    dirs = list(site.getsitepackages()) + [site.getusersitepackages()]
    for d in dirs:
        g = sorted(glob.glob(os.path.join(d, "opencv_python_headless.libs",
                                          "libopenblasp-r0-*.so")))
        if g:
            return g[0]
    return None


def set_threads(n: int) -> None:
    _lib().orc_set_threads(int(n))


# ---- op-level wrappers (restatement) ----
def layer_norm(x, w, b, eps=1e-5):
    x = _f32(x)
    D = x.shape[-1]
    out = np.empty_like(x)
    _lib().orc_layer_norm(_fp(x), x.size // D, D, _fp(_f32(w)) if w is not None else None,
                          _fp(_f32(b)) if b is not None else None, eps, _fp(out))
    return out


def gemm_nt(a, w, bias=None, act=0):
    a, w = _f32(a), _f32(w)
    M, K = a.shape
    N = w.shape[0]
    out = np.empty((M, N), np.float32)
    bb = _f32(bias) if bias is not None else None
    _lib().orc_gemm_nt(_fp(a), M, K, _fp(w), N, _fp(bb), act, _fp(out))
    return out


def geglu(a, wi):
    a, wi = _f32(a), _f32(wi)
    M, K = a.shape
    F = wi.shape[0] // 2
    out = np.empty((M, F), np.float32)
    _lib().orc_geglu(_fp(a), M, K, _fp(wi), F, _fp(out))
    return out


def rope_table(theta, Dh, L):
    c = np.empty((L, Dh // 2), np.float32)
    s = np.empty((L, Dh // 2), np.float32)
    _lib().orc_rope_table(float(theta), int(Dh), int(L), _fp(c), _fp(s))
    return c, s


def rope(qkv, cos_t, sin_t, L, H, Dh):
    q = _f32(qkv).copy()
    _lib().orc_rope(_fp(q), q.shape[0], _fp(_f32(cos_t)), _fp(_f32(sin_t)), L, H, Dh)
    return q


def attention(q, k, v, lens=None, window=0):
    """q/k/v [B, H, L, Dh] fp32 -> [B, H, L, Dh]."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    B, H, L, Dh = q.shape
    out = np.empty_like(q)
    ln = None if lens is None else np.ascontiguousarray(lens, dtype=np.int64)
    _lib().orc_attention(_fp(q), _fp(k), _fp(v), B, H, L, Dh, _ip(ln), window, _fp(out))
    return out


def attention_packed_np(q, k, v, lengths, window=0, kv_lens=None, dtype=np.float64):
    """attention_packed restated with matrix products (NumPy BLAS), for
    segments too long for the scalar C loop: per (segment, head) the same
    steps as src/tensor.cpp:156-228 — scores q.k / sqrt(Dh) over keys
    [max(0, i - w), min(kv_len, i + w + 1)) (w = 0: [0, kv_len)), max
    subtracted, exponentials summed, o = sum p v / sum p; no visible key
    gives 0.  q/k/v [T, H, Dh]; returns float32 [T, H, Dh].  Pinned against
    the C restatement in tests/test_oracle.py.  dtype float32 halves the time
    of the largest cases (its error, ~1e-6 relative, is far below the bf16
    bars it checks)."""
    q = np.asarray(q, dtype)
    k = np.asarray(k, dtype)
    v = np.asarray(v, dtype)
    T, H, Dh = q.shape
    out = np.zeros((T, H, Dh), np.float32)
    cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    scale = 1.0 / np.sqrt(np.float32(Dh))
    for b in range(len(lengths)):
        s0, e = int(cu[b]), int(cu[b + 1])
        n = e - s0
        if n == 0:
            continue
        nk = n if kv_lens is None else min(int(kv_lens[b]), n)
        if nk == 0:
            continue
        i = np.arange(n)[:, None]
        j = np.arange(nk)[None, :]
        vis = np.ones((n, nk), bool) if window <= 0 else (np.abs(i - j) <= window)
        for h in range(H):
            s = (q[s0:e, h] @ k[s0:s0 + nk, h].T) * scale
            s = np.where(vis, s, -np.inf)
            m = s.max(1, keepdims=True)
            m = np.where(np.isfinite(m), m, 0.0)
            p = np.where(vis, np.exp(s - m), 0.0)
            lsum = p.sum(1, keepdims=True)
            o = (p @ v[s0:s0 + nk, h]) / np.where(lsum > 0, lsum, 1.0)
            out[s0:e, h] = o.astype(np.float32)
    return out


def attention_packed(q, k, v, lengths, window=0, kv_lens=None):
    """Packed varlen attention: q/k/v [T, H, Dh]; one segment per sequence."""
    out = np.empty_like(_f32(q))
    cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    for b in range(len(lengths)):
        s, e = int(cu[b]), int(cu[b + 1])
        if e == s:
            continue
        kl = None if kv_lens is None else np.array([kv_lens[b]], np.int64)
        qb = q[s:e].transpose(1, 0, 2)[None]
        kb = k[s:e].transpose(1, 0, 2)[None]
        vb = v[s:e].transpose(1, 0, 2)[None]
        ob = attention(qb, kb, vb, kl, window)
        out[s:e] = ob[0].transpose(1, 0, 2)
    return out


# ---- model-level (restatement) ----
class Oracle:
    """The C restatement holding one checkpoint's fp32 weights."""

    def __init__(self, cfg, tensors: dict[str, np.ndarray]):
        self.cfg = cfg
        self.t = {k: _f32(v) for k, v in tensors.items()}
        c = cfg
        D, H = c.hidden_size, c.num_attention_heads
        Dh = D // H
        self._keep = []
        self.cos_f, self.sin_f = rope_table(c.rope_theta_full, Dh, c.max_position_embeddings)
        self.cos_s, self.sin_s = rope_table(c.rope_theta_sliding, Dh, c.max_position_embeddings)
        layers = (_Layer * c.num_hidden_layers)()
        for i in range(c.num_hidden_layers):
            p = f"encoder.layers.{i}."
            an = self.t.get(p + "attn_norm.weight")
            layers[i] = _Layer(_fp(an), _fp(self.t[p + "attn.Wqkv.weight"]),
                               _fp(self.t[p + "attn.Wo.weight"]),
                               _fp(self.t[p + "mlp_norm.weight"]),
                               _fp(self.t[p + "mlp.Wi.weight"]), _fp(self.t[p + "mlp.Wo.weight"]),
                               c.layer_window(i), int(c.layer_sliding(i)))
        self._layers = layers
        la, lb = self.t.get("lora_A.weight"), self.t.get("lora_B.weight")
        self._m = _Model(D, H, c.intermediate_size, c.vocab_size, c.num_hidden_layers,
                         c.max_position_embeddings, c.norm_eps,
                         _fp(self.t["encoder.embeddings.tok_embeddings.weight"]),
                         _fp(self.t["encoder.embeddings.norm.weight"]),
                         _fp(self.t["encoder.final_norm.weight"]),
                         layers, _fp(self.cos_f), _fp(self.sin_f), _fp(self.cos_s),
                         _fp(self.sin_s), 0 if la is None else la.shape[0], _fp(la), _fp(lb))

    def encode_padded(self, ids, mask):
        ids = np.ascontiguousarray(ids, np.int64)
        mask = np.ascontiguousarray(mask, np.int64)
        B, L = ids.shape
        out = np.empty((B, L, self.cfg.hidden_size), np.float32)
        rc = _lib().orc_encode(C.byref(self._m), _ip(ids), _ip(mask), B, L, _fp(out))
        if rc != 0:
            raise ValueError(f"orc_encode failed ({rc})")
        return out

    def encode_packed(self, ids, lengths):
        """Packed varlen: each sequence encoded alone (valid rows are batch-independent)."""
        D = self.cfg.hidden_size
        cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
        out = np.empty((int(cu[-1]), D), np.float32)
        for b in range(len(lengths)):
            s, e = int(cu[b]), int(cu[b + 1])
            if e == s:
                continue
            ids_b = np.asarray(ids[s:e], np.int64)[None]
            out[s:e] = self.encode_padded(ids_b, np.ones_like(ids_b))[0]
        return out

    def forward_padded(self, ids, mask, marker_pos, marker_mask, qtype):
        """Full DecisionModel forward: (logits [B, K], act [B, n_act])."""
        c, t = self.cfg, self.t
        h = self.encode_padded(ids, mask)
        B, L = np.asarray(ids).shape
        marker_pos = np.ascontiguousarray(marker_pos, np.int64)
        marker_mask = np.ascontiguousarray(marker_mask, np.uint8)
        qtype = np.ascontiguousarray(qtype, np.int64)
        K = marker_pos.shape[1]
        hl = (_HeadLayer * max(1, c.head_layers))()
        for i in range(c.head_layers):
            p = f"head.layers.{i}."
            hl[i] = _HeadLayer(*[_fp(t[p + s]) for s in (
                "norm1.weight", "norm1.bias", "norm2.weight", "norm2.bias",
                "self_attn.in_proj_weight", "self_attn.in_proj_bias",
                "self_attn.out_proj.weight", "self_attn.out_proj.bias",
                "linear1.weight", "linear1.bias", "linear2.weight", "linear2.bias")])
        n_act = t["act_head.2.weight"].shape[0]
        hd = _Head(_fp(t["type_emb.weight"]), c.head_layers, hl,
                   _fp(t["scorer.0.weight"]), _fp(t.get("scorer.0.bias")),
                   _fp(t["scorer.1.weight"]), _fp(t.get("scorer.1.bias")),
                   _fp(t["scorer.3.weight"]), _fp(t.get("scorer.3.bias")),
                   _fp(t["act_head.0.weight"]), _fp(t["act_head.0.bias"]),
                   _fp(t["act_head.2.weight"]), _fp(t["act_head.2.bias"]), n_act)
        logits = np.empty((B, K), np.float32)
        act = np.empty((B, n_act), np.float32)
        _lib().orc_forward_head(C.byref(self._m), C.byref(hd), _fp(h),
                                _ip(np.ascontiguousarray(mask, np.int64)), B, L,
                                _ip(marker_pos), marker_mask.ctypes.data_as(_U8), K,
                                _ip(qtype), _fp(logits), _fp(act))
        return logits, act


def embed_mean(hidden, mask):
    """Agent::embed's pooling (src/agent.cpp:347-354): per row, the fp32 sum of
    the hidden states at its valid positions in position order, divided by
    max(1, n).  hidden [B, L, D], mask [B, L] (right-padded) -> [B, D]."""
    hidden = np.asarray(hidden, np.float32)
    lens = np.asarray(mask).astype(np.int64).sum(axis=1)
    B, _, D = hidden.shape
    out = np.zeros((B, D), np.float32)
    for b in range(B):
        acc = np.zeros(D, np.float32)
        for i in range(int(lens[b])):
            acc += hidden[b, i]
        out[b] = acc / np.float32(max(1, int(lens[b])))
    return out


def task_heads(cls_hidden, tensors, heads):
    """Config decision heads on the [CLS] rows, fp64: list of [B, n_out] probabilities."""
    x = np.asarray(cls_hidden, np.float64)
    outs = []
    for i, h in enumerate(heads):
        w = np.asarray(tensors[f"task_heads.{i}.weight"], np.float64)
        b = np.asarray(tensors[f"task_heads.{i}.bias"], np.float64)
        z = x @ w.T + b
        if h.kind == 1:
            outs.append(1.0 / (1.0 + np.exp(-z)))
        else:
            z = z - z.max(axis=1, keepdims=True)
            e = np.exp(z)
            outs.append(e / e.sum(axis=1, keepdims=True))
    return outs


# ------------------------------------------------------------------ reference
_REF = {}


def ref_available(noblas: bool = False) -> bool:
    return os.path.exists(os.path.join(HERE, "_ref",
                                       "libsjref_noblas.so" if noblas else "libsjref.so"))


def _ref(noblas=False):
    key = bool(noblas)
    if key not in _REF:
        path = os.path.join(HERE, "_ref", "libsjref_noblas.so" if noblas else "libsjref.so")
        lib = C.CDLL(path)
        lib.sjref_load.argtypes = [C.c_char_p]
        lib.sjref_load.restype = C.c_void_p
        lib.sjref_last_error.restype = C.c_char_p
        lib.sjref_free.argtypes = [C.c_void_p]
        lib.sjref_n_act.argtypes = [C.c_void_p]
        lib.sjref_encode.argtypes = [C.c_void_p, _I64, _I64, C.c_int64, C.c_int64, _F]
        lib.sjref_forward.argtypes = [C.c_void_p, _I64, _I64, C.c_int64, C.c_int64, _I64, _U8,
                                      C.c_int64, _I64, _F, _F]
        lib.sjref_layer_norm.argtypes = [_F, C.c_int64, C.c_int64, _F, _F, C.c_float, _F]
        lib.sjref_gemm_nt.argtypes = [_F, C.c_int64, C.c_int64, _F, C.c_int64, _F, C.c_int, _F]
        lib.sjref_geglu.argtypes = [_F, C.c_int64, C.c_int64, _F, C.c_int64, _F]
        lib.sjref_attention.argtypes = [_F, _F, _F, C.c_int64, C.c_int64, C.c_int64, C.c_int64,
                                        _I64, C.c_int, _F]
        lib.sjref_rope.argtypes = [_F, C.c_int64, _F, _F, C.c_int64, C.c_int64, C.c_int64]
        lib.sjref_sj_load.argtypes = [C.c_char_p]
        lib.sjref_sj_load.restype = C.c_void_p
        lib.sjref_sj_free.argtypes = [C.c_void_p]
        lib.sjref_sj_encode.argtypes = [C.c_void_p, _I64, _I64, C.c_int64, C.c_int64,
                                        C.c_int64, _F]
        lib.sjref_sj_forward.argtypes = [C.c_void_p, _I64, _I64, C.c_int64, C.c_int64, _I64,
                                         _U8, C.c_int64, _I64, _F, _F]
        _REF[key] = lib
    return _REF[key]


class RefModel:
    """The reference DecisionModel, loaded from a checkpoint directory."""

    def __init__(self, ckpt_dir: str, noblas: bool = False):
        self.lib = _ref(noblas)
        self.h = self.lib.sjref_load(ckpt_dir.encode())
        if not self.h:
            raise RuntimeError(self.lib.sjref_last_error().decode())
        self.n_act = self.lib.sjref_n_act(self.h)

    def __del__(self):
        if getattr(self, "h", None):
            self.lib.sjref_free(self.h)
            self.h = None

    def encode(self, ids, mask, D):
        ids = np.ascontiguousarray(ids, np.int64)
        mask = np.ascontiguousarray(mask, np.int64)
        B, L = ids.shape
        out = np.empty((B, L, D), np.float32)
        if self.lib.sjref_encode(self.h, _ip(ids), _ip(mask), B, L, _fp(out)) != 0:
            raise RuntimeError(self.lib.sjref_last_error().decode())
        return out

    def forward(self, ids, mask, marker_pos, marker_mask, qtype):
        ids = np.ascontiguousarray(ids, np.int64)
        mask = np.ascontiguousarray(mask, np.int64)
        mp = np.ascontiguousarray(marker_pos, np.int64)
        mm = np.ascontiguousarray(marker_mask, np.uint8)
        qt = np.ascontiguousarray(qtype, np.int64)
        B, L = ids.shape
        K = mp.shape[1]
        logits = np.empty((B, K), np.float32)
        act = np.empty((B, self.n_act), np.float32)
        if self.lib.sjref_forward(self.h, _ip(ids), _ip(mask), B, L, _ip(mp),
                                  mm.ctypes.data_as(_U8), K, _ip(qt), _fp(logits),
                                  _fp(act)) != 0:
            raise RuntimeError(self.lib.sjref_last_error().decode())
        return logits, act


def _erf(x):
    """erf elementwise (math.erf on float64), as the reference's erff."""
    import math
    return np.vectorize(math.erf, otypes=[np.float64])(np.asarray(x, np.float64))


class SjOracle:
    """NumPy restatement of the SjModel forward (reference src/sj_model.cpp), fp32
    GEMMs with fp64 LN statistics and softmax sums like the reference's tensor ops:
    * embeddings: word[ids] + position[min(i, max_positions - 1)], LN with bias (:217-233);
    * per layer (:235-245): X += o(attn(LN_a(X))), X += w2(gelu(w1(LN_f(X))));
      attention with separate biased q/k/v/o (:40-88), keys j < lens[b];
    * final LN with bias (:246);
    * forward (:277-368): + type_emb[qtype], head layers of the same shape,
      scorer on the marker rows, act = [top1, 1 - top1]."""

    def __init__(self, cfg, tensors):
        self.cfg = cfg
        self.t = {k: np.asarray(v, np.float32) for k, v in tensors.items()}

    def _ln(self, x, name, eps=None):
        eps = self.cfg.norm_eps if eps is None else eps
        xd = x.astype(np.float64)
        mu = xd.mean(-1, keepdims=True)
        var = ((xd - mu) ** 2).mean(-1, keepdims=True)
        y = (xd - mu) / np.sqrt(var + eps)
        return (y * self.t[name + ".weight"] + self.t[name + ".bias"]).astype(np.float32)

    def _lin(self, x, name, act=0):
        y = x @ self.t[name + ".weight"].T + self.t[name + ".bias"]
        if act == 1:
            y = (0.5 * y * (1.0 + _erf(y / np.sqrt(2.0)))).astype(np.float32)
        return y.astype(np.float32)

    def _attn(self, Y, p, lens):
        B, L, D = Y.shape
        H = self.cfg.num_heads
        Dh = D // H
        q = self._lin(Y, p + "attn.q").reshape(B, L, H, Dh)
        k = self._lin(Y, p + "attn.k").reshape(B, L, H, Dh)
        v = self._lin(Y, p + "attn.v").reshape(B, L, H, Dh)
        s = np.einsum("bihd,bjhd->bhij", q, k) / np.float32(np.sqrt(Dh))
        keep = np.arange(L)[None, :] < np.asarray(lens)[:, None]       # [B, L] keys
        s = np.where(keep[:, None, None, :], s, -np.inf)
        m = s.max(-1, keepdims=True)
        e = np.exp((s - m).astype(np.float32))
        o = np.einsum("bhij,bjhd->bihd", e, v) / e.astype(np.float64).sum(-1)[..., None].transpose(0, 2, 1, 3)
        return self._lin(o.reshape(B, L, D).astype(np.float32), p + "attn.o")

    def _layer(self, X, p, lens, n1, n2):
        X = X + self._attn(self._ln(X, p + n1), p, lens)
        return X + self._lin(self._lin(self._ln(X, p + n2), p + "ffn.w1", 1), p + "ffn.w2")

    def encode_padded(self, ids, mask):
        c = self.cfg
        ids = np.asarray(ids, np.int64)
        B, L = ids.shape
        lens = np.asarray(mask, np.int64).sum(1)
        pos = np.minimum(np.arange(L), c.max_positions - 1)
        X = self.t["sj.embeddings.word.weight"][ids] + self.t["sj.embeddings.position.weight"][pos][None]
        X = self._ln(X, "sj.embeddings.norm")
        for i in range(c.num_layers):
            X = self._layer(X, f"sj.encoder.layers.{i}.", lens, "attn_norm", "ffn_norm")
        return self._ln(X, "sj.encoder.final_norm")

    def forward_padded(self, ids, mask, marker_pos, marker_mask, qtype):
        c = self.cfg
        h = self.encode_padded(ids, mask)
        B, L, D = h.shape
        lens = np.asarray(mask, np.int64).sum(1)
        h = h + self.t["sj.type_emb.weight"][np.asarray(qtype, np.int64)][:, None, :]
        for i in range(c.head_layers):
            h = self._layer(h, f"sj.head.layers.{i}.", lens, "norm1", "norm2")
        pos = np.clip(np.asarray(marker_pos, np.int64), 0, L - 1)
        m = h[np.arange(B)[:, None], pos]                                   # [B, K, D]
        s = self._lin(self._lin(self._ln(m, "sj.scorer.norm"), "sj.scorer.w1", 1), "sj.scorer.w2")
        logits = np.where(np.asarray(marker_mask) != 0, s[..., 0], np.float32(-1e4)).astype(np.float32)
        mx = logits.max(1, keepdims=True)
        e = np.exp((logits - mx).astype(np.float32)).astype(np.float64)
        top1 = (e / e.sum(1, keepdims=True)).max(1)
        return logits, np.stack([top1, 1.0 - top1], 1).astype(np.float32)


class RefSjModel:
    """The reference SjModel (src/sj_model.cpp), loaded from an sj_config.json +
    model.safetensors directory: encode (:257-275) and forward (:277-368)."""

    def __init__(self, ckpt_dir: str, hidden_size: int, noblas: bool = False):
        self.lib = _ref(noblas)
        self.D = hidden_size
        self.h = self.lib.sjref_sj_load(ckpt_dir.encode())
        if not self.h:
            raise RuntimeError(self.lib.sjref_last_error().decode())

    def __del__(self):
        if getattr(self, "h", None):
            self.lib.sjref_sj_free(self.h)
            self.h = None

    def encode(self, ids, mask):
        ids = np.ascontiguousarray(ids, np.int64)
        mask = np.ascontiguousarray(mask, np.int64)
        B, L = ids.shape
        out = np.empty((B, L, self.D), np.float32)
        if self.lib.sjref_sj_encode(self.h, _ip(ids), _ip(mask), B, L, self.D, _fp(out)) != 0:
            raise RuntimeError(self.lib.sjref_last_error().decode())
        return out

    def forward(self, ids, mask, marker_pos, marker_mask, qtype):
        ids = np.ascontiguousarray(ids, np.int64)
        mask = np.ascontiguousarray(mask, np.int64)
        mp = np.ascontiguousarray(marker_pos, np.int64)
        mm = np.ascontiguousarray(marker_mask, np.uint8)
        qt = np.ascontiguousarray(qtype, np.int64)
        B, L = ids.shape
        K = mp.shape[1]
        logits = np.empty((B, K), np.float32)
        act = np.empty((B, 2), np.float32)
        if self.lib.sjref_sj_forward(self.h, _ip(ids), _ip(mask), B, L, _ip(mp),
                                     mm.ctypes.data_as(_U8), K, _ip(qt), _fp(logits),
                                     _fp(act)) != 0:
            raise RuntimeError(self.lib.sjref_last_error().decode())
        return logits, act


def ref_layer_norm(x, w, b, eps=1e-5, noblas=False):
    x = _f32(x)
    D = x.shape[-1]
    out = np.empty_like(x)
    _ref(noblas).sjref_layer_norm(_fp(x), x.size // D, D, _fp(_f32(w)) if w is not None
                                  else None, _fp(_f32(b)) if b is not None else None, eps,
                                  _fp(out))
    return out


def ref_gemm_nt(a, w, bias=None, act=0, noblas=False):
    a, w = _f32(a), _f32(w)
    M, K = a.shape
    N = w.shape[0]
    out = np.empty((M, N), np.float32)
    _ref(noblas).sjref_gemm_nt(_fp(a), M, K, _fp(w), N,
                               _fp(_f32(bias)) if bias is not None else None, act, _fp(out))
    return out


def ref_geglu(a, wi, noblas=False):
    a, wi = _f32(a), _f32(wi)
    M, K = a.shape
    F = wi.shape[0] // 2
    out = np.empty((M, F), np.float32)
    _ref(noblas).sjref_geglu(_fp(a), M, K, _fp(wi), F, _fp(out))
    return out


def ref_attention(q, k, v, lens=None, window=0, noblas=False):
    q, k, v = _f32(q), _f32(k), _f32(v)
    B, H, L, Dh = q.shape
    out = np.empty_like(q)
    ln = None if lens is None else np.ascontiguousarray(lens, dtype=np.int64)
    _ref(noblas).sjref_attention(_fp(q), _fp(k), _fp(v), B, H, L, Dh, _ip(ln), window,
                                 _fp(out))
    return out


def ref_rope(qkv, cos_t, sin_t, L, H, Dh, noblas=False):
    q = _f32(qkv).copy()
    _ref(noblas).sjref_rope(_fp(q), q.shape[0], _fp(_f32(cos_t)), _fp(_f32(sin_t)), L, H, Dh)
    return q
