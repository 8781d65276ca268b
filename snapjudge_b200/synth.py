"""Seeded synthetic checkpoints and request batches for the benchmark configs.

No real snapjudge checkpoint or dataset is available offline, so every config
is generated from numpy ``default_rng(seed)``:

* weights ``N(0, 0.02)`` float32 in the reference tensor schema
  (reference ``src/model.cpp:96-171``), LayerNorm weights 1, no LayerNorm bias
  (``norm_bias=false``), no layer-0 ``attn_norm`` (reference convention,
  ``python/make_tiny_ckpt.py:29-32``);
* the decision-model head tensors (type_emb, head layers, scorer, act head) so
  that the reference ``DecisionModel::load`` accepts the file;
* per-config "task heads": linear layers on the [CLS] (position 0) hidden state,
  stored as extra ``task_heads.<i>.weight/bias`` tensors that the reference
  loader ignores;
* token ids uniform in ``[0, V)``; lengths uniform / log-normal-clipped / fixed.

Config names follow the benchmark list: ``c1`` tiny fp32 encoder, ``c2``
attention-only op, ``c3`` base encoder, ``c4`` long-context encoder, ``c5``
serving batch (c3 architecture), and ``tiny`` = the reference's own tiny
test checkpoint shape (D=16, H=2, F=8, sliding layer 1, window 4).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .checkpoint import EncoderConfig, SjConfig

# task head kinds
SOFTMAX = 0
SIGMOID = 1


@dataclass
class TaskHead:
    name: str
    n_out: int
    kind: int  # SOFTMAX or SIGMOID


@dataclass
class SynthSpec:
    name: str
    cfg: EncoderConfig
    seed: int
    heads: list[TaskHead]
    batch: int
    lengths: str           # "fixed:<n>", "uniform:<lo>:<hi>", "lognormal:<median>:<sigma>:<lo>:<hi>"
    precision: str         # "fp32" | "bf16"


def _enc(D, H, F, V, layers, *, local_attention=0, layer_types=None, max_pos=8192,
         head_layers=1):
    return EncoderConfig(hidden_size=D, num_hidden_layers=layers, num_attention_heads=H,
                         intermediate_size=F, vocab_size=V, max_position_embeddings=max_pos,
                         local_attention=local_attention,
                         layer_types=layer_types or ["full_attention"] * layers,
                         head_layers=head_layers)


SPECS: dict[str, SynthSpec] = {
    "tiny": SynthSpec("tiny", _enc(16, 2, 8, 512, 2, local_attention=8,
                                   layer_types=["full_attention", "sliding_attention"],
                                   max_pos=128),
                      7, [TaskHead("choice3", 3, SOFTMAX)], 3, "uniform:5:40", "fp32"),
    "c1": SynthSpec("c1", _enc(64, 4, 256, 1000, 2), 0,
                    [TaskHead("choice3", 3, SOFTMAX)], 4, "fixed:32", "fp32"),
    "c3": SynthSpec("c3", _enc(768, 12, 2048, 32768, 12), 2,
                    [TaskHead("choice3", 3, SOFTMAX)], 256, "lognormal:128:0.6:8:512", "bf16"),
    "c4": SynthSpec("c4", _enc(1024, 16, 2816, 50368, 24), 3,
                    [TaskHead("noul", 1, SIGMOID)], 32, "fixed:2048", "bf16"),
    "c5": SynthSpec("c5", _enc(768, 12, 2048, 32768, 12), 4,
                    [TaskHead("choice3", 3, SOFTMAX), TaskHead("choice8", 8, SOFTMAX),
                     TaskHead("score5", 5, SOFTMAX), TaskHead("noul", 1, SIGMOID)],
                    32768, "lognormal:48:0.8:4:512", "bf16"),
}


def make_weights(spec: SynthSpec, std: float = 0.02) -> dict[str, np.ndarray]:
    """Seeded fp32 weights in the reference schema (+ task heads)."""
    c = spec.cfg
    D, F, V = c.hidden_size, c.intermediate_size, c.vocab_size
    rng = np.random.default_rng(spec.seed)
    s = np.float32(std)

    def n(*shape):
        return rng.standard_normal(shape, dtype=np.float32) * s

    ones = lambda k: np.ones(k, dtype=np.float32)  # noqa: E731
    zeros = lambda k: np.zeros(k, dtype=np.float32)  # noqa: E731
    t: dict[str, np.ndarray] = {}
    t["encoder.embeddings.tok_embeddings.weight"] = n(V, D)
    t["encoder.embeddings.norm.weight"] = ones(D)
    for i in range(c.num_hidden_layers):
        p = f"encoder.layers.{i}."
        if i > 0:
            t[p + "attn_norm.weight"] = ones(D)
        t[p + "attn.Wqkv.weight"] = n(3 * D, D)
        t[p + "attn.Wo.weight"] = n(D, D)
        t[p + "mlp_norm.weight"] = ones(D)
        t[p + "mlp.Wi.weight"] = n(2 * F, D)
        t[p + "mlp.Wo.weight"] = n(D, F)
    t["encoder.final_norm.weight"] = ones(D)
    t["type_emb.weight"] = n(3, D)
    for i in range(c.head_layers):
        p = f"head.layers.{i}."
        t[p + "norm1.weight"] = ones(D)
        t[p + "norm1.bias"] = zeros(D)
        t[p + "norm2.weight"] = ones(D)
        t[p + "norm2.bias"] = zeros(D)
        t[p + "self_attn.in_proj_weight"] = n(3 * D, D)
        t[p + "self_attn.in_proj_bias"] = n(3 * D)
        t[p + "self_attn.out_proj.weight"] = n(D, D)
        t[p + "self_attn.out_proj.bias"] = n(D)
        t[p + "linear1.weight"] = n(4 * D, D)
        t[p + "linear1.bias"] = n(4 * D)
        t[p + "linear2.weight"] = n(D, 4 * D)
        t[p + "linear2.bias"] = n(D)
    t["scorer.0.weight"] = ones(D)
    t["scorer.1.weight"] = n(D, D)
    t["scorer.1.bias"] = n(D)
    t["scorer.3.weight"] = n(1, D)
    t["scorer.3.bias"] = n(1)
    t["act_head.0.weight"] = n(256, D + 4)
    t["act_head.0.bias"] = n(256)
    t["act_head.2.weight"] = n(c.n_act, 256)
    t["act_head.2.bias"] = n(c.n_act)
    for i, h in enumerate(spec.heads):
        # task heads: std 1/sqrt(D) so the [CLS] logits are O(1), as in a trained head
        t[f"task_heads.{i}.weight"] = (rng.standard_normal((h.n_out, D), dtype=np.float32)
                                       * np.float32(1.0 / np.sqrt(D)))
        t[f"task_heads.{i}.bias"] = rng.standard_normal((h.n_out,), dtype=np.float32) * s
    return t


# SjModel (reference src/sj_model.cpp) checkpoints: a tiny one for the committed
# goldens and one at the C3 width for the tensor-core paths.
SJ_SPECS: dict[str, tuple[SjConfig, int]] = {
    "sj_tiny": (SjConfig(vocab_size=500, hidden_size=32, num_layers=2, num_heads=2,
                         intermediate_size=64, max_positions=64, head_layers=1,
                         head_intermediate=128), 21),
    "sj_base": (SjConfig(vocab_size=32768, hidden_size=768, num_layers=12, num_heads=12,
                         intermediate_size=3072, max_positions=512, head_layers=1), 22),
}


def make_sj_weights(cfg: SjConfig, seed: int, std: float = 0.02) -> dict[str, np.ndarray]:
    """Seeded fp32 SjModel weights in its schema (sj.* names, src/sj_model.cpp:117-202);
    LN weights 1, every bias drawn like the weights so the bias paths are exercised."""
    D, F, V = cfg.hidden_size, cfg.intermediate_size, cfg.vocab_size
    rng = np.random.default_rng(seed)
    s = np.float32(std)

    def n(*shape):
        return rng.standard_normal(shape, dtype=np.float32) * s

    ones = lambda k: np.ones(k, dtype=np.float32)  # noqa: E731
    t: dict[str, np.ndarray] = {}
    t["sj.embeddings.word.weight"] = n(V, D)
    t["sj.embeddings.position.weight"] = n(cfg.max_positions, D)
    t["sj.embeddings.norm.weight"] = ones(D)
    t["sj.embeddings.norm.bias"] = n(D)

    def layer(p, ffn, norms):
        t[p + norms[0] + ".weight"] = ones(D)
        t[p + norms[0] + ".bias"] = n(D)
        for x in "qkvo":
            t[p + f"attn.{x}.weight"] = n(D, D)
            t[p + f"attn.{x}.bias"] = n(D)
        t[p + norms[1] + ".weight"] = ones(D)
        t[p + norms[1] + ".bias"] = n(D)
        t[p + "ffn.w1.weight"] = n(ffn, D)
        t[p + "ffn.w1.bias"] = n(ffn)
        t[p + "ffn.w2.weight"] = n(D, ffn)
        t[p + "ffn.w2.bias"] = n(D)

    for i in range(cfg.num_layers):
        layer(f"sj.encoder.layers.{i}.", F, ("attn_norm", "ffn_norm"))
    t["sj.encoder.final_norm.weight"] = ones(D)
    t["sj.encoder.final_norm.bias"] = n(D)
    t["sj.type_emb.weight"] = n(cfg.n_types, D)
    for i in range(cfg.head_layers):
        layer(f"sj.head.layers.{i}.", cfg.head_intermediate, ("norm1", "norm2"))
    t["sj.scorer.norm.weight"] = ones(D)
    t["sj.scorer.norm.bias"] = n(D)
    t["sj.scorer.w1.weight"] = n(D, D)
    t["sj.scorer.w1.bias"] = n(D)
    t["sj.scorer.w2.weight"] = n(1, D)
    t["sj.scorer.w2.bias"] = n(1)
    return t


def make_lengths(spec: SynthSpec, batch: int | None = None, seed: int | None = None) -> np.ndarray:
    """Per-request valid lengths, int64 [batch]."""
    b = spec.batch if batch is None else batch
    rng = np.random.default_rng(spec.seed + 1000 if seed is None else seed)
    kind, *a = spec.lengths.split(":")
    if kind == "fixed":
        return np.full(b, int(a[0]), dtype=np.int64)
    if kind == "uniform":
        return rng.integers(int(a[0]), int(a[1]) + 1, size=b).astype(np.int64)
    if kind == "lognormal":
        med, sig, lo, hi = float(a[0]), float(a[1]), int(a[2]), int(a[3])
        x = np.round(np.exp(rng.normal(np.log(med), sig, size=b)))
        return np.clip(x, lo, hi).astype(np.int64)
    raise ValueError(spec.lengths)


def make_ids(spec: SynthSpec, lengths: np.ndarray, seed: int | None = None) -> np.ndarray:
    """Packed token ids int64 [sum(lengths)], uniform in [0, V)."""
    rng = np.random.default_rng(spec.seed + 2000 if seed is None else seed)
    return rng.integers(0, spec.cfg.vocab_size, size=int(lengths.sum())).astype(np.int64)


def cu_seqlens(lengths: np.ndarray) -> np.ndarray:
    cu = np.zeros(len(lengths) + 1, dtype=np.int32)
    np.cumsum(lengths, out=cu[1:])
    return cu


def pad_batch(ids: np.ndarray, lengths: np.ndarray, pad_id: int = 0,
              L: int | None = None) -> tuple[np.ndarray, np.ndarray]:
    """Right-pad packed ids to [B, L] + attention mask (reference collate layout)."""
    B = len(lengths)
    L = int(lengths.max()) if L is None else L
    out = np.full((B, L), pad_id, dtype=np.int64)
    mask = np.zeros((B, L), dtype=np.int64)
    cu = cu_seqlens(lengths)
    for b in range(B):
        n = int(lengths[b])
        out[b, :n] = ids[cu[b]:cu[b] + n]
        mask[b, :n] = 1
    return out, mask


def attention_inputs(batch=64, H=12, Dh=64, lo=32, hi=512, seed=1):
    """C2 inputs: lengths U[lo,hi], packed q/k/v N(0,1) as float32 [T, H, Dh] each."""
    rng = np.random.default_rng(seed)
    lengths = rng.integers(lo, hi + 1, size=batch).astype(np.int64)
    T = int(lengths.sum())
    q = rng.standard_normal((T, H, Dh), dtype=np.float32)
    k = rng.standard_normal((T, H, Dh), dtype=np.float32)
    v = rng.standard_normal((T, H, Dh), dtype=np.float32)
    return lengths, q, k, v
