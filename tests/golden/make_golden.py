#!/usr/bin/env python3
"""Regenerate the committed golden fixtures (needs the snapjudge reference tree).

Writes, next to this script:

* ``tensor_ops_ref.npz`` — the reference's own op-level golden vectors
  (``tests/golden/tensor_ops.json`` of the reference, produced by its
  ``python/make_tensor_golden.py``): gemm / gelu / relu / geglu / layer_norm /
  attention (lens [6, 4], window 0 and 2) / RoPE, converted to numpy arrays.
* ``encoder_ref.npz`` — outputs of the reference's own ``DecisionModel::encode``
  and ``DecisionModel::forward`` (``src/model.cpp``, compiled unchanged into
  ``oracle/_ref/libsjref.so`` by ``oracle/Makefile``) on seeded synthetic
  checkpoints (``snapjudge_b200.synth``): the ``tiny`` shape (D=16, Dh=8,
  sliding layer) and config ``c1`` (D=64, Dh=16), on packed-equivalent single
  sequences and on a right-padded ragged batch (padded rows included).
* ``sjmodel_ref.npz`` — outputs of the reference's own ``SjModel::encode`` and
  ``SjModel::forward`` (``src/sj_model.cpp``, compiled into the same library)
  on the seeded ``sj_tiny`` checkpoint: single sequences and a ragged padded
  batch.

Usage:  python tests/golden/make_golden.py [--reference /path/to/snapjudge]
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import oracle  # noqa: E402
from snapjudge_b200 import synth  # noqa: E402
from snapjudge_b200.checkpoint import save_checkpoint, save_sj_checkpoint  # noqa: E402


def convert_tensor_ops(ref_root: str) -> None:
    with open(os.path.join(ref_root, "tests", "golden", "tensor_ops.json")) as f:
        g = json.load(f)
    out = {}
    for case, fields in g.items():
        for k, v in fields.items():
            out[f"{case}.{k}"] = np.asarray(v, dtype=np.float64 if k != "lens" else np.int64)
    np.savez_compressed(os.path.join(HERE, "tensor_ops_ref.npz"), **out)
    print("wrote tensor_ops_ref.npz:", len(out), "arrays")


def markers(rng, lengths, K):
    B = len(lengths)
    pos = np.zeros((B, K), np.int64)
    mm = np.zeros((B, K), np.uint8)
    for b in range(B):
        k = int(rng.integers(1, K + 1))
        pos[b, :k] = rng.integers(0, lengths[b], size=k)
        mm[b, :k] = 1
    return pos, mm


def encoder_goldens() -> None:
    out = {}
    for name, lens_list in (("tiny", [[5], [17], [40], [40, 23, 1]]),
                            ("c1", [[32], [32, 32, 32, 32], [32, 17, 1, 9]])):
        spec = synth.SPECS[name]
        tensors = synth.make_weights(spec)
        with tempfile.TemporaryDirectory() as d:
            save_checkpoint(d, spec.cfg, tensors)
            ref = oracle.RefModel(d)
            rng = np.random.default_rng(123)
            for ci, lens in enumerate(lens_list):
                lengths = np.asarray(lens, np.int64)
                ids = synth.make_ids(spec, lengths, seed=500 + ci)
                pid, mask = synth.pad_batch(ids, lengths)
                h = ref.encode(pid, mask, spec.cfg.hidden_size)
                pos, mm = markers(rng, lengths, 4)
                qt = rng.integers(0, 3, size=len(lengths)).astype(np.int64)
                logits, act = ref.forward(pid, mask, pos, mm, qt)
                p = f"{name}.{ci}."
                out[p + "lengths"] = lengths
                out[p + "ids"] = ids
                out[p + "hidden"] = h
                out[p + "marker_pos"] = pos
                out[p + "marker_mask"] = mm
                out[p + "qtype"] = qt
                out[p + "logits"] = logits
                out[p + "act"] = act
    np.savez_compressed(os.path.join(HERE, "encoder_ref.npz"), **out)
    print("wrote encoder_ref.npz:", len(out), "arrays")


def sjmodel_goldens() -> None:
    cfg, seed = synth.SJ_SPECS["sj_tiny"]
    tensors = synth.make_sj_weights(cfg, seed)
    out = {}
    with tempfile.TemporaryDirectory() as d:
        save_sj_checkpoint(d, cfg, tensors)
        ref = oracle.RefSjModel(d, cfg.hidden_size)
        rng = np.random.default_rng(321)
        for ci, lens in enumerate([[7], [40], [40, 23, 1, 64]]):
            lengths = np.asarray(lens, np.int64)
            L = int(lengths.max())
            ids = rng.integers(0, cfg.vocab_size, size=int(lengths.sum())).astype(np.int64)
            pid, mask = synth.pad_batch(ids, lengths)
            h = ref.encode(pid, mask)
            pos, mm = markers(rng, lengths, 4)
            qt = rng.integers(0, cfg.n_types, size=len(lengths)).astype(np.int64)
            logits, act = ref.forward(pid, mask, pos, mm, qt)
            p = f"sj_tiny.{ci}."
            out[p + "lengths"] = lengths
            out[p + "ids"] = ids
            out[p + "hidden"] = h
            out[p + "marker_pos"] = pos
            out[p + "marker_mask"] = mm
            out[p + "qtype"] = qt
            out[p + "logits"] = logits
            out[p + "act"] = act
            assert L <= cfg.max_positions
    np.savez_compressed(os.path.join(HERE, "sjmodel_ref.npz"), **out)
    print("wrote sjmodel_ref.npz:", len(out), "arrays")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=oracle.reference_tree(), required=oracle.reference_tree() is None,
                    help="snapjudge reference checkout (default: $SNAPJUDGE_REFERENCE, else a "
                         "'reference' directory beside this repository)")
    a = ap.parse_args()
    oracle.build()
    convert_tensor_ops(a.reference)
    encoder_goldens()
    sjmodel_goldens()


if __name__ == "__main__":
    main()
