"""Checkpoint directory I/O in the snapjudge on-disk schema.

A checkpoint directory holds ``rl_agent_config.json``, ``encoder/config.json``
and ``model.safetensors``.  The encoder hyper-parameters are read exactly the
way the reference ``DecisionModel::load`` reads them
(reference ``src/model.cpp:59-111``): defaults for missing keys, window =
``local_attention // 2`` on ``sliding_attention`` layers, two RoPE thetas, and
a layer-0 ``attn_norm`` that may be absent (identity).

Tensors are returned as float32 numpy arrays whatever the on-disk dtype
(F32/F16/BF16), like ``SafeTensors::data_f32`` (reference
``src/safetensors.cpp:113-135``).
"""
from __future__ import annotations

import json
import os
import struct
from dataclasses import dataclass, field

import numpy as np

_DT_READ = {"F32": np.float32, "F16": np.float16, "BF16": None,
            "I64": np.int64, "I32": np.int32}


def read_safetensors(path: str) -> dict[str, np.ndarray]:
    """Read every tensor of a safetensors file as a numpy array (floats → fp32)."""
    with open(path, "rb") as f:
        buf = f.read()
    if len(buf) < 8:
        raise ValueError(f"not a safetensors file (too small): {path}")
    (hlen,) = struct.unpack("<Q", buf[:8])
    if 8 + hlen > len(buf):
        raise ValueError(f"bad header length in {path}")
    hdr = json.loads(buf[8:8 + hlen])
    base = 8 + hlen
    out: dict[str, np.ndarray] = {}
    for name, ent in hdr.items():
        if name == "__metadata__":
            continue
        o0, o1 = ent["data_offsets"]
        raw = buf[base + o0: base + o1]
        shape = tuple(ent["shape"])
        dt = ent["dtype"]
        if dt == "BF16":
            u = np.frombuffer(raw, dtype=np.uint16).astype(np.uint32) << 16
            arr = u.view(np.float32)
        elif dt in _DT_READ:
            arr = np.frombuffer(raw, dtype=_DT_READ[dt])
            if arr.dtype == np.float16:
                arr = arr.astype(np.float32)
        else:
            raise ValueError(f"unsupported dtype {dt} for {name}")
        out[name] = np.ascontiguousarray(arr.reshape(shape))
    return out


def write_safetensors(path: str, tensors: dict[str, np.ndarray]) -> None:
    """Write float32 tensors as an F32 safetensors file (8-byte aligned header)."""
    header = {}
    off = 0
    order = list(tensors.keys())
    for k in order:
        v = tensors[k]
        if v.dtype != np.float32:
            raise ValueError(f"{k}: only float32 is written, got {v.dtype}")
        n = v.nbytes
        header[k] = {"dtype": "F32", "shape": list(v.shape), "data_offsets": [off, off + n]}
        off += n
    hj = json.dumps(header).encode()
    hj += b" " * ((8 - (8 + len(hj)) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        for k in order:
            f.write(np.ascontiguousarray(tensors[k]).tobytes())


@dataclass
class EncoderConfig:
    """Encoder hyper-parameters, parsed like reference ``src/model.cpp:59-111``."""
    hidden_size: int
    num_hidden_layers: int
    num_attention_heads: int
    intermediate_size: int
    vocab_size: int
    max_position_embeddings: int = 8192
    norm_eps: float = 1e-5
    norm_bias: bool = False
    local_attention: int = 0
    layer_types: list[str] = field(default_factory=list)
    rope_theta_full: float = 10000.0
    rope_theta_sliding: float = 10000.0
    head_layers: int = 2
    max_len: int = 512
    n_act: int = 1

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_attention_heads

    def layer_window(self, i: int) -> int:
        """Half-width of the bidirectional window of layer i (0 = full)."""
        t = self.layer_types[i] if i < len(self.layer_types) else "full_attention"
        if t == "sliding_attention" and self.local_attention > 0:
            return self.local_attention // 2
        return 0

    def layer_sliding(self, i: int) -> bool:
        t = self.layer_types[i] if i < len(self.layer_types) else "full_attention"
        return t == "sliding_attention"

    def to_json(self) -> dict:
        return {
            "hidden_size": self.hidden_size,
            "num_hidden_layers": self.num_hidden_layers,
            "num_attention_heads": self.num_attention_heads,
            "intermediate_size": self.intermediate_size,
            "max_position_embeddings": self.max_position_embeddings,
            "vocab_size": self.vocab_size,
            "norm_eps": self.norm_eps,
            "norm_bias": self.norm_bias,
            "attention_bias": False,
            "mlp_bias": False,
            "local_attention": self.local_attention,
            "layer_types": list(self.layer_types),
            "rope_parameters": {
                "full_attention": {"rope_theta": self.rope_theta_full, "rope_type": "default"},
                "sliding_attention": {"rope_theta": self.rope_theta_sliding,
                                      "rope_type": "default"},
            },
        }

    @staticmethod
    def from_json(enc: dict, rl: dict | None = None) -> "EncoderConfig":
        rl = rl or {}
        c = EncoderConfig(
            hidden_size=int(enc.get("hidden_size", 0)),
            num_hidden_layers=int(enc.get("num_hidden_layers", 0)),
            num_attention_heads=int(enc.get("num_attention_heads", 0)),
            intermediate_size=int(enc.get("intermediate_size", 0)),
            vocab_size=int(enc.get("vocab_size", 0)),
            max_position_embeddings=int(enc.get("max_position_embeddings", 8192)),
            norm_eps=float(enc.get("norm_eps", 1e-5)),
            norm_bias=bool(enc.get("norm_bias", False)),
            local_attention=int(enc.get("local_attention", 0)),
            layer_types=list(enc.get("layer_types", [])),
        )
        rp = enc.get("rope_parameters", {})
        if "full_attention" in rp:
            c.rope_theta_full = float(rp["full_attention"].get("rope_theta", c.rope_theta_full))
        if "sliding_attention" in rp:
            c.rope_theta_sliding = float(rp["sliding_attention"].get("rope_theta",
                                                                     c.rope_theta_sliding))
        c.head_layers = int(rl.get("head_layers", 2))
        c.max_len = int(rl.get("max_len", 512))
        costs = rl.get("act_costs", {})
        c.n_act = (len(costs) if isinstance(costs, dict) else 0) + 1
        return c


def load_checkpoint(path: str) -> tuple[EncoderConfig, dict[str, np.ndarray]]:
    """Load (config, fp32 tensors) from a snapjudge checkpoint directory."""
    with open(os.path.join(path, "rl_agent_config.json")) as f:
        rl = json.load(f)
    with open(os.path.join(path, "encoder", "config.json")) as f:
        enc = json.load(f)
    for k in ("encoder", "head_layers"):
        if k not in rl:
            raise ValueError(f"Incompatible model config for '{path}': missing configuration "
                             f"keys ['{k}']")
    cfg = EncoderConfig.from_json(enc, rl)
    return cfg, read_safetensors(os.path.join(path, "model.safetensors"))


def save_checkpoint(path: str, cfg: EncoderConfig, tensors: dict[str, np.ndarray],
                    extra_rl: dict | None = None) -> None:
    """Write a checkpoint directory loadable by the reference ``Agent`` loader."""
    os.makedirs(os.path.join(path, "encoder"), exist_ok=True)
    rl = {"encoder": "synthetic", "head_layers": cfg.head_layers, "max_len": cfg.max_len,
          "head_max_len": 48, "act_costs": {}, "amp_dtype": "fp32",
          "model_name": "snapjudge-synthetic", "temperature": [1.0, 1.0, 1.0]}
    if extra_rl:
        rl.update(extra_rl)
    with open(os.path.join(path, "rl_agent_config.json"), "w") as f:
        json.dump(rl, f, indent=1)
    with open(os.path.join(path, "encoder", "config.json"), "w") as f:
        json.dump(cfg.to_json(), f, indent=1)
    write_safetensors(os.path.join(path, "model.safetensors"), tensors)


# ---------------------------------------------------------------- SjModel
@dataclass
class SjConfig:
    """SjModel hyper-parameters, read as ``SjModel::load`` reads ``sj_config.json``
    (reference ``src/sj_model.cpp:88-110``): a BERT-style pre-LN encoder with
    learned positions, separate biased q/k/v/o projections and a biased GELU FFN."""
    vocab_size: int
    hidden_size: int
    num_layers: int
    num_heads: int
    intermediate_size: int = 0     # 0 -> 4 * hidden_size
    max_positions: int = 512
    norm_eps: float = 1e-5
    head_layers: int = 1
    head_intermediate: int = 0     # 0 -> 4 * hidden_size
    n_types: int = 3

    def __post_init__(self):
        if self.intermediate_size <= 0:
            self.intermediate_size = 4 * self.hidden_size
        if self.head_intermediate <= 0:
            self.head_intermediate = 4 * self.hidden_size

    def to_json(self) -> dict:
        return {"vocab_size": self.vocab_size, "hidden_size": self.hidden_size,
                "num_layers": self.num_layers, "num_heads": self.num_heads,
                "intermediate_size": self.intermediate_size,
                "max_positions": self.max_positions, "norm_eps": self.norm_eps,
                "head_layers": self.head_layers, "head_intermediate": self.head_intermediate,
                "n_types": self.n_types}

    @classmethod
    def from_json(cls, j: dict) -> "SjConfig":
        for k in ("vocab_size", "hidden_size", "num_layers", "num_heads"):
            if k not in j:
                raise ValueError("config missing required keys "
                                 "(vocab_size/hidden_size/num_layers/num_heads)")
        D = int(j["hidden_size"])
        return cls(vocab_size=int(j["vocab_size"]), hidden_size=D,
                   num_layers=int(j["num_layers"]), num_heads=int(j["num_heads"]),
                   intermediate_size=int(j.get("intermediate_size", 4 * D)),
                   max_positions=int(j.get("max_positions", 512)),
                   norm_eps=float(j.get("norm_eps", 1e-5)),
                   head_layers=int(j.get("head_layers", 1)),
                   head_intermediate=int(j.get("head_intermediate", 4 * D)),
                   n_types=int(j.get("n_types", 3)))


def load_sj_checkpoint(path: str) -> tuple[SjConfig, dict[str, np.ndarray]]:
    """Load (config, fp32 tensors) from an SjModel directory (sj_config.json +
    model.safetensors)."""
    with open(os.path.join(path, "sj_config.json")) as f:
        cfg = SjConfig.from_json(json.load(f))
    return cfg, read_safetensors(os.path.join(path, "model.safetensors"))


def save_sj_checkpoint(path: str, cfg: SjConfig, tensors: dict[str, np.ndarray]) -> None:
    """Write an SjModel directory loadable by the reference ``SjModel::load``."""
    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "sj_config.json"), "w") as f:
        json.dump(cfg.to_json(), f, indent=1)
    write_safetensors(os.path.join(path, "model.safetensors"), tensors)
