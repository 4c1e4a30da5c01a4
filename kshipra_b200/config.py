"""Model configurations for the quantized forward path.

A ``ModelConfig`` carries exactly the hyper-parameters that
``KshipraModel.__init__`` reads from a HuggingFace config
(engine/model.py:69-75 of the reference) plus the few the HF modules use
internally (RMSNorm epsilon, tied embeddings, q/k/v bias).

``rope_theta`` is carried explicitly.  Under transformers 5.x the HF config
keeps it in ``config.rope_parameters['rope_theta']``; the reference reads the
(absent) ``config.rope_theta`` attribute and silently falls back to 10000.0
(engine/model.py:74).  ``from_hf_config`` reads both places.
"""

from __future__ import annotations

from dataclasses import dataclass, asdict
from typing import Dict


@dataclass(frozen=True)
class ModelConfig:
    name: str
    arch: str                 # "llama" | "qwen2"
    hidden: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int
    rope_theta: float
    rms_eps: float = 1e-6
    tie_embeddings: bool = False
    qkv_bias: bool = False
    max_positions: int = 32768

    @property
    def q_size(self) -> int:
        return self.heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.kv_heads * self.head_dim

    @property
    def gqa_group(self) -> int:
        return self.heads // self.kv_heads

    def to_dict(self) -> Dict:
        return asdict(self)

    # ------------------------------------------------------------------ #
    # HF interop
    # ------------------------------------------------------------------ #

    def to_hf_config(self):
        """Build the matching ``LlamaConfig`` / ``Qwen2Config``."""
        if self.arch == "llama":
            from transformers import LlamaConfig as C
        elif self.arch == "qwen2":
            from transformers import Qwen2Config as C
        else:  # pragma: no cover - guarded by the presets
            raise ValueError(f"unknown arch {self.arch!r}")
        kw = dict(
            vocab_size=self.vocab,
            hidden_size=self.hidden,
            intermediate_size=self.intermediate,
            num_hidden_layers=self.layers,
            num_attention_heads=self.heads,
            num_key_value_heads=self.kv_heads,
            max_position_embeddings=self.max_positions,
            rms_norm_eps=self.rms_eps,
            tie_word_embeddings=self.tie_embeddings,
            rope_theta=self.rope_theta,
        )
        if self.arch == "llama":
            kw["head_dim"] = self.head_dim
        cfg = C(**kw)
        # transformers 5.x stores theta under rope_parameters.
        rp = getattr(cfg, "rope_parameters", None)
        if isinstance(rp, dict):
            rp["rope_theta"] = self.rope_theta
        return cfg

    @staticmethod
    def from_hf_config(cfg, name: str = "hf") -> "ModelConfig":
        heads = int(cfg.num_attention_heads)
        kv = int(getattr(cfg, "num_key_value_heads", None) or heads)
        head_dim = getattr(cfg, "head_dim", None) or cfg.hidden_size // heads
        theta = getattr(cfg, "rope_theta", None)
        rp = getattr(cfg, "rope_parameters", None)
        if theta is None and isinstance(rp, dict):
            theta = rp.get("rope_theta")
        if theta is None:
            theta = 10000.0
        mt = getattr(cfg, "model_type", "llama")
        arch = "qwen2" if mt == "qwen2" else "llama"
        return ModelConfig(
            name=name,
            arch=arch,
            hidden=int(cfg.hidden_size),
            layers=int(cfg.num_hidden_layers),
            heads=heads,
            kv_heads=kv,
            head_dim=int(head_dim),
            intermediate=int(cfg.intermediate_size),
            vocab=int(cfg.vocab_size),
            rope_theta=float(theta),
            rms_eps=float(getattr(cfg, "rms_norm_eps", 1e-6)),
            tie_embeddings=bool(getattr(cfg, "tie_word_embeddings", False)),
            qkv_bias=(arch == "qwen2"),
            max_positions=int(getattr(cfg, "max_position_embeddings", 32768)),
        )


# Presets: the model shapes the benchmark configurations name.
TINY_LLAMA = ModelConfig(
    name="tiny-llama", arch="llama", hidden=256, layers=2, heads=4, kv_heads=2,
    head_dim=64, intermediate=688, vocab=1024, rope_theta=10000.0,
    max_positions=2048,
)

QWEN25_05B = ModelConfig(
    name="qwen2.5-0.5b", arch="qwen2", hidden=896, layers=24, heads=14, kv_heads=2,
    head_dim=64, intermediate=4864, vocab=151936, rope_theta=1000000.0,
    tie_embeddings=True, qkv_bias=True, max_positions=32768,
)

LLAMA3_8B = ModelConfig(
    name="llama-3-8b", arch="llama", hidden=4096, layers=32, heads=32, kv_heads=8,
    head_dim=128, intermediate=14336, vocab=128256, rope_theta=500000.0,
    max_positions=8192,
)

PRESETS = {c.name: c for c in (TINY_LLAMA, QWEN25_05B, LLAMA3_8B)}


def truncated(cfg: ModelConfig, layers: int) -> ModelConfig:
    """Same shapes with fewer layers (for oracle runs of the 8B shape)."""
    d = cfg.to_dict()
    d["layers"] = layers
    d["name"] = f"{cfg.name}-L{layers}"
    return ModelConfig(**d)
