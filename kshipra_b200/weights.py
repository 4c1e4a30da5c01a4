"""Seeded synthetic weights with HuggingFace parameter names.

No checkpoint is available to this build, so every model is random-init:
each linear / embedding weight is N(0, 0.02) drawn from one
``torch.Generator`` seeded once, in a fixed parameter order; RMSNorm weights
are 1; biases (Qwen2 q/k/v) are 0.  The order is fixed by this module, not by
HF's module-init order, so the same seed gives the same tensors whichever
transformers version builds the HF model around them.

On CPU the stream is bit-reproducible across machines running the same torch
build, which is what the golden fixtures rely on.  ``device="cuda"`` draws
from the CUDA generator instead (fast, used for the large benchmark shapes,
not comparable with the CPU stream).
"""

from __future__ import annotations

from collections import OrderedDict
from typing import Iterator, Tuple

import torch

from .config import ModelConfig

STD = 0.02


def param_specs(cfg: ModelConfig) -> Iterator[Tuple[str, Tuple[int, ...], str]]:
    """Yield (hf_name, shape, kind) in generation order.

    kind: "normal" (N(0, STD)), "ones" or "zeros".
    """
    h, qs, kvs, inter = cfg.hidden, cfg.q_size, cfg.kv_size, cfg.intermediate
    yield "model.embed_tokens.weight", (cfg.vocab, h), "normal"
    for i in range(cfg.layers):
        p = f"model.layers.{i}."
        yield p + "self_attn.q_proj.weight", (qs, h), "normal"
        yield p + "self_attn.k_proj.weight", (kvs, h), "normal"
        yield p + "self_attn.v_proj.weight", (kvs, h), "normal"
        if cfg.qkv_bias:
            yield p + "self_attn.q_proj.bias", (qs,), "zeros"
            yield p + "self_attn.k_proj.bias", (kvs,), "zeros"
            yield p + "self_attn.v_proj.bias", (kvs,), "zeros"
        yield p + "self_attn.o_proj.weight", (h, qs), "normal"
        yield p + "mlp.gate_proj.weight", (inter, h), "normal"
        yield p + "mlp.up_proj.weight", (inter, h), "normal"
        yield p + "mlp.down_proj.weight", (h, inter), "normal"
        yield p + "input_layernorm.weight", (h,), "ones"
        yield p + "post_attention_layernorm.weight", (h,), "ones"
    yield "model.norm.weight", (h,), "ones"
    if not cfg.tie_embeddings:
        yield "lm_head.weight", (cfg.vocab, h), "normal"


def synthetic_state_dict(cfg: ModelConfig, seed: int = 0,
                         device: str | torch.device = "cpu") -> "OrderedDict[str, torch.Tensor]":
    dev = torch.device(device)
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    sd: "OrderedDict[str, torch.Tensor]" = OrderedDict()
    for name, shape, kind in param_specs(cfg):
        if kind == "normal":
            t = torch.randn(shape, generator=gen, dtype=torch.float32, device=dev)
            t.mul_(STD)
        elif kind == "ones":
            t = torch.ones(shape, dtype=torch.float32, device=dev)
        else:
            t = torch.zeros(shape, dtype=torch.float32, device=dev)
        sd[name] = t
    if cfg.tie_embeddings:
        sd["lm_head.weight"] = sd["model.embed_tokens.weight"]
    return sd


def build_hf_model(cfg: ModelConfig, state_dict=None, seed: int = 0):
    """Construct the HF ``*ForCausalLM`` holding ``state_dict`` (fp32, CPU)."""
    from transformers import LlamaForCausalLM, Qwen2ForCausalLM

    hf_cfg = cfg.to_hf_config()
    klass = Qwen2ForCausalLM if cfg.arch == "qwen2" else LlamaForCausalLM
    if state_dict is None:
        state_dict = synthetic_state_dict(cfg, seed)
    model = klass(hf_cfg)
    sd = {k: v for k, v in state_dict.items()
          if not (cfg.tie_embeddings and k == "lm_head.weight")}
    missing, unexpected = model.load_state_dict(sd, strict=False)
    bad = [k for k in missing if not (cfg.tie_embeddings and k == "lm_head.weight")
           and "rotary" not in k]
    if bad or unexpected:
        raise RuntimeError(f"state dict mismatch: missing={bad} unexpected={unexpected}")
    if cfg.tie_embeddings:
        model.tie_weights()
    return model.eval()


def weights_checksum(sd) -> float:
    """Order-dependent float64 checksum used to pin the generator stream."""
    acc = 0.0
    for i, (name, t) in enumerate(sd.items()):
        acc += float(t.double().sum()) * (i + 1) + float(t.double().abs().sum())
    return acc
