"""torch-CPU restatement of the reference quantized forward.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Follows engine/model.py of the reference:

* ``compute_rope`` / ``apply_rope`` / ``rotate_half``  -- model.py:30-55
* ``OracleModel.forward``  -- model.py:93-151: embed -> per layer [RMSNorm ->
  q/k/v (dequantize every call, then ``F.linear``; quantization.py:394-396)
  -> RoPE at absolute positions -> per-token scatter of K/V into the block
  pool (model.py:124-129) -> ``chunked_attention`` over the pool -> o_proj ->
  residual -> RMSNorm -> SwiGLU MLP -> residual] -> final RMSNorm -> fp32
  ``lm_head`` (never quantized).
* ``OracleModel.generate`` -- model.py:154-205 (fresh pool, prefill, greedy
  ``argmax``, one-token decode loop), with an optional prefill chunk size that
  drives ``forward(prefix_len=...)`` chunk by chunk, the recipe the benchmark
  configurations use.

The HF module arithmetic the reference calls is restated too:
``LlamaRMSNorm`` (fp32 ``x * rsqrt(mean(x^2) + eps)`` times weight) and
``LlamaMLP`` (``down(silu(gate(x)) * up(x))``).  Dequantization follows
quantization.py:226-230 / 321-344 with torch ops, so the CPU cost profile
(materialised dequant per forward) is the reference's own.
"""

from __future__ import annotations

from typing import Dict, List, Optional, Tuple

import numpy as np
import torch
import torch.nn.functional as F

from . import quant as oq
from .attention import chunked_attention


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    x1, x2 = x.chunk(2, dim=-1)
    return torch.cat([-x2, x1], dim=-1)


def compute_rope(head_dim: int, position_ids: torch.Tensor, theta: float):
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2).float() / head_dim))
    freqs = torch.einsum("bi,j->bij", position_ids.float(), inv_freq)
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos(), emb.sin()


def apply_rope(q, k, cos, sin):
    cos = cos.unsqueeze(1)
    sin = sin.unsqueeze(1)
    return q * cos + rotate_half(q) * sin, k * cos + rotate_half(k) * sin


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    dt = x.dtype
    h = x.to(torch.float32)
    var = h.pow(2).mean(-1, keepdim=True)
    h = h * torch.rsqrt(var + eps)
    return w * h.to(dt)


class OracleLinear:
    """fp32 / INT8 / INT4 linear with the reference's per-call dequant."""

    def __init__(self, w: torch.Tensor, bias: Optional[torch.Tensor], scheme: Optional[str],
                 group_size: int = 128):
        self.scheme = scheme
        self.bias = None if bias is None else bias.detach().clone().float()
        self.out_features, self.in_features = w.shape
        wn = w.detach().float().contiguous().numpy()
        if scheme is None:
            self.w = torch.from_numpy(wn.copy())
        elif scheme == "int8":
            p, s = oq.quantize_int8_per_channel(wn)
            self.payload = torch.from_numpy(p)
            self.scales = torch.from_numpy(s)
        elif scheme == "int4":
            p, s, kp = oq.quantize_int4_per_group(wn, group_size)
            self.payload = torch.from_numpy(p)
            self.scales = torch.from_numpy(s)
            self.group_size = group_size
            self.in_features_padded = kp
        else:
            raise ValueError(f"scheme must be None, 'int8' or 'int4', got {scheme!r}")

    def weight(self) -> torch.Tensor:
        if self.scheme is None:
            return self.w
        if self.scheme == "int8":
            return self.payload.to(torch.float32) * self.scales.to(torch.float32).unsqueeze(1)
        n, kp, g = self.out_features, self.in_features_padded, self.group_size
        low = (self.payload & 0x0F).to(torch.int16)
        high = ((self.payload >> 4) & 0x0F).to(torch.int16)
        qu = torch.stack([low, high], dim=-1).reshape(n, kp)
        q = torch.where(qu >= 8, qu - 16, qu).to(torch.int8)
        se = self.scales.to(torch.float32).unsqueeze(-1).expand(-1, -1, g).reshape(n, kp)
        return (q.to(torch.float32) * se)[:, : self.in_features]

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        return F.linear(x, self.weight().to(x.dtype), self.bias)


class OracleModel:
    def __init__(self, cfg, state_dict: Dict[str, torch.Tensor], quantize: Optional[str] = None,
                 group_size: int = 128):
        self.cfg = cfg
        self.n_heads = cfg.heads
        self.n_kv_heads = cfg.kv_heads
        self.head_dim = cfg.head_dim
        self.n_layers = cfg.layers
        self.rope_theta = float(cfg.rope_theta)
        self.eps = cfg.rms_eps
        sd = {k: v.detach().float().cpu() for k, v in state_dict.items()}
        self.embed = sd["model.embed_tokens.weight"]
        self.layers = []
        for i in range(cfg.layers):
            p = f"model.layers.{i}."
            lin = lambda n, b=None: OracleLinear(sd[p + n + ".weight"],
                                                 sd.get(p + n + ".bias"), quantize, group_size)
            self.layers.append(dict(
                ln1=sd[p + "input_layernorm.weight"], ln2=sd[p + "post_attention_layernorm.weight"],
                q=lin("self_attn.q_proj"), k=lin("self_attn.k_proj"), v=lin("self_attn.v_proj"),
                o=lin("self_attn.o_proj"), gate=lin("mlp.gate_proj"), up=lin("mlp.up_proj"),
                down=lin("mlp.down_proj")))
        self.norm = sd["model.norm.weight"]
        self.lm_head = sd["lm_head.weight"] if "lm_head.weight" in sd else self.embed

    def new_pool(self, num_blocks: int, block_size: int) -> torch.Tensor:
        # BlockAllocator layout, prefix_cache.py:67-71
        return torch.zeros((num_blocks, self.n_layers, 2, self.n_kv_heads, block_size,
                            self.head_dim), dtype=torch.float32)

    @torch.inference_mode()
    def forward(self, input_ids: torch.Tensor, position_ids: torch.Tensor, pool: torch.Tensor,
                block_table: List[int], slot_mapping: List[int], prefix_len: int) -> torch.Tensor:
        assert input_ids.shape[0] == 1
        _, L = input_ids.shape
        bs = pool.shape[4]
        hidden = F.embedding(input_ids, self.embed)
        cos, sin = compute_rope(self.head_dim, position_ids, self.rope_theta)
        for i, ly in enumerate(self.layers):
            residual = hidden
            hidden = rms_norm(hidden, ly["ln1"], self.eps)
            q = ly["q"](hidden).view(1, L, self.n_heads, self.head_dim).transpose(1, 2)
            k = ly["k"](hidden).view(1, L, self.n_kv_heads, self.head_dim).transpose(1, 2)
            v = ly["v"](hidden).view(1, L, self.n_kv_heads, self.head_dim).transpose(1, 2)
            q, k = apply_rope(q, k, cos, sin)
            for t in range(L):
                slot = slot_mapping[t]
                pool[slot // bs, i, 0, :, slot % bs, :] = k[0, :, t, :]
                pool[slot // bs, i, 1, :, slot % bs, :] = v[0, :, t, :]
            attn = chunked_attention(q[0], pool[:, i, 0], pool[:, i, 1], block_table,
                                     prefix_len=prefix_len, chunk_len=L, block_size=bs)
            attn = attn.transpose(0, 1).reshape(1, L, self.n_heads * self.head_dim)
            hidden = residual + ly["o"](attn)
            residual = hidden
            hidden = rms_norm(hidden, ly["ln2"], self.eps)
            hidden = ly["down"](F.silu(ly["gate"](hidden)) * ly["up"](hidden))
            hidden = residual + hidden
        hidden = rms_norm(hidden, self.norm, self.eps)
        return F.linear(hidden, self.lm_head)

    @torch.inference_mode()
    def generate(self, prompt_ids: List[int], max_new_tokens: int = 20,
                 eos_token_id: Optional[int] = None, block_size: int = 64,
                 prefill_chunk: Optional[int] = None,
                 return_logits: bool = False):
        lp = len(prompt_ids)
        nb = (lp + max_new_tokens + block_size - 1) // block_size
        pool = self.new_pool(nb, block_size)
        bt = list(range(nb))
        chunk = prefill_chunk or lp
        logits_log = []
        pos = 0
        logits = None
        while pos < lp:
            c = min(chunk, lp - pos)
            ids = torch.tensor([prompt_ids[pos:pos + c]], dtype=torch.long)
            positions = torch.arange(pos, pos + c).unsqueeze(0)
            slots = [bt[p // block_size] * block_size + p % block_size for p in range(pos, pos + c)]
            logits = self.forward(ids, positions, pool, bt, slots, prefix_len=pos)
            pos += c
        tok = int(logits[0, -1].argmax().item())
        out = [tok]
        if return_logits:
            logits_log.append(logits[0, -1].clone())
        if eos_token_id is not None and tok == eos_token_id:
            return (out, logits_log) if return_logits else out
        for step in range(1, max_new_tokens):
            p = lp + step - 1
            slot = bt[p // block_size] * block_size + p % block_size
            logits = self.forward(torch.tensor([[out[-1]]]), torch.tensor([[p]]), pool, bt,
                                  [slot], prefix_len=p)
            tok = int(logits[0, -1].argmax().item())
            out.append(tok)
            if return_logits:
                logits_log.append(logits[0, -1].clone())
            if eos_token_id is not None and tok == eos_token_id:
                break
        return (out, logits_log) if return_logits else out


def top2_margin(logits: torch.Tensor) -> float:
    v = torch.topk(logits.float(), 2).values
    return float(v[0] - v[1])
