"""torch-CPU restatement of the reference paged attention.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

* ``chunked_attention``     -- engine/chunked_prefill.py:93-140: per KV block
  of the block table, scores ``q K^T / sqrt(D)``, causal mask only on blocks
  that reach past ``prefix_len``, running max / sum / accumulator merge with
  ``m_safe = 0`` when the running max is still -inf, GQA by repeating each KV
  head ``g = Hq / Hkv`` times; output ``acc / l``.
* ``monolithic_attention``  -- engine/chunked_prefill.py:47-90: contiguous K/V
  with a ``[C, P+C]`` mask through SDPA (no GQA).
* ``gather_contiguous``     -- helper that builds contiguous K/V from a pool
  and block table, for monolithic checks of paged layouts.

The ops are the reference's own (bmm, exp, max) in the same order, so on the
same machine the output is bit-identical to the reference.
"""

from __future__ import annotations

import math
from typing import List

import torch
import torch.nn.functional as F


def chunked_attention(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
                      block_table: List[int], prefix_len: int, chunk_len: int,
                      block_size: int) -> torch.Tensor:
    hq = q.shape[0]
    hkv = k_pool.shape[1]
    if hq % hkv != 0:
        raise ValueError(f"GQA requires H_q ({hq}) % H_kv ({hkv}) == 0")
    g = hq // hkv
    _, c, d = q.shape
    scale = 1.0 / math.sqrt(d)
    total = prefix_len + chunk_len
    m = torch.full((hq, c), float("-inf"))
    l = torch.zeros((hq, c))
    acc = torch.zeros((hq, c, d))
    qpos = prefix_len + torch.arange(c)
    for j in range((total + block_size - 1) // block_size):
        bid = block_table[j]
        start = j * block_size
        end = min(start + block_size, total)
        nv = end - start
        kt = k_pool[bid, :, :nv, :]
        vt = v_pool[bid, :, :nv, :]
        if g > 1:
            kt = kt.repeat_interleave(g, dim=0)
            vt = vt.repeat_interleave(g, dim=0)
        s = torch.bmm(q, kt.transpose(1, 2)) * scale
        if end > prefix_len:
            kpos = start + torch.arange(nv)
            mask = kpos.unsqueeze(0) > qpos.unsqueeze(1)
            s.masked_fill_(mask.unsqueeze(0), float("-inf"))
        m_new = torch.max(m, s.max(dim=-1).values)
        m_safe = torch.where(torch.isinf(m_new), torch.zeros_like(m_new), m_new)
        p = torch.exp(s - m_safe.unsqueeze(-1))
        corr = torch.exp(m - m_safe)
        l = l * corr + p.sum(dim=-1)
        acc = acc * corr.unsqueeze(-1) + torch.bmm(p, vt)
        m = m_new
    return acc / l.unsqueeze(-1)


def monolithic_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                         prefix_len: int, chunk_len: int) -> torch.Tensor:
    mask = torch.ones((chunk_len, prefix_len + chunk_len), dtype=torch.bool)
    mask[:, prefix_len:] = torch.tril(torch.ones((chunk_len, chunk_len), dtype=torch.bool))
    out = F.scaled_dot_product_attention(q.unsqueeze(0), k_cache.unsqueeze(0),
                                         v_cache.unsqueeze(0),
                                         attn_mask=mask.unsqueeze(0).unsqueeze(0))
    return out.squeeze(0)


def gather_contiguous(pool_kv: torch.Tensor, block_table: List[int], total: int) -> torch.Tensor:
    """pool_kv [nb, H, B, D] -> [H, total, D] following the block table."""
    b = pool_kv.shape[2]
    nblk = (total + b - 1) // b
    parts = [pool_kv[block_table[j]] for j in range(nblk)]
    return torch.cat(parts, dim=1)[:, :total, :]
