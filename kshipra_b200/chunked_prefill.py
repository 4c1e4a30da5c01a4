"""Paged online-softmax attention on the B200 (drop-in for engine/chunked_prefill.py).

``chunked_attention`` keeps the reference signature (chunked_prefill.py:93):
``q [Hq, C, D]``, ``k_pool`` / ``v_pool`` ``[num_blocks, Hkv, B, D]``, a
block-table list, ``prefix_len``, ``chunk_len``, ``block_size`` -> ``[Hq, C, D]``.
When ``k_pool`` / ``v_pool`` are the ``pool[:, layer, 0]`` / ``pool[:, layer, 1]``
views of one ``BlockAllocator`` pool the kernel reads the pool in place;
separately allocated K and V pools are first interleaved into the pool layout.

``paged_attention`` is the batched (varlen) form the model uses.
"""

from __future__ import annotations

import math
from typing import List, Optional

import torch

from . import _lib
from ._lib import call, ptr, stream_ptr


class AttentionWorkspace:
    """Grow-only split-K scratch: one buffer for the prefill attention (its
    entry point clears its counters per call) and one for the fused decode
    attention's key-split states (zeroed here once; its kernels leave the
    counters at zero)."""

    def __init__(self):
        self.buf: Optional[torch.Tensor] = None
        self.dec: Optional[torch.Tensor] = None

    def get(self, nbytes: int, device) -> torch.Tensor:
        if self.buf is None or self.buf.numel() < nbytes or self.buf.device != device:
            self.buf = torch.zeros(max(nbytes, 1 << 16), dtype=torch.uint8, device=device)
        return self.buf

    def decode(self, nbytes: int, device) -> torch.Tensor:
        if self.dec is None or self.dec.numel() < nbytes or self.dec.device != device:
            self.dec = torch.zeros(max(nbytes, 1 << 16), dtype=torch.uint8, device=device)
        return self.dec


_WS = AttentionWorkspace()


def paged_attention(q: torch.Tensor, pool: torch.Tensor, layer: int, block_tables: torch.Tensor,
                    q_start: torch.Tensor, prefix_lens: torch.Tensor, max_q_len: int,
                    max_total_len: int, out: torch.Tensor, flags: Optional[torch.Tensor] = None,
                    ws: AttentionWorkspace = _WS, pool_base: Optional[int] = None,
                    num_layers: Optional[int] = None) -> torch.Tensor:
    """Batched paged attention.

    q [T, Hq, D] fp32; pool [nb, L, 2, Hkv, B, D]; block_tables int32 [S, max_blocks];
    q_start int32 [S+1]; prefix_lens int32 [S]; out [T, Hq, D].
    """
    nb, L, _, hkv, bs, d = pool.shape
    hq = q.shape[1]
    S, max_blocks = block_tables.shape
    wsz = int(_lib.lib().ksh_paged_attention_workspace_size(S, hq, hkv, d, max_q_len, max_total_len))
    buf = ws.get(wsz, q.device)
    call("ksh_paged_attention", ptr(q), hq, d, pool_base if pool_base is not None else ptr(pool),
         nb, num_layers if num_layers is not None else L, layer, hkv, bs, ptr(block_tables),
         max_blocks, ptr(q_start), ptr(prefix_lens), S, max_q_len, max_total_len, ptr(out),
         ptr(buf), buf.numel(), ptr(flags), stream_ptr())
    return out


def _pool_view_info(k_pool: torch.Tensor, v_pool: torch.Tensor):
    """If k/v are pool[:, l, 0] / pool[:, l, 1] views, return (base_ptr, L)."""
    nb, hkv, bs, d = k_pool.shape
    row = hkv * bs * d
    if k_pool.stride()[1:] != (bs * d, d, 1) or v_pool.stride() != k_pool.stride():
        return None
    if k_pool.stride(0) % (2 * row) != 0:
        return None
    if v_pool.data_ptr() - k_pool.data_ptr() != row * k_pool.element_size():
        return None
    return k_pool.data_ptr(), k_pool.stride(0) // (2 * row)


def chunked_attention(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
                      block_table: List[int], prefix_len: int, chunk_len: int,
                      block_size: int) -> torch.Tensor:
    """Drop-in for chunked_attention (chunked_prefill.py:93-140), on the GPU."""
    hq, C, D = q.shape
    hkv = k_pool.shape[1]
    if hq % hkv != 0:
        raise AssertionError(f"GQA requires H_q ({hq}) % H_kv ({hkv}) == 0")
    dev = q.device if q.is_cuda else torch.device("cuda")
    q = q.to(dev, torch.float32)
    k_pool = k_pool.to(dev, torch.float32)
    v_pool = v_pool.to(dev, torch.float32)
    total = prefix_len + chunk_len
    nblk = (total + block_size - 1) // block_size
    bt = torch.tensor([list(block_table[:nblk])], dtype=torch.int32, device=dev)
    info = _pool_view_info(k_pool, v_pool)
    if info is None:
        pool = torch.stack([k_pool, v_pool], dim=1).unsqueeze(1).contiguous()  # [nb,1,2,H,B,D]
        base, L = pool.data_ptr(), 1
    else:
        pool = None
        base, L = info
    qt = q.transpose(0, 1).contiguous()              # [C, Hq, D]
    out = torch.empty_like(qt)
    q_start = torch.tensor([0, C], dtype=torch.int32, device=dev)
    pl = torch.tensor([prefix_len], dtype=torch.int32, device=dev)
    flags = torch.zeros(1, dtype=torch.int32, device=dev)
    shape_pool = torch.empty((k_pool.shape[0], L, 2, hkv, k_pool.shape[2], D), device="meta")
    with torch.cuda.device(dev):
        paged_attention(qt, shape_pool, 0, bt, q_start, pl, C, total, out, flags,
                        pool_base=base, num_layers=L)
    f = int(flags.item())
    if f:
        raise IndexError(f"paged attention reported device flags {f:#x}")
    del pool
    return out.transpose(0, 1).contiguous()


class ChunkedPrefillEngine:
    """Chunked prefill over one sequence with a PrefixCache (chunked_prefill.py:148-246)."""

    def __init__(self, prefix_cache, chunk_size: int, num_heads: int, num_kv_heads: int,
                 head_dim: int) -> None:
        self.cache = prefix_cache
        self.block_size = prefix_cache.block_size
        self.chunk_size = chunk_size
        self.num_heads = num_heads
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.gqa_ratio = num_heads // num_kv_heads

    def prefill(self, token_ids: List[int], embedding_layer, rope_fn, layer_fn) -> torch.Tensor:
        """Chunked prefill of ``token_ids`` after the prefix the radix tree
        holds (chunked_prefill.py:168-246).  Each chunk's rotated K and V are
        written into its blocks of the pool in one indexed store per chunk
        (every layer of the pool, as the reference's scatter does), then the
        chunk attends over the pool's layer-0 views on the GPU."""
        P = len(token_ids)
        matched_blocks, matched_len, node = self.cache.tree.match(token_ids)
        self.cache.tree.pin(node)
        remaining = P - matched_len
        need = math.ceil((matched_len % self.block_size + remaining) / self.block_size)
        new_blocks = self.cache.allocate_blocks(need)
        block_table = matched_blocks + new_blocks
        pool = self.cache.allocator.pool
        bt_dev = torch.as_tensor(block_table, dtype=torch.int64, device=pool.device)
        pos = matched_len
        hidden = None
        while pos < P:
            chunk = token_ids[pos: pos + self.chunk_size]
            C = len(chunk)
            x = embedding_layer(torch.tensor(chunk, device=pool.device))

            def attn_fn(q, k, v, pos=pos, C=C):
                positions = pos + torch.arange(C, device=q.device)
                q, k = rope_fn(q, k, positions)
                p = torch.arange(pos, pos + C, device=pool.device)
                blk = bt_dev[p // self.block_size]
                off = p % self.block_size
                # pool[blk[i], :, 0 | 1, :, off[i], :] = k | v[:, i, :] for all i
                pool[blk, :, 0, :, off, :] = k.transpose(0, 1).unsqueeze(1).to(pool.dtype)
                pool[blk, :, 1, :, off, :] = v.transpose(0, 1).unsqueeze(1).to(pool.dtype)
                return chunked_attention(q, pool[:, 0, 0], pool[:, 0, 1], block_table,
                                         prefix_len=pos, chunk_len=C, block_size=self.block_size)

            hidden = layer_fn(x, attn_fn)
            pos += C
        self.cache.tree.unpin(node)
        return hidden
