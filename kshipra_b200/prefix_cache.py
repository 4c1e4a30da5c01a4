"""Block pool + radix prefix cache (host-side control plane).

Interface and decisions follow the reference's engine/prefix_cache.py so the
allocator, tree and cache are drop-ins:

* ``BlockAllocator`` (prefix_cache.py:51-82): one preallocated pool tensor of
  layout ``[num_blocks, num_layers, 2, num_kv_heads, block_size, head_dim]``
  (the layout the attention kernels read through block tables) and a LIFO
  free list of block ids;
* ``TokenArena`` (:90-106): flat int32 token storage for tree nodes;
* ``RadixTree`` (:141-302): match with block-aligned split of a partially
  matched node, insert of an unmatched suffix, ref-count pin/unpin along the
  root path, LRU eviction of unpinned leaves that re-scans after every
  eviction so it cascades to parents;
* ``PrefixCache.allocate_blocks`` (:328-335): allocate, evicting on
  ``OutOfBlocksError``.  As in the reference, ids popped before an
  allocation failure are not returned to the free list.

Only the pool tensor lives on the GPU; everything else is host state.
"""

from __future__ import annotations

import time
from typing import Dict, List, Optional, Tuple

import torch


class OutOfBlocksError(RuntimeError):
    """Raised when the allocator cannot satisfy a request without eviction."""


class BlockAllocator:
    def __init__(self, num_blocks: int, block_size: int, num_layers: int, num_kv_heads: int,
                 head_dim: int, dtype: torch.dtype = torch.float16,
                 device: torch.device = torch.device("cpu")) -> None:
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.pool = torch.zeros((num_blocks, num_layers, 2, num_kv_heads, block_size, head_dim),
                                dtype=dtype, device=device)
        self.free_blocks: List[int] = list(range(num_blocks))

    def alloc(self) -> int:
        if not self.free_blocks:
            raise OutOfBlocksError("No free blocks available")
        return self.free_blocks.pop()

    def free(self, block_id: int) -> None:
        self.free_blocks.append(block_id)


class TokenArena:
    def __init__(self, capacity: int) -> None:
        self.capacity = capacity
        self.storage = torch.zeros(capacity, dtype=torch.int32)
        self.ptr = 0

    def alloc(self, tokens: List[int]) -> Tuple[int, int]:
        n = len(tokens)
        if self.ptr + n > self.capacity:
            raise RuntimeError("TokenArena out of memory")
        start = self.ptr
        if n:
            self.storage[start:start + n] = torch.tensor(tokens, dtype=torch.int32)
        self.ptr += n
        return start, n

    def tokens(self, start: int, length: int) -> List[int]:
        return self.storage[start:start + length].tolist()


class RadixNode:
    __slots__ = ("parent", "children", "ref_count", "last_access", "block_ids", "token_start",
                 "token_len")

    def __init__(self, parent: Optional["RadixNode"], token_start: int, token_len: int,
                 block_ids: List[int]) -> None:
        self.parent = parent
        self.children: Dict[int, "RadixNode"] = {}
        self.ref_count = 0
        self.last_access = time.monotonic()
        self.block_ids = block_ids
        self.token_start = token_start
        self.token_len = token_len


class RadixTree:
    def __init__(self, allocator: BlockAllocator, token_arena: TokenArena, block_size: int) -> None:
        self.allocator = allocator
        self.token_arena = token_arena
        self.block_size = block_size
        self.root = RadixNode(None, 0, 0, [])

    def _first_token(self, node: RadixNode) -> int:
        return int(self.token_arena.storage[node.token_start].item())

    def match(self, token_ids: List[int]) -> Tuple[List[int], int, Optional[RadixNode]]:
        """Longest cached prefix: (block ids, matched length, last node).

        A node matched only partially is split at the last whole block of the
        common part; the partial block is recomputed by the caller.
        """
        node = self.root
        blocks: List[int] = []
        matched = 0
        n = len(token_ids)
        while matched < n:
            child = node.children.get(token_ids[matched])
            if child is None:
                break
            ctoks = self.token_arena.tokens(child.token_start, child.token_len)
            limit = min(len(ctoks), n - matched)
            common = 0
            while common < limit and ctoks[common] == token_ids[matched + common]:
                common += 1
            if common == len(ctoks):
                blocks.extend(child.block_ids)
                matched += common
                node = child
                continue
            if common > 0:
                aligned = (common // self.block_size) * self.block_size
                if aligned > 0:
                    self._split_node(child, aligned)
                    blocks.extend(child.block_ids)
                    matched += aligned
                    node = child
            break
        return blocks, matched, node

    def _split_node(self, node: RadixNode, split_len: int) -> None:
        keep = split_len // self.block_size
        tail_tokens = self.token_arena.tokens(node.token_start + split_len,
                                              node.token_len - split_len)
        tail_start, tail_len = self.token_arena.alloc(tail_tokens)
        tail = RadixNode(node, tail_start, tail_len, node.block_ids[keep:])
        tail.ref_count = node.ref_count
        tail.children = node.children
        for c in tail.children.values():
            c.parent = tail
        node.token_len = split_len
        node.block_ids = node.block_ids[:keep]
        node.children = {self._first_token(tail): tail}

    def insert(self, token_ids: List[int], block_ids: List[int], matched_len: int,
               curr: RadixNode) -> RadixNode:
        if len(token_ids) == matched_len:
            return curr
        suffix = token_ids[matched_len:]
        start, length = self.token_arena.alloc(suffix)
        node = RadixNode(curr, start, length, block_ids)
        curr.children[suffix[0]] = node
        return node

    def pin(self, node: Optional[RadixNode]) -> None:
        while node is not None:
            node.ref_count += 1
            node.last_access = time.monotonic()
            node = node.parent

    def unpin(self, node: Optional[RadixNode]) -> None:
        while node is not None:
            node.ref_count -= 1
            node = node.parent

    def _evictable_leaves(self) -> List[RadixNode]:
        out = []
        stack = [self.root]
        while stack:
            nd = stack.pop()
            if nd is not self.root and not nd.children and nd.ref_count == 0:
                out.append(nd)
            stack.extend(nd.children.values())
        return out

    def evict(self, num_blocks_needed: int) -> int:
        """Evict LRU unpinned leaves until enough blocks are freed; returns blocks freed."""
        freed = 0
        while freed < num_blocks_needed:
            leaves = self._evictable_leaves()
            if not leaves:
                break
            victim = min(leaves, key=lambda nd: nd.last_access)
            del victim.parent.children[self._first_token(victim)]
            for b in victim.block_ids:
                self.allocator.free(b)
            freed += len(victim.block_ids)
        return freed


class PrefixCache:
    def __init__(self, num_blocks: int, block_size: int, num_layers: int, num_kv_heads: int,
                 head_dim: int, dtype: torch.dtype = torch.float16,
                 device: torch.device = torch.device("cpu")) -> None:
        self.block_size = block_size
        self.allocator = BlockAllocator(num_blocks, block_size, num_layers, num_kv_heads,
                                        head_dim, dtype, device)
        self.token_arena = TokenArena(capacity=1024 * 1024)
        self.tree = RadixTree(self.allocator, self.token_arena, block_size)

    def allocate_blocks(self, num_blocks: int) -> List[int]:
        try:
            return [self.allocator.alloc() for _ in range(num_blocks)]
        except OutOfBlocksError:
            if self.tree.evict(num_blocks) < num_blocks:
                raise OutOfBlocksError("Not enough evictable memory to satisfy request")
            return [self.allocator.alloc() for _ in range(num_blocks)]
