"""Tensor-parallel sharding of the packed weights (8B-class models).

Column-parallel projections (q/k/v by heads, gate/up by intermediate rows,
the lm_head by vocabulary rows) keep a subset of output rows; row-parallel
ones (o, down) keep a slice of the input columns, and their partial outputs
are summed by an NCCL all-reduce.  Every shard is cut out of the packed bytes
of the full-matrix quantization, never re-quantized: an INT8 row keeps its
per-channel scale, and an INT4 column slice starts and ends on a group
boundary with the groups' scales, so the rank's bytes are exactly the
reference's bytes for those rows / columns (quantization.py:196-318).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

import torch

from .quantization import QuantizationError, QuantizedWeight


@dataclass(frozen=True)
class TPShape:
    """Per-rank sizes of a tensor-parallel layout."""

    rank: int
    world: int
    heads: int          # query heads on this rank
    kv_heads: int       # K/V heads on this rank
    inter: int          # intermediate rows on this rank
    vocab: int          # lm_head rows on this rank
    vocab_start: int


def tp_shape(cfg, rank: int, world: int, group_size: Optional[int] = None) -> TPShape:
    """Validate that ``cfg`` splits over ``world`` ranks and give rank's sizes.

    Heads, K/V heads, intermediate rows and vocabulary must divide evenly; for
    INT4 the row-parallel input slices (q_size / world, intermediate / world)
    must be whole groups."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad tensor-parallel rank {rank} of {world}")
    for name, v in (("heads", cfg.heads), ("kv_heads", cfg.kv_heads),
                    ("intermediate", cfg.intermediate), ("vocab", cfg.vocab)):
        if v % world:
            raise ValueError(f"{name} = {v} does not split over {world} ranks")
    if group_size and world > 1:
        for name, v in (("q_size", cfg.heads * cfg.head_dim), ("intermediate", cfg.intermediate)):
            if (v // world) % group_size:
                raise ValueError(f"{name} / {world} is not a whole number of {group_size}-groups")
    vl = cfg.vocab // world
    return TPShape(rank, world, cfg.heads // world, cfg.kv_heads // world,
                   cfg.intermediate // world, vl, rank * vl)


def _row_index(ranges: Sequence[Tuple[int, int]], device) -> torch.Tensor:
    return torch.cat([torch.arange(a, b, device=device) for a, b in ranges])


def take_rows(qw: QuantizedWeight, ranges: Sequence[Tuple[int, int]]) -> QuantizedWeight:
    """Output rows ``ranges`` (concatenated, in order) of a packed weight."""
    idx = _row_index(ranges, qw.payload.device)
    n = int(idx.numel())
    return QuantizedWeight(payload=qw.payload.index_select(0, idx).contiguous(),
                           scales=qw.scales.index_select(0, idx).contiguous(), scheme=qw.scheme,
                           original_shape=(n, qw.original_shape[1]), group_size=qw.group_size,
                           in_features_padded=qw.in_features_padded)


def take_cols(qw: QuantizedWeight, c0: int, c1: int) -> QuantizedWeight:
    """Input columns [c0, c1) of a packed weight.  INT4: c0 must be a group
    boundary, and c1 too unless it is the last column (the zero padding up
    to ``in_features_padded`` then comes along)."""
    n, k = qw.original_shape
    if not 0 <= c0 < c1 <= k:
        raise ValueError(f"columns [{c0}, {c1}) outside [0, {k})")
    if qw.scheme == "int8_per_channel":
        return QuantizedWeight(payload=qw.payload[:, c0:c1].contiguous(), scales=qw.scales,
                               scheme=qw.scheme, original_shape=(n, c1 - c0))
    g = qw.group_size
    kp = qw.in_features_padded
    end = kp if c1 == k else c1
    if c0 % g or end % g:
        raise QuantizationError(f"INT4 column slice [{c0}, {c1}) is not on {g}-groups")
    return QuantizedWeight(payload=qw.payload[:, c0 // 2:end // 2].contiguous(),
                           scales=qw.scales[:, c0 // g:end // g].contiguous(), scheme=qw.scheme,
                           original_shape=(n, c1 - c0), group_size=g, in_features_padded=end - c0)


def qkv_row_ranges(cfg, s: TPShape) -> List[Tuple[int, int]]:
    """Rows of the fused [q; k; v] projection that rank ``s.rank`` keeps."""
    d = cfg.head_dim
    qs, kvs = cfg.heads * d, cfg.kv_heads * d
    q0 = s.rank * s.heads * d
    k0 = s.rank * s.kv_heads * d
    return [(q0, q0 + s.heads * d), (qs + k0, qs + k0 + s.kv_heads * d),
            (qs + kvs + k0, qs + kvs + k0 + s.kv_heads * d)]


def gate_up_row_ranges(cfg, s: TPShape) -> List[Tuple[int, int]]:
    """Rows of the fused [gate; up] projection that rank ``s.rank`` keeps."""
    i0 = s.rank * s.inter
    return [(i0, i0 + s.inter), (cfg.intermediate + i0, cfg.intermediate + i0 + s.inter)]


def o_col_range(cfg, s: TPShape) -> Tuple[int, int]:
    c0 = s.rank * s.heads * cfg.head_dim
    return c0, c0 + s.heads * cfg.head_dim


def down_col_range(cfg, s: TPShape) -> Tuple[int, int]:
    c0 = s.rank * s.inter
    return c0, c0 + s.inter


def merge_argmax(values: torch.Tensor, indices: torch.Tensor) -> torch.Tensor:
    """Global greedy token from per-rank (max logit, global index) pairs.

    ``values``/``indices`` are [world, m]; ranks own increasing vocabulary
    ranges and each reports its first maximum, so the first rank holding the
    largest value gives the first index of the global maximum, which is what
    torch.argmax over the full logits returns (model.py:187,200)."""
    best = torch.argmax(values, dim=0)
    return indices.gather(0, best.view(1, -1)).view(-1)
