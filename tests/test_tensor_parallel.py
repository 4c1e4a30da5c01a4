"""Tensor-parallel sharding, checked on the CPU with two gloo ranks.

The helpers in kshipra_b200.tensor_parallel decide which packed rows / columns
each rank keeps; the GPU model uses exactly these.  Here one Llama layer is
computed in plain torch from the dequantized shards (column-parallel q/k/v and
gate/up, row-parallel o and down with the residual added on rank 0 and an
all-reduce) and compared with the unsharded layer; the vocabulary-parallel
argmax merge is compared with torch.argmax, ties across ranks included.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from kshipra_b200.config import TINY_LLAMA
from kshipra_b200.quantization import QuantizationError, QuantizedWeight
from kshipra_b200.tensor_parallel import (down_col_range, gate_up_row_ranges, merge_argmax,
                                          o_col_range, qkv_row_ranges, take_cols, take_rows,
                                          tp_shape)
from oracle import quant as oq


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _q8(w):
    p, s = oq.quantize_int8_per_channel(w.numpy())
    return QuantizedWeight(payload=torch.from_numpy(p), scales=torch.from_numpy(s),
                           scheme="int8_per_channel", original_shape=tuple(w.shape))


def _q4(w, g=128):
    p, s, kp = oq.quantize_int4_per_group(w.numpy(), g)
    return QuantizedWeight(payload=torch.from_numpy(p), scales=torch.from_numpy(s),
                           scheme="int4_per_group", original_shape=tuple(w.shape), group_size=g,
                           in_features_padded=kp)


def _deq(qw):
    if qw.scheme == "int8_per_channel":
        return torch.from_numpy(oq.dequantize_int8(qw.payload.numpy(), qw.scales.numpy()))
    return torch.from_numpy(oq.dequantize_int4(qw.payload.numpy(), qw.scales.numpy(),
                                               qw.original_shape[1], qw.group_size))


def test_shards_are_slices_of_the_full_packing():
    g = torch.Generator().manual_seed(0)
    w = torch.randn((96, 640), generator=g) * 0.02
    for qw in (_q8(w), _q4(w)):
        full = _deq(qw)
        r = take_rows(qw, [(8, 24), (40, 48)])
        assert torch.equal(_deq(r), torch.cat([full[8:24], full[40:48]]))
        c = take_cols(qw, 128, 384)
        assert torch.equal(_deq(c), full[:, 128:384])
        assert torch.equal(c.payload, qw.payload[:, 128:384] if qw.scheme == "int8_per_channel"
                           else qw.payload[:, 64:192])
    # the last INT4 slice keeps the zero padding; inner slices must be group-aligned
    w2 = torch.randn((16, 700), generator=g) * 0.02
    q4 = _q4(w2)
    tail = take_cols(q4, 512, 700)
    assert tail.in_features_padded == 256 and torch.equal(_deq(tail), _deq(q4)[:, 512:700])
    with pytest.raises(QuantizationError):
        take_cols(q4, 100, 356)


def test_tp_shape_validation():
    from kshipra_b200.config import LLAMA3_8B, QWEN25_05B
    s = tp_shape(LLAMA3_8B, 3, 8, 128)
    assert (s.heads, s.kv_heads, s.inter, s.vocab, s.vocab_start) == (4, 1, 1792, 16032, 48096)
    with pytest.raises(ValueError):
        tp_shape(QWEN25_05B, 0, 4)          # 14 heads do not split over 4 ranks


def _rms(x, w, eps):
    return x / torch.sqrt((x * x).mean(-1, keepdim=True) + eps) * w


def _rope(x, pos, theta):
    d = x.shape[-1]
    inv = 1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.float64) / d))
    f = pos.double()[:, None] * inv[None]
    cos, sin = torch.cat([f.cos(), f.cos()], -1), torch.cat([f.sin(), f.sin()], -1)
    x1, x2 = x[..., : d // 2], x[..., d // 2:]
    return x * cos[:, None] + torch.cat([-x2, x1], -1) * sin[:, None]


def _layer(x, wts, heads, kv_heads, cfg, rank0=True, reduce=None):
    """One Llama layer in float64: q/k/v, RoPE, causal GQA attention, o, SwiGLU."""
    d = cfg.head_dim
    T = x.shape[0]
    xn = _rms(x, wts["ln1"], cfg.rms_eps)
    qkv = xn @ wts["qkv"].T
    q = qkv[:, : heads * d].view(T, heads, d)
    k = qkv[:, heads * d: (heads + kv_heads) * d].view(T, kv_heads, d)
    v = qkv[:, (heads + kv_heads) * d:].view(T, kv_heads, d)
    pos = torch.arange(T)
    q, k = _rope(q, pos, cfg.rope_theta), _rope(k, pos, cfg.rope_theta)
    grp = heads // kv_heads
    k, v = k.repeat_interleave(grp, 1), v.repeat_interleave(grp, 1)
    s = torch.einsum("thd,shd->hts", q, k) / d ** 0.5
    s = s.masked_fill(torch.triu(torch.ones(T, T, dtype=torch.bool), 1), float("-inf"))
    a = torch.einsum("hts,shd->thd", torch.softmax(s, -1), v).reshape(T, heads * d)
    h = a @ wts["o"].T + (x if rank0 else 0)
    if reduce:
        h = reduce(h)
    hn = _rms(h, wts["ln2"], cfg.rms_eps)
    gu = hn @ wts["gate_up"].T
    n = gu.shape[1] // 2
    act = torch.nn.functional.silu(gu[:, :n]) * gu[:, n:]
    out = act @ wts["down"].T + (h if rank0 else 0)
    if reduce:
        out = reduce(out)
    return out


def _weights(cfg, seed):
    g = torch.Generator().manual_seed(seed)
    r = lambda *s: torch.randn(s, generator=g) * 0.05
    qs, kvs = cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim
    return dict(qkv=_q8(r(qs + 2 * kvs, cfg.hidden)), o=_q8(r(cfg.hidden, qs)),
                gate_up=_q8(r(2 * cfg.intermediate, cfg.hidden)),
                down=_q8(r(cfg.hidden, cfg.intermediate)),
                ln1=1.0 + 0.1 * r(cfg.hidden), ln2=1.0 + 0.1 * r(cfg.hidden))


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = TINY_LLAMA
        s = tp_shape(cfg, rank, world)
        W = _weights(cfg, 3)
        x = torch.randn((9, cfg.hidden), generator=torch.Generator().manual_seed(4)).double()
        full = {k: (_deq(v).double() if isinstance(v, QuantizedWeight) else v.double())
                for k, v in W.items()}
        ref = _layer(x, full, cfg.heads, cfg.kv_heads, cfg)
        shard = dict(qkv=_deq(take_rows(W["qkv"], qkv_row_ranges(cfg, s))).double(),
                     o=_deq(take_cols(W["o"], *o_col_range(cfg, s))).double(),
                     gate_up=_deq(take_rows(W["gate_up"], gate_up_row_ranges(cfg, s))).double(),
                     down=_deq(take_cols(W["down"], *down_col_range(cfg, s))).double(),
                     ln1=W["ln1"].double(), ln2=W["ln2"].double())

        def reduce(t):
            t = t.clone()
            dist.all_reduce(t)
            return t
        got = _layer(x, shard, s.heads, s.kv_heads, cfg, rank0=(rank == 0), reduce=reduce)
        err = float((got - ref).abs().max() / ref.abs().max())
        # vocabulary-parallel greedy argmax with a tie between the ranks' ranges
        g = torch.Generator().manual_seed(5)
        logits = torch.randn((6, cfg.vocab), generator=g)
        logits[2, 10] = logits[2, cfg.vocab - 3] = logits[2].max() + 1.0     # tie: index 10 wins
        vl = s.vocab
        loc = logits[:, s.vocab_start:s.vocab_start + vl]
        li = torch.argmax(loc, 1)
        vals = [torch.empty(6) for _ in range(world)]
        idxs = [torch.empty(6, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(vals, loc.gather(1, li.view(-1, 1)).view(-1).contiguous())
        dist.all_gather(idxs, (li + s.vocab_start).contiguous())
        tok = merge_argmax(torch.stack(vals), torch.stack(idxs))
        ok_tok = torch.equal(tok, torch.argmax(logits, 1)) and int(tok[2]) == 10
        out[rank] = (err, ok_tok)
    finally:
        dist.destroy_process_group()


def test_sharded_layer_and_argmax_match_unsharded_two_ranks():
    world = 2
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.spawn(_worker, args=(world, _free_port(), out), nprocs=world, join=True)
    for r in range(world):
        err, ok_tok = out[r]
        assert err < 1e-12, (r, err)
        assert ok_tok, r
