"""KshipraModel on the B200: the quantized forward through the CUDA kernels.

Drop-in for the reference's engine/model.py ``KshipraModel``:

* ``KshipraModel(hf_model, device, quantize)`` (model.py:61-91) takes a HF
  Llama / Qwen2 ``*ForCausalLM`` and quantizes all seven projections per
  layer (INT8 per channel or INT4 per group of 128; ``None`` keeps fp32);
  embeddings and ``lm_head`` stay fp32;
* ``forward(input_ids, position_ids, pool, block_table, slot_mapping,
  prefix_len)`` (model.py:93-151) returns logits ``[1, L, vocab]`` and writes
  the chunk's K/V into ``pool`` (BlockAllocator layout);
* ``generate(prompt_ids, max_new_tokens, eos_token_id, block_size)``
  (model.py:154-205) is greedy decoding with a fresh pool.

Per layer the forward runs: RMSNorm -> fused q/k/v dequant-linear (+bias) ->
RoPE + K/V scatter into the pool -> paged attention -> o_proj with the
residual add fused -> RMSNorm -> fused gate/up dequant-linear with SwiGLU ->
down_proj with the residual add fused.  The decode step of ``generate``
(embedding -> layers -> final norm -> lm_head + argmax -> on-device position /
slot advance) is captured once in a CUDA graph and replayed per token, so
greedy decoding has no host round trip until the end.

Weights for q/k/v and gate/up are packed into one buffer each (per-row
quantization makes that byte-identical to packing them separately); the
per-projection ``QuantizedLinear`` modules exposed on ``layers[i]`` are views
into those buffers.
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence

import torch

from . import _lib
from ._lib import call, ptr, stream_ptr
from .chunked_prefill import AttentionWorkspace, paged_attention
from .config import ModelConfig
from .prefix_cache import BlockAllocator
from .tensor_parallel import (down_col_range, gate_up_row_ranges, merge_argmax, o_col_range,
                              qkv_row_ranges, take_cols, take_rows, tp_shape)
from .quantization import (QuantizedLinear, QuantizedWeight, Workspace, linear_launch,
                           quantize_int4_per_group, quantize_int8_per_channel, swiglu_launch)

FLAG_NAMES = {1: "non-finite weight", 2: "block id out of range", 4: "slot out of range",
              8: "position outside the RoPE table", 16: "token id out of range",
              32: "sequence longer than its block table", 64: "a bounded device wait gave up"}
FLAG_TIMEOUT = 64
LM_GEMV_ROWS = 16            # lm_head rows served by the fp32 GEMV; more go to tensor cores
PEER_AR_ROWS = 256           # token rows of a row-parallel sum done over peer memory


# GQA group sizes the fused decode-attention kernel is instantiated for, per head dim.
_DECODE_GROUPS = {64: (1, 2, 4, 7, 8), 128: (1, 2, 4, 8)}


class KshipraDeviceError(IndexError):
    """A kernel reported a data-dependent error through the device status word."""


class KshipraDeviceTimeout(TimeoutError):
    """A kernel's bounded wait gave up (KSH_FLAG_TIMEOUT); its outputs are invalid."""


def _check_flags(flags: torch.Tensor) -> None:
    f = int(flags.item())
    if f:
        names = [n for b, n in FLAG_NAMES.items() if f & b]
        flags.zero_()
        msg = "device reported: " + ", ".join(names)
        if f & FLAG_TIMEOUT:
            raise KshipraDeviceTimeout(msg)
        raise KshipraDeviceError(msg)


def rope_tables(head_dim: int, theta: float, max_pos: int):
    """cos / sin of position * inv_freq, [max_pos, head_dim/2], by the
    reference's formula (model.py:35-44) evaluated on the CPU in fp32."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2).float() / head_dim))
    pos = torch.arange(max_pos).float()
    freqs = torch.einsum("i,j->ij", pos, inv_freq)
    return freqs.cos().contiguous(), freqs.sin().contiguous()


@dataclass
class _Proj:
    """One (possibly fused) projection: quantized or fp32."""
    qw: Optional[QuantizedWeight]
    w: Optional[torch.Tensor]
    bias: Optional[torch.Tensor]
    n: int


class _Layer:
    pass


class KshipraModel:
    """Runs a Llama / Qwen2 model through the B200 kernels."""

    def __init__(self, hf_model=None, device: torch.device = None, quantize: Optional[str] = None,
                 *, config: Optional[ModelConfig] = None,
                 state_dict: Optional[Dict[str, torch.Tensor]] = None, group_size: int = 128,
                 tp: Optional[tuple] = None) -> None:
        """``tp=(rank, world, group)`` builds rank's tensor-parallel shard: heads,
        intermediate rows and lm_head vocabulary split over ``world`` ranks
        (one process per GPU), row-parallel sums all-reduced over ``group``
        (a torch.distributed NCCL group; None = the default group)."""
        if quantize not in (None, "int8", "int4"):
            raise ValueError(f"quantize must be None, 'int8' or 'int4', got {quantize!r}")
        if device is None or torch.device(device).type != "cuda":
            if not torch.cuda.is_available():
                raise _lib.KshipraLibraryError("KshipraModel runs on CUDA only (no CPU path)")
            device = torch.device("cuda", torch.cuda.current_device())
        self.device = torch.device(device)
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        if hf_model is not None:
            config = ModelConfig.from_hf_config(hf_model.config)
            state_dict = hf_model.state_dict()
        if config is None or state_dict is None:
            raise ValueError("pass an HF model, or config= and state_dict=")
        _lib.lib()
        self.model = hf_model
        self.cfg = config
        self.quantize = quantize
        self.group_size = group_size
        self.tp_rank, self.tp_world, self.tp_group = (0, 1, None) if tp is None else tp
        self.tp = tp_shape(config, self.tp_rank, self.tp_world,
                           group_size if quantize == "int4" else None)
        self.n_heads = self.tp.heads                 # per rank
        self.n_kv_heads = self.tp.kv_heads
        self.head_dim = config.head_dim
        self.n_layers = config.layers
        self.vocab_size = config.vocab
        self.hidden = config.hidden
        self.inter = self.tp.inter
        self.eps = float(config.rms_eps)
        self._rope_theta = float(config.rope_theta)
        self._rope = None
        self.max_positions = config.max_positions
        self.flags = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._lin_ws = Workspace()
        self._attn_ws = AttentionWorkspace()
        self._lm_ws: Optional[torch.Tensor] = None
        self._lm_hl = None
        self.lm_tc = True            # > 16 lm_head rows on the tensor-core kernel
        self._gen_cache: Dict[tuple, tuple] = {}
        self.fused_decode = True
        with torch.cuda.device(self.device):
            self._load(state_dict)
        # Row-parallel sums of up to PEER_AR_ROWS rows over peer memory (a
        # collective set-up: every rank builds its shard at the same point);
        # KSH_PEER_AR=0 in the environment keeps NCCL for them.
        self._peer_ar = None
        if self.tp_world > 1 and os.environ.get("KSH_PEER_AR", "1") != "0":
            from .peer_allreduce import PeerAllReduce
            self._peer_ar = PeerAllReduce(self.tp_group, self.device, PEER_AR_ROWS * self.hidden)

    # ------------------------------------------------------------------ #
    # weights
    # ------------------------------------------------------------------ #

    def _pack(self, w: torch.Tensor) -> _Proj:
        if self.quantize == "int8":
            return _Proj(quantize_int8_per_channel(w), None, None, w.shape[0])
        if self.quantize == "int4":
            return _Proj(quantize_int4_per_group(w, self.group_size), None, None, w.shape[0])
        return _Proj(None, w.to(self.device, torch.float32).contiguous(), None, w.shape[0])

    def _view(self, proj: _Proj, r0: int, r1: int, bias=None):
        """QuantizedLinear / fp32 weight view of rows [r0, r1) of a fused projection."""
        if proj.qw is None:
            lin = torch.nn.Linear(proj.w.shape[1], r1 - r0, bias=bias is not None,
                                  device="meta")
            lin.weight = torch.nn.Parameter(proj.w[r0:r1], requires_grad=False)
            if bias is not None:
                lin.bias = torch.nn.Parameter(bias, requires_grad=False)
            return lin
        qw = proj.qw
        sub = QuantizedWeight(payload=qw.payload[r0:r1], scales=qw.scales[r0:r1], scheme=qw.scheme,
                              original_shape=(r1 - r0, qw.original_shape[1]),
                              group_size=qw.group_size, in_features_padded=qw.in_features_padded)
        return QuantizedLinear.from_quantized(sub, bias)

    def _shard_rows(self, proj: _Proj, ranges) -> _Proj:
        if self.tp_world == 1:
            return proj
        if proj.qw is not None:
            return _Proj(take_rows(proj.qw, ranges), None, None, sum(b - a for a, b in ranges))
        w = torch.cat([proj.w[a:b] for a, b in ranges]).contiguous()
        return _Proj(None, w, None, w.shape[0])

    def _shard_cols(self, proj: _Proj, c0: int, c1: int) -> _Proj:
        if self.tp_world == 1:
            return proj
        if proj.qw is not None:
            return _Proj(take_cols(proj.qw, c0, c1), None, None, proj.qw.original_shape[0])
        return _Proj(None, proj.w[:, c0:c1].contiguous(), None, proj.w.shape[0])

    def _load(self, sd: Dict[str, torch.Tensor]) -> None:
        dev = self.device
        g = lambda k: sd[k].detach().to(dev, torch.float32)
        self.embed = g("model.embed_tokens.weight").contiguous()
        lm = (self.embed if ("lm_head.weight" not in sd or self.cfg.tie_embeddings)
              else g("lm_head.weight").contiguous())
        v0 = self.tp.vocab_start
        self.lm_head = lm if self.tp_world == 1 else lm[v0:v0 + self.tp.vocab].contiguous()
        self.norm_w = g("model.norm.weight").contiguous()
        qs, kvs = self.cfg.q_size, self.cfg.kv_size
        tpr = self.tp
        qkv_rows = qkv_row_ranges(self.cfg, tpr)
        gu_rows = gate_up_row_ranges(self.cfg, tpr)
        self.layers: List[_Layer] = []
        for i in range(self.n_layers):
            p = f"model.layers.{i}."
            L = _Layer()
            L.ln1 = g(p + "input_layernorm.weight").contiguous()
            L.ln2 = g(p + "post_attention_layernorm.weight").contiguous()
            wq, wk, wv = g(p + "self_attn.q_proj.weight"), g(p + "self_attn.k_proj.weight"), g(
                p + "self_attn.v_proj.weight")
            L.qkv = self._shard_rows(self._pack(torch.cat([wq, wk, wv], dim=0)), qkv_rows)
            bq = sd.get(p + "self_attn.q_proj.bias")
            if bq is not None:
                bias = torch.cat([g(p + "self_attn.q_proj.bias"), g(p + "self_attn.k_proj.bias"),
                                  g(p + "self_attn.v_proj.bias")])
                if self.tp_world > 1:
                    bias = torch.cat([bias[a:b] for a, b in qkv_rows])
                L.qkv.bias = bias.contiguous()
            del wq, wk, wv
            L.o = self._shard_cols(self._pack(g(p + "self_attn.o_proj.weight")),
                                   *o_col_range(self.cfg, tpr))
            L.gate_up = self._shard_rows(self._pack(torch.cat([g(p + "mlp.gate_proj.weight"),
                                                               g(p + "mlp.up_proj.weight")], dim=0)),
                                         gu_rows)
            L.down = self._shard_cols(self._pack(g(p + "mlp.down_proj.weight")),
                                      *down_col_range(self.cfg, tpr))
            self.layers.append(L)
            if self.tp_world > 1:
                continue            # the per-projection drop-in views are single-GPU only
            b = L.qkv.bias
            L.q_proj = self._view(L.qkv, 0, qs, None if b is None else b[:qs])
            L.k_proj = self._view(L.qkv, qs, qs + kvs, None if b is None else b[qs:qs + kvs])
            L.v_proj = self._view(L.qkv, qs + kvs, qs + 2 * kvs, None if b is None else b[qs + kvs:])
            L.o_proj = self._view(L.o, 0, self.hidden)
            L.gate_proj = self._view(L.gate_up, 0, self.inter)
            L.up_proj = self._view(L.gate_up, self.inter, 2 * self.inter)
            L.down_proj = self._view(L.down, 0, self.hidden)
        torch.cuda.synchronize(dev)

    def weight_bytes(self) -> Dict[str, int]:
        """Bytes one decode step streams, by kind (algorithmic HBM traffic)."""
        def pb(p: _Proj) -> int:
            if p.qw is not None:
                return p.qw.storage_bytes()
            return p.w.numel() * 4
        layers = sum(pb(L.qkv) + pb(L.o) + pb(L.gate_up) + pb(L.down) for L in self.layers)
        return {"layers": layers, "lm_head": self.lm_head.numel() * 4}

    # ------------------------------------------------------------------ #
    # RoPE
    # ------------------------------------------------------------------ #

    @property
    def rope_theta(self) -> float:
        return self._rope_theta

    @rope_theta.setter
    def rope_theta(self, v: float) -> None:
        self._rope_theta = float(v)
        self._rope = None
        self._gen_cache.clear()      # captured graphs point at the old tables

    def _rope_tables(self):
        if self._rope is None:
            c, s = rope_tables(self.head_dim, self._rope_theta, self.max_positions)
            self._rope = (c.to(self.device), s.to(self.device))
        return self._rope

    # ------------------------------------------------------------------ #
    # core: one pass over a varlen batch of token rows
    # ------------------------------------------------------------------ #

    def _alloc_acts(self, T: int) -> Dict[str, torch.Tensor]:
        dev, f = self.device, torch.float32
        return dict(
            hidden=torch.empty((T, self.hidden), dtype=f, device=dev),
            xn=torch.empty((T, self.hidden), dtype=f, device=dev),
            qkv=torch.empty((T, (self.n_heads + 2 * self.n_kv_heads) * self.head_dim), dtype=f,
                            device=dev),
            q=torch.empty((T, self.n_heads, self.head_dim), dtype=f, device=dev),
            attn=torch.empty((T, self.n_heads, self.head_dim), dtype=f, device=dev),
            h=torch.empty((T, self.inter), dtype=f, device=dev),
        )

    def _run_layers(self, acts, ids, positions, slots, block_tables, q_start, prefix_lens,
                    num_seqs: int, max_q_len: int, max_total_len: int, pool: torch.Tensor,
                    lin_ws: Workspace, attn_ws: AttentionWorkspace) -> torch.Tensor:
        T = ids.shape[0]
        s = stream_ptr()
        hid, xn, qkv, q, attn, h = (acts[k] for k in ("hidden", "xn", "qkv", "q", "attn", "h"))
        nb, L, _, hkv, bs, d = pool.shape
        if pool.dtype != torch.float32 or not pool.is_contiguous():
            raise ValueError("the pool must be a contiguous fp32 CUDA tensor")
        rc, rs = self._rope_tables()
        call("ksh_embedding", ptr(ids), T, ptr(self.embed), self.vocab_size, self.hidden, ptr(hid),
             ptr(self.flags), s)
        eps = self.eps
        # decode step (one token per sequence, position == prefix length): the
        # fused RoPE + K/V write + attention kernel
        fused = (max_q_len == 1 and T == num_seqs and self.fused_decode and bs % 16 == 0
                 and d in (64, 128) and self.n_heads // self.n_kv_heads in _DECODE_GROUPS[d])
        if fused:   # key-split partial states (zeroed once; the kernels leave the counters at 0)
            dec_ws = attn_ws.decode(int(_lib.lib().ksh_decode_attention_workspace_size(
                T, self.n_heads, self.n_kv_heads, d)), self.device)
        for i, Ly in enumerate(self.layers):
            linear_launch(hid, Ly.qkv.qw, Ly.qkv.w, Ly.qkv.bias, qkv, ws=lin_ws, norm_w=Ly.ln1,
                          eps=eps)
            if fused:
                call("ksh_decode_attention_ws", ptr(qkv), T, self.n_heads, self.n_kv_heads, d,
                     ptr(positions), ptr(slots), ptr(rc), ptr(rs), rc.shape[0], ptr(pool), nb, L,
                     i, bs, ptr(block_tables), block_tables.shape[1], max_total_len, ptr(attn),
                     ptr(dec_ws), dec_ws.numel(), ptr(self.flags), s)
            else:
                call("ksh_rope_kv_write", ptr(qkv), T, self.n_heads, self.n_kv_heads,
                     self.head_dim, ptr(positions), ptr(slots), ptr(rc), ptr(rs), rc.shape[0],
                     ptr(q), ptr(pool), nb, L, i, bs, ptr(self.flags), s)
                paged_attention(q, pool, i, block_tables, q_start, prefix_lens, max_q_len,
                                max_total_len, attn, self.flags, ws=attn_ws)
            self._row_parallel(attn.view(T, -1), Ly.o, hid, lin_ws)
            swiglu_launch(hid, Ly.gate_up.qw, Ly.gate_up.w, self.inter, h, ws=lin_ws,
                          norm_w=Ly.ln2, eps=eps)
            self._row_parallel(h, Ly.down, hid, lin_ws)
        return hid

    def _row_parallel(self, x_in: torch.Tensor, proj: "_Proj", hid: torch.Tensor,
                      lin_ws: Workspace) -> None:
        """hid += x_in @ W^T, W split by input columns over the ranks: rank 0
        adds the residual, every rank its partial sum, then the sum over the
        ranks.  Up to the peer buffer's size the partial goes straight into
        symmetric memory and this library's peer all-reduce sums it; larger
        ones (prefill chunks) use NCCL."""
        if self.tp_world == 1:
            linear_launch(x_in, proj.qw, proj.w, None, hid, residual=hid, ws=lin_ws)
            return
        res = hid if self.tp_rank == 0 else None
        n = hid.numel()
        par = self._peer_ar
        if par is not None and n <= par.n_max and n % 4 == 0:
            dst = par.partial(n).view(hid.shape)
            linear_launch(x_in, proj.qw, proj.w, None, dst, residual=res, ws=lin_ws)
            par.reduce(hid, n)
        else:
            linear_launch(x_in, proj.qw, proj.w, None, hid, residual=res, ws=lin_ws)
            torch.distributed.all_reduce(hid, group=self.tp_group)

    def lm_ws_bytes(self, m: int) -> int:
        """Workspace bytes of the lm_head call for ``m`` rows."""
        n = int(_lib.lib().ksh_lm_head_workspace_size(m, self.tp.vocab))
        if m > LM_GEMV_ROWS and self.lm_tc:
            n = max(n, int(_lib.lib().ksh_lm_head_tc_workspace_size(m, self.hidden, self.tp.vocab)))
        return n

    def _lm_workspace(self, m: int) -> torch.Tensor:
        need = self.lm_ws_bytes(m)
        if self._lm_ws is None or self._lm_ws.numel() < need:
            self._lm_ws = torch.empty(need, dtype=torch.uint8, device=self.device)
        return self._lm_ws

    def lm_head_split(self):
        """The lm_head weight (this rank's vocabulary rows) split once into
        fp16 hi / lo terms with a power-of-two scale per row, for the
        tensor-core lm_head of more than 16 rows (same 4 bytes per weight as
        the fp32 copy, which the GEMV path keeps reading).  Made on first use;
        callers that capture CUDA graphs make it before the capture."""
        if self._lm_hl is None:
            V, H = self.lm_head.shape
            with torch.cuda.device(self.device):
                hi = torch.empty((V, H), dtype=torch.float16, device=self.device)
                lo = torch.empty((V, H), dtype=torch.float16, device=self.device)
                inv = torch.empty(V, dtype=torch.float32, device=self.device)
                call("ksh_lm_head_split_weight", ptr(self.lm_head), V, H, ptr(hi), ptr(lo),
                     ptr(inv), ptr(self.flags), stream_ptr())
                _check_flags(self.flags)
            self._lm_hl = (hi, lo, inv)
        return self._lm_hl

    def _lm_head_call(self, x: torch.Tensor, m: int, logits: Optional[torch.Tensor],
                      tokens: Optional[torch.Tensor], ws: torch.Tensor) -> None:
        """Fused final norm + lm_head (+ argmax): a GEMV up to 16 rows, above
        that the tensor-core kernel on the split weight (one pass over the
        weight per 64 rows)."""
        vl = self.tp.vocab
        if m > LM_GEMV_ROWS and self.lm_tc:
            hi, lo, inv = self.lm_head_split()
            call("ksh_lm_head_argmax_tc", ptr(x), m, self.hidden, ptr(self.norm_w), self.eps,
                 ptr(hi), ptr(lo), ptr(inv), vl, ptr(logits), ptr(tokens), ptr(ws), ws.numel(),
                 stream_ptr())
        else:
            call("ksh_lm_head_argmax", ptr(x), m, self.hidden, ptr(self.norm_w), self.eps,
                 ptr(self.lm_head), vl, ptr(logits), ptr(tokens), ptr(ws), ws.numel(),
                 stream_ptr())

    def _lm_head_argmax(self, x: torch.Tensor, tokens: torch.Tensor,
                        ws: Optional[torch.Tensor] = None, logits: Optional[torch.Tensor] = None):
        m = x.shape[0]
        if ws is None:
            ws = self._lm_workspace(m)
        if self.tp_world > 1 and logits is None:
            logits = self._tp_logits(m)
        self._lm_head_call(x, m, logits, tokens, ws)
        if self.tp_world > 1:
            # vocabulary-parallel: every rank's (max logit, global index), then
            # the first index of the overall maximum
            val = logits[:m].gather(1, tokens.view(-1, 1)).view(-1)
            idx = tokens + self.tp.vocab_start
            vals = torch.empty((self.tp_world, m), dtype=val.dtype, device=val.device)
            idxs = torch.empty((self.tp_world, m), dtype=idx.dtype, device=idx.device)
            torch.distributed.all_gather_into_tensor(vals, val.contiguous(), group=self.tp_group)
            torch.distributed.all_gather_into_tensor(idxs, idx.contiguous(), group=self.tp_group)
            tokens.copy_(merge_argmax(vals, idxs))

    def _tp_logits(self, m: int) -> torch.Tensor:
        buf = getattr(self, "_tp_lg", None)
        if buf is None or buf.shape[0] < m:
            buf = torch.empty((m, self.tp.vocab), dtype=torch.float32, device=self.device)
            self._tp_lg = buf
        return buf[:m]

    # ------------------------------------------------------------------ #
    # reference API
    # ------------------------------------------------------------------ #

    @torch.inference_mode()
    def forward(self, input_ids: torch.Tensor, position_ids: torch.Tensor, pool: torch.Tensor,
                block_table: List[int], slot_mapping: List[int], prefix_len: int) -> torch.Tensor:
        """Logits [1, L, vocab]; writes the chunk's K/V into ``pool``."""
        assert input_ids.shape[0] == 1, "KshipraModel expects batch=1"
        L = input_ids.shape[1]
        dev = self.device
        with torch.cuda.device(dev):
            ids = input_ids.reshape(-1).to(dev, torch.int64)
            pos = position_ids.reshape(-1).to(dev, torch.int64)
            slots = torch.as_tensor(list(slot_mapping), dtype=torch.int64).to(dev)
            bs = pool.shape[4]
            nblk = (prefix_len + L + bs - 1) // bs
            bt = torch.as_tensor([list(block_table)[:max(nblk, 1)]], dtype=torch.int32).to(dev)
            q_start = torch.tensor([0, L], dtype=torch.int32, device=dev)
            pl = torch.tensor([prefix_len], dtype=torch.int32, device=dev)
            acts = self._alloc_acts(L)
            xn = self._run_layers(acts, ids, pos, slots, bt, q_start, pl, 1, L, prefix_len + L,
                                  pool, self._lin_ws, self._attn_ws)
            vl = self.tp.vocab
            logits = torch.empty((L, vl), dtype=torch.float32, device=dev)
            if L > LM_GEMV_ROWS and self.lm_tc:
                self._lm_head_call(xn, L, logits, None, self._lm_workspace(L))
            else:
                linear_launch(xn, None, self.lm_head, None, logits, ws=self._lin_ws,
                              norm_w=self.norm_w, eps=self.eps)
            if self.tp_world > 1:           # vocabulary shards -> full rows
                parts = torch.empty((self.tp_world, L, vl), dtype=torch.float32, device=dev)
                torch.distributed.all_gather_into_tensor(parts, logits, group=self.tp_group)
                logits = parts.permute(1, 0, 2).reshape(L, self.vocab_size)
            _check_flags(self.flags)
        return logits.view(1, L, self.vocab_size)

    def new_pool(self, num_blocks: int, block_size: int) -> BlockAllocator:
        return BlockAllocator(num_blocks=num_blocks, block_size=block_size, num_layers=self.n_layers,
                              num_kv_heads=self.n_kv_heads, head_dim=self.head_dim,
                              dtype=torch.float32, device=self.device)

    @torch.inference_mode()
    def prefill(self, prompt_ids: Sequence[int], pool: torch.Tensor, block_table: List[int],
                prefill_chunk: Optional[int] = None, start: int = 0) -> torch.Tensor:
        """Chunked prefill of ``prompt_ids[start:]``; returns the greedy next token [1] (device)."""
        dev = self.device
        bs = pool.shape[4]
        lp = len(prompt_ids)
        chunk = prefill_chunk or (lp - start)
        bt = torch.as_tensor([list(block_table)], dtype=torch.int32).to(dev)
        ids_all = torch.as_tensor(list(prompt_ids), dtype=torch.int64).to(dev)
        pos_all = torch.arange(lp, dtype=torch.int64, device=dev)
        bl = torch.as_tensor(list(block_table), dtype=torch.int64)
        p = torch.arange(lp)
        slots_all = (bl[p // bs] * bs + p % bs).to(dev)
        tok = torch.empty(1, dtype=torch.int64, device=dev)
        acts = self._alloc_acts(min(chunk, lp - start) if lp > start else 1)
        pos = start
        while pos < lp:
            c = min(chunk, lp - pos)
            a = acts if c == acts["hidden"].shape[0] else self._alloc_acts(c)
            q_start = torch.tensor([0, c], dtype=torch.int32, device=dev)
            pl = torch.tensor([pos], dtype=torch.int32, device=dev)
            xn = self._run_layers(a, ids_all[pos:pos + c], pos_all[pos:pos + c],
                                  slots_all[pos:pos + c], bt, q_start, pl, 1, c, pos + c, pool,
                                  self._lin_ws, self._attn_ws)
            pos += c
        self._lm_head_argmax(xn[-1:], tok)
        return tok

    @torch.inference_mode()
    def run_batch(self, pool: torch.Tensor, seqs) -> List[Optional[int]]:
        """One forward pass over several sequences at once (continuous batching).

        ``seqs`` holds ``(tokens, start_pos, block_table, want_token)`` per
        sequence: a decode step (one token at its position) or a prefill chunk
        (the prompt tokens ``[start_pos, start_pos + len)``).  All of them go
        through one varlen pass of the kernels; each writes its K/V into its own
        blocks of ``pool`` and attends over its positions ``[0, start_pos +
        len)``.  Returns, per sequence, the greedy next token after its last
        input token when ``want_token`` is set, else None.  This is the batched
        step the reference's ContinuousEngine only simulates
        (engine/continuous.py:229-261); the token of a sequence is the one
        ``generate`` produces for it."""
        if not seqs:
            return []
        dev = self.device
        bs = pool.shape[4]
        n = len(seqs)
        lens = [len(t) for t, _, _, _ in seqs]
        if min(lens) < 1:
            raise ValueError("every sequence of a batch needs at least one token")
        ids, pos, slots = [], [], []
        for (toks, start, bt, _), c in zip(seqs, lens):
            ids.extend(int(x) for x in toks)
            for p in range(start, start + c):
                if p // bs >= len(bt):
                    raise IndexError(f"position {p} lies past the sequence's block table")
                pos.append(p)
                slots.append(bt[p // bs] * bs + p % bs)
        max_blocks = max(len(bt) for _, _, bt, _ in seqs)
        bt_rows = [list(bt) + [0] * (max_blocks - len(bt)) for _, _, bt, _ in seqs]
        q_start = [0]
        for c in lens:
            q_start.append(q_start[-1] + c)
        T = q_start[-1]
        ids_t = torch.as_tensor(ids, dtype=torch.int64).to(dev)
        pos_t = torch.as_tensor(pos, dtype=torch.int64).to(dev)
        slots_t = torch.as_tensor(slots, dtype=torch.int64).to(dev)
        bt_t = torch.as_tensor(bt_rows, dtype=torch.int32).to(dev)
        qs_t = torch.as_tensor(q_start, dtype=torch.int32).to(dev)
        pl_t = torch.as_tensor([s for _, s, _, _ in seqs], dtype=torch.int32).to(dev)
        max_total = max(s + c for (_, s, _, _), c in zip(seqs, lens))
        acts = self._alloc_acts(T)
        hid = self._run_layers(acts, ids_t, pos_t, slots_t, bt_t, qs_t, pl_t, n, max(lens),
                               max_total, pool, self._lin_ws, self._attn_ws)
        want = [i for i, (_, _, _, w) in enumerate(seqs) if w]
        out: List[Optional[int]] = [None] * n
        if want:
            rows = torch.as_tensor([q_start[i + 1] - 1 for i in want], dtype=torch.int64,
                                   device=dev)
            x = hid.index_select(0, rows)
            tok = torch.empty(len(want), dtype=torch.int64, device=dev)
            self._lm_head_argmax(x, tok)
            for i, t in zip(want, tok.tolist()):
                out[i] = t
        _check_flags(self.flags)
        return out

    @torch.inference_mode()
    def generate(self, prompt_ids: List[int], max_new_tokens: int = 20,
                 eos_token_id: Optional[int] = None, block_size: int = 64,
                 prefill_chunk: Optional[int] = None, use_graph: bool = True) -> List[int]:
        """Greedy generation; returns the new token ids (model.py:154-205)."""
        lp = len(prompt_ids)
        nb = (lp + max_new_tokens + block_size - 1) // block_size
        with torch.cuda.device(self.device):
            # The reference allocates a fresh zeroed pool per call; every slot
            # the forward reads was written earlier in the same call, so a
            # cached pool of the same shape is equivalent and keeps the
            # captured decode graph valid across calls.
            key = (nb, block_size, max_new_tokens)
            cached = self._gen_cache.get(key) if use_graph else None
            if cached is None:
                alloc = self.new_pool(nb, block_size)
                bt = list(range(nb))
                st = DecodeState(self, alloc.pool, [bt], max_new_tokens)
                if use_graph:
                    self._gen_cache[key] = (alloc, bt, st)
            else:
                alloc, bt, st = cached
            first = self.prefill(prompt_ids, alloc.pool, bt, prefill_chunk)
            hist = self._decode_with(st, first, lp, max_new_tokens, use_graph)
            _check_flags(self.flags)
            toks = hist.tolist()
        if eos_token_id is not None and eos_token_id in toks:
            toks = toks[: toks.index(eos_token_id) + 1]
        return toks

    # ------------------------------------------------------------------ #
    # decode loop (single sequence) with CUDA-graph replay
    # ------------------------------------------------------------------ #

    @torch.inference_mode()
    def decode(self, first_tok: torch.Tensor, prompt_len: int, pool: torch.Tensor,
               block_table: List[int], max_new_tokens: int, use_graph: bool = True) -> torch.Tensor:
        """Greedy decode after a prefill: returns all ``max_new_tokens`` tokens
        (the first one included) as a device tensor, host-synchronised."""
        st = DecodeState(self, pool, [list(block_table)], max_new_tokens)
        return self._decode_with(st, first_tok, prompt_len, max_new_tokens, use_graph)

    def _decode_with(self, st: "DecodeState", first_tok: torch.Tensor, prompt_len: int,
                     max_new_tokens: int, use_graph: bool) -> torch.Tensor:
        st.start(first_tok.view(1), [prompt_len])
        steps = max_new_tokens - 1
        if steps > 0:
            if use_graph and steps > 1:
                if st.graph is None:
                    st.step_eager()          # first call: eager step, then capture
                    steps -= 1
                g = st.capture()
                for _ in range(steps):
                    g.replay()
            else:
                for _ in range(steps):
                    st.step_eager()
        torch.cuda.current_stream().synchronize()
        return st.history[0, :max_new_tokens].cpu()


class DecodeState:
    """Static device buffers for batched greedy decode (graph-capturable).

    Per sequence b: ids[b] (last token), positions[b] (its position),
    prefix_lens[b] (= position: tokens already in the pool), slots[b], a row
    of block_tables; ``history[b, step]`` collects generated tokens.
    """

    def __init__(self, model: KshipraModel, pool: torch.Tensor, block_tables: List[List[int]],
                 max_new_tokens: int):
        dev = model.device
        self.m = model
        self.pool = pool
        B = len(block_tables)
        maxb = max(len(r) for r in block_tables)
        bt = torch.zeros((B, maxb), dtype=torch.int32)
        for i, r in enumerate(block_tables):
            bt[i, :len(r)] = torch.tensor(r, dtype=torch.int32)
        self.B = B
        self.block_tables = bt.to(dev)
        self.capacity = maxb * pool.shape[4]
        self.ids = torch.zeros(B, dtype=torch.int64, device=dev)
        self.positions = torch.zeros(B, dtype=torch.int64, device=dev)
        self.prefix_lens = torch.zeros(B, dtype=torch.int32, device=dev)
        self.slots = torch.zeros(B, dtype=torch.int64, device=dev)
        self.q_start = torch.arange(B + 1, dtype=torch.int32, device=dev)
        self.next = torch.zeros(B, dtype=torch.int64, device=dev)
        self.history = torch.zeros((B, max(max_new_tokens, 1)), dtype=torch.int64, device=dev)
        self.step_ctr = torch.zeros(1, dtype=torch.int64, device=dev)
        self.acts = model._alloc_acts(B)
        self.lin_ws = Workspace()
        self.attn_ws = AttentionWorkspace()
        nbytes = int(_lib.lib().ksh_paged_attention_workspace_size(
            B, model.n_heads, model.n_kv_heads, model.head_dim, 1, self.capacity))
        self.attn_ws.get(nbytes, dev)
        self.attn_ws.decode(int(_lib.lib().ksh_decode_attention_workspace_size(
            B, model.n_heads, model.n_kv_heads, model.head_dim)), dev)
        self.lm_ws = torch.empty(model.lm_ws_bytes(B), dtype=torch.uint8, device=dev)
        if B > LM_GEMV_ROWS and model.lm_tc:
            model.lm_head_split()        # before any graph capture of the step
        self.graph: Optional[torch.cuda.CUDAGraph] = None

    def start(self, first_tokens: torch.Tensor, prompt_lens: List[int]) -> None:
        """Seed with each sequence's first generated token (from prefill)."""
        self.next.copy_(first_tokens.view(-1))
        self.positions.copy_(torch.tensor([p - 1 for p in prompt_lens], dtype=torch.int64))
        self.step_ctr.zero_()
        self._advance()

    def _advance(self) -> None:
        call("ksh_decode_advance", ptr(self.next), self.B, ptr(self.ids), ptr(self.positions),
             ptr(self.prefix_lens), ptr(self.slots), ptr(self.block_tables),
             self.block_tables.shape[1], self.pool.shape[4], ptr(self.history),
             self.history.shape[1], ptr(self.step_ctr), ptr(self.m.flags), stream_ptr())

    def _step(self) -> None:
        m = self.m
        xn = m._run_layers(self.acts, self.ids, self.positions, self.slots, self.block_tables,
                           self.q_start, self.prefix_lens, self.B, 1, self.capacity, self.pool,
                           self.lin_ws, self.attn_ws)
        m._lm_head_argmax(xn, self.next, ws=self.lm_ws)
        self._advance()

    def step_eager(self) -> None:
        self._step()

    def capture(self) -> torch.cuda.CUDAGraph:
        if self.graph is None:
            g = torch.cuda.CUDAGraph()
            s = torch.cuda.Stream(device=self.m.device)
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                with torch.cuda.graph(g, stream=s):
                    self._step()
            torch.cuda.current_stream().wait_stream(s)
            self.graph = g
        return self.graph
