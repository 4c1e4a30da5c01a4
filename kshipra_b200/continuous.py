"""Continuous-batching iteration scheduler (host side).

Interface and scheduling policy follow the reference's engine/continuous.py:

* request state machine WAITING -> PREFILLING -> RUNNING -> FINISHED
  (continuous.py:32-64);
* admission only if ``new_need + active_reserved <= free - h_evict``
  (:121-142), blocks reserved for prompt + max_new_tokens up front;
* per iteration, every RUNNING request decodes one token and the prefill
  token budget ``int(itl_budget / t_tok) - n_decodes`` is handed out in
  chunks to PREFILLING requests in admission order (:148-183);
* swap-out preemption of a victim's blocks to pinned host memory
  (:206-223), asynchronous on a side stream, and swap-in that resumes the
  request where it stopped.

Without a model the step sleeps ``total_tokens * t_tok_s`` like the
reference's simulated forward (:229-261), so the scheduling decisions are
the reference's.  With ``model=KshipraModel`` the step runs the real batched
forward: all scheduled prefill chunks and decode tokens of the iteration go
through one varlen pass of the kernels; the chunk that completes a prompt
yields its first token (as ``generate`` does), each decode step the next one.

With a model the radix tree also saves work (the reference matches prefixes
but recomputes them): a request's prefill starts after the whole blocks of
its prompt that the tree already holds (the last prompt token is always
computed, it yields the first output token), and once its prompt is
prefilled the prompt's whole blocks are published into the tree, so later
requests with the same prefix reuse them.  Published blocks belong to the
tree (freed by eviction once no request pins them), not to the request.
"""

from __future__ import annotations

import math
import time
from dataclasses import dataclass, field
from enum import Enum
from typing import Dict, List, Optional, Tuple

import torch

from .prefix_cache import OutOfBlocksError, PrefixCache  # noqa: F401  (re-export)


class SeqState(Enum):
    WAITING = "waiting"
    PREFILLING = "prefilling"
    RUNNING = "running"
    FINISHED = "finished"


@dataclass
class Request:
    req_id: int
    prompt_tokens: List[int]
    max_new_tokens: int
    arrival_time: float = field(default_factory=time.monotonic)
    state: SeqState = SeqState.WAITING
    prefill_pos: int = 0
    generated_tokens: List[int] = field(default_factory=list)
    block_table: List[int] = field(default_factory=list)
    swapped_kv: Optional[torch.Tensor] = None
    first_token_time: Optional[float] = None
    finish_time: Optional[float] = None
    itl_times: List[float] = field(default_factory=list)

    @property
    def seq_len(self) -> int:
        return len(self.prompt_tokens) + len(self.generated_tokens)


@dataclass
class SchedulerOutput:
    decodes: List[Request]
    prefills: List[Tuple[Request, int]]
    total_tokens: int


def _runs(blocks: List[int], start: int = 0):
    """(index, first block, count) for each run of consecutive block ids, so a
    swap copies whole contiguous ranges of the pool at once."""
    out = []
    i = 0
    while i < len(blocks):
        j = i + 1
        while j < len(blocks) and blocks[j] == blocks[j - 1] + 1:
            j += 1
        out.append((start + i, blocks[i], j - i))
        i = j
    return out


class ContinuousEngine:
    def __init__(self, prefix_cache: PrefixCache, block_size: int, max_batch_tokens: int,
                 itl_budget_s: float, t_tok_s: float, model=None) -> None:
        self.cache = prefix_cache
        self.block_size = block_size
        self.max_batch_tokens = max_batch_tokens
        self.itl_budget_s = itl_budget_s
        self.t_tok_s = t_tok_s
        self.model = model
        self.waiting_queue: List[Request] = []
        self.active_sequences: Dict[int, Request] = {}
        self._next_req_id = 0
        self._total_finished = 0
        self.finished: List[Request] = []

    # ---------------- admission ----------------

    def add_request(self, prompt_tokens: List[int], max_new_tokens: int) -> Request:
        req = Request(req_id=self._next_req_id, prompt_tokens=list(prompt_tokens),
                      max_new_tokens=max_new_tokens)
        self._next_req_id += 1
        self.waiting_queue.append(req)
        return req

    def _required_blocks(self, req: Request) -> int:
        return math.ceil((len(req.prompt_tokens) + req.max_new_tokens) / self.block_size)

    def _active_reserved(self) -> int:
        return sum(max(0, self._required_blocks(r) - len(r.block_table))
                   for r in self.active_sequences.values())

    def _admission_check(self, req: Request) -> bool:
        need = self._required_blocks(req)
        toks = req.prompt_tokens if self.model is None else req.prompt_tokens[:-1]
        matched, _, node = self.cache.tree.match(toks)
        h_evict = 0
        cur = node
        while cur is not None and cur.parent is not None:
            if cur.ref_count == 0:
                h_evict += len(cur.block_ids)
            cur = cur.parent
        free = len(self.cache.allocator.free_blocks)
        return need - len(matched) + self._active_reserved() <= free - h_evict

    # ---------------- scheduling ----------------

    def schedule(self) -> SchedulerOutput:
        for req in list(self.waiting_queue):
            if self._admission_check(req):
                self.waiting_queue.remove(req)
                self._init_sequence(req)
                self.active_sequences[req.req_id] = req
        decodes = [r for r in self.active_sequences.values() if r.state == SeqState.RUNNING]
        budget = int(self.itl_budget_s / self.t_tok_s + 1e-9)
        c_max = max(0, budget - len(decodes))
        prefills: List[Tuple[Request, int]] = []
        left = c_max
        for req in self.active_sequences.values():
            if left <= 0:
                break
            if req.state != SeqState.PREFILLING or req.prefill_pos >= len(req.prompt_tokens):
                continue
            c = min(len(req.prompt_tokens) - req.prefill_pos, left, self.max_batch_tokens)
            if c > 0:
                prefills.append((req, c))
                left -= c
        return SchedulerOutput(decodes, prefills, len(decodes) + (c_max - left))

    def _init_sequence(self, req: Request) -> None:
        # With a model the last prompt token is never taken from the tree: its
        # position starts the prefill, in a block of the request's own.
        toks = req.prompt_tokens if self.model is None else req.prompt_tokens[:-1]
        matched, matched_len, node = self.cache.tree.match(toks)
        self.cache.tree.pin(node)
        req._pinned = node  # type: ignore[attr-defined]
        new = self.cache.allocate_blocks(max(0, self._required_blocks(req) - len(matched)))
        req._own_blocks = list(new)  # type: ignore[attr-defined]
        req.block_table = matched + new
        req.state = SeqState.PREFILLING
        if req.swapped_kv is not None:
            self._swap_in(req, len(matched))
        elif self.model is not None:
            req.prefill_pos = matched_len             # the tree's blocks hold these positions

    def _publish_prompt(self, req: Request) -> None:
        """Insert the whole blocks of a prefilled prompt into the radix tree.

        The tree is matched again first: blocks another request published
        meanwhile stay the tree's, this request's copies of them stay its own
        (freed when it finishes), and only the remainder is inserted.  The
        request's pin moves to the deepest node of its prompt."""
        bsz = self.block_size
        full = len(req.prompt_tokens) // bsz
        if full == 0:
            return
        toks = req.prompt_tokens[:full * bsz]
        _, have, node = self.cache.tree.match(toks)
        if have < full * bsz:
            given = req.block_table[have // bsz:full]
            node = self.cache.tree.insert(toks, given, have, node)
            gone = set(given)
            req._own_blocks = [b for b in req._own_blocks if b not in gone]  # type: ignore[attr-defined]
        self.cache.tree.pin(node)
        self._unpin(req)
        req._pinned = node  # type: ignore[attr-defined]

    # ---------------- preemption ----------------

    def _preempt(self, victim: Request) -> None:
        """Swap the victim's K/V blocks out to pinned host memory and requeue
        it at the head of the waiting queue (continuous.py:206-223).

        On a CUDA pool the device-to-host copies run on a side stream, after
        the work already queued on the current stream (so they see the
        victim's latest K/V); the current stream then waits on the copies'
        event, a device-side wait, so no later kernel can overwrite the freed
        blocks before they are saved and the host never blocks.  The event is
        kept on the request (``swap_event``) for a caller that wants to read
        ``swapped_kv`` on the host.  The request resumes where it stopped:
        a decoding request comes back RUNNING, a partly prefilled one
        PREFILLING at the same prompt position (the reference comes back
        PREFILLING at the prompt's end, where its scheduler never picks the
        request up again)."""
        victim._resume_running = victim.state == SeqState.RUNNING  # type: ignore[attr-defined]
        victim._resume_pos = victim.prefill_pos  # type: ignore[attr-defined]
        victim.state = SeqState.WAITING
        if victim.block_table:
            pool = self.cache.allocator.pool
            n = len(victim.block_table)
            host = torch.empty((n, *pool.shape[1:]), dtype=pool.dtype, pin_memory=pool.is_cuda)
            if pool.is_cuda:
                cur = torch.cuda.current_stream(pool.device)
                side = self._side_stream(pool.device)
                side.wait_stream(cur)
                with torch.cuda.stream(side):
                    for i0, b0, cnt in _runs(victim.block_table):
                        host[i0:i0 + cnt].copy_(pool[b0:b0 + cnt], non_blocking=True)
                    ev = torch.cuda.Event()
                    ev.record(side)
                cur.wait_event(ev)
                victim.swap_event = ev  # type: ignore[attr-defined]
            else:
                for i0, b0, cnt in _runs(victim.block_table):
                    host[i0:i0 + cnt].copy_(pool[b0:b0 + cnt])
            # blocks the request took from (or gave to) the radix tree stay the tree's
            for b in getattr(victim, "_own_blocks", victim.block_table):
                self.cache.allocator.free(b)
            victim._own_blocks = []  # type: ignore[attr-defined]
            victim.swapped_kv = host
            victim.block_table = []
        self._unpin(victim)
        self.waiting_queue.insert(0, victim)
        self.active_sequences.pop(victim.req_id, None)

    def _side_stream(self, device) -> "torch.cuda.Stream":
        s = getattr(self, "_swap_stream", None)
        if s is None:
            s = torch.cuda.Stream(device=device)
            self._swap_stream = s
        return s

    def _swap_in(self, req: Request, n_matched: int) -> None:
        """Copy the swapped K/V back into the request's own blocks.  The first
        ``n_matched`` entries of its new block table come from the radix tree
        (the same tokens' K/V, possibly pinned and read by other requests), so
        they are left as they are."""
        pool = self.cache.allocator.pool
        n = min(len(req.block_table), req.swapped_kv.shape[0])
        if pool.is_cuda:
            ev = getattr(req, "swap_event", None)
            if ev is not None:
                torch.cuda.current_stream(pool.device).wait_event(ev)
        for i0, b0, cnt in _runs(req.block_table[n_matched:n], start=n_matched):
            pool[b0:b0 + cnt].copy_(req.swapped_kv[i0:i0 + cnt], non_blocking=pool.is_cuda)
        req.swapped_kv = None
        req.swap_event = None  # type: ignore[attr-defined]
        if getattr(req, "_resume_running", True):
            req.prefill_pos = len(req.prompt_tokens)
            req.state = SeqState.RUNNING
        else:
            req.prefill_pos = getattr(req, "_resume_pos", 0)

    # ---------------- step ----------------

    def step(self) -> bool:
        sched = self.schedule()
        if not sched.decodes and not sched.prefills:
            return False
        if self.model is None:
            time.sleep(sched.total_tokens * self.t_tok_s)
            first: Dict[int, int] = {}
            nxt = {r.req_id: 0 for r in sched.decodes}
        else:
            first, nxt = self._run_model(sched)
        finished_any = False
        now = time.monotonic()
        for req, c in sched.prefills:
            req.prefill_pos += c
            if req.prefill_pos >= len(req.prompt_tokens):
                req.state = SeqState.RUNNING
                if self.model is not None:
                    self._publish_prompt(req)
                if req.req_id in first:
                    self._emit(req, first[req.req_id], now)
                    if len(req.generated_tokens) >= req.max_new_tokens:
                        self._finish(req)
                        finished_any = True
        for req in sched.decodes:
            self._emit(req, nxt[req.req_id], now)
            if len(req.generated_tokens) >= req.max_new_tokens:
                self._finish(req)
                finished_any = True
        return finished_any

    def _emit(self, req: Request, tok: int, now: float) -> None:
        req.generated_tokens.append(int(tok))
        if req.first_token_time is None:
            req.first_token_time = now
        if req.itl_times:
            req.itl_times.append(now - req.itl_times[-1])
        else:
            req.itl_times.append(now - req.arrival_time)

    def _run_model(self, sched: SchedulerOutput):
        seqs = []
        for req in sched.decodes:
            pos = len(req.prompt_tokens) + len(req.generated_tokens) - 1
            seqs.append(([req.generated_tokens[-1]], pos, req.block_table, True))
        for req, c in sched.prefills:
            done = req.prefill_pos + c >= len(req.prompt_tokens)
            seqs.append((req.prompt_tokens[req.prefill_pos:req.prefill_pos + c], req.prefill_pos,
                         req.block_table, done))
        toks = self.model.run_batch(self.cache.allocator.pool, seqs)
        nxt = {r.req_id: toks[i] for i, r in enumerate(sched.decodes)}
        first = {}
        for j, (req, _) in enumerate(sched.prefills):
            t = toks[len(sched.decodes) + j]
            if t is not None:
                first[req.req_id] = t
        return first, nxt

    def _unpin(self, req: Request) -> None:
        node = getattr(req, "_pinned", None)
        if node is not None:
            self.cache.tree.unpin(node)
            req._pinned = None  # type: ignore[attr-defined]

    def _finish(self, req: Request) -> None:
        req.state = SeqState.FINISHED
        req.finish_time = time.monotonic()
        # Free only the blocks this request allocated; blocks it matched in the
        # radix tree stay owned by the tree (the request only unpins them).
        own = getattr(req, "_own_blocks", req.block_table)
        for b in own:
            self.cache.allocator.free(b)
        self._unpin(req)
        req.block_table = []
        self.active_sequences.pop(req.req_id, None)
        self._total_finished += 1
        self.finished.append(req)
