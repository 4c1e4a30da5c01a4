"""Host-side control plane: block allocator, radix tree, prefix cache, scheduler.

Behavioural tests follow the reference's tests/test_prefix_cache.py and
tests/test_continuous.py; the trace tests replay a deterministic operation
sequence and compare every decision with the reference's own
(``tests/golden/cache_trace.json``).
"""

import json
import os
import time

import pytest
import torch

import make_golden
from kshipra_b200 import continuous as kc
from kshipra_b200 import prefix_cache as kp
from kshipra_b200.continuous import ContinuousEngine, SeqState
from kshipra_b200.prefix_cache import (BlockAllocator, OutOfBlocksError, PrefixCache, RadixTree,
                                       TokenArena)

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def test_block_allocator_lifo():
    alloc = BlockAllocator(num_blocks=4, block_size=16, num_layers=2, num_kv_heads=2, head_dim=8)
    b1, b2 = alloc.alloc(), alloc.alloc()
    assert (b1, b2) == (3, 2)
    alloc.free(b1)
    assert alloc.alloc() == 3
    assert tuple(alloc.pool.shape) == (4, 2, 2, 2, 16, 8)
    alloc.alloc(), alloc.alloc()
    with pytest.raises(OutOfBlocksError):
        alloc.alloc()


def test_token_arena():
    arena = TokenArena(capacity=10)
    assert arena.alloc([1, 2, 3]) == (0, 3)
    assert arena.storage[0:3].tolist() == [1, 2, 3]
    with pytest.raises(RuntimeError):
        arena.alloc(list(range(8)))


def _tree(nb=100, bs=4):
    arena = TokenArena(1000)
    alloc = BlockAllocator(num_blocks=nb, block_size=bs, num_layers=1, num_kv_heads=1, head_dim=1)
    return RadixTree(alloc, arena, block_size=bs), alloc


def test_radix_match_exact_and_split():
    tree, alloc = _tree()
    toks = [1, 2, 3, 4, 5, 6, 7, 8]
    blocks = [alloc.alloc(), alloc.alloc()]
    node = tree.insert(toks, blocks, 0, tree.root)
    tree.pin(node)
    assert tree.match(toks) == (blocks, 8, node)
    mb, ml, last = tree.match([1, 2, 3, 4, 9, 10, 11, 12])
    assert (mb, ml) == ([blocks[0]], 4)
    assert last.token_len == 4 and last.block_ids == [blocks[0]]
    tail = list(last.children.values())[0]
    assert tail.token_len == 4 and tail.block_ids == [blocks[1]]
    assert tail.ref_count == last.ref_count == 1
    # partial match shorter than a block is not taken
    assert tree.match([1, 2, 9])[1] == 0


def test_eviction_lru_refcount_and_cascade():
    tree, alloc = _tree(nb=10)
    n1 = tree.insert([1, 2, 3, 4], [alloc.alloc()], 0, tree.root)
    tree.pin(n1)
    b2 = [alloc.alloc()]
    n2 = tree.insert([5, 6, 7, 8], b2, 0, tree.root)
    tree.pin(n2)
    tree.unpin(n2)
    assert len(alloc.free_blocks) == 8
    tree.evict(1)
    assert len(alloc.free_blocks) == 9 and alloc.free_blocks[-1] == b2[0]
    assert n1.ref_count == 1
    tree2, alloc2 = _tree(nb=10)
    m1 = tree2.insert([1, 2, 3, 4], [alloc2.alloc()], 0, tree2.root)
    tree2.insert([1, 2, 3, 4, 5, 6, 7, 8], [alloc2.alloc()], 4, m1)
    assert tree2.evict(2) == 2
    assert len(alloc2.free_blocks) == 10 and not tree2.root.children


def test_prefix_cache_allocate_with_eviction():
    cache = PrefixCache(num_blocks=4, block_size=4, num_layers=1, num_kv_heads=1, head_dim=1)
    nodes = []
    for t in ([1, 2, 3, 4], [5, 6, 7, 8], [9, 10, 11, 12]):
        b = cache.allocate_blocks(1)
        n = cache.tree.insert(t, b, 0, cache.tree.root)
        cache.tree.pin(n)
        nodes.append(n)
    cache.tree.unpin(nodes[1])
    cache.tree.unpin(nodes[2])
    assert len(cache.allocate_blocks(2)) == 2
    assert nodes[0].ref_count == 1


def _engine(pool_blocks=100):
    cache = PrefixCache(num_blocks=pool_blocks, block_size=64, num_layers=2, num_kv_heads=2,
                        head_dim=8)
    return ContinuousEngine(prefix_cache=cache, block_size=64, max_batch_tokens=1024,
                            itl_budget_s=0.1, t_tok_s=0.01)


def test_admission_strict_reservation():
    e = _engine(10)
    r = e.add_request([0] * 600, 40)
    assert e._admission_check(r)
    e.schedule()
    assert r.state == SeqState.PREFILLING and len(r.block_table) == 10
    assert not e._admission_check(e.add_request([0] * 64, 10))


def test_scheduler_interleaves_prefill_and_decode():
    e = _engine()
    rd = e.add_request([0] * 128, 10)
    e.schedule()
    rd.prefill_pos, rd.state, rd.generated_tokens = 128, SeqState.RUNNING, [0]
    rp = e.add_request([1] * 512, 10)
    s = e.schedule()
    assert s.decodes == [rd] and s.prefills == [(rp, 9)] and s.total_tokens == 10


def test_preemption_swap():
    e = _engine(12)
    r = e.add_request([0] * 640, 10)
    e.schedule()
    assert len(r.block_table) == 11 and len(e.cache.allocator.free_blocks) == 1
    r.prefill_pos, r.state = 640, SeqState.RUNNING
    pool = e.cache.allocator.pool
    pool[r.block_table] = torch.arange(11, dtype=pool.dtype).view(
        11, 1, 1, 1, 1, 1).expand(11, *pool.shape[1:])
    r.generated_tokens = [0, 0, 0]
    e._preempt(r)
    assert r.state == SeqState.WAITING and r.block_table == []
    assert r.swapped_kv is not None and r.swapped_kv.shape[0] == 11
    assert len(e.cache.allocator.free_blocks) == 12
    assert e.waiting_queue[0] is r
    # re-admission restores the K/V into the new blocks and resumes decoding
    s = e.schedule()
    assert r.state == SeqState.RUNNING and s.decodes == [r] and s.prefills == []
    assert r.swapped_kv is None and len(r.block_table) == 11
    got = e.cache.allocator.pool[r.block_table][:, 0, 0, 0, 0, 0]
    assert got.tolist() == [float(i) for i in range(11)]
    while r.state != SeqState.FINISHED:
        e.step()
    assert len(r.generated_tokens) == 10 and r in e.finished
    assert len(e.cache.allocator.free_blocks) == 12


def test_preemption_mid_prefill_resumes_at_its_position():
    e = _engine(12)
    r = e.add_request([0] * 100, 10)
    s = e.schedule()
    assert s.prefills and s.prefills[0][0] is r
    r.prefill_pos = 48
    e._preempt(r)
    s = e.schedule()
    assert r.state == SeqState.PREFILLING and r.prefill_pos == 48
    assert s.prefills == [(r, min(52, s.prefills[0][1]))]


def test_itl_budget_bound():
    e = _engine()
    for _ in range(5):
        r = e.add_request([0] * 64, 10)
        e.schedule()
        r.prefill_pos, r.state, r.generated_tokens = 64, SeqState.RUNNING, [0]
    e.add_request([1] * 256, 10)
    s = e.schedule()
    assert len(s.prefills) == 1 and s.prefills[0][1] == 5 and s.total_tokens == 10


def test_mock_step_runs_to_completion(monkeypatch):
    monkeypatch.setattr(kc.time, "sleep", lambda s: None)
    e = _engine()
    for i in range(50):
        e.add_request([i % 100] * 64, 5)
    for _ in range(5000):
        e.step()
        if not e.active_sequences and not e.waiting_queue:
            break
    assert e._total_finished == 50
    assert len(e.cache.allocator.free_blocks) == 100


def _with_clock(fn):
    clock = make_golden._Clock()
    orig = time.monotonic
    time.monotonic = clock
    try:
        return fn(clock)
    finally:
        time.monotonic = orig


def _jsonable(x):
    return json.loads(json.dumps(x))


def test_cache_trace_matches_reference():
    ref = json.load(open(os.path.join(GOLDEN, "cache_trace.json")))
    got = _with_clock(lambda c: make_golden.cache_scenario((kp.PrefixCache, kp.OutOfBlocksError), c))
    assert _jsonable(got) == ref["cache"]


def test_scheduler_trace_matches_reference():
    ref = json.load(open(os.path.join(GOLDEN, "cache_trace.json")))
    got = _with_clock(lambda c: make_golden.scheduler_scenario((kp.PrefixCache, kc.ContinuousEngine), c))
    assert _jsonable(got) == ref["scheduler"]
