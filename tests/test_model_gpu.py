"""End-to-end parity of the B200 forward with the reference (golden fixtures).

* greedy token streams must match the reference bit-exactly;
* logits must match within 1e-3 relative (max-abs error / max-abs logit),
  the bound the path's specification states for fp32 accumulation.
"""

import numpy as np
import pytest
import torch

import cases
from kshipra_b200.config import QWEN25_05B, TINY_LLAMA
from kshipra_b200.model import KshipraModel
from kshipra_b200.weights import build_hf_model, synthetic_state_dict
from oracle.model import OracleModel

pytestmark = pytest.mark.gpu

LOGIT_RTOL = 1e-3


def logit_err(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / np.abs(b).max())


@pytest.fixture(scope="module")
def tiny_sd():
    return synthetic_state_dict(TINY_LLAMA, seed=0)


@pytest.mark.parametrize("scheme", ["int8", "int4", "none"])
def test_tiny_generate_matches_reference(golden, tiny_sd, scheme):
    g = golden("model_tiny.npz")
    q = None if scheme == "none" else scheme
    km = KshipraModel(config=TINY_LLAMA, state_dict=tiny_sd, quantize=q)
    prompt = g["prompt"].tolist()
    toks = km.generate(prompt, max_new_tokens=16, block_size=16, prefill_chunk=16)
    assert toks == g[f"{scheme}/tokens"].tolist()
    # eager decode (no graph) and one-shot prefill give the same stream
    assert km.generate(prompt, 16, block_size=16, use_graph=False) == toks
    assert g[f"{scheme}/tokens_oneshot"].tolist() == toks


@pytest.mark.parametrize("scheme", ["int8", "int4"])
def test_tiny_forward_logits_match_reference(golden, tiny_sd, scheme):
    """The reference-facing forward(): chunked prefill then decode, logits per step."""
    g = golden("model_tiny.npz")
    km = KshipraModel(config=TINY_LLAMA, state_dict=tiny_sd, quantize=scheme)
    prompt = g["prompt"].tolist()
    ref_logits = g[f"{scheme}/logits"]
    ref_toks = g[f"{scheme}/tokens"].tolist()
    B = 16
    alloc = km.new_pool((len(prompt) + 16 + B - 1) // B, B)
    bt = list(range(alloc.pool.shape[0]))
    pos = 0
    while pos < len(prompt):
        c = min(16, len(prompt) - pos)
        ids = torch.tensor([prompt[pos:pos + c]])
        positions = torch.arange(pos, pos + c).unsqueeze(0)
        slots = [bt[p // B] * B + p % B for p in range(pos, pos + c)]
        logits = km.forward(ids, positions, alloc.pool, bt, slots, prefix_len=pos)
        pos += c
    assert logit_err(logits[0, -1].cpu(), ref_logits[0]) < LOGIT_RTOL
    toks = [int(logits[0, -1].argmax())]
    for step in range(1, 16):
        p = len(prompt) + step - 1
        logits = km.forward(torch.tensor([[toks[-1]]]), torch.tensor([[p]]), alloc.pool, bt,
                            [bt[p // B] * B + p % B], prefix_len=p)
        assert logit_err(logits[0, -1].cpu(), ref_logits[step]) < LOGIT_RTOL
        toks.append(int(logits[0, -1].argmax()))
    assert toks == ref_toks


def test_drop_in_from_hf_model(golden, tiny_sd):
    """KshipraModel(hf_model, device, quantize) as the reference constructs it."""
    g = golden("model_tiny.npz")
    hf = build_hf_model(TINY_LLAMA, tiny_sd)
    km = KshipraModel(hf, torch.device("cuda"), "int8")
    km.rope_theta = TINY_LLAMA.rope_theta
    toks = km.generate(g["prompt"].tolist(), max_new_tokens=16, block_size=16)
    assert toks == g["int8/tokens"].tolist()
    assert km.layers[0].q_proj.weight.payload.shape == (256, 256)
    y = km.layers[0].k_proj(torch.randn(3, 256, device="cuda"))
    assert tuple(y.shape) == (3, 128)


def test_forward_matches_oracle_with_prefix(tiny_sd):
    """forward() over a shuffled block table with a prefix, vs the oracle."""
    gen = torch.Generator().manual_seed(0)
    km = KshipraModel(config=TINY_LLAMA, state_dict=tiny_sd, quantize="int4")
    orc = OracleModel(TINY_LLAMA, tiny_sd, "int4")
    B = 8
    nb = 12
    bt = torch.randperm(nb, generator=gen).tolist()
    ids = torch.randint(0, TINY_LLAMA.vocab, (1, 60), generator=gen)
    alloc = km.new_pool(nb, B)
    opool = orc.new_pool(nb, B)
    for (a, b) in ((0, 23), (23, 41), (41, 42), (42, 60)):
        positions = torch.arange(a, b).unsqueeze(0)
        slots = [bt[p // B] * B + p % B for p in range(a, b)]
        got = km.forward(ids[:, a:b], positions, alloc.pool, bt, slots, prefix_len=a).cpu()
        ref = orc.forward(ids[:, a:b], positions, opool, bt, slots, prefix_len=a)
        assert logit_err(got, ref) < LOGIT_RTOL
        assert logit_err(got, ref) < 1e-5
    np.testing.assert_allclose(alloc.pool.cpu().numpy(), opool.numpy(), rtol=1e-5, atol=1e-5)


@pytest.fixture(scope="module")
def qwen_sd():
    return synthetic_state_dict(QWEN25_05B, seed=0)


@pytest.mark.parametrize("scheme", ["int8", "int4"])
def test_qwen05b_tokens_match_reference(golden, qwen_sd, scheme):
    """Config: Qwen2.5-0.5B shape, 512-token prompt in 128-token chunks, 50 greedy tokens."""
    g = golden("model_qwen05b.npz")
    km = KshipraModel(config=QWEN25_05B, state_dict=qwen_sd, quantize=scheme)
    prompt = g["prompt"].tolist()
    toks = km.generate(prompt, max_new_tokens=50, block_size=16, prefill_chunk=128)
    ref = g[f"{scheme}/tokens"].tolist()
    if toks != ref:
        i = next(i for i, (a, b) in enumerate(zip(toks, ref)) if a != b)
        pytest.fail(f"first mismatch at {i}: margin there {g[f'{scheme}/margins'][i]}")
    # logits after the prefill
    B = 16
    alloc = km.new_pool(33, B)
    bt = list(range(33))
    pos = 0
    while pos < 512:
        positions = torch.arange(pos, pos + 128).unsqueeze(0)
        logits = km.forward(torch.tensor([prompt[pos:pos + 128]]), positions, alloc.pool, bt,
                            list(range(pos, pos + 128)), prefix_len=pos)
        pos += 128
    err = logit_err(logits[0, -1].cpu(), g[f"{scheme}/logits0"])
    assert err < LOGIT_RTOL, err


def _engine_run(km, prompts, new_tokens, block_size=16, budget_tokens=48, num_blocks=256):
    """Drive the continuous-batching scheduler with the real batched forward."""
    from kshipra_b200.continuous import ContinuousEngine
    from kshipra_b200.prefix_cache import PrefixCache
    cfg = km.cfg
    cache = PrefixCache(num_blocks, block_size, cfg.layers, cfg.kv_heads, cfg.head_dim,
                        dtype=torch.float32, device=torch.device("cuda"))
    eng = ContinuousEngine(cache, block_size=block_size, max_batch_tokens=budget_tokens,
                           itl_budget_s=budget_tokens * 1e-3, t_tok_s=1e-3, model=km)
    reqs = [eng.add_request(list(p), new_tokens) for p in prompts]
    for _ in range(10000):
        if all(r in eng.finished for r in reqs):
            break
        eng.step()
    return reqs


@pytest.mark.parametrize("scheme", ["int8", "int4"])
def test_continuous_engine_batched_forward_matches_generate(tiny_sd, scheme):
    """Requests of different lengths prefill in chunks and decode together in
    the same batched passes; each one's greedy tokens equal those of running
    it alone through generate()."""
    km = KshipraModel(config=TINY_LLAMA, state_dict=tiny_sd, quantize=scheme)
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, TINY_LLAMA.vocab, (n,), generator=g).tolist()
               for n in (20, 33, 7, 50, 16)]
    reqs = _engine_run(km, prompts, new_tokens=6)
    for p, r in zip(prompts, reqs):
        assert len(r.generated_tokens) == 6
        solo = km.generate(p, max_new_tokens=6, block_size=16)
        assert r.generated_tokens == solo, (len(p), r.generated_tokens, solo)


def test_continuous_engine_reuses_radix_prefix(tiny_sd):
    """With a model the engine starts a prefill after the prompt blocks the
    radix tree holds: request B shares 48 tokens (three blocks) with the
    already finished request A, computes only its own tail, and still yields
    the tokens of generate() run alone."""
    from kshipra_b200.continuous import ContinuousEngine
    from kshipra_b200.prefix_cache import PrefixCache
    km = KshipraModel(config=TINY_LLAMA, state_dict=tiny_sd, quantize="int8")
    cfg = km.cfg
    g = torch.Generator().manual_seed(9)
    shared = torch.randint(0, cfg.vocab, (48,), generator=g).tolist()
    pa = shared + torch.randint(0, cfg.vocab, (21,), generator=g).tolist()
    pb = shared + torch.randint(0, cfg.vocab, (10,), generator=g).tolist()
    cache = PrefixCache(64, 16, cfg.layers, cfg.kv_heads, cfg.head_dim, dtype=torch.float32,
                        device=torch.device("cuda"))
    eng = ContinuousEngine(cache, block_size=16, max_batch_tokens=32, itl_budget_s=0.032,
                           t_tok_s=1e-3, model=km)
    computed = []
    orig = km.run_batch

    def counting(pool, seqs):
        computed.append(sum(len(t) for t, _, _, _ in seqs))
        return orig(pool, seqs)
    km.run_batch = counting
    ra = eng.add_request(pa, 5)
    while ra not in eng.finished:
        eng.step()
    done_a = sum(computed)
    rb = eng.add_request(pb, 5)
    while rb not in eng.finished:
        eng.step()
    km.run_batch = orig
    # A: its whole prompt + 4 decode tokens; B: only its 10-token tail + 4 decode tokens
    assert done_a == len(pa) + 4
    assert sum(computed) - done_a == 10 + 4
    assert ra.generated_tokens == km.generate(pa, max_new_tokens=5, block_size=16)
    assert rb.generated_tokens == km.generate(pb, max_new_tokens=5, block_size=16)
    # the published blocks stay in the tree; the requests' own blocks went back
    blocks, matched, _ = cache.tree.match(pa)
    assert matched == 64 and len(blocks) == 4


def test_run_batch_mixed_prefill_and_decode_vs_oracle(tiny_sd):
    """One pass holding a prefill chunk and decode steps of other sequences
    gives each sequence the oracle's next token."""
    km = KshipraModel(config=TINY_LLAMA, state_dict=tiny_sd, quantize="int8")
    om = OracleModel(TINY_LLAMA, tiny_sd, quantize="int8")
    alloc = km.new_pool(64, 16)
    pool = alloc.pool
    g = torch.Generator().manual_seed(11)
    pa = torch.randint(0, TINY_LLAMA.vocab, (21,), generator=g).tolist()
    pb = torch.randint(0, TINY_LLAMA.vocab, (9,), generator=g).tolist()
    bta = [alloc.alloc() for _ in range(3)]
    btb = [alloc.alloc() for _ in range(3)]
    # a: whole prompt first; b: first 5 prompt tokens, then the rest with a's decode
    ta = km.run_batch(pool, [(pa, 0, bta, True), (pb[:5], 0, btb, False)])
    assert ta[1] is None
    out = km.run_batch(pool, [([ta[0]], len(pa), bta, True), (pb[5:], 5, btb, True)])
    ref_a = om.generate(pa, 2)
    ref_b = om.generate(pb, 1)
    assert [ta[0], out[0]] == ref_a
    assert out[1] == ref_b[0]


def test_preempted_request_resumes_with_generate_tokens(tiny_sd):
    """A decoding request is swapped out (asynchronous device-to-host copy on
    a side stream), its freed blocks are overwritten by later work on the
    main stream, and after re-admission (host-to-device copy into its new
    blocks) it finishes with the tokens generate() gives it alone."""
    from kshipra_b200.continuous import ContinuousEngine, SeqState
    from kshipra_b200.prefix_cache import PrefixCache
    km = KshipraModel(config=TINY_LLAMA, state_dict=tiny_sd, quantize="int8")
    cfg = km.cfg
    g = torch.Generator().manual_seed(13)
    pa = torch.randint(0, cfg.vocab, (37,), generator=g).tolist()
    pb = torch.randint(0, cfg.vocab, (21,), generator=g).tolist()
    cache = PrefixCache(32, 16, cfg.layers, cfg.kv_heads, cfg.head_dim, dtype=torch.float32,
                        device=torch.device("cuda"))
    eng = ContinuousEngine(cache, block_size=16, max_batch_tokens=64, itl_budget_s=0.064,
                           t_tok_s=1e-3, model=km)
    ra, rb = eng.add_request(pa, 9), eng.add_request(pb, 9)
    while len(ra.generated_tokens) < 4:
        eng.step()
    assert ra.state == SeqState.RUNNING
    freed = list(ra._own_blocks)
    eng._preempt(ra)
    assert ra.state == SeqState.WAITING and ra.swapped_kv is not None and freed
    # later work on the main stream overwrites the freed blocks
    cache.allocator.pool[torch.tensor(freed, device="cuda")] = float("nan")
    for _ in range(1000):
        if ra in eng.finished and rb in eng.finished:
            break
        eng.step()
    assert ra.generated_tokens == km.generate(pa, max_new_tokens=9, block_size=16)
    assert rb.generated_tokens == km.generate(pb, max_new_tokens=9, block_size=16)
