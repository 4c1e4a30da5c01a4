"""Parity with the reference beyond the batch-1 small shapes (golden fixtures
made by running the reference itself, tests/golden/make_golden.py):

* the Llama-3-8B architecture cut to two layers (head_dim 128, 32 / 8
  heads, untied fp32 lm_head, vocabulary 128256), INT8 and INT4 G=128:
  ``generate`` (chunked prefill + CUDA-graph decode) and the reference-facing
  ``forward`` logits, and a batch of 20 short requests served together by
  ``ContinuousEngine`` with the real batched forward, so the decode steps run
  the 17..64-row linears and the batch lm_head at the 8B shapes;
* shortened config-3 requests on the Qwen2.5-0.5B shape (INT4): two waves of
  20 requests served by the engine, the second wave finding the first wave's
  system-prefix blocks in the radix tree.

Greedy tokens must be identical to the reference's; logits within 1e-3 of the
largest |logit| (the bound the path's specification states).  A token that
differs is reported with the reference's top-2 margin at that step.
"""

import numpy as np
import pytest
import torch

import cases
from kshipra_b200.config import QWEN25_05B
from kshipra_b200.model import KshipraModel
from kshipra_b200.weights import synthetic_state_dict, weights_checksum

pytestmark = pytest.mark.gpu

LOGIT_RTOL = 1e-3


def logit_err(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / np.abs(b).max())


def _same_tokens(got, ref, margins, what):
    if list(got) != list(ref):
        i = next((i for i, (a, b) in enumerate(zip(got, ref)) if a != b), min(len(got), len(ref)))
        m = float(margins[i]) if i < len(margins) else float("nan")
        pytest.fail(f"{what}: first token mismatch at step {i} (reference top-2 margin {m:.3g}): "
                    f"{list(got)} vs {list(ref)}")


def _engine(km, num_blocks, budget):
    from kshipra_b200.continuous import ContinuousEngine
    from kshipra_b200.prefix_cache import PrefixCache
    cfg = km.cfg
    cache = PrefixCache(num_blocks, 16, cfg.layers, cfg.kv_heads, cfg.head_dim,
                        dtype=torch.float32, device=km.device)
    return ContinuousEngine(cache, block_size=16, max_batch_tokens=budget,
                            itl_budget_s=budget * 1e-3, t_tok_s=1e-3, model=km)


def _drain(eng, reqs):
    for _ in range(100000):
        if all(r in eng.finished for r in reqs):
            return
        eng.step()
    raise AssertionError("engine did not finish its requests")


class _RowLog:
    """Wraps run_batch to record how many token rows each pass computed."""

    def __init__(self, km):
        self.km, self.rows, self.orig = km, [], km.run_batch

    def __enter__(self):
        def counting(pool, seqs):
            self.rows.append(sum(len(t) for t, _, _, _ in seqs))
            return self.orig(pool, seqs)
        self.km.run_batch = counting
        return self

    def __exit__(self, *exc):
        self.km.run_batch = self.orig


@pytest.fixture(scope="module")
def l8_sd(golden):
    cfg = cases.llama8b_l2()
    sd = synthetic_state_dict(cfg, seed=0)
    g = golden("model_llama8b_l2.npz")
    assert weights_checksum(sd) == pytest.approx(float(g["weights_checksum"]), rel=1e-12)
    return sd


@pytest.mark.parametrize("scheme", ["int8", "int4"])
def test_llama8b_l2_generate_and_forward_match_reference(golden, l8_sd, scheme):
    g = golden("model_llama8b_l2.npz")
    cfg = cases.llama8b_l2()
    km = KshipraModel(config=cfg, state_dict=l8_sd, quantize=scheme)
    prompt = g["prompt"].tolist()
    toks = km.generate(prompt, max_new_tokens=cases.L8B_NEW, block_size=16,
                       prefill_chunk=cases.L8B_CHUNK)
    _same_tokens(toks, g[f"{scheme}/tokens"], g[f"{scheme}/margins"], f"8B-L2 {scheme} generate")
    # the reference-facing forward: 16-token chunks, then one-token decode steps
    B, new = 16, cases.L8B_NEW
    alloc = km.new_pool((len(prompt) + new + B - 1) // B, B)
    bt = list(range(alloc.pool.shape[0]))
    pos = 0
    while pos < len(prompt):
        c = min(cases.L8B_CHUNK, len(prompt) - pos)
        logits = km.forward(torch.tensor([prompt[pos:pos + c]]),
                            torch.arange(pos, pos + c).unsqueeze(0), alloc.pool, bt,
                            [bt[p // B] * B + p % B for p in range(pos, pos + c)], prefix_len=pos)
        pos += c
    assert logit_err(logits[0, -1].cpu(), g[f"{scheme}/logits_first"]) < LOGIT_RTOL
    ref = g[f"{scheme}/tokens"].tolist()
    for step in range(1, new):
        p = len(prompt) + step - 1
        logits = km.forward(torch.tensor([[ref[step - 1]]]), torch.tensor([[p]]), alloc.pool, bt,
                            [bt[p // B] * B + p % B], prefix_len=p)
    assert logit_err(logits[0, -1].cpu(), g[f"{scheme}/logits_last"]) < LOGIT_RTOL


@pytest.mark.parametrize("scheme", ["int8", "int4"])
def test_llama8b_l2_batched_engine_matches_reference(golden, l8_sd, scheme):
    """20 requests at once: prefill chunks mixed with decode rows, then
    20-row decode passes (the batched-decode linears and the batch lm_head)."""
    g = golden("model_llama8b_l2.npz")
    cfg = cases.llama8b_l2()
    km = KshipraModel(config=cfg, state_dict=l8_sd, quantize=scheme)
    prompts = cases.llama8b_batch_prompts(cfg.vocab)
    eng = _engine(km, num_blocks=128, budget=160)
    with _RowLog(km) as log:
        reqs = [eng.add_request(p, cases.L8B_BATCH_NEW) for p in prompts]
        _drain(eng, reqs)
    assert any(17 <= r <= 64 for r in log.rows), log.rows
    for i, r in enumerate(reqs):
        _same_tokens(r.generated_tokens, g[f"{scheme}/batch{i}/tokens"],
                     g[f"{scheme}/batch{i}/margins"], f"8B-L2 {scheme} batch request {i}")


@pytest.fixture(scope="module")
def qwen_sd():
    return synthetic_state_dict(QWEN25_05B, seed=0)


def test_cb_requests_batched_with_radix_reuse_match_reference(golden, qwen_sd):
    """Config-3 requests, shortened: wave A (20 requests) runs from an empty
    radix tree; wave B (20 more, same two system prefixes) starts its
    prefills after the prefix blocks wave A published.  Every request's
    tokens are the reference's (each computed there alone, from scratch)."""
    g = golden("model_cb_requests.npz")
    assert weights_checksum(qwen_sd) == pytest.approx(float(g["weights_checksum"]), rel=1e-12)
    km = KshipraModel(config=QWEN25_05B, state_dict=qwen_sd, quantize="int4")
    prompts = cases.cb_requests(QWEN25_05B.vocab)
    eng = _engine(km, num_blocks=512, budget=192)
    W = cases.CB_WAVE
    with _RowLog(km) as log_a:
        wave_a = [eng.add_request(p, cases.CB_NEW) for p in prompts[:W]]
        _drain(eng, wave_a)
    with _RowLog(km) as log_b:
        wave_b = [eng.add_request(p, cases.CB_NEW) for p in prompts[W:]]
        _drain(eng, wave_b)
    assert any(17 <= r <= 64 for r in log_a.rows + log_b.rows)
    prompt_b = sum(len(p) for p in prompts[W:])
    decode_b = W * (cases.CB_NEW - 1)
    # every wave-B request reuses at least its two system-prefix blocks
    assert sum(log_b.rows) <= prompt_b + decode_b - W * cases.CB_SYSTEM
    assert sum(log_a.rows) == sum(len(p) for p in prompts[:W]) + W * (cases.CB_NEW - 1)
    for i, r in enumerate(wave_a + wave_b):
        _same_tokens(r.generated_tokens, g[f"req{i}/tokens"], g[f"req{i}/margins"],
                     f"config-3 request {i}")
