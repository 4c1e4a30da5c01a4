"""Generate the golden fixtures by running the reference implementation itself.

Usage::

    python tests/golden/make_golden.py --reference <path to the Kshipra checkout> [--skip-05b]

The reference is pure Python (PyTorch + transformers); its ``engine``
package is imported from the checkout given on the command line and run on
the CPU on the seeded inputs of ``tests/golden/cases.py``.  Only outputs are
stored (inputs are regenerated from their seeds by the tests):

* ``quant.npz``        -- ``quantize_int8_per_channel`` / ``quantize_int4_per_group``
                          payload bytes and fp16 scales (engine/quantization.py:196-318)
* ``qlinear.npz``      -- ``QuantizedLinear.forward`` outputs (quantization.py:394-396)
* ``attention.npz``    -- ``chunked_attention`` outputs (chunked_prefill.py:93-140)
                          and the monolithic oracle for the same inputs
* ``model_tiny.npz``   -- ``KshipraModel.forward`` driven as chunked prefill +
                          greedy decode on the tiny Llama config (model.py:93-205):
                          tokens and per-step logits for int8 / int4 / fp32
* ``model_qwen05b.npz`` -- the same on the Qwen2.5-0.5B shape (int8, int4):
                          tokens, top-2 margins, logits after the prefill
* ``model_llama8b_l2.npz`` -- the Llama-3-8B shape cut to two layers (int8,
                          int4): one 64-token prompt in 16-token chunks + 12
                          greedy tokens (tokens, margins, logits of the first
                          and last step), and 20 short prompts with 4 greedy
                          tokens each (tokens, margins)
* ``model_cb_requests.npz`` -- 40 shortened config-3 requests (two 32-token
                          system prefixes + Poisson-trace suffixes) on the
                          Qwen2.5-0.5B shape, int4, 5 greedy tokens each,
                          every request run alone (tokens, margins)
* ``cache_trace.json`` -- block allocator / radix tree / scheduler decisions on
                          a deterministic operation sequence (prefix_cache.py,
                          continuous.py), with the clock replaced by a counter.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))   # repo root
sys.path.insert(0, HERE)

import cases  # noqa: E402
from kshipra_b200.config import TINY_LLAMA, QWEN25_05B  # noqa: E402
from kshipra_b200.weights import synthetic_state_dict, build_hf_model, weights_checksum  # noqa: E402


def _ref_generate(km, prompt, max_new, block_size, chunk):
    """Chunked prefill through ``KshipraModel.forward(prefix_len=...)`` then greedy decode."""
    from engine.prefix_cache import BlockAllocator
    lp = len(prompt)
    nb = (lp + max_new + block_size - 1) // block_size
    alloc = BlockAllocator(nb, block_size, km.n_layers, km.n_kv_heads, km.head_dim,
                           dtype=torch.float32)
    pool, bt = alloc.pool, list(range(nb))
    logs = []
    pos = 0
    with torch.inference_mode():
        while pos < lp:
            c = min(chunk, lp - pos)
            ids = torch.tensor([prompt[pos:pos + c]])
            positions = torch.arange(pos, pos + c).unsqueeze(0)
            slots = [bt[p // block_size] * block_size + p % block_size for p in range(pos, pos + c)]
            logits = km.forward(ids, positions, pool, bt, slots, prefix_len=pos)
            pos += c
        out = [int(logits[0, -1].argmax())]
        logs.append(logits[0, -1].clone())
        for step in range(1, max_new):
            p = lp + step - 1
            slot = bt[p // block_size] * block_size + p % block_size
            logits = km.forward(torch.tensor([[out[-1]]]), torch.tensor([[p]]), pool, bt, [slot],
                                prefix_len=p)
            out.append(int(logits[0, -1].argmax()))
            logs.append(logits[0, -1].clone())
    return out, logs


def make_quant(out_dir):
    from engine.quantization import quantize_int8_per_channel, quantize_int4_per_group
    d = {}
    for name, w, scheme, g in cases.quant_cases():
        if scheme == "int8":
            qw = quantize_int8_per_channel(w)
        else:
            qw = quantize_int4_per_group(w, g)
        d[f"{name}/payload"] = qw.payload.numpy()
        d[f"{name}/scales"] = qw.scales.numpy()
    np.savez_compressed(os.path.join(out_dir, "quant.npz"), **d)


def make_qlinear(out_dir):
    import torch.nn as nn
    from engine.quantization import QuantizedLinear
    d = {}
    for name, x, w, b, scheme, g in cases.qlinear_cases():
        lin = nn.Linear(w.shape[1], w.shape[0], bias=b is not None)
        with torch.no_grad():
            lin.weight.copy_(w)
            if b is not None:
                lin.bias.copy_(b)
        ql = QuantizedLinear(lin, scheme=scheme, group_size=g)
        with torch.no_grad():
            d[name] = ql(x).numpy()
    np.savez_compressed(os.path.join(out_dir, "qlinear.npz"), **d)


def make_attention(out_dir):
    from engine.chunked_prefill import chunked_attention, monolithic_attention
    d = {}
    for c in cases.attention_cases():
        q, kp, vp, bt = cases.attention_inputs(c)
        out = chunked_attention(q, kp, vp, bt, c["P"], c["C"], c["B"])
        d[c["name"]] = out.numpy()
        if c["hq"] == c["hkv"]:
            from oracle.attention import gather_contiguous
            k = gather_contiguous(kp, bt, c["P"] + c["C"])
            v = gather_contiguous(vp, bt, c["P"] + c["C"])
            d[c["name"] + "/monolithic"] = monolithic_attention(q, k, v, c["P"], c["C"]).numpy()
    q, kp, vp, bt, P, C, B = cases.mask_kat_inputs()
    d["mask_kat"] = chunked_attention(q, kp, vp, bt, P, C, B).numpy()
    np.savez_compressed(os.path.join(out_dir, "attention.npz"), **d)


def _kshipra(cfg, sd, quantize):
    from engine.model import KshipraModel
    hf = build_hf_model(cfg, sd)
    km = KshipraModel(hf, quantize=quantize)
    km.rope_theta = float(cfg.rope_theta)   # transformers 5.x hides rope_theta
    return km


def make_model_tiny(out_dir):
    cfg = TINY_LLAMA
    sd = synthetic_state_dict(cfg, seed=0)
    prompt = cases.prompt_ids(cfg.vocab, 32, seed=0)
    d = {"prompt": np.array(prompt), "weights_checksum": np.array(weights_checksum(sd))}
    for q in ("int8", "int4", "none"):
        km = _kshipra(cfg, sd, None if q == "none" else q)
        toks, logs = _ref_generate(km, prompt, 16, block_size=16, chunk=16)
        d[f"{q}/tokens"] = np.array(toks)
        d[f"{q}/logits"] = torch.stack(logs).numpy()
        # one-shot prefill through the reference's own generate (model.py:154-205)
        d[f"{q}/tokens_oneshot"] = np.array(km.generate(prompt, max_new_tokens=16, block_size=16))
    np.savez_compressed(os.path.join(out_dir, "model_tiny.npz"), **d)


def make_model_05b(out_dir):
    cfg = QWEN25_05B
    sd = synthetic_state_dict(cfg, seed=0)
    prompt = cases.prompt_ids(cfg.vocab, 512, seed=0)
    d = {"prompt": np.array(prompt), "weights_checksum": np.array(weights_checksum(sd))}
    for q in ("int8", "int4"):
        t0 = time.time()
        km = _kshipra(cfg, sd, q)
        toks, logs = _ref_generate(km, prompt, 50, block_size=16, chunk=128)
        L = torch.stack(logs)
        top = torch.topk(L, 2, dim=-1).values
        d[f"{q}/tokens"] = np.array(toks)
        d[f"{q}/margins"] = (top[:, 0] - top[:, 1]).numpy()
        d[f"{q}/logits0"] = L[0].numpy()
        print(f"  0.5B {q}: {time.time() - t0:.1f}s tokens[:8]={toks[:8]}", flush=True)
        del km
    np.savez_compressed(os.path.join(out_dir, "model_qwen05b.npz"), **d)


def _margins(logs):
    top = torch.topk(torch.stack(logs), 2, dim=-1).values
    return (top[:, 0] - top[:, 1]).numpy()


def make_model_8b(out_dir):
    cfg = cases.llama8b_l2()
    sd = synthetic_state_dict(cfg, seed=0)
    prompt = cases.prompt_ids(cfg.vocab, cases.L8B_PROMPT, seed=0)
    batch = cases.llama8b_batch_prompts(cfg.vocab)
    d = {"prompt": np.array(prompt), "weights_checksum": np.array(weights_checksum(sd))}
    for q in ("int8", "int4"):
        t0 = time.time()
        km = _kshipra(cfg, sd, q)
        toks, logs = _ref_generate(km, prompt, cases.L8B_NEW, block_size=16,
                                   chunk=cases.L8B_CHUNK)
        d[f"{q}/tokens"] = np.array(toks)
        d[f"{q}/margins"] = _margins(logs)
        d[f"{q}/logits_first"] = logs[0].numpy()
        d[f"{q}/logits_last"] = logs[-1].numpy()
        for i, p in enumerate(batch):
            bt, bl = _ref_generate(km, p, cases.L8B_BATCH_NEW, block_size=16, chunk=len(p))
            d[f"{q}/batch{i}/tokens"] = np.array(bt)
            d[f"{q}/batch{i}/margins"] = _margins(bl)
        print(f"  8B-L2 {q}: {time.time() - t0:.1f}s tokens[:8]={toks[:8]}", flush=True)
        del km
    np.savez_compressed(os.path.join(out_dir, "model_llama8b_l2.npz"), **d)


def make_cb_requests(out_dir):
    cfg = QWEN25_05B
    sd = synthetic_state_dict(cfg, seed=0)
    reqs = cases.cb_requests(cfg.vocab)
    d = {"weights_checksum": np.array(weights_checksum(sd))}
    km = _kshipra(cfg, sd, "int4")
    t0 = time.time()
    for i, p in enumerate(reqs):
        toks, logs = _ref_generate(km, p, cases.CB_NEW, block_size=16, chunk=len(p))
        d[f"req{i}/tokens"] = np.array(toks)
        d[f"req{i}/margins"] = _margins(logs)
    print(f"  cb requests: {time.time() - t0:.1f}s", flush=True)
    np.savez_compressed(os.path.join(out_dir, "model_cb_requests.npz"), **d)


class _Clock:
    def __init__(self):
        self.t = 0.0

    def __call__(self):
        self.t += 1.0
        return self.t


def cache_scenario(mods, clock):
    """Deterministic admission / release / eviction sequence over a PrefixCache.

    ``mods`` supplies ``PrefixCache`` and ``OutOfBlocksError``; the same
    scenario runs against the reference and against this package.
    """
    PrefixCache, OutOfBlocksError = mods
    rng = np.random.default_rng(5)
    B = 4
    cache = PrefixCache(num_blocks=40, block_size=B, num_layers=1, num_kv_heads=1, head_dim=1)
    systems = [list(rng.integers(0, 50, 12)) for _ in range(3)]
    live = []
    log = []
    for it in range(60):
        op = rng.integers(0, 4)
        if op <= 1 or not live:
            sp = systems[int(rng.integers(0, 3))]
            cut = int(rng.integers(0, len(sp) + 1))
            toks = [int(t) for t in sp[:cut]] + [int(t) for t in rng.integers(50, 60, int(rng.integers(1, 10)))]
            mb, ml, node = cache.tree.match(toks)
            cache.tree.pin(node)
            need = (len(toks) - ml + B - 1) // B
            try:
                nb = cache.allocate_blocks(need)
            except OutOfBlocksError:
                cache.tree.unpin(node)
                log.append(["oom", toks, list(mb), ml])
                continue
            leaf = cache.tree.insert(toks, nb, ml, node)
            cache.tree.pin(leaf)
            cache.tree.unpin(node)
            live.append(leaf)
            log.append(["admit", toks, list(mb), ml, list(nb), len(cache.allocator.free_blocks)])
        elif op == 2:
            leaf = live.pop(int(rng.integers(0, len(live))))
            cache.tree.unpin(leaf)
            log.append(["release", len(cache.allocator.free_blocks)])
        else:
            n = int(rng.integers(1, 6))
            ev = cache.tree.evict(n)
            log.append(["evict", n, ev, list(cache.allocator.free_blocks)])
    return log


def scheduler_scenario(mods, clock):
    """ContinuousEngine decisions on Poisson-shaped traffic (no real forward)."""
    PrefixCache, ContinuousEngine = mods
    cache = PrefixCache(num_blocks=64, block_size=16, num_layers=1, num_kv_heads=1, head_dim=1)
    eng = ContinuousEngine(cache, block_size=16, max_batch_tokens=48, itl_budget_s=0.1,
                           t_tok_s=0.001)
    rng = np.random.default_rng(9)
    log = []
    pending = [(int(rng.integers(20, 200)), int(rng.integers(2, 12))) for _ in range(12)]
    for it in range(400):
        if pending and it % 3 == 0:
            pl, mn = pending.pop(0)
            eng.add_request([int(t) for t in rng.integers(0, 100, pl)], mn)
        sched = eng.schedule()
        log.append([[r.req_id for r in sched.decodes], [[r.req_id, c] for r, c in sched.prefills],
                    sched.total_tokens, len(cache.allocator.free_blocks)])
        # apply the state transitions of ContinuousEngine.step (continuous.py:238-261)
        for r, c in sched.prefills:
            r.prefill_pos += c
            if r.prefill_pos >= len(r.prompt_tokens):
                r.state = type(r.state).RUNNING
        for r in sched.decodes:
            r.generated_tokens.append(0)
            if len(r.generated_tokens) >= r.max_new_tokens:
                eng._finish(r)
        if not pending and not eng.active_sequences and not eng.waiting_queue:
            break
    return log


def make_cache_trace(out_dir):
    import engine.prefix_cache as pc
    import engine.continuous as ct
    clock = _Clock()
    orig = time.monotonic
    pc.time.monotonic = clock
    try:
        trace = {
            "cache": cache_scenario((pc.PrefixCache, pc.OutOfBlocksError), clock),
            "scheduler": scheduler_scenario((pc.PrefixCache, ct.ContinuousEngine), clock),
        }
    finally:
        pc.time.monotonic = orig
    with open(os.path.join(out_dir, "cache_trace.json"), "w") as f:
        json.dump(trace, f)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--skip-05b", action="store_true")
    ap.add_argument("--only", default=None)
    a = ap.parse_args()
    sys.path.insert(0, os.path.abspath(a.reference))
    torch.set_num_threads(os.cpu_count() or 1)
    steps = [("quant", make_quant), ("qlinear", make_qlinear), ("attention", make_attention),
             ("model_tiny", make_model_tiny), ("cache_trace", make_cache_trace)]
    if not a.skip_05b:
        steps += [("model_qwen05b", make_model_05b), ("model_llama8b_l2", make_model_8b),
                  ("model_cb_requests", make_cb_requests)]
    for name, fn in steps:
        if a.only and name not in a.only.split(","):
            continue
        t0 = time.time()
        fn(HERE)
        print(f"{name}: {time.time() - t0:.1f}s", flush=True)


if __name__ == "__main__":
    main()
