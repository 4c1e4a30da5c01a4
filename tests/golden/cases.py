"""Seeded input builders shared by the fixture generator and the tests.

Every input is rebuilt from a seed with ``torch.Generator`` on the CPU, so the
committed fixtures only hold outputs; the tests regenerate identical inputs
(same torch build) and compare.
"""

from __future__ import annotations

from typing import Dict, List, Tuple

import torch


def _randn(shape, seed: int, std: float = 1.0) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randn(shape, generator=g, dtype=torch.float32) * std


# ---------------------------------------------------------------------------
# Quantizer cases: (name, weight, scheme, group_size)
# ---------------------------------------------------------------------------

def quant_cases() -> List[Tuple[str, torch.Tensor, str, int]]:
    cases = []
    cases.append(("gauss_64x512", _randn((64, 512), 1), "int8", 0))
    cases.append(("gauss_96x896_w002", _randn((96, 896), 2, 0.02), "int8", 0))
    cases.append(("k500", _randn((16, 500), 3), "int8", 0))
    cases.append(("k100", _randn((16, 100), 8), "int8", 0))
    cases.append(("one_by_one", torch.tensor([[1.5]]), "int8", 0))
    cases.append(("zeros_4x128", torch.zeros(4, 128), "int8", 0))
    # Rows whose fp16 scale underflows to 0 or to a subnormal.
    tiny = torch.zeros(6, 128)
    tiny[0, :4] = torch.tensor([1e-7, 0.0, -2e-7, 3e-9])
    tiny[1, :] = 1e-5
    tiny[2, :] = _randn((128,), 11, 1e-6)
    tiny[3, :] = _randn((128,), 12, 3e-3)
    tiny[4, 7] = -4e-6
    tiny[5, :] = _randn((128,), 13, 1e-4)
    cases.append(("tiny_scales", tiny, "int8", 0))
    # Exact ties: values at k + 0.5 of the scale exercise round-half-even.
    # Row absmax 63.5 gives scale exactly 0.5; the other entries j/2 + 0.25
    # land on j + 0.5 after division.
    body = (torch.arange(-126, 126, dtype=torch.float32) / 2.0 + 0.25).reshape(2, 126)
    ties = torch.cat([torch.full((2, 1), 63.5), body], dim=1)
    cases.append(("ties", ties, "int8", 0))

    cases.append(("g128_32x512", _randn((32, 512), 2), "int4", 128))
    cases.append(("g128_k500", _randn((16, 500), 3), "int4", 128))
    cases.append(("g128_k100", _randn((16, 100), 8), "int4", 128))
    cases.append(("g128_in1", torch.tensor([[0.5], [-0.3]]), "int4", 128))
    cases.append(("g32_64x512", _randn((64, 512), 6), "int4", 32))
    cases.append(("g256_64x512", _randn((64, 512), 6), "int4", 256))
    cases.append(("g2_8x10", _randn((8, 10), 21), "int4", 2))
    cases.append(("g6_8x20", _randn((8, 20), 22), "int4", 6))
    cases.append(("g128_tiny", tiny, "int4", 128))
    cases.append(("g128_zeros", torch.zeros(4, 256), "int4", 128))
    cases.append(("g128_96x896_w002", _randn((96, 896), 2, 0.02), "int4", 128))
    return cases


# ---------------------------------------------------------------------------
# Quantized-linear cases: (name, x, weight, bias|None, scheme, group_size)
# ---------------------------------------------------------------------------

def qlinear_cases():
    cases = []
    for m in (1, 3, 8, 16, 64, 130):
        x = _randn((m, 512), 100 + m)
        w = _randn((384, 512), 200, 0.05)
        b = _randn((384,), 300, 0.1)
        cases.append((f"w8_m{m}", x, w, b, "int8", 128))
        cases.append((f"w4_m{m}", x, w, None, "int4", 128))
    cases.append(("w8_k500", _randn((4, 500), 41), _randn((40, 500), 42, 0.05), None, "int8", 128))
    cases.append(("w4_k500", _randn((4, 500), 41), _randn((40, 500), 42, 0.05),
                  _randn((40,), 43), "int4", 128))
    cases.append(("w4_g32", _randn((2, 256), 44), _randn((72, 256), 45, 0.05), None, "int4", 32))
    return cases


# ---------------------------------------------------------------------------
# Paged attention cases
# ---------------------------------------------------------------------------

def attention_cases() -> List[Dict]:
    """Each case: hq, hkv, C, D, P, B, seed, permute (shuffle block ids)."""
    return [
        # engine tests: test_chunked_prefill.py:22-52, :55-82, :85-110
        dict(name="h4_c128_p256", hq=4, hkv=4, C=128, D=64, P=256, B=16, seed=42, permute=False),
        dict(name="decode_p1024", hq=4, hkv=4, C=1, D=64, P=1024, B=16, seed=42, permute=False),
        dict(name="unaligned_p37", hq=4, hkv=4, C=16, D=64, P=37, B=16, seed=42, permute=False),
        # GQA and paged layouts
        dict(name="gqa2_c16_p32", hq=4, hkv=2, C=16, D=64, P=32, B=16, seed=7, permute=True),
        dict(name="gqa7_decode_p549", hq=14, hkv=2, C=1, D=64, P=549, B=16, seed=8, permute=True),
        dict(name="gqa7_c48_p384", hq=14, hkv=2, C=48, D=64, P=384, B=16, seed=9, permute=True),
        dict(name="gqa4_d128_decode_p700", hq=8, hkv=2, C=1, D=128, P=700, B=16, seed=10, permute=True),
        dict(name="gqa4_d128_c40_p17", hq=8, hkv=2, C=40, D=128, P=17, B=16, seed=11, permute=True),
        dict(name="b64_c5_p0", hq=4, hkv=2, C=5, D=64, P=0, B=64, seed=12, permute=True),
        dict(name="b1_c3_p4", hq=2, hkv=1, C=3, D=64, P=4, B=1, seed=13, permute=True),
    ]


def attention_inputs(case: Dict):
    """Returns q [Hq,C,D], k_pool, v_pool [nb,Hkv,B,D], block_table (list)."""
    hq, hkv, C, D, P, B = case["hq"], case["hkv"], case["C"], case["D"], case["P"], case["B"]
    s = case["seed"]
    total = P + C
    nblk = (total + B - 1) // B
    nb = nblk + 3                     # spare blocks that must never be read
    q = _randn((hq, C, D), s)
    k_pool = _randn((nb, hkv, B, D), s + 1)
    v_pool = _randn((nb, hkv, B, D), s + 2)
    if case.get("permute"):
        g = torch.Generator().manual_seed(s + 3)
        bt = torch.randperm(nb, generator=g)[:nblk].tolist()
    else:
        bt = list(range(nblk))
    return q, k_pool, v_pool, bt


def mask_kat_inputs():
    """test_chunked_prefill.py:113-136: H=1, C=4, D=1, P=2, B=1, v = position."""
    H, C, D, P, B = 1, 4, 1, 2, 1
    q = torch.ones(H, C, D)
    k_pool = torch.ones(P + C, H, B, D)
    v_pool = torch.arange(P + C, dtype=torch.float32).view(P + C, 1, 1, 1).expand(P + C, H, B, D).clone()
    return q, k_pool, v_pool, list(range(P + C)), P, C, B


# ---------------------------------------------------------------------------
# Model cases
# ---------------------------------------------------------------------------

def prompt_ids(vocab: int, n: int, seed: int = 0) -> List[int]:
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, vocab, (n,), generator=g).tolist()


def batch_prompts(vocab: int, n: int, lo: int, hi: int, seed: int) -> List[List[int]]:
    """``n`` prompts of uniform random ids, lengths uniform in [lo, hi]."""
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(lo, hi + 1, (n,), generator=g).tolist()
    return [torch.randint(0, vocab, (ln,), generator=g).tolist() for ln in lens]


# Llama-3-8B shape cut to two layers (head_dim 128, 32 / 8 heads, untied
# lm_head, vocabulary 128256): one request chunk-prefilled in 16-token chunks
# with per-step logits, and a batch of short requests (4 greedy tokens each).
L8B_PROMPT, L8B_CHUNK, L8B_NEW = 64, 16, 12
L8B_BATCH, L8B_BATCH_NEW = 20, 4


def llama8b_l2():
    from kshipra_b200.config import LLAMA3_8B, truncated
    return truncated(LLAMA3_8B, 2)


def llama8b_batch_prompts(vocab: int) -> List[List[int]]:
    return batch_prompts(vocab, L8B_BATCH, 5, 40, seed=31)


# Config-3 requests, shortened: the first 40 draws of the config's Poisson
# trace (benchmarks/traffic.py:23-55 semantics: 8 req/s, prompts 256-2048,
# seed 42; the first 32 are the benchmark's own trace), each prompt length
# divided by 32, behind one of two 32-token system prefixes (request i uses
# prefix i % 2) so that a second wave of requests finds the first wave's
# prompt blocks in the radix tree.  Qwen2.5-0.5B shape, INT4, 5 greedy tokens.
CB_REQUESTS, CB_WAVE, CB_NEW, CB_SYSTEM = 40, 20, 5, 32


def cb_requests(vocab: int) -> List[List[int]]:
    import importlib.util
    import os
    root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    spec = importlib.util.spec_from_file_location("_bench_trace", os.path.join(root, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    trace = bench.poisson_trace(CB_REQUESTS, 8.0, (256, 2048), (128, 128), 42)
    systems = [prompt_ids(vocab, CB_SYSTEM, seed=100 + s) for s in range(2)]
    out = []
    for i, (_, plen, _) in enumerate(trace):
        out.append(systems[i % 2] + prompt_ids(vocab, plen // 32, seed=200 + i))
    return out
