"""Benchmark of the quantized forward path (one JSON line on rank 0).

Default workload (the path that shards): the Llama-3-8B
architecture, random-init N(0, 0.02), INT4 per-group (G = 128) weights, fp32
activations; 64 sequences decoding at context 4096 (K/V of the earlier
positions synthetic), KV block size 16, tensor parallel over the GPUs: heads,
MLP rows and the vocabulary are split, with two NCCL all-reduces per layer.
One step = one decode token for all 64 sequences (a CUDA-graph replay of
embedding -> 32 layers -> vocabulary-parallel lm_head + argmax -> on-device
position advance).  ``value`` = 64 tokens / step time for the whole job
(strong scaling: the same batch over more GPUs); ``per_gpu`` = value / N.
The 2048-token prefill chunk is timed beside it, and the Qwen2.5-0.5B INT8
batch-1 request workload (config 2: 512-token prompt in 128-token chunks +
50 greedy tokens; one independent replica per rank) is reported under
``qwen05b_int8``.

``--workload`` selects the other configurations (``qwen05b-int8``,
``qwen05b-int4``, ``qwen05b-int4-cb`` for config 3's continuous batching,
``llama8b-int8``, ``attn-prefix`` and ``micro`` for config 5).
``--impl reference`` times the CPU oracle (a restatement of the reference's
own algorithm, see oracle/) on this box's host cores instead.
"""

from __future__ import annotations

import argparse
import dataclasses
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOADS = {
    "qwen05b-int8": dict(preset="qwen2.5-0.5b", quantize="int8", prompt=512, chunk=128, new=50,
                         block=16),
    "qwen05b-int4": dict(preset="qwen2.5-0.5b", quantize="int4", prompt=512, chunk=128, new=50,
                         block=16),
    "tiny-int8": dict(preset="tiny-llama", quantize="int8", prompt=32, chunk=16, new=16, block=16),
    # config 4: Llama-3-8B shape, decode batch 64 at context 4096 (+ one
    # 2048-token prefill chunk), tensor parallel over the ranks
    "llama8b-int4": dict(preset="llama-3-8b", quantize="int4", batch=64, context=4096,
                         prefill=2048, block=16, tp=True),
    "llama8b-int8": dict(preset="llama-3-8b", quantize="int8", batch=64, context=4096,
                         prefill=2048, block=16, tp=True),
    # config 3: continuous batching of 32 concurrent requests (Poisson trace,
    # prompts 256-2048, 128 new tokens each), INT4 0.5B, replicas over ranks
    "qwen05b-int4-cb": dict(preset="qwen2.5-0.5b", quantize="int4", requests=32, rate=8.0,
                            prompt_range=(256, 2048), new=128, block=16, budget=2048, seed=42,
                            cb=True),
    # microbench part 2: decode attention of 64 requests sharing a radix-cached
    # 1024-token system prefix, plus 1-3072-token unique suffixes (8B heads)
    "attn-prefix": dict(preset="llama-3-8b", requests=64, prefix=1024, suffix=(1, 3072), block=16,
                        seed=0, attn=True),
}


def poisson_trace(num_requests, rate, prompt_range, new_range, seed):
    """(arrival_s, prompt_len, max_new_tokens) per request, from the same
    sequence of draws as the reference's generate_poisson_traffic
    (benchmarks/traffic.py:23-55): per request one exponential inter-arrival
    gap, then the prompt length, then the new-token count, from one
    random.Random(seed)."""
    import random
    rng = random.Random(seed)
    t, out = 0.0, []
    for _ in range(num_requests):
        t += rng.expovariate(rate)
        p = rng.randint(*prompt_range)
        n = rng.randint(*new_range)
        out.append((t, p, n))
    return out


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------

class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d.get("bf16_tflops"), "measured"
    return 6650.0, 1590.0, "fallback"


REPLICA_METRIC = ("decode tok/s, whole job (generated tokens of all ranks / request time incl. "
                  "512-token chunked prefill; one request per GPU)")
TP_METRIC = ("decode tok/s, whole job (Llama-3-8B shape, 64 sequences at context 4096, one "
             "token each per step, tensor parallel over the GPUs; per GPU = value / n_gpus)")


def replica_config(name, cfg, wl):
    return {"workload": name, "model": cfg.name, "quantize": wl["quantize"], "batch_per_gpu": 1,
            "prompt_len": wl["prompt"], "prefill_chunk": wl["chunk"], "new_tokens": wl["new"],
            "block_size": wl["block"],
            "l2": "inputs larger than L2 (every weight is streamed once per decode token)"}


def tp_config(name, cfg, wl):
    return {"workload": name, "model": cfg.name, "quantize": wl["quantize"],
            "global_batch": wl["batch"], "context": wl["context"], "block_size": wl["block"],
            "kv_cache": "fp32, synthetic values for the context positions",
            "l2": "inputs larger than L2 (weights + K/V read per step: tens of GB, >> 126 MB)"}


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------

def time_linear_family(km, T, reps=20):
    """The quantized linears of one decode step -- every layer's fused q/k/v
    (RMSNorm folded in), o, gate/up + SwiGLU (RMSNorm folded in) and down --
    at T token rows, captured in one CUDA graph (the same launches, with
    programmatic dependent launch, as in the decode graph) and replayed.
    Returns (ms per pass, algorithmic bytes per pass: packed weights + scales
    + fp32 activations in and out)."""
    from kshipra_b200.quantization import Workspace, linear_launch, swiglu_launch
    acts = km._alloc_acts(T)
    for t in acts.values():
        t.normal_()
    lws = Workspace()

    def once():
        for Ly in km.layers:
            linear_launch(acts["hidden"], Ly.qkv.qw, Ly.qkv.w, Ly.qkv.bias, acts["qkv"], ws=lws,
                          norm_w=Ly.ln1, eps=km.eps)
            linear_launch(acts["attn"].view(T, -1), Ly.o.qw, Ly.o.w, None, acts["xn"], ws=lws)
            swiglu_launch(acts["hidden"], Ly.gate_up.qw, Ly.gate_up.w, km.inter, acts["h"],
                          ws=lws, norm_w=Ly.ln2, eps=km.eps)
            linear_launch(acts["h"], Ly.down.qw, Ly.down.w, None, acts["xn"], ws=lws)
    once()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            once()
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    stream = torch.cuda.current_stream()
    e0.record(stream)
    for _ in range(reps):
        g.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    del g
    H, I = km.hidden, km.inter
    qkv = acts["qkv"].shape[1]
    act = 4 * T * sum([H + qkv, acts["attn"].view(T, -1).shape[1] + H, H + I, I + H])
    return ms, km.weight_bytes()["layers"] + km.n_layers * act


def time_lm_head(km, T, reps=30):
    """The fused final norm + fp32 lm_head + argmax at T rows, launched alone
    (the model's own call: the GEMV up to 16 rows, the tensor-core kernel on
    the split weight above)."""
    dev = km.device
    x = torch.randn((T, km.hidden), device=dev)
    tok = torch.empty(T, dtype=torch.int64, device=dev)
    ws = torch.empty(km.lm_ws_bytes(T), dtype=torch.uint8, device=dev)
    lg = km._tp_logits(T) if km.tp_world > 1 else None
    stream = torch.cuda.current_stream()

    def once():
        km._lm_head_call(x, T, lg, tok, ws)
    for _ in range(3):
        once()
    r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    r0.record(stream)
    for _ in range(reps):
        once()
    r1.record(stream)
    torch.cuda.synchronize()
    ms = r0.elapsed_time(r1) / reps
    nbytes = km.lm_head.numel() * 4 + T * km.hidden * 4 + (0 if lg is None else T * km.tp.vocab * 4)
    return ms, nbytes


def roofline_entry(kernel, nbytes, ms, hbm, peak_kind, traffic=None, source=None):
    achieved = nbytes / (ms * 1e-3) / 1e9
    return {"kernel": kernel, "bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
            "frac": achieved / hbm, "peak_kind": peak_kind, "traffic": traffic,
            "traffic_source": source, "algorithmic_bytes_per_launch": nbytes, "launch_ms": ms}


def measure_replica(args, wl, wl_name, ws, rank, local, dev, with_cpu_baseline):
    """One Qwen2.5-0.5B request per rank (512-token chunked prefill + 50 greedy
    tokens): an independent replica per rank, no data-path collective.  The
    caller owns the process group."""
    from kshipra_b200.config import PRESETS
    from kshipra_b200.model import KshipraModel, DecodeState
    from kshipra_b200.weights import synthetic_state_dict
    import kshipra_b200._lib as L

    cfg = PRESETS[wl["preset"]]
    sd = synthetic_state_dict(cfg, seed=0, device=dev)
    km = KshipraModel(config=cfg, state_dict=sd, quantize=wl["quantize"], device=dev)
    del sd
    torch.cuda.empty_cache()
    P, C, NEW, B = wl["prompt"], wl["chunk"], wl["new"], wl["block"]
    g = torch.Generator().manual_seed(rank)
    prompt = torch.randint(0, cfg.vocab, (P,), generator=g).tolist()
    nb = (P + NEW + B - 1) // B
    alloc = km.new_pool(nb, B)
    bt = list(range(nb))

    # One decode state reused by every step: the graph is captured once.
    st = DecodeState(km, alloc.pool, [bt], NEW)

    def device_step():
        first = km.prefill(prompt, alloc.pool, bt, C)
        st.start(first.view(1), [P])
        st.step_eager() if st.graph is None else st.graph.replay()
        for _ in range(NEW - 2):
            st.graph.replay()

    # warm-up (captures the graph); the library's launch counter gives the
    # kernels of one request: the prefill chunks and start, and the kernels
    # recorded into the decode graph (one step)
    n0 = L.lib().ksh_kernel_launches()
    first = km.prefill(prompt, alloc.pool, bt, C)
    st.start(first.view(1), [P])
    per_prefill = L.lib().ksh_kernel_launches() - n0
    st.step_eager()
    n0 = L.lib().ksh_kernel_launches()
    st.capture()
    per_tok = L.lib().ksh_kernel_launches() - n0
    for _ in range(max(args.warmup, 3)):
        device_step()
    torch.cuda.synchronize()

    def barrier():
        if ws > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier()
        e0.record(stream)
        for _ in range(args.steps):
            device_step()
        e1.record(stream)
        barrier()
    ms = e0.elapsed_time(e1) / args.steps
    tokens = st.history[0, :NEW].cpu().tolist()

    # decode-only rate: graph replays alone
    d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    first = km.prefill(prompt, alloc.pool, bt, C)
    st.start(first.view(1), [P])
    torch.cuda.synchronize()
    d0.record(stream)
    for _ in range(NEW - 1):
        st.graph.replay()
    d1.record(stream)
    torch.cuda.synchronize()
    decode_ms_per_tok = d0.elapsed_time(d1) / (NEW - 1)

    # end to end through the public API: host prompt list in, host token list out
    h2d = P * 8
    d2h = NEW * 8
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    a0.record(stream)
    for _ in range(args.steps):
        out = km.generate(prompt, max_new_tokens=NEW, block_size=B, prefill_chunk=C)
    a1.record(stream)
    barrier()
    e2e_ms = a0.elapsed_time(a1) / args.steps
    assert out == tokens, "public API and device loop disagree"

    # the dominant kernel family of a decode token, the quantized linears,
    # timed in graph replay; the lm_head (the largest single launch) beside it
    hbm, _, peak_kind = measured_peaks()
    lin_ms, lin_bytes = time_linear_family(km, 1)
    lm_ms, lm_bytes = time_lm_head(km, 1)

    # max over ranks
    t = torch.tensor([ms, e2e_ms, decode_ms_per_tok], dtype=torch.float64, device=dev)
    if ws > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms, e2e_ms, decode_ms_per_tok = t.tolist()
    wb = km.weight_bytes()
    res = dict(
        metric=REPLICA_METRIC,
        value=ws * NEW / (ms * 1e-3), unit="tok/s", n_gpus=ws, steps=args.steps,
        warmup=max(args.warmup, 3), ms_per_step=ms, higher_is_better=True, scaling="weak",
        vs_baseline=None, dtype="fp32 act / " + wl["quantize"] + " weights", data="synthetic",
        config=replica_config(wl_name, cfg, wl),
        parallelism=f"replicas x{ws} (no data-path collective)",
        per_gpu={"value": NEW / (ms * 1e-3), "unit": "tok/s/GPU"},
        decode_only={"value": ws * 1e3 / decode_ms_per_tok, "unit": "tok/s",
                     "ms_per_token": decode_ms_per_tok,
                     "bytes_per_token": wb["layers"] + wb["lm_head"],
                     "hbm_frac_of_" + peak_kind: (wb["layers"] + wb["lm_head"]) /
                     (decode_ms_per_tok * 1e-3) / 1e9 / hbm},
        e2e={"value": ws * NEW / (e2e_ms * 1e-3), "unit": "tok/s", "h2d_bytes_per_step": h2d,
             "d2h_bytes_per_step": d2h},
        roofline=roofline_entry("decode quantized linears of one token (q/k/v, o, gate/up + "
                                "SwiGLU, down; all layers, one CUDA-graph replay)",
                                lin_bytes, lin_ms, hbm, peak_kind),
        roofline_lm_head=roofline_entry("lm_head fp32 GEMV + argmax (ksh_lm_head_argmax)",
                                        lm_bytes, lm_ms, hbm, peak_kind,
                                        profiled_traffic(f"lm_head_{wl['preset']}"),
                                        f"profiles/lm_head_{wl['preset']}.md (ncu, one launch)"),
        gpu_launches=args.steps * (per_prefill + (NEW - 1) * per_tok),
        clocks=clk.summary(),
    )
    if rank == 0 and with_cpu_baseline and ws == 1:
        res["cpu_baseline"] = cpu_baseline(wl, cfg, prompt, samples=1)
    st.graph = None
    del st, km, alloc
    torch.cuda.empty_cache()
    return res


def run_ours(args, wl):
    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=dev)
    res = measure_replica(args, wl, args.workload, ws, rank, local, dev,
                          not args.no_cpu_baseline)
    if ws > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    return res, rank


# ---------------------------------------------------------------------------
# CPU oracle (reference algorithm) timing
# ---------------------------------------------------------------------------

def cpu_baseline(wl, cfg, prompt, samples=1):
    """Bounded sample of the workload on the CPU oracle: the full chunked
    prefill plus 2 decode tokens, extrapolated to the workload's tok/s."""
    from oracle.model import OracleModel
    from kshipra_b200.weights import synthetic_state_dict
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    sd = synthetic_state_dict(cfg, seed=0)
    om = OracleModel(cfg, sd, wl["quantize"])
    P, C, NEW, B = wl["prompt"], wl["chunk"], wl["new"], wl["block"]
    tp, td = [], []
    for _ in range(samples):
        nb = (P + NEW + B - 1) // B
        pool = om.new_pool(nb, B)
        bt = list(range(nb))
        t0 = time.perf_counter()
        pos = 0
        while pos < P:
            c = min(C, P - pos)
            ids = torch.tensor([prompt[pos:pos + c]])
            om.forward(ids, torch.arange(pos, pos + c).unsqueeze(0), pool, bt,
                       [bt[p // B] * B + p % B for p in range(pos, pos + c)], prefix_len=pos)
            pos += c
        tp.append(time.perf_counter() - t0)
        for s in range(2):
            p = P + s
            t0 = time.perf_counter()
            om.forward(torch.tensor([[1]]), torch.tensor([[p]]), pool, bt,
                       [bt[p // B] * B + p % B], prefix_len=p)
            td.append(time.perf_counter() - t0)
    t_pref = statistics.mean(tp)
    t_dec = statistics.mean(td)
    value = NEW / (t_pref + NEW * t_dec)
    return {"value": value, "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"oracle.model on {threads} threads: {samples}x (full {P}-token prefill "
                      f"({t_pref:.2f}s) + 2 decode tokens ({t_dec:.2f}s/token)); the "
                      f"{NEW}-token request = prefill + {NEW} decode tokens",
            "prefill_s": t_pref, "decode_s_per_token": t_dec,
            "sample_s": t_pref + 2 * t_dec}


def cpu_decode_8b(wl, steps, warmup):
    """The CPU oracle (the reference's algorithm) on config 4's decode step,
    sampled: the reference serves one request at a time (model.py:103), so a
    batch of 64 costs 64 single-request decode tokens.  One sample step is one
    decode token of one request at context ``wl['context']`` through the
    model cut to ONE layer (INT4/INT8 dequant + linears, RoPE, K/V write,
    chunked attention over the context, MLP) and through the model with NO
    layer (embedding, final norm, the untied fp32 lm_head); the full model's
    token costs ``t0 + 32 * (t1 - t0)``.  K/V of the context are synthetic
    (the cost does not depend on them).  Returns the sample and per-step
    times."""
    import copy
    from oracle.model import OracleModel
    from kshipra_b200.config import PRESETS, truncated
    from kshipra_b200.weights import synthetic_state_dict
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    full = PRESETS[wl["preset"]]
    cfg1 = truncated(full, 1)
    sd = synthetic_state_dict(cfg1, seed=0)
    om1 = OracleModel(cfg1, sd, wl["quantize"])
    del sd
    om0 = copy.copy(om1)
    om0.layers, om0.n_layers = [], 0
    ctx, bs = wl["context"], wl["block"]
    nb = ctx // bs + 1
    pool1 = om1.new_pool(nb, bs).uniform_(-1.0, 1.0)
    pool0 = om0.new_pool(nb, bs)
    bt = list(range(nb))

    def token(om, pool):
        p = ctx
        om.forward(torch.tensor([[1]]), torch.tensor([[p]]), pool, bt,
                   [bt[p // bs] * bs + p % bs], prefix_len=p)

    for _ in range(warmup):
        token(om1, pool1)
        token(om0, pool0)
    t1, t0, step_s = [], [], []
    for _ in range(steps):
        a = time.perf_counter()
        token(om1, pool1)
        b = time.perf_counter()
        token(om0, pool0)
        c = time.perf_counter()
        t1.append(b - a)
        t0.append(c - b)
        step_s.append(c - a)
    m1, m0 = statistics.median(t1), statistics.median(t0)
    t_tok = m0 + full.layers * max(m1 - m0, 0.0)
    value = 1.0 / t_tok
    return {"value": value, "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"oracle.model on {threads} threads, one request at a time: decode token at "
                      f"context {ctx} through the 1-layer cut ({m1:.2f}s) and the 0-layer cut "
                      f"({m0:.3f}s), x{steps} steps; {full.layers}-layer token = "
                      f"t0 + {full.layers}*(t1 - t0) = {t_tok:.2f}s; a batch of "
                      f"{wl['batch']} costs {wl['batch']} such tokens",
            "s_per_token_full_model": t_tok, "s_per_layer": m1 - m0, "s_embed_lm_head": m0}, \
        statistics.mean(step_s)


def run_reference(args, wl):
    ws, rank, local = dist_env()
    if rank != 0:
        return None, rank
    if wl.get("tp"):
        from kshipra_b200.config import PRESETS
        cfg = PRESETS[wl["preset"]]
        cb, step_s = cpu_decode_8b(wl, steps=args.steps, warmup=min(args.warmup, 2))
        res = dict(metric=TP_METRIC, value=cb["value"], unit="tok/s", n_gpus=ws, steps=args.steps,
                   warmup=min(args.warmup, 2), ms_per_step=step_s * 1e3, higher_is_better=True,
                   scaling="strong", vs_baseline=None,
                   dtype="fp32 act / " + wl["quantize"] + " weights", data="synthetic",
                   config=tp_config(args.workload, cfg, wl),
                   parallelism="cpu, one request at a time (the reference's forward is batch 1)",
                   impl="reference", cpu_baseline=cb,
                   e2e={"value": cb["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0})
        return res, rank
    from kshipra_b200.config import PRESETS
    cfg = PRESETS[wl["preset"]]
    g = torch.Generator().manual_seed(0)
    if wl.get("cb"):
        # The reference serves one request at a time: the trace's time is the
        # sum of its requests' times.  Sample one 256-token request (chunked
        # prefill + 2 decode tokens) and extrapolate with the per-token
        # prefill and decode costs over every prompt length of the trace.
        trace = poisson_trace(wl["requests"], wl["rate"], wl["prompt_range"],
                              (wl["new"], wl["new"]), wl["seed"])
        sample = dict(wl, prompt=256, chunk=128)
        prompt = torch.randint(0, cfg.vocab, (256,), generator=g).tolist()
        cb = cpu_baseline(sample, cfg, prompt, samples=1)
        t_total = sum(cb["prefill_s"] * p / 256 + n * cb["decode_s_per_token"] for _, p, n in trace)
        gen = sum(n for _, _, n in trace)
        value = gen / t_total
        cb = dict(cb, value=value, sample=cb["sample"] + f"; trace of {len(trace)} requests "
                  f"extrapolated per token ({t_total:.0f} s serial)")
        res = dict(metric="decode tok/s/GPU (generated tokens / trace time, 32 concurrent requests)",
                   value=value, unit="tok/s", n_gpus=ws, steps=args.steps, warmup=args.warmup,
                   ms_per_step=t_total * 1e3, higher_is_better=True, scaling="weak",
                   vs_baseline=None, dtype="fp32 act / " + wl["quantize"] + " weights",
                   data="synthetic",
                   config={"workload": args.workload, "model": cfg.name, "quantize": wl["quantize"],
                           "requests": wl["requests"], "new_tokens_per_request": wl["new"],
                           "parallelism": "cpu, one request at a time"},
                   impl="reference", cpu_baseline=cb,
                   e2e={"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0})
        return res, rank
    prompt = torch.randint(0, cfg.vocab, (wl["prompt"],), generator=g).tolist()
    # one step = one sample of the request: the full chunked prefill and two
    # decode tokens (timed), from which the 50-token request rate follows
    cb = cpu_baseline(wl, cfg, prompt, samples=max(1, args.steps))
    res = dict(metric=REPLICA_METRIC,
               value=cb["value"], unit="tok/s", n_gpus=ws, steps=args.steps,
               warmup=0, ms_per_step=1e3 * cb["sample_s"],
               higher_is_better=True, scaling="weak", vs_baseline=None,
               dtype="fp32 act / " + wl["quantize"] + " weights", data="synthetic",
               config=replica_config(args.workload, cfg, wl),
               parallelism="cpu, one request at a time",
               impl="reference", cpu_baseline=cb,
               e2e={"value": cb["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0})
    return res, rank


MICRO_SHAPES = [(4096, 6144), (4096, 28672), (14336, 4096)]   # K x N (Llama-3-8B projections)
MICRO_M = [1, 8, 64, 512, 4096]


def micro_case(scheme, m, k, n, dev):
    """Quantized weight + activations of one microbench point (N(0,1) activations)."""
    from kshipra_b200.quantization import quantize_int4_per_group, quantize_int8_per_channel
    g = torch.Generator(device=dev).manual_seed(m * 7 + k + n)
    w = torch.randn((n, k), generator=g, device=dev) * 0.02
    qw = quantize_int8_per_channel(w) if scheme == "int8" else quantize_int4_per_group(w, 128)
    del w
    x = torch.randn((m, k), generator=g, device=dev)
    y = torch.empty((m, n), device=dev)
    return qw, x, y


def run_micro(args):
    """Config: W4/W8 dequant-linear sweep, M in {1,8,64,512,4096} over the 8B shapes."""
    from kshipra_b200.quantization import Workspace, linear_launch
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    hbm, tc_peak, peak_kind = measured_peaks()
    ws = Workspace()
    flt = args.micro_filter.split(",") if args.micro_filter else None
    results = []
    points = [(sc, m, k, n) for sc in ("int4", "int8") for (k, n) in MICRO_SHAPES for m in MICRO_M]
    if flt:
        # any scheme:M:KxN point, also M outside the sweep (e.g. a 2048-row prefill chunk)
        points = []
        for tag in flt:
            sc, m, kn = tag.split(":")
            k, n = kn.split("x")
            points.append((sc, int(m), int(k), int(n)))
    for scheme, m, k, n in points:
        qw, x, y = micro_case(scheme, m, k, n, dev)
        # Enough weight copies that one pass over them exceeds twice the
        # L2, so every launch streams its weights from HBM; the launches
        # replay from a CUDA graph, so host overhead is not timed.
        ncopy = max(1, min(64, -(-300_000_000 // qw.storage_bytes())))
        if m > 64:
            ncopy = 1
        copies = [qw] + [dataclasses.replace(qw, payload=qw.payload.clone(),
                                             scales=qw.scales.clone())
                         for _ in range(ncopy - 1)]
        for c in copies:
            linear_launch(x, c, None, None, y, ws=ws)
        torch.cuda.synchronize()
        if args.profile:
            torch.cuda.cudart().cudaProfilerStart()
            linear_launch(x, qw, None, None, y, ws=ws)
            torch.cuda.synchronize()
            torch.cuda.cudart().cudaProfilerStop()
            continue
        rounds = max(1, 64 // ncopy) if m <= 64 else 3
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(rounds):
                for c in copies:
                    linear_launch(x, c, None, None, y, ws=ws)
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        graph.replay()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (rounds * ncopy)
        del graph, copies
        wbytes = qw.storage_bytes()
        nbytes = wbytes + m * k * 4 + m * n * 4
        flops = 2.0 * m * n * k
        results.append({"scheme": scheme, "m": m, "k": k, "n": n, "us": us,
                        "gb_s": nbytes / us / 1e3, "hbm_frac": nbytes / us / 1e3 / hbm,
                        "tflop_s": flops / us / 1e6,
                        "tensor_frac": flops / us / 1e6 / tc_peak})
        del qw, x, y
    if args.profile:
        print(json.dumps({"profile": "micro", "filter": args.micro_filter}))
        return
    gemv4 = [r for r in results if r["scheme"] == "int4" and r["m"] == 1]
    head = sum(r["hbm_frac"] for r in gemv4) / max(len(gemv4), 1)
    res = dict(metric="INT4 decode GEMV (M=1) fraction of measured HBM peak, 8B shapes",
               value=head, unit="fraction", n_gpus=1, steps=1, warmup=3, ms_per_step=None,
               higher_is_better=True, scaling="none", vs_baseline=None,
               dtype="fp32 act / int4|int8 weights", data="synthetic",
               config={"workload": "micro", "shapes_KxN": MICRO_SHAPES, "m": MICRO_M,
                       "l2": "M<=64: CUDA-graph replay over weight copies totalling >= 300 MB (> 2x L2) so every launch reads HBM; M>64: graph of 3 launches"},
               peaks={"hbm_gbs": hbm, "tensor_tflops": tc_peak, "kind": peak_kind},
               sweep=results)
    print(json.dumps(res))


def run_tp(args, wl):
    """Config 4: batched greedy decode of the 8B shape, tensor parallel.

    Every rank holds 1/N of the heads, intermediate rows and vocabulary; one
    step is one decode token for all ``batch`` sequences (a CUDA-graph replay
    of embedding -> 32 layers with two NCCL all-reduces each -> vocabulary-
    parallel lm_head + argmax -> on-device position advance).  The K/V cache
    of the ``context`` earlier positions is filled with synthetic values (the
    decode cost does not depend on them); the 2048-token prefill chunk is
    timed separately.  value = batch tokens per step / step time (whole job),
    strong scaling: the same batch over more GPUs."""
    from kshipra_b200 import _lib as L
    from kshipra_b200.config import PRESETS
    from kshipra_b200.model import DecodeState, KshipraModel
    from kshipra_b200.weights import synthetic_state_dict

    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=dev)
    cfg = PRESETS[wl["preset"]]
    sd = synthetic_state_dict(cfg, seed=0, device=dev)          # the same weights on every rank
    km = KshipraModel(config=cfg, state_dict=sd, quantize=wl["quantize"], device=dev,
                      tp=(rank, ws, None) if ws > 1 else None)
    del sd
    torch.cuda.empty_cache()
    Bt, ctx, bs, PF = wl["batch"], wl["context"], wl["block"], wl["prefill"]
    steps_total = max(args.warmup, 3) + args.steps + 4
    nbs = (ctx + steps_total + bs) // bs + 1
    npf = (PF + bs - 1) // bs + 1
    alloc = km.new_pool(Bt * nbs + npf, bs)
    pool = alloc.pool
    pool.uniform_(-1.0, 1.0)                                    # synthetic K/V of the context
    bts = [list(range(i * nbs, (i + 1) * nbs)) for i in range(Bt)]
    st = DecodeState(km, pool, bts, steps_total)
    g = torch.Generator().manual_seed(1)
    first = torch.randint(0, cfg.vocab, (Bt,), generator=g).to(dev)
    st.start(first, [ctx] * Bt)

    def barrier():
        if ws > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    n0 = L.lib().ksh_kernel_launches()
    st.step_eager()
    per_step = L.lib().ksh_kernel_launches() - n0               # this library's kernels per step
    graph = True
    try:
        st.capture()
    except Exception as e:                                      # eager steps if capture fails
        graph = False
        if rank == 0:
            print(f"# decode graph capture failed, eager steps: {e}", file=sys.stderr)
    step = (lambda: st.graph.replay()) if graph else st.step_eager
    for _ in range(max(args.warmup, 3)):
        step()
    barrier()
    if args.profile:
        # one decode step between cudaProfilerStart/Stop (ncu --profile-from-start off)
        torch.cuda.cudart().cudaProfilerStart()
        step()
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStop()
        if graph:
            st.graph = None
        if ws > 1:
            torch.distributed.destroy_process_group()
        return {"profile": args.workload, "decode_graph": graph, "batch": Bt,
                "launches_per_step": per_step}, rank
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier()
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        barrier()
    ms = e0.elapsed_time(e1) / args.steps

    # end to end: every step the batch's input tokens come from pinned host
    # memory and the generated tokens are read back
    h_in = torch.randint(0, cfg.vocab, (Bt,), generator=g).pin_memory()
    h_out = torch.empty(Bt, dtype=torch.int64).pin_memory()
    barrier()
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record(stream)
    for _ in range(args.steps):
        st.ids.copy_(h_in, non_blocking=True)
        step()
        h_out.copy_(st.next, non_blocking=True)
    a1.record(stream)
    barrier()
    e2e_ms = a0.elapsed_time(a1) / args.steps

    # dominant kernel: decode attention of one layer, timed alone
    nb_, L_, _, hkv, bs_, d = pool.shape
    rc, rs = km._rope_tables()
    qkv = st.acts["qkv"]
    attn = st.acts["attn"]

    dws = st.attn_ws.dec

    def attn_once():
        L.call("ksh_decode_attention_ws", qkv.data_ptr(), Bt, km.n_heads, km.n_kv_heads, d,
               st.positions.data_ptr(), st.slots.data_ptr(), rc.data_ptr(), rs.data_ptr(),
               rc.shape[0], pool.data_ptr(), nb_, L_, 0, bs_, st.block_tables.data_ptr(),
               st.block_tables.shape[1], st.capacity, attn.data_ptr(), dws.data_ptr(),
               dws.numel(), km.flags.data_ptr(), L.stream_ptr())
    for _ in range(3):
        attn_once()
    r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    R = 20
    r0.record(stream)
    for _ in range(R):
        attn_once()
    r1.record(stream)
    torch.cuda.synchronize()
    attn_ms = r0.elapsed_time(r1) / R
    ctx_now = int(st.positions[0]) + 1
    attn_bytes = Bt * ctx_now * 2 * hkv * d * 4 + Bt * (km.n_heads * d * 4) * 2

    # one prefill chunk of PF tokens on fresh blocks
    pf_bt = list(range(Bt * nbs, Bt * nbs + npf))
    prompt = torch.randint(0, cfg.vocab, (PF,), generator=g).tolist()
    km.prefill(prompt, pool, pf_bt, PF)
    barrier()
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record(stream)
    km.prefill(prompt, pool, pf_bt, PF)
    p1.record(stream)
    barrier()
    pf_ms = p0.elapsed_time(p1)

    # the batch's quantized linears (one graph replay over all layers) and the
    # vocabulary-parallel lm_head, each timed alone at the step's 64 rows
    lin_ms, lin_bytes = time_linear_family(km, Bt)
    lm_ms, lm_bytes = time_lm_head(km, Bt)

    t = torch.tensor([ms, e2e_ms, attn_ms, pf_ms, lin_ms, lm_ms], dtype=torch.float64, device=dev)
    if ws > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms, e2e_ms, attn_ms, pf_ms, lin_ms, lm_ms = t.tolist()
    hbm, _, peak_kind = measured_peaks()
    wb = km.weight_bytes()
    step_bytes = wb["layers"] + wb["lm_head"] + L_ * attn_bytes
    res = dict(
        metric=TP_METRIC,
        value=Bt / (ms * 1e-3), unit="tok/s", n_gpus=ws, steps=args.steps,
        warmup=max(args.warmup, 3), ms_per_step=ms, higher_is_better=True, scaling="strong",
        vs_baseline=None, dtype="fp32 act / " + wl["quantize"] + " weights", data="synthetic",
        config=tp_config(args.workload, cfg, wl),
        parallelism=(f"tensor parallel x{ws}: heads, MLP rows and vocabulary split, two NCCL "
                     "all-reduces per layer" if ws > 1 else "one GPU (tp1)"),
        decode_graph=graph,
        per_gpu={"value": Bt / (ms * 1e-3) / ws, "unit": "tok/s/GPU"},
        decode_step={"bytes_rank0": step_bytes,
                     "hbm_frac_of_" + peak_kind: step_bytes / (ms * 1e-3) / 1e9 / hbm,
                     "share_attention": L_ * attn_ms / ms, "share_linears": lin_ms / ms,
                     "share_lm_head": lm_ms / ms},
        prefill={"tokens": PF, "ms": pf_ms, "tok_s": PF / (pf_ms * 1e-3)},
        e2e={"value": Bt / (e2e_ms * 1e-3), "unit": "tok/s", "h2d_bytes_per_step": Bt * 8,
             "d2h_bytes_per_step": Bt * 8},
        roofline=roofline_entry(
            "fused decode attention (ksh_decode_attention_ws), one layer",
            attn_bytes, attn_ms, hbm, peak_kind,
            profiled_traffic("decode_attention_llama8b_b64_ctx4096") if ws == 1 else None,
            "profiles/decode_attention_llama8b_b64_ctx4096.md (ncu, one launch, TP1)"),
        roofline_linears=roofline_entry(
            "batched-decode quantized linears of one step at 64 rows (q/k/v, o, gate/up + "
            "SwiGLU, down; all layers, one CUDA-graph replay)", lin_bytes, lin_ms, hbm, peak_kind),
        roofline_lm_head=roofline_entry(
            "batch lm_head + argmax at 64 rows (ksh_lm_head_argmax_tc on the split fp16 weight, "
            "vocabulary shard)",
            lm_bytes, lm_ms, hbm, peak_kind),
        gpu_launches=args.steps * per_step,
        clocks=clk.summary(),
    )
    if graph:
        st.graph = None                 # release the captured NCCL calls before teardown
    torch.cuda.synchronize()
    del st, km, pool, alloc
    torch.cuda.empty_cache()
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"], _ = cpu_decode_8b(wl, steps=2, warmup=1)
    if not args.no_replica:
        # the 0.5B batch-1 request workload (config 2) beside it: one
        # independent replica per rank
        rep = measure_replica(args, WORKLOADS["qwen05b-int8"], "qwen05b-int8", ws, rank, local,
                              dev, with_cpu_baseline=False)
        res["qwen05b_int8"] = {k: rep[k] for k in ("metric", "value", "unit", "ms_per_step",
                                                   "config", "parallelism", "per_gpu",
                                                   "decode_only", "e2e", "roofline",
                                                   "roofline_lm_head", "gpu_launches")}
    if ws > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    return res, rank


def run_cb(args, wl):
    """Config 3: continuous batching through ContinuousEngine with the real
    batched forward (run_batch: mixed prefill chunks and decode tokens in one
    varlen pass per iteration).

    One step = the whole trace: 32 requests from the Poisson trace, all
    admitted at the start so that they run concurrently (arrival order kept),
    each prefilled in chunks out of a 2048-token iteration budget and decoded
    for 128 tokens.  value = generated tokens / trace time.  The engine reads
    every iteration's tokens back to the host, so each step is end to end by
    construction.  Multi-GPU: one independent replica per rank (weak scaling)."""
    from kshipra_b200 import _lib as L
    from kshipra_b200.config import PRESETS
    from kshipra_b200.continuous import ContinuousEngine
    from kshipra_b200.model import KshipraModel
    from kshipra_b200.prefix_cache import PrefixCache
    from kshipra_b200.weights import synthetic_state_dict

    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=dev)
    cfg = PRESETS[wl["preset"]]
    sd = synthetic_state_dict(cfg, seed=0, device=dev)
    km = KshipraModel(config=cfg, state_dict=sd, quantize=wl["quantize"], device=dev)
    del sd
    torch.cuda.empty_cache()
    trace = poisson_trace(wl["requests"], wl["rate"], wl["prompt_range"], (wl["new"], wl["new"]),
                          wl["seed"])
    g = torch.Generator().manual_seed(rank)
    prompts = [torch.randint(0, cfg.vocab, (p,), generator=g).tolist() for _, p, _ in trace]
    bs = wl["block"]
    nblocks = sum((p + n + bs - 1) // bs for _, p, n in trace) + 16

    def run_trace():
        cache = PrefixCache(nblocks, bs, cfg.layers, cfg.kv_heads, cfg.head_dim,
                            dtype=torch.float32, device=dev)
        eng = ContinuousEngine(cache, block_size=bs, max_batch_tokens=wl["budget"],
                               itl_budget_s=wl["budget"] * 1e-3, t_tok_s=1e-3, model=km)
        reqs = [eng.add_request(p, n) for p, (_, _, n) in zip(prompts, trace)]
        t0 = time.monotonic()
        for r in reqs:
            r.arrival_time = t0
        # token emission times, taken here: the engine's itl_times keep the
        # reference's arithmetic (continuous.py:252-255), not intervals
        seen = [0] * len(reqs)
        last = [t0] * len(reqs)
        ttft, itl, it_pf, it_dec = [], [], [], []
        iters = 0
        profiled = False
        while not all(r.state.value == "finished" for r in reqs):
            decode_only = all(r.state.value in ("running", "finished") for r in reqs)
            if args.profile and decode_only and not profiled:
                # one decode-only iteration between cudaProfilerStart/Stop
                torch.cuda.synchronize()
                torch.cuda.cudart().cudaProfilerStart()
                eng.step()
                torch.cuda.synchronize()
                torch.cuda.cudart().cudaProfilerStop()
                profiled = True
            else:
                eng.step()
            iters += 1
            now = time.monotonic()
            (it_dec if decode_only else it_pf).append(now - max(last + [t0]))
            for j, r in enumerate(reqs):
                k = len(r.generated_tokens)
                if k > seen[j]:
                    (ttft if seen[j] == 0 else itl).append(now - last[j])
                    seen[j], last[j] = k, now
        return reqs, iters, sorted(ttft), sorted(itl), sorted(it_pf), sorted(it_dec)

    profile = args.profile
    args.profile = False
    for _ in range(max(args.warmup, 3) if not profile else 1):
        run_trace()
    if profile:
        args.profile = True
        run_trace()
        if ws > 1:
            torch.distributed.destroy_process_group()
        return {"profile": args.workload, "captured": "one decode-only engine iteration"}, rank

    def barrier():
        if ws > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n0 = L.lib().ksh_kernel_launches()
    with ClockSampler(local) as clk:
        barrier()
        w0 = time.perf_counter()
        e0.record(stream)
        for _ in range(args.steps):
            reqs, iters, ttft, itl, it_pf, it_dec = run_trace()
        e1.record(stream)
        barrier()
        wall = (time.perf_counter() - w0) / args.steps
    launches = L.lib().ksh_kernel_launches() - n0
    ms = e0.elapsed_time(e1) / args.steps
    gen = sum(len(r.generated_tokens) for r in reqs)
    t = torch.tensor([ms, wall * 1e3], dtype=torch.float64, device=dev)
    if ws > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms, wall_ms = t.tolist()

    def pct(v, q):
        return v[min(len(v) - 1, int(q * len(v)))] * 1e3 if v else None

    prompt_tokens = sum(p for _, p, _ in trace)
    res = dict(
        metric="decode tok/s/GPU (generated tokens / trace time, 32 concurrent requests)",
        value=ws * gen / (ms * 1e-3), unit="tok/s", n_gpus=ws, steps=args.steps,
        warmup=max(args.warmup, 3), ms_per_step=ms, higher_is_better=True, scaling="weak",
        vs_baseline=None, dtype="fp32 act / " + wl["quantize"] + " weights", data="synthetic",
        config={"workload": args.workload, "model": cfg.name, "quantize": wl["quantize"],
                "requests": wl["requests"], "prompt_tokens": prompt_tokens,
                "new_tokens_per_request": wl["new"], "arrival": "Poisson trace order, all admitted at t0",
                "iteration_budget_tokens": wl["budget"], "block_size": bs,
                "parallelism": f"replicas{ws}",
                "l2": "inputs larger than L2 (weights + growing K/V per iteration)"},
        per_gpu={"value": gen / (ms * 1e-3), "unit": "tok/s/GPU"},
        engine={"iterations": iters, "ttft_ms_p50": pct(ttft, 0.5), "ttft_ms_p99": pct(ttft, 0.99),
                "itl_ms_p50": pct(itl, 0.5), "itl_ms_p99": pct(itl, 0.99),
                "prefill_iterations": len(it_pf), "prefill_iter_ms_p50": pct(it_pf, 0.5),
                "decode_iterations": len(it_dec), "decode_iter_ms_p50": pct(it_dec, 0.5),
                "decode_iterations_ms_total": sum(it_dec) * 1e3},
        e2e={"value": ws * gen / (wall_ms * 1e-3), "unit": "tok/s",
             "h2d_bytes_per_step": 8 * (prompt_tokens + gen), "d2h_bytes_per_step": 8 * (gen + iters)},
        gpu_launches=launches,
        clocks=clk.summary(),
    )
    if ws > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    return res, rank


def run_attn_prefix(args, wl):
    """Microbench part 2: one decode-attention layer (ksh_decode_attention:
    RoPE, K/V write, paged GQA attention) for 64 requests whose block tables
    share the 64 blocks of a 1024-token prefix.  The prefix is inserted once
    into the RadixTree; each request matches it (the shared blocks) and pins
    the node, then allocates blocks for its unique suffix and the new token.

    value = logical K/V bytes (every request's keys, the shared prefix counted
    per request) / launch time; the unique bytes (prefix counted once) are
    reported beside it -- the prefix stays in L2 across the requests that
    share it, so the logical rate can exceed the HBM peak."""
    from kshipra_b200 import _lib as L
    from kshipra_b200.config import PRESETS
    from kshipra_b200.model import rope_tables
    from kshipra_b200.prefix_cache import PrefixCache

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = PRESETS[wl["preset"]]
    hq, hkv, d, bs = cfg.heads, cfg.kv_heads, cfg.head_dim, wl["block"]
    R, P = wl["requests"], wl["prefix"]
    g = torch.Generator().manual_seed(wl["seed"])
    sfx = torch.randint(wl["suffix"][0], wl["suffix"][1] + 1, (R,), generator=g).tolist()
    nblocks = P // bs + sum((s + 1 + bs - 1) // bs + 1 for s in sfx) + 8
    cache = PrefixCache(nblocks, bs, 1, hkv, d, dtype=torch.float32, device=dev)
    prefix = torch.randint(0, cfg.vocab, (P,), generator=g).tolist()
    pblocks = cache.allocate_blocks(P // bs)
    cache.tree.insert(prefix, pblocks, 0, cache.tree.root)
    tables, positions = [], []
    for s in sfx:
        toks = prefix + torch.randint(0, cfg.vocab, (s,), generator=g).tolist()
        blocks, matched, node = cache.tree.match(toks)
        assert matched == P and blocks == pblocks
        cache.tree.pin(node)
        own = cache.allocate_blocks((len(toks) + 1 - matched + bs - 1) // bs)
        tables.append(blocks + own)
        positions.append(len(toks))                    # the new token's position
    maxb = max(len(t) for t in tables)
    bt = torch.full((R, maxb), -1, dtype=torch.int32)
    for i, t in enumerate(tables):
        bt[i, :len(t)] = torch.tensor(t, dtype=torch.int32)
    pool = cache.allocator.pool
    pool.uniform_(-1.0, 1.0)
    btd = bt.to(dev)
    pos = torch.tensor(positions, dtype=torch.int64, device=dev)
    slots = torch.tensor([tables[i][p // bs] * bs + p % bs for i, p in enumerate(positions)],
                         dtype=torch.int64, device=dev)
    qkv = torch.randn((R, (hq + 2 * hkv) * d), device=dev)
    rc, rs = (t.to(dev) for t in rope_tables(d, cfg.rope_theta, max(positions) + 1))
    out = torch.empty((R, hq, d), device=dev)
    flags = torch.zeros(1, dtype=torch.int32, device=dev)
    s_ = L.stream_ptr()

    def run():
        L.call("ksh_decode_attention", qkv.data_ptr(), R, hq, hkv, d, pos.data_ptr(), slots.data_ptr(),
               rc.data_ptr(), rs.data_ptr(), rc.shape[0], pool.data_ptr(), pool.shape[0], 1, 0, bs,
               btd.data_ptr(), maxb, max(positions) + 1, out.data_ptr(), flags.data_ptr(), s_)
    for _ in range(max(args.warmup, 3)):
        run()
    torch.cuda.synchronize()
    if int(flags.item()):
        raise RuntimeError(f"decode attention raised flags {int(flags.item())}")
    n0 = L.lib().ksh_kernel_launches()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        torch.cuda.synchronize()
        e0.record()
        for _ in range(args.steps):
            run()
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    row = 2 * hkv * d * 4                               # K and V of one token, all kv heads
    logical = sum(p + 1 for p in positions) * row + R * hq * d * 8
    unique = (P + sum(p + 1 - P for p in positions)) * row + R * hq * d * 8
    hbm, _, peak_kind = measured_peaks()
    ach = logical / (ms * 1e-3) / 1e9
    res = dict(
        metric="paged GQA decode attention, logical K/V GB/s (64 requests sharing a 1024-token prefix)",
        value=ach, unit="GB/s", n_gpus=1, steps=args.steps, warmup=max(args.warmup, 3),
        ms_per_step=ms, higher_is_better=True, scaling="weak", vs_baseline=None, dtype="fp32",
        data="synthetic",
        config={"workload": args.workload, "model_heads": f"{hq}/{hkv} x {d}", "requests": R,
                "shared_prefix": P, "suffix_range": list(wl["suffix"]),
                "suffix_total": sum(sfx), "block_size": bs,
                "l2": "prefix shared through L2 by construction; the suffix K/V (%.2f GB) exceed L2"
                      % ((unique - P * row) / 1e9)},
        unique={"bytes": unique, "gb_s": unique / (ms * 1e-3) / 1e9,
                "frac_of_" + peak_kind: unique / (ms * 1e-3) / 1e9 / hbm},
        e2e={"value": ach, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        roofline={"kernel": "fused decode attention (ksh_decode_attention), one layer", "bound": "hbm",
                  "achieved": ach, "peak": hbm, "unit": "GB/s", "frac": ach / hbm,
                  "peak_kind": peak_kind, "traffic": None, "algorithmic_bytes_per_launch": logical,
                  "launch_ms": ms},
        gpu_launches=int(L.lib().ksh_kernel_launches() - n0),
        clocks=clk.summary(),
    )
    return res, 0


def run_reference_attn(args, wl):
    """Reference arm of the shared-prefix microbench: the oracle's restatement
    of chunked_attention (chunked_prefill.py:93-140, chunk_len 1) on the host
    cores, one request at a time as the reference runs it, over a sample of
    the workload's requests (same prefix and suffix lengths), in logical
    K/V GB/s."""
    ws, rank, _ = dist_env()
    if rank != 0:
        return None, rank
    from kshipra_b200.config import PRESETS
    from oracle.attention import chunked_attention
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    cfg = PRESETS[wl["preset"]]
    hq, hkv, d, bs = cfg.heads, cfg.kv_heads, cfg.head_dim, wl["block"]
    R, P = wl["requests"], wl["prefix"]
    g = torch.Generator().manual_seed(wl["seed"])
    sfx = torch.randint(wl["suffix"][0], wl["suffix"][1] + 1, (R,), generator=g).tolist()
    sample = sfx[:4]
    nb = P // bs + max(sample) // bs + 2
    kp = torch.rand((nb, hkv, bs, d)) * 2 - 1
    vp = torch.rand((nb, hkv, bs, d)) * 2 - 1
    row = 2 * hkv * d * 4
    nbytes, t = 0, 0.0
    for s_ in sample:
        p = P + s_
        q = torch.randn((hq, 1, d))
        bt = list(range((p + 1 + bs - 1) // bs))
        t0 = time.perf_counter()
        chunked_attention(q, kp, vp, bt, p, 1, bs)
        t += time.perf_counter() - t0
        nbytes += (p + 1) * row
    value = nbytes / t / 1e9
    res = dict(metric="paged GQA decode attention, logical K/V GB/s (64 requests sharing a 1024-token prefix)",
               value=value, unit="GB/s", n_gpus=ws, steps=args.steps, warmup=args.warmup,
               ms_per_step=1e3 * t / len(sample) * R, higher_is_better=True, scaling="weak",
               vs_baseline=None, dtype="fp32", data="synthetic",
               config={"workload": args.workload, "parallelism": "cpu, one request at a time"},
               impl="reference",
               cpu_baseline={"value": value, "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": f"oracle chunked_attention, {len(sample)} of the {R} requests "
                                       f"(contexts {[P + x for x in sample]}), {threads} threads"},
               e2e={"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0})
    return res, rank


def run_profile_lm_head(args, wl):
    """The roofline kernel alone, for an ncu capture of a small case: the
    workload's fp32 lm_head weight [vocab, hidden] (544 MB for the 0.5B shape)
    and one ksh_lm_head_argmax call (fused final norm + GEMV + argmax, one
    token row) between cudaProfilerStart/Stop, after a warm-up."""
    from kshipra_b200 import _lib as L
    from kshipra_b200.config import PRESETS
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = PRESETS[wl["preset"]]
    g = torch.Generator(device=dev).manual_seed(0)
    w = torch.randn((cfg.vocab, cfg.hidden), generator=g, device=dev) * 0.02
    nw = torch.ones(cfg.hidden, device=dev)
    x = torch.randn((1, cfg.hidden), generator=g, device=dev)
    tok = torch.empty(1, dtype=torch.int64, device=dev)
    ws = torch.zeros(int(L.lib().ksh_lm_head_workspace_size(1, cfg.vocab)), dtype=torch.uint8, device=dev)
    s = L.stream_ptr()

    def run():
        L.call("ksh_lm_head_argmax", x.data_ptr(), 1, cfg.hidden, nw.data_ptr(), 1e-6, w.data_ptr(),
               cfg.vocab, None, tok.data_ptr(), ws.data_ptr(), ws.numel(), s)
    for _ in range(3):
        run()
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStart()
    run()
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStop()
    print(json.dumps({"profile": "lm_head", "workload": args.workload,
                      "algorithmic_bytes": cfg.vocab * cfg.hidden * 4 + cfg.hidden * 8}))


def run_profile_lm_head_tc(args, wl):
    """The batch lm_head alone for an ncu capture: the workload's vocabulary x
    hidden weight split into fp16 hi / lo (2.1 GB for the 8B shape; the fp32
    copy is freed after the split) and one ksh_lm_head_argmax_tc call at 64
    rows (fused final norm + tensor-core GEMM + argmax) between
    cudaProfilerStart/Stop, after a warm-up."""
    from kshipra_b200 import _lib as L
    from kshipra_b200.config import PRESETS
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = PRESETS[wl["preset"]]
    V, H, M = cfg.vocab, cfg.hidden, 64
    g = torch.Generator(device=dev).manual_seed(0)
    w = torch.randn((V, H), generator=g, device=dev) * 0.02
    hi = torch.empty((V, H), dtype=torch.float16, device=dev)
    lo = torch.empty_like(hi)
    inv = torch.empty(V, device=dev)
    s = L.stream_ptr()
    L.call("ksh_lm_head_split_weight", w.data_ptr(), V, H, hi.data_ptr(), lo.data_ptr(),
           inv.data_ptr(), None, s)
    torch.cuda.synchronize()
    del w
    nw = torch.ones(H, device=dev)
    x = torch.randn((M, H), generator=g, device=dev)
    tok = torch.empty(M, dtype=torch.int64, device=dev)
    ws = torch.empty(int(L.lib().ksh_lm_head_tc_workspace_size(M, H, V)), dtype=torch.uint8,
                     device=dev)

    def run():
        L.call("ksh_lm_head_argmax_tc", x.data_ptr(), M, H, nw.data_ptr(), 1e-6, hi.data_ptr(),
               lo.data_ptr(), inv.data_ptr(), V, None, tok.data_ptr(), ws.data_ptr(), ws.numel(), s)
    for _ in range(3):
        run()
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStart()
    run()
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStop()
    print(json.dumps({"profile": "lm_head_tc", "workload": args.workload, "rows": M,
                      "algorithmic_bytes": V * H * 4 + V * 4 + M * H * 4}))


def run_profile_decode_attention(args, wl):
    """The tensor-parallel workload's roofline kernel alone, for an ncu
    capture: one layer's block pool for ``batch`` sequences at ``context``
    earlier positions (fp32 K/V, 2.2 GB for the 8B shape at TP1) and one
    ksh_decode_attention_ws call (the model's) between
    cudaProfilerStart/Stop, after a warm-up."""
    from kshipra_b200 import _lib as L
    from kshipra_b200.config import PRESETS
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = PRESETS[wl["preset"]]
    Bt, ctx, bs = wl["batch"], wl["context"], wl["block"]
    hq, hkv, d = cfg.heads, cfg.kv_heads, cfg.head_dim
    nbs = (ctx + 1 + bs - 1) // bs
    pool = torch.empty((Bt * nbs, 1, 2, hkv, bs, d), device=dev).uniform_(-1.0, 1.0)
    bt = torch.arange(Bt * nbs, dtype=torch.int32, device=dev).view(Bt, nbs)
    g = torch.Generator(device=dev).manual_seed(0)
    qkv = torch.randn((Bt, (hq + 2 * hkv) * d), generator=g, device=dev)
    pos = torch.full((Bt,), ctx, dtype=torch.int64, device=dev)
    slots = torch.arange(Bt, dtype=torch.int64, device=dev) * nbs * bs + ctx
    ang = torch.arange(ctx + 1, device=dev, dtype=torch.float32)[:, None] * 1e-3
    rc, rs = torch.cos(ang.expand(-1, d // 2)).contiguous(), torch.sin(ang.expand(-1, d // 2)).contiguous()
    out = torch.empty((Bt, hq, d), device=dev)
    flags = torch.zeros(1, dtype=torch.int32, device=dev)
    wsz = int(L.lib().ksh_decode_attention_workspace_size(Bt, hq, hkv, d))
    dws = torch.zeros(wsz, dtype=torch.uint8, device=dev)
    s = L.stream_ptr()

    def run():
        L.call("ksh_decode_attention_ws", qkv.data_ptr(), Bt, hq, hkv, d, pos.data_ptr(),
               slots.data_ptr(), rc.data_ptr(), rs.data_ptr(), rc.shape[0], pool.data_ptr(),
               pool.shape[0], 1, 0, bs, bt.data_ptr(), nbs, ctx + 1, out.data_ptr(),
               dws.data_ptr(), wsz, flags.data_ptr(), s)
    for _ in range(3):
        run()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(10):
        run()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / 10
    torch.cuda.cudart().cudaProfilerStart()
    run()
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStop()
    if int(flags.abs().sum()):
        raise RuntimeError(f"decode attention raised flags {flags.tolist()}")
    nbytes = Bt * (ctx + 1) * 2 * hkv * d * 4 + Bt * hq * d * 8
    print(json.dumps({"profile": "decode_attention", "workload": args.workload,
                      "algorithmic_bytes": nbytes, "ms_unprofiled": ms,
                      "gb_s_unprofiled": nbytes / (ms * 1e-3) / 1e9}))


def profiled_traffic(name):
    """DRAM bytes per launch recorded in profiles/<name>.md (line
    'traffic_bytes_per_launch: N', from ncu dram__bytes_read.sum +
    dram__bytes_write.sum), or None."""
    p = os.path.join(ROOT, "profiles", name + ".md")
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.strip().startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


def run_profile(args, wl):
    """One request (chunked prefill + decode graph replays) between
    cudaProfilerStart/Stop, after a warm-up, for ncu --profile-from-start off."""
    from kshipra_b200.config import PRESETS
    from kshipra_b200.model import KshipraModel
    from kshipra_b200.weights import synthetic_state_dict
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = PRESETS[wl["preset"]]
    km = KshipraModel(config=cfg, state_dict=synthetic_state_dict(cfg, 0, dev),
                      quantize=wl["quantize"], device=dev)
    g = torch.Generator().manual_seed(0)
    prompt = torch.randint(0, cfg.vocab, (wl["prompt"],), generator=g).tolist()
    for _ in range(2):
        km.generate(prompt, wl["new"], block_size=wl["block"], prefill_chunk=wl["chunk"])
    torch.cuda.synchronize()
    if args.trace:
        # CUPTI activity trace of one request (in-graph kernel durations and
        # the idle gaps between them, which ncu's serialised replay hides).
        from torch.profiler import ProfilerActivity, profile
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            km.generate(prompt, wl["new"], block_size=wl["block"], prefill_chunk=wl["chunk"])
            torch.cuda.synchronize()
        evs = [e for e in prof.events() if e.device_type.name == "CUDA" and e.name]
        evs.sort(key=lambda e: e.time_range.start)
        # With programmatic dependent launch a kernel starts early and waits,
        # so its raw duration overlaps its predecessor.  Attribute to each
        # kernel the time it adds to the critical path: end - previous end.
        evs.sort(key=lambda e: e.time_range.end)
        agg = {}
        busy = 0.0
        prev_end = evs[0].time_range.start if evs else 0
        for e in evs:
            d = e.time_range.end - max(prev_end, e.time_range.start)
            early = prev_end - e.time_range.start        # > 0: started before its predecessor ended
            prev_end = max(prev_end, e.time_range.end)
            k = e.name.replace("void ", "").replace("ksh::(anonymous namespace)::", "")
            k = k.split("(")[0][:60]
            c, t, ea = agg.get(k, (0, 0.0, 0.0))
            agg[k] = (c + 1, t + d, ea + early)
            busy += d
        span = evs[-1].time_range.end - evs[0].time_range.start if evs else 0
        print(json.dumps({"trace": args.workload, "span_us": span, "busy_us": busy,
                          "kernels": {k: {"n": c, "total_us": t, "avg_us": t / c,
                                          "avg_early_start_us": ea / c}
                                      for k, (c, t, ea) in sorted(agg.items(),
                                                                  key=lambda x: -x[1][1])}}))
        return
    torch.cuda.cudart().cudaProfilerStart()
    toks = km.generate(prompt, wl["new"], block_size=wl["block"], prefill_chunk=wl["chunk"])
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStop()
    print(json.dumps({"profile": args.workload, "tokens": len(toks)}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="llama8b-int4", choices=sorted(WORKLOADS) + ["micro"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-replica", action="store_true",
                    help="default workload: skip the 0.5B replica figures reported beside it")
    ap.add_argument("--profile", action="store_true",
                    help="run one request inside cudaProfilerStart/Stop (for ncu)")
    ap.add_argument("--trace", action="store_true",
                    help="with --profile: CUPTI trace of one request, per-kernel summary")
    ap.add_argument("--profile-kernel", default=None,
                    choices=["lm_head", "lm_head_tc", "decode_attention"],
                    help="with --profile: only this kernel on the workload's shape (small ncu case)")
    ap.add_argument("--micro-filter", default=None,
                    help="micro workload: comma list of scheme:M:KxN points to run")
    args = ap.parse_args()
    if args.workload == "micro":
        run_micro(args)
        return
    wl = WORKLOADS[args.workload]
    if args.profile and args.profile_kernel == "lm_head":
        run_profile_lm_head(args, wl)
        return
    if args.profile and args.profile_kernel == "lm_head_tc":
        run_profile_lm_head_tc(args, wl)
        return
    if args.profile and args.profile_kernel == "decode_attention":
        run_profile_decode_attention(args, wl)
        return
    if args.profile and not wl.get("tp") and not wl.get("cb"):
        run_profile(args, wl)
        return
    if args.impl == "reference" and wl.get("attn"):
        res, rank = run_reference_attn(args, wl)
    elif args.impl == "reference":
        res, rank = run_reference(args, wl)
    elif wl.get("tp"):
        res, rank = run_tp(args, wl)
    elif wl.get("cb"):
        res, rank = run_cb(args, wl)
    elif wl.get("attn"):
        res, rank = run_attn_prefix(args, wl)
    else:
        res, rank = run_ours(args, wl)
    if rank == 0 and res is not None:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
