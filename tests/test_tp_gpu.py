"""Tensor parallelism on real GPUs: one NCCL rank per GPU (needs >= 2 GPUs;
skipped otherwise).

The sharded model must give the unsharded model's greedy tokens (CUDA-graph
decode with the all-reduces inside) and its logits within the 1e-3 relative
bound: the row-parallel partial sums are added in a different order, which
only moves the fp32 rounding.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cases():
    from kshipra_b200.config import LLAMA3_8B, TINY_LLAMA, truncated
    return [("tiny", TINY_LLAMA, "int8", 40, 12), ("8b-2l", truncated(LLAMA3_8B, 2), "int4", 48, 6)]


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    import datetime
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    try:
        from kshipra_b200.model import KshipraModel
        from kshipra_b200.weights import synthetic_state_dict
        res = {}
        for name, cfg, q, plen, new in _cases():
            sd = synthetic_state_dict(cfg, seed=0, device=dev)
            prompt = torch.randint(0, cfg.vocab, (plen,),
                                   generator=torch.Generator().manual_seed(7)).tolist()
            tp = KshipraModel(config=cfg, state_dict=sd, quantize=q, device=dev,
                              tp=(rank, world, None))
            toks = tp.generate(prompt, max_new_tokens=new, block_size=16)
            alloc = tp.new_pool(8, 16)
            ids = torch.tensor([prompt[:16]])
            lg = tp.forward(ids, torch.arange(16).view(1, -1), alloc.pool, list(range(8)),
                            list(range(16)), 0)[0].cpu()
            tp._gen_cache.clear()                      # release graphs holding NCCL calls
            del tp
            if rank == 0:
                solo = KshipraModel(config=cfg, state_dict=sd, quantize=q, device=dev)
                ref_toks = solo.generate(prompt, max_new_tokens=new, block_size=16)
                alloc1 = solo.new_pool(8, 16)
                ref_lg = solo.forward(ids, torch.arange(16).view(1, -1), alloc1.pool,
                                      list(range(8)), list(range(16)), 0)[0].cpu()
                err = float((lg - ref_lg).abs().max() / ref_lg.abs().max())
                res[name] = (toks, ref_toks, err)
                del solo
            del sd
            torch.cuda.synchronize()
            dist.barrier()
        if rank == 0:
            out.update(res)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_tensor_parallel_two_gpus_matches_single_gpu():
    out = mp.get_context("spawn").Manager().dict()
    mp.spawn(_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    assert set(out.keys()) == {name for name, *_ in _cases()}
    for name, (toks, ref, err) in out.items():
        assert toks == ref, (name, toks, ref)
        assert err < 1e-3, (name, err)
