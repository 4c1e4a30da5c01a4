"""Sum all-reduce of the tensor-parallel partial sums over peer memory.

The row-parallel projections (o_proj, down_proj) of a tensor-parallel layer
leave each rank a partial sum of the layer output; ``PeerAllReduce`` sums
them with this library's kernel (``ksh_peer_allreduce_f32``: a reduce-scatter
and an all-gather over NVLink peer loads, two flag barriers per call, every
wait bounded) instead of an NCCL all-reduce.  The producing GEMM writes its
partial straight into this rank's slot of a symmetric-memory buffer
(``partial(n)``), so nothing is copied before the reduction.

The buffer comes from ``torch.distributed._symmetric_memory`` (allocation
and the exchange of the peers' mappings are its job; multicast objects are not
used); the per-call state (alternating buffer parity, per-CTA epochs) lives
here and in device memory, so calls can be captured in a CUDA graph.  Calls
must come in the same order on every rank, as collectives do.
"""

from __future__ import annotations

import os

import torch

from . import _lib
from ._lib import call, ptr, stream_ptr


class PeerAllReduce:
    def __init__(self, group, device: torch.device, n_max: int):
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm
        os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")
        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        self.device = device
        self.n_max = (n_max + 3) // 4 * 4
        nfl = int(_lib.lib().ksh_peer_allreduce_buffer_floats(self.n_max, self.world))
        if nfl <= 0:
            raise ValueError(f"peer all-reduce needs 1..8 ranks, got {self.world}")
        try:                        # peer mappings through the CUDA driver (no NVSHMEM here)
            symm.set_backend("CUDA")
        except Exception:
            pass
        if hasattr(symm, "enable_symm_mem_for_group"):
            try:
                symm.enable_symm_mem_for_group(self.group.group_name)
            except Exception:
                pass
        self.buf = symm.empty(nfl, dtype=torch.float32, device=device)
        self.buf.zero_()                                   # flags start at 0
        self.handle = symm.rendezvous(self.buf, self.group)
        self.peers = torch.tensor([int(p) for p in self.handle.buffer_ptrs], dtype=torch.int64,
                                  device=device)
        self.epochs = torch.zeros(int(_lib.lib().ksh_peer_allreduce_epoch_words()),
                                  dtype=torch.int32, device=device)
        self.flags = torch.zeros(1, dtype=torch.int32, device=device)
        self.parity = 0
        torch.cuda.synchronize(device)
        dist.barrier(group=self.group)                     # every rank's flags are zero

    def partial(self, n: int) -> torch.Tensor:
        """This rank's slot for the next call's partial sum (n floats)."""
        if n > self.n_max:
            raise ValueError(f"{n} floats exceed the buffer's {self.n_max}")
        o = self.parity * self.n_max
        return self.buf[o:o + n]

    def reduce(self, out: torch.Tensor, n: int) -> torch.Tensor:
        """out[:n] = sum over ranks of their ``partial(n)``; every rank gets the same bits."""
        call("ksh_peer_allreduce_f32", ptr(self.peers), self.rank, self.world, n, self.n_max,
             self.parity, ptr(out), ptr(self.epochs), ptr(self.flags), stream_ptr())
        self.parity ^= 1
        return out
