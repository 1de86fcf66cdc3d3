"""One-shot all-reduce over NVLink peer memory for tensor parallelism.

Each rank allocates a data buffer (two slots) and a flag array, shares them
with the other ranks of the process group through CUDA IPC (torch's storage
sharing, the mechanism torch.multiprocessing uses for CUDA tensors), and maps
the peers' buffers; ``PeerAllReduce(t)`` then sums ``t`` over the ranks in
one kernel (gdsq_allreduce_sum_f16): stage the local slice, release-store an
epoch flag into every peer, wait for the peers' flags, add all ranks' slices
in rank order.  It replaces the NCCL all-reduce after the row-split o and
down projections (gdsllm_b200.tp); every rank must make the same sequence of
calls, as with any collective.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch
import torch.distributed as dist

from ._native import check, lib

MAX_RANKS = 8
MAX_CTAS = 32


class PeerAllReduce:
    def __init__(self, capacity: int, group: Optional[dist.ProcessGroup] = None, device=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > MAX_RANKS:
            raise ValueError(f"{self.world} ranks: at most {MAX_RANKS}")
        self.cap = (capacity + 7) // 8 * 8
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.data = torch.zeros(2 * self.cap, dtype=torch.float16, device=self.device)
        self.flags = torch.zeros(MAX_CTAS * MAX_RANKS, dtype=torch.int32, device=self.device)
        torch.cuda.synchronize(self.device)
        mine = (self.data.untyped_storage()._share_cuda_(), self.flags.untyped_storage()._share_cuda_())
        gathered = [None] * self.world
        dist.all_gather_object(gathered, mine, group=group)
        self._peer_storages = []
        bufs, flags = [], []
        me = self.device.index
        for r, (hd, hf) in enumerate(gathered):
            if r == self.rank:
                bufs.append(self.data.data_ptr())
                flags.append(self.flags.data_ptr())
                continue
            if hd[0] != me and not torch.cuda.can_device_access_peer(me, hd[0]):
                raise RuntimeError(f"GPU {me} cannot access GPU {hd[0]}'s memory (no peer access)")
            # Open the peer's allocation with this rank's own device current (the
            # first tuple entry selects the device whose context maps it): the
            # kernel runs on this device, and the runtime enables peer access
            # from here to the owner lazily when it maps the handle.
            sd = torch.UntypedStorage._new_shared_cuda(me, *hd[1:])
            sf = torch.UntypedStorage._new_shared_cuda(me, *hf[1:])
            self._peer_storages += [sd, sf]
            bufs.append(sd.data_ptr())
            flags.append(sf.data_ptr())
        self._bufs = (ctypes.c_void_p * self.world)(*bufs)
        self._flags = (ctypes.c_void_p * self.world)(*flags)
        dist.barrier(group=group)

    def __call__(self, t: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Sum of ``t`` (fp16, contiguous, numel % 8 == 0) over the ranks;
        in place unless ``out`` is given."""
        out = t if out is None else out
        stream = torch.cuda.current_stream(t.device).cuda_stream
        check(lib().gdsq_allreduce_sum_f16(t.data_ptr(), out.data_ptr(), t.numel(), self._bufs, self._flags,
                                           self.cap, self.rank, self.world, stream), "gdsq_allreduce_sum_f16")
        return out

    def close(self):
        self._peer_storages = []
