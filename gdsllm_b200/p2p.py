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


class PeerBuffers:
    """A device data buffer and an int32 flag array per rank, shared with every
    rank of the group through CUDA IPC.  ``bufs`` / ``flags`` are ctypes
    arrays of the ranks' device pointers as mapped into this process."""

    def __init__(self, data_bytes: int, flag_count: int, group: Optional[dist.ProcessGroup] = None,
                 device=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > MAX_RANKS:
            raise ValueError(f"{self.world} ranks: at most {MAX_RANKS}")
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.data = torch.zeros((data_bytes + 15) // 16 * 16, dtype=torch.uint8, device=self.device)
        self.flags_t = torch.zeros(flag_count, dtype=torch.int32, device=self.device)
        torch.cuda.synchronize(self.device)
        mine = (self.data.untyped_storage()._share_cuda_(), self.flags_t.untyped_storage()._share_cuda_())
        gathered = [None] * self.world
        dist.all_gather_object(gathered, mine, group=group)
        self._peer_storages = []
        bufs, flags = [], []
        me = self.device.index
        for r, (hd, hf) in enumerate(gathered):
            if r == self.rank:
                bufs.append(self.data.data_ptr())
                flags.append(self.flags_t.data_ptr())
                continue
            if hd[0] != me and not torch.cuda.can_device_access_peer(me, hd[0]):
                raise RuntimeError(f"GPU {me} cannot access GPU {hd[0]}'s memory (no peer access)")
            # Open the peer's allocation with this rank's own device current (the
            # first tuple entry selects the device whose context maps it): the
            # kernels run on this device, and the runtime enables peer access
            # from here to the owner lazily when it maps the handle.
            sd = torch.UntypedStorage._new_shared_cuda(me, *hd[1:])
            sf = torch.UntypedStorage._new_shared_cuda(me, *hf[1:])
            self._peer_storages += [sd, sf]
            bufs.append(sd.data_ptr())
            flags.append(sf.data_ptr())
        self.bufs = (ctypes.c_void_p * self.world)(*bufs)
        self.flags = (ctypes.c_void_p * self.world)(*flags)
        dist.barrier(group=group)

    def close(self):
        self._peer_storages = []


class PeerAllReduce:
    """One-shot sum of a fp16 vector over the ranks (gdsq_allreduce_sum_f16)."""

    def __init__(self, capacity: int, group: Optional[dist.ProcessGroup] = None, device=None):
        self.cap = (capacity + 7) // 8 * 8
        self.peer = PeerBuffers(2 * self.cap * 2, MAX_CTAS * MAX_RANKS, group, device)
        self.rank, self.world = self.peer.rank, self.peer.world

    def __call__(self, t: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Sum of ``t`` (fp16, contiguous, numel % 8 == 0) over the ranks;
        in place unless ``out`` is given."""
        out = t if out is None else out
        stream = torch.cuda.current_stream(t.device).cuda_stream
        check(lib().gdsq_allreduce_sum_f16(t.data_ptr(), out.data_ptr(), t.numel(), self.peer.bufs, self.peer.flags,
                                           self.cap, self.rank, self.world, stream), "gdsq_allreduce_sum_f16")
        return out

    def close(self):
        self.peer.close()


WORDS_MAX_ELEMS = 32768
WORDS_EPOCHS = 32  # one int per CTA of the word all-reduce


class PeerWordAllReduce:
    """One-shot sum of an fp16 or fp32 vector over the ranks with (value,
    epoch) 64-bit words (gdsq_allreduce_sum_words): every rank stores its
    elements into every rank's buffer and waits only on its own."""

    def __init__(self, capacity: int, group: Optional[dist.ProcessGroup] = None, device=None):
        if capacity > WORDS_MAX_ELEMS:
            raise ValueError(f"capacity {capacity}: at most {WORDS_MAX_ELEMS} elements")
        self.cap = capacity
        world = dist.get_world_size(group)
        # the flag array doubles as this rank's per-CTA epochs (never read by the peers)
        self.peer = PeerBuffers(2 * world * self.cap * 8, WORDS_EPOCHS, group, device)
        self.rank, self.world = self.peer.rank, self.peer.world

    # fp32 in, fp16 out (the sum clamped to the fp16 range) in one kernel
    finishes_fp16 = True

    def __call__(self, t: torch.Tensor, out: Optional[torch.Tensor] = None,
                 residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Sum of ``t`` (fp16 or fp32, contiguous) over the ranks; in place
        unless ``out`` is given.  fp32 ``t`` with an fp16 ``out`` gives the
        sum clamped to +-65504 and rounded to fp16 (``moe.finish``), plus
        ``residual`` (fp16) in fp16 when given."""
        out = t if out is None else out
        if t.dtype == torch.float32 and out.dtype == torch.float16:
            kind = 2
        else:
            if out.dtype != t.dtype:
                raise ValueError(f"allreduce words: {t.dtype} in, {out.dtype} out")
            kind = {torch.float16: 0, torch.float32: 1}[t.dtype]
        if residual is not None and (kind != 2 or residual.dtype != torch.float16 or
                                     residual.numel() != t.numel()):
            raise ValueError("allreduce words: a residual needs fp32 in, fp16 out and fp16 residual of the same size")
        stream = torch.cuda.current_stream(t.device).cuda_stream
        check(lib().gdsq_allreduce_sum_words_residual(kind, t.data_ptr(), out.data_ptr(), t.numel(), self.peer.bufs,
                                                      self.peer.flags_t.data_ptr(), self.cap, self.rank, self.world,
                                                      None if residual is None else residual.data_ptr(), stream),
              "gdsq_allreduce_sum_words_residual")
        return out

    def close(self):
        self.peer.close()


TP_MAX_ROW_GROUPS = 1024
TP_FLAG_INTS = 64  # call epoch and finisher count (local only)


class PeerRowGemv:
    """Row-split GGUF GEMV with the all-reduce inside the kernel's epilogue
    (gdsq_fused_gemv_allreduce): y [1, n] = sum over ranks of W_r . x_r."""

    def __init__(self, max_rows: int, group: Optional[dist.ProcessGroup] = None, device=None):
        self.rows = (max_rows + 31) // 32 * 32
        if self.rows // 32 > TP_MAX_ROW_GROUPS:
            raise ValueError(f"{max_rows} rows: at most {TP_MAX_ROW_GROUPS * 32}")
        world = dist.get_world_size(group)
        # [2 slots][world][rows] 64-bit (fp32 partial row, call epoch) words: every
        # rank stores its rows into every rank's buffer
        self.peer = PeerBuffers(2 * world * self.rows * 8, TP_FLAG_INTS, group, device)
        self.rank, self.world = self.peer.rank, self.peer.world

    def __call__(self, fmt: str, w: torch.Tensor, x_local: torch.Tensor, n: int, k_local: int,
                 out: Optional[torch.Tensor] = None) -> torch.Tensor:
        if out is None:
            out = torch.empty(1, n, dtype=torch.float16, device=x_local.device)
        stream = torch.cuda.current_stream(x_local.device).cuda_stream
        check(lib().gdsq_fused_gemv_allreduce(0 if fmt == "q4_0" else 1, w.data_ptr(), x_local.data_ptr(),
                                              out.data_ptr(), n, k_local, self.peer.bufs, self.peer.flags,
                                              self.rows, self.rank, self.world, stream), "gdsq_fused_gemv_allreduce")
        return out

    def close(self):
        self.peer.close()
