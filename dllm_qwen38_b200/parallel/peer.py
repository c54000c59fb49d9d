"""Symmetric peer memory for the ranks of one node (NVLink / NVSwitch) and its collectives.

`SymmetricHeap` allocates one device region of the same size on every rank, exchanges CUDA IPC
handles once through the process group, and maps every peer's region. Objects are carved out by
`alloc` in the same order on every rank, so an object at byte offset `o` of the heap is at
`ptrs[r] + o` on rank r. The collectives are single launches of this repository's kernels that
read peers' memory directly (csrc/peer.cu):

  all_gather(off, shard_bytes, out, epoch)      parameter shards -> full buffer, after every
                                                peer published parameter epoch >= `epoch`
  reduce_scatter(off, shard, in_f32, out, ...)  fp32 (1/world)-averaged shard of a flat gradient
                                                with its sum of squares, fused
  allreduce_f32(vals, out)                      a few floats, summed in rank order
  publish_epoch(e)                              tell peers this rank's shards are at epoch e

This is the B200 counterpart of the reference's NCCL collectives C2/C3/C6
(`fsdp_train.py:133-171,224-252`); the reference itself only calls NCCL through FSDP2.
"""

from __future__ import annotations

import os

import torch
import torch.distributed as dist

from ..ops import _native


def _count() -> None:
    from ..ops import cuda

    cuda.LAUNCHES[0] += 1


HEADER_BYTES = 64 * 1024
SLOT_EPOCH = 0


def _timeout_s() -> float:
    return float(os.environ.get("BDLLM_PEER_TIMEOUT_S", "60"))


class SymmetricHeap:
    def __init__(self, nbytes: int, device: torch.device, group=None):
        C = _native.require()
        self.C = C
        self.device = torch.device(device)
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 16:
            raise ValueError("SymmetricHeap: at most 16 ranks (one node)")
        self.nbytes = HEADER_BYTES + ((int(nbytes) + 4095) // 4096) * 4096
        with torch.cuda.device(self.device):
            self.base = C.peer_alloc(self.nbytes)
            handle = C.peer_handle(self.base)
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle.numpy().tobytes()), group=group)
            self.ptrs = []
            for r, h in enumerate(handles):
                if r == self.rank:
                    self.ptrs.append(self.base)
                else:
                    self.ptrs.append(C.peer_open(torch.frombuffer(bytearray(h), dtype=torch.uint8)))
        self.off = HEADER_BYTES
        self.rs_seq = 0
        self.ar_seq = 0
        self.epoch = 0
        self.timeout = _timeout_s()
        self._like = {}

    # ------------------------------------------------------------------ allocation
    def alloc(self, numel: int, dtype: torch.dtype) -> tuple[torch.Tensor, int]:
        """A zero-initialised tensor of `numel` elements in the heap and its byte offset."""
        like = self._like.get(dtype)
        if like is None:
            like = self._like[dtype] = torch.empty(0, dtype=dtype, device=self.device)
        esz = like.element_size()
        off = (self.off + 255) // 256 * 256
        end = off + numel * esz
        if end > self.nbytes:
            raise MemoryError(f"SymmetricHeap: {end} bytes needed, {self.nbytes} reserved")
        self.off = end
        return self.C.peer_view(self.base + off, numel, like), off

    # ------------------------------------------------------------------ collectives
    def all_gather(self, off: int, shard_bytes: int, out: torch.Tensor, epoch: int | None = None,
                   max_blocks: int = 148) -> None:
        self.C.peer_all_gather(self.ptrs, self.rank, off, shard_bytes, out,
                               self.epoch if epoch is None else epoch, max_blocks, self.timeout)
        _count()

    def gather_range(self, off: int, shard_bytes: int, out: torch.Tensor, lo: int, hi: int,
                     epoch: int | None = None) -> None:
        """Bytes [lo, hi) of the gathered buffer (rounded out to 16 bytes) from the owning shards."""
        self.C.peer_gather_range(self.ptrs, self.rank, off, shard_bytes, out, lo, hi,
                                 self.epoch if epoch is None else epoch, self.timeout)
        _count()

    def reduce_scatter(self, off: int, shard: int, in_f32: bool, out: torch.Tensor, scale: float,
                       sq: torch.Tensor | None = None, max_blocks: int = 64, adam=None) -> None:
        """adam = ((master, m, v, p_bf16), (lr, b1, b2, eps, wd, bc1, bc2)) applies AdamW to the
        reduced gradient in the same launch (no clipping: the gradient is not stored)."""
        self.rs_seq += 1
        st, hp = adam if adam is not None else ((), ())
        self.C.peer_reduce_scatter(self.ptrs, self.rank, off, shard, in_f32, out, scale, sq, self.rs_seq,
                                   max_blocks, self.timeout, list(st), [float(x) for x in hp])
        _count()

    def allreduce_f32(self, vals: torch.Tensor, out: torch.Tensor) -> None:
        self.ar_seq += 1
        self.C.peer_allreduce_f32(self.ptrs, self.rank, vals, out, self.ar_seq, self.timeout)
        _count()

    def publish_epoch(self, epoch: int) -> None:
        self.epoch = epoch
        self.C.peer_signal(self.ptrs, self.rank, SLOT_EPOCH, epoch)
        _count()

    def close(self) -> None:
        """Unmap peers and free the heap (call after every kernel using it has finished)."""
        if self.base is None:
            return
        torch.cuda.synchronize(self.device)
        for r, p in enumerate(self.ptrs):
            if r != self.rank:
                self.C.peer_close(p)
        dist.barrier()  # no peer still maps this heap
        self.C.peer_release(self.base)
        self.base = None
