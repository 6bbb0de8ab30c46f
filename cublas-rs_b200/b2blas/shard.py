"""Host-side partitioning for running the GEMM family on several GPUs, one
process per GPU (torch.distributed over NCCL for the plumbing).

Two strategies, neither in the reference (which is single-device,
crates/cublas-rs/src/lib.rs:57-68):

* batch sharding of strided-batched SGEMM: rank r owns a contiguous range of
  batches; independent units, no collective.
* column-block sharding of a large GEMM: A is replicated, rank r owns the
  column panel B[:, c0:c1] (k x w) and C[:, c0:c1] (m x w), stored as its own
  contiguous row-major panel.  Only when the caller asks for the full C do
  the ranks all-gather their panels (panel-major), after which
  b2b_panels_to_rowmajor lays the result out row-major -- or, fused,
  b2b_*gemm_gather writes each rank's panel straight into every rank's
  full C through the peer pointers PeerBuffers sets up.
"""
from __future__ import annotations

from typing import List, Tuple

import numpy as np


def split_range(total: int, parts: int, index: int, align: int = 1) -> Tuple[int, int]:
    """[begin, end) of part `index` when `total` items are split into `parts`
    contiguous pieces whose sizes differ by at most `align` (piece boundaries
    are multiples of `align`, except the last end)."""
    if parts <= 0 or not 0 <= index < parts:
        raise ValueError("bad partition")
    units = (total + align - 1) // align
    base, rem = divmod(units, parts)
    b = index * base + min(index, rem)
    e = b + base + (1 if index < rem else 0)
    return min(b * align, total), min(e * align, total)


def batch_shard(batch: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous batch range of `rank` for strided-batched sharding."""
    return split_range(batch, world, rank)


def column_panels(n: int, world: int, align: int = 8) -> List[int]:
    """Widths of the world column panels of an n-column C (multiples of
    `align` where possible, so every panel stays 16-byte aligned for f16)."""
    return [e - b for b, e in (split_range(n, world, r, align) for r in range(world))]


def panel_of(B: np.ndarray, k: int, n: int, c0: int, c1: int) -> np.ndarray:
    """Contiguous row-major copy of columns [c0, c1) of a row-major k x n B."""
    return np.ascontiguousarray(B.reshape(k, n)[:, c0:c1]).ravel()


def panels_to_rowmajor_host(panels: np.ndarray, m: int, widths: List[int]) -> np.ndarray:
    """Host restatement of b2b_panels_to_rowmajor: panel g (m x widths[g],
    row-major) back to back -> row-major m x sum(widths)."""
    out = np.empty((m, sum(widths)), panels.dtype)
    off = 0
    c = 0
    for w in widths:
        out[:, c:c + w] = panels[off:off + m * w].reshape(m, w)
        off += m * w
        c += w
    return out.ravel()


class PeerBuffers:
    """One library allocation per rank, mapped into every rank: after
    construction (collective over `group`), `ptrs[r]` is rank r's buffer as a
    device pointer valid in this process (CUDA IPC for the peers).  Used as
    the destinations of b2b_*gemm_gather.  Call close() (collectively) before
    the handle goes away."""

    def __init__(self, handle, length: int, dtype, group=None):
        import torch.distributed as dist

        self.handle = handle
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.buf = handle.alloc(length, dtype)
        mine = handle.ipc_get_handle(self.buf)
        handles = [None] * self.world
        dist.all_gather_object(handles, mine, group=group)
        self.ptrs = []
        for r, hd in enumerate(handles):
            self.ptrs.append(self.buf.ptr if r == self.rank else handle.ipc_open_handle(hd))

    def close(self) -> None:
        import torch.distributed as dist

        if not self.ptrs:
            return
        # Nobody may still be writing into a peer's buffer when it is unmapped
        # and freed.
        self.handle.synchronize()
        dist.barrier(group=self.group)
        for r, p in enumerate(self.ptrs):
            if r != self.rank:
                self.handle.ipc_close_handle(p)
        dist.barrier(group=self.group)
        self.buf.free()
        self.ptrs = []
