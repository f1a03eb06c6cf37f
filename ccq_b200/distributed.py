"""Multi-GPU helpers: shard the cleaning operator over ranks and reduce the gate gradients.

The operator has no data-path exchange: every (document, head) pair is
independent and the state never crosses a shard.  Ranks take whole batch rows (dense) or whole
documents (varlen, longest-processing-time-first by length), so each rank holds all heads of its
tokens and the per-head gate needs no communication.  The only collective is the sum of the
gate gradients dW [H, K] and db [H] over ranks, issued once per step after the backward.
"""
from __future__ import annotations

import heapq

import torch
import torch.distributed as dist


def shard_rows(B, world, rank):
    """Contiguous batch rows [lo, hi) of `rank` for a dense batch of B rows (B >= world)."""
    if B < world:
        raise ValueError(f'batch {B} smaller than world size {world}: shard heads instead')
    base, extra = divmod(B, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def shard_documents(lengths, world):
    """Assign documents to ranks, longest first onto the least-loaded rank (LPT).

    Returns one sorted list of document indices per rank; token counts are balanced to within
    the longest document."""
    heap = [(0, r) for r in range(world)]
    heapq.heapify(heap)
    out = [[] for _ in range(world)]
    for i in sorted(range(len(lengths)), key=lambda j: -int(lengths[j])):
        load, r = heapq.heappop(heap)
        out[r].append(i)
        heapq.heappush(heap, (load + int(lengths[i]), r))
    return [sorted(x) for x in out]


def local_cu_seqlens(lengths, docs, device=None):
    """cu_seqlens (int64) of the documents `docs` packed in order."""
    sizes = torch.tensor([0] + [int(lengths[i]) for i in docs], dtype=torch.int64)
    return torch.cumsum(sizes, 0).to(device) if device is not None else torch.cumsum(sizes, 0)


def allreduce_gate_grads(dW, db, group=None, async_op=False):
    """Sum the per-rank gate gradients over the process group (NCCL on GPUs, gloo on CPU).

    Both tensors are reduced in one flat buffer, so the step issues a single collective."""
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return None
    flat = torch.cat([dW.reshape(-1), db.reshape(-1)])
    work = dist.all_reduce(flat, group=group, async_op=True)

    def finish():
        work.wait()
        dW.copy_(flat[:dW.numel()].view_as(dW))
        db.copy_(flat[dW.numel():].view_as(db))

    if async_op:
        return finish
    finish()
    return None


class GateGradReducer:
    """Per-step sum of the gate gradients over ranks that the next step's kernels never wait for.

    The backward writes dW [H, K] and db [H] straight into one of ``depth`` flat buffers (``out()``
    gives the views to pass as its outputs); ``submit()`` starts the all-reduce of that buffer on
    NCCL's stream and returns at once.  A buffer is written again only ``depth`` steps later, after
    the compute stream has been made to wait for its previous all-reduce (long finished by then),
    and ``result()`` waits for the latest one where an optimizer would consume it.  With one rank
    nothing is communicated and ``result()`` returns the local gradients."""

    def __init__(self, H, K, device, group=None, depth=2):
        self.H, self.K, self.group = H, K, group
        self.bufs = [torch.empty(H * K + H, device=device, dtype=torch.float32) for _ in range(depth)]
        self.works = [None] * depth
        self.i = 0
        self.last = None

    def _active(self):
        return dist.is_available() and dist.is_initialized() and dist.get_world_size(self.group) > 1

    def out(self):
        """(dW, db) views of the next free buffer, for the backward to write into."""
        j = self.i % len(self.bufs)
        if self.works[j] is not None:
            self.works[j].wait()
            self.works[j] = None
        b = self.bufs[j]
        return b[:self.H * self.K].view(self.H, self.K), b[self.H * self.K:]

    def submit(self):
        """Start the sum of the buffer the backward just wrote."""
        j = self.i % len(self.bufs)
        if self._active():
            self.works[j] = dist.all_reduce(self.bufs[j], group=self.group, async_op=True)
        self.last = j
        self.i += 1

    def result(self):
        """(dW, db) summed over ranks for the latest submitted step."""
        j = self.last
        if j is None:
            return None
        if self.works[j] is not None:
            self.works[j].wait()
            self.works[j] = None
        b = self.bufs[j]
        return b[:self.H * self.K].view(self.H, self.K), b[self.H * self.K:]

    def drain(self):
        """Wait for every all-reduce still in flight (before the process group goes away)."""
        for j, w in enumerate(self.works):
            if w is not None:
                w.wait()
                self.works[j] = None
