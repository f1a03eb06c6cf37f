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
