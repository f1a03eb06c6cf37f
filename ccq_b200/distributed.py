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


class _StatePrefix(torch.autograd.Function):
    """Exclusive prefix over ranks of the partial (C, m) states of a document cut by rank boundaries.

    forward: every rank contributes ``part`` (its last local document's sum of k k^T and k, flattened)
    and ``pre`` (how many earlier ranks hold the start of its first document); one all-gather; the
    result is the sum of the parts of ranks rank-pre .. rank-1 (zeros when pre is 0).
    backward: one all-gather of the gradients on those sums; a rank's part receives the gradient of
    every later rank whose sum included it.  Both passes issue exactly one collective on every rank,
    whether or not the rank itself continues a document."""

    @staticmethod
    def forward(ctx, part, group, pre):
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        buf = torch.cat([part.reshape(-1), part.new_tensor([float(pre)])])
        gathered = [torch.empty_like(buf) for _ in range(world)]
        dist.all_gather(gathered, buf, group=group)
        pres = [int(g[-1].item()) for g in gathered]
        prefix = torch.zeros_like(part)
        for r in range(rank - pre, rank):
            prefix += gathered[r][:-1].view_as(part)
        ctx.group, ctx.rank, ctx.pres, ctx.shape = group, rank, pres, part.shape
        return prefix

    @staticmethod
    def backward(ctx, dprefix):
        world = len(ctx.pres)
        dprefix = dprefix.contiguous()
        gathered = [torch.empty_like(dprefix) for _ in range(world)]
        dist.all_gather(gathered, dprefix, group=ctx.group)
        dpart = torch.zeros_like(dprefix)
        for r in range(ctx.rank + 1, world):
            if r - ctx.pres[r] <= ctx.rank:
                dpart += gathered[r]
        return dpart, None, None


def cp_clean_read(q, k, lambda_h, cp_context, *, l2norm_qk=False, position_offset=0, initial_cov_state=None,
                  initial_mean_state=None, output_final_state=False, subtract_mean=True, clean_fn=None):
    """The cleaning operator under fla's context parallelism: each rank holds a contiguous slice of a
    packed varlen batch (``cp_context`` from ``fla.ops.cp.build_cp_context``), and a document cut by a
    rank boundary continues on the next rank with the running (C, m) state and positions it would
    have had on one GPU.  The reference's chunk path has no such exchange: its cleaning restarts the
    state at every rank boundary.

    The exchange is an exclusive prefix over ranks of (C, m) (``_StatePrefix``): each rank sums
    k k^T and k over its LAST local document (the one later ranks continue), and a rank whose first
    document started earlier (``cp_context.pre_num_ranks`` > 0) starts it from the sum of its
    predecessors' partial states, at position offset ``cp_context.pre_num_conv_tokens`` (the
    document's tokens on earlier ranks).  Autograd carries the gradient of that starting state back
    to the ranks whose keys formed it.

    q, k: [1, T_local, H, K] (raw when ``l2norm_qk``: normalised here, fla's l2norm, eps 1e-6).
    Returns (q_clean, k as the backbone reads it, final_cov [n_local, H, K, K] | None,
    final_mean | None).  ``clean_fn`` is the per-rank operator (default: this library's
    fused_ccq_clean_read); tests pass a CPU restatement to check the exchange on gloo ranks."""
    from . import ops
    if clean_fn is None:
        clean_fn = ops.fused_ccq_clean_read
    if initial_cov_state is not None or initial_mean_state is not None:
        raise NotImplementedError('context-parallel cleaning starts from zero states (no cache)')
    group = cp_context.group
    cu = cp_context.cu_seqlens_cpu
    if cu is None:
        cu = cp_context.cu_seqlens.cpu()
    cu = [int(x) for x in cu.tolist()]
    n_local = len(cu) - 1
    H, K = q.shape[2], q.shape[3]
    if l2norm_qk:
        q = ops.l2norm(q, eps=1e-6)
        k = ops.l2norm(k, eps=1e-6)
    # partial state of this rank's last local document; the prefix of the ranks before this one
    k_last = k[0, cu[-2]:cu[-1]].to(torch.promote_types(k.dtype, torch.float32))  # fp32 states (fp64 stays)
    part = torch.cat([torch.einsum('thk,thv->hkv', k_last, k_last).reshape(-1), k_last.sum(0).reshape(-1)])
    pre = int(cp_context.pre_num_ranks or 0)
    prefix = _StatePrefix.apply(part, group, pre)
    h0 = prefix[:H * K * K].view(1, H, K, K)
    m0 = prefix[H * K * K:].view(1, H, K) if subtract_mean else None
    off_first = position_offset + (int(cp_context.pre_num_conv_tokens or 0) if pre > 0 else 0)
    dev = q.device

    def call(lo, hi, cu_part, off, s0, s1):
        cut = torch.tensor(cu_part, dtype=torch.int64, device=dev)
        return clean_fn(q[:, lo:hi], k[:, lo:hi], _lambda_slice(lambda_h, lo, hi), position_offset=off,
                        initial_cov_state=s0, initial_mean_state=s1, output_final_state=output_final_state,
                        subtract_mean=subtract_mean, cu_seqlens=cut)

    # the first local document always takes the (possibly zero) prefix, so every rank's backward
    # reaches the exchange's collective
    outs = [call(cu[0], cu[1], [0, cu[1] - cu[0]], off_first, h0, m0)]
    if n_local > 1:
        outs.append(call(cu[1], cu[-1], [c - cu[1] for c in cu[1:]], position_offset, None, None))
    q_clean = torch.cat([o[0] for o in outs], dim=1) if len(outs) > 1 else outs[0][0]
    fc = fm = None
    if output_final_state:
        fc = torch.cat([o[1] for o in outs], dim=0)
        if subtract_mean:
            fm = torch.cat([o[2] for o in outs], dim=0)
    return q_clean, k, fc, fm


def _lambda_slice(lam, lo, hi):
    """lambda restricted to tokens [lo, hi) when it is per token ([1, T, H] or [1, T, H, 1])."""
    if isinstance(lam, torch.Tensor) and lam.ndim >= 3:
        return lam[:, lo:hi]
    return lam
