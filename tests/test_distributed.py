"""Sharding and the gate-gradient all-reduce on CPU ranks (gloo, world size 2)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from ccq_b200.distributed import allreduce_gate_grads, local_cu_seqlens, shard_documents, shard_rows
from oracle import ccq_oracle as O


def test_shard_rows_cover_batch():
    for B in (8, 9, 13, 64):
        for world in (1, 2, 4, 8):
            if B < world:
                continue
            parts = [shard_rows(B, world, r) for r in range(world)]
            assert parts[0][0] == 0 and parts[-1][1] == B
            assert all(parts[i][1] == parts[i + 1][0] for i in range(world - 1))
            sizes = [hi - lo for lo, hi in parts]
            assert max(sizes) - min(sizes) <= 1


def test_shard_documents_lpt_balance():
    rng = np.random.default_rng(0)
    lengths = rng.integers(128, 8193, size=32)
    for world in (2, 4, 8):
        docs = shard_documents(lengths, world)
        assert sorted(i for d in docs for i in d) == list(range(32))
        loads = [sum(int(lengths[i]) for i in d) for d in docs]
        assert max(loads) - min(loads) <= int(lengths.max())
        cu = local_cu_seqlens(lengths, docs[0])
        assert int(cu[-1]) == loads[0]


def _free_port():
    s = socket.socket()
    s.bind(('127.0.0.1', 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out):
    import torch.distributed as dist
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=world)
    try:
        # each rank computes the gate gradients of its batch shard with the oracle
        rng = np.random.default_rng(0)
        B, T, H, K = 4, 50, 2, 8
        q = rng.standard_normal((B, T, H, K))
        q /= np.linalg.norm(q, axis=-1, keepdims=True)
        k = rng.standard_normal((B, T, H, K))
        k /= np.linalg.norm(k, axis=-1, keepdims=True)
        W, b = rng.normal(0, 0.1, (H, K)), rng.uniform(-1, 1, H)
        g = rng.standard_normal((B, T, H, K))
        lo, hi = shard_rows(B, world, rank)
        lam = O.lambda_headwise_fwd(q[lo:hi], W, b)
        _, _, dl, _, _ = O.clean_read_bwd(q[lo:hi], k[lo:hi], lam, g[lo:hi])
        _, dW, db = O.lambda_headwise_bwd(q[lo:hi], W, lam, dl)
        dWt, dbt = torch.tensor(dW), torch.tensor(db)
        allreduce_gate_grads(dWt, dbt)
        out[rank] = (dWt.numpy(), dbt.numpy())
    finally:
        dist.destroy_process_group()


def test_gate_grad_allreduce_matches_single_process():
    world = 2
    port = _free_port()
    ctx = mp.get_context('spawn')
    mgr = ctx.Manager()
    out = mgr.dict()
    procs = [ctx.Process(target=_worker, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    rng = np.random.default_rng(0)
    B, T, H, K = 4, 50, 2, 8
    q = rng.standard_normal((B, T, H, K))
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    k = rng.standard_normal((B, T, H, K))
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    W, b = rng.normal(0, 0.1, (H, K)), rng.uniform(-1, 1, H)
    g = rng.standard_normal((B, T, H, K))
    lam = O.lambda_headwise_fwd(q, W, b)
    _, _, dl, _, _ = O.clean_read_bwd(q, k, lam, g)
    _, dW, db = O.lambda_headwise_bwd(q, W, lam, dl)
    for r in range(world):
        assert np.allclose(out[r][0], dW, atol=1e-10)
        assert np.allclose(out[r][1], db, atol=1e-10)


def _reducer_worker(rank, world, port, out):
    import torch.distributed as dist

    from ccq_b200.distributed import GateGradReducer
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=world)
    try:
        H, K = 3, 4
        red = GateGradReducer(H, K, torch.device('cpu'), depth=2)
        got = []
        for step in range(5):
            dW, db = red.out()  # the backward writes its gate gradients into these views
            dW.copy_(torch.full((H, K), float(10 * step + rank)))
            db.copy_(torch.arange(H, dtype=torch.float32) + 100 * step + rank)
            red.submit()
            if step % 2 == 1:  # consume every other step, as an optimizer a step late would
                rW, rb = red.result()
                got.append((step, rW.clone().numpy(), rb.clone().numpy()))
        rW, rb = red.result()
        got.append((4, rW.clone().numpy(), rb.clone().numpy()))
        red.drain()
        out[rank] = got
    finally:
        dist.destroy_process_group()


def test_gate_grad_reducer_double_buffered_sums():
    world = 2
    port = _free_port()
    ctx = mp.get_context('spawn')
    mgr = ctx.Manager()
    out = mgr.dict()
    procs = [ctx.Process(target=_reducer_worker, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    H, K = 3, 4
    for r in range(world):
        for step, W, b in out[r]:
            assert np.allclose(W, np.full((H, K), sum(10 * step + q for q in range(world))))
            assert np.allclose(b, sum(np.arange(H) + 100 * step + q for q in range(world)))
