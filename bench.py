#!/usr/bin/env python
"""Benchmark of the B200 CCQ cleaning operator: forward + backward throughput (tokens/s).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload c2|c4]

Workload c2 (default): per GPU B=8, T=4096, H=16, d_k=128, bf16 inputs with
fp32 accumulation; q, k ~ N(0,1) L2-normalised per head; lambda = sigmoid(W q + b) with the
per-head W_lambda (H x d_k) ~ N(0, 0.02) and b ~ U(-1, 1) fused into the kernels; upstream grad
~ N(0,1).  One step = forward + backward of the operator (q_clean, dq, dk, dW, db); with N > 1
ranks each rank runs its own batch shard (weak scaling) and dW/db are all-reduced over NCCL.
Workload c4: one decode step, batch 256, H=16, d_k=128, fp32 cache state.

Rank 0 prints one JSON line.  ``--impl reference`` times the CPU restatement of the operator
(the reference ships no CPU path; see oracle/ccq_torch_port.py) on a bounded sample instead.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

# algorithmic work per token-head at K=128, BT=64 (fwd 4K^2+4BT K, bwd 8K^2+12BT K, dense gate 6K)
FWD_BYTES_PER_TH = 768      # q, k read + q_clean write (bf16)
BWD_BYTES_PER_TH = 1280     # q, k, dq_clean read + dq, dk write (bf16)
FLOP_PER_TH = 339968
# DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) from one ncu capture of each
# kernel at c2; profiles/tc_fwd_kernel_c2.md and profiles/tc_bwd_kernel_c2.md give the command.
NCU_TRAFFIC_C2 = {'fwd': 270.7e6 + 108.9e6, 'bwd': 415.5e6 + 233.6e6}
NCU_TRAFFIC_C4 = 272.7e6 + 213.9e6  # decode_kernel, profiles/decode_kernel_c4.md
DECODE_BYTES_PER_TH = 2 * 128 * 128 * 4 + 2 * 128 * 4 + 4 * 128 * 2 + 2 * 2


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=200)
    ap.add_argument('--warmup', type=int, default=5)
    ap.add_argument('--impl', default='ours', choices=['ours', 'reference'])
    ap.add_argument('--workload', default='c2', choices=['c2', 'c4'])
    ap.add_argument('--e2e-steps', type=int, default=10)
    ap.add_argument('--no-cpu-baseline', action='store_true')
    return ap.parse_args()


def peaks():
    path = os.path.join(ROOT, 'MEASURED_PEAKS.json')
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p['hbm_gbs']), float(p['bf16_tflops']), 'measured'
    except Exception:
        return 6650.0, 1590.0, 'fallback'


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms while active."""

    FIELDS = ('index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,'
              'clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,'
              'clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap')

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(['nvidia-smi', '-i', str(self.index), f'--query-gpu={self.FIELDS}',
                                          '--format=csv,noheader,nounits', '-lms', '200'],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        time.sleep(0.25)
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap']
        for line in self.lines:
            parts = [p.strip() for p in line.split(',')]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, val in zip(names, parts[5:9]):
                if val.lower().startswith('active'):
                    reasons.add(nm)
        return {'sm_mhz': statistics.median(sm) if sm else None, 'sm_max_mhz': mx,
                'reasons': sorted(reasons), 'samples': len(sm)}


def unit(gen, shape, device, dtype):
    import torch
    x = torch.randn(shape, generator=gen, device=device, dtype=torch.float32)
    return (x / x.norm(dim=-1, keepdim=True)).to(dtype)


def cpu_port_sample(T=4096, Hs=2, K=128, reps=3, warm=1):
    """The CPU restatement (torch fp32, chunked, autograd) on B=1 x Hs heads of a T-token batch row.

    Returns (tokens/s for the full H=16 head set, seconds per sample, threads)."""
    import torch
    from oracle import ccq_torch_port as P
    g = torch.Generator().manual_seed(0)
    q = torch.randn(1, T, Hs, K, generator=g)
    q = q / q.norm(dim=-1, keepdim=True)
    k = torch.randn(1, T, Hs, K, generator=g)
    k = k / k.norm(dim=-1, keepdim=True)
    W = torch.randn(Hs, K, generator=g) * 0.02
    b = torch.rand(Hs, generator=g) * 2 - 1
    dqc = torch.randn(1, T, Hs, K, generator=g)
    for _ in range(warm):
        P.clean_step_fwd_bwd(q, k, W, b, dqc)
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        P.clean_step_fwd_bwd(q, k, W, b, dqc)
        times.append(time.perf_counter() - t0)
    t = min(times)
    return T * Hs / 16 / t, t, torch.get_num_threads()


C2_METRIC = 'CCQ clean fwd+bwd tokens/s/GPU (bf16, T=4096,H=16,dk=128) and % roofline'


def c2_config(world, B=8, T=4096, H=16, K=128):
    """The c2 workload description shared by both arms of the bench."""
    return {'workload': 'c2: B=8/GPU,T=4096,H=16,d_k=128 cleaning fwd+bwd, per-head gate fused',
            'global_batch': B * world, 'seq_len': T, 'heads': H, 'd_k': K,
            'parallelism': f'dp{world} (batch shards, NCCL all-reduce of dW,db)',
            'l2': 'inputs larger than L2 (q,k,dq_clean 384 MiB per GPU)'}


def run_reference(args, rank, world):
    """CPU restatement timed on the host cores (rank 0 only)."""
    if rank != 0:
        return
    import torch
    torch.set_num_threads(os.cpu_count() or 1)
    T, Hs = 4096, 2
    tps_list = []
    for i in range(args.warmup + args.steps):
        tps, t, thr = cpu_port_sample(T=T, Hs=Hs, reps=1, warm=0)
        if i >= args.warmup:
            tps_list.append(tps)
    value = statistics.median(tps_list) if tps_list else None
    sample = f'B=1,T={T},H={Hs} of 16 heads per step (fp32 torch restatement, chunk 64, autograd); tokens/s scaled by {Hs}/16'
    line = {
        'impl': 'reference', 'metric': C2_METRIC,
        'value': value, 'unit': 'tokens/s', 'n_gpus': world, 'steps': args.steps, 'warmup': args.warmup,
        'ms_per_step': 32768 / value * 1e3 if value else None, 'higher_is_better': True, 'scaling': 'weak',
        'vs_baseline': None, 'dtype': 'f32', 'data': 'synthetic',
        'config': c2_config(world),
        'cpu_baseline': {'value': value, 'unit': 'tokens/s', 'cores': thr, 'kind': 'port', 'sample': sample},
        'e2e': {'value': value, 'unit': 'tokens/s', 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    import ccq_b200
    from ccq_b200 import _lib, ops
    from ccq_b200.distributed import allreduce_gate_grads

    device = torch.device('cuda', local_rank)
    torch.cuda.set_device(device)
    _lib.load()
    hbm_peak, tf_peak, peak_kind = peaks()

    if args.workload == 'c4':
        return run_decode(args, rank, world, device, hbm_peak, peak_kind)

    B, T, H, K = 8, 4096, 16, 128
    gen = torch.Generator(device=device).manual_seed(1000 + rank)
    q = unit(gen, (B, T, H, K), device, torch.bfloat16)
    k = unit(gen, (B, T, H, K), device, torch.bfloat16)
    W = torch.randn(H, K, generator=gen, device=device) * 0.02
    bias = torch.rand(H, generator=gen, device=device) * 2 - 1
    dqc = torch.randn(B, T, H, K, generator=gen, device=device).to(torch.bfloat16)
    N = B

    def fwd():
        return ops.clean_fwd_raw(q, k, None, W, bias, 0, None, None, True, None, N)

    def bwd(fc, fm, aux):
        return ops.clean_bwd_raw(q, k, None, W, bias, 0, None, None, True, None, N, fc, fm, aux, dqc, None, None)

    def allreduce(dW, db):
        if world > 1:
            allreduce_gate_grads(dW, db)

    # Each step's gate-gradient all-reduce runs on NCCL's stream and is joined after the next step's
    # kernels are queued (the overlap a training loop gets); the last one is joined inside the timed
    # region.
    pending = []

    def allreduce_async(dW, db):
        if world > 1:
            pending.append(allreduce_gate_grads(dW, db, async_op=True))

    def join(keep=0):
        while len(pending) > keep:
            pending.pop(0)()

    stream = torch.cuda.current_stream(device)
    for _ in range(args.warmup):
        qc, fc, fm, aux = fwd()
        dq, dk, (dW, db), _, _ = bwd(fc, fm, aux)
        join()
        allreduce_async(dW, db)
    join()
    path_fwd = path_bwd = None
    n_launch = 0
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True),
           torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    with ClockSampler(local_rank) as clocks:
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        t_start.record(stream)
        for i in range(args.steps):
            e0, e1, e2 = ev[i]
            e0.record(stream)
            qc, fc, fm, aux = fwd()
            if path_fwd is None:
                path_fwd = _lib.last_path()
            n_launch += _lib.last_launch_count()
            e1.record(stream)
            dq, dk, (dW, db), _, _ = bwd(fc, fm, aux)
            if path_bwd is None:
                path_bwd = _lib.last_path()
            n_launch += _lib.last_launch_count()
            e2.record(stream)
            join()
            allreduce_async(dW, db)
        join()
        t_end.record(stream)
        torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    elapsed = t_start.elapsed_time(t_end) / 1e3
    if world > 1:
        tt = torch.tensor([elapsed], device=device)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        elapsed = float(tt.item())
    t_fwd = statistics.mean(e0.elapsed_time(e1) for e0, e1, _ in ev) / 1e3
    t_bwd = statistics.mean(e1.elapsed_time(e2) for _, e1, e2 in ev) / 1e3
    tokens = B * T * world * args.steps
    value = tokens / elapsed
    ms_per_step = elapsed / args.steps * 1e3
    th = B * T * H
    dom_bwd = t_bwd >= t_fwd
    dom_bytes = (BWD_BYTES_PER_TH if dom_bwd else FWD_BYTES_PER_TH) * th
    dom_t = t_bwd if dom_bwd else t_fwd
    achieved = dom_bytes / dom_t / 1e9
    roof_time = max(FLOP_PER_TH * th / (tf_peak * 1e12), (FWD_BYTES_PER_TH + BWD_BYTES_PER_TH) * th / (hbm_peak * 1e9))

    # end to end through the public API: pinned host inputs -> device, fwd + bwd via autograd, dW/db -> host
    e2e = None
    if args.e2e_steps > 0:
        hq, hk, hg = (t.cpu().pin_memory() for t in (q, k, dqc))
        hdW = torch.empty(H, K, pin_memory=True)
        hdb = torch.empty(H, pin_memory=True)
        Wp = W.clone().requires_grad_(True)
        bp = bias.clone().requires_grad_(True)
        dq_ = torch.empty_like(q)
        dk_ = torch.empty_like(k)
        dg_ = torch.empty_like(dqc)

        def e2e_step():
            dq_.copy_(hq, non_blocking=True)
            dk_.copy_(hk, non_blocking=True)
            dg_.copy_(hg, non_blocking=True)
            qq = dq_.detach().requires_grad_(True)
            kk = dk_.detach().requires_grad_(True)
            Wp.grad = None
            bp.grad = None
            out, _, _ = ccq_b200.fused_ccq_clean_gated(qq, kk, Wp, bp)
            out.backward(dg_)
            allreduce(Wp.grad, bp.grad)
            hdW.copy_(Wp.grad, non_blocking=True)
            hdb.copy_(bp.grad, non_blocking=True)

        for _ in range(2):
            e2e_step()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(device)
        s0 = torch.cuda.Event(enable_timing=True)
        s1 = torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        for _ in range(args.e2e_steps):
            e2e_step()
        s1.record(stream)
        torch.cuda.synchronize(device)
        et = s0.elapsed_time(s1) / 1e3
        if world > 1:
            tt = torch.tensor([et], device=device)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            et = float(tt.item())
        e2e = {'value': B * T * world * args.e2e_steps / et, 'unit': 'tokens/s',
               'h2d_bytes_per_step': 3 * q.numel() * q.element_size(),
               'd2h_bytes_per_step': (H * K + H) * 4}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            tps, t, thr = cpu_port_sample()
            cpu = {'value': tps, 'unit': 'tokens/s', 'cores': thr, 'kind': 'port',
                   'sample': f'B=1,T=4096,H=2 of C2 (fp32 torch restatement, chunk 64, autograd), {t * 1e3:.1f} ms per sample, scaled by 2/16 heads'}
        except Exception as exc:  # the baseline is informational
            cpu = {'value': None, 'unit': 'tokens/s', 'cores': None, 'kind': 'port', 'sample': f'failed: {exc}'}

    if rank == 0:
        line = {
            'metric': C2_METRIC,
            'value': value, 'unit': 'tokens/s', 'n_gpus': world, 'steps': args.steps, 'warmup': args.warmup,
            'ms_per_step': ms_per_step, 'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None,
            'dtype': 'bf16', 'data': 'synthetic (seeded; q,k unit-normalised N(0,1), W~N(0,0.02), b~U(-1,1))',
            'config': c2_config(world, B, T, H, K),
            'paths': {'fwd': path_fwd, 'bwd': path_bwd},
            'roofline': {'bound': 'hbm', 'achieved': achieved, 'peak': hbm_peak, 'unit': 'GB/s',
                         'frac': achieved / hbm_peak, 'traffic': NCU_TRAFFIC_C2['bwd' if dom_bwd else 'fwd'],
                         'traffic_unit': 'bytes per launch (ncu)',
                         'kernel': 'bwd' if dom_bwd else 'fwd', 'peak_kind': peak_kind,
                         'op_roofline_frac': roof_time / (elapsed / args.steps / 1),
                         'fwd_ms': t_fwd * 1e3, 'bwd_ms': t_bwd * 1e3},
            'clocks': clocks.summary(),
            'e2e': e2e,
            'gpu_launches': n_launch,
            'cpu_baseline': cpu,
        }
        print(json.dumps(line), flush=True)


def run_decode(args, rank, world, device, hbm_peak, peak_kind):
    import torch

    from ccq_b200 import _lib, ops
    N, H, K = 256, 16, 128
    gen = torch.Generator(device=device).manual_seed(2000 + rank)
    pre = unit(gen, (N, 2048, H, K), device, torch.float32)
    C = torch.einsum('nthk,nthv->nhkv', pre, pre).contiguous()
    m = pre.sum(1).contiguous()
    del pre
    steps = [(unit(gen, (N, 1, H, K), device, torch.bfloat16), unit(gen, (N, 1, H, K), device, torch.bfloat16),
              torch.rand(N, 1, H, generator=gen, device=device).to(torch.bfloat16)) for _ in range(16)]
    stream = torch.cuda.current_stream(device)
    off = 2048
    for i in range(args.warmup):
        qq, kk, ll = steps[i % 16]
        ops.decode_step(qq, kk, ll, C, m, position_offset=off, inplace=True)
        off += 1
    torch.cuda.synchronize(device)
    n_launch = 0
    with ClockSampler(device.index) as clocks:
        s0 = torch.cuda.Event(enable_timing=True)
        s1 = torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        for i in range(args.steps):
            qq, kk, ll = steps[i % 16]
            ops.decode_step(qq, kk, ll, C, m, position_offset=off, inplace=True)
            n_launch += _lib.last_launch_count()
            off += 1
        s1.record(stream)
        torch.cuda.synchronize(device)
    el = s0.elapsed_time(s1) / 1e3
    per = el / args.steps
    achieved = DECODE_BYTES_PER_TH * N * H / per / 1e9
    if rank == 0:
        print(json.dumps({
            'metric': 'CCQ decode step tokens/s (bf16 q/k, fp32 cache, batch 256, H=16, d_k=128)',
            'value': N / per, 'unit': 'tokens/s', 'n_gpus': world, 'steps': args.steps, 'warmup': args.warmup,
            'ms_per_step': per * 1e3, 'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None,
            'dtype': 'bf16', 'data': 'synthetic', 'config': {'workload': 'c4: decode batch 256, H=16, d_k=128'},
            'roofline': {'bound': 'hbm', 'achieved': achieved, 'peak': hbm_peak, 'unit': 'GB/s',
                         'frac': achieved / hbm_peak, 'traffic': NCU_TRAFFIC_C4,
                         'traffic_unit': 'bytes per launch (ncu)', 'peak_kind': peak_kind},
            'clocks': clocks.summary(), 'gpu_launches': n_launch}), flush=True)


def main():
    args = parse()
    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local_rank = int(os.environ.get('LOCAL_RANK', '0'))
    if args.impl == 'reference':
        run_reference(args, rank, world)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device('cuda', local_rank))
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == '__main__':
    main()
