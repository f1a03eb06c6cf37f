#!/usr/bin/env python
"""Benchmark of the B200 CCQ cleaning operator: forward + backward throughput (tokens/s).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload all|c2|c3|c4|c5]

Rank 0 prints one JSON line.  Its headline (``value``) is workload c2: per GPU B=8, T=4096, H=16,
d_k=128, bf16 inputs with fp32 accumulation; q, k ~ N(0,1) L2-normalised per head; lambda =
sigmoid(W q + b) with the per-head W_lambda (H x d_k) ~ N(0, 0.02) and b ~ U(-1, 1) fused into the
kernels; upstream grad ~ N(0,1).  One step = forward + backward of the operator (q_clean, dq, dk,
dW, db); with N > 1 ranks each rank runs its own batch shard (weak scaling) and dW/db are summed
over NCCL without the next step waiting for it.  ``value`` is the whole job's tokens/s.

With the default ``--workload all`` the same line also carries, each with its own roofline:
  c3  a packed varlen batch per GPU: 32 documents with lengths ~ U[128, 8192], H=16, d_k=128;
  c4  the decode step: batch 256, H=16, d_k=128, fp32 cache built from a 2048-token prefix,
      1024 single-token steps;
  c5  B=64, T=16384, H=16, d_k=128 split over the N ranks by batch rows (strong scaling);
  reference_triton_gpu  the reference's own Triton operator (fused_ccq_clean_read, bf16) timed on
      the same GPU at c2 beside this library's operator called through the same Python API.

``--impl reference`` times the reference's CPU path of the operator on the host cores (the
reference has no CPU kernels of its own; oracle/ccq_torch_port.py is the torch restatement of its
formula), one batch row of c2 per step.
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
# kernel on the c2 shapes at batch 4, doubled for batch 8 (traffic grows with the (document, head)
# count); profiles/tc_fwd_kernel_c2.md and profiles/tc_bwd_kernel_c2.md give the commands.
NCU_TRAFFIC_C2 = {'fwd': 2 * (134.3e6 + 41.6e6), 'bwd': 2 * (207.8e6 + 100.8e6)}  # batch-4 captures x 2 (profiles/)
NCU_TRAFFIC_C4 = 272.7e6 + 213.9e6  # decode_kernel, profiles/decode_kernel_c4.md
DECODE_BYTES_PER_TH = 2 * 128 * 128 * 4 + 2 * 128 * 4 + 4 * 128 * 2 + 2 * 2

METRIC = 'CCQ clean fwd+bwd tokens/s (bf16, T=4096, H=16, d_k=128; whole job) and % roofline'
DATA = 'synthetic (seeded; q,k unit-normalised N(0,1), W~N(0,0.02), b~U(-1,1), grad~N(0,1))'


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=50)
    ap.add_argument('--warmup', type=int, default=5)
    ap.add_argument('--impl', default='ours', choices=['ours', 'reference'])
    ap.add_argument('--workload', default='all', choices=['all', 'c2', 'c2_l2norm', 'c3', 'c4', 'c5'])
    ap.add_argument('--batch', type=int, default=8,
                    help='batch rows per GPU of c2 / c2_l2norm (8 is the benchmark; smaller for profiling)')
    ap.add_argument('--e2e-steps', type=int, default=10)
    ap.add_argument('--soak-s', type=float, default=1.5,
                    help='seconds of untimed c2 steps run under the clock sampler before the timed steps')
    ap.add_argument('--no-cpu-baseline', action='store_true')
    ap.add_argument('--no-triton', action='store_true', help='skip the reference Triton operator timing')
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
    """nvidia-smi clocks, utilisation and throttle reasons sampled every 200 ms while active."""

    FIELDS = ('index,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,clocks_event_reasons.active,'
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
        """Median SM clock over the samples taken while the GPU was busy (utilisation >= 50 %), the
        throttle reasons seen in any sample, and the sample counts."""
        busy, idle, mx, reasons = [], [], None, set()
        names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap']
        for line in self.lines:
            parts = [p.strip() for p in line.split(',')]
            if len(parts) < 10:
                continue
            try:
                sm = float(parts[1])
                mx = float(parts[2])
                util = float(parts[4])
            except ValueError:
                continue
            (busy if util >= 50 else idle).append(sm)
            for nm, val in zip(names, parts[6:10]):
                if val.lower().startswith('active'):
                    reasons.add(nm)
        return {'sm_mhz': statistics.median(busy) if busy else None, 'sm_max_mhz': mx, 'reasons': sorted(reasons),
                'samples': len(busy) + len(idle), 'samples_busy': len(busy)}


def unit(gen, shape, device, dtype):
    import torch
    x = torch.randn(shape, generator=gen, device=device, dtype=torch.float32)
    return (x / x.norm(dim=-1, keepdim=True)).to(dtype)


def c2_inputs(device, seed, B=8, T=4096, H=16, K=128):
    """The c2 inputs of one rank: q, k (bf16, unit rows), W [H,K], b [H] (fp32), dq_clean (bf16)."""
    import torch
    gen = torch.Generator(device=device).manual_seed(seed)
    q = unit(gen, (B, T, H, K), device, torch.bfloat16)
    k = unit(gen, (B, T, H, K), device, torch.bfloat16)
    W = torch.randn(H, K, generator=gen, device=device) * 0.02
    bias = torch.rand(H, generator=gen, device=device) * 2 - 1
    dqc = torch.randn(B, T, H, K, generator=gen, device=device).to(torch.bfloat16)
    return q, k, W, bias, dqc


def c3_lengths(seed, n_docs=32, lo=128, hi=8192):
    """Seeded document lengths ~ U[lo, hi] of one rank's packed varlen batch."""
    import torch
    g = torch.Generator().manual_seed(seed)
    return [int(x) for x in torch.randint(lo, hi + 1, (n_docs,), generator=g)]


def c2_config(world, B=8, T=4096, H=16, K=128):
    """The c2 workload description shared by both arms of the bench."""
    return {'workload': f'c2: B={B}/GPU,T={T},H={H},d_k={K} cleaning fwd+bwd, per-head gate fused',
            'global_batch': B * world, 'seq_len': T, 'heads': H, 'd_k': K,
            'parallelism': f'dp{world} (batch shards, NCCL all-reduce of dW,db)',
            'l2': f'inputs larger than L2 (q,k,dq_clean {3 * B * T * H * K * 2 >> 20} MiB per GPU)'}


def roofline_of(th, step_s, hbm_peak, tf_peak):
    """Op roofline of one fwd+bwd step over `th` token-heads (HBM-bound at K=128)."""
    t_roof = max(FLOP_PER_TH * th / (tf_peak * 1e12), (FWD_BYTES_PER_TH + BWD_BYTES_PER_TH) * th / (hbm_peak * 1e9))
    achieved = (FWD_BYTES_PER_TH + BWD_BYTES_PER_TH) * th / step_s / 1e9
    return {'bound': 'hbm', 'achieved': achieved, 'peak': hbm_peak, 'unit': 'GB/s', 'frac': achieved / hbm_peak,
            'op_roofline_frac': t_roof / step_s}


def max_over_ranks(x, world, device):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x, world, device):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], device=device, dtype=torch.float64)
    dist.all_reduce(t)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# ------------------------------------------------------------------------------------------------
# CPU: the reference's formula restated in torch (oracle/ccq_torch_port.py), on the host cores
# ------------------------------------------------------------------------------------------------

def cpu_row_sample(T=4096, H=16, K=128, seed=0):
    """Inputs of one c2 batch row (B=1) in fp32 on the CPU."""
    import torch
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(1, T, H, K, generator=g)
    q = q / q.norm(dim=-1, keepdim=True)
    k = torch.randn(1, T, H, K, generator=g)
    k = k / k.norm(dim=-1, keepdim=True)
    W = torch.randn(H, K, generator=g) * 0.02
    b = torch.rand(H, generator=g) * 2 - 1
    dqc = torch.randn(1, T, H, K, generator=g)
    return q, k, W, b, dqc


def cpu_step(inputs):
    from oracle import ccq_torch_port as P
    t0 = time.perf_counter()
    P.clean_step_fwd_bwd(*inputs)
    return time.perf_counter() - t0


CPU_SAMPLE = 'one batch row of c2 per step (B=1, T=4096, H=16, d_k=128; fp32 torch restatement, chunk 64, autograd)'


def run_reference(args, rank, world):
    """The reference's CPU path timed on the host cores (rank 0 only; other ranks exit)."""
    if rank != 0:
        return
    import torch
    torch.set_num_threads(os.cpu_count() or 1)
    inputs = cpu_row_sample()
    for _ in range(args.warmup):
        cpu_step(inputs)
    t0 = time.perf_counter()
    times = [cpu_step(inputs) for _ in range(args.steps)]
    total = time.perf_counter() - t0
    tokens = 4096 * args.steps
    value = tokens / total
    line = {
        'impl': 'reference', 'metric': METRIC,
        'value': value, 'unit': 'tokens/s', 'n_gpus': world, 'steps': args.steps, 'warmup': args.warmup,
        'ms_per_step': total / args.steps * 1e3, 'higher_is_better': True, 'scaling': 'weak',
        'vs_baseline': None, 'dtype': 'f32', 'data': DATA,
        'config': dict(c2_config(world), sample=CPU_SAMPLE),
        'cpu_baseline': {'value': value, 'unit': 'tokens/s', 'cores': torch.get_num_threads(), 'kind': 'port',
                         'sample': f'{CPU_SAMPLE}; median {statistics.median(times) * 1e3:.0f} ms per step'},
        'e2e': {'value': value, 'unit': 'tokens/s', 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------------
# GPU workloads
# ------------------------------------------------------------------------------------------------

def timed_steps(step, steps, stream, events=False):
    """Run `steps` calls of step() between CUDA events on `stream`; returns (seconds, per-step marks)."""
    import torch
    marks = []
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(steps):
        marks.append(step())
    t1.record(stream)
    torch.cuda.synchronize()
    return t0.elapsed_time(t1) / 1e3, marks


def run_c2(args, rank, world, device, hbm_peak, tf_peak, peak_kind, reducer):
    import torch

    import ccq_b200
    from ccq_b200 import _lib, ops

    B, T, H, K = args.batch, 4096, 16, 128
    q, k, W, bias, dqc = c2_inputs(device, 1000 + rank, B=B)
    stream = torch.cuda.current_stream(device)
    launches = [0]

    def step(ev=None):
        if ev is not None:
            ev[0].record(stream)
        qc, fc, fm, aux = ops.clean_fwd_raw(q, k, None, W, bias, 0, None, None, True, None, B)
        launches[0] += _lib.last_launch_count()
        if ev is not None:
            ev[1].record(stream)
        ops.clean_bwd_raw(q, k, None, W, bias, 0, None, None, True, None, B, fc, fm, aux, dqc, None, None,
                          gate_out=reducer.out())
        launches[0] += _lib.last_launch_count()
        if ev is not None:
            ev[2].record(stream)
        reducer.submit()

    for _ in range(args.warmup):
        step()
    paths = {}
    ops.clean_fwd_raw(q, k, None, W, bias, 0, None, None, True, None, B)
    paths['fwd'] = _lib.last_path()
    torch.cuda.synchronize(device)
    barrier(world)
    with ClockSampler(device.index) as clocks:
        # untimed soak of the same steps so the clock record covers the kernels under load
        t_end = time.time() + args.soak_s
        while time.time() < t_end:
            for _ in range(20):
                step()
            torch.cuda.synchronize(device)
        reducer.result()
        torch.cuda.synchronize(device)
        barrier(world)
        launches[0] = 0
        ev = [tuple(torch.cuda.Event(enable_timing=True) for _ in range(3)) for _ in range(args.steps)]
        s0 = torch.cuda.Event(enable_timing=True)
        s1 = torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        for i in range(args.steps):
            step(ev[i])
        reducer.result()  # the last step's reduced gate gradients, where an optimizer takes them
        s1.record(stream)
        torch.cuda.synchronize(device)
    paths['bwd'] = _lib.last_path()
    barrier(world)
    elapsed = max_over_ranks(s0.elapsed_time(s1) / 1e3, world, device)
    t_fwd = statistics.mean(a.elapsed_time(b) for a, b, _ in ev) / 1e3
    t_bwd = statistics.mean(b.elapsed_time(c) for _, b, c in ev) / 1e3
    th = B * T * H
    step_s = elapsed / args.steps
    dom_bwd = t_bwd >= t_fwd
    dom_bytes = (BWD_BYTES_PER_TH if dom_bwd else FWD_BYTES_PER_TH) * th
    dom_t = t_bwd if dom_bwd else t_fwd
    achieved = dom_bytes / dom_t / 1e9
    op = roofline_of(th, step_s, hbm_peak, tf_peak)
    out = {
        'value': B * T * world * args.steps / elapsed, 'ms_per_step': step_s * 1e3, 'paths': paths,
        'roofline': {'bound': 'hbm', 'achieved': achieved, 'peak': hbm_peak, 'unit': 'GB/s',
                     'frac': achieved / hbm_peak, 'traffic': NCU_TRAFFIC_C2['bwd' if dom_bwd else 'fwd'],
                     'traffic_unit': 'bytes per launch (ncu)', 'kernel': 'bwd' if dom_bwd else 'fwd',
                     'peak_kind': peak_kind, 'op_roofline_frac': op['op_roofline_frac'],
                     'fwd_ms': t_fwd * 1e3, 'bwd_ms': t_bwd * 1e3,
                     'fwd_frac': FWD_BYTES_PER_TH * th / t_fwd / 1e9 / hbm_peak,
                     'step_minus_kernels_us': (step_s - t_fwd - t_bwd) * 1e6},
        'clocks': clocks.summary(), 'gpu_launches': launches[0],
    }

    # end to end through the public API: pinned host inputs -> device, fwd + bwd via autograd, dW/db -> host
    if args.e2e_steps > 0:
        from ccq_b200.distributed import allreduce_gate_grads
        hq, hk, hg = (t.cpu().pin_memory() for t in (q, k, dqc))
        hdW = torch.empty(H, K, pin_memory=True)
        hdb = torch.empty(H, pin_memory=True)
        Wp = W.clone().requires_grad_(True)
        bp = bias.clone().requires_grad_(True)
        # Each step's inputs cross the host link on a copy stream into one of two device buffer sets
        # while the previous step computes; a buffer set is refilled once the step that read it is done.
        copy_stream = torch.cuda.Stream(device)
        bufs = [tuple(torch.empty_like(x) for x in (q, k, dqc)) for _ in range(2)]
        copied = [torch.cuda.Event() for _ in range(2)]
        consumed = [torch.cuda.Event() for _ in range(2)]

        def issue_copy(j):
            copy_stream.wait_event(consumed[j % 2])
            with torch.cuda.stream(copy_stream):
                for dst, src in zip(bufs[j % 2], (hq, hk, hg)):
                    dst.copy_(src, non_blocking=True)
            copied[j % 2].record(copy_stream)

        def e2e_step(j):
            stream.wait_event(copied[j % 2])
            issue_copy(j + 1)
            dq_, dk_, dg_ = bufs[j % 2]
            qq = dq_.detach().requires_grad_(True)
            kk = dk_.detach().requires_grad_(True)
            Wp.grad = None
            bp.grad = None
            o, _, _ = ccq_b200.fused_ccq_clean_gated(qq, kk, Wp, bp)
            o.backward(dg_)
            consumed[j % 2].record(stream)
            allreduce_gate_grads(Wp.grad, bp.grad)
            hdW.copy_(Wp.grad, non_blocking=True)
            hdb.copy_(bp.grad, non_blocking=True)

        issue_copy(0)
        for j in range(2):
            e2e_step(j)
        torch.cuda.synchronize(device)
        barrier(world)
        # timed: steps 2 .. K+1 and the K copies they issue (the inputs of steps 3 .. K+2); the input
        # copy of step 2 finished before the region starts, the last one is waited for inside it
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for j in range(2, 2 + args.e2e_steps):
            e2e_step(j)
        stream.wait_event(copied[(2 + args.e2e_steps) % 2])
        e1.record(stream)
        torch.cuda.synchronize(device)
        et = max_over_ranks(e0.elapsed_time(e1) / 1e3, world, device)
        out['e2e'] = {'value': B * T * world * args.e2e_steps / et, 'unit': 'tokens/s',
                      'h2d_bytes_per_step': 3 * q.numel() * q.element_size(),
                      'd2h_bytes_per_step': (H * K + H) * 4,
                      'ms_per_step': et / args.e2e_steps * 1e3,
                      'note': 'pinned host q, k, dq_clean copied in every step (host-link bound at this size), '
                              'on a second stream while the previous step computes'}
    return out


def run_c3(args, rank, world, device, hbm_peak, tf_peak):
    """Packed varlen batch per GPU: 32 documents, lengths ~ U[128, 8192], longest-first CTA order."""
    import torch

    from ccq_b200 import _lib, ops
    H, K = 16, 128
    lens = c3_lengths(3000 + rank)
    T = sum(lens)
    gen = torch.Generator(device=device).manual_seed(3100 + rank)
    q = unit(gen, (1, T, H, K), device, torch.bfloat16)
    k = unit(gen, (1, T, H, K), device, torch.bfloat16)
    W = torch.randn(H, K, generator=gen, device=device) * 0.02
    bias = torch.rand(H, generator=gen, device=device) * 2 - 1
    dqc = torch.randn(1, T, H, K, generator=gen, device=device).to(torch.bfloat16)
    cu = torch.tensor([0] + lens, dtype=torch.int64).cumsum(0).to(device)
    N = len(lens)
    stream = torch.cuda.current_stream(device)
    launches = [0]

    def step():
        qc, fc, fm, aux = ops.clean_fwd_raw(q, k, None, W, bias, 0, None, None, True, cu, N)
        launches[0] += _lib.last_launch_count()
        ops.clean_bwd_raw(q, k, None, W, bias, 0, None, None, True, cu, N, fc, fm, aux, dqc, None, None)
        launches[0] += _lib.last_launch_count()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(device)
    barrier(world)
    launches[0] = 0
    el, _ = timed_steps(step, args.steps, stream)
    el = max_over_ranks(el, world, device)
    step_s = el / args.steps
    tokens = sum_over_ranks(T, world, device)
    th = T * H
    return {'workload': 'c3: per GPU 32 packed documents, lengths ~ U[128,8192] (seeded), H=16, d_k=128, '
                        'bf16 fwd+bwd, per-head gate fused, documents launched longest first',
            'tokens_rank0': T, 'value': tokens / step_s, 'unit': 'tokens/s', 'ms_per_step': step_s * 1e3,
            'steps': args.steps, 'roofline': roofline_of(th, step_s, hbm_peak, tf_peak),
            'gpu_launches': launches[0]}


def run_c4(args, rank, world, device, hbm_peak, peak_kind, steps=1024):
    """Decode: batch 256, H=16, d_k=128, fp32 cache from a 2048-token prefix, `steps` tokens."""
    import torch

    from ccq_b200 import _lib, ops
    N, H, K, P = 256, 16, 128, 2048
    gen = torch.Generator(device=device).manual_seed(2000 + rank)
    C = torch.zeros(N, H, K, K, device=device)
    m = torch.zeros(N, H, K, device=device)
    for p0 in range(0, P, 256):  # prefix state in slices, fp32
        pre = unit(gen, (N, 256, H, K), device, torch.float32)
        C += torch.einsum('nthk,nthv->nhkv', pre, pre)
        m += pre.sum(1)
        del pre
    sets = [(unit(gen, (N, 1, H, K), device, torch.bfloat16), unit(gen, (N, 1, H, K), device, torch.bfloat16),
             torch.rand(N, 1, H, generator=gen, device=device).to(torch.bfloat16)) for _ in range(16)]
    stream = torch.cuda.current_stream(device)
    off = [P]
    launches = [0]

    def step():
        qq, kk, ll = sets[off[0] % 16]
        ops.decode_step(qq, kk, ll, C, m, position_offset=off[0], inplace=True)
        launches[0] += _lib.last_launch_count()
        off[0] += 1

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(device)
    barrier(world)
    launches[0] = 0
    el, _ = timed_steps(step, steps, stream)
    el = max_over_ranks(el, world, device)
    per = el / steps
    achieved = DECODE_BYTES_PER_TH * N * H / per / 1e9
    return {'workload': 'c4: decode step, batch 256/GPU, H=16, d_k=128, bf16 q/k, fp32 cache from a 2048-token '
                        'prefix, 1024 single-token steps', 'value': N * world / per, 'unit': 'tokens/s',
            'ms_per_step': per * 1e3, 'steps': steps,
            'roofline': {'bound': 'hbm', 'achieved': achieved, 'peak': hbm_peak, 'unit': 'GB/s',
                         'frac': achieved / hbm_peak, 'traffic': NCU_TRAFFIC_C4,
                         'traffic_unit': 'bytes per launch (ncu)', 'peak_kind': peak_kind},
            'gpu_launches': launches[0]}


def run_c5(args, rank, world, device, hbm_peak, tf_peak, reducer):
    """B=64, T=16384 split over the ranks by batch rows (strong scaling); dW/db summed over NCCL."""
    import torch

    from ccq_b200 import _lib, ops
    from ccq_b200.distributed import shard_rows
    B_all, T, H, K = 64, 16384, 16, 128
    lo, hi = shard_rows(B_all, world, rank)
    B = hi - lo
    gen = torch.Generator(device=device).manual_seed(5000 + rank)
    q = unit(gen, (B, T, H, K), device, torch.bfloat16)
    k = unit(gen, (B, T, H, K), device, torch.bfloat16)
    W = torch.randn(H, K, generator=torch.Generator(device=device).manual_seed(5000), device=device) * 0.02
    bias = torch.zeros(H, device=device)
    dqc = torch.randn(B, T, H, K, generator=gen, device=device).to(torch.bfloat16)
    stream = torch.cuda.current_stream(device)
    launches = [0]

    def step():
        qc, fc, fm, aux = ops.clean_fwd_raw(q, k, None, W, bias, 0, None, None, True, None, B)
        launches[0] += _lib.last_launch_count()
        del qc
        ops.clean_bwd_raw(q, k, None, W, bias, 0, None, None, True, None, B, fc, fm, aux, dqc, None, None,
                          gate_out=reducer.out())
        launches[0] += _lib.last_launch_count()
        reducer.submit()

    for _ in range(args.warmup):
        step()
    reducer.result()
    torch.cuda.synchronize(device)
    barrier(world)
    launches[0] = 0
    steps = max(3, args.steps // 2)

    def timed():
        for _ in range(steps):
            step()
        reducer.result()

    el, _ = timed_steps(timed, 1, stream)
    el = max_over_ranks(el, world, device)
    step_s = el / steps
    return {'workload': f'c5: B=64, T=16384, H=16, d_k=128 bf16 fwd+bwd split over {world} GPU(s) by batch rows '
                        f'({B} per GPU), per-head gate fused, dW/db all-reduced over NCCL',
            'scaling': 'strong', 'value': B_all * T / step_s, 'unit': 'tokens/s', 'ms_per_step': step_s * 1e3,
            'steps': steps, 'roofline': roofline_of(B * T * H, step_s, hbm_peak, tf_peak),
            'gpu_launches': launches[0]}


def run_c2_l2norm(args, rank, world, device, hbm_peak, tf_peak):
    """c2 with RAW q and k: the l2norm of both (which the fused_chunk orchestrators apply right before
    the operator) fused into the kernels, fwd + bwd through the autograd API with the backbone's
    gradient on the normalised keys; beside it the same step with fla's l2norm as a separate pass
    (the reference's sequence) in front of this library's operator."""
    import torch

    import ccq_b200
    B, T, H, K = args.batch, 4096, 16, 128
    gen = torch.Generator(device=device).manual_seed(1500 + rank)
    q0 = torch.randn(B, T, H, K, generator=gen, device=device).to(torch.bfloat16)
    k0 = torch.randn(B, T, H, K, generator=gen, device=device).to(torch.bfloat16)
    lam0 = torch.rand(B, T, H, generator=gen, device=device).to(torch.bfloat16)
    dqc = torch.randn(B, T, H, K, generator=gen, device=device).to(torch.bfloat16)
    dkn = torch.randn(B, T, H, K, generator=gen, device=device).to(torch.bfloat16)
    stream = torch.cuda.current_stream(device)

    def fused():
        q, k, lam = (t.detach().requires_grad_(True) for t in (q0, k0, lam0))
        qc, kn, _, _ = ccq_b200.fused_ccq_clean_read_l2norm(q, k, lam)
        torch.autograd.backward([qc, kn], [dqc, dkn])

    res = {}
    arms = [('fused', fused)]
    try:
        from fla.modules.l2norm import l2norm as fla_l2norm

        def separate():
            q, k, lam = (t.detach().requires_grad_(True) for t in (q0, k0, lam0))
            qn, kn = fla_l2norm(q, eps=1e-6), fla_l2norm(k, eps=1e-6)
            qc, _, _ = ccq_b200.fused_ccq_clean_read(qn, kn, lam)
            torch.autograd.backward([qc, kn], [dqc, dkn])
        arms.append(('separate_fla_l2norm', separate))
    except Exception as exc:
        res['separate_fla_l2norm'] = {'unavailable': f'{type(exc).__name__}: {exc}'[:200]}
    for name, fn in arms:
        for _ in range(max(3, args.warmup)):
            fn()
        torch.cuda.synchronize(device)
        barrier(world)
        el, _ = timed_steps(fn, args.steps, stream)
        el = max_over_ranks(el, world, device)
        step_s = el / args.steps
        res[name] = {'ms_per_step': step_s * 1e3, 'value': B * T * world / step_s, 'unit': 'tokens/s'}
    # fused path, algorithmic bytes per token-head: fwd reads q, k and writes q_clean, k_norm (+16 B of
    # per-token side outputs); bwd reads q, k_norm, dq_clean and the backbone's gradient on k_norm
    # (+16 B) and writes dq and dk (the key gradient is mapped through the norm inside the kernel)
    th = B * T * H
    step_bytes = (1040 + 1552) * th
    ach = step_bytes / (res['fused']['ms_per_step'] * 1e-3) / 1e9
    res['fused']['roofline'] = {'bound': 'hbm', 'achieved': ach, 'peak': hbm_peak, 'unit': 'GB/s',
                                'frac': ach / hbm_peak, 'bytes_per_token_head': 2592}
    res['workload'] = ('c2 shapes with raw (un-normalised) bf16 q, k ~ N(0,1), per-token lambda, gradients on '
                       'q_clean and on the normalised keys; through the autograd API')
    return res


def reference_path():
    """Directory holding the reference package `ccq` (its install under baseline/_ref, or
    CCQ_REFERENCE_PATH), or None."""
    for cand in (os.environ.get('CCQ_REFERENCE_PATH'), os.path.join(ROOT, 'baseline', '_ref')):
        if cand and os.path.isdir(os.path.join(cand, 'ccq')):
            return cand
    return None


def run_triton_reference(args, device):
    """The reference's Triton fused_ccq_clean_read (fwd+bwd, bf16) at c2 on this GPU, next to this
    library's fused_ccq_clean_read called through the same Python signature on the same inputs."""
    import torch

    import ccq_b200
    path = reference_path()
    if path is None:
        return {'unavailable': 'reference package not installed under baseline/_ref'}
    if path not in sys.path:
        sys.path.insert(0, path)
    try:
        from ccq.ops.common import fused_read as R
    except Exception as exc:  # report, do not fail the bench
        return {'unavailable': f'import failed: {type(exc).__name__}: {exc}'[:300]}
    B, T, H, K = 8, 4096, 16, 128
    q0, k0, W, bias, dqc = c2_inputs(device, 1000)
    lam0 = torch.sigmoid(torch.einsum('bthk,hk->bth', q0.float(), W) + bias).to(torch.bfloat16)
    stream = torch.cuda.current_stream(device)

    def make(fn):
        def step():
            q = q0.detach().requires_grad_(True)
            k = k0.detach().requires_grad_(True)
            lam = lam0.detach().requires_grad_(True)
            out = fn(q, k, lam)[0]
            out.backward(dqc)
            return out, q.grad, k.grad, lam.grad
        return step

    res = {}
    outs = {}
    for name, fn in (('reference_triton', R.fused_ccq_clean_read), ('ours', ccq_b200.fused_ccq_clean_read)):
        step = make(fn)
        try:
            for _ in range(max(3, args.warmup)):
                o = step()
            torch.cuda.synchronize(device)
            outs[name] = [None if t is None else t.float() for t in o]
            el, _ = timed_steps(step, args.steps, stream)
            # forward alone, same call
            q = q0.detach().requires_grad_(True)
            k = k0.detach().requires_grad_(True)
            lam = lam0.detach().requires_grad_(True)
            ef, _ = timed_steps(lambda: fn(q, k, lam), args.steps, stream)
        except Exception as exc:
            res[name] = {'error': f'{type(exc).__name__}: {exc}'[:300]}
            continue
        res[name] = {'ms_per_step': el / args.steps * 1e3, 'fwd_ms': ef / args.steps * 1e3,
                     'tokens_per_s': B * T * args.steps / el}
        if name == 'ours':
            res[name]['path'] = ccq_b200.last_path()
    if 'reference_triton' in outs and 'ours' in outs:
        res['max_abs_diff'] = {n: float((a - b).abs().max().detach()) for n, a, b in
                               zip(('q_clean', 'dq', 'dk', 'dlam'), outs['ours'], outs['reference_triton'])
                               if a is not None and b is not None}
    if 'ms_per_step' in res.get('reference_triton', {}) and 'ms_per_step' in res.get('ours', {}):
        res['speedup'] = res['reference_triton']['ms_per_step'] / res['ours']['ms_per_step']
    res['workload'] = ('c2 (B=8, T=4096, H=16, d_k=128, bf16) fwd+bwd through fused_ccq_clean_read(q, k, lambda) '
                       'with per-token lambda [B,T,H] = sigmoid(W q + b) precomputed; both arms autograd, '
                       'same inputs, same GPU; the reference JIT-compiles its Triton kernels here')
    return res


def run_ours(args, rank, world, local_rank):
    import torch

    from ccq_b200 import _lib
    from ccq_b200.distributed import GateGradReducer

    device = torch.device('cuda', local_rank)
    torch.cuda.set_device(device)
    _lib.load()
    hbm_peak, tf_peak, peak_kind = peaks()
    reducer = GateGradReducer(16, 128, device)
    extra = {}
    try:
        if args.workload in ('all', 'c2'):
            main = run_c2(args, rank, world, device, hbm_peak, tf_peak, peak_kind, reducer)
        if args.workload in ('all', 'c2_l2norm'):
            extra['c2_l2norm'] = run_c2_l2norm(args, rank, world, device, hbm_peak, tf_peak)
        if args.workload in ('all', 'c3'):
            extra['c3'] = run_c3(args, rank, world, device, hbm_peak, tf_peak)
        if args.workload in ('all', 'c4'):
            extra['c4'] = run_c4(args, rank, world, device, hbm_peak, peak_kind)
        torch.cuda.empty_cache()
        if args.workload in ('all', 'c5'):
            extra['c5'] = run_c5(args, rank, world, device, hbm_peak, tf_peak, reducer)
        torch.cuda.empty_cache()
    finally:
        reducer.drain()
    if rank == 0 and world == 1 and args.workload == 'all' and not args.no_triton:
        extra['reference_triton_gpu'] = run_triton_reference(args, device)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.workload in ('all', 'c2'):
        try:
            import torch as _t
            _t.set_num_threads(os.cpu_count() or 1)
            inputs = cpu_row_sample()
            cpu_step(inputs)
            t = cpu_step(inputs)
            cpu = {'value': 4096 / t, 'unit': 'tokens/s', 'cores': _t.get_num_threads(), 'kind': 'port',
                   'sample': f'{CPU_SAMPLE}; {t * 1e3:.0f} ms for the sample'}
        except Exception as exc:  # the baseline is informational
            cpu = {'value': None, 'unit': 'tokens/s', 'cores': None, 'kind': 'port', 'sample': f'failed: {exc}'}

    if rank != 0:
        return
    if args.workload == 'c2_l2norm':
        w = extra['c2_l2norm']
        print(json.dumps({'metric': 'CCQ c2_l2norm tokens/s', 'n_gpus': world, 'steps': args.steps,
                          'warmup': args.warmup, 'higher_is_better': True, 'dtype': 'bf16', 'data': DATA,
                          'config': {'workload': w['workload'], 'batch_per_gpu': args.batch}, 'c2_l2norm': w}),
              flush=True)
        return
    if args.workload not in ('all', 'c2'):
        # a single extra workload as the line's headline
        w = extra[args.workload]
        line = {'metric': f'CCQ {args.workload} tokens/s', 'value': w['value'], 'unit': 'tokens/s', 'n_gpus': world,
                'steps': w.get('steps', args.steps), 'warmup': args.warmup, 'ms_per_step': w['ms_per_step'],
                'higher_is_better': True, 'scaling': w.get('scaling', 'weak'), 'vs_baseline': None, 'dtype': 'bf16',
                'data': DATA, 'config': {'workload': w['workload']}, 'roofline': w['roofline'],
                'gpu_launches': w['gpu_launches']}
        print(json.dumps(line), flush=True)
        return
    line = {
        'metric': METRIC,
        'value': main['value'], 'unit': 'tokens/s', 'n_gpus': world, 'steps': args.steps, 'warmup': args.warmup,
        'ms_per_step': main['ms_per_step'], 'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None,
        'dtype': 'bf16', 'data': DATA,
        'config': c2_config(world, B=args.batch),
        'paths': main['paths'],
        'roofline': main['roofline'],
        'clocks': main['clocks'],
        'e2e': main.get('e2e'),
        'gpu_launches': main['gpu_launches'],
        'cpu_baseline': cpu,
    }
    line.update(extra)
    print(json.dumps(line), flush=True)


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
