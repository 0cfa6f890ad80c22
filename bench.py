#!/usr/bin/env python
"""Benchmark of the B200 hot path: pair-biased attention fwd+bwd (headline) and the pair-stack
fusions, printed as one JSON line by rank 0.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
  python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N ...

Headline workload (BASELINE.json's metric, quoted at N_res=512): MSA row attention with pair
bias, N_seq=512 sequences x N_res=512 residues, H=8 heads of d=32, bf16; q, k, v = LN(m) W for a
synthetic MSA m [512, 512, 256] ~ N(0,1) and W ~ N(0, 1/sqrt(256)); bias [8, 512, 512] ~ N(0,1);
upstream gradient ~ N(0,1); seed 0. One step = VoltaMma (with lse) + VoltaMmaBwd (with dBias)
over every sequence; with N GPUs the sequences are split across ranks (strong scaling) and the
dBias partials are summed by an NCCL all-reduce. value = algorithmic FLOPs of the step
(4 N H S^2 d forward + 10 N H S^2 d backward) / device time, max over ranks. L2 is flushed
(a 256 MiB write) before every timed step.

--impl reference times the reference's CPU arithmetic for the same path (the float32 port of
its closed-form oracle, oracle/attention.py) on this host's cores, one bounded sample per step.

The line also carries the e2e leg (the same step from pinned host buffers through the public
API, in 8 chunks of sequences on copy-in / kernel / copy-out streams), the pair fusions on
BASELINE configs[3] and the large-protein inference leg; --no-e2e, --no-fusions,
--no-inference and --no-cpu skip legs, and --only-fusion NAME runs one fusion line alone (the
form the ncu captures use).
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, 'colabfold-legacy-kernels_b200', 'src'))
sys.path.insert(0, ROOT)

METRIC = ("attn fwd+bwd TFLOP/s & %bf16 peak at N_res=512; pair-fusion GB/s & %HBM, "
          "1/2/4/8 GPU")
N_SEQ, N_RES, HEADS, HEAD_DIM, C_M = 512, 512, 8, 32, 256
FALLBACK_PEAKS = {'hbm_gbs': 6650.0, 'bf16_tflops': 1590.0, 'bf16_tflops_sustained': 1400.0}
CPU_SAMPLE_SEQ = 32      # sequences per CPU step (of 512)


def peaks():
    path = os.path.join(ROOT, 'MEASURED_PEAKS.json')
    try:
        with open(path) as f:
            p = json.load(f)
        return p, 'measured'
    except (OSError, ValueError):
        return dict(FALLBACK_PEAKS), 'fallback'


def attn_flops(n, h=HEADS, s=N_RES, d=HEAD_DIM):
    return 14.0 * n * h * s * s * d


# ------------------------------------------------------------------------------------------
# CPU: the reference's arithmetic (float32 port of its closed form, and the fusion oracle), on
# all host cores: a spawn pool of one single-threaded process per core, each given a share of a
# bounded sample of batch rows (rows are independent, so the sample scales by rows)
# ------------------------------------------------------------------------------------------
TRI_RES, TRI_H, TRI_MASKED = 384, 4, 38
CPU_SAMPLE = {'msa': 32, 'triangle': 48, 'inference': 16}   # batch rows per CPU step
CPU_FUSION_ROWS = 1 << 16                   # rows of the pair per CPU fusion sample


def _attn_shape(kind):
    if kind == 'msa':
        return HEADS, N_RES, 0
    if kind == 'triangle':
        return TRI_H, TRI_RES, TRI_MASKED
    return BIG_H, BIG_RES, BIG_RES - int(BIG_RES * 0.95)


def _cpu_worker(args):
    """Seconds for n batch rows of one attention workload (inputs made before the clock)."""
    import numpy as np
    from oracle import attention as oa
    kind, seed, n = args
    h, s, masked = _attn_shape(kind)
    rng = np.random.default_rng(seed)
    q, k, v, dout = (rng.standard_normal((n, h, s, HEAD_DIM), dtype=np.float32)
                     for _ in range(4))
    bias = rng.standard_normal((h, s, s), dtype=np.float32)
    km = np.ones((n, s), np.uint8)
    if masked:
        km[:, s - masked:] = 0
    t0 = time.perf_counter()
    if kind == 'inference':
        oa.attention_forward_f32(q, k, v, bias, km, HEAD_DIM ** -0.5)
    else:
        oa.attention_grads_f32(q, k, v, bias, km, dout, HEAD_DIM ** -0.5)
    return time.perf_counter() - t0


def _fusion_cpu_inputs(name, rows, rng):
    """Inputs of one pair fusion for `rows` rows (BASELINE configs[3] distributions) and the
    oracle call that computes it."""
    import numpy as np
    from oracle import fused as of
    f = np.float32
    x = rng.standard_normal((rows, C_Z), dtype=f)
    ones, zeros = np.ones(C_Z, f), np.zeros(C_Z, f)
    w = C_Z ** -0.5
    if name.startswith('ln_gated_dual_proj'):
        ci = int(name.split('=')[1])
        wpT, wgT = (rng.standard_normal((2 * ci, C_Z), dtype=f) * w for _ in range(2))
        bp, bg, mask = np.zeros(2 * ci, f), np.ones(2 * ci, f), np.ones(rows, f)
        return lambda: of.ln_gdp(x, ones, zeros, wpT, bp, wgT, bg, mask, 1e-5, 'bf16', 128)
    if name.startswith('trimul_epilogue'):
        c = int(name.split('=')[1].split()[0])
        x_cm = rng.standard_normal((c, rows), dtype=f)
        woT = rng.standard_normal((C_Z, c), dtype=f) * c ** -0.5
        wgT = rng.standard_normal((C_Z, C_Z), dtype=f) * w
        bo, bg = np.zeros(C_Z, f), np.zeros(C_Z, f)
        return lambda: of.trimul_epilogue(x_cm, x, ones, zeros, np.ones(c, f), np.zeros(c, f),
                                          woT, bo, wgT, bg, None, 1e-5, True, 'bf16', 128)
    if name.startswith('ln_projection'):
        wT, wbT = rng.standard_normal((512, C_Z), dtype=f) * w, \
            rng.standard_normal((4, C_Z), dtype=f) * w
        return lambda: of.ln_projection(x, ones, zeros, wT, wbT, None, 1e-5, 'bf16', 128)
    if name.startswith('output_projection'):
        woT, bo = rng.standard_normal((C_Z, C_Z), dtype=f) * w, np.zeros(C_Z, f)
        res = rng.standard_normal((rows, C_Z), dtype=f)
        return lambda: of.output_projection(x, woT, bo, res, None, 'bf16', 128)
    if name.startswith('gated_dual_proj'):
        wp, wg = (rng.standard_normal((C_Z, C_Z), dtype=f) * w for _ in range(2))
        b0, mask = np.zeros(C_Z, f), np.ones(rows, f)
        return lambda: of.gdp(x, wp, b0, wg, b0, mask, 0, 'bf16')
    if name.startswith('layer_norm'):
        return lambda: of.layer_norm_one_pass(x, ones, zeros, 1e-5, 'bf16')
    if name.startswith('transition'):
        w1T = rng.standard_normal((512, C_Z), dtype=f) * w
        w2T = rng.standard_normal((512 * C_Z,), dtype=f) * 512 ** -0.5
        b1, b2 = np.zeros(512, f), np.zeros(C_Z, f)
        return lambda: of.transition(x, ones, zeros, w1T, b1, w2T, b2, None, 1e-5, True, 'bf16',
                                     128)
    raise KeyError(name)


# The next rows (the triangle contraction, the outer product mean, VoltaGdp at the channel-major
# width) on BASELINE configs[3]'s pair: name -> (units of the workload, the unit's name, units a
# CPU worker takes). Algorithmic bytes and FLOPs in next_row_work().
OPM_K, OPM_C, OPM_F = 16 * 32, 32, 128   # 16 MSA rows x 32 channels, c_z out
NEXT_ROWS = {
    'trimul_contract outgoing C=128': (128, 'channels', 1),
    'trimul_contract incoming C=128': (128, 'channels', 1),
    'opm_update K=512 F=128': (768, 'rows of b', 8),
    'opm_outer C=E=32 F=128': (768, 'rows of b', 4),
    'gated_dual_proj K=128 N=256 sigmoid': (768 * 768, 'rows', 1 << 14),
}


def next_row_work(name, units):
    """(algorithmic bytes, FLOPs) of `units` units of a next-row workload: every input read once
    and every output written once (16-bit; float32 x_cm and OPM norms), intermediates none."""
    n = PAIR
    if name.startswith('trimul_contract'):
        return units * n * n * (2 + 2 + 4), 2.0 * units * n ** 3
    if name.startswith('opm_update'):
        return (units * OPM_K * 2 + OPM_K * n * OPM_F * 2 + 2 * units * n * OPM_F * 2 +
                units * n * 4), 2.0 * units * OPM_K * n * OPM_F
    if name.startswith('opm_outer'):
        ce = OPM_C * 32
        return ((16 * units * OPM_C + 16 * n * 32 + OPM_F * ce + units * n * OPM_F) * 2,
                2.0 * units * n * ce * (16 + OPM_F))
    if name.startswith('gated_dual_proj'):
        return units * (C_Z * 2 + 256 * 2 + 2) + 2 * C_Z * 256 * 2, 2.0 * units * C_Z * 256 * 2
    raise KeyError(name)


def _next_cpu_inputs(name, units, rng):
    """Inputs of `units` units of a next-row workload and the oracle call that computes them."""
    import numpy as np
    from oracle import fused as of
    f = np.float32
    n = PAIR
    if name.startswith('trimul_contract'):
        a = rng.standard_normal((units, n, n), dtype=f)
        b = rng.standard_normal((units, n, n), dtype=f)
        return lambda: of.trimul_contract(a, b, 'incoming' in name)
    if name.startswith('opm_update'):
        lhs = rng.standard_normal((units, OPM_K), dtype=f)
        t = rng.standard_normal((OPM_K, n, OPM_F), dtype=f) * OPM_K ** -0.5
        bias, norm = np.zeros(OPM_F, f), np.ones((units, n), f)
        res = rng.standard_normal((units, n, OPM_F), dtype=f)
        return lambda: of.opm_update(lhs, t, bias, norm, res, 1e-3, 'bf16')
    if name.startswith('opm_outer'):
        left = rng.standard_normal((16, units, OPM_C), dtype=f)
        right = rng.standard_normal((16, n, 32), dtype=f)
        wT = rng.standard_normal((OPM_F, OPM_C * 32), dtype=f) * (OPM_C * 32) ** -0.5
        return lambda: of.opm_outer(left, right, wT, 'bf16')
    if name.startswith('gated_dual_proj'):
        x = rng.standard_normal((units, C_Z), dtype=f)
        wp, wg = (rng.standard_normal((C_Z, 256), dtype=f) * C_Z ** -0.5 for _ in range(2))
        b0, mask = np.zeros(256, f), np.ones(units, f)
        return lambda: of.gdp(x, wp, b0, wg, b0, mask, 0, 'bf16')
    raise KeyError(name)


def _cpu_next_worker(args):
    import numpy as np
    name, seed, units = args
    fn = _next_cpu_inputs(name, units, np.random.default_rng(seed))
    t0 = time.perf_counter()
    fn()
    return time.perf_counter() - t0


def _cpu_fusion_worker(args):
    import numpy as np
    name, seed, rows = args
    fn = _fusion_cpu_inputs(name, rows, np.random.default_rng(seed))
    t0 = time.perf_counter()
    fn()
    return time.perf_counter() - t0


class CpuBaseline:
    """A spawn pool of one process per host core, each running single-threaded BLAS."""

    def __init__(self):
        import multiprocessing as mp
        self.cores = os.cpu_count() or 1
        for var in ('OMP_NUM_THREADS', 'OPENBLAS_NUM_THREADS', 'MKL_NUM_THREADS'):
            os.environ[var] = '1'
        self.pool = mp.get_context('spawn').Pool(self.cores)
        self.pool.map(_cpu_worker, [('msa', 0, 1)] * self.cores)  # import and warm every worker

    def step(self, kind='msa', rows=None):
        """Seconds of wall time for `rows` batch rows of a workload, spread over the pool."""
        rows = CPU_SAMPLE[kind] if rows is None else rows
        t0 = time.perf_counter()
        self.pool.map(_cpu_worker, [(kind, i, 1) for i in range(rows)])
        return time.perf_counter() - t0

    def fusion_step(self, name, rows=CPU_FUSION_ROWS):
        share = -(-rows // self.cores)
        t0 = time.perf_counter()
        self.pool.map(_cpu_fusion_worker, [(name, i, share) for i in range(self.cores)])
        return time.perf_counter() - t0, share * self.cores

    def next_step(self, name):
        share = NEXT_ROWS[name][2]
        t0 = time.perf_counter()
        self.pool.map(_cpu_next_worker, [(name, i, share) for i in range(self.cores)])
        return time.perf_counter() - t0, share * self.cores

    def close(self):
        self.pool.close()
        self.pool.join()


def cpu_attention_line(cpu, kind, steps, warmup):
    """The CPU baseline of an attention workload: TFLOP/s of the reference's closed form (float32
    port) over a bounded sample of batch rows."""
    for _ in range(warmup):
        cpu.step(kind)
    times = [cpu.step(kind) for _ in range(steps)]
    t = sum(times) / len(times)
    n = CPU_SAMPLE[kind]
    h, s, _ = _attn_shape(kind)
    flops = (4.0 if kind == 'inference' else 14.0) * n * h * s * s * HEAD_DIM
    total = {'msa': N_SEQ, 'triangle': TRI_RES, 'inference': BIG_RES}[kind]
    what = 'fwd only' if kind == 'inference' else 'fwd+bwd'
    return {'value': flops / t / 1e12, 'unit': 'TFLOP/s', 'cores': cpu.cores, 'kind': 'port',
            'sample': '%d of %d batch rows per step (%s, float32 numpy, one process per core), '
                      '%.2f s per step' % (n, total, what, t)}, t


def cpu_fusion_lines(cpu):
    """The CPU baseline of each pair fusion: GB/s of the fusion oracle (oracle/fused.py, the
    restatement of the reference kernels) over a bounded sample of rows, algorithmic bytes as the
    GPU lines count them."""
    out = {}
    for name, per_row in FUSION_BYTES_PER_ROW.items():
        t, rows = cpu.fusion_step(name)
        out[name] = {'value': per_row * rows / t / 1e9, 'unit': 'GB/s', 'cores': cpu.cores,
                     'kind': 'port',
                     'sample': '%d of %d rows (numpy oracle, one process per core), %.2f s'
                               % (rows, PAIR * PAIR, t)}
    return out


def cpu_next_lines(cpu):
    """The CPU baseline of each next-row workload: the oracle over a bounded sample of its units,
    GB/s and TFLOP/s as the GPU lines count them."""
    out = {}
    for name, (total, unit, _) in NEXT_ROWS.items():
        t, units = cpu.next_step(name)
        nbytes, flops = next_row_work(name, units)
        out[name] = {'value': nbytes / t / 1e9, 'unit': 'GB/s', 'TFLOP/s': flops / t / 1e12,
                     'cores': cpu.cores, 'kind': 'port',
                     'sample': '%d of %d %s (numpy oracle, one process per core), %.2f s'
                               % (units, total, unit, t)}
    return out


def cpu_sample_line(steps, warmup):
    cpu = CpuBaseline()
    try:
        return cpu_attention_line(cpu, 'msa', steps, warmup)
    finally:
        cpu.close()


def run_reference(args):
    rank = int(os.environ.get('RANK', '0'))
    if rank != 0:
        return
    line, t = cpu_sample_line(max(args.steps, 1), max(args.warmup, 0))
    out = {'impl': 'reference', 'metric': METRIC, 'value': line['value'], 'unit': 'TFLOP/s',
           'n_gpus': args.gpus, 'steps': args.steps, 'warmup': args.warmup,
           'ms_per_step': t * 1e3, 'higher_is_better': True, 'scaling': 'strong',
           'vs_baseline': None, 'dtype': 'f32', 'data': 'synthetic',
           'config': workload_config(1),
           'cpu_baseline': line,
           'e2e': {'value': line['value'], 'unit': 'TFLOP/s', 'h2d_bytes_per_step': 0,
                   'd2h_bytes_per_step': 0}}
    print(json.dumps(out), flush=True)


def workload_config(world):
    return {'workload': 'MSA row attention fwd+bwd with pair bias and dBias (BASELINE '
                        'configs[2]): N_seq=512, N_res=512, H=8, d=32, bf16',
            'N_seq': N_SEQ, 'N_res': N_RES, 'H': HEADS, 'd': HEAD_DIM, 'c_m': C_M,
            'step': 'VoltaMma(want_lse) + VoltaMmaBwd(want_dbias)' +
                    (' + NCCL dBias all-reduce' if world > 1 else ''),
            'parallelism': 'dp%d over sequences' % world,
            'l2': 'flushed before every timed step (256 MiB write)'}


# ------------------------------------------------------------------------------------------
# GPU
# ------------------------------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi sampling of this GPU's clocks and throttle reasons during a timed region."""

    FIELDS = ('clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,'
              'clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,'
              'clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap')

    def __init__(self, bus_id):
        self.proc = None
        try:
            cmd = ['nvidia-smi', '--query-gpu=' + self.FIELDS, '--format=csv,noheader,nounits',
                   '-lms', '200']
            if bus_id:
                cmd += ['-i', bus_id]
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                                         text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], None, set()
        names = ('hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap')
        for line in out.splitlines():
            f = [x.strip() for x in line.split(',')]
            if len(f) < 8:
                continue
            try:
                sm.append(float(f[0]))
                mx = float(f[1])
            except ValueError:
                continue
            for name, val in zip(names, f[4:8]):
                if val.lower().startswith('active'):
                    reasons.add(name)
        if not sm:
            return None
        return {'sm_mhz': statistics.median(sm), 'sm_max_mhz': mx, 'samples': len(sm),
                'reasons': sorted(reasons)}


def bus_id(torch, dev):
    try:
        p = torch.cuda.get_device_properties(dev)
        return '%08x:%02x:%02x.0' % (p.pci_domain_id, p.pci_bus_id, p.pci_device_id)
    except Exception:  # noqa: BLE001 - older torch without the PCI fields
        return None


def make_inputs(torch, dev, rank, world, n_seq=N_SEQ):
    """Config 3's inputs, generated whole from one seed on every rank, then this rank's slice
    (the first n_seq sequences when a profiling run asks for fewer)."""
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    bf = torch.bfloat16
    m = torch.randn(N_SEQ, N_RES, C_M, generator=g, device=dev, dtype=torch.float32)
    m = torch.nn.functional.layer_norm(m, (C_M,)).to(bf)
    proj = []
    for _ in range(3):
        w = (torch.randn(C_M, HEADS * HEAD_DIM, generator=g, device=dev) * C_M ** -0.5).to(bf)
        x = (m @ w).view(N_SEQ, N_RES, HEADS, HEAD_DIM).permute(0, 2, 1, 3).contiguous()
        proj.append(x)
    del m
    bias = torch.randn(HEADS, N_RES, N_RES, generator=g, device=dev).to(bf)
    dout = torch.randn(N_SEQ, HEADS, N_RES, HEAD_DIM, generator=g, device=dev).to(bf)
    kmask = torch.ones(N_SEQ, N_RES, dtype=torch.uint8, device=dev)
    per = min(n_seq, N_SEQ) // world
    sl = slice(rank * per, (rank + 1) * per)
    q, k, v = (x[sl].contiguous() for x in proj)
    return q, k, v, bias, kmask[sl].contiguous(), dout[sl].contiguous()


def make_gate(torch, dev, shape):
    """The gate of configs[2]'s gated attention: gate = LN(m) W_g, here a unit-variance bf16
    tensor of q's shape drawn from its own seed (the q/k/v draws stay unchanged), and the gate
    bias 1.0 that the config names, [H, d]."""
    g = torch.Generator(device=dev)
    g.manual_seed(3)
    gate = torch.randn(*shape, generator=g, device=dev).to(torch.bfloat16)
    gb = torch.ones(shape[1], shape[3], dtype=torch.bfloat16, device=dev)
    return gate, gb


def run_ours(args):
    import torch
    import torch.distributed as dist
    from colabfold_legacy_kernels import b200

    rank = int(os.environ.get('RANK', '0'))
    world = int(os.environ.get('WORLD_SIZE', '1'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    torch.cuda.set_device(local)
    dev = torch.device('cuda', local)
    if world > 1:
        import datetime
        dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=300),
                                device_id=dev)
    pk, pk_kind = peaks()

    if args.only_fusion or args.only_next:
        # one pair-fusion or next-row line alone (profiling runs): its warm-up and timed
        # launches only
        flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
        if args.only_fusion:
            res = {'fusions': bench_fusions(torch, b200, dev, rank, world, args.steps,
                                            args.warmup, flush, pk, only=args.only_fusion)}
        else:
            only = None if args.only_next == 'all' else args.only_next
            res = {'next_rows': bench_next_rows(torch, b200, dev, rank, world, args.steps,
                                                args.warmup, flush, pk, only=only)}
        if rank == 0:
            print(json.dumps(res), flush=True)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return

    cpu_line, cpu_more = None, {}
    if rank == 0 and world == 1 and not args.no_cpu:
        # before any CUDA work (the pool is spawned, never forked): the headline's CPU baseline,
        # and those of the triangle, inference and fusion legs that this run includes
        cpu = CpuBaseline()
        try:
            cpu_line, _ = cpu_attention_line(cpu, 'msa', 2, 1)
            if not args.no_triangle:
                cpu_more['triangle'] = cpu_attention_line(cpu, 'triangle', 2, 1)[0]
            if not args.no_inference:
                cpu_more['inference'] = cpu_attention_line(cpu, 'inference', 1, 0)[0]
            if not args.no_fusions:
                cpu_more['fusions'] = cpu_fusion_lines(cpu)
            if not args.no_next:
                cpu_more['next'] = cpu_next_lines(cpu)
        finally:
            cpu.close()

    q, k, v, bias, kmask, dout = make_inputs(torch, dev, rank, world, args.n_seq)
    n_local = q.shape[0]
    scale = HEAD_DIM ** -0.5
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    from colabfold_legacy_kernels import distributed as cd

    def step():
        return cd.attention_fwd_bwd(q, k, v, bias, kmask, dout, scale=scale)[5]

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if b200.device_status() != 0:
        raise RuntimeError('a kernel reported a wait that gave up')

    clocks = ClockSampler(bus_id(torch, dev)) if rank == 0 else None
    time.sleep(0.3)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    for i in range(args.steps):
        flush.fill_(i & 0xff)
        starts[i].record()
        step()
        ends[i].record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop() if clocks else None
    ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / args.steps
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    value = attn_flops(n_local * world) / (ms * 1e-3) / 1e12

    # per-kernel device time (the forward is one launch, the backward call four), L2 flushed
    def timed(fn, reps):
        evs = []
        for _ in range(reps):
            flush.fill_(1)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            evs.append((a, b))
        torch.cuda.synchronize()
        return sum(a.elapsed_time(b) for a, b in evs) / reps

    out, lse = b200.volta_mma(q, k, v, bias, kmask, scale=scale)
    fwd_ms = timed(lambda: b200.volta_mma(q, k, v, bias, kmask, scale=scale), args.steps)
    bwd_ms = timed(lambda: b200.volta_mma_bwd(q, k, v, bias, kmask, out, dout, lse,
                                              scale=scale), args.steps)
    fwd_tf = 4.0 * n_local * HEADS * N_RES ** 2 * HEAD_DIM / (fwd_ms * 1e-3) / 1e12
    bwd_tf = 10.0 * n_local * HEADS * N_RES ** 2 * HEAD_DIM / (bwd_ms * 1e-3) / 1e12

    # the gated training step of configs[2] (gate bias 1.0): the fused gated forward (with lse)
    # and the gate-aware backward, which the reference composes from VoltaMma, an XLA gate and
    # VoltaMmaBwd; same algorithmic FLOPs (the gate's elementwise work is not counted)
    gate, gb = make_gate(torch, dev, q.shape)

    def gated_step():
        y, l2 = b200.volta_mma_gated(q, k, v, gate, gb, bias, kmask, scale=scale)
        return b200.volta_mma_gated_bwd(q, k, v, gate, gb, bias, kmask, y, dout, l2,
                                        scale=scale)

    gated_step()
    gated_ms = timed(gated_step, args.steps)
    del gate, gb

    e2e = None if args.no_e2e else run_e2e(args, torch, dist, b200, dev, world, q, k, v, bias,
                                           kmask, dout, scale)

    tri = None
    if not args.no_triangle:
        tri = bench_triangle(torch, b200, dev, rank, world, args.steps, args.warmup, flush, pk)
        if 'triangle' in cpu_more:
            tri['cpu_baseline'] = cpu_more['triangle']

    fusions = None
    if not args.no_fusions:
        fusions = bench_fusions(torch, b200, dev, rank, world, args.steps, args.warmup, flush,
                                pk)
        for name, line in cpu_more.get('fusions', {}).items():
            if name in fusions:
                fusions[name]['cpu_baseline'] = line

    nxt = None
    if not args.no_next:
        nxt = bench_next_rows(torch, b200, dev, rank, world, args.steps, args.warmup, flush, pk)
        for name, line in cpu_more.get('next', {}).items():
            if name in nxt:
                nxt[name]['cpu_baseline'] = line

    big = None
    if not args.no_inference:
        big = bench_inference(torch, b200, dev, rank, world, max(2, args.steps // 3), 2, flush,
                              pk)
        if 'inference' in cpu_more:
            big['cpu_baseline'] = cpu_more['inference']

    if rank == 0:
        peak = pk['bf16_tflops']
        line = {
            'metric': METRIC, 'value': value, 'unit': 'TFLOP/s', 'n_gpus': world,
            'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': ms,
            'higher_is_better': True, 'scaling': 'strong', 'vs_baseline': None,
            'dtype': 'bf16', 'data': 'synthetic',
            'config': dict(workload_config(world), N_seq=n_local * world),
            'frac_of_bf16_peak': value / (peak * world),
            'roofline': {
                'kernel': 'VoltaMmaBwd (attn_bwd_kernel + row_delta + dq_convert + fills)',
                'bound': 'tensor', 'achieved': bwd_tf, 'peak': peak,
                'peak_kind': pk_kind + ' burst bf16', 'unit': 'TFLOP/s',
                'frac': bwd_tf / peak, 'traffic': BWD_DRAM_BYTES_PER_SEQ * n_local,
                'traffic_unit': 'bytes per launch',
                'traffic_source': 'ncu dram__bytes_read.sum + dram__bytes_write.sum of '
                                  'attn_bwd_kernel at N_seq=256 (526.2 MB), scaled by the '
                                  'sequences processed'},
            'gated_step': {'ms': gated_ms,
                           'TFLOP/s': attn_flops(n_local) / (gated_ms * 1e-3) / 1e12,
                           'what': 'VoltaMma-gated (with lse) + gated backward, gate bias 1.0, '
                                   'this GPU\'s sequences'},
            'kernels': {'fwd_ms': fwd_ms, 'fwd_tflops': fwd_tf, 'fwd_frac': fwd_tf / peak,
                        'bwd_ms': bwd_ms, 'bwd_tflops': bwd_tf, 'bwd_frac': bwd_tf / peak,
                        'sequences_per_gpu': n_local},
            'e2e': e2e,
            # per step: attn_fwd_kernel; row_delta_kernel, bias_transpose_kernel,
            # attn_bwd_kernel, dq_convert_kernel
            'gpu_launches': 5 * args.steps,
            'clocks': clk,
        }
        if cpu_line is not None:
            line['cpu_baseline'] = cpu_line
        if tri is not None:
            line['triangle_384'] = tri
        if fusions is not None:
            line['fusions'] = fusions
        if nxt is not None:
            line['next_rows'] = nxt
        if big is not None:
            line['inference_2048'] = big
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def make_triangle_inputs(torch, dev, rank, world):
    """BASELINE configs[1]'s inputs, generated whole from one seed on every rank: pair z
    [384, 384, 128] ~ N(0,1); q, k, v = LN(z) W with W ~ N(0, 1/sqrt(128)) reshaped to H=4, d=32
    (starting node: row i attends along j, so batch row i holds q[i, h, j, :]); bias
    [4, 384, 384] = LN(z) W_b; the last 38 residues masked as keys; upstream gradient ~ N(0,1).
    Returns this rank's rows (q, k, v, dout, kmask) and the whole bias."""
    from colabfold_legacy_kernels import distributed as cd
    S, H, d = TRI_RES, TRI_H, HEAD_DIM
    g = torch.Generator(device=dev)
    g.manual_seed(2)
    z = torch.randn(S, S, C_Z, generator=g, device=dev)
    z = torch.nn.functional.layer_norm(z, (C_Z,)).to(torch.bfloat16)
    proj = []
    for _ in range(3):
        w = (torch.randn(C_Z, H * d, generator=g, device=dev) * C_Z ** -0.5).to(torch.bfloat16)
        proj.append((z @ w).view(S, S, H, d).permute(0, 2, 1, 3).contiguous())
    wb = (torch.randn(C_Z, H, generator=g, device=dev) * C_Z ** -0.5).to(torch.bfloat16)
    bias = (z @ wb).permute(2, 0, 1).contiguous()
    dout = torch.randn(S, H, S, d, generator=g, device=dev).to(torch.bfloat16)
    kmask = torch.ones(S, S, dtype=torch.uint8, device=dev)
    kmask[:, S - TRI_MASKED:] = 0
    a, b = cd.row_range(S, world, rank)
    q, k, v = (x[a:b].contiguous() for x in proj)
    return q, k, v, bias, kmask[a:b].contiguous(), dout[a:b].contiguous()


def bench_triangle(torch, b200, dev, rank, world, steps, warmup, flush, pk):
    """triangle attention (starting node) fwd+bwd with dBias reduced over
    the 384 rows, rows sharded across ranks with the NCCL dBias all-reduce; the step is VoltaMma
    (with lse) + VoltaMmaBwd (the gate is applied outside these targets, as the reference
    composes it). TFLOP/s over device time (max over ranks), L2 flushed before every step."""
    import torch.distributed as dist
    from colabfold_legacy_kernels import distributed as cd
    q, k, v, bias, kmask, dout = make_triangle_inputs(torch, dev, rank, world)
    scale = HEAD_DIM ** -0.5

    def step():
        return cd.attention_fwd_bwd(q, k, v, bias, kmask, dout, scale=scale)[5]

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    evs = []
    for _ in range(steps):
        flush.fill_(7)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        step()
        e1.record()
        evs.append((e0, e1))
    torch.cuda.synchronize()
    ms = sum(x.elapsed_time(y) for x, y in evs) / steps
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    flops = 14.0 * TRI_RES * TRI_H * TRI_RES ** 2 * HEAD_DIM
    tf = flops / (ms * 1e-3) / 1e12
    if b200.device_status() != 0:
        raise RuntimeError('a kernel reported a wait that gave up')
    return {'ms': ms, 'TFLOP/s': tf, 'frac_bf16': tf / (pk['bf16_tflops'] * world),
            'flops': flops, 'config': 'triangle attention (starting node) fwd+bwd with dBias, '
            'pair 384x384, H=4, d=32, last 38 residues masked, rows sharded over %d GPU(s)'
            % world}


PAIR = 768            # pair [768, 768, 128]
C_Z = 128
# algorithmic bytes per row of each pair fusion: every input read once, every output written
# once (bf16; float32 for x_cm), weights (read once per launch) added separately
FUSION_BYTES_PER_ROW = {
    'ln_gated_dual_proj ci=64': C_Z * 2 + 2 + 2 * 64 * 2,
    'ln_gated_dual_proj ci=128': C_Z * 2 + 2 + 2 * 128 * 2,
    'trimul_epilogue C=64 CA=O=128 add_input': 64 * 4 + C_Z * 2 + C_Z * 2,
    'trimul_epilogue C=128 CA=O=128 add_input': 128 * 4 + C_Z * 2 + C_Z * 2,
    'ln_projection n=512 heads=4': C_Z * 2 + 512 * 2 + 4 * 2,
    'output_projection 128->128 + residual': C_Z * 2 * 3,
    'gated_dual_proj K=N=128 sigmoid': C_Z * 2 + C_Z * 2 + 2,
    'layer_norm C=128': C_Z * 2 * 2,
    'transition 128->512->128 add_input': C_Z * 2 * 2,
}


def bench_fusions(torch, b200, dev, rank, world, steps, warmup, flush, pk, only=None):
    """Pair-stack fusions on BASELINE configs[3] (pair [768, 768, 128] ~ N(0,1), M = 589,824
    rows, W ~ N(0, 1/sqrt(128)), bf16), rows sharded across ranks. Algorithmic bytes: every
    input read once and every output written once (bf16; float32 for x_cm and the LN
    parameters), weights once. GB/s = bytes / device time (max over ranks)."""
    import torch.distributed as dist
    M_all = PAIR * PAIR
    M = M_all // world
    g = torch.Generator(device=dev)
    g.manual_seed(1)
    bf = torch.bfloat16

    def rn(*shape, s=1.0, dt=bf):
        return (torch.randn(*shape, generator=g, device=dev) * s).to(dt)

    x = rn(M, C_Z)
    ones = torch.ones(C_Z, device=dev)
    zeros = torch.zeros(C_Z, device=dev)
    keep1 = torch.ones(1, dtype=bf, device=dev)
    mask = torch.ones(M, dtype=bf, device=dev)
    w = C_Z ** -0.5
    ops = []
    for ci in (64, 128):
        wpT, wgT = rn(2 * ci, C_Z, s=w), rn(2 * ci, C_Z, s=w)
        bp, bg = torch.zeros(2 * ci, dtype=bf, device=dev), torch.ones(2 * ci, dtype=bf, device=dev)
        ops.append(('ln_gated_dual_proj ci=%d' % ci,
                    (lambda wpT=wpT, wgT=wgT, bp=bp, bg=bg: b200.volta_ln_gdp(
                        x, ones, zeros, wpT, bp, wgT, bg, mask, eps=1e-5)),
                    M * (C_Z * 2 + 2 + 2 * ci * 2) + 4 * ci * C_Z * 2, 2.0 * M * C_Z * 4 * ci))
    for c in (64, 128):
        x_cm = rn(c, M, dt=torch.float32)
        woT, wgT = rn(C_Z, c, s=c ** -0.5), rn(C_Z, C_Z, s=w)
        bo, bg = torch.zeros(C_Z, dtype=bf, device=dev), torch.zeros(C_Z, dtype=bf, device=dev)
        lsc, lof = torch.ones(c, device=dev), torch.zeros(c, device=dev)
        ops.append(('trimul_epilogue C=%d CA=O=128 add_input' % c,
                    (lambda x_cm=x_cm, woT=woT, wgT=wgT, bo=bo, bg=bg, lsc=lsc, lof=lof:
                     b200.volta_trimul_epilogue(x_cm, x, ones, zeros, lsc, lof, woT, bo, wgT, bg,
                                                keep1, eps=1e-5, add_input=True,
                                                has_keep=False)),
                    M * (c * 4 + C_Z * 2 + C_Z * 2), 2.0 * M * C_Z * (c + C_Z)))
    wT, wbT = rn(512, C_Z, s=w), rn(4, C_Z, s=w)
    ops.append(('ln_projection n=512 heads=4',
                lambda: b200.volta_ln_proj(x, ones, zeros, wT, wbT, keep1, eps=1e-5, n=512,
                                           heads=4, has_keep=False),
                M * (C_Z * 2 + 512 * 2 + 4 * 2), 2.0 * M * C_Z * 516))
    o, woT, bo, res = rn(M, C_Z), rn(C_Z, C_Z, s=w), rn(C_Z, s=0.1), rn(M, C_Z)
    ops.append(('output_projection 128->128 + residual',
                lambda: b200.volta_out_proj(o, woT, bo, res, keep1, has_residual=True,
                                            has_keep=False),
                M * C_Z * 2 * 3, 2.0 * M * C_Z * C_Z))
    gwp, gwg = rn(C_Z, C_Z, s=w), rn(C_Z, C_Z, s=w)
    gbp, gbg = rn(C_Z, s=0.1), rn(C_Z, s=0.1)
    g_out = torch.empty_like(x)
    ops.append(('gated_dual_proj K=N=128 sigmoid',
                lambda: b200.volta_gdp(x, gwp, gbp, gwg, gbg, mask, activation=0, out=g_out),
                M * (C_Z * 2 + C_Z * 2 + 2) + 2 * C_Z * C_Z * 2, 2.0 * M * C_Z * C_Z * 2))
    ln_out = torch.empty_like(x)
    ops.append(('layer_norm C=128',
                lambda: b200.volta_layer_norm(x, ones, zeros, eps=1e-5, out=ln_out),
                M * C_Z * 2 * 2, 0.0))
    w1T, b1 = rn(512, C_Z, s=w), rn(512, s=0.1)
    w2T, b2 = rn(512 * C_Z, s=512 ** -0.5), rn(C_Z, s=0.1)
    ops.append(('transition 128->512->128 add_input',
                lambda: b200.volta_transition(x, ones, zeros, w1T, b1, w2T, b2, keep1, eps=1e-5,
                                              add_input=True, has_keep=False),
                M * C_Z * 2 * 2, 2.0 * M * C_Z * 512 * 2))
    res_out = {}
    for name, fn, nbytes, flops in ops:
        if only is not None and not name.startswith(only):
            continue
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        evs = []
        for _ in range(steps):
            flush.fill_(3)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            evs.append((a, b))
        torch.cuda.synchronize()
        ms = sum(a.elapsed_time(b) for a, b in evs) / steps
        t = torch.tensor([ms], device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        gbs = nbytes * world / (ms * 1e-3) / 1e9
        tf = flops * world / (ms * 1e-3) / 1e12
        res_out[name] = {'ms': ms, 'GB/s': gbs, 'frac_hbm': gbs / (pk['hbm_gbs'] * world),
                         'TFLOP/s': tf, 'frac_bf16': tf / (pk['bf16_tflops'] * world),
                         'bytes': nbytes * world, 'rows': M_all}
    if b200.device_status() != 0:
        raise RuntimeError('a fused kernel reported a wait that gave up')
    return res_out


def bench_next_rows(torch, b200, dev, rank, world, steps, warmup, flush, pk, only=None):
    """The next rows on BASELINE configs[3]'s pair (768 residues, bf16, N(0,1) activations,
    weights ~ N(0, 1/sqrt(fan-in))): the triangle contraction of ln_gdp's ci = 128 halves (both
    edge directions, float32 out), VoltaOpmUpdate (16 MSA rows x 32 channels contracted against
    t [512, 768, 128], norms 1, with the residual), VoltaOpmOuter (16 rows, C = E = 32, F = 128),
    VoltaGdp at the channel-major width K = 128, N = 256 on the pair's rows. Each rank takes its
    share of the leading units. 'roofline_frac' = max(bytes / measured HBM, FLOPs / measured
    bf16 peak) / device time."""
    import torch.distributed as dist
    n = PAIR
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    bf = torch.bfloat16

    def rn(*shape, s=1.0, dt=bf):
        return (torch.randn(*shape, generator=g, device=dev) * s).to(dt)

    ops = []
    for name, (total, _, _) in NEXT_ROWS.items():
        if only is not None and not name.startswith(only):
            continue
        units = total // world
        if name.startswith('trimul_contract'):
            a, b = rn(units, n, n), rn(units, n, n)
            out = torch.empty(units, n, n, device=dev)
            inc = 'incoming' in name
            fn = (lambda a=a, b=b, out=out, inc=inc: b200.trimul_contract(a, b, incoming=inc,
                                                                          out=out))
        elif name.startswith('opm_update'):
            lhs, t = rn(units, OPM_K), rn(OPM_K, n, OPM_F, s=OPM_K ** -0.5)
            bias, norm = torch.zeros(OPM_F, device=dev), torch.ones(units, n, device=dev)
            res, out = rn(units, n, OPM_F), torch.empty(units, n, OPM_F, dtype=bf, device=dev)
            fn = (lambda lhs=lhs, t=t, bias=bias, norm=norm, res=res, out=out:
                  b200.volta_opm_update(lhs, t, bias, norm, res, eps=1e-3, out=out))
        elif name.startswith('opm_outer'):
            left, right = rn(16, units, OPM_C), rn(16, n, 32)
            wT = rn(OPM_F, OPM_C * 32, s=(OPM_C * 32) ** -0.5)
            out = torch.empty(units, n, OPM_F, dtype=bf, device=dev)
            wsn = b200.opm_outer_workspace_size(units, OPM_C, n, 32)
            ws = torch.empty(wsn, dtype=torch.uint8, device=dev)
            fn = (lambda left=left, right=right, wT=wT, out=out, ws=ws:
                  b200.volta_opm_outer(left, right, wT, out=out, workspace=ws))
        else:
            x = rn(units, C_Z)
            wp, wg = rn(C_Z, 256, s=C_Z ** -0.5), rn(C_Z, 256, s=C_Z ** -0.5)
            bp, bg = rn(256, s=0.1), rn(256, s=0.1)
            mask = torch.ones(units, dtype=bf, device=dev)
            out = torch.empty(units, 256, dtype=bf, device=dev)
            fn = (lambda x=x, wp=wp, bp=bp, wg=wg, bg=bg, mask=mask, out=out:
                  b200.volta_gdp(x, wp, bp, wg, bg, mask, activation=0, out=out))
        nbytes, flops = next_row_work(name, units)
        ops.append((name, fn, nbytes, flops))
    res_out = {}
    for name, fn, nbytes, flops in ops:
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        evs = []
        for _ in range(steps):
            flush.fill_(3)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            evs.append((a, b))
        torch.cuda.synchronize()
        ms = sum(a.elapsed_time(b) for a, b in evs) / steps
        t = torch.tensor([ms], device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        gbs = nbytes * world / (ms * 1e-3) / 1e9
        tf = flops * world / (ms * 1e-3) / 1e12
        t_hbm = nbytes / (pk['hbm_gbs'] * 1e9)
        t_tc = flops / (pk['bf16_tflops'] * 1e12)
        res_out[name] = {'ms': ms, 'GB/s': gbs, 'frac_hbm': gbs / (pk['hbm_gbs'] * world),
                         'TFLOP/s': tf, 'frac_bf16': tf / (pk['bf16_tflops'] * world),
                         'bound': 'hbm' if t_hbm >= t_tc else 'tensor',
                         'roofline_frac': max(t_hbm, t_tc) / (ms * 1e-3),
                         'bytes': nbytes * world, 'flops': flops * world}
    if b200.device_status() != 0:
        raise RuntimeError('a next-row kernel reported a wait that gave up')
    return res_out


# DRAM bytes (read + written) of one attn_bwd_kernel launch per sequence of the headline shape,
# from one ncu capture at N_seq=256 (526.20 MB / 256; the contiguous (n, h) schedule the full
# size runs); the full-size launch is larger than the profiling size rule allows and its traffic
# grows with the sequences processed
BWD_DRAM_BYTES_PER_SEQ = 526.20e6 / 256

BIG_RES, BIG_H = 2048, 4


def make_inference_inputs(torch, dev, rank, world, rows=None):
    """BASELINE configs[4]'s inputs: pair z [2048, 2048, 128] ~ N(0,1) generated in row blocks
    from one seed (every rank sees the same pair), q/k/v = LN(z) W reshaped to H=4, d=32 with
    W ~ N(0, 1/sqrt(128)), bias [4, 2048, 2048] ~ N(0,1), the last 5% of residues masked; this
    rank's rows [a, b) of the pair (or `rows` = (a, b) when given)."""
    from colabfold_legacy_kernels import distributed as cd
    S, H, d = BIG_RES, BIG_H, HEAD_DIM
    a, b = rows if rows is not None else cd.row_range(S, world, rank)
    n = b - a
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    w = [(torch.randn(C_Z, H * d, generator=g, device=dev) * C_Z ** -0.5).to(torch.bfloat16)
         for _ in range(3)]
    bias = torch.randn(H, S, S, generator=g, device=dev).to(torch.bfloat16)
    qkv = [torch.empty(n, H, S, d, dtype=torch.bfloat16, device=dev) for _ in range(3)]
    for r0 in range(0, S, 256):
        # rows [r0, r0+256) of the pair, generated in order so every rank sees the same pair
        z = torch.randn(min(256, S - r0), S, C_Z, generator=g, device=dev)
        z = torch.nn.functional.layer_norm(z, (C_Z,)).to(torch.bfloat16)
        lo, hi = max(a, r0), min(b, r0 + z.shape[0])
        if lo < hi:
            zz = z[lo - r0:hi - r0]
            for t, wt in zip(qkv, w):
                t[lo - a:hi - a] = (zz @ wt).view(hi - lo, S, H, d).permute(0, 2, 1, 3)
    kmask = torch.ones(n, S, dtype=torch.uint8, device=dev)
    kmask[:, int(S * 0.95):] = 0
    return qkv[0], qkv[1], qkv[2], bias, kmask


def bench_inference(torch, b200, dev, rank, world, steps, warmup, flush, pk):
    """triangle attention forward only (want_lse off, one-element lse),
    pair [2048, 2048, 128] ~ N(0,1), q/k/v = LN(z) W reshaped to H=4, d=32, bias [4, 2048, 2048]
    ~ N(0,1), the last 5% of residues masked; rows sharded across ranks, then the output
    all-gather. Reports the forward alone and forward + gather (device time, max over ranks)."""
    import torch.distributed as dist
    S, H, d = BIG_RES, BIG_H, HEAD_DIM
    q, k, v, bias, kmask = make_inference_inputs(torch, dev, rank, world)
    one = torch.empty(1, device=dev)
    scale = d ** -0.5

    def fwd():
        return b200.volta_mma(q, k, v, bias, kmask, scale=scale, want_lse=False, lse=one)[0]

    full = torch.empty(S, H, S, d, dtype=torch.bfloat16, device=dev) if world > 1 else None

    def fwd_gather():
        out = fwd()
        if world > 1:
            # rows are equal across ranks for S divisible by the world size
            dist.all_gather_into_tensor(full, out)
        return out

    res = {}
    for name, fn in (('fwd', fwd), ('fwd+all_gather', fwd_gather)):
        if name != 'fwd' and world == 1:
            continue
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        evs = []
        for _ in range(steps):
            flush.fill_(5)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            evs.append((e0, e1))
        torch.cuda.synchronize()
        ms = sum(x.elapsed_time(y) for x, y in evs) / steps
        t = torch.tensor([ms], device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        tf = 4.0 * S * H * S * S * d / (ms * 1e-3) / 1e12
        res[name] = {'ms': ms, 'TFLOP/s': tf, 'frac_bf16': tf / (pk['bf16_tflops'] * world)}
    res['config'] = 'pair 2048x2048, H=4, d=32, fwd only (want_lse off), last 5%% masked, ' \
                    'rows sharded over %d GPU(s)' % world
    return res


E2E_CHUNKS = 8


def run_e2e(args, torch, dist, b200, dev, world, q, k, v, bias, kmask, dout, scale):
    """The same step through the public API from pinned host buffers, inputs copied in and the
    gradients copied out inside the timed region. The batch goes through in E2E_CHUNKS chunks of
    sequences on three streams, so that the copies in, the kernels and the copies out overlap
    (PCIe carries both directions at once): chunk i's q/k/v/dout/mask copy in while chunk i-1
    computes and chunk i-2's dq/dk/dv copy out. The bias is copied once a step; the chunks'
    dBias partial sums add up on the device and dBias is read back after the last chunk."""
    N = q.shape[0]
    nch = E2E_CHUNKS if N % E2E_CHUNKS == 0 else 1
    cn = N // nch
    per_seq = [t.cpu().pin_memory() for t in (q, k, v, kmask, dout)]
    bias_h = bias.cpu().pin_memory()
    devs = [torch.empty_like(t) for t in (q, k, v, kmask, dout)]
    bias_d = torch.empty_like(bias)
    outs_h = [torch.empty(q.shape, dtype=q.dtype).pin_memory() for _ in range(3)]
    dbias_h = torch.empty(bias.shape, dtype=torch.float32).pin_memory()
    dbias_d = torch.empty(bias.shape, dtype=torch.float32, device=dev)
    h2d = sum(t.numel() * t.element_size() for t in per_seq) + bias_h.numel() * 2
    d2h = sum(t.numel() * t.element_size() for t in outs_h) + dbias_h.numel() * 4
    s_in, s_comp, s_out = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
    main = torch.cuda.current_stream()

    def step():
        s_in.wait_stream(main)
        s_comp.wait_stream(main)
        s_out.wait_stream(main)
        ev_in, ev_done = [], []
        with torch.cuda.stream(s_in):
            bias_d.copy_(bias_h, non_blocking=True)
            for c in range(nch):
                for d, h in zip(devs, per_seq):
                    d[c * cn:(c + 1) * cn].copy_(h[c * cn:(c + 1) * cn], non_blocking=True)
                e = torch.cuda.Event()
                e.record(s_in)
                ev_in.append(e)
        for c in range(nch):
            with torch.cuda.stream(s_comp):
                s_comp.wait_event(ev_in[c])
                tq, tk, tv, tm, td = (d[c * cn:(c + 1) * cn] for d in devs)
                out, lse = b200.volta_mma(tq, tk, tv, bias_d, tm, scale=scale)
                dq, dk, dv, dbias = b200.volta_mma_bwd(tq, tk, tv, bias_d, tm, out, td, lse,
                                                       scale=scale)
                if c == 0:
                    dbias_d.copy_(dbias)
                else:
                    dbias_d.add_(dbias)
                e = torch.cuda.Event()
                e.record(s_comp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(e)
                for h, d in zip(outs_h, (dq, dk, dv)):
                    h[c * cn:(c + 1) * cn].copy_(d, non_blocking=True)
                    d.record_stream(s_out)
        with torch.cuda.stream(s_comp):
            if world > 1:
                dist.all_reduce(dbias_d)
            e = torch.cuda.Event()
            e.record(s_comp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(e)
            dbias_h.copy_(dbias_d, non_blocking=True)
        main.wait_stream(s_out)
        main.wait_stream(s_in)
        main.wait_stream(s_comp)

    step()
    torch.cuda.synchronize()
    reps = max(3, min(args.steps, 10))
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    a.record()
    for _ in range(reps):
        step()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / reps
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    return {'value': attn_flops(q.shape[0] * world) / (ms * 1e-3) / 1e12, 'unit': 'TFLOP/s',
            'ms_per_step': ms, 'h2d_bytes_per_step': h2d, 'd2h_bytes_per_step': d2h,
            'chunks': nch, 'streams': 'copy-in / kernels / copy-out',
            'api': 'colabfold_legacy_kernels.b200.volta_mma / volta_mma_bwd (C ABI)'}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=20)
    ap.add_argument('--warmup', type=int, default=5)
    ap.add_argument('--impl', choices=('ours', 'reference'), default='ours')
    ap.add_argument('--no-cpu', action='store_true', help='skip the cpu_baseline sample')
    ap.add_argument('--no-fusions', action='store_true', help='skip the pair-fusion lines')
    ap.add_argument('--only-next', default=None, metavar='NAME',
                    help="run only the next-row line whose name starts with NAME ('all': each)")
    ap.add_argument('--no-next', action='store_true',
                    help='skip the next-row lines (triangle contraction, OPM, wide Gdp)')
    ap.add_argument('--no-e2e', action='store_true', help='skip the host-buffer end-to-end leg')
    ap.add_argument('--no-inference', action='store_true',
                    help='skip the large-protein inference leg (BASELINE configs[4])')
    ap.add_argument('--no-triangle', action='store_true',
                    help='skip the triangle-attention leg (BASELINE configs[1])')
    ap.add_argument('--only-fusion', default=None, metavar='NAME',
                    help='run only the pair-fusion lines whose name starts with NAME (e.g. '
                         'ln_projection, trimul_epilogue, transition) and print them')
    ap.add_argument('--n-seq', type=int, default=N_SEQ,
                    help='sequences of the attention workload (smaller for profiling runs)')
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == 'ours':
        args.warmup = 3
    if args.impl == 'reference':
        run_reference(args)
    else:
        run_ours(args)


if __name__ == '__main__':
    main()
