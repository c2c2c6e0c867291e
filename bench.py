"""Benchmark: fused packed-GGUF dequant GEMV / small-batch GEMM on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: one Q4_K weight matrix of 6144 rows x 2048 cols
(256-element superblocks of 144 bytes: fp16 d and dmin = |N(0,1)|*0.01,
12 random sub-scale bytes, 128 random nibble bytes), f32 activations N(0,1),
token batch swept over 1, 4, 16 and 64.  One step = one pass of the sweep:
four launches, each over a different resident copy of the weights (the
copies rotate through more than twice the L2 capacity, so every launch
streams its weights from HBM).  The metric is algorithmic bytes (packed
weights + f32 activations + f32 outputs) per second.

Arms:
  ours       device-resident timing of the CUDA library (CUDA graph of the K
             timed steps, CUDA events between kernels), plus `e2e` through
             the public gpu.backend.GPUBackend API with host activations and
             host outputs, and (rank 0, N=1) the single-thread CPU oracle on a
             bounded row sample as `cpu_baseline`.
  reference  the reference's CPU implementation of the path -- its Vx
             kernels cannot be compiled here, so the C restatement in
             oracle/ (OpenMP build, all host cores) -- on a row sample.

Multi-GPU: the path does not shard (a single projection), so N GPUs run N
independent replicas ("replicas only"); torch.distributed over gloo carries
only the barrier and the max-over-ranks of the device times.
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path[:0] = [str(ROOT), str(ROOT / 'glm-vx_b200')]

METRIC = 'fused dequant-GEMV HBM GB/s vs 8 TB/s peak'
KIND, ROWS, COLS = 12, 6144, 2048           # Q4_K
BATCHES = (1, 4, 16, 64)
BLOCK, BLOCK_BYTES = 256, 144
WEIGHT_BYTES = ROWS * (COLS // BLOCK) * BLOCK_BYTES  # 7,077,888
# dram bytes per launch from the committed ncu capture (profiles/), None until captured.
NCU_TRAFFIC = {}


def algorithmic_bytes(batch, rows=ROWS):
    return rows * (COLS // BLOCK) * BLOCK_BYTES + batch * COLS * 4 + batch * rows * 4


def synthetic_q4k(rows, seed=0):
    """Config-1 synthetic Q4_K superblocks."""
    rng = np.random.default_rng(seed)
    blocks = rows * (COLS // BLOCK)
    raw = rng.integers(0, 256, size=(blocks, BLOCK_BYTES), dtype=np.uint8)
    d = (np.abs(rng.normal(size=(blocks, 2))) * 0.01).astype(np.float16)
    raw[:, 0:4] = d.view(np.uint8).reshape(blocks, 4)
    return raw.reshape(-1)


def peaks():
    try:
        data = json.loads((ROOT / 'MEASURED_PEAKS.json').read_text())
        return float(data['hbm_gbs']), 'measured'
    except (OSError, KeyError, ValueError):
        return 6650.0, 'fallback'


# ----------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampled every 100 ms; keeps samples inside marked windows."""
    FIELDS = ('timestamp,clocks.sm,clocks.max.sm,utilization.gpu,clocks_event_reasons.hw_slowdown,'
              'clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,'
              'clocks_event_reasons.sw_power_cap')
    NAMES = ('hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap')

    def __init__(self, gpu_index):
        self.samples, self.windows, self.proc = [], [], None
        try:
            self.proc = subprocess.Popen(['nvidia-smi', '-i', str(gpu_index), f'--query-gpu={self.FIELDS}',
                                          '--format=csv,noheader,nounits', '-lms', '100'],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(',')]
            if len(parts) >= 8:
                self.samples.append((time.time(), parts))

    def window(self, t0, t1):
        self.windows.append((t0 - 0.15, t1 + 0.15))

    def summary(self):
        time.sleep(0.25)
        if self.proc:
            self.proc.terminate()
        picked = [p for t, p in self.samples if any(a <= t <= b for a, b in self.windows)]
        if not picked and self.samples:
            picked = [p for _, p in self.samples]
        if not picked:
            return {'sm_mhz': None, 'sm_max_mhz': None, 'reasons': ['nvidia-smi unavailable']}
        sm = [float(p[1]) for p in picked if p[1].replace('.', '').isdigit()]
        mx = [float(p[2]) for p in picked if p[2].replace('.', '').isdigit()]
        reasons = sorted({n for p in picked for n, v in zip(self.NAMES, p[4:8]) if v.lower() == 'active'})
        return {'sm_mhz': statistics.median(sm) if sm else None, 'sm_max_mhz': max(mx) if mx else None,
                'reasons': reasons, 'samples': len(picked)}


# ------------------------------------------------------------ distributed
class Ranks:
    def __init__(self):
        self.rank = int(os.environ.get('RANK', 0))
        self.world = int(os.environ.get('WORLD_SIZE', 1))
        self.local = int(os.environ.get('LOCAL_RANK', 0))
        self.dist = None
        if self.world > 1:
            import datetime
            import torch.distributed as dist
            dist.init_process_group('gloo', timeout=datetime.timedelta(seconds=300))
            self.dist = dist

    def barrier(self):
        if self.dist:
            self.dist.barrier()

    def max(self, value):
        if not self.dist:
            return value
        import torch
        t = torch.tensor([float(value)], dtype=torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.dist:
            self.dist.destroy_process_group()


# ------------------------------------------------------------ CPU oracle
def oracle_sweep(lib_path, rows, deadline_s, steps=None):
    """Run the config-1 sweep on a `rows`-row prefix through the oracle's
    reference C ABI.  Returns (bytes processed, seconds, steps)."""
    from kernels.backend import VxBackend
    cpu = VxBackend(str(lib_path))
    raw = synthetic_q4k(rows, seed=0)
    xs = {b: np.random.default_rng(b).normal(size=(b, COLS)).astype(np.float32) for b in BATCHES}
    done, nbytes, t0 = 0, 0, time.perf_counter()
    while (steps is None and (done == 0 or time.perf_counter() - t0 < deadline_s)) or (steps is not None and done < steps):
        for b in BATCHES:
            if b == 1:
                cpu.packed_matvec(raw, KIND, (rows, COLS), xs[b][0])
            else:
                cpu.packed_linear_batch(raw, KIND, (rows, COLS), xs[b])
            nbytes += algorithmic_bytes(b, rows)
        done += 1
    return nbytes, time.perf_counter() - t0, done


def run_reference(args, ranks):
    """The reference arm: the CPU implementation of the path on host cores."""
    if ranks.rank != 0:
        return 0
    from oracle import loader
    cores = len(os.sched_getaffinity(0))
    os.environ['OMP_NUM_THREADS'] = str(cores)
    lib = loader.parallel()
    sample_rows = 768  # 1/8 of the matrix per step keeps K steps within minutes
    oracle_sweep(lib, sample_rows, 0, steps=args.warmup)
    nbytes, secs, steps = oracle_sweep(lib, sample_rows, 0, steps=args.steps)
    value = nbytes / secs / 1e9
    sample = f'{sample_rows} of {ROWS} rows per step, batches {list(BATCHES)}; C restatement of the Vx kernels (OpenMP)'
    line = {
        'impl': 'reference', 'metric': METRIC, 'value': value, 'unit': 'GB/s', 'n_gpus': args.gpus,
        'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': secs / steps * 1e3, 'higher_is_better': True,
        'scaling': 'weak', 'vs_baseline': None, 'dtype': 'f32', 'data': 'synthetic',
        'config': {'workload': 'config1_q4_k_6144x2048_batch_sweep', 'rows_sampled': sample_rows,
                   'batches': list(BATCHES), 'parallelism': 'host cores'},
        'cpu_baseline': {'value': value, 'unit': 'GB/s', 'cores': cores, 'kind': 'port', 'sample': sample},
        'e2e': {'value': value, 'unit': 'GB/s', 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- ours
def run_ours(args, ranks):
    import ctypes as C
    from gpu import runtime as rt
    from gpu.backend import GPUBackend, PackedWeight

    dev = rt.Device(ranks.local)
    lib = rt.library()
    stream = rt.Stream()
    copies = max(4, math.ceil(2.5 * dev.l2_bytes / WEIGHT_BYTES))
    stride = (WEIGHT_BYTES + 255) // 256 * 256
    raw = synthetic_q4k(ROWS, seed=0)
    wbuf = rt.DeviceBuffer(stride * copies)
    for c in range(copies):
        wbuf.upload(raw, stream.handle, offset=c * stride)
    xs = {b: np.random.default_rng(b).normal(size=(b, COLS)).astype(np.float32) for b in BATCHES}
    xbuf = {b: rt.DeviceBuffer(xs[b].nbytes) for b in BATCHES}
    obuf = {b: rt.DeviceBuffer(4 * b * ROWS) for b in BATCHES}
    for b in BATCHES:
        xbuf[b].upload(xs[b], stream.handle)
    stream.synchronize()
    paths = {}

    def launch(step):
        for i, b in enumerate(BATCHES):
            w = wbuf.ptr + ((step * len(BATCHES) + i) % copies) * stride
            path = C.c_int32()
            rt.check(lib, lib.glmvx_packed_gemm_path(KIND, obuf[b].ptr, w, xbuf[b].ptr, ROWS, COLS, b,
                                                     stream.handle, C.byref(path)), 'glmvx_packed_gemm')
            paths[b] = path.value

    def capture(fn):
        g = rt.Graph(stream)
        g.begin()
        fn()
        g.end()
        g.launch()  # untimed replay: the first launch of a graph is not timed
        stream.synchronize()
        return g

    def sweep_steps():
        for s in range(args.steps):
            for i, b in enumerate(BATCHES):
                w = wbuf.ptr + ((s * len(BATCHES) + i) % copies) * stride
                rt.check(lib, lib.glmvx_packed_gemm(KIND, obuf[b].ptr, w, xbuf[b].ptr, ROWS, COLS, b,
                                                    stream.handle), 'glmvx_packed_gemm')

    def one_batch(i, b):
        def fn():
            for s in range(args.steps):
                w = wbuf.ptr + ((s * len(BATCHES) + i) % copies) * stride
                rt.check(lib, lib.glmvx_packed_gemm(KIND, obuf[b].ptr, w, xbuf[b].ptr, ROWS, COLS, b,
                                                    stream.handle), 'glmvx_packed_gemm')
        return fn

    start, end = rt.Event(), rt.Event()

    def timed(graph):
        ranks.barrier()
        dev.synchronize()
        t0 = time.time()
        start.record(stream)
        graph.launch()
        end.record(stream)
        end.synchronize()
        t1 = time.time()
        ranks.barrier()
        clocks.window(t0, t1)
        return start.elapsed_ms(end)

    # warm-up, then the timed region: K steps captured as one CUDA graph,
    # bracketed by events on the launching stream.
    for s in range(args.warmup):
        launch(s)
    stream.synchronize()
    graph = capture(sweep_steps)
    clocks = ClockSampler(int(os.environ.get('CUDA_VISIBLE_DEVICES', str(ranks.local)).split(',')[0])
                          if os.environ.get('CUDA_VISIBLE_DEVICES', '').split(',')[0].isdigit() else ranks.local)
    time.sleep(0.3)
    total_ms = ranks.max(timed(graph))
    graph.close()
    dev.check_device_error()
    step_bytes = sum(algorithmic_bytes(b) for b in BATCHES)
    value = ranks.world * step_bytes * args.steps / (total_ms * 1e-3) / 1e9
    # Per-kernel durations: each batch size alone, K back-to-back launches.
    avg = []
    for i, b in enumerate(BATCHES):
        g = capture(one_batch(i, b))
        avg.append(ranks.max(timed(g)) / args.steps)
        g.close()
    avg = np.array(avg)
    dev.check_device_error()

    # e2e through the public API: resident weights, host activations/outputs.
    backend = GPUBackend(ranks.local)
    handles = [PackedWeight(wbuf, KIND, (ROWS, COLS), WEIGHT_BYTES, offset=c * stride, owner=False)
               for c in range(copies)]
    e2e_steps = max(1, min(args.steps, 2000))

    def api_step(s):
        for i, b in enumerate(BATCHES):
            h = handles[(s * len(BATCHES) + i) % copies]
            if b == 1:
                backend.packed_matvec(h, KIND, (ROWS, COLS), xs[b][0])
            else:
                backend.packed_linear_batch(h, KIND, (ROWS, COLS), xs[b])

    for s in range(args.warmup):
        api_step(s)
    ranks.barrier()
    t2 = time.perf_counter()
    w2 = time.time()
    for s in range(e2e_steps):
        api_step(s)
    e2e_s = time.perf_counter() - t2
    clocks.window(w2, time.time())
    e2e_s = ranks.max(e2e_s)
    ranks.barrier()
    e2e_value = ranks.world * step_bytes * e2e_steps / e2e_s / 1e9
    backend.close()

    peak, peak_kind = peaks()
    dom = int(np.argmax(avg))
    b_dom = BATCHES[dom]

    def roof(i):
        b = BATCHES[i]
        achieved = algorithmic_bytes(b) / (avg[i] * 1e-3) / 1e9
        return {'bound': 'hbm', 'achieved': achieved, 'peak': peak, 'unit': 'GB/s', 'frac': achieved / peak,
                'traffic': NCU_TRAFFIC.get(b), 'kernel_batch': b, 'peak_source': peak_kind,
                'avg_launch_us': float(avg[i] * 1e3)}

    line = {
        'metric': METRIC, 'value': value, 'unit': 'GB/s', 'n_gpus': ranks.world, 'steps': args.steps,
        'warmup': args.warmup, 'ms_per_step': total_ms / args.steps, 'higher_is_better': True, 'scaling': 'weak',
        'vs_baseline': None, 'dtype': 'f32', 'data': 'synthetic',
        'config': {'workload': 'config1_q4_k_6144x2048_batch_sweep', 'format': 'Q4_K', 'rows': ROWS, 'cols': COLS,
                   'batches': list(BATCHES), 'global_batch': sum(BATCHES), 'parallelism': f'replicas x{ranks.world}',
                   'l2_policy': f'inputs larger than L2: {copies} rotating weight copies, '
                                f'{copies * WEIGHT_BYTES / 1e6:.0f} MB vs {dev.l2_bytes / 1e6:.0f} MB L2',
                   'kernel_paths': {str(b): paths.get(b) for b in BATCHES},
                   'per_batch_us': {str(b): float(avg[i] * 1e3) for i, b in enumerate(BATCHES)},
                   'per_batch_gbs': {str(b): algorithmic_bytes(b) / (avg[i] * 1e-3) / 1e9
                                     for i, b in enumerate(BATCHES)}},
        'roofline': roof(dom),
        'roofline_gemv_b1': roof(0),
        'e2e': {'value': e2e_value, 'unit': 'GB/s', 'steps': e2e_steps,
                'h2d_bytes_per_step': sum(b * COLS * 4 for b in BATCHES),
                'd2h_bytes_per_step': sum(b * ROWS * 4 for b in BATCHES),
                'api': 'gpu.backend.GPUBackend.packed_matvec / packed_linear_batch (resident PackedWeight)'},
        'gpu_launches': len(BATCHES) * args.steps,
        'clocks': clocks.summary(),
    }
    if ranks.rank == 0 and ranks.world == 1 and not args.no_cpu_baseline:
        from oracle import loader
        sample_rows = 256
        nbytes, secs, steps = oracle_sweep(loader.serial(), sample_rows, args.cpu_seconds)
        line['cpu_baseline'] = {'value': nbytes / secs / 1e9, 'unit': 'GB/s', 'cores': 1, 'kind': 'port',
                                'sample': f'{steps} sweeps (batches {list(BATCHES)}) over a {sample_rows}-row '
                                          f'prefix of the {ROWS}x{COLS} Q4_K matrix, single-thread C oracle'}
    if ranks.rank == 0:
        print(json.dumps(line), flush=True)
    wbuf.close()
    return 0


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=2000)
    ap.add_argument('--warmup', type=int, default=20)
    ap.add_argument('--impl', choices=('ours', 'reference'), default='ours')
    ap.add_argument('--cpu-seconds', type=float, default=10.0)
    ap.add_argument('--no-cpu-baseline', action='store_true')
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error('--warmup must be >= 3')
    ranks = Ranks()
    try:
        return run_reference(args, ranks) if args.impl == 'reference' else run_ours(args, ranks)
    finally:
        ranks.close()


if __name__ == '__main__':
    sys.exit(main())
