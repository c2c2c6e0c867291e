"""Benchmark: IQ1_S routed-MoE decode layer on B200 (+ fused dequant-GEMV GB/s).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline workload (the largest configuration that fits
one GPU): one GLM-MoE-DSA sparse feed-forward layer -- 256 routed experts +
1 shared expert, hidden 6144, moe_intermediate 2048, all IQ1_S (fp16
d = |N(0,1)|*0.02, uniform random qs/qh bytes); F32 router 6144x256
~ N(0, 0.02) with correction bias ~ N(0, 0.01); sigmoid top-8, renormalised,
scale 2.5; SwiGLU.  One step = one layer forward for a decode batch of
TOKENS=32 token rows ~ N(0,1) (the top of the config's 1-32 range).  The
metric is decode tokens per second through the layer; the layer streams its
1.9 GB of experts from HBM (far more than L2), so every step reads weights
from DRAM.  Synthetic, seeded data: the reference publishes no dataset.

Also reported (key `fused_gemv`): BASELINE config 0 (Q8_0 2048x6144, batch 1)
and config 1 (Q4_K 6144x2048, batch 1/4/16/64) fused dequant-GEMV GB/s, and
the FP8 E4M3 block-scaled projection (6144x6144, batch 1), rotating weight
copies beyond L2.  Key `dsa_decode` (N=1): BASELINE config 3, the fused DSA
decode attention (indexer over 32768 cached positions, top-2048, absorbed
MLA with 64 heads x rank 512 + rope 64) for 1 and 16 queries.

Arms:
  ours       device-resident timing (CUDA graph of the K timed steps, CUDA
             events on the launching stream), `e2e` through the public
             gpu.moe.MoELayer.forward API (host activations in, host outputs
             out), and (rank 0, N=1) the single-thread C oracle on a bounded
             token sample as `cpu_baseline`.
  reference  the reference's own Python path for the layer
             (glm_vx GlmMoeDsaModel._feed_forward with its kernels/backend.py
             VxBackend and kernels/packed.py, installed unmodified in
             baseline/_ref) over the OpenMP C restatement of its uncompilable
             Vx kernels, one token per step, all host cores.

Multi-GPU (N>1, one process per GPU under torchrun): the headline is the
same layer EXPERT-PARALLEL over the N GPUs (gpu/ep.py, csrc/ep.cu): 256/N
experts per GPU, router and shared expert replicated, TOKENS rows per GPU
per step, token rows and expert outputs moved by this library's kernels over
peer memory (NVLink), one captured graph of K steps per rank, max over
ranks.  Its line carries the per-rank parity against the full single-GPU
layer (bit-identical expected).  The N independent replicas are reported
beside it (`replicas`).  torch.distributed over gloo carries only barriers,
the max of device times and the one-time swap of IPC handles.
"""
import argparse
import ctypes as C
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
METRIC = 'decode tok/s (1/2/4/8 B200) + fused dequant-GEMV HBM GB/s vs 8 TB/s peak'
EXPERTS, HIDDEN, INTER, TOPK, SCALE, KIND = 256, 6144, 2048, 8, 2.5, 19
TOKENS = 32
PROFILE_EXPERTS = 32
IQ1_BLOCK, IQ1_BYTES = 256, 50
EXPERT_MATRIX_BYTES = INTER * (HIDDEN // IQ1_BLOCK) * IQ1_BYTES  # 2,457,600; gate, up and down are equal


# the full synthetic GLM-MoE-DSA decoder.  Widths from the
# BASELINE line; the remaining architecture fields (DSA indexer every fourth
# layer after the first three, RoPE theta) from the reference's model config.
CONFIG4 = dict(num_hidden_layers=78, first_k_dense_replace=3, hidden_size=6144, vocab_size=154880,
               num_attention_heads=64, q_lora_rank=2048, kv_lora_rank=512, qk_nope_head_dim=192,
               qk_rope_head_dim=64, v_head_dim=256, index_n_heads=32, index_head_dim=128, index_topk=2048,
               index_topk_freq=4, index_skip_topk_offset=3, intermediate_size=12288, moe_intermediate_size=2048,
               n_routed_experts=256, n_shared_experts=1, num_experts_per_tok=8, routed_scaling_factor=2.5,
               rms_norm_eps=1e-5, rope_parameters={'rope_theta': 8000000, 'rope_type': 'default'},
               attention_bias=False, tie_word_embeddings=False)


def traffic_row(workload):
    """roofline.traffic for `workload` from profiles/traffic_per_launch.txt
    (one-pass ncu captures): (bytes per launch, source) or (None, reason)."""
    path = ROOT / 'profiles' / 'traffic_per_launch.txt'
    try:
        for line in path.read_text().splitlines():
            if line.startswith('#') or not line.strip():
                continue
            cols = line.split('\t')
            if cols[0] == workload:
                return float(cols[2]), f'{path.relative_to(ROOT)} row {workload}: {cols[1]}; captured by: {cols[3]}'
    except (OSError, IndexError, ValueError):
        pass
    return None, f'no ncu capture recorded for workload {workload}'


def use_ours():
    sys.path[:0] = [str(ROOT), str(ROOT / 'glm-vx_b200')]


def peaks():
    try:
        data = json.loads((ROOT / 'MEASURED_PEAKS.json').read_text())
        return float(data['hbm_gbs']), 'measured'
    except (OSError, KeyError, ValueError):
        return 6650.0, 'fallback'


def synthetic_layer(seed=0, experts=EXPERTS):
    """BASELINE config-2 weights as host arrays (about 1.9 GB at 256 experts)."""
    rng = np.random.default_rng(seed)

    def iq1(count, rows, cols):
        blocks = count * rows * cols // IQ1_BLOCK
        raw = rng.integers(0, 256, size=(blocks, IQ1_BYTES), dtype=np.uint8)
        raw[:, :2] = (np.abs(rng.normal(size=(blocks, 1))) * 0.02).astype(np.float16).view(np.uint8)
        return raw.reshape(-1)

    return dict(router=(rng.normal(size=(experts, HIDDEN)) * 0.02).astype(np.float32),
                bias=(rng.normal(size=experts) * 0.01).astype(np.float32),
                gate=iq1(experts, INTER, HIDDEN), up=iq1(experts, INTER, HIDDEN), down=iq1(experts, HIDDEN, INTER),
                shared=(iq1(1, INTER, HIDDEN), iq1(1, INTER, HIDDEN), iq1(1, HIDDEN, INTER)))


def layer_bytes(unique_experts, tokens):
    """Algorithmic bytes of one layer forward: every routed expert used at
    least once plus the shared expert (gate, up, down each), the F32 router,
    token rows in and out."""
    return (unique_experts + 1) * 3 * EXPERT_MATRIX_BYTES + EXPERTS * HIDDEN * 4 + 2 * tokens * HIDDEN * 4


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


def gpu_index(local):
    vis = os.environ.get('CUDA_VISIBLE_DEVICES', '').split(',')
    return int(vis[local]) if local < len(vis) and vis[local].strip().isdigit() else local


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


# --------------------------------------------------------- reference arm
class _PackedLayerWeights:
    """The object glm_vx.model expects for packed weights (.linear and a name
    lookup), over host arrays of one synthetic layer."""

    def __init__(self, layer):
        self.layer = layer
        self.gu = INTER * (HIDDEN // IQ1_BLOCK) * IQ1_BYTES
        self.dn = HIDDEN * (INTER // IQ1_BLOCK) * IQ1_BYTES

    def _packed(self, name):
        p = 'model.layers.0.mlp.'
        rest = name[len(p):]
        if rest == 'gate.weight':
            return self.layer['router'].reshape(-1).view(np.uint8), 0, (EXPERTS, HIDDEN)
        shared = rest.startswith('shared_experts.')
        proj = rest.split('.')[-2]
        if shared:
            i = {'gate_proj': 0, 'up_proj': 1, 'down_proj': 2}[proj]
            raw = self.layer['shared'][i]
        else:
            e = int(rest.split('.')[1])
            src = {'gate_proj': 'gate', 'up_proj': 'up', 'down_proj': 'down'}[proj]
            n = self.dn if proj == 'down_proj' else self.gu
            raw = self.layer[src][e * n:(e + 1) * n]
        shape = (HIDDEN, INTER) if proj == 'down_proj' else (INTER, HIDDEN)
        return raw, KIND, shape

    def linear(self, name, x, backend):
        raw, kind, shape = self._packed(name)
        return backend.packed_matvec(raw, kind, shape, x)

    def linear_batch(self, name, x, backend):
        raw, kind, shape = self._packed(name)
        return backend.packed_linear_batch(raw, kind, shape, x)

    def __call__(self, name):
        if name.endswith('e_score_correction_bias'):
            return self.layer['bias']
        raise KeyError(name)


def reference_model(layer, library):
    """One sparse layer of the reference model class, stock code path."""
    from glm_vx.model import GlmMoeDsaModel
    from kernels.backend import VxBackend
    config = dict(num_hidden_layers=1, hidden_size=HIDDEN, num_attention_heads=1, kv_lora_rank=1,
                  qk_nope_head_dim=1, qk_rope_head_dim=2, v_head_dim=1, index_n_heads=1, index_head_dim=2,
                  index_topk=1, mlp_layer_types=['sparse'], indexer_types=['full'], num_experts_per_tok=TOPK,
                  routed_scaling_factor=SCALE, n_shared_experts=1, vocab_size=1)
    return GlmMoeDsaModel(config, _PackedLayerWeights(layer), VxBackend(str(library)), packed_weights=True)


def oracle_ffn(cpu, layer, x):
    """One token through the layer with the reference's semantics
    (glm_vx/model.py:289-324), every primitive on the C oracle `cpu`."""
    gu = INTER * (HIDDEN // IQ1_BLOCK) * IQ1_BYTES
    dn = HIDDEN * (INTER // IQ1_BLOCK) * IQ1_BYTES

    def mlp(g, u, d):
        a = cpu.swiglu(cpu.packed_matvec(g, KIND, (INTER, HIDDEN), x), cpu.packed_matvec(u, KIND, (INTER, HIDDEN), x))
        return cpu.packed_matvec(d, KIND, (HIDDEN, INTER), a)

    ids, w = cpu.route(cpu.matvec(layer['router'], x), layer['bias'], TOPK, SCALE)
    result = np.zeros(HIDDEN, np.float32)
    for slot in np.argsort(ids, kind='stable'):
        e = int(ids[slot])
        result += mlp(layer['gate'][e * gu:(e + 1) * gu], layer['up'][e * gu:(e + 1) * gu],
                      layer['down'][e * dn:(e + 1) * dn]) * float(w[slot])
    return result + mlp(*layer['shared'])


def workload_config():
    """The config dict both arms print for the headline workload."""
    return {'workload': 'config2_iq1_s_moe_decode_layer', 'experts': EXPERTS, 'shared_experts': 1,
            'hidden': HIDDEN, 'moe_intermediate': INTER, 'top_k': TOPK, 'routed_scale': SCALE, 'format': 'IQ1_S',
            'tokens_per_step': TOKENS}


def run_reference(args):
    """The reference arm: the reference's own Python over the C oracle, host cores.

    A step is the headline's step: TOKENS token rows through one full config-2
    layer, here by the reference's grouped path for a chunk of rows
    (glm_vx/prefill.py:44-81 `_feed_forward`: batched router logits, rows
    grouped by expert through packed_linear_batch / batch_v2, ascending-id
    combine, shared expert over the whole chunk).  Under torchrun only rank 0
    works; no process group is created, so no torch import can fix the
    OpenMP runtime at one thread before the oracle library sets its count."""
    if int(os.environ.get('RANK', 0)) != 0:
        return 0
    ref_root = ROOT / 'baseline' / '_ref'
    have_ref = (ref_root / 'glm_vx').exists()
    sys.path[:0] = ([str(ref_root)] if have_ref else []) + [str(ROOT)]
    if not have_ref:
        sys.path.insert(1, str(ROOT / 'glm-vx_b200'))
    cores = len(os.sched_getaffinity(0))
    os.environ['OMP_NUM_THREADS'] = str(cores)
    from oracle import loader
    lib = loader.parallel()
    threads = int(C.CDLL(str(lib)).glm_vx_ref_set_threads(cores))
    layer = synthetic_layer(0)
    if have_ref:
        from glm_vx import prefill
        model = reference_model(layer, lib)
        run = lambda v: prefill._feed_forward(model, 0, v)
        source = 'baseline/_ref glm_vx.prefill._feed_forward + GlmMoeDsaModel + kernels.backend.VxBackend'
    else:  # reference Python not installed: the same semantics composed here, token by token
        from kernels.backend import VxBackend
        cpu = VxBackend(str(lib))
        run = lambda v: np.stack([oracle_ffn(cpu, layer, row) for row in v])
        source = 'reference semantics composed over the oracle (baseline/_ref not installed)'
    x = np.random.default_rng(1).normal(size=(args.steps + args.warmup, TOKENS, HIDDEN)).astype(np.float32)
    for i in range(args.warmup):
        run(x[i])
    t0 = time.perf_counter()
    for i in range(args.steps):
        run(x[args.warmup + i])
    secs = time.perf_counter() - t0
    value = TOKENS * args.steps / secs
    line = {
        'impl': 'reference', 'metric': METRIC, 'value': value, 'unit': 'tok/s', 'n_gpus': args.gpus,
        'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': secs / args.steps * 1e3, 'higher_is_better': True,
        'scaling': 'weak', 'vs_baseline': None, 'dtype': 'f32', 'data': 'synthetic',
        'config': {**workload_config(), 'global_batch': TOKENS, 'parallelism': f'host cores ({threads} OpenMP threads)'},
        'cpu_baseline': {'value': value, 'unit': 'tok/s', 'cores': threads, 'kind': 'port',
                         'sample': f'{TOKENS} token rows per step through one full config-2 layer: {source} over '
                                   f'the OpenMP C restatement of the Vx kernels ({threads} threads reported by the '
                                   'library)'},
        'e2e': {'value': value, 'unit': 'tok/s', 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- ours
def graph_time(rt, stream, fn, reps, ranks=None, clocks=None):
    """Capture `fn` (issuing work on `stream`) `reps` times into a graph, run
    it once untimed, then time one launch with events on the stream."""
    g = rt.Graph(stream)
    g.begin()
    for i in range(reps):
        fn(i)
    g.end()
    g.launch()
    stream.synchronize()
    e0, e1 = rt.Event(), rt.Event()
    if ranks:
        ranks.barrier()
    rt.call('glmvx_device_synchronize')
    t0 = time.time()
    e0.record(stream)
    g.launch()
    e1.record(stream)
    e1.synchronize()
    if clocks:
        clocks.window(t0, time.time())
    if ranks:
        ranks.barrier()
    ms = e0.elapsed_ms(e1)
    g.close()
    return ms


PATH_NAMES = {1: 'stream', 2: 'generic', 5: 'mma_int8', 6: 'gemm_f16', 7: 'mma_int8_col_segments', 8: 'gemm_f16_col_segments',
              9: 'gemm_tcgen05_bf16x3'}


def fused_gemv_sweep(rt, lib, dev, stream, steps, peak):
    """Configs 0 and 1: GB/s of the fused dequant-GEMV/GEMM per launch; for
    token batches on the f16 GEMM also the tensor-core rate (two limbs)."""
    res = {}
    try:
        bf16_peak = float(json.loads((ROOT / 'MEASURED_PEAKS.json').read_text())['bf16_tflops'])
    except (OSError, KeyError, ValueError):
        bf16_peak = 1590.0
    rng = np.random.default_rng(0)
    for name, kind, rows, cols, blk, size, batches in (('config0_q8_0_2048x6144', 8, 2048, 6144, 32, 34, (1,)),
                                                       ('config1_q4_k_6144x2048', 12, 6144, 2048, 256, 144,
                                                        (1, 4, 16, 64))):
        wbytes = rows * (cols // blk) * size
        nblocks = rows * cols // blk
        raw = rng.integers(0, 256, size=(nblocks, size), dtype=np.uint8)
        sc = (np.abs(rng.normal(size=(nblocks, 2))) * 0.01).astype(np.float16).view(np.uint8)
        raw[:, :2 if kind == 8 else 4] = sc[:, :2 if kind == 8 else 4]
        raw = raw.reshape(-1)
        copies = max(4, math.ceil(2.5 * dev.l2_bytes / wbytes))
        stride = (wbytes + 255) // 256 * 256
        wbuf = rt.DeviceBuffer(stride * copies)
        for c in range(copies):
            wbuf.upload(raw, stream.handle, offset=c * stride)
        for b in batches:
            x = rng.normal(size=(b, cols)).astype(np.float32)
            xd, od = rt.DeviceBuffer(x.nbytes), rt.DeviceBuffer(4 * b * rows)
            xd.upload(x, stream.handle)

            def launch(i, b=b, xd=xd, od=od):
                rt.check(lib, lib.glmvx_packed_gemm(kind, od.ptr, wbuf.ptr + (i % copies) * stride, xd.ptr, rows,
                                                    cols, b, stream.handle), 'glmvx_packed_gemm')
            reps = max(20, min(steps, 400))
            for i in range(3):
                launch(i)
            us = graph_time(rt, stream, launch, reps) / reps * 1e3
            path = C.c_int32(-1)
            rt.check(lib, lib.glmvx_packed_gemm_path(kind, od.ptr, wbuf.ptr, xd.ptr, rows, cols, b, stream.handle,
                                                     C.byref(path)), 'glmvx_packed_gemm_path')
            stream.synchronize()
            alg = wbytes + x.nbytes + 4 * b * rows
            line = {'us': us, 'gbs': alg / us / 1e3, 'frac_of_measured_hbm': alg / us / 1e3 / peak,
                    'path': PATH_NAMES.get(path.value, str(path.value)), 'gflops': 2 * rows * cols * b / us / 1e3}
            if path.value == 6:  # f16 tensor-core GEMM: two f16 limbs per activation
                tf = 2 * 2 * rows * cols * b / us / 1e6
                line.update({'tensor_tflops': tf, 'frac_of_measured_bf16': tf / bf16_peak})
            res[f'{name}_b{b}'] = line
            xd.close()
            od.close()
        wbuf.close()
    # FP8 E4M3 block-scaled projection (gpu/fp8.vx contract), 6144x6144, batch 1.
    rows = cols = 6144
    w8 = rng.integers(0, 256, size=rows * cols, dtype=np.uint8)
    w8[(w8 & 0x7F) == 0x7F] = 0x3C
    sc = (np.abs(rng.normal(size=(rows // 128) * (cols // 128))) * 0.02 + 1e-3).astype(np.float32)
    x = rng.normal(size=cols).astype(np.float32)
    wbytes = w8.nbytes
    copies = max(4, math.ceil(2.5 * dev.l2_bytes / wbytes))
    stride = (wbytes + 255) // 256 * 256
    wbuf, sd, xd, od = rt.DeviceBuffer(stride * copies), rt.DeviceBuffer(sc.nbytes), rt.DeviceBuffer(x.nbytes), \
        rt.DeviceBuffer(4 * rows)
    for c in range(copies):
        wbuf.upload(w8, stream.handle, offset=c * stride)
    sd.upload(sc, stream.handle)
    xd.upload(x, stream.handle)

    def launch8(i):
        rt.check(lib, lib.glmvx_fp8_matvec(od.ptr, wbuf.ptr + (i % copies) * stride, sd.ptr, xd.ptr, rows, cols,
                                           stream.handle), 'glmvx_fp8_matvec')
    reps = max(20, min(steps, 400))
    for i in range(3):
        launch8(i)
    us = graph_time(rt, stream, launch8, reps) / reps * 1e3
    alg = wbytes + sc.nbytes + x.nbytes + 4 * rows
    res['fp8_e4m3_6144x6144_b1'] = {'us': us, 'gbs': alg / us / 1e3, 'frac_of_measured_hbm': alg / us / 1e3 / peak}
    for b in (xd, od):
        b.close()
    # The same weights for 16 and 32 tokens through glmvx_fp8_gemm (tcgen05).
    for b in (16, 32):
        xb = rng.normal(size=(b, cols)).astype(np.float32)
        xd, od, path = rt.DeviceBuffer(xb.nbytes), rt.DeviceBuffer(4 * rows * b), C.c_int32(-1)
        xd.upload(xb, stream.handle)

        def launch8b(i):
            rt.check(lib, lib.glmvx_fp8_gemm(od.ptr, wbuf.ptr + (i % copies) * stride, sd.ptr, xd.ptr, rows, cols, b,
                                             C.byref(path), stream.handle), 'glmvx_fp8_gemm')
        for i in range(3):
            launch8b(i)
        us = graph_time(rt, stream, launch8b, reps) / reps * 1e3
        alg = wbytes + sc.nbytes + xb.nbytes + 4 * rows * b
        res[f'fp8_e4m3_6144x6144_b{b}'] = {'us': us, 'gbs': alg / us / 1e3, 'frac_of_measured_hbm': alg / us / 1e3 / peak,
                                          'path': PATH_NAMES.get(path.value, str(path.value)),
                                          'us_per_token_gemv': res['fp8_e4m3_6144x6144_b1']['us']}
        xd.close()
        od.close()
    for b in (wbuf, sd):
        b.close()
    return res


DSA_CONTEXT, DSA_TOPK, DSA_HEADS, DSA_RANK, DSA_ROPE, DSA_IH, DSA_ID = 32768, 2048, 64, 512, 64, 32, 128


def dsa_sweep(rt, lib, backend, stream, steps, peak):
    """Config 3: fused DSA decode attention (gpu/dsa.py DSADecoder) for a
    batch of 1 and 16 decode queries, each over its own resident compressed
    cache of DSA_CONTEXT positions (f32 N(0,1)): indexer scores, stable
    top-2048, absorbed MLA.  `us` is the device time of the fused decode
    (a graph of launches, caches far beyond L2 for B=16; at B=1 the 23 MB of
    keys and selected rows may partly stay in L2 between launches), `e2e_us`
    one DSADecoder.step_pinned() call: inputs copied in from pinned memory,
    the new rows appended, the decode, outputs copied back."""
    from gpu.dsa import DSADecoder
    rng = np.random.default_rng(3)
    T = DSA_CONTEXT
    lat = rng.normal(size=(T, DSA_RANK)).astype(np.float32)
    rk = rng.normal(size=(T, DSA_ROPE)).astype(np.float32)
    ik = rng.normal(size=(T, DSA_ID)).astype(np.float32)
    # per query: every index key, the selected latent + rope rows, queries and outputs
    per_query = 4 * (T * DSA_ID + DSA_TOPK * (DSA_RANK + DSA_ROPE) + DSA_HEADS * (2 * DSA_RANK + DSA_ROPE)
                     + DSA_IH * (DSA_ID + 1) + T + DSA_TOPK)
    # multiply-adds of the f32 algorithm (indexer dots, MLA scores and values)
    fma_per_query = T * DSA_IH * DSA_ID + DSA_HEADS * DSA_TOPK * (2 * DSA_RANK + DSA_ROPE)
    res = {}
    for B in (1, 16):
        dec = DSADecoder(backend, B, T)
        warm = 3
        reps = max(5, min(steps, 20))
        n0 = T - (warm + reps + 2)
        for i in range(B):
            dec.load(i, lat[:n0], rk[:n0], ik[:n0])
        io = dec.pinned_io()
        for k in ('new_latent', 'new_rope', 'new_index_key', 'q_index'):
            io[k][...] = rng.normal(size=io[k].shape)
        io['q_latent'][...] = rng.normal(size=io['q_latent'].shape) * 0.05
        io['q_rope'][...] = rng.normal(size=io['q_rope'].shape) * 0.05
        io['head_weights'][...] = rng.normal(size=io['head_weights'].shape) * DSA_IH ** -0.5
        for _ in range(warm):
            dec.step_pinned()

        def decode(i, dec=dec, B=B):
            rt.check(lib, lib.glmvx_dsa_decode(
                dec._ptr('out'), dec._ptr('selected'), dec._ptr('q_latent'), dec._ptr('q_rope'), dec._ptr('q_index'),
                dec._ptr('head_weights'), dec.latents.ptr, dec.rope_keys.ptr, dec.index_keys.ptr, dec.lens_dev.ptr,
                B, DSA_HEADS, DSA_RANK, DSA_ROPE, DSA_IH, DSA_ID, T, DSA_TOPK, dec.index_scale, dec.scale,
                dec._scratch.ptr, dec._scratch_bytes, stream.handle), 'glmvx_dsa_decode')
        us = graph_time(rt, stream, decode, reps) / reps * 1e3
        t0 = time.perf_counter()
        for _ in range(reps):
            dec.step_pinned()
        e2e_us = (time.perf_counter() - t0) / reps * 1e6
        backend.device.check_device_error()
        alg = B * per_query
        res[f'config3_b{B}'] = {
            'us': us, 'queries_s': B / (us * 1e-6), 'e2e_us': e2e_us, 'e2e_queries_s': B / (e2e_us * 1e-6),
            'gbs': alg / us / 1e3, 'frac_of_measured_hbm': alg / us / 1e3 / peak,
            'algorithmic_tflops': 2 * B * fma_per_query / us / 1e6,
            'algorithmic_bytes': alg, 'context': T, 'topk': DSA_TOPK}
        dec.close()
    return res


def attention_config3(rt, backend, steps, peak):
    """Config 3 with its projections: one DSA attention sub-step of the
    resident decoder (gpu/decoder.py) at config-3 widths (64 heads, q_lora
    2048, kv_lora 512, rope 64, nope 192, v 256, indexer 32 x 128 top-2048,
    RoPE theta 1e6) with Q8_0 random projections (q_a, q_b, kv_a, o_proj,
    indexer wq_b / wk; the indexer head weights F32 and kv_b F32 as the
    reference model keeps them), 1 and 16 queries over 32768 cached
    positions: rmsnorm, projections, indexer, append, top-2048, absorbed MLA,
    o_proj, residual, as a graph replayed per step."""
    from gpu.decoder import ResidentDecoder, SyntheticWeights
    cfg = dict(CONFIG4, num_hidden_layers=1, first_k_dense_replace=1,
               rope_parameters={'rope_theta': 1000000, 'rope_type': 'default'})
    ctx = DSA_CONTEXT
    res = {}
    for B in (1, 16):
        reps = max(3, min(steps, 10))
        dec = ResidentDecoder(backend, cfg, SyntheticWeights(cfg, seed=33, attention_kind=8), batch=B,
                              capacity=ctx + 8 + reps, layers=1)
        try:
            dec.fill_caches(ctx)
            dec.set_tokens(np.arange(B) * 11)
            rt.check(backend.lib, backend.lib.glmvx_embed_rows(dec.x, dec.embed[0], dec.embed[1], dec.tokens, B,
                                                               dec.vocab, dec.hidden, dec.s), 'glmvx_embed_rows')
            g = dec.attention_graph(0)
            for _ in range(3):
                g.launch()
            dec.check()
            e0, e1 = rt.Event(), rt.Event()
            e0.record(backend.stream)
            for _ in range(reps):
                g.launch()
            e1.record(backend.stream)
            e1.synchronize()
            dec.check()
            us = e0.elapsed_ms(e1) / reps * 1e3
            g.close()
        finally:
            dec.close()
        H, Q = cfg['hidden_size'], cfg['q_lora_rank']
        heads, R, P, N, V = 64, 512, 64, 192, 256
        q8 = lambda r, c: r * c // 32 * 34
        proj = (q8(Q, H) + q8(heads * (N + P), Q) + q8(R + P, H) + q8(H, heads * V) + q8(32 * 128, Q) + q8(128, H)
                + 4 * 32 * H + 4 * heads * (N + V) * R)
        per_query = 4 * (ctx * 128 + DSA_TOPK * (R + P))
        alg = proj + B * per_query
        res[f'config3_b{B}'] = {'us': us, 'queries_s': B / (us * 1e-6), 'algorithmic_bytes': alg,
                                'gbs': alg / us / 1e3, 'frac_of_measured_hbm': alg / us / 1e3 / peak,
                                'projection_bytes': proj, 'context': ctx, 'topk': DSA_TOPK}
    res['note'] = ('one attention sub-step of the resident decoder with Q8_0 projections (kv_b and the indexer head '
                   'weights F32 as the reference model keeps them); graph-timed, caches synthetic')
    return res


def decoder_sweep(rt, backend, steps, ranks=None):
    """Config 4 on one GPU: the resident batched greedy decoder (gpu/decoder.py)
    at BASELINE config-4 widths, B=64 sequences whose caches hold 4096
    synthetic positions (a stand-in for prefilling the 4096-token prompts),
    device-generated random weights (IQ1_S experts, Q4_K attention, Q8_0
    embedding / lm_head).  The 78-layer model (~150 GB of experts plus
    ~58 GB of caches) does not fit one GPU, so the step is measured at 4
    layers (3 dense + 1 sparse) and 6 (3 dense + 3 sparse): the sparse layer's
    time is the difference / 2 and the 78-layer step is extrapolated as
    t(4) + 74 * t_sparse (labelled as such)."""
    from gpu.decoder import ResidentDecoder, SyntheticWeights, expert_parallel_moe
    B, ctx = 64, 4096
    N = ranks.world if ranks else 1
    local = B // N
    reps = max(3, min(steps, 10))
    out = {}

    def allgather(data):
        got = [None] * N
        ranks.dist.all_gather_object(got, data)
        return got

    for L in (4, 6):
        factory = expert_parallel_moe(ranks.rank, N, allgather) if N > 1 else None
        dec = ResidentDecoder(backend, CONFIG4, SyntheticWeights(CONFIG4, seed=44), batch=local,
                              capacity=ctx + 16 + reps, layers=L, moe_layer_factory=factory)
        try:
            dec.fill_caches(ctx, seed=1 + (ranks.rank if ranks else 0))
            dec.set_tokens(np.random.default_rng(L * 100 + (ranks.rank if ranks else 0)).integers(
                0, CONFIG4['vocab_size'], local))
            for _ in range(3):
                dec.step()
            dec.check()
            if ranks:
                ranks.barrier()
            e0, e1 = rt.Event(), rt.Event()
            e0.record(backend.stream)
            for _ in range(reps):
                dec.step()
            e1.record(backend.stream)
            e1.synchronize()
            dec.check()
            ms = e0.elapsed_ms(e1) / reps
            out[L] = ranks.max(ms) if ranks else ms
        finally:
            dec.close(barrier=ranks.barrier if N > 1 else None)
    t_sparse = (out[6] - out[4]) / 2
    t78 = out[4] + 74 * t_sparse
    return {'batch': B, 'sequences_per_gpu': local, 'context': ctx, 'ms_per_step_4_layers': out[4],
            'ms_per_step_6_layers': out[6], 'tok_s_6_layers': B / (out[6] * 1e-3), 'sparse_layer_ms': t_sparse,
            'extrapolated_78_layer_ms_per_step': t78, 'extrapolated_78_layer_tok_s': B / (t78 * 1e-3),
            'parallelism': (f'expert x{N} for the sparse layers ({CONFIG4["n_routed_experts"] // N} experts per GPU), '
                            f'data-parallel attention ({local} sequences per GPU)') if N > 1 else 'single GPU',
            'note': 'measured at 4 and 6 layers (3 dense + 1 or 3 sparse); 78 layers extrapolated as '
                    't(4) + 74 * (t(6) - t(4)) / 2 (the full model does not fit one GPU); caches filled '
                    'synthetically, weights random'}


def expert_parallel_step(args, ranks, backend, layer, moe, x, clocks):
    """N>1 headline: the config-2 layer with its 256 experts sharded over the
    N GPUs (gpu/ep.py, csrc/ep.cu: 256/N experts per GPU, router and shared
    expert replicated), TOKENS rows per GPU per step.  Each rank captures K
    steps in one CUDA graph; the ranks' graphs run together (the steps pace
    each other through the mailbox flags); device time per rank from CUDA
    events on the launching stream, max over ranks.  Also: the per-rank
    output against the full single-GPU layer (bit-identical expected), the
    end-to-end rate through ExpertParallelLayer.forward_pinned, per-phase
    times of one un-graphed step, and the bytes that cross NVLink."""
    from gpu import runtime as rt
    from gpu.ep import ExpertParallelLayer, split_layer
    N, r = ranks.world, ranks.rank
    stream = backend.stream
    g, u, d = split_layer(layer, N, r)
    ep = ExpertParallelLayer(backend, r, N, layer['router'], layer['bias'], KIND, g, u, d, EXPERTS, HIDDEN, INTER,
                             TOPK, SCALE, shared=layer['shared'], max_tokens=TOKENS)

    def allgather(data):
        out = [None] * N
        ranks.dist.all_gather_object(out, data)
        return out

    ep.connect_ipc(allgather)
    xd, yd, idd = rt.DeviceBuffer(x.nbytes), rt.DeviceBuffer(x.nbytes), rt.DeviceBuffer(4 * TOKENS * TOPK)
    xd.upload(x, stream.handle)
    stream.synchronize()
    ranks.barrier()
    for _ in range(args.warmup):
        ep.forward_device(yd.ptr, xd.ptr, TOKENS)
    stream.synchronize()
    backend.device.check_device_error()
    ms = ranks.max(graph_time(rt, stream, lambda i: ep.forward_device(yd.ptr, xd.ptr, TOKENS), args.steps, ranks,
                              clocks))
    backend.device.check_device_error()
    value = N * TOKENS * args.steps / (ms * 1e-3)

    # parity: this rank's rows through the expert-parallel step and through
    # the full single-GPU layer (same kernels per token: bytes must agree)
    io = ep.pinned_io(TOKENS)
    np.copyto(io['x'], x)
    y_ep, ids_ep, _ = (a.copy() for a in ep.forward_pinned(TOKENS))
    y_1, ids_1, _ = moe.forward(x)
    rel = float(np.linalg.norm(y_ep - y_1) / np.linalg.norm(y_1))
    mism = float(ids_ep.tolist() != ids_1.tolist()) + float(y_ep.tobytes() != y_1.tobytes())
    worst_rel, worst_mism = ranks.max(rel), ranks.max(mism)

    # end to end through the public API: pinned rows in, pinned outputs out
    e2e_steps = min(max(args.steps, 50), 200)
    for _ in range(3):
        ep.forward_pinned(TOKENS)
    ranks.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        ep.forward_pinned(TOKENS)
    e2e_s = ranks.max(time.perf_counter() - t0)
    h2d, d2h = ep.step_copy_bytes(TOKENS)

    # phases of one un-graphed step (events between them; the wait for the
    # slowest peer lands in the phase that waits)
    ev = [rt.Event() for _ in range(4)]
    sums = np.zeros(3)
    reps = 10
    ranks.barrier()
    for _ in range(reps):
        ev[0].record(stream)
        ep.dispatch(xd.ptr, TOKENS, idd.ptr)
        ev[1].record(stream)
        ep.run_experts(TOKENS)
        ev[2].record(stream)
        ep.combine(yd.ptr, TOKENS)
        ev[3].record(stream)
        ev[3].synchronize()
        sums += [ev[i].elapsed_ms(ev[i + 1]) for i in range(3)]
    backend.device.check_device_error()
    phases = dict(zip(('route_and_dispatch', 'experts_and_return', 'wait_and_combine'), (sums / reps * 1e3).tolist()))

    # bytes per step: this rank's pairs to other ranks (prepared rows out,
    # f32 rows back), and the owner's expert weights (distinct local experts
    # routed by all ranks + the shared expert) read from HBM
    ids = np.empty(TOKENS * TOPK, np.int32)
    idd.download(ids)
    per = EXPERTS // N
    remote = int(np.sum(ids // per != r))
    xstride = ((4 * HIDDEN + 4 * (HIDDEN // 256) + 15) // 16 * 16 + 4 * (HIDDEN // 32) + 255) // 256 * 256
    nvlink = remote * (xstride + 4 * HIDDEN)
    all_ids = allgather(ids.tobytes())
    routed = np.concatenate([np.frombuffer(b, np.int32) for b in all_ids])
    local = len(np.unique(routed[routed // per == r]))
    weight_bytes = (local + 1) * 3 * EXPERT_MATRIX_BYTES + EXPERTS * HIDDEN * 4
    step_s = ms * 1e-3 / args.steps
    res = {'tok_s': value, 'ms_per_step': ms / args.steps, 'steps': args.steps, 'experts_per_gpu': per,
           'tokens_per_gpu': TOKENS,
           'parity': {'max_rel_err_vs_single_gpu_layer': worst_rel, 'ranks_not_bit_identical': worst_mism,
                      'reference': 'gpu.moe.MoELayer (full 256-expert layer on the same rows; pinned to the oracle '
                                   'by tests/test_gpu_moe.py)'},
           'e2e': {'value': N * TOKENS * e2e_steps / e2e_s, 'unit': 'tok/s', 'steps': e2e_steps,
                   'h2d_bytes_per_step': h2d, 'd2h_bytes_per_step': d2h,
                   'api': 'gpu.ep.ExpertParallelLayer.forward_pinned (pinned rows in, pinned outputs + routing out)'},
           'phase_us_rank0_view': phases,
           'nvlink_bytes_per_step_per_gpu': {'out': nvlink - remote * 4 * HIDDEN, 'back': remote * 4 * HIDDEN},
           'owner_distinct_experts': local,
           'hbm_bytes_per_step_per_gpu': weight_bytes,
           'hbm_gbs_per_gpu': weight_bytes / step_s / 1e9,
           'transport': 'own kernels over peer memory: prepared rows stored into the owners\' IPC-mapped mailboxes, '
                        'down-GEMV outputs stored straight back into the senders\' mailboxes, epoch flags with '
                        'system-scope release/acquire (bounded 2 s waits); no NCCL, no host round trip'}
    ranks.barrier()
    for b in (xd, yd, idd):
        b.close()
    ep.close(barrier=ranks.barrier)
    return res


def run_ours(args, ranks):
    use_ours()
    from gpu import runtime as rt
    from gpu.backend import GPUBackend
    from gpu.moe import MoELayer

    backend = GPUBackend(ranks.local)
    dev, lib, stream = backend.device, backend.lib, backend.stream
    layer = synthetic_layer(0)
    moe = MoELayer(backend, layer['router'], layer['bias'], KIND, layer['gate'], layer['up'], layer['down'],
                   HIDDEN, INTER, TOPK, SCALE, shared=layer['shared'])
    rng = np.random.default_rng(100 + ranks.rank)
    xs = {t: rng.normal(size=(t, HIDDEN)).astype(np.float32) for t in (1, 8, TOKENS)}
    bufs = {}
    for t, x in xs.items():
        xd, yd, idd = rt.DeviceBuffer(x.nbytes), rt.DeviceBuffer(x.nbytes), rt.DeviceBuffer(4 * t * TOPK)
        xd.upload(x, stream.handle)
        bufs[t] = (xd, yd, idd)
    stream.synchronize()

    def step(t):
        xd, yd, _ = bufs[t]
        return lambda i: moe.forward_device(yd.ptr, xd.ptr, t)

    clocks = ClockSampler(gpu_index(ranks.local))
    for i in range(args.warmup):
        step(TOKENS)(i)
    stream.synchronize()
    time.sleep(0.3)
    total_ms = ranks.max(graph_time(rt, stream, step(TOKENS), args.steps, ranks, clocks))
    dev.check_device_error()
    value = ranks.world * TOKENS * args.steps / (total_ms * 1e-3)

    # Per decode-batch size: layer time, unique experts, stage breakdown.
    peak, peak_kind = peaks()
    per_tokens, stage_names = {}, ['router_logits', 'routing', 'grouping', 'gate_up', 'down', 'combine']
    for t in xs:
        xd, yd, idd = bufs[t]
        moe.forward_device(yd.ptr, xd.ptr, t, idd.ptr)
        ids = np.empty(t * TOPK, np.int32)
        stream.synchronize()
        idd.download(ids)
        unique = len(np.unique(ids))
        reps = max(5, min(args.steps, 100))
        ms = graph_time(rt, stream, step(t), reps) / reps
        # stage durations (events between the six launches, no graph)
        events = [rt.Event() for _ in range(7)]
        ev_arr = C.cast((C.c_void_p * 7)(*[e.handle for e in events]), C.c_void_p)
        sums = np.zeros(6)
        ws = moe._workspace(t)
        for _ in range(reps):
            rt.check(lib, lib.glmvx_moe_ffn_profiled(
                yd.ptr, xd.ptr, t, HIDDEN, INTER, moe.router_w, moe.router_bias, EXPERTS, TOPK, SCALE, KIND,
                moe.gate, moe.up, moe.down, *moe.shared, ws, moe._ws_bytes, ev_arr, stream.handle), 'moe profiled')
            events[-1].synchronize()
            sums += [events[i].elapsed_ms(events[i + 1]) for i in range(6)]
        stages = dict(zip(stage_names, (sums / reps * 1e3).tolist()))
        alg = layer_bytes(unique, t)
        per_tokens[str(t)] = {'us_per_layer': ms * 1e3, 'tok_s': t / (ms * 1e-3), 'unique_experts': unique,
                              'layer_gbs': alg / (ms * 1e-3) / 1e9, 'stage_us': stages}
    dom_t = per_tokens[str(TOKENS)]
    gu_us = dom_t['stage_us']['gate_up']
    gu_bytes = (dom_t['unique_experts'] + 1) * 2 * EXPERT_MATRIX_BYTES + (TOKENS * TOPK + TOKENS) * 2 * INTER * 4
    achieved = gu_bytes / (gu_us * 1e-6) / 1e9
    traffic = traffic_row(f'config2_t{TOKENS}_gate_up')
    dev.check_device_error()

    # e2e through the public API: token rows in pinned host memory, copied to
    # the device, the layer, outputs copied back to pinned host memory and
    # checked there (MoELayer.forward_pinned), every step.
    e2e_steps = min(max(args.steps, 50), 200)
    e2e_h2d, e2e_d2h = moe.step_copy_bytes(TOKENS)
    np.copyto(moe.pinned_io(TOKENS)['x'], xs[TOKENS])
    for i in range(min(args.warmup, 3)):
        moe.forward_pinned(TOKENS)
    ranks.barrier()
    t0 = time.perf_counter()
    w0 = time.time()
    for _ in range(e2e_steps):
        moe.forward_pinned(TOKENS)
    e2e_s = ranks.max(time.perf_counter() - t0)
    clocks.window(w0, time.time())
    e2e_value = ranks.world * TOKENS * e2e_steps / e2e_s

    gemv = fused_gemv_sweep(rt, lib, dev, stream, args.steps, peak)
    dsa = dsa_sweep(rt, lib, backend, stream, args.steps, peak) if ranks.world == 1 else None
    if dsa is not None:
        dsa['with_projections'] = attention_config3(rt, backend, args.steps, peak)
    decoder = (decoder_sweep(rt, backend, args.steps, ranks if ranks.world > 1 else None)
               if not args.no_decoder and 64 % ranks.world == 0 else None)
    ep = (expert_parallel_step(args, ranks, backend, layer, moe, xs[TOKENS], clocks)
          if ranks.world > 1 and EXPERTS % ranks.world == 0 else None)
    single = {'tok_s': value, 'ms_per_step': total_ms / args.steps,
              'e2e': {'value': e2e_value, 'unit': 'tok/s', 'steps': e2e_steps, 'h2d_bytes_per_step': e2e_h2d,
                      'd2h_bytes_per_step': e2e_d2h,
                      'api': 'gpu.moe.MoELayer.forward_pinned (pinned host rows in, pinned host rows + routing out)'}}
    roofline = {'bound': 'hbm', 'achieved': achieved, 'peak': peak, 'unit': 'GB/s', 'frac': achieved / peak,
                'traffic': traffic[0], 'traffic_source': traffic[1],
                'kernel': 'mma_rows_kernel<IQ1_S> gate+up job lists of the single-GPU layer (tensor-core int8; '
                          'two- and four-token jobs, two launches)',
                'algorithmic_bytes_per_launch': gu_bytes, 'avg_launch_us': gu_us, 'peak_source': peak_kind}
    config = {**workload_config(), 'global_batch': TOKENS * ranks.world,
              'l2_policy': 'inputs larger than L2: every step streams its experts from HBM (1.2 GB per GPU at N=1)',
              'per_tokens': per_tokens}
    if ep:
        # N > 1: the expert-parallel step is the headline; replicas beside it
        config['parallelism'] = f'expert x{ranks.world} ({EXPERTS // ranks.world} experts per GPU, router and ' \
                                'shared expert replicated)'
        headline = {'value': ep['tok_s'], 'ms_per_step': ep['ms_per_step'], 'e2e': ep['e2e'],
                    # prep x, router logits, top-k, dispatch, grouping, gate+up (two lists), prep h, down (two
                    # lists), return signal, combine
                    'gpu_launches': 12 * args.steps}
        ep_roof = {'bound': 'hbm', 'achieved': ep['hbm_gbs_per_gpu'], 'peak': peak, 'unit': 'GB/s',
                   'frac': ep['hbm_gbs_per_gpu'] / peak, 'traffic': None,
                   'traffic_source': 'no ncu capture of a multi-rank step (ncu runs on one GPU only)',
                   'kernel': 'whole expert-parallel step per GPU: owner expert weights (distinct local experts + '
                             'shared) + router over the step time',
                   'algorithmic_bytes_per_step': ep['hbm_bytes_per_step_per_gpu'], 'peak_source': peak_kind}
        extra = {'expert_parallel': ep, 'replicas': single, 'single_gpu_roofline': roofline}
        roofline = ep_roof
    else:
        config['parallelism'] = 'single GPU'
        headline = {'value': value, 'ms_per_step': total_ms / args.steps, 'e2e': single['e2e'],
                    # prep x, router logits, top-k, grouping, gate+up (two lists), prep h, down (two lists), combine
                    'gpu_launches': 10 * args.steps}
        extra = {}
    line = {
        'metric': METRIC, 'value': headline['value'], 'unit': 'tok/s', 'n_gpus': ranks.world, 'steps': args.steps,
        'warmup': args.warmup, 'ms_per_step': headline['ms_per_step'], 'higher_is_better': True, 'scaling': 'weak',
        'vs_baseline': None, 'dtype': 'f32', 'data': 'synthetic', 'config': config, 'roofline': roofline,
        'fused_gemv': gemv,
        **({'dsa_decode': dsa} if dsa else {}),
        **({'full_decoder_config4': decoder} if decoder else {}),
        **extra,
        'e2e': headline['e2e'],
        'gpu_launches': headline['gpu_launches'],
        'clocks': clocks.summary(),
    }
    if ranks.rank == 0 and ranks.world == 1 and not args.no_cpu_baseline:
        from oracle import loader
        from kernels.backend import VxBackend
        cpu = VxBackend(str(loader.serial()))  # the checker's library, here as the timed CPU baseline
        n, t0 = 0, time.perf_counter()
        while n == 0 or (time.perf_counter() - t0 < args.cpu_seconds and n < 8):
            oracle_ffn(cpu, layer, xs[1][0])
            n += 1
        secs = time.perf_counter() - t0
        line['cpu_baseline'] = {'value': n / secs, 'unit': 'tok/s', 'cores': 1, 'kind': 'port',
                                'sample': f'{n} token(s) through the full config-2 layer, reference semantics '
                                          '(glm_vx/model.py:289-324) on the single-thread C oracle'}
    if ranks.rank == 0:
        print(json.dumps(line), flush=True)
    moe.close()
    for t in bufs:
        for b in bufs[t]:
            b.close()
    backend.close()
    return 0


def run_profile_case(args):
    """Small cases for kernel captures (one status line, no benchmark numbers).
    moe: the config-2 layer shapes with only PROFILE_EXPERTS experts (about
    240 MB of IQ1_S, still above L2), TOKENS rows, six forwards.
    gemm: glmvx_gemm tf32_rna at 2048^3 (N(0,1) operands), three launches.
    dsa: the config-3 fused DSA decode for 16 queries over caches of 32768
    positions (DSADecoder.step_pinned), three steps."""
    use_ours()
    if args.profile_case == 'gemm':
        return profile_gemm()
    if args.profile_case in ('dsa', 'dsa1'):  # 16 queries, or the single-query step
        return profile_dsa(16 if args.profile_case == 'dsa' else 1)
    if args.profile_case == 'decoder':
        return profile_decoder()
    if args.profile_case == 'packed_gemm':
        return profile_packed_gemm()
    if args.profile_case == 'fp8_gemm':
        return profile_fp8_gemm()
    if args.profile_case == 'fp8_matvec':
        return profile_fp8_matvec()
    if args.profile_case == 'packed_gemm_tc':
        return profile_packed_gemm('glmvx_packed_gemm_tc')
    if args.profile_case in ('attention3', 'attention3_16'):
        return profile_attention3(16 if args.profile_case == 'attention3_16' else 1)
    from gpu.backend import GPUBackend
    from gpu import runtime as rt
    from gpu.moe import MoELayer
    backend = GPUBackend(0)
    layer = synthetic_layer(0, PROFILE_EXPERTS)
    moe = MoELayer(backend, layer['router'], layer['bias'], KIND, layer['gate'], layer['up'], layer['down'],
                   HIDDEN, INTER, TOPK, SCALE, shared=layer['shared'])
    x = np.random.default_rng(100).normal(size=(TOKENS, HIDDEN)).astype(np.float32)
    xd, yd = rt.DeviceBuffer(x.nbytes), rt.DeviceBuffer(x.nbytes)
    xd.upload(x, backend.stream.handle)
    for _ in range(6):
        moe.forward_device(yd.ptr, xd.ptr, TOKENS)
    backend.stream.synchronize()
    backend.device.check_device_error()
    print(f'profile case ok: {PROFILE_EXPERTS} experts, {TOKENS} tokens, 6 forwards', flush=True)
    xd.close()
    yd.close()
    moe.close()
    backend.close()
    return 0


def profile_decoder(layers=4, steps=2):
    """The config-4 resident decoder at 4 layers (3 dense + 1 sparse), 64
    sequences over 4096 synthetic cache rows: `steps` eager (un-graphed)
    steps, so a launch list shows every kernel of a step."""
    from gpu.backend import GPUBackend
    from gpu.decoder import ResidentDecoder, SyntheticWeights
    backend = GPUBackend(0)
    dec = ResidentDecoder(backend, CONFIG4, SyntheticWeights(CONFIG4, seed=44), batch=64, capacity=4096 + 16,
                          layers=layers)
    dec.fill_caches(4096)
    dec.set_tokens(np.arange(64) * 7)
    for _ in range(steps):
        dec._step_launches()
    dec.check()
    print(f'profile case ok: config-4 decoder, {layers} layers, 64 sequences, {steps} steps', flush=True)
    dec.close()
    backend.close()
    return 0


def profile_attention3(B, steps=2):
    """Config 3's attention sub-step with its Q8_0 projections (the resident
    decoder's layer-0 attention at config-3 widths, B queries over 32768
    synthetic cache rows), `steps` eager passes so a launch list shows every
    kernel."""
    from gpu.backend import GPUBackend
    from gpu.decoder import ResidentDecoder, SyntheticWeights
    backend = GPUBackend(0)
    cfg = dict(CONFIG4, num_hidden_layers=1, first_k_dense_replace=1,
               rope_parameters={'rope_theta': 1000000, 'rope_type': 'default'})
    dec = ResidentDecoder(backend, cfg, SyntheticWeights(cfg, seed=33, attention_kind=8), batch=B,
                          capacity=DSA_CONTEXT + 8 + steps, layers=1)
    dec.fill_caches(DSA_CONTEXT)
    dec.set_tokens(np.arange(B) * 11)
    from gpu import runtime as rt
    rt.check(backend.lib, backend.lib.glmvx_embed_rows(dec.x, dec.embed[0], dec.embed[1], dec.tokens, B, dec.vocab,
                                                       dec.hidden, dec.s), 'glmvx_embed_rows')
    L = dec.layers[0]
    for _ in range(steps):
        dec._rmsnorm(dec.n, dec.x, L['in_norm'], dec.hidden, dec.eps)
        dec._attention(0, L, None)
    dec.check()
    print(f'profile case ok: config-3 attention with projections, {B} queries, {steps} steps', flush=True)
    dec.close()
    backend.close()
    return 0


def profile_packed_gemm(entry='glmvx_packed_gemm'):
    """The packed GEMM for token batches (`entry`: the dispatching
    glmvx_packed_gemm, or glmvx_packed_gemm_tc for the tcgen05 kernel) on
    BASELINE config 1 at 64 tokens (Q4_K 6144 x 2048) and on the config-4
    lm_head shape at 32 tokens (Q8_0 154880 x 6144, 1 GB, larger than L2):
    three launches each."""
    from gpu.backend import GPUBackend
    from gpu import runtime as rt
    backend = GPUBackend(0)
    s = backend.stream.handle
    rng = np.random.default_rng(0)
    for kind, rows, cols, batch in ((12, 6144, 2048, 64), (8, 154880, 6144, 32)):
        blk, size = (256, 144) if kind == 12 else (32, 34)
        nb = rows * cols // blk
        w = rt.DeviceBuffer(nb * size)
        rt.check(backend.lib, backend.lib.glmvx_fill_random(w.ptr, kind, nb, 7, 0.01, 0, s), 'glmvx_fill_random')
        x = rng.normal(size=(batch, cols)).astype(np.float32)
        xd, od = rt.DeviceBuffer(x.nbytes), rt.DeviceBuffer(4 * batch * rows)
        xd.upload(x, s)
        for _ in range(3):
            rt.check(backend.lib, getattr(backend.lib, entry)(kind, od.ptr, w.ptr, xd.ptr, rows, cols, batch, s),
                     entry)
        backend.stream.synchronize()
        for b in (w, xd, od):
            b.close()
    backend.device.check_device_error()
    print(f'profile case ok: {entry}, config-1 Q4_K x64 and config-4 lm_head Q8_0 x32, 3 launches each', flush=True)
    backend.close()
    return 0


def profile_fp8_matvec(rows=16384, cols=6144):
    """glmvx_fp8_matvec on a 16384 x 6144 FP8 projection (100 MB, larger than
    L2): three launches."""
    from gpu.backend import GPUBackend
    from gpu import runtime as rt
    backend = GPUBackend(0)
    s = backend.stream.handle
    rng = np.random.default_rng(0)
    w8 = rng.integers(0, 256, size=rows * cols, dtype=np.uint8)
    w8[(w8 & 0x7F) == 0x7F] = 0x3C
    sc = (np.abs(rng.normal(size=(rows // 128) * (cols // 128))) * 0.02 + 1e-3).astype(np.float32)
    x = rng.normal(size=cols).astype(np.float32)
    bufs = [rt.DeviceBuffer(a.nbytes) for a in (w8, sc, x)] + [rt.DeviceBuffer(4 * rows)]
    for b, a in zip(bufs, (w8, sc, x)):
        b.upload(a, s)
    for _ in range(3):
        rt.check(backend.lib, backend.lib.glmvx_fp8_matvec(bufs[3].ptr, bufs[0].ptr, bufs[1].ptr, bufs[2].ptr, rows,
                                                           cols, s), 'glmvx_fp8_matvec')
    backend.stream.synchronize()
    for b in bufs:
        b.close()
    backend.device.check_device_error()
    print(f'profile case ok: glmvx_fp8_matvec {rows} x {cols}, 3 launches', flush=True)
    backend.close()
    return 0


def profile_fp8_gemm():
    """glmvx_fp8_gemm (tcgen05) at 32 tokens on the bench's FP8 6144 x 6144
    projection and on 24576 x 6144 (151 MB, larger than L2): three launches
    each."""
    from gpu.backend import GPUBackend
    from gpu import runtime as rt
    backend = GPUBackend(0)
    s = backend.stream.handle
    rng = np.random.default_rng(0)
    for rows, cols, batch in ((6144, 6144, 32), (24576, 6144, 32)):
        w8 = rng.integers(0, 256, size=rows * cols, dtype=np.uint8)
        w8[(w8 & 0x7F) == 0x7F] = 0x3C
        sc = (np.abs(rng.normal(size=(rows // 128) * (cols // 128))) * 0.02 + 1e-3).astype(np.float32)
        x = rng.normal(size=(batch, cols)).astype(np.float32)
        bufs = [rt.DeviceBuffer(a.nbytes) for a in (w8, sc, x)] + [rt.DeviceBuffer(4 * batch * rows)]
        for b, a in zip(bufs, (w8, sc, x)):
            b.upload(a, s)
        path = C.c_int32(-1)
        for _ in range(3):
            rt.check(backend.lib, backend.lib.glmvx_fp8_gemm(bufs[3].ptr, bufs[0].ptr, bufs[1].ptr, bufs[2].ptr, rows,
                                                             cols, batch, C.byref(path), s), 'glmvx_fp8_gemm')
        backend.stream.synchronize()
        assert path.value == 9, path.value
        for b in bufs:
            b.close()
    backend.device.check_device_error()
    print('profile case ok: glmvx_fp8_gemm x32 at 6144 x 6144 and 24576 x 6144, 3 launches each', flush=True)
    backend.close()
    return 0


def profile_gemm(n=2048):
    from gpu.backend import GPUBackend
    from gpu import runtime as rt
    backend = GPUBackend(0)
    s = backend.stream.handle
    a = np.random.default_rng(0).normal(size=(n, n)).astype(np.float32)
    bufs = [rt.DeviceBuffer(a.nbytes) for _ in range(3)]
    bufs[0].upload(a, s)
    bufs[1].upload(a, s)
    for _ in range(3):
        rt.check(backend.lib, backend.lib.glmvx_gemm(bufs[2].ptr, bufs[0].ptr, bufs[1].ptr, n, n, n, 1,
                                                     backend.device.error_address(), s), 'glmvx_gemm')
    backend.stream.synchronize()
    backend.device.check_device_error()
    print(f'profile case ok: tf32 GEMM {n}^3, 3 launches', flush=True)
    for b in bufs:
        b.close()
    backend.close()
    return 0


def profile_dsa(batch=16):
    from gpu.backend import GPUBackend
    from gpu.dsa import DSADecoder
    backend = GPUBackend(0)
    rng = np.random.default_rng(3)
    T = DSA_CONTEXT
    lat = rng.normal(size=(T - 8, DSA_RANK)).astype(np.float32)
    rk = rng.normal(size=(T - 8, DSA_ROPE)).astype(np.float32)
    ik = rng.normal(size=(T - 8, DSA_ID)).astype(np.float32)
    dec = DSADecoder(backend, batch, T)
    for i in range(batch):
        dec.load(i, lat, rk, ik)
    io = dec.pinned_io()
    for k in ('new_latent', 'new_rope', 'new_index_key', 'q_index'):
        io[k][...] = rng.normal(size=io[k].shape)
    io['q_latent'][...] = rng.normal(size=io['q_latent'].shape) * 0.05
    io['q_rope'][...] = rng.normal(size=io['q_rope'].shape) * 0.05
    io['head_weights'][...] = rng.normal(size=io['head_weights'].shape) * DSA_IH ** -0.5
    for _ in range(3):
        dec.step_pinned()
    backend.device.check_device_error()
    print(f'profile case ok: DSA decode, {batch} queries x {T} positions, 3 steps', flush=True)
    dec.close()
    backend.close()
    return 0


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=20)
    ap.add_argument('--warmup', type=int, default=5)
    ap.add_argument('--impl', choices=('ours', 'reference'), default='ours')
    ap.add_argument('--cpu-seconds', type=float, default=10.0)
    ap.add_argument('--no-cpu-baseline', action='store_true')
    ap.add_argument('--no-decoder', action='store_true', help='skip the config-4 decoder measurement')
    ap.add_argument('--profile-case', nargs='?', const='moe', choices=('moe', 'gemm', 'dsa', 'dsa1', 'decoder', 'packed_gemm', 'fp8_gemm', 'fp8_matvec',
                                                                 'attention3', 'attention3_16', 'packed_gemm_tc'),
                    help='run a small kernel-capture case (one GPU) instead of the benchmark')
    args = ap.parse_args()
    if args.profile_case:
        return run_profile_case(args)
    if args.warmup < 3:
        ap.error('--warmup must be >= 3')
    if args.impl == 'reference':
        return run_reference(args)
    ranks = Ranks()
    try:
        return run_ours(args, ranks)
    finally:
        ranks.close()


if __name__ == '__main__':
    sys.exit(main())
