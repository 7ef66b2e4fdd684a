"""Benchmark of the Motif Chord hot path on B200: 172M-class bf16 prefill (config 4).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (one process per GPU)

One step = one `MotifChordModel.forward` over this rank's share of config 4's batch: the 32 x
4096-token batch is split by sequence across the N ranks (32/N each; strong scaling, no
collective on the hot path), logits over all positions included.  `--weak` instead gives every
rank 32 sequences.  Config 5's decode splits its 64 requests the same way.  Prints ONE JSON
line on rank 0.

* `value`      — whole-job prefill tokens/s, inputs resident in HBM, device time (CUDA
                 events on the launching stream), max over ranks.
* `e2e`        — the same metric through the public API with host buffers: pinned int64
                 ids -> device, forward, greedy next token -> host, every step.
* `roofline`   — the dominant kernel of this library (by time), its algorithmic work per
                 launch over its CUDA-event duration inside the timed region (tensor fraction
                 against the sustained bf16 peak: the kernel runs inside a long step).
* `kernels`    — per-kernel breakdown of one instrumented step (CUDA events per call).
* `ops`        — configs 2 and 3 (the GDN and Chord ops alone), each with its roofline.
* `decode`     — config 5 (64 requests at context 8192, greedy CUDA-graph steps).
* `reference_gpu` — the reference's own GPU path (its Triton kernels, from `baseline/_ref`)
                 timed on the same box, configs 2-4, when that package is present.
* `cpu_baseline` — the CPU oracle (the reference's torch algorithm restated) timed on this
                 box's host cores on a bounded sample (B=1 x T=4096), rank 0 at N=1.
* `--impl reference` times that CPU implementation alone on the same metric.
"""

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

GLOBAL_BATCH = 32   # config 4: sequences per step, split across the ranks
SEQ_LEN = 4096
METRIC = 'prefill_tokens_per_s'
UNIT = 'tokens/s'
FALLBACK_PEAKS = {'hbm_gbs': 6650.0, 'bf16_tflops': 1590.0}


def peaks():
    p = os.path.join(ROOT, 'MEASURED_PEAKS.json')
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {'hbm_gbs': float(d['hbm_gbs']), 'bf16_tflops': float(d['bf16_tflops']),
                'bf16_tflops_sustained': float(d.get('bf16_tflops_sustained', d['bf16_tflops'])),
                'source': 'measured'}
    return dict(FALLBACK_PEAKS, bf16_tflops_sustained=1400.0, source='fallback')


# ---------------------------------------------------------------- algorithmic work
def kernel_work(name, cfg, B, T):
    """(flops, bytes) one launch of `name` does on a [B, T] prefill of `cfg` (bf16)."""
    d, H, Hkv = cfg.model_dim, cfg.num_heads, cfg.kv_heads
    dk, dv, D, hid, V = cfg.gdn_dk, cfg.gdn_dv, cfg.head_dim, cfg.mlp_hidden, cfg.vocab_size
    M = B * T
    C = 64
    if name == 'motif_b200_gdn_prefill_ws':
        # whole GDN layer from the projections: per token per head the chunked delta rule's
        # flops; bytes = q, k, v, a, b projection columns in, gate in, gated o out, + state out
        f_tok = 3 * 2 * C * dk + 2 * 2 * C * dv + 3 * 2 * dk * dv
        by_tok = 2 * (2 * dk + dv) + 2 * 2 + 2 * dv + 2 * dv
        return M * H * f_tok, M * H * by_tok + B * H * dk * dv * 4
    if name in ('motif_b200_gdn_chunk_gated', 'motif_b200_gdn_chunk_gated_ws'):
        # per token per head: G1, QK, W (2*C*dk each), U (2*C*dv), WS, qS, K^T X (2*dk*dv each), Aq X (2*C*dv)
        f_tok = 3 * 2 * C * dk + 2 * 2 * C * dv + 3 * 2 * dk * dv
        by_tok = 2 * (2 * dk + dv) + 8 + 2 * dv + 2 * dv  # q,k,v in, beta+g, gate in, o out
        return M * H * f_tok, M * H * by_tok + B * H * dk * dv * 4
    if name == 'motif_b200_chord_attention':
        pairs = T * (T + 1) / 2
        return 4 * B * H * D * pairs, M * (2 * H + 2 * Hkv) * D * 2
    if name == 'motif_b200_gdn_prep':
        cin = H * (2 * dk + dv) + 2 * H
        return 0, M * cin * 2 + M * H * (2 * dk + dv) * 2 + M * H * 8
    if name == 'motif_b200_attn_res_norm':
        return 0, None  # depends on the source count; filled by the caller
    if name == 'motif_b200_swiglu':
        return 0, M * hid * 3 * 2
    if name == 'motif_b200_chord_prep':
        return 0, M * (H + 2 * Hkv) * D * 2 * 2
    if name == 'motif_b200_gate_residual':
        return 0, M * d * 4 * 2
    if name == 'motif_b200_embed':
        return 0, M * d * 2 * 2 + M * 8
    return 0, 0


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per unit of work, from one ncu
# capture of each kernel on a smaller case of the same layer (B = 4 x T = 4096); traffic grows in
# proportion to the units, so a full launch's traffic is this figure times its units.
#   gdn_prefill_ws  : per token-head, the layer's three kernels at B = 4
#                     (profiles/gdn_split_b4_t4096.txt: UT transform 216.9 MB + state scan
#                     202.6 MB + gated norm 114.4 MB = 533.9 MB / 196608)
#   gdn_chunk_gated : per token-head, profiles/gdn_chunk_fast_b4_t4096.txt (186.2 MB / 196608)
#   chord_attention : per token, profiles/chord_tc_b4_t4096.txt (38.35 MB / 16384)
NCU_TRAFFIC = {
    'motif_b200_gdn_chunk_gated': (186.15e6 / (4 * 4096 * 12), 'token_head'),
    'motif_b200_gdn_prefill_ws': (533.9e6 / (4 * 4096 * 12), 'token_head'),
    'motif_b200_chord_attention': (38.35e6 / (4 * 4096), 'token'),
}


def ncu_traffic(name, cfg, B, T):
    if name not in NCU_TRAFFIC:
        return None
    per, unit = NCU_TRAFFIC[name]
    units = B * T * (cfg.num_heads if unit == 'token_head' else 1)
    return per * units


def gemm_flops(cfg, B, T):
    """Total cuBLAS GEMM flops of one forward (packed projections, K-concat residual, lm_head)."""
    d, H, Hkv = cfg.model_dim, cfg.num_heads, cfg.kv_heads
    dk, dv, D, hid, V = cfg.gdn_dk, cfg.gdn_dv, cfg.head_dim, cfg.mlp_hidden, cfg.vocab_size
    M = B * T
    n_gdn = sum(t != 'chord' for t in cfg.block) * cfg.block_n
    n_chord = sum(t == 'chord' for t in cfg.block) * cfg.block_n
    gdn = 2 * M * d * (2 * H * dk + 2 * H * dv + 2 * H + 2 * hid) + 2 * M * d * (H * dv + hid)
    chord = 2 * M * d * (2 * d + 2 * Hkv * D + 2 * hid) + 2 * M * d * d + 2 * M * d * hid
    return n_gdn * gdn + n_chord * chord + 2 * M * d * V


# ---------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ('index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,'
              'clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,'
              'clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap')

    def __init__(self, gpu_index):
        self.proc = None
        self.idx = gpu_index

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(['nvidia-smi', f'--query-gpu={self.FIELDS}', '--format=csv,noheader,nounits',
                                          '-lms', '50', '-i', str(self.idx)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap']
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(',')]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith('active'):
                    reasons.add(n)
        if not sm:
            return {'sm_mhz': None, 'sm_max_mhz': mx, 'reasons': ['unsampled'], 'samples': 0}
        load = [s for s in sm if mx is None or s > 0.5 * mx] or sm
        return {'sm_mhz': statistics.median(load), 'sm_max_mhz': mx, 'reasons': sorted(reasons),
                'samples': len(sm)}


# ---------------------------------------------------------------- distributed
# One process per GPU through motif_b200.runner: NCCL process group (short timeout), barrier,
# max over ranks.  No collective inside a forward.
_CTX = None


def dist_setup():
    global _CTX
    from motif_b200 import runner
    _CTX = runner.init(timeout_s=300.0)
    return _CTX.world, _CTX.rank, _CTX.local


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    from motif_b200 import runner
    return runner.max_over_ranks(x, _CTX)


def barrier(world):
    if world > 1:
        from motif_b200 import runner
        runner.barrier(_CTX)


# ---------------------------------------------------------------- CPU baseline
_CPU_PARAMS = {}


def cpu_oracle_rate(seq_len=SEQ_LEN, batch=1):
    """The CPU oracle (reference torch algorithm) forward at batch x seq_len, fp32, all cores."""
    from motif_b200.config import config_172m
    from oracle import model as om
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    cfg = config_172m()
    if 'P' not in _CPU_PARAMS:
        _CPU_PARAMS['P'] = om.make_params(cfg, 0, dtype=torch.float32)
    P = _CPU_PARAMS['P']
    ids = torch.randint(0, cfg.vocab_size, (batch, seq_len), generator=torch.Generator().manual_seed(0))
    t0 = time.perf_counter()
    om.forward(P, cfg, ids)
    dt = time.perf_counter() - t0
    return batch * seq_len / dt, threads, dt


def run_reference(args, world, rank):
    if rank != 0:
        return
    steps, warm = args.steps, args.warmup
    rates = []
    threads = os.cpu_count() or 1
    t_all = time.perf_counter()
    sample_len = args.ref_seq_len
    for i in range(warm + steps):
        r, threads, _ = cpu_oracle_rate(seq_len=sample_len)
        if i >= warm:
            rates.append(r)
    value = statistics.mean(rates)
    sample = f'B=1 x T={sample_len} prefill of the 172M config per step, fp32 CPU oracle (reference torch path)'
    line = {'metric': METRIC, 'value': value, 'unit': UNIT, 'n_gpus': world, 'steps': steps, 'warmup': warm,
            'ms_per_step': 1000.0 * sample_len / value, 'higher_is_better': True, 'scaling': 'strong',
            'vs_baseline': None, 'dtype': 'fp32', 'data': 'synthetic', 'impl': 'reference',
            'config': {'workload': '172M prefill (bounded CPU sample)', 'global_batch': 1, 'seq_len': sample_len},
            'cpu_baseline': {'value': value, 'unit': UNIT, 'cores': threads, 'kind': 'port', 'sample': sample},
            'e2e': {'value': value, 'unit': UNIT, 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0},
            'wall_s': time.perf_counter() - t_all}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- our arm
def run_ours(args, world, rank, local):
    from motif_b200 import _lib
    from motif_b200.config import config_172m
    from motif_b200.init import init_params
    from motif_b200.model import MotifChordModel

    dev = torch.device('cuda', local)
    torch.cuda.set_device(dev)
    cfg = config_172m()
    from motif_b200 import runner
    weak = args.weak
    gb = args.global_batch * world if weak else args.global_batch
    lo, hi = runner.shard_range(gb, world, rank)
    B = hi - lo
    if B == 0:
        raise SystemExit(f'global batch {gb} leaves rank {rank} of {world} without a sequence')
    T = args.seq_len
    torch.manual_seed(0)
    model = MotifChordModel(cfg)
    init_params(model, seed=0)
    model = model.to(dev, torch.bfloat16).eval()
    if args.mode == 'ops':
        # the op-level lines alone (configs 2 and 3, the projection shapes): for profiling
        if rank == 0:
            print(json.dumps({'metric': 'ops', 'ops': run_ops(dev, peaks(), args)}), flush=True)
        return
    if args.mode == 'decode':
        # decode measurement alone, printed as the line's headline (profiling captures)
        d = run_decode(model, cfg, args, world, rank, local, dev, torch.cuda.current_stream(dev), peaks())
        if rank == 0:
            line = dict(d, n_gpus=world, warmup=3, dtype='bf16', data='synthetic', vs_baseline=None)
            line['roofline'] = {'bound': 'hbm', 'achieved': d['hbm']['achieved_gbs_per_gpu'], 'peak': d['hbm']['peak'],
                                'unit': 'GB/s', 'frac': d['hbm']['frac'], 'traffic': None,
                                'kernel': 'whole decode step (all kernels)'}
            print(json.dumps(line), flush=True)
        return
    ids_all = torch.randint(0, cfg.vocab_size, (gb, T), generator=torch.Generator().manual_seed(0))
    ids_host = ids_all[lo:hi].contiguous().pin_memory()
    ids_dev = ids_host.to(dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        return model(ids_dev).logits

    # warm-up (also builds the packed weights and the cuBLAS handles)
    for _ in range(args.warmup):
        out = step()
    torch.cuda.synchronize(dev)
    del out

    # one instrumented step: per-kernel CUDA-event breakdown (outside the timed region)
    tr = _lib.Tracker(timed=None)
    _lib.set_tracker(tr)
    out = step()
    torch.cuda.synchronize(dev)
    _lib.set_tracker(None)
    del out
    summ = tr.summary()
    # the roofline kernel: the slowest of this library's kernels whose work is known per launch
    mine = {k: v for k, v in summ.items()
            if k.startswith('motif_b200_') and kernel_work(k, cfg, B, T)[1]}
    dominant = max(mine, key=lambda k: mine[k][1])

    # timed region: events only around the dominant kernel's launches
    tr = _lib.Tracker(timed={dominant})
    barrier(world)
    torch.cuda.synchronize(dev)
    with ClockSampler(local) as clk:
        _lib.set_tracker(tr)
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(args.steps):
            out = step()
        end.record(stream)
        torch.cuda.synchronize(dev)
        _lib.set_tracker(None)
    barrier(world)
    del out
    elapsed_ms = max_over_ranks(start.elapsed_time(end), world)
    dom = tr.summary().get(dominant, (0, 0.0))
    launches = tr.launches

    # end to end through the public API with host buffers
    def e2e_step():
        ids = ids_host.to(dev, non_blocking=True)
        o = model(ids)
        tok = o.next_token()
        return tok.to('cpu')

    e2e_step()
    torch.cuda.synchronize(dev)
    barrier(world)
    e_start = torch.cuda.Event(enable_timing=True)
    e_end = torch.cuda.Event(enable_timing=True)
    e_start.record(stream)
    for _ in range(args.steps):
        tok = e2e_step()
    e_end.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = max_over_ranks(e_start.elapsed_time(e_end), world)

    tokens = gb * T * args.steps
    value = tokens / (elapsed_ms / 1000.0)
    pk = peaks()
    kernels = {}
    for name, (calls, tot) in sorted(summ.items(), key=lambda kv: -kv[1][1]):
        kernels[name.replace('motif_b200_', '')] = {'calls': calls, 'ms': round(tot, 4)}
    gf = gemm_flops(cfg, B, T)
    if 'cublas_gemm' in summ:
        kernels['cublas_gemm']['tflops'] = round(gf / (summ['cublas_gemm'][1] / 1000.0) / 1e12, 1)
    flops, byts = kernel_work(dominant, cfg, B, T)
    avg_s = dom[1] / max(dom[0], 1) / 1000.0
    # the kernel runs inside a long step under the power cap: the sustained bf16 peak applies
    tpk = pk['bf16_tflops_sustained']
    if flops and flops / max(byts, 1) > tpk * 1e12 / (pk['hbm_gbs'] * 1e9):
        roof = {'bound': 'tensor', 'achieved': flops / avg_s / 1e12, 'peak': tpk, 'unit': 'TFLOP/s'}
    else:
        roof = {'bound': 'hbm', 'achieved': byts / avg_s / 1e9, 'peak': pk['hbm_gbs'], 'unit': 'GB/s'}
    roof['frac'] = roof['achieved'] / roof['peak']
    roof['traffic'] = ncu_traffic(dominant, cfg, B, T)
    roof['kernel'] = dominant
    roof['launches_timed'] = dom[0]
    roof['avg_launch_ms'] = avg_s * 1000.0
    roof['algorithmic_bytes'] = byts
    if flops:
        roof['algorithmic_flops'] = flops
        roof['tflops'] = flops / avg_s / 1e12
        roof['tensor_frac_of_measured_sustained_bf16'] = roof['tflops'] / tpk
    roof['gbs'] = byts / avg_s / 1e9
    roof['hbm_frac_of_measured'] = roof['gbs'] / pk['hbm_gbs']
    roof['peak_source'] = pk['source'] + (' (sustained bf16 peak)' if roof['bound'] == 'tensor' else ' (copy peak)')

    result = {
        'metric': METRIC, 'value': value, 'unit': UNIT, 'n_gpus': world, 'steps': args.steps, 'warmup': args.warmup,
        'ms_per_step': elapsed_ms / args.steps, 'higher_is_better': True, 'scaling': 'weak' if weak else 'strong',
        'vs_baseline': None,
        'dtype': 'bf16', 'data': 'synthetic',
        'config': {'workload': '172M-class MotifChord prefill, logits over all positions (config 4)',
                   'global_batch': gb, 'seq_len': T, 'per_rank_batch': B,
                   'parallelism': f'sequence-sharded replicas x{world} ({"weak: " + str(B) + " per rank" if weak else "strong: the batch split " + str(gb) + "/" + str(world)}), no hot-path collective',
                   'l2': 'inputs larger than L2 (every activation >= 200 MB at B=32)'},
        'e2e': {'value': tokens / (e2e_ms / 1000.0), 'unit': UNIT, 'h2d_bytes_per_step': ids_host.numel() * 8,
                'd2h_bytes_per_step': int(tok.numel() * 8)},
        'gpu_launches': launches,
        'roofline': roof,
        'kernels': kernels,
        'clocks': clk.summary(),
        'peaks': pk,
    }
    if args.decode_steps > 0:
        result['decode'] = run_decode(model, cfg, args, world, rank, local, dev, stream, pk)
    if not args.no_ops:
        result['ops'] = run_ops(dev, pk, args)
    if rank == 0 and world == 1 and not args.no_reference_gpu:
        result['reference_gpu'] = run_reference_gpu(dev, args)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rate, threads, dt = cpu_oracle_rate(seq_len=args.ref_seq_len)
        result['cpu_baseline'] = {'value': rate, 'unit': UNIT, 'cores': threads, 'kind': 'port',
                                  'sample': f'one B=1 x T={args.ref_seq_len} forward of the fp32 CPU oracle '
                                            f'(reference torch algorithm), {dt:.1f} s'}
    if rank == 0:
        print(json.dumps(result), flush=True)


# ---------------------------------------------------------------- ops (configs 2 and 3)
def _time_ms(fn, warm=3, iters=10):
    """Mean device time of fn() over `iters` calls after `warm` calls (CUDA events on the current
    stream, synchronised on both sides)."""
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters


def op_inputs(dev, which, dtype=torch.bfloat16):
    """Seeded synthetic inputs of config 2 ('gdn') or config 3 ('chord'), on `dev`."""
    import torch.nn.functional as F
    g = torch.Generator().manual_seed(0)
    B, H, T, D = 8, 12, 4096, 64
    if which == 'gdn':
        q = F.normalize(torch.randn(B, H, T, D, generator=g), dim=-1)
        k = F.normalize(torch.randn(B, H, T, D, generator=g), dim=-1)
        v = torch.randn(B, H, T, D, generator=g)
        beta = torch.sigmoid(torch.randn(B, H, T, generator=g))
        gg = -F.softplus(torch.randn(B, H, T, generator=g)) * 0.1
        return [t.to(dev, dtype) for t in (q, k, v)] + [beta.to(dev), gg.to(dev)]
    q, k, v = (torch.randn(B, H, T, D, generator=g).to(dev, dtype) for _ in range(3))
    alpha = (0.5 + 1.5 * torch.rand(H, generator=g)).to(dev)
    beta = torch.rand(H, generator=g).to(dev)
    mu = torch.ones(H, device=dev)
    ssmax = torch.ones(H, device=dev)
    log_n = torch.log(torch.arange(1, T + 1, dtype=torch.float32)).view(1, T).expand(B, T).contiguous().to(dev)
    return [q, k, v, alpha, beta, mu, ssmax, log_n]


OP_WORK = {
    # config 2: per token-head flops of the chunked delta rule (C = dk = dv = 64); bytes = q, k, v,
    # o bf16 + beta, g fp32 + the final state fp32
    'gdn': (8 * 12 * 4096 * (3 * 2 * 64 * 64 + 2 * 2 * 64 * 64 + 3 * 2 * 64 * 64),
            4 * 8 * 12 * 4096 * 64 * 2 + 2 * 8 * 12 * 4096 * 4 + 8 * 12 * 64 * 64 * 4),
    # config 3: causal half of QK^T and PV; bytes = q, k, v, o bf16
    'chord': (4 * 8 * 12 * 64 * 4096 * 4097 / 2, 4 * 8 * 12 * 4096 * 64 * 2),
}


def run_ops(dev, pk, args):
    """Configs 2 and 3 through the public ops (`motif_b200.ops`), timed alone (burst peaks)."""
    from motif_b200 import ops
    out = {}
    a = op_inputs(dev, 'gdn')
    ms = _time_ms(lambda: ops.chunk_gated_delta_rule(*a))
    f, b = OP_WORK['gdn']
    out['gdn_op'] = {'config': 'B=8 H=12 T=4096 dk=dv=64 chunk 64, bf16 q/k/v, fp32 beta/g/state (config 2)',
                     'ms': ms, 'tokens_per_s': 8 * 4096 / (ms / 1000.0),
                     'roofline': {'bound': 'hbm', 'achieved': b / (ms / 1000.0) / 1e9, 'peak': pk['hbm_gbs'],
                                  'unit': 'GB/s', 'frac': b / (ms / 1000.0) / 1e9 / pk['hbm_gbs'],
                                  'algorithmic_bytes': b, 'algorithmic_flops': f,
                                  'tflops': f / (ms / 1000.0) / 1e12,
                                  'tensor_frac_of_measured_bf16': f / (ms / 1000.0) / 1e12 / pk['bf16_tflops']}}
    del a
    a = op_inputs(dev, 'chord')
    ms = _time_ms(lambda: ops.apply_chord_attention(*a))
    f, b = OP_WORK['chord']
    out['chord_op'] = {'config': 'B=8 H=12 (kv 12) T=4096 D=64 bf16, GGD bias in-kernel (config 3)',
                       'ms': ms, 'tokens_per_s': 8 * 4096 / (ms / 1000.0),
                       'roofline': {'bound': 'tensor', 'achieved': f / (ms / 1000.0) / 1e12,
                                    'peak': pk['bf16_tflops'], 'unit': 'TFLOP/s',
                                    'frac': f / (ms / 1000.0) / 1e12 / pk['bf16_tflops'],
                                    'algorithmic_flops': f, 'algorithmic_bytes': b,
                                    'gbs': b / (ms / 1000.0) / 1e9}}
    del a
    torch.cuda.empty_cache()
    out['gemm_shapes'] = run_gemm_shapes(dev, pk)
    out['decode_gemm_shapes'] = {f'M={m}': run_decode_gemm_shapes(dev, pk, M=m) for m in (64, 8)}
    return out


# config 5's products (M = 64 requests): name -> (N, K)
DECODE_GEMM_SHAPES = {'gdn_in_proj': (8728, 768), 'gdn_out_proj': (768, 3584), 'chord_in_proj': (6016, 768),
                      'chord_o_proj': (768, 768), 'chord_down_proj': (768, 2048), 'lm_head': (32000, 768)}


def run_decode_gemm_shapes(dev, pk, M=64, reps=24):
    """The skinny GEMM (`motif_b200_skinny_gemm` on fragment-packed weights, 'ours') and the
    tensor-core decode GEMM (`motif_b200_skinny_gemm_tc`, 'tc') against the library GEMM (torch.mm
    -> cuBLAS) on config 5's decode products at M rows (64: one GPU; 8: eight GPUs of the strong
    split), bf16: each timed as a CUDA graph of
    `reps` back-to-back products whose weights rotate through enough copies to exceed L2 twice
    (every product streams its weight from HBM, as in the decode step)."""
    from motif_b200 import _lib
    from motif_b200.model import _skinny_packed
    res = {}
    g = torch.Generator(device=dev).manual_seed(0)
    l2 = 126 << 20
    for name, (N, K) in DECODE_GEMM_SHAPES.items():
        wbytes = N * K * 2
        copies = max(2, -(-2 * l2 // wbytes))
        ws = [(torch.randn((N, K), device=dev, generator=g) * K ** -0.5).bfloat16() for _ in range(copies)]
        ps = [_skinny_packed(w) for w in ws]
        x = torch.randn((M, K), device=dev, generator=g).bfloat16()
        y = torch.empty((M, N), device=dev, dtype=torch.bfloat16)

        def ours():
            for i in range(reps):
                _lib.call('motif_b200_skinny_gemm', x.data_ptr(), K, ps[i % copies].data_ptr(), y.data_ptr(), N, M, N,
                          K, 0, 0, _lib.MB_BF16, _lib.stream_ptr(dev))

        def lib():
            for i in range(reps):
                torch.mm(x, ws[i % copies].t(), out=y)

        def ours_tc():
            for i in range(reps):
                _lib.call('motif_b200_skinny_gemm_tc', x.data_ptr(), K, ws[i % copies].data_ptr(), K, y.data_ptr(), N,
                          M, N, K, 0, _lib.MB_BF16, _lib.stream_ptr(dev))

        r = {'M': M, 'N': N, 'K': K, 'weight_bytes': wbytes}
        for tag, fn in (('ours', ours), ('tc', ours_tc), ('cublas', lib)):
            s_ = torch.cuda.Stream(dev)
            s_.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(s_):
                fn()
                torch.cuda.synchronize(dev)
                gr = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gr, stream=s_):
                    fn()
            torch.cuda.current_stream(dev).wait_stream(s_)
            ms = _time_ms(gr.replay, warm=3, iters=10) / reps
            r[f'{tag}_us'] = ms * 1000.0
            r[f'{tag}_weight_gbs'] = wbytes / (ms / 1000.0) / 1e9
            del gr
        r['ours_frac_of_measured_hbm'] = r['ours_weight_gbs'] / pk['hbm_gbs']
        r['tc_frac_of_measured_hbm'] = r['tc_weight_gbs'] / pk['hbm_gbs']
        res[name] = r
        del ws, ps, x, y
        torch.cuda.empty_cache()
    return res


# config 4's projection shapes (M = 32 x 4096 tokens): name -> (N, K)
GEMM_SHAPES = {'gdn_in_proj': (8728, 768), 'gdn_out_proj': (768, 3584), 'chord_in_proj': (6016, 768),
               'chord_down_proj': (768, 2048), 'lm_head': (32000, 768)}


def run_gemm_shapes(dev, pk, M=32 * 4096):
    """The tcgen05 projection kernel (`motif_b200_gemm`, plain store epilogue) against the library
    GEMM (torch.mm -> cuBLAS) on config 4's shapes, bf16, alone (burst peak)."""
    from motif_b200 import _lib
    res = {}
    g = torch.Generator(device=dev).manual_seed(0)
    for name, (N, K) in GEMM_SHAPES.items():
        a = torch.randn((M, K), device=dev, generator=g).bfloat16()
        w = (torch.randn((N, K), device=dev, generator=g) * K ** -0.5).bfloat16()
        y = torch.empty((M, N), device=dev, dtype=torch.bfloat16)

        def ours():
            _lib.call('motif_b200_gemm', a.data_ptr(), K, w.data_ptr(), K, y.data_ptr(), N, M, N, K, _lib.MB_BF16,
                      _lib.stream_ptr(dev))

        ms_o = _time_ms(ours, warm=2, iters=5)
        ms_c = _time_ms(lambda: torch.mm(a, w.t(), out=y), warm=2, iters=5)
        f = 2.0 * M * N * K
        res[name] = {'M': M, 'N': N, 'K': K, 'ours_ms': ms_o, 'cublas_ms': ms_c,
                     'ours_tflops': f / (ms_o / 1000.0) / 1e12, 'cublas_tflops': f / (ms_c / 1000.0) / 1e12,
                     'ours_frac_of_measured_bf16': f / (ms_o / 1000.0) / 1e12 / pk['bf16_tflops']}
        del a, w, y
    torch.cuda.empty_cache()
    res['gdn_in_proj_fused'] = run_gdn_prep_shape(dev, M)
    return res


def run_gdn_prep_shape(dev, M):
    """The GDN input projection as the model runs it (`motif_b200_gemm_gdn_prep`: conv, SiLU,
    norms, beta / g and SwiGLU in the epilogue) at config 4's shape."""
    from motif_b200 import _lib
    from motif_b200.config import config_172m
    cfg = config_172m()
    H, dk, dv, hid, d = cfg.num_heads, cfg.gdn_dk, cfg.gdn_dv, cfg.mlp_hidden, cfg.model_dim
    B, T = M // SEQ_LEN, SEQ_LEN
    n = 2 * H * dk + 2 * H * dv + 2 * H + 2 * hid
    C = H * (2 * dk + dv)
    g = torch.Generator(device=dev).manual_seed(1)
    x = torch.randn((M, d), device=dev, generator=g).bfloat16()
    w = (torch.randn((n, d), device=dev, generator=g) * d ** -0.5).bfloat16()
    cw = torch.randn((C, 4), device=dev, generator=g).bfloat16()
    al, db = torch.rand(H, device=dev, generator=g).bfloat16(), torch.rand(H, device=dev, generator=g).bfloat16()
    q = torch.empty((M, H * dk), device=dev, dtype=torch.bfloat16)
    k, v, gate = torch.empty_like(q), torch.empty((M, H * dv), device=dev, dtype=torch.bfloat16), torch.empty(
        (M, H * dv), device=dev, dtype=torch.bfloat16)
    be, gg = torch.empty((M, H), device=dev), torch.empty((M, H), device=dev)
    act = torch.empty((M, hid), device=dev, dtype=torch.bfloat16)
    co = torch.empty((B, 3, C), device=dev, dtype=torch.bfloat16)

    def run():
        _lib.call('motif_b200_gemm_gdn_prep', x.data_ptr(), d, w.data_ptr(), d, B, T, d, H, dk, dv, hid, cw.data_ptr(),
                  al.data_ptr(), db.data_ptr(), None, co.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(),
                  be.data_ptr(), gg.data_ptr(), gate.data_ptr(), act.data_ptr(), hid, _lib.MB_BF16,
                  _lib.stream_ptr(dev))

    ms = _time_ms(run, warm=2, iters=5)
    f = 2.0 * M * n * d
    out = {'M': M, 'N': n, 'K': d, 'ours_ms': ms, 'ours_tflops': f / (ms / 1000.0) / 1e12}
    del x, w, q, k, v, gate, act
    torch.cuda.empty_cache()
    return out


# ---------------------------------------------------------------- the reference's GPU path
REF_DIR = os.path.join(ROOT, 'baseline', '_ref')


def run_reference_gpu(dev, args):
    """The reference's own GPU path, unmodified, from the package installed in `baseline/_ref`
    (its Triton kernels: `chunk_gated_delta_rule_triton`, `apply_chord_attention`, and
    `MotifChordModel.forward`, which dispatches to them on CUDA), on configs 2, 3 and 4.  The
    reference's GDN layer runs its delta rule in fp32 (`gdn_attn.py:197`), so config 2 is timed
    on fp32 inputs there; config 4 runs at B = 4 x 4096 (its per-token rate)."""
    if not os.path.isdir(os.path.join(REF_DIR, 'motif')):
        return {'unavailable': 'baseline/_ref is not installed'}
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    res = {'source': 'baseline/_ref (reference package, Triton GPU path)'}
    try:
        from motif.ops.chord_attention import apply_chord_attention as ref_chord
        from motif.ops.gated_deltanet import chunk_gated_delta_rule_triton as ref_gdn
    except Exception as e:  # noqa: BLE001 - reported, not raised
        return {'unavailable': f'import failed: {type(e).__name__}: {e}'}
    with torch.no_grad():
        try:
            a = op_inputs(dev, 'gdn', dtype=torch.float32)
            ms = _time_ms(lambda: ref_gdn(*a), warm=2, iters=5)
            res['gdn_op'] = {'ms': ms, 'tokens_per_s': 8 * 4096 / (ms / 1000.0), 'dtype': 'fp32'}
            del a
        except Exception as e:  # noqa: BLE001
            res['gdn_op'] = {'unavailable': f'{type(e).__name__}: {e}'[:300]}
        torch.cuda.empty_cache()
        try:
            a = op_inputs(dev, 'chord')
            ms = _time_ms(lambda: ref_chord(*a), warm=2, iters=5)
            res['chord_op'] = {'ms': ms, 'tokens_per_s': 8 * 4096 / (ms / 1000.0), 'dtype': 'bf16',
                               'tflops': OP_WORK['chord'][0] / (ms / 1000.0) / 1e12}
            del a
        except Exception as e:  # noqa: BLE001
            res['chord_op'] = {'unavailable': f'{type(e).__name__}: {e}'[:300]}
        torch.cuda.empty_cache()
        try:
            from motif.model.config import MotifChordConfig as RefConfig
            from motif.model.motif import MotifChordModel as RefModel
            from motif_b200.config import config_172m
            from motif_b200.init import init_params
            c = config_172m()
            rcfg = RefConfig(vocab_size=c.vocab_size, model_dim=c.model_dim, num_heads=c.num_heads,
                             num_kv_heads=c.num_kv_heads, head_k_dim=c.head_k_dim, block=tuple(c.block),
                             block_n=c.block_n)
            torch.manual_seed(0)
            rm = RefModel(rcfg)
            init_params(rm, seed=0)
            rm = rm.to(dev, torch.bfloat16).eval()
            Bref = 4
            ids = torch.randint(0, c.vocab_size, (Bref, SEQ_LEN), generator=torch.Generator().manual_seed(0)).to(dev)
            ms = _time_ms(lambda: rm(ids), warm=2, iters=3)
            res['prefill_172m'] = {'ms': ms, 'batch': Bref, 'seq_len': SEQ_LEN,
                                   'tokens_per_s': Bref * SEQ_LEN / (ms / 1000.0), 'dtype': 'bf16'}
            del rm, ids
        except Exception as e:  # noqa: BLE001
            res['prefill_172m'] = {'unavailable': f'{type(e).__name__}: {e}'[:300]}
        torch.cuda.empty_cache()
    return res


# ---------------------------------------------------------------- decode (config 5)
DECODE_BATCH = 64      # config 5: requests, split across the ranks
DECODE_CONTEXT = 8192


def decode_step_bytes(model, B, S):
    """HBM bytes one greedy decode step must move at cache length S (new token included):
    every packed weight once, each Chord layer's K and V over S positions plus the new
    row, each GDN layer's fp32 state read + written and conv window read + written, the
    embedding rows, the logits written and read by the argmax."""
    cfg = model.config
    decs, lm = model.packed()
    wb = lm.numel() * lm.element_size()
    kv = gdn = 0
    for blk in decs:
        for pk in blk:
            for name in ('w_in', 'w_out', 'w_o', 'w_down'):
                t = getattr(pk, name, None)
                if t is not None:
                    wb += t.numel() * t.element_size()
            if hasattr(pk, 'Hkv'):
                kv += 2 * B * pk.Hkv * (S + 1) * pk.D * 2
            else:
                C = pk.H * (2 * pk.dk + pk.dv)
                gdn += 2 * B * pk.H * pk.dk * pk.dv * 4 + 2 * B * 3 * C * 2
    d = cfg.model_dim
    return wb + kv + gdn + B * d * 2 + 2 * B * cfg.vocab_size * 2


def _decode_kernels(brk, graph_ms):
    """Per-kernel share of the decode step: eager event times averaged over 32 steps (which
    include launch gaps the graph does not have), normalised so the shares sum to 1 and scaled to
    the graph step's measured time."""
    tot = sum(t for _, t in brk.values()) or 1.0
    out = {'_note': 'eager steps (32, events per launch) scaled to the graph step: ms = share x graph ms/step'}
    for k, (c, t) in sorted(brk.items(), key=lambda kv: -kv[1][1]):
        out[k.replace('motif_b200_', '')] = {'calls_per_step': c, 'eager_ms': round(t, 4), 'share': round(t / tot, 4),
                                             'ms': round(t / tot * graph_ms, 4)}
    return out


def run_decode(model, cfg, args, world, rank, local, dev, stream, pk):
    """Config 5: B=64 sequences per GPU at context 8192, then `--decode-steps` greedy steps,
    one CUDA-graph replay per step.  The caches are filled directly with seeded random
    contents at length 8192 (decode speed does not depend on them), as a prefill of
    64 x 8192 tokens would leave them."""
    from motif_b200 import _lib
    from motif_b200.decode import GraphDecoder, fill_cache_random
    from motif_b200 import runner
    gbd = args.decode_batch * world if args.weak else args.decode_batch
    lo, hi = runner.shard_range(gbd, world, rank)
    B, L, n = hi - lo, DECODE_CONTEXT, args.decode_steps
    cache = fill_cache_random(model, model.create_cache(), B, L, L + 2 * n, seed=rank)
    dec = GraphDecoder(model, cache, max_steps=2 * n)
    g = torch.Generator().manual_seed(rank)
    first_host = torch.randint(0, cfg.vocab_size, (B, 1), generator=g).pin_memory()
    first = first_host.to(dev)
    # per-kernel breakdown, 32 eager steps with events around every launch (outside the timed
    # region); reported as shares of the graph step
    brk = dec.breakdown(first, steps=32)
    # warm-up replays (also the first touch of every cache page), then the caches' lengths
    # are rewound so the timed steps start at context 8192
    dec.run(first, min(3, n))
    torch.cuda.synchronize(dev)
    dec.taken = 0
    dec.lens.copy_(torch.tensor([L, L + 1], dtype=torch.int32))
    dec.step_idx.zero_()
    barrier(world)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        t0.record(stream)
        toks = dec.run(first, n)
        t1.record(stream)
        torch.cuda.synchronize(dev)
    ms = max_over_ranks(t0.elapsed_time(t1), world)
    # end to end through the public API: host ids in, n graph steps, host tokens out
    dec.taken = 0
    dec.lens.copy_(torch.tensor([L, L + 1], dtype=torch.int32))
    dec.step_idx.zero_()
    barrier(world)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    toks = dec.run(first_host.to(dev, non_blocking=True), n).to('cpu')
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world)
    total_tok = gbd * n
    byts = sum(decode_step_bytes(model, B, L + i) for i in range(n))
    gbs = byts / (ms / 1000.0) / 1e9
    out = {
        'metric': 'decode_tokens_per_s', 'value': total_tok / (ms / 1000.0), 'unit': 'tokens/s',
        'higher_is_better': True, 'scaling': 'weak' if args.weak else 'strong', 'steps': n, 'ms_per_step': ms / n,
        'config': {'workload': '172M-class greedy decode (config 5), one CUDA-graph replay per token',
                   'per_rank_batch': B, 'global_batch': gbd, 'context': L,
                   'cache_fill': 'seeded random KV / GDN states at length 8192 (stands in for the prefill)',
                   'l2': 'working set per step > 2 GB, larger than L2'},
        'hbm': {'achieved_gbs_per_gpu': gbs, 'peak': pk['hbm_gbs'], 'frac': gbs / pk['hbm_gbs'],
                'algorithmic_bytes_per_step': byts / n},
        'e2e': {'value': total_tok / (e2e_ms / 1000.0), 'unit': 'tokens/s',
                'h2d_bytes_per_step': first_host.numel() * 8 / n, 'd2h_bytes_per_step': toks.numel() * 8 / n},
        'gpu_launches': dec.launches_per_step * n,
        'kernels': _decode_kernels(brk, ms / n),
        'clocks': clk.summary(),
    }
    dec.release()
    del cache
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=10)
    ap.add_argument('--warmup', type=int, default=3)
    ap.add_argument('--impl', choices=['ours', 'reference'], default='ours')
    ap.add_argument('--seq-len', type=int, default=SEQ_LEN)
    ap.add_argument('--global-batch', type=int, default=GLOBAL_BATCH,
                    help=f'config-4 sequences per step, split across the ranks (default {GLOBAL_BATCH}); small '
                         'values are for profiling captures')
    ap.add_argument('--weak', action='store_true',
                    help='weak scaling: every rank runs --global-batch prefill sequences and --decode-batch requests')
    ap.add_argument('--no-ops', action='store_true', help='skip the op-level lines (configs 2 and 3)')
    ap.add_argument('--no-reference-gpu', action='store_true',
                    help="skip timing the reference's own GPU (Triton) path from baseline/_ref")
    ap.add_argument('--ref-seq-len', type=int, default=SEQ_LEN)
    ap.add_argument('--no-cpu-baseline', action='store_true')
    ap.add_argument('--mode', choices=['all', 'decode', 'ops'], default='all',
                    help="'decode' runs only the config-5 decode measurement, 'ops' only the op-level lines "
                         "(configs 2 and 3, the projection shapes); both for profiling")
    ap.add_argument('--decode-batch', type=int, default=DECODE_BATCH,
                    help=f'config-5 decode requests, split across the ranks (default {DECODE_BATCH})')
    ap.add_argument('--decode-steps', type=int, default=256,
                    help='greedy decode steps of the config-5 decode measurement (0 skips it)')
    args = ap.parse_args()
    world, rank, local = dist_setup() if args.impl == 'ours' else (
        int(os.environ.get('WORLD_SIZE', '1')), int(os.environ.get('RANK', '0')), 0)
    if world != args.gpus:
        print(f'warning: --gpus {args.gpus} but WORLD_SIZE {world}', file=sys.stderr)
    try:
        if args.impl == 'reference':
            run_reference(args, world, rank)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1 and args.impl == 'ours':
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == '__main__':
    main()
