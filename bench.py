"""Benchmark of the Veda sparse-attention layer on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config cfg3]
    python bench.py --impl reference ...   # the reference algorithm on CPU
    python bench.py --config cfg5 ...      # the stage-2 training step
    python bench.py --only backward|heat   # one stage on one head group

One step = one Veda attention layer forward over synthetic q, k, v already
resident in HBM: permute + pool q/k/v, predictor logits, budgeted top-k
lists, tcgen05 block-sparse attention, inverse permutation. The default
workload is the H3-scale config (cfg3: 48 heads, two tile shapes, 1024
text rows). With N > 1:
  --parallel ulysses  (default) one clip, heads split over the ranks by an
                      all-to-all from the sequence-sharded layout; strong
                      scaling, the value is the time of one layer;
  --parallel clips    every rank runs the layer on its own clip (the
                      reference's one-clip-per-GPU data parallelism, no
                      collective on the data path; weak scaling, the value
                      is ms per layer of the whole job).
Prints one JSON line on rank 0.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from miowtion_b200 import attention as veda_attention  # noqa: E402
from miowtion_b200 import kernels  # noqa: E402
from miowtion_b200 import mask as veda_mask  # noqa: E402
from miowtion_b200 import plan as veda_plan  # noqa: E402
from miowtion_b200 import predictor as veda_predictor  # noqa: E402
from miowtion_b200 import tiling  # noqa: E402
from miowtion_b200.pipeline import HostPipeline  # noqa: E402
from miowtion_b200 import ulysses  # noqa: E402

METRIC = ('sparse-attn ms/layer @90% sparsity; effective TFLOP/s; '
          'frac of bf16 peak')
BLOCK_FLOPS = 4 * 128 * 128 * 128  # QK^T + PV of one 128x128 block, fwd

# BASELINE.json configs 2-4 (config 1 is the CPU-sized parity case).
CONFIGS = {
    'cfg2': dict(desc='1xB200 fwd, 24 heads, grid (20,32,56)=35840 tokens, '
                      'tile 2x8x8, 280x280 tiles, 28 key tiles/row (90%)',
                 heads=24, seq_len=35840, used=35840, target=(0, (20, 32, 56)),
                 cond=None, shapes=[(2, 8, 8)], head_shape=[0] * 24,
                 target_ratio=0.1, ref_ratio=None, seed=1),
    'cfg3': dict(desc='H3-scale fwd, 48 heads, 1024 text + grid (26,45,80), '
                      'heads 0-23 tile 2x8x8, 24-47 tile 1x8x16, 90% budget',
                 heads=48, seq_len=94624, used=94624,
                 target=(1024, (26, 45, 80)), cond=None,
                 shapes=[(2, 8, 8), (1, 8, 16)],
                 head_shape=[0] * 24 + [1] * 24, target_ratio=0.1,
                 ref_ratio=None, seed=2),
    'cfg4': dict(desc='Ref2VA fwd, 48 heads, ref grid (4,45,80) at 95% + '
                      'target grid (26,45,80) at 90%, tile 2x8x8',
                 heads=48, seq_len=108000, used=108000,
                 target=(14400, (26, 45, 80)), cond=(0, (4, 45, 80)),
                 shapes=[(2, 8, 8)], head_shape=[0] * 48, target_ratio=0.1,
                 ref_ratio=0.05, seed=3),
    # Config 5: the config-3 layer as a stage-2 training step.
    'cfg5': dict(desc='stage-2 step on the config-3 shapes: dense fwd + LSE, '
                      'teacher heat (sum) for all query tiles, sparse student '
                      'fwd + bwd (transposed lists), dO ~N(0,1) seed 4',
                 heads=48, seq_len=94624, used=94624,
                 target=(1024, (26, 45, 80)), cond=None,
                 shapes=[(2, 8, 8), (1, 8, 16)],
                 head_shape=[0] * 24 + [1] * 24, target_ratio=0.1,
                 ref_ratio=None, seed=2, dout_seed=4, train=True),
}


def load_peaks() -> dict:
    path = os.path.join(ROOT, 'MEASURED_PEAKS.json')
    if os.path.exists(path):
        with open(path) as f:
            peaks = json.load(f)
        peaks['source'] = 'measured'
        return peaks
    return {'hbm_gbs': 6650.0, 'bf16_tflops': 1590.0,
            'bf16_tflops_sustained': 1400.0, 'source': 'fallback'}


# A timed region at least this long runs under the power cap: its kernel is
# compared with the sustained bf16 figure (a GEMM loop of seconds), a shorter
# one with the burst figure.
SUSTAINED_AFTER_S = 1.0


def tensor_roofline(peaks: dict, achieved: float, timed_s: float,
                    kernel: str, traffic) -> dict:
    """The roofline object of a tensor-bound kernel: `achieved` TFLOP/s
    over the burst or the sustained measured peak, by the length of the timed
    region, with both fractions."""
    sustained = timed_s >= SUSTAINED_AFTER_S
    burst, sus = peaks['bf16_tflops'], peaks['bf16_tflops_sustained']
    peak = sus if sustained else burst
    return {'bound': 'tensor', 'kernel': kernel, 'achieved': achieved,
            'peak': peak, 'unit': 'TFLOP/s', 'frac': achieved / peak,
            'traffic': traffic,
            'peak_source': (f'{peaks["source"]} bf16 '
                            f'{"sustained" if sustained else "burst"} '
                            f'(timed region {timed_s:.2f} s)'),
            'frac_of_burst': achieved / burst,
            'frac_of_sustained': achieved / sus}


def build_student(cfg, device, heads_plan=None):
    layout = veda_attention.PackedLayout(
        cfg['seq_len'], cfg['used'],
        (veda_attention.VideoSpan(cfg['target'][0], cfg['target'][1]),))
    cond = ()
    if cfg['cond'] is not None:
        cond = (tiling.TiledSpan(cfg['cond'][0], cfg['cond'][1],
                                 tiling.TileShape(2, 8, 8)),)
    config = veda_attention.VedaConfig(
        target_budget=veda_mask.Budget(ratio=cfg['target_ratio']),
        ref_budget=(veda_mask.Budget(ratio=cfg['ref_ratio'])
                    if cfg['ref_ratio'] else None))
    clip = veda_attention.ClipTiling(layout, config, device, cond)
    plan = heads_plan or veda_plan.TilePlan(
        'bench', cfg['target'][1],
        [tiling.TileShape(*s) for s in cfg['shapes']], [cfg['head_shape']])
    local_heads = len(plan.head_shape[0])
    pred = predictor_for(cfg, device)
    return veda_attention.SparseStudent(clip, plan, pred), clip, plan, \
        local_heads


def predictor_for(cfg, device):
    """Random-init predictor of the reference architecture, N(0, 0.02)."""
    gen = torch.Generator().manual_seed(1000 + cfg['seed'])
    pred = veda_predictor.TileScorePredictor(1, cfg['heads'], 128)
    with torch.no_grad():
        for p in (pred.layers[0].proj_q, pred.layers[0].proj_k):
            p.copy_(torch.randn(p.shape, generator=gen) * 0.02)
    return pred.to(device)


def synthetic_qkv(cfg, rows, row0, device, clip=0):
    """q, k, v rows [row0, row0+rows) of ~N(0,1) bf16 [S, H, 128], drawn
    per 4096-row chunk from a seeded device generator (so every rank draws
    the same global tensors); `clip` > 0 draws a different clip."""
    heads = cfg['heads']
    out = []
    for t in range(3):
        x = torch.empty(rows, heads, 128, dtype=torch.bfloat16, device=device)
        chunk = 4096
        for c0 in range(row0 - row0 % chunk, row0 + rows, chunk):
            gen = torch.Generator(device=device)
            gen.manual_seed(cfg['seed'] * 1_000_003 + t * 7919 + c0 // chunk
                            + clip * 104_729)
            blk = torch.randn(chunk, heads, 128, generator=gen, device=device)
            lo, hi = max(c0, row0), min(c0 + chunk, row0 + rows)
            x[lo - row0:hi - row0] = blk[lo - c0:hi - c0].to(torch.bfloat16)
        out.append(x)
    return out


class ClockSampler:
    """nvidia-smi clocks and throttle reasons while the timed region runs."""

    QUERY = ('index,clocks.sm,clocks.max.sm,power.draw,'
             'clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,'
             'clocks_event_reasons.hw_thermal_slowdown,'
             'clocks_event_reasons.sw_thermal_slowdown,'
             'clocks_event_reasons.sw_power_cap')

    def __init__(self, device: torch.device):
        # nvidia-smi ignores CUDA_VISIBLE_DEVICES: address the GPU by UUID.
        try:
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            self.index = uuid if uuid.startswith('GPU-') else f'GPU-{uuid}'
        except (AttributeError, RuntimeError):
            self.index = str(device.index)
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ['nvidia-smi', f'--id={self.index}',
                 f'--query-gpu={self.QUERY}', '--format=csv,noheader,nounits',
                 '-lms', '20'], stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.perf_counter(), line.strip()))

    def mark(self, name: str) -> None:
        setattr(self, name, time.perf_counter())

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        """Samples taken between mark('t0') and mark('t1') only."""
        mhz, max_mhz, reasons = [], None, set()
        names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown',
                 'sw_power_cap']
        t0 = getattr(self, 't0', 0.0)
        t1 = getattr(self, 't1', float('inf'))
        for stamp, line in self.lines:
            if not t0 <= stamp <= t1:
                continue
            parts = [p.strip() for p in line.split(',')]
            if len(parts) < 9:
                continue
            try:
                mhz.append(float(parts[1]))
                max_mhz = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == 'active':
                    reasons.add(name)
        return {'sm_mhz': statistics.median(mhz) if mhz else None,
                'sm_max_mhz': max_mhz, 'reasons': sorted(reasons),
                'samples': len(mhz)}


def cpu_baseline(cfg, budget_s=12.0, timed_steps=None):
    """The reference algorithm (the oracle restatement) on the host cores:
    the full layer for a time-bounded sample of heads, extrapolated to all
    heads (heads are independent with equal per-head cost)."""
    from oracle import veda_oracle as vo
    import threadpoolctl
    # Every host core, whatever OMP_NUM_THREADS the launcher set (torchrun
    # sets 1): numpy's BLAS pool and torch's intra-op pool.
    cores = os.cpu_count() or 1
    threadpoolctl.threadpool_limits(cores)
    torch.set_num_threads(cores)
    seq_len, used = cfg['seq_len'], cfg['used']
    gen = torch.Generator().manual_seed(1000 + cfg['seed'])
    pq = (torch.randn(cfg['heads'], 384, 128, generator=gen) * 0.02).numpy()
    pk = (torch.randn(cfg['heads'], 384, 128, generator=gen) * 0.02).numpy()
    spans_target = cfg['target']
    layouts = {}
    times = []
    head = 0
    t_all = time.perf_counter()
    while True:
        shape = tuple(cfg['shapes'][cfg['head_shape'][head]])
        if shape not in layouts:
            spans = []
            if cfg['cond'] is not None:
                spans.append(vo.Span(cfg['cond'][0], cfg['cond'][1],
                                     (2, 8, 8)))
            spans.append(vo.Span(spans_target[0], spans_target[1], shape))
            layouts[shape] = vo.build_tile_layout(spans, used, seq_len)
        gen_h = torch.Generator().manual_seed(cfg['seed'] * 31 + head)
        q, k, v = (torch.randn(seq_len, 1, 128, generator=gen_h).to(
            torch.bfloat16).float().numpy() for _ in range(3))
        t0 = time.perf_counter()
        vo.sparse_student_layer(
            q, k, v, [(layouts[shape], np.array([0]))], pq[head:head + 1],
            pk[head:head + 1], vo.Budget(ratio=cfg['target_ratio']),
            vo.Budget(ratio=cfg['ref_ratio']) if cfg['ref_ratio'] else None,
            used=used)
        times.append(time.perf_counter() - t0)
        head = (head + 1) % cfg['heads']
        if timed_steps is not None:
            if len(times) >= timed_steps:
                break
        elif time.perf_counter() - t_all > budget_s:
            break
    per_head = sum(times) / len(times)
    threads = max([i.get('num_threads', 1)
                   for i in threadpoolctl.threadpool_info()] or [1])
    return per_head * cfg['heads'] * 1e3, len(times), threads, times


def reference_layer_head(ref, cfg, head, sample_tiles, layouts, seed):
    """One head of the layer through the reference's own CPU functions
    (installed unmodified under baseline/_ref): build_tile_layout (cached per
    shape, as the reference caches it), gather_tiles of q, k, v,
    pool_tiles, LayerPredictor.forward, column_blocks, select_video_blocks,
    dense_block_mask, scatter_tiles_, all at full size; the token-level
    reference attention (kernels/reference.py:23-56) on `sample_tiles`
    random query tiles, in chunks of 8 tiles (the function takes any
    subset of query tiles with their mask rows). Returns (seconds of the
    full-size stages, seconds of the sampled attention, tiles sampled,
    tiles in the layout)."""
    from miowtion.kernels import reference as rref
    from miowtion.veda import mask as rmask
    from miowtion.veda import predictor as rpred
    from miowtion.veda import tiling as rtiling
    seq_len, used = cfg['seq_len'], cfg['used']
    shape = tuple(cfg['shapes'][cfg['head_shape'][head]])
    if shape not in layouts:
        spans = []
        if cfg['cond'] is not None:
            spans.append(rtiling.TiledSpan(cfg['cond'][0],
                                           tuple(cfg['cond'][1]),
                                           rtiling.TileShape(2, 8, 8)))
        spans.append(rtiling.TiledSpan(cfg['target'][0],
                                       tuple(cfg['target'][1]),
                                       rtiling.TileShape(*shape)))
        layouts[shape] = rtiling.build_tile_layout(spans, used, seq_len)
    lay = layouts[shape]
    gen = torch.Generator().manual_seed(cfg['seed'] * 31 + head)
    q, k, v = (torch.randn(seq_len, 1, 128, generator=gen).to(torch.bfloat16)
               for _ in range(3))
    gen_w = torch.Generator().manual_seed(1000 + cfg['seed'])
    pq = torch.randn(cfg['heads'], 384, 128, generator=gen_w) * 0.02
    pk = torch.randn(cfg['heads'], 384, 128, generator=gen_w) * 0.02
    pred = rpred.TileScorePredictor(1, 1, 128)
    with torch.no_grad():
        pred.layers[0].proj_q.copy_(pq[head:head + 1])
        pred.layers[0].proj_k.copy_(pk[head:head + 1])
    one = torch.tensor([0])
    with torch.no_grad():
        t0 = time.perf_counter()
        qt, kt, vt = (rtiling.gather_tiles(x, lay, one) for x in (q, k, v))
        fq = rpred.pool_tiles(qt, lay)
        fk = rpred.pool_tiles(kt, lay)
        logits = pred.layers[0](fq, fk, one)
        blocks = rmask.column_blocks(
            lay, rmask.Budget(ratio=cfg['target_ratio']),
            rmask.Budget(ratio=cfg['ref_ratio']) if cfg['ref_ratio'] else None)
        sel = rmask.select_video_blocks(logits[:, :lay.n_video_tiles], lay,
                                        blocks)
        block_mask = rmask.dense_block_mask(sel, lay)
        out = torch.zeros(seq_len + 1, 1, 128, dtype=torch.bfloat16)
        rtiling.scatter_tiles_(out, qt, lay, one)  # a full-size scatter
        t_stages = time.perf_counter() - t0
        pick = torch.randperm(lay.n_tiles, generator=torch.Generator()
                              .manual_seed(seed))[:sample_tiles].sort().values
        t0 = time.perf_counter()
        for c0 in range(0, pick.numel(), 8):
            tiles = pick[c0:c0 + 8]
            rows = (tiles[:, None] * 128 + torch.arange(128)).view(-1)
            rref.block_sparse_attention(qt[rows], kt, vt,
                                        block_mask[:, tiles],
                                        lay.valid_count)
        t_attn = time.perf_counter() - t0
    return t_stages, t_attn, int(pick.numel()), lay.n_tiles


def reference_cpu_ms(cfg, timed_steps=None, budget_s=12.0, sample_tiles=32):
    """ms per layer of the reference's own CPU path (reference_layer_head),
    one head per step, extrapolated: the sampled attention over all query
    tiles, every head the cost of the heads timed. Returns (ms, steps,
    threads, per-step ms, sample description) or None without the
    reference installed."""
    try:
        ref = reference_package()
    except Exception:  # pylint: disable=broad-except
        ref = None
    if ref is None:
        return None
    import threadpoolctl
    cores = os.cpu_count() or 1
    threadpoolctl.threadpool_limits(cores)
    torch.set_num_threads(cores)
    layouts: dict = {}
    per_step = []
    t_all = time.perf_counter()
    head = 0
    while True:
        t_st, t_at, n_s, n_t = reference_layer_head(
            ref, cfg, head, sample_tiles, layouts, seed=len(per_step))
        per_step.append((t_st + t_at * n_t / n_s) * cfg['heads'] * 1e3)
        head = (head + 1) % cfg['heads']
        if timed_steps is not None:
            if len(per_step) >= timed_steps:
                break
        elif time.perf_counter() - t_all > budget_s:
            break
    sample = (f'per step one head (of {cfg["heads"]}) through the '
              "reference's own CPU functions (baseline/_ref, unmodified): "
              'layout, gather, pool, predictor, selection, block mask and '
              'scatter at full size; its token-level attention on '
              f'{sample_tiles} random query tiles, scaled to all query '
              f'tiles; x{cfg["heads"]} heads')
    return per_step, cores, sample


def run_reference(args, cfg):
    """The reference arm: the reference's own CPU implementation of the
    layer on the host cores (reference_cpu_ms), or the oracle port when the
    reference is not installed. Rank 0 alone runs it."""
    rank = int(os.environ.get('RANK', '0'))
    if rank != 0:
        return
    warm = max(0, args.warmup)
    steps = max(1, args.steps)
    got = reference_cpu_ms(cfg, timed_steps=warm + steps)
    if got is not None:
        per_step, threads, sample = got
        timed = per_step[warm:]
        ms = sum(timed) / len(timed)
        kind = 'reference'
    else:
        _, _, threads, times = cpu_baseline(cfg, timed_steps=warm + steps)
        timed = times[warm:]
        ms = sum(timed) / len(timed) * cfg['heads'] * 1e3
        kind = 'port'
        sample = (f'per step one head (of {cfg["heads"]}) of the full layer '
                  f'through the oracle (numpy restatement of the reference), '
                  f'x{cfg["heads"]} heads')
    line = {
        'metric': METRIC, 'value': ms, 'unit': 'ms/layer', 'impl': 'reference',
        'n_gpus': args.gpus, 'steps': steps, 'warmup': warm,
        'ms_per_step': ms, 'higher_is_better': False, 'scaling': 'strong',
        'vs_baseline': None, 'dtype': 'f32', 'data': 'synthetic',
        'config': {'workload': f'{args.config}: {cfg["desc"]}',
                   'parallelism': 'cpu'},
        'cpu_baseline': {'value': ms, 'unit': 'ms/layer', 'cores': threads,
                         'kind': kind, 'sample': sample},
        'e2e': {'value': ms, 'unit': 'ms/layer', 'h2d_bytes_per_step': 0,
                'd2h_bytes_per_step': 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=400)
    ap.add_argument('--warmup', type=int, default=5)
    ap.add_argument('--config', default='cfg3', choices=sorted(CONFIGS))
    ap.add_argument('--impl', default='b200', choices=['b200', 'reference'])
    ap.add_argument('--no-cpu-baseline', action='store_true')
    ap.add_argument('--no-comparators', action='store_true',
                    help='skip the same-box GPU comparators (N=1)')
    ap.add_argument('--exchange', choices=['auto', 'nccl', 'copy'],
                    default='auto',
                    help='ulysses at N > 1: NCCL all-to-alls, copy-engine '
                         'copies between IPC-mapped buffers, or (auto) the '
                         'one measured faster at N: copy at 2 GPUs, NCCL '
                         'above')
    ap.add_argument('--fwd-groups', type=int, choices=[1, 2], default=2,
                    help="the attention forward's softmax: two groups of "
                         'warps on alternate key blocks (2) or one (1)')
    ap.add_argument('--only', choices=['backward', 'heat', 'teacher',
                                       'compensation', 'search'],
                    default=None,
                    help='time one stage on head group 0 of the config '
                         '(for kernel profiling)')
    ap.add_argument('--reduce', choices=['sum', 'max'], default='sum',
                    help="heat reduction for --only heat")
    ap.add_argument('--teacher', choices=['fused', 'separate'],
                    default='fused',
                    help='cfg5 teacher: one fused dense + LSE + heat pass per '
                         'head group, or the dense kernel then the heat kernel')
    ap.add_argument('--query-tiles', type=int, default=40,
                    help='sampled query tiles for --only search (the '
                         "reference's SearchConfig default)")
    ap.add_argument('--pieces', type=int, default=1,
                    help='ulysses: head pieces whose exchanges overlap')
    ap.add_argument('--reserve-sms', type=int, default=16,
                    help='ulysses: SMs the attention leaves to NCCL while '
                    'pieces overlap')
    ap.add_argument('--parallel', choices=['clips', 'ulysses'],
                    default='ulysses',
                    help='multi-GPU mode: heads split over the ranks '
                         '(ulysses) or one clip per rank (clips)')
    args = ap.parse_args()
    cfg = CONFIGS[args.config]
    if args.impl == 'reference':
        run_reference(args, cfg)
        return
    kernels.set_fwd_groups(args.fwd_groups)
    if args.warmup < 3:
        raise SystemExit('use at least 3 warm-up steps')
    if args.only:
        run_stage(args, cfg)
        return
    if cfg.get('train'):
        run_train_step(args, cfg)
        return

    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local_rank = int(os.environ.get('LOCAL_RANK', '0'))
    if world != args.gpus:
        raise SystemExit(f'--gpus {args.gpus} but WORLD_SIZE={world}')
    device = torch.device('cuda', local_rank)
    torch.cuda.set_device(device)
    if world > 1:
        import datetime
        dist.init_process_group('nccl', device_id=device,
                                timeout=datetime.timedelta(seconds=120))

    seq_len, heads = cfg['seq_len'], cfg['heads']
    mode = args.parallel
    heads_split = world > 1 and mode == 'ulysses'
    if heads_split and (heads % world or seq_len % world):
        raise SystemExit('heads and sequence must divide by the GPU count')
    full_plan = veda_plan.TilePlan(
        'bench', cfg['target'][1],
        [tiling.TileShape(*s) for s in cfg['shapes']], [cfg['head_shape']])
    plan = ulysses.local_plan(full_plan, rank, world) if heads_split else None
    student, clip, plan, local_heads = build_student(cfg, device, plan)
    if heads_split:
        shard = seq_len // world
        q, k, v = synthetic_qkv(cfg, shard, rank * shard, device)
        exchange = args.exchange
        if exchange == 'auto':
            # cfg3 on B200: 2 GPUs copy 15.4 ms/layer against NCCL 17.1;
            # 8 GPUs copy 4.76 against NCCL 4.59 (narrower strided rows per
            # peer, more host barriers).
            exchange = 'copy' if world == 2 else 'nccl'
        args.exchange = exchange
        fn = ulysses.UlyssesSparseStudent(student, pieces=args.pieces,
                                          reserve_sms=args.reserve_sms,
                                          transport=exchange)
    else:
        # The whole layer on this rank's own clip (clip 0 on one GPU).
        q, k, v = synthetic_qkv(cfg, seq_len, 0, device, clip=rank)
        fn = student
    events = veda_attention.StageEvents()

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    with torch.no_grad():
        for _ in range(args.warmup):
            fn(q, k, v, 0)
        barrier()
        student.events = events
        events.clear()
        stream = torch.cuda.current_stream()
        start = torch.cuda.Event(enable_timing=True)
        stop = torch.cuda.Event(enable_timing=True)
        with ClockSampler(device) as clocks:
            start.record(stream)
            clocks.mark('t0')
            for _ in range(args.steps):
                fn(q, k, v, 0)
            stop.record(stream)
            barrier()
            clocks.mark('t1')
        student.events = veda_attention._NO_EVENTS  # pylint: disable=protected-access
        ms = start.elapsed_time(stop) / args.steps
        stages = {n: t / args.steps for n, t in events.totals_ms().items()}
        # Algorithmic work of the local heads (counted after the timing).
        blocks = 0
        for group in plan.head_groups(0, device):
            tl = clip.get(group.shape)
            qt, fq = tiling.gather_and_pool(ulysses.seq_to_heads(q)
                                            if heads_split else q, tl,
                                            group.heads)
            kt, fk = tiling.gather_and_pool(ulysses.seq_to_heads(k)
                                            if heads_split else k, tl,
                                            group.heads)
            logits = student.predictor.layers[0](
                fq, fk, group.heads + (rank * local_heads if heads_split
                                       else 0))
            lists = veda_mask.select_block_lists(
                logits[:, :tl.n_video_tiles], tl, clip.blocks(tl))
            blocks += int(lists.part_cnt.sum() + lists.full_cnt.sum())
            del qt, kt
        # End to end through the public API with host buffers: every step
        # copies its q, k, v shard from pinned host memory, runs the layer
        # and copies the output back (HostPipeline: step i + 1's inputs and
        # step i - 1's output move while step i computes).
        host = [t.cpu().pin_memory() for t in (q, k, v)]
        out_host = torch.empty_like(host[0]).pin_memory()
        pipe = HostPipeline(fn, q.shape, q.dtype, device)
        e2e_steps = min(args.steps, 30)
        for _ in range(2):
            pipe(*host, 0, out_host)
        pipe.synchronize()
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(pipe.h2d)
        for _ in range(e2e_steps):
            pipe(*host, 0, out_host)
        pipe.wait_on(stream)
        e1.record(stream)
        barrier()
        e2e_ms = e0.elapsed_time(e1) / e2e_steps

        dense = dense_comparison(cfg, q, k, v) if world == 1 else None
        comp = (comparators(cfg, clip, plan, student, q, k, v)
                if world == 1 and not args.no_comparators else None)

    vals = torch.tensor([ms, e2e_ms, stages.get('attention', 0.0),
                         float(blocks)], dtype=torch.float64, device=device)
    if world > 1:
        mx = vals[:3].clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        tot = vals[3:].clone()
        dist.all_reduce(tot, op=dist.ReduceOp.SUM)
        vals = torch.cat([mx, tot])
    ms, e2e_ms, attn_ms, total_blocks = vals.tolist()
    # Clips mode: `world` layers ran in the max-over-ranks time, so the whole
    # job spends ms / world per layer.
    layers = 1 if heads_split else world
    step_ms = ms
    ms, e2e_ms = ms / layers, e2e_ms / layers
    if rank == 0:
        peaks = load_peaks()
        peak = peaks['bf16_tflops']
        flops = total_blocks * BLOCK_FLOPS
        dense_flops = 4.0 * cfg['used'] ** 2 * 128 * heads * layers
        eff = flops / (ms * layers * 1e-3) / 1e12
        attn_tflops = (flops / world) / (attn_ms * 1e-3) / 1e12
        clk = clocks.summary()
        line = {
            'metric': METRIC, 'value': ms, 'unit': 'ms/layer',
            'n_gpus': world, 'steps': args.steps, 'warmup': args.warmup,
            'ms_per_step': step_ms, 'higher_is_better': False,
            'scaling': 'strong' if heads_split or world == 1 else 'weak',
            'vs_baseline': None, 'dtype': 'bf16',
            'data': 'synthetic (seeded N(0,1) q/k/v, random-init predictor '
                    'N(0,0.02))',
            'config': {'workload': f'{args.config}: {cfg["desc"]}',
                       'heads': heads, 'seq_len': seq_len, 'head_dim': 128,
                       'parallelism': (f'clip per GPU x{world}'
                                       if mode == 'clips' else
                                       f'ulysses-heads x{world}'),
                       'softmax_groups': args.fwd_groups,
                       'exchange': (args.exchange if heads_split
                                    else None),
                       'l2': 'inputs exceed L2 (q/k/v/tiles >> 126 MB)'},
            'effective_tflops': eff,
            'frac_of_peak': eff / peak,
            'computed_blocks': int(total_blocks),
            'dense_equiv_tflop': dense_flops / 1e12,
            'stages_ms': stages,
            'roofline': tensor_roofline(
                peaks, attn_tflops, step_ms * args.steps * 1e-3,
                'bsa_fwd_kernel',
                FWD_TRAFFIC.get(args.config) if world == 1 else None),
            # Bytes of all ranks per step (each rank copies its q, k, v in
            # and its output back).
            'e2e': {'value': e2e_ms, 'unit': 'ms/layer', 'steps': e2e_steps,
                    'h2d_bytes_per_step': world * 3 * q.numel() * 2,
                    'd2h_bytes_per_step': world * q.numel() * 2},
            'gpu_launches': args.steps * launches_per_step(
                clip, plan, heads_split, args.pieces if heads_split else 1),
            'clocks': clk,
        }
        if dense is not None:
            best = min(dense, key=dense.get)
            line['dense'] = {
                'ms': dense, 'unit': 'ms/layer', 'fastest': best,
                'speedup_vs_fastest_dense': dense[best] / ms,
                'note': 'dense attention of the same q, k, v over the used '
                        'rows (no permutation, predictor or top-k), timed '
                        'with CUDA events; the sparse layer is the whole '
                        'Veda path'}
        if comp is not None:
            line['comparators'] = comp
        if world == 1 and not args.no_cpu_baseline:
            got = reference_cpu_ms(cfg)
            if got is not None:
                per_step, threads, sample = got
                line['cpu_baseline'] = {
                    'value': sum(per_step) / len(per_step),
                    'unit': 'ms/layer', 'cores': threads,
                    'kind': 'reference',
                    'sample': f'{len(per_step)} steps: {sample}'}
            else:
                cpu_ms, n_heads, threads, _ = cpu_baseline(cfg)
                line['cpu_baseline'] = {
                    'value': cpu_ms, 'unit': 'ms/layer', 'cores': threads,
                    'kind': 'port',
                    'sample': f'{n_heads} heads of {heads} through the '
                              'oracle (numpy restatement), full layer per '
                              'head, extrapolated linearly over heads'}
        print(json.dumps(line), flush=True)
    if heads_split:
        fn.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# DRAM bytes (read + write) of one bsa_fwd_kernel launch (one head group),
# from single-pass ncu captures of the two-group kernel
# (dram__bytes_read.sum + dram__bytes_write.sum): config 2, and config 3 at
# full size (3.18 GB + 0.57 GB per launch). Other configs: null.
FWD_TRAFFIC = {'cfg2': 864.2e6, 'cfg3': 3.748e9}


def dense_comparison(cfg, q, k, v, reps=3):
    """ms per call of dense attention of the same q, k, v over the used rows:
    this library's dense kernel and torch's fused SDPA backends (cuDNN,
    flash) where they run on this device. Each backend is timed after one
    warm-up call; backends that raise are left out."""
    from miowtion_b200 import kernels
    import torch.nn.functional as F
    from torch.nn.attention import SDPBackend, sdpa_kernel
    used = cfg['used']
    out = {}

    def timed(fn):
        fn()
        torch.cuda.synchronize()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / reps

    with torch.no_grad():
        out['b200_dense_kernel'] = timed(
            lambda: kernels.dense_attention(q, k, v, 128 ** -0.5, False,
                                            used=used))
        # [1, H, used, D] views in the layout SDPA wants (copies made once,
        # outside the timed calls).
        qs, ks, vs = (t[:used].permute(1, 0, 2).unsqueeze(0).contiguous()
                      for t in (q, k, v))
        for name, backend in (('sdpa_cudnn', SDPBackend.CUDNN_ATTENTION),
                              ('sdpa_flash', SDPBackend.FLASH_ATTENTION)):
            try:
                with sdpa_kernel(backend):
                    out[name] = timed(lambda: F.scaled_dot_product_attention(
                        qs, ks, vs))
            except RuntimeError:
                continue
        del qs, ks, vs
    return out


REF_DIR = os.path.join(ROOT, 'baseline', '_ref')


def reference_package():
    """The reference's own package, installed unmodified (`pip install
    --no-deps` of the reference project) under baseline/_ref, or None when
    that install is absent."""
    if not os.path.isdir(os.path.join(REF_DIR, 'miowtion')):
        return None
    if REF_DIR not in sys.path:
        sys.path.append(REF_DIR)
    import importlib
    return importlib.import_module('miowtion')


def _timed_ms(fn, reps):
    fn()
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / reps


def _rel_err(got, want):
    got, want = got.float(), want.float()
    return float((got - want).abs().max() / want.abs().max().clamp(min=1e-30))


def comparators(cfg, clip, plan, student, q, k, v, reps=3):
    """Same-box GPU comparators for head group 0 of the layer: this
    library's kernels beside the reference's own GPU kernels, run
    unmodified from baseline/_ref through their public functions
    (kernels/tile_gather_triton.py:156-224, kernels/block_heat_triton.py:
    140-173), torch flex_attention with a BlockMask of the same lists
    through the reference's benchmark backend (kernels/bench.py:241-262),
    and FA4 SM100 where it can be imported. ms per call, CUDA events,
    after one warm-up call; each entry that cannot run says why. Every
    pair is checked to compute the same thing (max relative difference)."""
    from miowtion_b200 import heatmap
    device = q.device
    res: dict = {}
    group = plan.head_groups(0, device)[0]
    tl = clip.get(group.shape)
    heads = group.heads
    res['workload'] = (f'head group 0 ({heads.numel()} heads, tile '
                       f'{group.shape.t}x{group.shape.h}x{group.shape.w}, '
                       f'{tl.n_tiles} tiles)')
    with torch.no_grad():
        qt, fq = tiling.gather_and_pool(q, tl, heads)
        kt, fk = tiling.gather_and_pool(k, tl, heads)
        vt = tiling.gather_tiles(v, tl, heads)
        logits = student.predictor.layers[0](fq, fk, heads)
        lists = veda_mask.select_block_lists(
            logits[:, :tl.n_video_tiles], tl, clip.blocks(tl),
            want_mask=True)
        ours = {
            'gather_pool_q_k_gather_v': _timed_ms(lambda: (
                tiling.gather_and_pool(q, tl, heads),
                tiling.gather_and_pool(k, tl, heads),
                tiling.gather_tiles(v, tl, heads)), reps),
            'packed_pool_q_images_k_v': _timed_ms(lambda: (
                tiling.pool_features(q, tl, heads),
                tiling.gather_images(k, tl, heads, pool=True),
                tiling.gather_images(v, tl, heads)), reps)}
        buf = torch.zeros(q.shape[0] + 1, q.shape[1], 128,
                          dtype=q.dtype, device=device)
        ours['scatter'] = _timed_ms(
            lambda: tiling.scatter_tiles_(buf, qt, tl, heads), reps)
        ot = kernels.block_sparse_attention_lists(qt, kt, vt, lists, tl)
        ours['block_sparse_attention'] = _timed_ms(
            lambda: kernels.block_sparse_attention_lists(qt, kt, vt, lists,
                                                         tl), reps)
        _, lse = kernels.dense_attention(q, k, v, 128 ** -0.5, True,
                                         used=cfg['used'])
        lse_t = tiling.gather_lse(lse, tl, heads)
        del lse
        rows = torch.arange(tl.n_tiles, device=device)
        heat = heatmap.teacher_heat(qt, kt, lse_t, tl, rows, 'sum')
        ours['teacher_heat_sum_all_query_tiles'] = _timed_ms(
            lambda: heatmap.teacher_heat(qt, kt, lse_t, tl, rows, 'sum'), 1)
        res['b200_ms'] = ours

        ref = None
        try:
            ref = reference_package()
        except Exception as exc:  # pylint: disable=broad-except
            res['reference_triton'] = f'unavailable: import failed ({exc})'
        if ref is None and 'reference_triton' not in res:
            res['reference_triton'] = ('unavailable: the reference is not '
                                       'installed under baseline/_ref')
        if ref is not None:
            theirs, same = {}, {}
            try:
                from miowtion.kernels import block_heat_triton as rbh
                from miowtion.kernels import tile_gather_triton as rtg
                from miowtion.veda import tiling as rtiling
                spans = []
                if cfg['cond'] is not None:
                    spans.append(rtiling.TiledSpan(
                        cfg['cond'][0], tuple(cfg['cond'][1]),
                        rtiling.TileShape(2, 8, 8)))
                spans.append(rtiling.TiledSpan(
                    cfg['target'][0], tuple(cfg['target'][1]),
                    rtiling.TileShape(group.shape.t, group.shape.h,
                                      group.shape.w)))
                rl = rtiling.build_tile_layout(spans, cfg['used'],
                                               q.shape[0], device)
                rqt, rfq = rtg.gather_and_pool(q, rl, heads)
                same['gather_tiles_equal'] = bool(torch.equal(rqt, qt))
                same['pool_rel_diff'] = _rel_err(rfq, fq)
                theirs['gather_pool_q_k_gather_v'] = _timed_ms(lambda: (
                    rtg.gather_and_pool(q, rl, heads),
                    rtg.gather_and_pool(k, rl, heads),
                    rtg.gather_tiles(v, rl, heads)), reps)
                rbuf = torch.zeros_like(buf)
                rtg.scatter_tiles_(rbuf, qt, rl, heads)
                tiling.scatter_tiles_(buf, qt, tl, heads)
                same['scatter_equal'] = bool(torch.equal(rbuf, buf))
                theirs['scatter'] = _timed_ms(
                    lambda: rtg.scatter_tiles_(rbuf, qt, rl, heads), reps)
                del rbuf, rqt, rfq
            except Exception as exc:  # pylint: disable=broad-except
                theirs['error'] = f'{type(exc).__name__}: {exc}'[:300]
            try:
                rheat = rbh.teacher_heat(qt, kt, lse_t, rl, rows, 'sum')
                same['teacher_heat_rel_diff'] = _rel_err(heat, rheat)
                theirs['teacher_heat_sum_all_query_tiles'] = _timed_ms(
                    lambda: rbh.teacher_heat(qt, kt, lse_t, rl, rows,
                                             'sum'), 1)
                del rheat
            except Exception as exc:  # pylint: disable=broad-except
                # Triton 3.6 (the image's) fails to compile this kernel
                # for sm_100: an MLIR pass error, not a wrong result.
                theirs['teacher_heat_sum_all_query_tiles'] = (
                    'unavailable: the Triton compile failed on this box '
                    f'({type(exc).__name__}: {str(exc)[:120]})')
            res['reference_triton_ms'] = theirs
            res['agreement'] = same
            try:
                from miowtion.kernels import bench as rbench
                flex = rbench._Flex(qt, kt, vt)  # pylint: disable=protected-access
                meta = flex.prepare(lists.mask.bool())
                fo = flex.run(meta)
                res['flex_attention_ms'] = _timed_ms(lambda: flex.run(meta),
                                                     reps)
                # The reference backend's BlockMask has no partial tiles:
                # flex attends every slot of a kept tile, the zero padding
                # keys included. This library's forward does the same when
                # told every tile has 128 real rows, so compare against that
                # on every row.
                res['flex_note'] = (
                    'torch.compile(flex_attention) with the same kept '
                    'blocks as full blocks (the reference backend, '
                    'kernels/bench.py:241-262); tile-ordered q, k, v; '
                    'agreement against this library\'s forward with every '
                    'tile taken as full')
                import dataclasses
                as_full = dataclasses.replace(
                    tl, valid_count=torch.full_like(tl.valid_count, 128))
                of = kernels.block_sparse_attention_lists(qt, kt, vt, lists,
                                                          as_full)
                res['flex_rel_diff'] = _rel_err(fo, of)
                del of
                del flex, meta, fo
            except Exception as exc:  # pylint: disable=broad-except
                res['flex_attention_ms'] = (
                    f'unavailable: {type(exc).__name__}: {exc}'[:300])
        import importlib.util
        if importlib.util.find_spec('flash_attn') is None or \
                importlib.util.find_spec('flash_attn.cute') is None:
            res['fa4_sm100'] = ('not installable on this box: flash-attn-4 '
                                '(flash_attn.cute @ d15f1531) is not in the '
                                'image and there is no network')
    return res


def run_stage(args, cfg):
    """One stage on one GPU, head group 0 of the config: the block-sparse
    backward (prep, dq, dk/dv), the teacher heat for every query tile, the
    zero-order compensation of every query tile, or the tile-search oracle
    error of one candidate shape. The line's unit is ms per call of that
    stage."""
    from miowtion_b200 import heatmap
    from miowtion_b200 import kernels
    device = torch.device('cuda', 0)
    torch.cuda.set_device(device)
    student, clip, plan, _ = build_student(cfg, device)
    q, k, v = synthetic_qkv(cfg, cfg['seq_len'], 0, device)
    group = plan.head_groups(0, device)[0]
    tl = clip.get(group.shape)
    heads = group.heads.numel()
    if args.only == 'backward':
        qt, fq = tiling.gather_and_pool(q, tl, group.heads)
        kt, fk = tiling.gather_and_pool(k, tl, group.heads)
        vt = tiling.gather_tiles(v, tl, group.heads)
        del q, k, v
        with torch.no_grad():
            logits = student.predictor.layers[0](fq, fk, group.heads)
            lists = veda_mask.select_block_lists(
                logits[:, :tl.n_video_tiles], tl, clip.blocks(tl),
                want_mask=True)
        t_lists = kernels.index_lists_from_mask(lists.mask, tl)
        out, lse = kernels.block_sparse_attention_lists(qt, kt, vt, lists, tl,
                                                        return_lse=True)
        gen = torch.Generator(device=device).manual_seed(cfg.get('dout_seed',
                                                                 4))
        dout = torch.randn(qt.shape, generator=gen, device=device).to(
            torch.bfloat16)
        blocks = int((lists.part_cnt.long() + lists.full_cnt.long()).sum())
        flops = 2.5 * blocks * BLOCK_FLOPS

        def call():
            kernels.block_sparse_attention_bwd(qt, kt, vt, out, dout, lse,
                                               lists, t_lists, tl)
        what = 'block-sparse backward (prep + dq + dk/dv)'
    elif args.only == 'teacher':
        qt = tiling.gather_tiles(q, tl, group.heads)
        kt = tiling.gather_tiles(k, tl, group.heads)
        vt = tiling.gather_tiles(v, tl, group.heads)
        del q, k, v
        blocks = tl.n_tiles ** 2 * heads
        # Dense QK^T and PV of every block; the heat reuses the scores.
        flops = 4.0 * blocks * 128 ** 3

        def call():
            heatmap.fused_dense_heat(qt, kt, vt, tl, args.reduce)
        what = (f'fused dense attention + LSE + heat (reduce={args.reduce}), '
                'all query tiles')
    elif args.only == 'compensation':
        from miowtion_b200 import compensation
        qt, fq = tiling.gather_and_pool(q, tl, group.heads)
        kt, fk = tiling.gather_and_pool(k, tl, group.heads)
        vt = tiling.gather_tiles(v, tl, group.heads)
        del q, k, v
        with torch.no_grad():
            logits = student.predictor.layers[0](fq, fk, group.heads)
            lists = veda_mask.select_block_lists(
                logits[:, :tl.n_video_tiles], tl, clip.blocks(tl))
        o_kept, lse = kernels.block_sparse_attention_lists(
            qt, kt, vt, lists, tl, return_lse=True)
        out = torch.empty_like(o_kept)
        blocks = tl.n_tiles * heads  # (query tile, head) items
        # Two GEMMs per (query tile, head) against every key centroid.
        flops = 4.0 * blocks * 128 * tl.n_tiles * 128

        def call():
            compensation.compensate_lists(o_kept, lse, qt, kt, vt, lists, tl,
                                          out=out)
        what = ('zero-order compensation (centroid summaries + tcgen05 '
                'centroid pass), all query tiles')
    elif args.only == 'search':
        from miowtion_b200 import search
        qg, kg, vg = (t.index_select(1, group.heads).contiguous()
                      for t in (q, k, v))
        del q, k, v
        with torch.no_grad():
            dense, lse = kernels.dense_attention(qg, kg, vg, 128 ** -0.5,
                                                 True, used=cfg['used'])
        gen = torch.Generator().manual_seed(0)
        count = min(args.query_tiles, tl.n_video_tiles)
        rows = torch.randperm(tl.n_video_tiles, generator=gen)[:count].sort(
        ).values.to(device)
        blocks = count * heads
        # Heat QK^T of the sampled tiles against every key tile; the sparse
        # forward of the kept blocks is small beside it.
        flops = 2.0 * blocks * tl.n_tiles * 128 ** 3

        def call():
            search.oracle_rel_mse(qg, kg, vg, tl, clip.blocks(tl), rows,
                                  dense_out=dense, lse=lse)
        what = (f'tile-search oracle rel-MSE of one candidate, {count} '
                'sampled query tiles')
    else:
        with torch.no_grad():
            _, lse = kernels.dense_attention(q, k, v, 128 ** -0.5, True,
                                             used=cfg['used'])
        lse_t = tiling.gather_lse(lse, tl, group.heads)
        qt = tiling.gather_tiles(q, tl, group.heads)
        kt = tiling.gather_tiles(k, tl, group.heads)
        del q, k, v, lse
        rows = torch.arange(tl.n_tiles, device=device)
        blocks = tl.n_tiles ** 2 * heads
        flops = 2.0 * blocks * 128 ** 3

        def call():
            heatmap.teacher_heat(qt, kt, lse_t, tl, rows, args.reduce)
        what = f'teacher heat (reduce={args.reduce}), all query tiles'
    for _ in range(args.warmup):
        call()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        call()
    stop.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(stop) / args.steps
    peaks = load_peaks()
    print(json.dumps({
        'metric': f'{args.only} ms per call', 'value': ms, 'unit': 'ms',
        'n_gpus': 1, 'steps': args.steps, 'warmup': args.warmup,
        'higher_is_better': False, 'dtype': 'bf16', 'data': 'synthetic',
        'config': {'workload': f'{args.config} head group 0 ({heads} heads, '
                               f'{tl.n_tiles} tiles): {what}'},
        'blocks': blocks,
        'tflops': flops / (ms * 1e-3) / 1e12,
        'frac_of_peak': flops / (ms * 1e-3) / 1e12 / peaks['bf16_tflops'],
        'flops_accounting': {
            'backward': "2.5 x the forward per computed block (the "
                        "reference's)",
            'heat': '2 x 128^3 per block of QK^T',
            'teacher': '4 x 128^3 per block (QK^T and PV, every block)',
            'compensation': '4 x 128 x n_tiles x 128 per (query tile, head)',
            'search': '2 x 128^3 per heat block of the sampled tiles',
        }[args.only]}), flush=True)


def run_train_step(args, cfg):
    """Config 5: the teacher (dense forward with LSE and the block heat
    with reduce='sum' for every query tile) and the sparse student forward +
    backward on the same q, k, v.

    `--teacher fused` (default): per head group, q, k, v in tile order, one
    pass of the fused dense + LSE + heat kernel, and the teacher output
    scattered back to its rows. `--teacher separate`: the dense kernel over
    the packed sequence, the LSE gathered into tile order, and the heat
    kernel recomputing QK^T.

    On N GPUs the heads are split (Ulysses): each rank holds a [S/N, H, D]
    shard of q, k, v and dO; one all-to-all per tensor brings the rank's
    H/N heads of every row, the teacher and the student run on them, and
    the student's output returns to the shard through the inverse exchange.
    The backward exchanges dO into the head layout and dQ, dK, dV back to
    the shards (autograd through the exchanges). Strong scaling: the value
    is the time of one step of the whole clip, the max over ranks."""
    from miowtion_b200 import heatmap
    from miowtion_b200 import kernels
    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local_rank = int(os.environ.get('LOCAL_RANK', '0'))
    if world != args.gpus:
        raise SystemExit(f'--gpus {args.gpus} but WORLD_SIZE={world}')
    if world > 1 and args.parallel != 'ulysses':
        raise SystemExit('cfg5 on several GPUs splits the heads '
                         '(--parallel ulysses)')
    device = torch.device('cuda', local_rank)
    torch.cuda.set_device(device)
    if world > 1:
        import datetime
        dist.init_process_group('nccl', device_id=device,
                                timeout=datetime.timedelta(seconds=120))
    seq_len, heads = cfg['seq_len'], cfg['heads']
    if heads % world or seq_len % world:
        raise SystemExit('heads and sequence must divide by the GPU count')
    full_plan = veda_plan.TilePlan(
        'bench', cfg['target'][1],
        [tiling.TileShape(*s) for s in cfg['shapes']], [cfg['head_shape']])
    plan = ulysses.local_plan(full_plan, rank, world) if world > 1 else None
    student, clip, plan, _ = build_student(cfg, device, plan)
    shard = seq_len // world
    rows = slice(rank * shard, (rank + 1) * shard)
    q, k, v = synthetic_qkv(cfg, shard, rank * shard, device)
    gen = torch.Generator(device=device).manual_seed(cfg['dout_seed'])
    dout = torch.randn(seq_len, heads, 128, generator=gen,
                       device=device).to(torch.bfloat16)[rows].contiguous()
    uly = ulysses.UlyssesSparseStudent(student) if world > 1 else None
    local = uly.local(0) if uly is not None else student
    scale = 128 ** -0.5
    groups = plan.head_groups(0, device)  # this rank's heads
    stream = torch.cuda.current_stream()
    fused = args.teacher == 'fused'
    names = ['exchange_in']
    names += (['teacher_gather', 'teacher_fused'] if fused else
              ['dense_fwd_lse', 'heat'])
    names += ['student_fwd', 'student_bwd']
    stage_ms = dict.fromkeys(names, 0.0)
    local_heads = len(plan.head_shape[0])
    teacher_out = torch.empty(seq_len + 1, local_heads, 128,
                              dtype=torch.bfloat16, device=device)

    def step(qs, ks, vs, dos, timed):
        marks = [torch.cuda.Event(enable_timing=True)
                 for _ in range(len(names) + 1)]
        marks[0].record(stream)
        leaves = [t.detach().requires_grad_(True) for t in (qs, ks, vs)]
        with torch.enable_grad():
            if uly is not None:
                qh, kh, vh = (uly.to_heads(t) for t in leaves)
            else:
                qh, kh, vh = leaves
        marks[1].record(stream)
        with torch.no_grad():
            tq, tk, tv = (t.detach() for t in (qh, kh, vh))
            heat_sum = 0.0
            if fused:
                tiles = []
                for g in groups:
                    tl = clip.get(g.shape)
                    tiles.append([tiling.gather_tiles(t, tl, g.heads)
                                  for t in (tq, tk, tv)])
                marks[2].record(stream)
                for g, (qt, kt, vt) in zip(groups, tiles):
                    tl = clip.get(g.shape)
                    out_t, _, heat = heatmap.fused_dense_heat(qt, kt, vt, tl,
                                                              'sum')
                    tiling.scatter_tiles_(teacher_out, out_t, tl, g.heads)
                    heat_sum = heat_sum + heat.sum()
                del tiles
            else:
                _, lse = kernels.dense_attention(tq, tk, tv, scale, True,
                                                 used=cfg['used'])
                marks[2].record(stream)
                for g in groups:
                    tl = clip.get(g.shape)
                    lse_t = tiling.gather_lse(lse, tl, g.heads)
                    qt = tiling.gather_tiles(tq, tl, g.heads)
                    kt = tiling.gather_tiles(tk, tl, g.heads)
                    heat = heatmap.teacher_heat(
                        qt, kt, lse_t, tl,
                        torch.arange(tl.n_tiles, device=device), 'sum')
                    heat_sum = heat_sum + heat.sum()
                    del qt, kt, lse_t
            marks[3].record(stream)
        with torch.enable_grad():
            out = local(qh, kh, vh, 0)
            if uly is not None:
                out = uly.to_seq(out)
            marks[4].record(stream)
            out.backward(dos)
        marks[5].record(stream)
        if timed:
            torch.cuda.synchronize()
            for i, n in enumerate(names):
                stage_ms[n] += marks[i].elapsed_time(marks[i + 1])
        return heat_sum + leaves[0].grad.float().abs().sum() * 0

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step(q, k, v, dout, False)
    barrier()
    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)
    with ClockSampler(device) as clocks:
        start.record(stream)
        clocks.mark('t0')
        for _ in range(args.steps):
            step(q, k, v, dout, False)
        stop.record(stream)
        barrier()
        clocks.mark('t1')
    ms = start.elapsed_time(stop) / args.steps
    # Stage split (separate, synchronised passes).
    for _ in range(2):
        step(q, k, v, dout, True)
    barrier()
    stages = {n: t / 2 for n, t in stage_ms.items()}
    # End to end: H2D of this step's q, k, v, dO shards from pinned memory,
    # the step, D2H of its scalar result.
    host = [t.cpu().pin_memory() for t in (q, k, v, dout)]
    dev_in = [torch.empty_like(t) for t in (q, k, v, dout)]
    res_host = torch.empty((), dtype=torch.float32).pin_memory()
    e2e_steps = max(1, min(args.steps, 5))
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        for d, h in zip(dev_in, host):
            d.copy_(h, non_blocking=True)
        res_host.copy_(step(*dev_in, False), non_blocking=True)
    e1.record(stream)
    barrier()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    # Algorithmic work of this rank's heads (counted after timing).
    blocks = 0
    with torch.no_grad():
        qh = uly.to_heads(q) if uly is not None else q
        kh = uly.to_heads(k) if uly is not None else k
        for g in groups:
            tl = clip.get(g.shape)
            _, fq = tiling.gather_and_pool(qh, tl, g.heads)
            _, fk = tiling.gather_and_pool(kh, tl, g.heads)
            logits = local.predictor.layers[0](fq, fk,
                                               g.heads + local.head_offset)
            lists = veda_mask.select_block_lists(
                logits[:, :tl.n_video_tiles], tl, clip.blocks(tl))
            blocks += int(lists.part_cnt.sum() + lists.full_cnt.sum())
        del qh, kh
    used = cfg['used']
    heat_flops = sum(2.0 * (clip.get(g.shape).n_tiles * 128) ** 2 * 128 *
                     g.heads.numel() for g in groups)
    # The fused pass runs the dense attention over the tile-ordered rows
    # (padding slots included) and no second QK^T.
    fused_exec_flops = sum(4.0 * (clip.get(g.shape).n_tiles * 128) ** 2 *
                           128 * g.heads.numel() for g in groups)
    qtile_heads = sum(clip.get(g.shape).n_tiles * g.heads.numel()
                      for g in groups)
    maxv = torch.tensor([ms, e2e_ms] + [stages[n] for n in names],
                        dtype=torch.float64, device=device)
    sums = torch.tensor([float(blocks), heat_flops, fused_exec_flops,
                         float(qtile_heads)], dtype=torch.float64,
                        device=device)
    if world > 1:
        dist.all_reduce(maxv, op=dist.ReduceOp.MAX)
        dist.all_reduce(sums, op=dist.ReduceOp.SUM)
    ms, e2e_ms, *stage_vals = maxv.tolist()
    stages = dict(zip(names, stage_vals))
    if world == 1:
        del stages['exchange_in']
    blocks, heat_flops, fused_exec_flops, qtile_heads = sums.tolist()
    blocks = int(blocks)
    dense_flops = 4.0 * used ** 2 * 128 * heads
    sparse_flops = 3.5 * blocks * BLOCK_FLOPS  # fwd + bwd (2.5x fwd)
    total = dense_flops + heat_flops + sparse_flops
    if rank == 0:
        peaks = load_peaks()
        peak = peaks['bf16_tflops']
        # Per-GPU rates: each rank's share of the work over its stage time.
        bwd_tflops = 2.5 * blocks * BLOCK_FLOPS / world / \
            stages['student_bwd'] / 1e9
        if fused:
            achieved = fused_exec_flops / world / stages['teacher_fused'] / 1e9
            stage_tflops = {
                'teacher_fused_executed': achieved,
                'teacher_reference_accounting': (dense_flops + heat_flops) /
                                                world /
                                                stages['teacher_fused'] / 1e9,
                'student_bwd_attention_equiv': bwd_tflops}
            kernel = (('pair_fwd_kernel<heat>' if args.fwd_groups == 2 else
                       'bsa_fwd_kernel<heat>') +
                      ' (fused dense + LSE + heat, executed FLOPs over '
                      'tile-ordered rows)')
        else:
            achieved = dense_flops / world / stages['dense_fwd_lse'] / 1e9
            stage_tflops = {
                'dense_fwd_lse': achieved,
                'heat': heat_flops / world / stages['heat'] / 1e9,
                'student_bwd_attention_equiv': bwd_tflops}
            kernel = 'bsa_fwd_kernel (dense mode)'
        roofline = tensor_roofline(peaks, achieved,
                                   ms * args.steps * 1e-3, kernel, None)
        # Ours per step and rank. Teacher, separate: dense fwd, then per
        # group gather_lse, gather q, k, heat (1 + 4 per group); fused: per
        # group gather q, k, v, keep-all lists, fused pass, scatter (6).
        # Student per group: fwd gather+pool q, k, embed, logits, select,
        # transposed lists, gather v, attention, scatter (9 + 1), backward
        # gather dO, prep, dq, dkdv, scatter x3 (7). Head split: 4 packing
        # kernels around the forward exchanges and 4 around the backward's.
        per_step = ((6 * len(groups)) if fused else (1 + 4 * len(groups))) \
            + 17 * len(groups) + (8 if world > 1 else 0)
        line = {
            'metric': METRIC, 'value': ms, 'unit': 'ms/step',
            'n_gpus': world, 'steps': args.steps, 'warmup': args.warmup,
            'ms_per_step': ms, 'higher_is_better': False,
            'scaling': 'strong', 'vs_baseline': None, 'dtype': 'bf16',
            'data': 'synthetic (seeded N(0,1) q/k/v and dO, random-init '
                    'predictor N(0,0.02))',
            'config': {'workload': f'{args.config}: {cfg["desc"]}',
                       'heads': heads, 'seq_len': seq_len,
                       'head_dim': 128,
                       'parallelism': (f'ulysses-heads x{world}'
                                       if world > 1 else 'single GPU'),
                       'l2': 'inputs exceed L2 (q/k/v >> 126 MB)'},
            'stages_ms': stages,
            'computed_blocks': blocks,
            'algorithmic_tflop': total / 1e12,
            'effective_tflops': total / (ms * 1e-3) / 1e12,
            'frac_of_peak': total / (ms * 1e-3) / 1e12 / peak / world,
            'teacher': args.teacher,
            'stage_tflops': stage_tflops,
            'roofline': roofline,
            'e2e': {'value': e2e_ms, 'unit': 'ms/step', 'steps': e2e_steps,
                    'h2d_bytes_per_step': world * 4 * q.numel() * 2,
                    'd2h_bytes_per_step': world * 4},
            'gpu_launches': args.steps * world * per_step,
            'clocks': clocks.summary(),
            'query_tile_heads': int(qtile_heads),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def launches_per_step(clip, plan, heads_split, pieces=1):
    """Our kernels per layer. Per head group on the packed path: pool q,
    k and v to tile images (k pooled too), embed, logits, select, attention
    (7), plus the gather of the global query tiles when there are any; on
    the tile path gather+pool q, k, gather v, embed, logits, select,
    attention, scatter (8). Head-parallel: per piece three packs and an
    unpack of the exchange buffers."""
    n = 0
    for group in plan.head_groups(0, 'cpu'):
        tl = clip.get(group.shape)
        if kernels.packed_supported(tl) and not clip.config.compensated:
            n += 7 + (1 if tl.n_global_tiles else 0)
        else:
            n += 8
    if heads_split:
        n *= pieces
        n += 4 * pieces
    return n


if __name__ == '__main__':
    main()
