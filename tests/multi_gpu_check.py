"""Two-rank check of the head-parallel layer, run by tests/test_gpu_multi.py
under torchrun (one process per GPU, NCCL): on every rank, the exchanged
layer (both transports) and its gradients equal that rank's rows of one
process running every head, bit for bit."""

import datetime
import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, 'tests', 'golden'))

import inputs  # noqa: E402
from miowtion_b200 import attention as veda_attention  # noqa: E402
from miowtion_b200 import mask as veda_mask  # noqa: E402
from miowtion_b200 import plan as veda_plan  # noqa: E402
from miowtion_b200 import predictor as veda_predictor  # noqa: E402
from miowtion_b200 import tiling  # noqa: E402
from miowtion_b200 import ulysses  # noqa: E402


def main() -> None:
    rank = int(os.environ['RANK'])
    world = int(os.environ['WORLD_SIZE'])
    dev = torch.device('cuda', int(os.environ['LOCAL_RANK']))
    torch.cuda.set_device(dev)
    dist.init_process_group('nccl', device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    text, grid = 130, (4, 12, 20)
    heads = max(4, 2 * world)
    used = text + grid[0] * grid[1] * grid[2]
    seq_len = used + 2
    seq_len += (-seq_len) % world
    layout = veda_attention.PackedLayout(
        seq_len, used, (veda_attention.VideoSpan(text, grid),))
    config = veda_attention.VedaConfig(
        target_budget=veda_mask.Budget(ratio=0.3))
    clip = veda_attention.ClipTiling(layout, config, dev)
    full_plan = veda_plan.TilePlan(
        'u', grid, [tiling.TileShape(2, 8, 8), tiling.TileShape(1, 8, 16)],
        [[h % 2 for h in range(heads)]])
    pred = veda_predictor.TileScorePredictor(1, heads, 128)
    pq, pk = inputs.predictor_weights(heads, 128, 53, 0.02)
    with torch.no_grad():
        pred.layers[0].proj_q.copy_(pq)
        pred.layers[0].proj_k.copy_(pk)
    pred = pred.to(dev)
    q, k, v = (t.to(dev) for t in inputs.qkv(seq_len, heads, 128, 54,
                                             torch.bfloat16))
    dout = inputs.dout(q.shape, 55).to(dev)
    whole = veda_attention.SparseStudent(clip, full_plan, pred)
    shard = seq_len // world
    rows = slice(rank * shard, (rank + 1) * shard)
    local = veda_attention.SparseStudent(
        clip, ulysses.local_plan(full_plan, rank, world), pred)
    failures = []
    with torch.no_grad():
        want = whole(q, k, v, 0)[rows]
        for transport in ('nccl', 'copy'):
            fn = ulysses.UlyssesSparseStudent(local, transport=transport)
            for _ in range(2):
                got = fn(*(t[rows].contiguous() for t in (q, k, v)), 0)
                torch.cuda.synchronize()
                if not torch.equal(got, want):
                    failures.append(f'forward, {transport}')
            fn.close()
    leaves = [t.clone().requires_grad_(True) for t in (q, k, v)]
    whole(*leaves, 0).backward(dout)
    parts = [t[rows].clone().requires_grad_(True) for t in (q, k, v)]
    fn = ulysses.UlyssesSparseStudent(local)
    fn(*parts, 0).backward(dout[rows].contiguous())
    torch.cuda.synchronize()
    for name, a, b in zip('qkv', parts, leaves):
        if not torch.equal(a.grad, b.grad[rows]):
            failures.append(f'd{name}')
    flags = torch.tensor([len(failures)], device=dev)
    dist.all_reduce(flags)
    dist.barrier()
    dist.destroy_process_group()
    if failures:
        print(f'rank {rank}: mismatch in {failures}', flush=True)
    if int(flags.item()):
        sys.exit(1)
    print(f'rank {rank}: exchanged layer and gradients equal the '
          'one-process layer', flush=True)


if __name__ == '__main__':
    main()
