"""The head-parallel wrapper on one GPU (a one-rank NCCL group): every
piece student scores its heads with their global predictor indices, so the
pieced, exchanged layer equals the plain SparseStudent bit for bit (heads
are independent through every kernel). The multi-rank exchange itself is
tested over gloo on the CPU (tests/test_ulysses.py) and measured by
bench.py --gpus N --config cfg3."""

import os
import tempfile

import pytest
import torch
import torch.distributed as dist

import inputs
from miowtion_b200 import attention as veda_attention
from miowtion_b200 import mask as veda_mask
from miowtion_b200 import plan as veda_plan
from miowtion_b200 import predictor as veda_predictor
from miowtion_b200 import tiling
from miowtion_b200 import ulysses

pytestmark = pytest.mark.gpu

DEV = torch.device('cuda', 0)


@pytest.fixture(scope='module')
def one_rank_group():
    torch.cuda.set_device(DEV)
    with tempfile.TemporaryDirectory() as tmp:
        store = dist.FileStore(os.path.join(tmp, 'store'), 1)
        dist.init_process_group('nccl', store=store, rank=0, world_size=1,
                                device_id=DEV)
        yield
        dist.destroy_process_group()


@pytest.mark.parametrize('pieces', [1, 3])
def test_pieced_layer_equals_plain_student(one_rank_group, pieces):
    text, grid, heads = 130, (4, 12, 20), 5
    used = text + grid[0] * grid[1] * grid[2]
    seq_len = used + 14
    layout = veda_attention.PackedLayout(
        seq_len, used, (veda_attention.VideoSpan(text, grid),))
    config = veda_attention.VedaConfig(
        target_budget=veda_mask.Budget(ratio=0.3))
    clip = veda_attention.ClipTiling(layout, config, DEV)
    plan = veda_plan.TilePlan('u', grid, [tiling.TileShape(2, 8, 8),
                                          tiling.TileShape(1, 8, 16)],
                              [[0, 1, 1, 0, 1]])
    pred = veda_predictor.TileScorePredictor(1, heads, 128)
    pq, pk = inputs.predictor_weights(heads, 128, 44, 0.02)
    with torch.no_grad():
        pred.layers[0].proj_q.copy_(pq)
        pred.layers[0].proj_k.copy_(pk)
    student = veda_attention.SparseStudent(clip, plan, pred.to(DEV))
    q, k, v = (t.to(DEV) for t in inputs.qkv(seq_len, heads, 128, 45,
                                             torch.bfloat16))
    with torch.no_grad():
        want = student(q, k, v, 0)
        got = ulysses.UlyssesSparseStudent(student, pieces=pieces)(q, k, v, 0)
    torch.cuda.synchronize()
    assert torch.equal(got[:used], want[:used])


def test_copy_engine_exchange_equals_plain_student(one_rank_group):
    """The copy-engine transport (IPC-mapped buffers, 2-D copies, IPC
    events and host barriers) on one rank: the layer equals the plain
    SparseStudent bit for bit, on three calls in a row (the receive and
    result buffers are reused). Across GPUs the same code copies between
    devices; bench.py --exchange copy measures it."""
    text, grid, heads = 130, (4, 12, 20), 4
    used = text + grid[0] * grid[1] * grid[2]
    seq_len = used + 14
    layout = veda_attention.PackedLayout(
        seq_len, used, (veda_attention.VideoSpan(text, grid),))
    config = veda_attention.VedaConfig(
        target_budget=veda_mask.Budget(ratio=0.3))
    clip = veda_attention.ClipTiling(layout, config, DEV)
    plan = veda_plan.TilePlan('u', grid, [tiling.TileShape(2, 8, 8),
                                          tiling.TileShape(1, 8, 16)],
                              [[1, 0, 1, 0]])
    pred = veda_predictor.TileScorePredictor(1, heads, 128)
    pq, pk = inputs.predictor_weights(heads, 128, 49, 0.02)
    with torch.no_grad():
        pred.layers[0].proj_q.copy_(pq)
        pred.layers[0].proj_k.copy_(pk)
    student = veda_attention.SparseStudent(clip, plan, pred.to(DEV))
    fn = ulysses.UlyssesSparseStudent(student, transport='copy')
    try:
        for seed in (50, 51, 52):
            q, k, v = (t.to(DEV) for t in inputs.qkv(seq_len, heads, 128,
                                                     seed, torch.bfloat16))
            with torch.no_grad():
                want = student(q, k, v, 0)
                got = fn(q, k, v, 0)
            torch.cuda.synchronize()
            assert torch.equal(got, want), seed
    finally:
        fn.close()


def test_exchanged_layer_gradients_equal_plain_student(one_rank_group):
    """The stage-2 student through the exchange (autograd across the NCCL
    all-to-alls): output and dq, dk, dv equal the plain SparseStudent's bit
    for bit on one rank. The multi-rank exchange of gradients is tested over
    gloo on the CPU (tests/test_ulysses.py)."""
    text, grid, heads = 130, (4, 12, 20), 4
    used = text + grid[0] * grid[1] * grid[2]
    seq_len = used + 14
    layout = veda_attention.PackedLayout(
        seq_len, used, (veda_attention.VideoSpan(text, grid),))
    config = veda_attention.VedaConfig(
        target_budget=veda_mask.Budget(ratio=0.3))
    clip = veda_attention.ClipTiling(layout, config, DEV)
    plan = veda_plan.TilePlan('u', grid, [tiling.TileShape(2, 8, 8),
                                          tiling.TileShape(1, 8, 16)],
                              [[0, 1, 1, 0]])
    pred = veda_predictor.TileScorePredictor(1, heads, 128)
    pq, pk = inputs.predictor_weights(heads, 128, 46, 0.02)
    with torch.no_grad():
        pred.layers[0].proj_q.copy_(pq)
        pred.layers[0].proj_k.copy_(pk)
    student = veda_attention.SparseStudent(clip, plan, pred.to(DEV))
    q, k, v = (t.to(DEV) for t in inputs.qkv(seq_len, heads, 128, 47,
                                             torch.bfloat16))
    dout = inputs.dout(q.shape, 48).to(DEV)
    runs = []
    for fn in (student, ulysses.UlyssesSparseStudent(student)):
        leaves = [t.clone().requires_grad_(True) for t in (q, k, v)]
        out = fn(*leaves, 0)
        out.backward(dout)
        runs.append([out.detach()] + [t.grad for t in leaves])
    torch.cuda.synchronize()
    for name, a, b in zip(('out', 'dq', 'dk', 'dv'), *runs):
        assert torch.equal(a, b), name
    assert runs[0][1][:used].abs().max() > 0


@pytest.mark.parametrize('world,start,stop', [(2, 0, 24), (8, 0, 6),
                                              (4, 3, 9)])
def test_head_blocks_pack_and_unpack_are_exact(world, start, stop):
    rows, heads = 1000, 48
    per = heads // world
    gen = torch.Generator().manual_seed(world)
    x = torch.randn(rows, heads, 128, generator=gen).to(DEV, torch.bfloat16)
    packed = ulysses._pack(x, world, start, stop)  # pylint: disable=protected-access
    want = x.view(rows, world, per, 128)[:, :, start:stop].transpose(0, 1)
    assert torch.equal(packed, want)
    back = torch.zeros_like(x)
    ulysses._head_blocks(packed, back, world, start, stop, pack=False)  # pylint: disable=protected-access
    mask = torch.zeros(heads, dtype=torch.bool)
    for p in range(world):
        mask[p * per + start:p * per + stop] = True
    assert torch.equal(back[:, mask.to(DEV)], x[:, mask.to(DEV)])
    assert (back[:, ~mask.to(DEV)] == 0).all()
