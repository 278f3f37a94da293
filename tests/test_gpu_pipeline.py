"""HostPipeline: host-resident q, k, v through a SparseStudent with the
copies overlapped gives exactly the outputs of direct device calls."""

import pytest
import torch

import inputs
from miowtion_b200 import attention as veda_attention
from miowtion_b200 import mask as veda_mask
from miowtion_b200 import plan as veda_plan
from miowtion_b200 import predictor as veda_predictor
from miowtion_b200 import tiling
from miowtion_b200.pipeline import HostPipeline

pytestmark = pytest.mark.gpu

DEV = torch.device('cuda')


@pytest.mark.parametrize('depth', [1, 2])
def test_host_pipeline_matches_device_calls(depth):
    text, grid, heads = 130, (4, 16, 24), 3
    used = text + grid[0] * grid[1] * grid[2]
    seq_len = used + 7
    layout = veda_attention.PackedLayout(
        seq_len, used, (veda_attention.VideoSpan(text, grid),))
    config = veda_attention.VedaConfig(
        target_budget=veda_mask.Budget(ratio=0.3))
    clip = veda_attention.ClipTiling(layout, config, DEV)
    plan = veda_plan.TilePlan('pipe', grid, [tiling.TileShape(2, 8, 8)],
                              [[0, 0, 0]])
    pred = veda_predictor.TileScorePredictor(1, heads, 128)
    pq, pk = inputs.predictor_weights(heads, 128, 5, 0.02)
    with torch.no_grad():
        pred.layers[0].proj_q.copy_(pq)
        pred.layers[0].proj_k.copy_(pk)
    student = veda_attention.SparseStudent(clip, plan, pred.to(DEV))
    calls = [inputs.qkv(seq_len, heads, 128, 100 + i, torch.bfloat16)
             for i in range(4)]
    with torch.no_grad():
        want = [student(*(t.to(DEV) for t in c), 0).cpu() for c in calls]
        pipe = HostPipeline(student, (seq_len, heads, 128), torch.bfloat16,
                            DEV, depth=depth)
        outs = [torch.empty(seq_len, heads, 128,
                            dtype=torch.bfloat16).pin_memory()
                for _ in calls]
        for c, o in zip(calls, outs):
            pipe(*(t.pin_memory() for t in c), 0, o)
        pipe.synchronize()
    for got, w in zip(outs, want):
        assert torch.equal(got, w)


def test_host_pipeline_rejects_device_tensors():
    pipe = HostPipeline(lambda q, k, v, i: q, (4, 1, 128), torch.bfloat16,
                        DEV)
    x = torch.zeros(4, 1, 128, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(ValueError, match='pinned host'):
        pipe(x, x, x, 0, x)
