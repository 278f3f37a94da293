"""GPU parity of the tile-search oracle error ((f) row 2): the device path
(`search.oracle_rel_mse`: heat-based selection, row-subset forward,
`veda_rel_mse`) against the CPU oracle's restatement of the reference's
kernel path, and against the reference's own fp32 numbers (fixture)."""

import os

import numpy as np
import pytest
import torch

import inputs
from miowtion_b200 import _lib
from miowtion_b200 import attention as veda_attention
from miowtion_b200 import kernels
from miowtion_b200 import mask as veda_mask
from miowtion_b200 import search
from miowtion_b200 import tiling
from oracle import veda_oracle as vo

pytestmark = pytest.mark.gpu

DEV = 'cuda'
GOLDEN = os.path.join(os.path.dirname(__file__), 'golden')


@pytest.fixture(autouse=True)
def _status_clean():
    _lib.device_status(reset=True)
    yield
    assert _lib.device_status(reset=True) == 0, 'a kernel wait timed out'


@pytest.fixture(scope='module')
def case():
    spec = inputs.SEARCH
    q, k, v = inputs.qkv(spec['seq_len'], spec['heads'], spec['dim'],
                         spec['seed'], torch.bfloat16)
    packed = veda_attention.PackedLayout(
        spec['seq_len'], spec['used'],
        (veda_attention.VideoSpan(spec['text'], spec['grid']),))
    return spec, packed, q, k, v


def test_rel_mse_kernel_matches_torch():
    gen = torch.Generator().manual_seed(3)
    n_rows, heads, seq = 6, 5, 1000
    o_sparse = torch.randn(n_rows * 128, heads, 128, generator=gen).to(
        torch.bfloat16).to(DEV)
    o_dense = torch.randn(seq, heads + 2, 128, generator=gen).to(
        torch.bfloat16).to(DEV)
    seq_row = torch.randint(0, seq, (n_rows * 128,), generator=gen)
    seq_row[torch.rand(n_rows * 128, generator=gen) < 0.2] = -1
    seq_row[128:256] = -1  # a tile with no real row
    hd = torch.tensor([6, 0, 2, 3, 5])
    got = search.rel_mse(o_sparse, o_dense, seq_row.to(DEV), hd.to(DEV))
    real = seq_row >= 0
    a = o_sparse.float().cpu()[real]
    b = o_dense.float().cpu()[seq_row[real]][:, hd]
    want = (a - b).square().sum((0, 2)) / b.square().sum((0, 2))
    torch.testing.assert_close(got.cpu(), want, rtol=1e-5, atol=0)
    again = search.rel_mse(o_sparse, o_dense, seq_row.to(DEV), hd.to(DEV))
    assert torch.equal(got, again), 'rel_mse must be deterministic'
    # No real row at all: 0 / tiny = 0.
    none = search.rel_mse(o_sparse[:128], o_dense,
                          torch.full((128,), -1, device=DEV), hd.to(DEV))
    assert torch.equal(none.cpu(), torch.zeros(heads))


def test_gather_tile_rows_is_a_slice_of_the_tile_order(case):
    spec, packed, q, _, _ = case
    clip = veda_attention.ClipTiling(packed, veda_attention.VedaConfig(), DEV)
    lay = clip.get(tiling.TileShape(*spec['candidates'][0]))
    rows = torch.tensor([0, 3, 4, lay.n_video_tiles - 1], device=DEV)
    heads = torch.tensor([2, 0], device=DEV)
    full = tiling.gather_tiles(q.to(DEV), lay, heads)
    sub = tiling.gather_tile_rows(q.to(DEV), lay, rows, heads)
    slots = (rows[:, None] * 128 + torch.arange(128, device=DEV)).reshape(-1)
    assert torch.equal(sub, full.index_select(0, slots))


@pytest.mark.parametrize('ci', range(len(inputs.SEARCH['candidates'])))
def test_oracle_rel_mse_matches_oracle_and_reference(case, ci):
    spec, packed, q, k, v = case
    config = veda_attention.VedaConfig(
        target_budget=veda_mask.Budget(ratio=spec['ratio']))
    clip = veda_attention.ClipTiling(packed, config, DEV)
    shape = tiling.TileShape(*spec['candidates'][ci])
    lay = clip.get(shape)
    rows = inputs.search_rows(lay.n_video_tiles, spec['query_tiles'],
                              spec['sample_seed'])
    qd, kd, vd = (t.to(DEV) for t in (q, k, v))
    out, lse = kernels.dense_attention(qd, kd, vd, 128**-0.5,
                                       return_lse=True, used=spec['used'])
    got = search.oracle_rel_mse(qd, kd, vd, lay, clip.blocks(lay),
                                rows.to(DEV), dense_out=out, lse=lse).cpu()
    # The same with the dense teacher computed inside.
    got2 = search.oracle_rel_mse(qd, kd, vd, lay, clip.blocks(lay),
                                 rows.to(DEV)).cpu()
    torch.testing.assert_close(got, got2, rtol=0, atol=0)
    ref = vo.build_tile_layout([vo.Span(spec['text'], spec['grid'],
                                        spec['candidates'][ci])],
                               spec['used'], spec['seq_len'])
    blocks = vo.column_blocks(ref, vo.Budget(ratio=spec['ratio']))
    qf, kf, vf = (t.float().numpy() for t in (q, k, v))
    o_np, lse_np = vo.dense_attention(qf, kf, vf, spec['used'],
                                      return_lse=True)
    want = vo.oracle_rel_mse(qf, kf, vf, ref, blocks, rows.numpy(), o_np,
                             lse_np)
    np.testing.assert_allclose(got.numpy(), want, rtol=2e-2)
    golden = np.load(os.path.join(GOLDEN, 'search.npz'))[f'c{ci}_rel_mse']
    np.testing.assert_allclose(got.numpy(), golden, rtol=2e-2)


def test_oracle_scorer_returns_dense_and_scores_every_candidate(case):
    spec, packed, q, k, v = case
    cands = [tiling.TileShape(*c) for c in spec['candidates']]
    config = veda_attention.VedaConfig(
        target_budget=veda_mask.Budget(ratio=spec['ratio']))
    scorer = search.OracleScorer(packed, cands, config,
                                 spec['query_tiles'], spec['sample_seed'],
                                 torch.device(DEV))
    qd, kd, vd = (t.to(DEV) for t in (q, k, v))
    out = scorer(qd, kd, vd, 0)
    dense, _ = kernels.dense_attention(qd, kd, vd, 128**-0.5, False,
                                       used=spec['used'])
    assert torch.equal(out, dense)
    table = scorer.scores[0]
    assert table.shape == (len(cands), spec['heads'])
    golden = np.load(os.path.join(GOLDEN, 'search.npz'))
    for ci in range(len(cands)):
        np.testing.assert_allclose(table[ci].numpy(),
                                   golden[f'c{ci}_rel_mse'], rtol=2e-2)
