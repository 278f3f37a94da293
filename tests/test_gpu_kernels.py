"""GPU parity: every kernel of the C ABI against the CPU oracle.

Bit-exact for index work (permutation, lists, selection) and for gathers,
max/min pooling; fp tolerances are the reference's own (pool mean 1e-5,
attention outputs 2e-2, lse 1e-3 absolute in natural-log units).
"""

import math

import numpy as np
import pytest
import torch

import inputs
import parity
from miowtion_b200 import _lib
from miowtion_b200 import kernels
from miowtion_b200 import mask as veda_mask
from miowtion_b200 import predictor as veda_predictor
from miowtion_b200 import tiling
from oracle import veda_oracle as vo

pytestmark = pytest.mark.gpu

DEV = 'cuda'


def spans_of(spec):
    return [tiling.TiledSpan(s, tuple(g), tiling.TileShape(*sh))
            for s, g, sh in spec['spans']]


def oracle_layout(spec):
    return vo.build_tile_layout(
        [vo.Span(s, tuple(g), tuple(sh)) for s, g, sh in spec['spans']],
        spec['used'], spec['seq_len'])


def qkv(seq_len, heads, seed):
    return [t.to(DEV) for t in inputs.qkv(seq_len, heads, 128, seed,
                                          torch.bfloat16)]


def np32(t):
    return t.detach().float().cpu().numpy()


@pytest.fixture(autouse=True)
def _status_clean():
    _lib.device_status(reset=True)
    yield
    assert _lib.device_status(reset=True) == 0, 'a kernel wait timed out'


# --- tcgen05 operand / accumulator layouts --------------------------------

@pytest.mark.parametrize('mode', [0, 1])
def test_umma_probe_matches_matmul(mode):
    gen = torch.Generator().manual_seed(3)
    a = torch.randn(128, 128, generator=gen).to(DEV, torch.bfloat16)
    b = torch.randn(128, 128, generator=gen).to(DEV, torch.bfloat16)
    d = torch.empty(128, 128, dtype=torch.float32, device=DEV)
    _lib.call('veda_probe_umma', a.data_ptr(), b.data_ptr(), d.data_ptr(),
              mode, _lib.stream_ptr())
    want = a.float() @ (b.float().T if mode == 0 else b.float())
    torch.testing.assert_close(d, want, rtol=1e-4, atol=1e-3)


# --- a1: layout -------------------------------------------------------------

LAYOUT_SPECS = {**inputs.SMALL_LAYOUTS, 'padded': inputs.PADDED,
                'segmented': inputs.SEGMENTED, **inputs.BENCH_LAYOUTS}


@pytest.mark.parametrize('name', sorted(LAYOUT_SPECS))
def test_layout_is_bit_exact(name):
    spec = LAYOUT_SPECS[name]
    lay = tiling.build_tile_layout(spans_of(spec), spec['used'],
                                   spec['seq_len'], DEV)
    ref = oracle_layout(spec)
    np.testing.assert_array_equal(lay.perm.cpu().numpy(), ref.perm)
    np.testing.assert_array_equal(lay.valid_count.cpu().numpy(),
                                  ref.valid_count)
    assert (lay.n_video_tiles, lay.n_ref_tiles, lay.n_global_tiles) == (
        ref.n_video_tiles, ref.n_ref_tiles, ref.n_global_tiles)
    np.testing.assert_array_equal(lay.partial_tiles.cpu().numpy(),
                                  ref.partial_tiles)
    np.testing.assert_array_equal(lay.pad_slots.cpu().numpy(), ref.pad_slots)


# --- a2/a3/a12/a14: gather, pool, scatter, lse ------------------------------

@pytest.fixture(scope='module')
def padded():
    spec = dict(inputs.PADDED, heads=4, group_heads=[0, 2, 3])
    lay = tiling.build_tile_layout(spans_of(spec), spec['used'],
                                   spec['seq_len'], DEV)
    ref = oracle_layout(spec)
    q, k, v = qkv(spec['seq_len'], spec['heads'], spec['seed'])
    heads = torch.tensor(spec['group_heads'], device=DEV)
    return spec, lay, ref, q, k, v, heads


@pytest.mark.parametrize('second', [False, True])
def test_gather_pool_matches_oracle(padded, second):
    spec, lay, ref, q, _, _, heads = padded
    res = tiling.gather_and_pool(q, lay, heads, second=second)
    tiles, feats = res[0], res[1]
    hn = heads.cpu().numpy()
    want_tiles = vo.gather_tiles(np32(q), ref, hn)
    np.testing.assert_array_equal(np32(tiles), want_tiles)
    want = vo.pool_tiles(want_tiles, ref)
    got = feats.cpu().numpy()
    np.testing.assert_array_equal(got[..., 128:], want[..., 128:])
    np.testing.assert_allclose(got[..., :128], want[..., :128], rtol=1e-5,
                               atol=1e-6)
    if second:
        np.testing.assert_allclose(res[2].cpu().numpy(),
                                   vo.pool_tiles(want_tiles, ref, 'raw'),
                                   rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(res[3].cpu().numpy(),
                                   vo.pool_tiles(want_tiles, ref, 'central'),
                                   rtol=1e-4, atol=1e-6)
    # Pooling already tile-ordered rows (predictor.pool_tiles) agrees.
    again = veda_predictor.pool_tiles(tiles, lay)
    torch.testing.assert_close(again, feats, rtol=1e-6, atol=1e-7)


def test_scatter_round_trip_and_lse_gather(padded):
    spec, lay, ref, q, _, _, heads = padded
    tiles = tiling.gather_tiles(q, lay, heads)
    out = torch.zeros(spec['seq_len'] + 1, spec['heads'], 128,
                      dtype=torch.bfloat16, device=DEV)
    tiling.scatter_tiles_(out, tiles, lay, heads)
    want = np.zeros((spec['seq_len'] + 1, spec['heads'], 128), np.float32)
    vo.scatter_tiles(want, vo.gather_tiles(np32(q), ref, heads.cpu().numpy()),
                     ref, heads.cpu().numpy())
    np.testing.assert_array_equal(np32(out)[:spec['seq_len']],
                                  want[:spec['seq_len']])
    lse = torch.randn(spec['seq_len'], spec['heads'], device=DEV)
    got = tiling.gather_lse(lse, lay, heads)
    np.testing.assert_array_equal(got.cpu().numpy(),
                                  vo.gather_lse(lse.cpu().numpy(), ref,
                                                heads.cpu().numpy()))


# --- a4: predictor ----------------------------------------------------------

def test_predictor_logits_match_oracle(padded):
    spec, lay, ref, q, k, _, heads = padded
    _, fq = tiling.gather_and_pool(q, lay, heads)
    _, fk = tiling.gather_and_pool(k, lay, heads)
    pq, pk = inputs.predictor_weights(spec['heads'], 128, 5, 0.02)
    logits = veda_predictor.predict_logits(fq, fk, pq.to(DEV), pk.to(DEV),
                                           heads)
    want = vo.predictor_logits(fq.cpu().numpy(), fk.cpu().numpy(),
                               pq.numpy(), pk.numpy(), heads.cpu().numpy())
    np.testing.assert_allclose(logits.cpu().numpy(), want, rtol=1e-4,
                               atol=1e-5)
    parity.assert_rel(logits, want, 1e-4, 'predictor logits')


# --- a5-a8: selection and lists --------------------------------------------

def _case(spec_name):
    if spec_name == 'segmented':
        spec = inputs.SEGMENTED
        budgets = (veda_mask.Budget(ratio=spec['target_ratio']),
                   veda_mask.Budget(ratio=spec['ref_ratio']))
        obudgets = (vo.Budget(ratio=spec['target_ratio']),
                    vo.Budget(ratio=spec['ref_ratio']))
    elif spec_name == 'padded':
        spec = inputs.PADDED
        budgets = (veda_mask.Budget(ratio=spec['ratio']), None)
        obudgets = (vo.Budget(ratio=spec['ratio']), None)
    else:
        spec = inputs.BENCH_LAYOUTS[spec_name]
        budgets = (veda_mask.Budget(ratio=0.1),
                   veda_mask.Budget(ratio=0.05))
        obudgets = (vo.Budget(ratio=0.1), vo.Budget(ratio=0.05))
    lay = tiling.build_tile_layout(spans_of(spec), spec['used'],
                                   spec['seq_len'], DEV)
    ref = oracle_layout(spec)
    return lay, ref, budgets, obudgets


@pytest.mark.parametrize('name', ['padded', 'segmented', 'cfg2', 'cfg3_a',
                                  'cfg4'])
def test_select_lists_bit_exact(name):
    lay, ref, budgets, obudgets = _case(name)
    heads = 2
    scores = inputs.scores(heads, lay.n_tiles, 17)
    blocks = veda_mask.column_blocks(lay, *budgets) if lay.n_ref_tiles else (
        veda_mask.column_blocks(lay, budgets[0]))
    oblocks = vo.column_blocks(ref, *obudgets) if ref.n_ref_tiles else (
        vo.column_blocks(ref, obudgets[0]))
    s_np = scores.numpy()[:, :lay.n_video_tiles]
    index, keep = vo.select_video_blocks(s_np, ref, oblocks)
    omask = vo.dense_block_mask(index, keep, ref)
    # Selection in the reference's rank order.
    sel = veda_mask.select_video_blocks(
        scores[:, :lay.n_video_tiles].to(DEV), lay, blocks)
    np.testing.assert_array_equal(sel.index.cpu().numpy(), index)
    np.testing.assert_array_equal(sel.keep.cpu().numpy(), keep)
    np.testing.assert_array_equal(
        veda_mask.dense_block_mask(sel, lay).cpu().numpy(), omask)
    # Fused scores -> mask + lists with tails, exactly the reference's.
    lists = veda_mask.select_block_lists(
        scores[:, :lay.n_video_tiles].to(DEV), lay, blocks, want_mask=True,
        fill_tails=True)
    np.testing.assert_array_equal(lists.mask.cpu().numpy().astype(bool),
                                  omask)
    for got, want in zip(lists.as_fa4(), vo.index_lists(omask, ref)):
        np.testing.assert_array_equal(got.cpu().numpy(), want)
    # Lists of an arbitrary mask, both directions.
    mask_t = torch.from_numpy(omask).to(DEV)
    for transpose in (False, True):
        got = kernels.index_lists(mask_t, lay, transpose=transpose)
        want = vo.index_lists(omask, ref, transpose=transpose)
        for g, w in zip(got, want):
            np.testing.assert_array_equal(g.cpu().numpy(), w)


def test_select_row_subset_follows_tile_ids():
    lay, ref, budgets, obudgets = _case('segmented')
    blocks = veda_mask.column_blocks(lay, *budgets)
    oblocks = vo.column_blocks(ref, *obudgets)
    scores = inputs.scores(3, lay.n_tiles, 23).numpy()
    rows = np.array(inputs.SEGMENTED['subset_rows'])
    index, keep = vo.select_video_blocks(scores[:, rows], ref, oblocks, rows)
    sel = veda_mask.select_video_blocks(
        torch.from_numpy(scores[:, rows]).to(DEV), lay, blocks,
        torch.from_numpy(rows).to(DEV))
    np.testing.assert_array_equal(sel.index.cpu().numpy(), index)
    np.testing.assert_array_equal(sel.keep.cpu().numpy(), keep)


def test_select_ties_rank_the_lower_column_first():
    lay, ref, budgets, obudgets = _case('padded')
    blocks = veda_mask.column_blocks(lay, budgets[0])
    oblocks = vo.column_blocks(ref, obudgets[0])
    gen = torch.Generator().manual_seed(0)
    scores = torch.randint(0, 4, (2, lay.n_video_tiles, lay.n_tiles),
                           generator=gen).float()
    index, keep = vo.select_video_blocks(scores.numpy(), ref, oblocks)
    sel = veda_mask.select_video_blocks(scores.to(DEV), lay, blocks)
    np.testing.assert_array_equal(sel.index.cpu().numpy(), index)
    np.testing.assert_array_equal(sel.keep.cpu().numpy(), keep)


# --- a9/a11: attention forward ---------------------------------------------

def _random_mask(heads, lay, density, seed):
    gen = torch.Generator().manual_seed(seed)
    n = lay.n_tiles
    m = torch.rand(heads, n, n, generator=gen) < density
    m[:, torch.arange(n), torch.arange(n)] = True
    return m


@pytest.mark.parametrize('density', [0.3, 1.0])
def test_block_sparse_forward_matches_oracle(padded, density):
    spec, lay, ref, q, k, v, heads = padded
    qt, kt, vt = (tiling.gather_tiles(t, lay, heads) for t in (q, k, v))
    mask = _random_mask(heads.numel(), lay, density, 31)
    mask[:, 5, :] = False  # a query tile with no key at all
    out, lse = kernels.block_sparse_attention(qt, kt, vt, mask.to(DEV), lay,
                                              return_lse=True)
    want, want_lse = vo.block_sparse_attention(
        np32(qt), np32(kt), np32(vt), mask.numpy(), ref.valid_count,
        return_lse=True)
    real = ref.slot_valid.astype(bool)
    np.testing.assert_allclose(np32(out)[real], want[real], rtol=2e-2,
                               atol=2e-2)
    parity.assert_rel(np32(out), want, parity.FWD,
                      f'sparse forward, padded layout, density {density}',
                      where=real)
    got_lse = lse.cpu().numpy()
    assert np.isneginf(got_lse[:, 5 * 128:6 * 128]).all()
    assert (np32(out)[5 * 128:6 * 128] == 0).all()
    fin = np.isfinite(want_lse)
    np.testing.assert_allclose(got_lse[:, real][fin[:, real]],
                               want_lse[:, real][fin[:, real]], rtol=0,
                               atol=2e-3)


def test_sparse_is_closer_to_sparse_than_dense(padded):
    """Guards against a kernel that silently ignores the block pattern."""
    spec, lay, ref, q, k, v, heads = padded
    qt, kt, vt = (tiling.gather_tiles(t, lay, heads) for t in (q, k, v))
    mask = _random_mask(heads.numel(), lay, 0.2, 7)
    out = np32(kernels.block_sparse_attention(qt, kt, vt, mask.to(DEV), lay))
    sparse = vo.block_sparse_attention(np32(qt), np32(kt), np32(vt),
                                       mask.numpy(), ref.valid_count)
    dense = vo.block_sparse_attention(np32(qt), np32(kt), np32(vt),
                                      np.ones_like(mask.numpy()),
                                      ref.valid_count)
    real = ref.slot_valid.astype(bool)
    assert np.abs(out - sparse)[real].max() < np.abs(out - dense)[real].max()


def test_dense_attention_matches_oracle():
    q, k, v = qkv(1300, 3, 41)
    used = 1100
    out, lse = kernels.dense_attention(q, k, v, 128 ** -0.5, True, used=used)
    want, want_lse = vo.dense_attention(np32(q), np32(k), np32(v), used,
                                        return_lse=True)
    np.testing.assert_allclose(np32(out), want, rtol=2e-2, atol=2e-2)
    parity.assert_rel(np32(out), want, parity.FWD, 'dense forward')
    np.testing.assert_allclose(lse.cpu().numpy(), want_lse, rtol=0,
                               atol=2e-3)
    assert (np32(out)[used:] == 0).all() and (lse[used:] == 0).all()


def test_large_uniform_lists_forward():
    """Many query tiles with long lists (the bench pattern, one head)."""
    spec = inputs.BENCH_LAYOUTS['cfg2']
    lay = tiling.build_tile_layout(spans_of(spec), spec['used'],
                                   spec['seq_len'], DEV)
    ref = oracle_layout(spec)
    q, k, v = qkv(spec['seq_len'], 1, 1)
    heads = torch.tensor([0], device=DEV)
    qt, kt, vt = (tiling.gather_tiles(t, lay, heads) for t in (q, k, v))
    scores = inputs.scores(1, lay.n_tiles, 3).to(DEV)
    blocks = veda_mask.column_blocks(lay, veda_mask.Budget(ratio=0.1))
    lists = veda_mask.select_block_lists(scores, lay, blocks, want_mask=True)
    assert int(lists.full_cnt.min()) == 28 and int(lists.full_cnt.max()) == 28
    out = kernels.block_sparse_attention_lists(qt, kt, vt, lists, lay)
    rows = np.array([0, 1, 137, 279])
    sub = (rows[:, None] * 128 + np.arange(128)[None]).reshape(-1)
    mask = lists.mask.cpu().numpy().astype(bool)
    want = vo.block_sparse_attention(np32(qt)[sub], np32(kt), np32(vt),
                                     mask[:, rows], ref.valid_count)
    np.testing.assert_allclose(np32(out)[sub], want, rtol=2e-2, atol=2e-2)
    parity.assert_rel(np32(out)[sub], want, parity.FWD,
                      'sparse forward, cfg2 lists, sampled query tiles')


def test_lse_is_natural_log():
    q, k, v = qkv(256, 1, 2)
    _, lse = kernels.dense_attention(q, k, v, 128 ** -0.5, True)
    s = (q.float()[:, 0] @ k.float()[:, 0].T) / math.sqrt(128)
    torch.testing.assert_close(lse[:, 0], torch.logsumexp(s, -1), rtol=0,
                               atol=2e-3)


# --- the forward's two softmax organisations ---------------------------------

@pytest.fixture
def fwd_groups():
    """Sets the forward's softmax groups for one test; restores the
    default."""
    def set_groups(g):
        kernels.set_fwd_groups(g)
    yield set_groups
    kernels.set_fwd_groups(kernels.DEFAULT_FWD_GROUPS)


@pytest.mark.parametrize('density', [0.3, 1.0])
def test_softmax_groups_agree_and_match_oracle(padded, fwd_groups, density):
    """Two groups on alternate key blocks (own accumulators, merged at the
    end) and one group on every block compute the same attention and LSE;
    both match the oracle."""
    spec, lay, ref, q, k, v, heads = padded
    qt, kt, vt = (tiling.gather_tiles(t, lay, heads) for t in (q, k, v))
    mask = _random_mask(heads.numel(), lay, density, 33)
    mask[:, 4, 1:] = False  # a query tile with a single key tile
    mask[:, 6, :] = False   # and one with none
    outs = {}
    for g in (1, 2):
        fwd_groups(g)
        outs[g] = kernels.block_sparse_attention(qt, kt, vt, mask.to(DEV),
                                                 lay, return_lse=True)
    want, want_lse = vo.block_sparse_attention(
        np32(qt), np32(kt), np32(vt), mask.numpy(), ref.valid_count,
        return_lse=True)
    real = ref.slot_valid.astype(bool)
    for g, (out, lse) in outs.items():
        parity.assert_rel(np32(out), want, parity.FWD,
                          f'sparse forward, {g} softmax group(s), density '
                          f'{density}', where=real)
        got_lse = lse.cpu().numpy()
        fin = np.isfinite(want_lse)
        np.testing.assert_allclose(got_lse[:, real][fin[:, real]],
                                   want_lse[:, real][fin[:, real]], rtol=0,
                                   atol=2e-3)
        assert np.isneginf(got_lse[:, 6 * 128:7 * 128]).all()
        assert (np32(out)[6 * 128:7 * 128] == 0).all()
    parity.assert_rel(np32(outs[2][0]), np32(outs[1][0]), 1e-2,
                      'two softmax groups against one', where=real)


def test_softmax_reference_jumps(padded, fwd_groups):
    """Scores that grow from block to block by more than the lazy-rescale
    threshold: the two-group softmax recomputes P against the new reference
    and rescales its accumulator, as the one-group softmax does."""
    spec, lay, ref, q, k, v, heads = padded
    qt, kt, vt = (tiling.gather_tiles(t, lay, heads) for t in (q, k, v))
    # Key tile j scaled by (1 + (n - 1 - j) / 2): the lists are walked from
    # their ends, so later blocks reach far above the first block's
    # maximum.
    n = lay.n_tiles
    scale = (1.0 + torch.arange(n - 1, -1, -1, dtype=torch.float32)
             .repeat_interleave(128) / 2.0).to(DEV)
    kt = (kt.float() * scale[:, None, None]).to(torch.bfloat16)
    mask = _random_mask(heads.numel(), lay, 0.6, 35)
    want = vo.block_sparse_attention(np32(qt), np32(kt), np32(vt),
                                     mask.numpy(), ref.valid_count)
    real = ref.slot_valid.astype(bool)
    for g in (1, 2):
        fwd_groups(g)
        out = kernels.block_sparse_attention(qt, kt, vt, mask.to(DEV), lay)
        parity.assert_rel(np32(out), want, parity.FWD,
                          f'sparse forward with growing scores, {g} '
                          'softmax group(s)', where=real)


def test_dense_two_groups_match_oracle(fwd_groups):
    q, k, v = qkv(1500, 2, 42)
    used = 1300
    want, want_lse = vo.dense_attention(np32(q), np32(k), np32(v), used,
                                        return_lse=True)
    for g in (1, 2):
        fwd_groups(g)
        out, lse = kernels.dense_attention(q, k, v, 128 ** -0.5, True,
                                           used=used)
        parity.assert_rel(np32(out), want, parity.FWD,
                          f'dense forward, {g} softmax group(s)')
        np.testing.assert_allclose(lse.cpu().numpy(), want_lse, rtol=0,
                                   atol=2e-3)
        assert (np32(out)[used:] == 0).all()
