"""The packed attention path: q, k, v read in place as TMA boxes of the
packed [S, H, D] tensors and the output written straight to its rows.

Checks the box layout against the span geometry (exactly), the packed
forward against the tile-ordered path (gather, forward, scatter) and the
oracle, and that nothing outside the group's rows [0, used) is written."""

import numpy as np
import pytest
import torch

import inputs
import parity
from miowtion_b200 import _lib
from miowtion_b200 import kernels
from miowtion_b200 import tiling
from oracle import veda_oracle as vo

pytestmark = pytest.mark.gpu

DEV = 'cuda'

LAYOUT_SPECS = {**inputs.SMALL_LAYOUTS, 'padded': inputs.PADDED,
                'segmented': inputs.SEGMENTED, **inputs.BENCH_LAYOUTS}


def spans_of(spec):
    return [tiling.TiledSpan(s, tuple(g), tiling.TileShape(*sh))
            for s, g, sh in spec['spans']]


def oracle_layout(spec):
    return vo.build_tile_layout(
        [vo.Span(s, tuple(g), tuple(sh)) for s, g, sh in spec['spans']],
        spec['used'], spec['seq_len'])


def np32(t):
    return t.detach().float().cpu().numpy()


@pytest.fixture(autouse=True)
def _status_clean():
    _lib.device_status(reset=True)
    yield
    assert _lib.device_status(reset=True) == 0, 'a kernel wait timed out'


def box_perm_of(spec, ref):
    """Box order of every video tile from the span geometry (numpy)."""
    out = ref.perm.copy()
    tile = 0
    for start, (T, H, W), (st, sh, sw) in spec['spans']:
        nbt, nbh, nbw = -(-T // st), -(-H // sh), -(-W // sw)
        pos = np.arange(128)
        dt, dh, dw = pos // (sh * sw), (pos // sw) % sh, pos % sw
        for lt in range(nbt * nbh * nbw):
            bt, bw, bh = lt % nbt, (lt // nbt) % nbw, lt // (nbt * nbw)
            t, h, w = bt * st + dt, bh * sh + dh, bw * sw + dw
            ok = (t < T) & (h < H) & (w < W)
            out[tile * 128:(tile + 1) * 128] = np.where(
                ok, start + (t * H + h) * W + w, -1)
            tile += 1
    assert tile == ref.n_video_tiles
    return out


@pytest.mark.parametrize('name', sorted(LAYOUT_SPECS))
def test_box_layout_matches_the_span_geometry(name):
    spec = LAYOUT_SPECS[name]
    lay = tiling.build_tile_layout(spans_of(spec), spec['used'],
                                   spec['seq_len'], DEV)
    ref = oracle_layout(spec)
    box = lay.box_perm.cpu().numpy()
    np.testing.assert_array_equal(box, box_perm_of(spec, ref))
    # Every tile holds the same rows as the reference's tile, reordered.
    per_tile = lambda a: np.sort(a.reshape(-1, 128), axis=1)  # noqa: E731
    np.testing.assert_array_equal(per_tile(box), per_tile(ref.perm))
    bits = (lay.key_mask.cpu().numpy().astype(np.int64) & 0xffffffff)
    want = ((box >= 0).reshape(-1, 32) << np.arange(32)).sum(axis=1)
    np.testing.assert_array_equal(bits, want)


def tile_image(tiles):
    """Shared-memory image of tile-ordered rows [N, H', 128] (torch): per
    head and tile two 64-column halves of 128 rows, chunk c of row r at
    position c ^ (r % 8)."""
    n, heads = tiles.shape[0] // 128, tiles.shape[1]
    x = tiles.view(n, 128, heads, 2, 8, 8).permute(2, 0, 3, 1, 4, 5)
    r = torch.arange(128, device=tiles.device).view(128, 1)
    c = torch.arange(8, device=tiles.device).view(1, 8)
    idx = (c ^ (r & 7)).view(1, 1, 1, 128, 8, 1).expand(heads, n, 2, 128, 8,
                                                          8)
    return torch.gather(x.contiguous(), 4, idx).reshape(heads, n, 2, 128, 64)


@pytest.mark.parametrize('name', ['padded', 'l_cond', 'cfg3_b'])
def test_gather_images_are_swizzled_tiles(name):
    spec = LAYOUT_SPECS[name]
    lay = tiling.build_tile_layout(spans_of(spec), spec['used'],
                                   spec['seq_len'], DEV)
    x = inputs.qkv(spec['seq_len'], 3, 128, 71, torch.bfloat16)[0].to(DEV)
    hd = torch.tensor([2, 0], device=DEV)
    tiles, feats = tiling.gather_and_pool(x, lay, hd)
    image, feats_i = tiling.gather_images(x, lay, hd, pool=True)
    assert torch.equal(image, tile_image(tiles))
    assert torch.equal(feats_i, feats)
    assert torch.equal(tiling.pool_features(x, lay, hd), feats)


def _lists(mask, lay):
    return kernels.index_lists_from_mask(mask.to(DEV), lay, transpose=False)


@pytest.mark.parametrize('kv_tiles', [True, 'images', False])
@pytest.mark.parametrize('name,heads', [('padded', [2, 0]),
                                        ('l_cond', [1]),
                                        ('l_ragged', [0, 1, 2]),
                                        ('segmented', [0, 2])])
def test_packed_forward_matches_tile_path_and_oracle(name, heads, kv_tiles):
    spec = LAYOUT_SPECS[name]
    total = 3
    lay = tiling.build_tile_layout(spans_of(spec), spec['used'],
                                   spec['seq_len'], DEV)
    ref = oracle_layout(spec)
    q, k, v = (t.to(DEV) for t in inputs.qkv(spec['seq_len'], total, 128,
                                             61, torch.bfloat16))
    hd = torch.tensor(heads, device=DEV)
    gen = torch.Generator().manual_seed(13)
    n = lay.n_tiles
    mask = torch.rand(len(heads), n, n, generator=gen) < 0.35
    mask[:, torch.arange(n), torch.arange(n)] = True
    if n > 3:
        mask[:, 3, :] = False  # a query tile with no key at all
    lists = _lists(mask, lay)
    # Tile-ordered path.
    qt, kt, vt = (tiling.gather_tiles(t, lay, hd) for t in (q, k, v))
    o_tiles = kernels.block_sparse_attention_lists(qt, kt, vt, lists, lay)
    want_tp = torch.zeros_like(q)
    tiling.scatter_rows_(want_tp, o_tiles, lay, hd)
    # Packed path, into a buffer of sentinels.
    out = torch.full_like(q, 7.0)
    if kv_tiles == 'images':
        kernels.block_sparse_attention_packed(
            q, tiling.gather_images(k, lay, hd), tiling.gather_images(v, lay, hd),
            lists, lay, hd, out, kv_tiles='images')
    elif kv_tiles:
        kernels.block_sparse_attention_packed(q, kt, vt, lists, lay, hd, out,
                                              kv_tiles=True)
    else:
        kernels.block_sparse_attention_packed(q, k, v, lists, lay, hd, out)
    torch.cuda.synchronize()
    used = spec['used']
    got = np32(out)
    other = [h for h in range(total) if h not in heads]
    assert (got[:, other] == 7.0).all(), 'wrote heads outside the group'
    assert (got[used:] == 7.0).all(), 'wrote rows >= used'
    sel = got[:used][:, heads]
    np.testing.assert_allclose(sel, np32(want_tp)[:used][:, heads],
                               rtol=1e-2, atol=1e-2)
    # The oracle over the tile order, scattered back.
    want = vo.block_sparse_attention(np32(qt), np32(kt), np32(vt),
                                     mask.numpy(), ref.valid_count)
    seq = np.zeros((spec['seq_len'] + 1, len(heads), 128), np.float32)
    vo.scatter_tiles(seq, want, ref, np.arange(len(heads)))
    np.testing.assert_allclose(sel, seq[:used], rtol=2e-2, atol=2e-2)
    parity.assert_rel(sel, seq[:used], parity.FWD,
                      f'packed forward ({kv_tiles or "boxes"}), {name}, '
                      f'heads {heads}')
    # The empty query tile's rows are zero.
    if n > 3:
        rows = ref.perm[3 * 128:4 * 128]
        rows = rows[rows >= 0]
        assert (got[rows][:, heads] == 0).all()


def test_packed_forward_full_size_rows_cfg3():
    """cfg3 group a at full size (two shapes of heads are separate layouts):
    sampled query tiles of the packed output against the oracle."""
    spec = inputs.BENCH_LAYOUTS['cfg3_a']
    lay = tiling.build_tile_layout(spans_of(spec), spec['used'],
                                   spec['seq_len'], DEV)
    ref = oracle_layout(spec)
    total = 2
    q, k, v = (t.to(DEV) for t in inputs.qkv(spec['seq_len'], total, 128,
                                             62, torch.bfloat16))
    hd = torch.tensor([1], device=DEV)
    n = lay.n_tiles
    gen = torch.Generator().manual_seed(14)
    mask = torch.rand(1, n, n, generator=gen) < 0.09
    mask[:, torch.arange(n), torch.arange(n)] = True
    mask[:, :, lay.n_video_tiles:] = True   # global columns
    mask[:, lay.n_video_tiles:, :] = True   # global rows
    lists = _lists(mask, lay)
    qt, kt, vt = (tiling.gather_tiles(t, lay, hd) for t in (q, k, v))
    out = torch.zeros_like(q)
    kernels.block_sparse_attention_packed(
        q, tiling.gather_images(k, lay, hd), tiling.gather_images(v, lay, hd),
        lists, lay, hd, out, kv_tiles='images')
    sample = np.array(ref.partial_tiles[:3].tolist() + [0, 411, n - 1])
    q_rows = (sample[:, None] * 128 + np.arange(128)).reshape(-1)
    want = vo.block_sparse_attention(
        np32(qt)[q_rows], np32(kt), np32(vt), mask.numpy()[:, sample],
        ref.valid_count)
    rows = ref.perm[q_rows]
    real = rows >= 0
    got = np32(out)[rows[real], 1]
    np.testing.assert_allclose(got, want[real][:, 0], rtol=2e-2, atol=2e-2)
    parity.assert_rel(got, want[real][:, 0], parity.FWD,
                      'packed forward, cfg3 group a full size, sampled tiles')


def test_packed_forward_full_size_rows_cfg4():
    """cfg4 (Ref2VA) at full size: the reference segment at 95% and the
    target at 90% sparsity, lists from the selection kernel with both
    segments' budgets; sampled query tiles of both segments (partial tiles
    included) of the packed output against the oracle."""
    from miowtion_b200 import mask as veda_mask
    spec = inputs.BENCH_LAYOUTS['cfg4']
    lay = tiling.build_tile_layout(spans_of(spec), spec['used'],
                                   spec['seq_len'], DEV)
    ref = oracle_layout(spec)
    total = 2
    q, k, v = (t.to(DEV) for t in inputs.qkv(spec['seq_len'], total, 128,
                                             65, torch.bfloat16))
    hd = torch.tensor([0], device=DEV)
    ref_ratio, target_ratio = spec['budgets'][0]
    blocks = veda_mask.column_blocks(lay, veda_mask.Budget(ratio=target_ratio),
                                     veda_mask.Budget(ratio=ref_ratio))
    scores = inputs.scores(1, lay.n_tiles, 17)[:, :lay.n_video_tiles]
    lists = veda_mask.select_block_lists(scores.to(DEV), lay, blocks,
                                         want_mask=True)
    n_ref = 120  # (4,45,80) in (2,8,8) tiles: 2 x 6 x 10
    # Every row keeps k_lo or k_lo + 1 key tiles of each column block:
    # 5.32 per row of the reference segment's columns (95%), 68.70 of the
    # target's (90%).
    kept = lists.mask[0].cpu()
    assert set(kept[:, :n_ref].sum(-1).tolist()) == {5, 6}
    assert set(kept[:, n_ref:].sum(-1).tolist()) == {68, 69}
    out = torch.zeros_like(q)
    kernels.block_sparse_attention_packed(
        q, tiling.gather_images(k, lay, hd), tiling.gather_images(v, lay, hd),
        lists, lay, hd, out, kv_tiles='images')
    partial = [t for t in ref.partial_tiles.tolist()]
    sample = np.array(sorted({0, 57, n_ref - 1, n_ref, 500, lay.n_tiles - 1,
                              *[t for t in partial if t < n_ref][:2],
                              *[t for t in partial if t >= n_ref][:2]}))
    q_rows = (sample[:, None] * 128 + np.arange(128)).reshape(-1)
    qt, kt, vt = (tiling.gather_tiles(t, lay, hd) for t in (q, k, v))
    mask = lists.mask.cpu().numpy().astype(bool)
    want = vo.block_sparse_attention(np32(qt)[q_rows], np32(kt), np32(vt),
                                     mask[:, sample], ref.valid_count)
    rows = ref.perm[q_rows]
    real = rows >= 0
    got = np32(out)[rows[real], 0]
    np.testing.assert_allclose(got, want[real][:, 0], rtol=2e-2, atol=2e-2)
    parity.assert_rel(got, want[real][:, 0], parity.FWD,
                      'packed forward, cfg4 full size, both segments')
    in_ref = np.repeat(sample < n_ref, 128)[real]
    parity.assert_rel(got[in_ref], want[real][in_ref, 0], parity.FWD,
                      'packed forward, cfg4 reference-segment query tiles')


def test_sm_reserve_changes_the_grid_not_the_result():
    spec = LAYOUT_SPECS['padded']
    lay = tiling.build_tile_layout(spans_of(spec), spec['used'],
                                   spec['seq_len'], DEV)
    q, k, v = (t.to(DEV) for t in inputs.qkv(spec['seq_len'], 3, 128, 63,
                                             torch.bfloat16))
    hd = torch.tensor([0, 1, 2], device=DEV)
    n = lay.n_tiles
    gen = torch.Generator().manual_seed(15)
    mask = torch.rand(3, n, n, generator=gen) < 0.3
    mask[:, torch.arange(n), torch.arange(n)] = True
    lists = _lists(mask, lay)
    ki, vi = (tiling.gather_images(t, lay, hd) for t in (k, v))
    outs = []
    for reserve in (0, 120, 0):
        _lib.call('veda_set_sm_reserve', reserve)
        out = torch.zeros_like(q)
        kernels.block_sparse_attention_packed(q, ki, vi, lists, lay, hd, out,
                                              kv_tiles='images')
        outs.append(out)
    _lib.call('veda_set_sm_reserve', 0)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])


def test_work_order_covers_every_item_and_keeps_the_bits():
    """The balanced work order (global query rows dealt first, then video
    rows to the least-loaded CTA) holds every (head, query tile) once, and
    the forward's output does not depend on it."""
    from miowtion_b200 import mask as veda_mask
    spec = inputs.BENCH_LAYOUTS['cfg3_a']
    lay = tiling.build_tile_layout(spans_of(spec), spec['used'],
                                   spec['seq_len'], DEV)
    heads = 2
    blocks = veda_mask.column_blocks(lay, veda_mask.Budget(ratio=0.1))
    order = kernels.work_order(lay, heads, blocks, torch.device(DEV))
    assert order is not None and order.dtype == torch.int32
    items = order[order >= 0].cpu().numpy()
    assert sorted(items.tolist()) == list(range(heads * lay.n_tiles))
    # Every CTA starts with at most one global query row's worth of work
    # more than the others: the global rows go to different CTAs first.
    first = order[0].cpu().numpy()
    assert ((first % lay.n_tiles) >= lay.n_video_tiles).sum() == min(
        order.shape[1], heads * lay.n_global_tiles)
    assert kernels.work_order(lay, heads, blocks, torch.device(DEV)) is order
    q, k, v = (t.to(DEV) for t in inputs.qkv(spec['seq_len'], heads, 128,
                                             64, torch.bfloat16))
    hd = torch.arange(heads, device=DEV)
    n = lay.n_tiles
    gen = torch.Generator().manual_seed(16)
    mask = torch.rand(heads, n, n, generator=gen) < 0.08
    mask[:, torch.arange(n), torch.arange(n)] = True
    mask[:, lay.n_video_tiles:, :] = True
    lists = _lists(mask, lay)
    ki, vi = (tiling.gather_images(t, lay, hd) for t in (k, v))
    outs = []
    for o in (None, order):
        out = torch.zeros_like(q)
        kernels.block_sparse_attention_packed(q, ki, vi, lists, lay, hd, out,
                                              kv_tiles='images', order=o)
        outs.append(out)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])
