"""GPU parity of the block-sparse backward (a10) against the CPU oracle.

The oracle restates the gradients of the reference's token-level attention
(`miowtion/kernels/reference.py:23-56` through autograd); the tolerance and
the "closer to the sparse than to the dense gradients" check are those of
the reference's own backward test
(`tests/gpu/test_kernels_gpu.py:200-250`: rtol = atol = 3e-2 on real rows);
the normalized error max|got - want| / max|want| must also stay within
2e-2 (`parity.GRAD`).
"""

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


def np32(t):
    return t.detach().float().cpu().numpy()


@pytest.fixture(autouse=True)
def _status_clean():
    _lib.device_status(reset=True)
    yield
    assert _lib.device_status(reset=True) == 0, 'a kernel wait timed out'


@pytest.fixture(scope='module')
def padded():
    spec = dict(inputs.PADDED, heads=4, group_heads=[0, 2, 3])
    lay = tiling.build_tile_layout(
        [tiling.TiledSpan(s, tuple(g), tiling.TileShape(*sh))
         for s, g, sh in spec['spans']], spec['used'], spec['seq_len'], DEV)
    ref = vo.build_tile_layout(
        [vo.Span(s, tuple(g), tuple(sh)) for s, g, sh in spec['spans']],
        spec['used'], spec['seq_len'])
    q, k, v = (t.to(DEV) for t in inputs.qkv(spec['seq_len'], spec['heads'],
                                              128, spec['seed'],
                                              torch.bfloat16))
    heads = torch.tensor(spec['group_heads'], device=DEV)
    qt, kt, vt = (tiling.gather_tiles(t, lay, heads) for t in (q, k, v))
    return lay, ref, qt, kt, vt


def _mask(heads, n, density, seed):
    gen = torch.Generator().manual_seed(seed)
    m = torch.rand(heads, n, n, generator=gen) < density
    m[:, torch.arange(n), torch.arange(n)] = True
    m[:, 5, :] = False  # a query tile with no key
    m[:, :, 7] = False  # a key tile no query attends
    return m


def _grads(qt, kt, vt, mask, lay, dout):
    ts = [t.detach().clone().requires_grad_(True) for t in (qt, kt, vt)]
    out = kernels.block_sparse_attention(ts[0], ts[1], ts[2], mask, lay)
    out.backward(dout)
    return [t.grad for t in ts]


@pytest.mark.parametrize('density', [0.3, 1.0])
def test_backward_matches_oracle(padded, density):
    lay, ref, qt, kt, vt = padded
    heads = qt.shape[1]
    mask = _mask(heads, lay.n_tiles, density, 41)
    gen = torch.Generator().manual_seed(4)
    dout = torch.randn(qt.shape, generator=gen).to(DEV, torch.bfloat16)
    got = _grads(qt, kt, vt, mask.to(DEV), lay, dout)
    want = vo.block_sparse_attention_bwd(np32(qt), np32(kt), np32(vt),
                                         np32(dout), mask.numpy(),
                                         ref.valid_count)
    real = ref.slot_valid.astype(bool)
    dense = vo.block_sparse_attention_bwd(
        np32(qt), np32(kt), np32(vt), np32(dout),
        np.ones_like(mask.numpy()), ref.valid_count) if density < 1 else None
    for name, g, w, i in zip('qkv', got, want, range(3)):
        g = np32(g)
        np.testing.assert_allclose(g[real], w[real], rtol=3e-2, atol=3e-2,
                                   err_msg=f'd{name}')
        parity.assert_rel(g, w, parity.GRAD,
                          f'backward d{name}, padded layout, density '
                          f'{density}', where=real)
        assert not (g[real] == 0).all(), f'd{name} is all zeros'
        if dense is not None:
            sparse_err = np.abs(g[real] - w[real]).max()
            dense_err = np.abs(g[real] - dense[i][real]).max()
            assert sparse_err < dense_err, (
                f'd{name} is as close to the dense gradient as to the sparse '
                'one: the block pattern was likely ignored')
    # Tiles without any block: zero gradients.
    assert (np32(got[0])[5 * 128:6 * 128] == 0).all()
    assert (np32(got[1])[7 * 128:8 * 128] == 0).all()
    assert (np32(got[2])[7 * 128:8 * 128] == 0).all()


def test_backward_is_deterministic(padded):
    lay, _, qt, kt, vt = padded
    mask = _mask(qt.shape[1], lay.n_tiles, 0.5, 43).to(DEV)
    gen = torch.Generator().manual_seed(5)
    dout = torch.randn(qt.shape, generator=gen).to(DEV, torch.bfloat16)
    a = _grads(qt, kt, vt, mask, lay, dout)
    b = _grads(qt, kt, vt, mask, lay, dout)
    for x, y in zip(a, b):
        assert torch.equal(x, y)


def test_backward_linear_in_dout(padded):
    """dq, dk, dv are linear in dO: doubling dO doubles every gradient
    (exactly, as every step scales by a power of two)."""
    lay, _, qt, kt, vt = padded
    mask = _mask(qt.shape[1], lay.n_tiles, 0.4, 47).to(DEV)
    gen = torch.Generator().manual_seed(6)
    dout = torch.randn(qt.shape, generator=gen).to(DEV, torch.bfloat16)
    a = _grads(qt, kt, vt, mask, lay, dout)
    b = _grads(qt, kt, vt, mask, lay, dout * 2)
    for x, y in zip(a, b):
        torch.testing.assert_close(y.float(), 2 * x.float(), rtol=2e-2,
                                   atol=2e-2)


def test_backward_full_size_cfg3_sampled_tiles():
    """cfg3 group a at full size (788 tiles, 1024 text rows), one head,
    lists from the selection kernel at the 90% budget: dQ of sampled query
    tiles and dK / dV of sampled key tiles against the oracle. A query
    tile's dQ needs only its own row of the mask; a key tile's dK / dV
    needs every query tile that keeps it, so the oracle runs on exactly
    those rows."""
    from miowtion_b200 import mask as veda_mask
    spec = inputs.BENCH_LAYOUTS['cfg3_a']
    spans = [tiling.TiledSpan(st, tuple(g), tiling.TileShape(*sh))
             for st, g, sh in spec['spans']]
    lay = tiling.build_tile_layout(spans, spec['used'], spec['seq_len'], DEV)
    ref = vo.build_tile_layout(
        [vo.Span(st, tuple(g), tuple(sh)) for st, g, sh in spec['spans']],
        spec['used'], spec['seq_len'])
    q, k, v = (t.to(DEV) for t in inputs.qkv(spec['seq_len'], 2, 128, 91,
                                              torch.bfloat16))
    hd = torch.tensor([1], device=DEV)
    qt, kt, vt = (tiling.gather_tiles(t, lay, hd) for t in (q, k, v))
    blocks = veda_mask.column_blocks(lay, veda_mask.Budget(ratio=0.1))
    scores = inputs.scores(1, lay.n_tiles, 23)[:, :lay.n_video_tiles]
    lists = veda_mask.select_block_lists(scores.to(DEV), lay, blocks,
                                         want_mask=True)
    mask = lists.mask.bool()
    dout = inputs.dout(qt.shape, 24).to(DEV)
    dq, dk, dv = _grads(qt, kt, vt, mask, lay, dout)
    torch.cuda.synchronize()
    m = mask.cpu().numpy()
    n = lay.n_tiles
    tile_rows = lambda t: (np.asarray(t)[:, None] * 128 +  # noqa: E731
                           np.arange(128)).reshape(-1)
    real = ref.slot_valid.astype(bool)
    # dQ of sampled query tiles: partial, full, last video and global.
    qs = np.array(sorted({*ref.partial_tiles[:2].tolist(), 0, 411,
                          lay.n_video_tiles - 1, n - 1}))
    rows = tile_rows(qs)
    want_dq, _, _ = vo.block_sparse_attention_bwd(
        np32(qt)[rows], np32(kt), np32(vt), np32(dout)[rows], m[:, qs],
        ref.valid_count)
    ok = real[rows]
    got_dq = np32(dq)[rows]
    np.testing.assert_allclose(got_dq[ok], want_dq[ok], rtol=3e-2, atol=3e-2)
    parity.assert_rel(got_dq, want_dq, parity.GRAD,
                      'backward dq, cfg3 full size, sampled query tiles',
                      where=ok)
    # dK, dV of sampled key tiles (one partial), from every query tile
    # that keeps them.
    ks = np.array(sorted({int(ref.partial_tiles[5]), 300, 777}))
    users = np.nonzero(m[0][:, ks].any(-1))[0]
    urows = tile_rows(users)
    _, want_dk, want_dv = vo.block_sparse_attention_bwd(
        np32(qt)[urows], np32(kt), np32(vt), np32(dout)[urows],
        m[:, users], ref.valid_count)
    krows = tile_rows(ks)
    kok = real[krows]
    for name, got, want in (('dk', dk, want_dk), ('dv', dv, want_dv)):
        g, w = np32(got)[krows], want[krows]
        np.testing.assert_allclose(g[kok], w[kok], rtol=3e-2, atol=3e-2,
                                   err_msg=name)
        parity.assert_rel(g, w, parity.GRAD,
                          f'backward {name}, cfg3 full size, sampled key '
                          'tiles', where=kok)
