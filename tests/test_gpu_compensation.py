"""GPU parity of the zero-order compensation ((f) row 4) against the CPU
oracle, which is pinned to the reference's torch form
(tests/test_compensation.py). The kernel stores the key centroids and value
sums in bf16, as the reference's Triton form does, so the oracle runs with
bf16 summaries; tolerance 2e-2, the reference's forward tolerance."""

import dataclasses

import numpy as np
import pytest
import torch

import inputs
import parity
from miowtion_b200 import _lib
from miowtion_b200 import attention as veda_attention
from miowtion_b200 import compensation
from miowtion_b200 import kernels
from miowtion_b200 import mask as veda_mask
from miowtion_b200 import plan as veda_plan
from miowtion_b200 import predictor as veda_predictor
from miowtion_b200 import tiling
from oracle import veda_oracle as vo

pytestmark = pytest.mark.gpu

DEV = 'cuda'
TOL = dict(rtol=2e-2, atol=2e-2)


@pytest.fixture(autouse=True)
def _status_clean():
    _lib.device_status(reset=True)
    yield
    assert _lib.device_status(reset=True) == 0, 'a kernel wait timed out'


def np32(t):
    return t.detach().float().cpu().numpy()


def build(spans, used, seq_len, heads, seed, score_seed, ratio):
    lay = tiling.build_tile_layout(
        [tiling.TiledSpan(s, tuple(g), tiling.TileShape(*sh))
         for s, g, sh in spans], used, seq_len, DEV)
    ref = vo.build_tile_layout(
        [vo.Span(s, tuple(g), tuple(sh)) for s, g, sh in spans], used,
        seq_len)
    q, k, v = inputs.qkv(seq_len, heads, 128, seed, torch.bfloat16)
    hd = torch.arange(heads, device=DEV)
    qt, kt, vt = (tiling.gather_tiles(t.to(DEV), lay, hd) for t in (q, k, v))
    scores = inputs.scores(heads, ref.n_tiles, score_seed).numpy()
    blocks = vo.column_blocks(ref, vo.Budget(ratio=ratio))
    index, keep = vo.select_video_blocks(scores[:, :ref.n_video_tiles], ref,
                                         blocks)
    mask = vo.dense_block_mask(index, keep, ref)
    return lay, ref, qt, kt, vt, mask


def oracle_out(ref, qt, kt, vt, mask, rows=None):
    qf, kf, vf = np32(qt), np32(kt), np32(vt)
    if rows is not None:
        slots = (np.asarray(rows)[:, None] * 128 + np.arange(128)).reshape(-1)
        qf = qf[slots]
    o, lse = vo.block_sparse_attention(qf, kf, vf, mask, ref.valid_count,
                                       return_lse=True)
    return vo.zero_order_compensation(o, lse, qf, kf, vf, mask, ref,
                                      bf16_summaries=True)


@pytest.fixture(scope='module')
def padded():
    spec = inputs.COMPENSATION
    return build(spec['spans'], spec['used'], spec['seq_len'], spec['heads'],
                 spec['seed'], spec['score_seed'], spec['ratio'])


def test_compensation_matches_oracle(padded):
    lay, ref, qt, kt, vt, mask = padded
    m = torch.from_numpy(mask).to(DEV)
    o_kept, lse = kernels.block_sparse_attention(qt, kt, vt, m, lay,
                                                 return_lse=True)
    got = compensation.compensate(o_kept, lse, qt, kt, vt, m, lay)
    want = oracle_out(ref, qt, kt, vt, mask)
    valid = ref.slot_valid.astype(bool)
    np.testing.assert_allclose(np32(got)[valid], want[valid], **TOL)
    parity.assert_rel(np32(got), want, parity.FWD,
                      'zero-order compensation', where=valid)
    assert (got.float() - o_kept.float()).abs().max() > 1e-2
    # End to end, and in place, give the same bits.
    e2e = compensation.attention(qt, kt, vt, m, lay)
    assert torch.equal(e2e, got)
    again = compensation.compensate(o_kept, lse, qt, kt, vt, m, lay)
    assert torch.equal(again, got), 'the compensation must be deterministic'


def test_keep_all_is_the_identity(padded):
    lay, _, qt, kt, vt, mask = padded
    m = torch.ones(mask.shape, dtype=torch.bool, device=DEV)
    o_kept, lse = kernels.block_sparse_attention(qt, kt, vt, m, lay,
                                                 return_lse=True)
    got = compensation.compensate(o_kept, lse, qt, kt, vt, m, lay)
    assert torch.equal(got, o_kept)


def test_query_tile_subset(padded):
    lay, ref, qt, kt, vt, mask = padded
    rows = [1, 4, 9, lay.n_tiles - 1]
    m = torch.from_numpy(mask[:, rows]).to(DEV)
    slots = (torch.tensor(rows)[:, None] * 128 + torch.arange(128)).reshape(
        -1).to(DEV)
    q_sub = qt.index_select(0, slots).contiguous()
    o_kept, lse = kernels.block_sparse_attention(q_sub, kt, vt, m, lay,
                                                 return_lse=True)
    got = compensation.zero_order_compensation(o_kept, lse, q_sub, kt, vt, m,
                                               lay)
    want = oracle_out(ref, qt, kt, vt, mask[:, rows], rows=rows)
    valid = ref.slot_valid.astype(bool)[slots.cpu().numpy()]
    np.testing.assert_allclose(np32(got)[valid], want[valid], **TOL)
    parity.assert_rel(np32(got), want, parity.FWD,
                      'zero-order compensation', where=valid)
    with pytest.raises(ValueError, match='same id'):
        compensation.compensate(o_kept, lse, q_sub, kt, vt, m, lay)


def test_many_chunks_and_partial_last_chunk():
    # 26 x 45 x 80 / (2 x 8 x 8) -> 780 video tiles behind 1024 text rows:
    # seven 128-tile chunks of centroids, the last one partial. Two query
    # tiles' worth of rows per head keeps the oracle quick.
    spans = [(1024, (26, 45, 80), (2, 8, 8))]
    lay, ref, qt, kt, vt, mask = build(spans, 94624, 94624, 2, 41, 42, 0.1)
    rows = [0, 333, 779, lay.n_tiles - 1]
    m = torch.from_numpy(mask[:, rows]).to(DEV)
    slots = (torch.tensor(rows)[:, None] * 128 + torch.arange(128)).reshape(
        -1).to(DEV)
    q_sub = qt.index_select(0, slots).contiguous()
    o_kept, lse = kernels.block_sparse_attention(q_sub, kt, vt, m, lay,
                                                 return_lse=True)
    got = compensation.zero_order_compensation(o_kept, lse, q_sub, kt, vt, m,
                                               lay)
    want = oracle_out(ref, qt, kt, vt, mask[:, rows], rows=rows)
    valid = ref.slot_valid.astype(bool)[slots.cpu().numpy()]
    np.testing.assert_allclose(np32(got)[valid], want[valid], **TOL)
    parity.assert_rel(np32(got), want, parity.FWD,
                      'zero-order compensation', where=valid)


def test_sparse_student_compensation_arm():
    spec = inputs.COMPENSATION
    (start, grid, shape), = spec['spans']
    packed = veda_attention.PackedLayout(
        spec['seq_len'], spec['used'], (veda_attention.VideoSpan(start,
                                                                 grid),))
    plan = veda_plan.TilePlan('c', grid, [tiling.TileShape(*shape)],
                              [[0] * spec['heads']])
    pred = veda_predictor.TileScorePredictor(1, spec['heads'], 128).to(DEV)
    with torch.no_grad():
        for prm in (pred.layers[0].proj_q, pred.layers[0].proj_k):
            prm.normal_(std=0.02)
    q, k, v = (t.to(DEV) for t in inputs.qkv(
        spec['seq_len'], spec['heads'], 128, spec['seed'], torch.bfloat16))
    outs = {}
    for ratio in (0.3, 1.0):
        plain = veda_attention.VedaConfig(
            target_budget=veda_mask.Budget(ratio=ratio))
        for name, cfg in (('plain', plain),
                          ('comp', dataclasses.replace(
                              plain, zero_order_compensation=True))):
            clip = veda_attention.ClipTiling(packed, cfg, DEV)
            with torch.no_grad():
                outs[name, ratio] = veda_attention.SparseStudent(
                    clip, plan, pred)(q, k, v, 0)
    used = spec['used']
    # Inert at full density, active below it.
    assert torch.equal(outs['plain', 1.0][:used], outs['comp', 1.0][:used])
    assert (outs['plain', 0.3][:used].float() -
            outs['comp', 0.3][:used].float()).abs().max() > 1e-2
    with pytest.raises(NotImplementedError):
        veda_attention.SparseStudent(
            veda_attention.ClipTiling(packed, veda_attention.VedaConfig(
                fused_compensation=True), DEV), plan, pred)
