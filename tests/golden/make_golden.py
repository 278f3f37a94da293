"""Generate golden vectors from the reference implementation (run in the
build container, where the reference's Python can be imported).

    PYTHONPATH=<path to the reference checkout> python tests/golden/make_golden.py

Writes `tests/golden/*.npz`. Inputs are regenerated from the stated torch
seeds by `tests/golden/inputs.py` (shared with the tests), and a checksum of
every input is stored so a change in the RNG is caught instead of silently
changing the comparison. Large outputs are subsampled (rows [::8]) to keep
the fixtures small; the oracle is checked on the same subsample.
"""

from __future__ import annotations

import hashlib
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

import inputs  # noqa: E402  (tests/golden/inputs.py)

from miowtion.h3 import attention as h3_attention  # noqa: E402
from miowtion.h3 import layout as h3_layout  # noqa: E402
from miowtion.kernels import fa4  # noqa: E402
from miowtion.kernels import reference  # noqa: E402
from miowtion.veda import attention as veda_attention  # noqa: E402
from miowtion.veda import heatmap  # noqa: E402
from miowtion.veda import mask as veda_mask  # noqa: E402
from miowtion.veda import plan as veda_plan  # noqa: E402
from miowtion.veda import predictor as veda_predictor  # noqa: E402
from miowtion.veda import tiling  # noqa: E402


def digest(t: torch.Tensor) -> str:
    return hashlib.sha256(t.detach().contiguous().view(-1).float()
                          .numpy().tobytes()).hexdigest()


def layout_arrays(prefix: str, lay) -> dict:
    return {
        f'{prefix}perm': lay.perm.numpy(),
        f'{prefix}valid_count': lay.valid_count.numpy(),
        f'{prefix}scalars': np.array([lay.n_video_tiles, lay.n_ref_tiles,
                                      lay.n_global_tiles, lay.ref_tokens,
                                      lay.target_tokens, lay.used,
                                      lay.seq_len], dtype=np.int64),
    }


def ref_layout(spec):
    spans = [tiling.TiledSpan(s, g, tiling.TileShape(*sh))
             for s, g, sh in spec['spans']]
    return tiling.build_tile_layout(spans, spec['used'], spec['seq_len'])


def half_rows(t: torch.Tensor) -> np.ndarray:
    """Rows [::4] as float16: the tolerances checked are >= 1e-2."""
    return t[::4].float().numpy().astype(np.float16)


def save(name: str, **arrays) -> None:
    path = os.path.join(HERE, f'{name}.npz')
    np.savez_compressed(path, **arrays)
    print(f'wrote {path} ({os.path.getsize(path) / 1024:.0f} KiB)')


# -- config 1: the whole SparseStudent layer on CPU ---------------------------

class _Clip(veda_attention.ClipTiling):
    """ClipTiling over a PackedLayout that holds only what it reads."""


def cfg1() -> None:
    spec = inputs.CFG1
    q, k, v = inputs.qkv(spec['seq_len'], spec['heads'], spec['dim'],
                         spec['seed'], torch.float32)
    proj_q, proj_k = inputs.predictor_weights(spec['heads'], spec['dim'],
                                              spec['pred_seed'],
                                              spec['pred_std'])
    packed = h3_layout.PackedLayout(
        seq_len=spec['seq_len'], used=spec['used'], text_len=0,
        img_pos=torch.arange(spec['used']),
        audio_pos=torch.zeros(0, dtype=torch.long),
        update_mask=torch.ones(spec['used'], dtype=torch.bool),
        audio_update_mask=torch.zeros(0, dtype=torch.bool),
        position_ids=torch.zeros(spec['seq_len'], 3, dtype=torch.float64),
        token_tags=torch.zeros(spec['seq_len'], dtype=torch.long),
        cu_seqlens=torch.tensor([0, spec['used'], spec['seq_len']],
                                dtype=torch.int32),
        spans=(h3_layout.VideoSpan(0, spec['grid'], 'target'),),
        visual_cond_shapes=(), audio_cond_lengths=())
    config = veda_attention.VedaConfig(
        target_budget=veda_mask.Budget(ratio=spec['ratio']))
    clip = veda_attention.ClipTiling(packed, config, torch.device('cpu'))
    shape = tiling.TileShape(*spec['shape'])
    plan = veda_plan.TilePlan('cfg1', spec['grid'], [shape],
                              [[0] * spec['heads']])
    predictor = veda_predictor.TileScorePredictor(1, spec['heads'],
                                                  spec['dim'])
    with torch.no_grad():
        predictor.layers[0].proj_q.copy_(proj_q)
        predictor.layers[0].proj_k.copy_(proj_k)
    student = veda_attention.SparseStudent(clip, plan, predictor,
                                           allow_reference_kernel=True)
    with torch.no_grad():
        out = student(q, k, v, 0)
    # Intermediates through the same functions SparseStudent uses.
    lay = clip.get(shape)
    heads = torch.arange(spec['heads'])
    qt = tiling.gather_tiles(q, lay, heads)
    kt = tiling.gather_tiles(k, lay, heads)
    fq = veda_predictor.pool_tiles(qt, lay)
    fk = veda_predictor.pool_tiles(kt, lay)
    with torch.no_grad():
        logits = predictor.layers[0](fq, fk, heads)
    sel = veda_mask.select_video_blocks(logits[:, :lay.n_video_tiles], lay,
                                        clip.blocks(lay))
    mask = veda_mask.dense_block_mask(sel, lay)
    lists = fa4.index_lists(mask, lay)
    lists_t = fa4.index_lists(mask, lay, transpose=True)
    save('cfg1',
         q_digest=np.array(digest(q)), k_digest=np.array(digest(k)),
         v_digest=np.array(digest(v)), p_digest=np.array(digest(proj_q)),
         **layout_arrays('', lay),
         feats_q=fq.numpy(), feats_k=fk.numpy(), logits=logits.numpy(),
         sel_index=sel.index.numpy(), sel_keep=sel.keep.numpy(),
         mask=mask.numpy(),
         **{f'lists_{n}': t.numpy() for n, t in zip(
             ('part_cnt', 'part_idx', 'full_cnt', 'full_idx'), lists)},
         **{f'tlists_{n}': t.numpy() for n, t in zip(
             ('part_cnt', 'part_idx', 'full_cnt', 'full_idx'), lists_t)},
         out_rows=out[::8].numpy())


# -- a padded layout with text rows: every kernel's contract ------------------

def padded() -> None:
    spec = inputs.PADDED
    lay = ref_layout(spec)
    assert lay.partial_tiles.numel() > 0
    q, k, v = inputs.qkv(spec['seq_len'], spec['heads'], spec['dim'],
                         spec['seed'], torch.bfloat16)
    heads = torch.tensor(spec['group_heads'])
    qt, kt, vt = (tiling.gather_tiles(t, lay, heads) for t in (q, k, v))
    fq = veda_predictor.pool_tiles(qt, lay)
    fk = veda_predictor.pool_tiles(kt, lay)
    fq_sq = veda_predictor.pool_tiles(qt, lay, veda_predictor.SECOND_RAW)
    fk_var = veda_predictor.pool_tiles(kt, lay,
                                       veda_predictor.SECOND_CENTRAL)
    proj_q, proj_k = inputs.predictor_weights(spec['heads'], spec['dim'],
                                              spec['pred_seed'], 0.02)
    layer = veda_predictor.LayerPredictor(spec['heads'], spec['dim'])
    with torch.no_grad():
        layer.proj_q.copy_(proj_q)
        layer.proj_k.copy_(proj_k)
        logits = layer(fq, fk, heads)
    blocks = veda_mask.column_blocks(lay, veda_mask.Budget(
        ratio=spec['ratio']))
    scores = inputs.scores(len(spec['group_heads']), lay.n_tiles,
                           spec['score_seed'])
    sel = veda_mask.select_video_blocks(scores[:, :lay.n_video_tiles], lay,
                                        blocks)
    mask = veda_mask.dense_block_mask(sel, lay)
    lists = fa4.index_lists(mask, lay)
    lists_t = fa4.index_lists(mask, lay, transpose=True)
    out, lse = reference.block_sparse_attention(qt, kt, vt, mask,
                                                lay.valid_count,
                                                return_lse=True)
    # Backward through autograd of the reference kernel.
    dout = inputs.dout(qt.shape, spec['dout_seed'])
    leaves = [t.detach().clone().requires_grad_(True) for t in (qt, kt, vt)]
    ref_out = reference.block_sparse_attention(*leaves, mask,
                                               lay.valid_count)
    ref_out.backward(dout)
    grads = [t.grad for t in leaves]
    # Dense attention with LSE (math backend) and the teacher heat.
    dout_dense, dlse = h3_attention.dense_attention(q, k, v, lay.used,
                                                    return_lse=True,
                                                    backend='math')
    lse_t = veda_attention._gather_lse(dlse, lay, heads)  # pylint: disable=protected-access
    rows = torch.tensor(spec['heat_rows'])
    heat_max = heatmap.teacher_heat_reference(qt, kt, lse_t, lay, rows,
                                              q_chunk=128, k_chunk=256,
                                              reduce='max')
    heat_sum = heatmap.teacher_heat_reference(qt, kt, lse_t, lay, rows,
                                              q_chunk=128, k_chunk=256,
                                              reduce='sum')
    # Scatter of the attention output into [S+1, H, D].
    buf = torch.zeros(lay.seq_len + 1, spec['heads'], spec['dim'],
                      dtype=torch.bfloat16)
    tiling.scatter_tiles_(buf, out, lay, heads)
    save('padded',
         q_digest=np.array(digest(q)), k_digest=np.array(digest(k)),
         v_digest=np.array(digest(v)), s_digest=np.array(digest(scores)),
         d_digest=np.array(digest(dout)),
         **layout_arrays('', lay),
         feats_q=fq.numpy(), feats_k=fk.numpy(), sq_q=fq_sq.numpy(),
         var_k=fk_var.numpy(), logits=logits.numpy(),
         sel_index=sel.index.numpy(), sel_keep=sel.keep.numpy(),
         mask=mask.numpy(),
         **{f'lists_{n}': t.numpy() for n, t in zip(
             ('part_cnt', 'part_idx', 'full_cnt', 'full_idx'), lists)},
         **{f'tlists_{n}': t.numpy() for n, t in zip(
             ('part_cnt', 'part_idx', 'full_cnt', 'full_idx'), lists_t)},
         attn_out=half_rows(out), attn_lse=lse.numpy(),
         dq=half_rows(grads[0]), dk=half_rows(grads[1]),
         dv=half_rows(grads[2]),
         dense_out=half_rows(dout_dense), dense_lse=dlse.numpy(),
         heat_max=heat_max.numpy(), heat_sum=heat_sum.numpy(),
         scatter=half_rows(buf))


# -- segmented (reference + target) budgets -----------------------------------

def segmented() -> None:
    spec = inputs.SEGMENTED
    lay = ref_layout(spec)
    blocks = veda_mask.column_blocks(
        lay, veda_mask.Budget(ratio=spec['target_ratio']),
        veda_mask.Budget(ratio=spec['ref_ratio']))
    scores = inputs.scores(spec['heads'], lay.n_tiles, spec['score_seed'])
    sel = veda_mask.select_video_blocks(scores[:, :lay.n_video_tiles], lay,
                                        blocks)
    mask = veda_mask.dense_block_mask(sel, lay)
    rows = torch.tensor(spec['subset_rows'])
    sub = veda_mask.select_video_blocks(scores[:, rows], lay, blocks, rows)
    sub_mask = veda_mask.dense_block_mask(sub, lay, global_rows=False)
    lists = fa4.index_lists(mask, lay)
    lists_t = fa4.index_lists(mask, lay, transpose=True)
    save('segmented',
         s_digest=np.array(digest(scores)),
         **layout_arrays('', lay),
         sel_index=sel.index.numpy(), sel_keep=sel.keep.numpy(),
         mask=mask.numpy(), sub_index=sub.index.numpy(),
         sub_keep=sub.keep.numpy(), sub_mask=sub_mask.numpy(),
         **{f'lists_{n}': t.numpy() for n, t in zip(
             ('part_cnt', 'part_idx', 'full_cnt', 'full_idx'), lists)},
         **{f'tlists_{n}': t.numpy() for n, t in zip(
             ('part_cnt', 'part_idx', 'full_cnt', 'full_idx'), lists_t)})


# -- small tiling layouts of the reference's own unit tests -------------------

def layouts() -> None:
    arrays = {}
    for name, spec in inputs.SMALL_LAYOUTS.items():
        arrays.update(layout_arrays(f'{name}_', ref_layout(spec)))
    # Budget facts of the benchmark configurations (full size).
    facts = []
    for name, spec in inputs.BENCH_LAYOUTS.items():
        lay = ref_layout(spec)
        h = hashlib.sha256(lay.perm.numpy().tobytes()).hexdigest()
        arrays[f'{name}_perm_sha256'] = np.array(h)
        arrays[f'{name}_valid_count'] = lay.valid_count.numpy()
        arrays[f'{name}_scalars'] = layout_arrays('', lay)['scalars']
        for budget in spec['budgets']:
            blocks = veda_mask.column_blocks(
                lay, veda_mask.Budget(ratio=budget[1]),
                None if budget[0] is None else veda_mask.Budget(
                    ratio=budget[0]))
            for b in blocks:
                per_row = b.budget.per_row(b.real_tokens, b.stop - b.start)
                k_lo, k_hi, frac = veda_mask.split_budget(per_row,
                                                          b.stop - b.start)
                extra = veda_mask.bresenham_extra(lay.n_video_tiles, frac,
                                                  'cpu')
                facts.append([b.start, b.stop, b.real_tokens, per_row,
                              k_lo, k_hi, frac, int(extra.sum())])
    arrays['budget_facts'] = np.array(facts, dtype=np.float64)
    # Bresenham / split_budget known answers of test_veda_predictor_mask.
    kat = []
    for budget in (1.0, 2.3, 3.75, 5.5, 68.69538461538462, 0.5, 100.0):
        k_lo, k_hi, frac = veda_mask.split_budget(budget, 64)
        extra = veda_mask.bresenham_extra(400, frac, 'cpu')
        kat.append([budget, k_lo, k_hi, frac, int(extra.sum()),
                    int(extra[:7].to(torch.int64) @ (2 ** torch.arange(7)))])
    arrays['split_kat'] = np.array(kat, dtype=np.float64)
    arrays['equal_cost'] = np.array(
        [veda_mask.Budget(ratio=0.1).per_row(37296, 330)])
    save('layouts', **arrays)


if __name__ == '__main__':
    torch.set_num_threads(8)
    np.set_printoptions(precision=4)
    layouts()
    segmented()
    padded()
    cfg1()
