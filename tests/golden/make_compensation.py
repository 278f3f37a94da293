"""Generate the zero-order compensation fixture from the reference
implementation, in the build container where its Python can be imported:

    PYTHONPATH=<path to the reference checkout> python tests/golden/make_compensation.py

Writes `tests/golden/compensation.npz` for the seeded `inputs.COMPENSATION`
case (fp32 q/k/v): the keep mask the reference selects from seeded block
scores, and the output of its torch `zero_order_compensation`
(miowtion/veda/attention.py:591-689) after its `reference.block_sparse_
attention(..., return_lse=True)`, stored as per-row checksums out . w for a
seeded w (all rows) plus the whole rows of one query tile.
"""

from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

import inputs  # noqa: E402

from miowtion.kernels import reference  # noqa: E402
from miowtion.veda import attention as veda_attention  # noqa: E402
from miowtion.veda import mask as veda_mask  # noqa: E402
from miowtion.veda import tiling  # noqa: E402


def main() -> None:
    spec = inputs.COMPENSATION
    lay = tiling.build_tile_layout(
        [tiling.TiledSpan(s, g, tiling.TileShape(*sh))
         for s, g, sh in spec['spans']], spec['used'], spec['seq_len'])
    q, k, v = inputs.qkv(spec['seq_len'], spec['heads'], spec['dim'],
                         spec['seed'], torch.float32)
    heads = torch.arange(spec['heads'])
    qt, kt, vt = (tiling.gather_tiles(t, lay, heads) for t in (q, k, v))
    scores = inputs.scores(spec['heads'], lay.n_tiles, spec['score_seed'])
    blocks = veda_mask.column_blocks(lay, veda_mask.Budget(
        ratio=spec['ratio']))
    sel = veda_mask.select_video_blocks(scores[:, :lay.n_video_tiles], lay,
                                        blocks)
    mask = veda_mask.dense_block_mask(sel, lay)
    with torch.no_grad():
        o_kept, lse = reference.block_sparse_attention(
            qt, kt, vt, mask, lay.valid_count, return_lse=True)
        out = veda_attention.zero_order_compensation(o_kept, lse, qt, kt, vt,
                                                     mask, lay)
    w = inputs.projection(spec['dim'], spec['proj_seed'])
    t = spec['full_tile']
    np.savez_compressed(
        os.path.join(HERE, 'compensation.npz'), mask=mask.numpy(),
        check_out=(out @ w).numpy(), check_kept=(o_kept @ w).numpy(),
        tile_out=out[t * 128:(t + 1) * 128].numpy().astype(np.float16))
    print('rows', out.shape, 'max |out - o_kept|',
          float((out - o_kept).abs().max()))


if __name__ == '__main__':
    main()
