"""Golden vectors of the reference's 'threshold' budget rule, run on CPU in
the build container:

    PYTHONPATH=<path to the reference checkout> python tests/golden/make_threshold.py

Stores `select_video_blocks(..., rule='threshold')` (index and keep) of
seeded scores on the padded layout (all video rows, then a row subset) and
on the segmented layout (condition and target budgets), and
`threshold_allowed` of seeded descending candidates with forced (+inf) and
invalid entries. Writes `tests/golden/threshold.npz`.
"""

from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

import inputs  # noqa: E402

from miowtion.veda import mask as veda_mask  # noqa: E402
from miowtion.veda import tiling  # noqa: E402


def layout(spec):
    return tiling.build_tile_layout(
        [tiling.TiledSpan(s, g, tiling.TileShape(*sh))
         for s, g, sh in spec['spans']], spec['used'], spec['seq_len'])


def main() -> None:
    out = {}
    gen = torch.Generator().manual_seed(inputs.THRESHOLD['seed'])
    pad, seg = inputs.PADDED, inputs.SEGMENTED
    cases = {
        'padded': (layout(pad), pad['heads'], None,
                   lambda lay: veda_mask.column_blocks(
                       lay, veda_mask.Budget(ratio=pad['ratio']))),
        'padded_rows': (layout(pad), pad['heads'],
                        inputs.THRESHOLD['rows'],
                        lambda lay: veda_mask.column_blocks(
                            lay, veda_mask.Budget(ratio=pad['ratio']))),
        'segmented': (layout(seg), seg['heads'], None,
                      lambda lay: veda_mask.column_blocks(
                          lay, veda_mask.Budget(ratio=seg['target_ratio']),
                          veda_mask.Budget(ratio=seg['ref_ratio']))),
    }
    for name, (lay, heads, rows, make_blocks) in cases.items():
        n_rows = lay.n_video_tiles if rows is None else len(rows)
        scores = torch.randn(heads, n_rows, lay.n_tiles, generator=gen)
        rows_t = None if rows is None else torch.tensor(rows)
        sel = veda_mask.select_video_blocks(scores, lay, make_blocks(lay),
                                            rows_t, rule='threshold')
        out[f'{name}_scores'] = scores.numpy()
        out[f'{name}_index'] = sel.index.numpy()
        out[f'{name}_keep'] = sel.keep.numpy()
    cand = torch.randn(3, 11, 9, generator=gen).sort(-1, descending=True)
    vals = cand.values
    vals[:, ::3, 0] = float('inf')           # forced diagonal
    vals[1, 2, 6:] = float('-inf')           # a short row
    valid = vals > float('-inf')
    out['allowed_vals'] = vals.numpy()
    out['allowed'] = veda_mask.threshold_allowed(
        vals, valid, torch.tensor(2.6), 9).numpy()
    path = os.path.join(HERE, 'threshold.npz')
    np.savez_compressed(path, **out)
    print(f'wrote {path} ({os.path.getsize(path) / 1024:.0f} KiB)')


if __name__ == '__main__':
    main()
