"""Generate the tile-search fixtures from the reference implementation, in
the build container where its Python can be imported:

    PYTHONPATH=<path to the reference checkout> python tests/golden/make_search.py

Writes `tests/golden/search.npz`: per candidate shape, the reference's own
fp32 `oracle_rel_mse_reference` (miowtion/veda/search.py:130-175) of the
seeded `inputs.SEARCH` case, with the sampled rows and the layout of each
candidate; and `tests/golden/search_plan.json`: the plans the reference's
`build_plan` (search.py:297-368) votes from seeded score tables.
"""

from __future__ import annotations

import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

import inputs  # noqa: E402

from miowtion.veda import mask as veda_mask  # noqa: E402
from miowtion.veda import search  # noqa: E402
from miowtion.veda import tiling  # noqa: E402


def main() -> None:
    spec = inputs.SEARCH
    q, k, v = inputs.qkv(spec['seq_len'], spec['heads'], spec['dim'],
                         spec['seed'], torch.bfloat16)
    arrays = {}
    for ci, shape in enumerate(spec['candidates']):
        lay = tiling.build_tile_layout(
            [tiling.TiledSpan(spec['text'], spec['grid'],
                              tiling.TileShape(*shape))],
            spec['used'], spec['seq_len'])
        blocks = veda_mask.column_blocks(lay, veda_mask.Budget(
            ratio=spec['ratio']))
        rows = inputs.search_rows(lay.n_video_tiles, spec['query_tiles'],
                                  spec['sample_seed'])
        err = search.oracle_rel_mse_reference(q, k, v, lay, blocks, rows)
        arrays[f'c{ci}_rows'] = rows.numpy()
        arrays[f'c{ci}_perm'] = lay.perm.numpy()
        arrays[f'c{ci}_rel_mse'] = err.numpy()
        print(shape, err.numpy())
    np.savez_compressed(os.path.join(HERE, 'search.npz'), **arrays)
    # The plan vote.
    cands = [tiling.TileShape.parse(s) for s in spec['vote_candidates']]
    entries = []
    for e, per_layer in enumerate(inputs.vote_tables(spec)):
        for layer, table in enumerate(per_layer):
            entries.append(search.ScoreEntry(f'clip{e % 2}', 10 * e, layer,
                                             table))
    plans = {}
    for max_padding, max_shapes in [(0.2, 2), (0.05, 1), (1.0, 3)]:
        try:
            plan = search.build_plan('16x9_t37', spec['vote_grid'], cands,
                                     entries, spec['vote_layers'],
                                     max_padding=max_padding,
                                     max_shapes_per_layer=max_shapes,
                                     meta={'keep_ratio': 0.1})
            plans[f'{max_padding}_{max_shapes}'] = plan.to_json()
        except ValueError as error:
            plans[f'{max_padding}_{max_shapes}'] = {'error': str(error)}
    with open(os.path.join(HERE, 'search_plan.json'), 'w') as f:
        json.dump(plans, f, indent=0)


if __name__ == '__main__':
    main()
