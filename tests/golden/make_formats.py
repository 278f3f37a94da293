"""Generate the format fixtures (geometry rounding, plan selection, predictor
bundles) from the reference implementation, in the build container where
its Python can be imported:

    PYTHONPATH=<path to the reference checkout> python tests/golden/make_formats.py

Writes `tests/golden/formats.json`, the fp32 weights of a seeded 2-layer x
3-head x 16-dim predictor (`bundle_weights.safetensors`) and the two bundles
the reference's own `bundle.save` writes from them (bf16 and fp8 storage,
`bundle_ref_{bf16,fp8}.safetensors`). Loaded tensors are recorded as sha256
digests of their bytes.
"""

from __future__ import annotations

import hashlib
import json
import os

import torch
from safetensors.torch import save_file

from miowtion.h3 import geometry as ref_geometry
from miowtion.veda import bundle as ref_bundle
from miowtion.veda import plan as ref_plan
from miowtion.veda import predictor as ref_predictor
from miowtion.veda import tiling as ref_tiling

HERE = os.path.dirname(os.path.abspath(__file__))

ASPECTS = ['16:9', '9:16', '4:3', '3:4', '1:1', '21:9', '9:21', '4:1', '1:4',
           '2:3', '5:4', '7:3']
SECONDS = [0.0, 0.1, 2.5, 5.0, 7.2, 10.0, 12.34, 15.0]


def digest(t: torch.Tensor) -> str:
    """sha256 of a tensor's bytes (row-major)."""
    return hashlib.sha256(
        t.detach().contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def geometry_row(g) -> dict:
    return {'aspect': g.aspect, 'width': g.width, 'height': g.height,
            'frame_count': g.frame_count, 'latent_t': g.latent_t,
            'latent_h': g.latent_h, 'latent_w': g.latent_w,
            'audio_t': g.audio_t, 'name': g.name,
            'video_grid': list(g.video_grid)}


def make_plans():
    """A small plan table: two searched-style plans for 16:9, one for 1:1,
    one for 4:3 with two shapes per layer."""
    s = ref_tiling.TileShape
    plans = []
    for aspect, lt, shapes, rows in [
            ('16:9', 37, [s(2, 8, 8), s(1, 8, 16)], [[0, 1, 0], [1, 1, 0]]),
            ('16:9', 102, [s(4, 4, 8)], [[0, 0, 0], [0, 0, 0]]),
            ('1:1', 72, [s(2, 8, 8), s(8, 4, 4)], [[0, 1, 1], [1, 0, 1]]),
            ('4:3', 37, [s(1, 16, 8), s(2, 4, 16)], [[1, 1, 0], [0, 0, 0]])]:
        g = ref_geometry.geometry_from_latent_t(aspect, lt)
        plans.append(ref_plan.TilePlan(g.name, g.video_grid, shapes, rows,
                                       {'source': 'fixture', 'keep': 0.1}))
    return ref_plan.PlanTable(plans)


def main() -> None:
    out = {'geometries': [], 'ladder': ref_geometry.latent_t_ladder(),
           'canvas_errors': []}
    for aspect in ASPECTS:
        for sec in SECONDS:
            out['geometries'].append(
                {'seconds': sec,
                 **geometry_row(ref_geometry.resolve_geometry(aspect, sec))})
    for aspect in ['5:1', '1:5', '9:40']:
        w, h = (int(v) for v in aspect.split(':'))
        try:
            ref_geometry.resolve_canvas(w, h)
            out['canvas_errors'].append([aspect, None])
        except ValueError as e:
            out['canvas_errors'].append([aspect, str(e)])
    table = make_plans()
    out['plans'] = {k: p.to_json() for k, p in table.plans.items()}
    out['mirrored'] = {}
    for name, p in table.plans.items():
        try:
            out['mirrored'][name] = p.mirrored().to_json()
        except ValueError as e:
            out['mirrored'][name] = {'error': str(e)}
    out['transposed'] = {k: p.transposed().to_json()
                         for k, p in table.plans.items()}
    out['select'] = []
    for aspect in ['16:9', '9:16', '1:1', '4:3', '3:4', '21:9']:
        for lt in [2, 37, 52, 72, 102, 167]:
            g = ref_geometry.geometry_from_latent_t(aspect, lt)
            try:
                chosen = table.select(g)
                out['select'].append([aspect, lt, chosen.to_json()])
            except KeyError as e:
                out['select'].append([aspect, lt, {'error': str(e)}])
    out['uniform'] = ref_plan.TilePlan.uniform(
        ref_geometry.geometry_from_latent_t('9:16', 52),
        ref_tiling.least_padding_shape(
            ref_geometry.geometry_from_latent_t('9:16', 52).video_grid),
        2, 3).to_json()
    # Bundles written by the reference.
    torch.manual_seed(7)
    model = ref_predictor.TileScorePredictor(2, 3, 16)
    with torch.no_grad():
        for i, layer in enumerate(model.layers):
            layer.proj_q.normal_(std=0.02)
            layer.proj_k.normal_(std=0.02 * (i + 1))
            layer.proj_k[1].mul_(1e3)  # a head far out of e4m3's range
            layer.proj_q[2].zero_()    # an all-zero head
    weights = {f'predictor.{k}': v for k, v in model.state_dict().items()}
    save_file({k: v.contiguous() for k, v in model.state_dict().items()},
              os.path.join(HERE, 'bundle_weights.safetensors'))
    for tag, dtype in [('bf16', torch.bfloat16),
                       ('fp8', torch.float8_e4m3fn)]:
        path = os.path.join(HERE, f'bundle_ref_{tag}.safetensors')
        ref_bundle.save(path, weights, table, num_layers=2, num_heads=3,
                        head_dim=16, keep_tiles=12.5, ref_keep_ratio=0.05,
                        tile_conditions=True, source='fixture',
                        source_weights='live', step=1234, dtype=dtype)
        loaded = ref_bundle.load(path)
        out[f'bundle_{tag}_metadata'] = loaded.metadata
        out[f'bundle_{tag}_loaded'] = {
            k: [str(v.dtype), list(v.shape), digest(v)]
            for k, v in loaded.predictor.state_dict().items()}
    with open(os.path.join(HERE, 'formats.json'), 'w') as f:
        json.dump(out, f, indent=0)


if __name__ == '__main__':
    main()
