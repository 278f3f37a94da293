"""On-disk inputs that choose head groups and weights: geometry rounding, the
tile-plan JSON and plan-table selection, and the safetensors predictor
bundle. Checked against fixtures the reference produced
(`tests/golden/make_formats.py`): bundles it wrote must load here to the same
tensors, and bundles written here must hold the same tensors and metadata.
"""

import hashlib
import json
import os

import pytest
import torch
from safetensors import safe_open
from safetensors.torch import load_file

from miowtion_b200 import bundle as veda_bundle
from miowtion_b200 import geometry as veda_geometry
from miowtion_b200 import mask as veda_mask
from miowtion_b200 import plan as veda_plan
from miowtion_b200 import tiling

GOLDEN = os.path.join(os.path.dirname(__file__), 'golden')


@pytest.fixture(scope='module')
def formats():
    with open(os.path.join(GOLDEN, 'formats.json')) as f:
        return json.load(f)


def _table(formats) -> veda_plan.PlanTable:
    return veda_plan.PlanTable([veda_plan.TilePlan.from_json(p)
                                for p in formats['plans'].values()])


def _digest(t: torch.Tensor) -> str:
    return hashlib.sha256(
        t.detach().contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def test_geometry_rounding_matches_reference(formats):
    for row in formats['geometries']:
        g = veda_geometry.resolve_geometry(row['aspect'], row['seconds'])
        got = {'width': g.width, 'height': g.height,
               'frame_count': g.frame_count, 'latent_t': g.latent_t,
               'latent_h': g.latent_h, 'latent_w': g.latent_w,
               'audio_t': g.audio_t, 'name': g.name,
               'video_grid': list(g.video_grid)}
        want = {k: row[k] for k in got}
        assert got == want, (row['aspect'], row['seconds'])
    assert veda_geometry.latent_t_ladder() == formats['ladder']
    for aspect, err in formats['canvas_errors']:
        w, h = (int(v) for v in aspect.split(':'))
        if err is None:
            veda_geometry.resolve_canvas(w, h)
        else:
            with pytest.raises(ValueError, match='out of range'):
                veda_geometry.resolve_canvas(w, h)
    with pytest.raises(ValueError):
        veda_geometry.frame_count_from_latent_t(38)


def test_plan_json_round_trip(formats):
    for name, data in formats['plans'].items():
        plan = veda_plan.TilePlan.from_json(data)
        assert plan.to_json() == data
        assert plan.geometry == name


def test_plan_mirrored_and_transposed(formats):
    table = _table(formats)
    for name, plan in table.plans.items():
        want = formats['mirrored'][name]
        if 'error' in want:
            with pytest.raises(ValueError):
                plan.mirrored()
        else:
            assert plan.mirrored().to_json() == want
        assert plan.transposed().to_json() == formats['transposed'][name]


def test_plan_table_select_matches_reference(formats):
    table = _table(formats)
    for aspect, lt, want in formats['select']:
        g = veda_geometry.geometry_from_latent_t(aspect, lt)
        if 'error' in want:
            with pytest.raises(KeyError):
                table.select(g)
        else:
            assert table.select(g).to_json() == want, (aspect, lt)


def test_plan_uniform_and_directory(formats, tmp_path):
    g = veda_geometry.geometry_from_latent_t('9:16', 52)
    plan = veda_plan.TilePlan.uniform(
        g, tiling.least_padding_shape(g.video_grid), 2, 3)
    assert plan.to_json() == formats['uniform']
    table = _table(formats)
    for p in table.plans.values():
        p.save(str(tmp_path / f'{p.geometry}.json'))
    again = veda_plan.PlanTable.load_dir(str(tmp_path))
    assert {k: p.to_json() for k, p in again.plans.items()} == \
        {k: p.to_json() for k, p in table.plans.items()}
    with pytest.raises(FileNotFoundError):
        veda_plan.PlanTable.load_dir(str(tmp_path / 'none'))
    with pytest.raises(ValueError, match='at most 2'):
        veda_plan.TilePlan('x', (1, 8, 16), [tiling.TileShape(1, 8, 16),
                                             tiling.TileShape(2, 8, 8),
                                             tiling.TileShape(1, 16, 8)],
                           [[0, 1, 2]])


@pytest.mark.parametrize('tag', ['bf16', 'fp8'])
def test_reference_bundle_loads(formats, tag):
    b = veda_bundle.load(os.path.join(GOLDEN, f'bundle_ref_{tag}.safetensors'))
    state = b.predictor.state_dict()
    want = formats[f'bundle_{tag}_loaded']
    assert set(state) == set(want)
    for k, (dtype, shape, digest) in want.items():
        assert str(state[k].dtype) == dtype and list(state[k].shape) == shape
        assert _digest(state[k]) == digest, k
    assert b.metadata == formats[f'bundle_{tag}_metadata']
    assert b.target_budget == veda_mask.Budget(tiles=12.5)
    assert b.ref_budget == veda_mask.Budget(ratio=0.05)
    assert b.tile_conditions and b.keep_ratio is None
    assert {k: p.to_json() for k, p in b.plans.plans.items()} == \
        formats['plans']


@pytest.mark.parametrize('tag,dtype', [('bf16', torch.bfloat16),
                                       ('fp8', torch.float8_e4m3fn)])
def test_bundle_written_here_matches_reference_file(formats, tmp_path, tag,
                                                    dtype):
    weights = load_file(os.path.join(GOLDEN, 'bundle_weights.safetensors'))
    path = str(tmp_path / 'b.safetensors')
    veda_bundle.save(path, {f'predictor.{k}': v for k, v in weights.items()},
                     _table(formats), num_layers=2, num_heads=3, head_dim=16,
                     keep_tiles=12.5, ref_keep_ratio=0.05,
                     tile_conditions=True, source='fixture',
                     source_weights='live', step=1234, dtype=dtype)
    ref_path = os.path.join(GOLDEN, f'bundle_ref_{tag}.safetensors')
    with safe_open(path, 'pt') as a, safe_open(ref_path, 'pt') as b:
        assert a.metadata() == b.metadata()
        assert sorted(a.keys()) == sorted(b.keys())
        for k in a.keys():
            x, y = a.get_tensor(k), b.get_tensor(k)
            assert x.dtype == y.dtype and _digest(x) == _digest(y), k


def test_bundle_errors(formats, tmp_path):
    weights = load_file(os.path.join(GOLDEN, 'bundle_weights.safetensors'))
    table = _table(formats)
    path = str(tmp_path / 'b.safetensors')
    common = dict(num_layers=2, num_heads=3, head_dim=16, source='s',
                  source_weights='live', step=0)
    with pytest.raises(ValueError, match='no predictor weights'):
        veda_bundle.save(path, {}, table, keep_ratio=0.1, **common)
    with pytest.raises(ValueError, match='exactly one'):
        veda_bundle.save(path, weights, table, **common)
    with pytest.raises(ValueError, match='requires tile_conditions'):
        veda_bundle.save(path, weights, table, keep_ratio=0.1,
                         ref_keep_ratio=0.1, **common)
    with pytest.raises(ValueError, match='requires a reference budget'):
        veda_bundle.save(path, weights, table, keep_ratio=0.1,
                         tile_conditions=True, **common)
    with pytest.raises(ValueError, match='unsupported storage dtype'):
        veda_bundle.save(path, weights, table, keep_ratio=0.1,
                         dtype=torch.float16, **common)
    mixed = dict(weights)
    mixed['predictor.layers.0.proj_q'] = mixed.pop('layers.0.proj_q')
    with pytest.raises(ValueError, match='mix prefixed'):
        veda_bundle.save(path, mixed, table, keep_ratio=0.1, **common)
    with pytest.raises(ValueError, match='without plans'):
        veda_bundle.save(path, weights, veda_plan.PlanTable([]),
                         keep_ratio=0.1, **common)
    # A float32 bundle with a legacy ratio loads as float32.
    veda_bundle.save(path, weights, table, keep_ratio=0.25,
                     dtype=torch.float32, **common)
    b = veda_bundle.load(path)
    assert b.keep_ratio == 0.25 and b.ref_budget is None
    assert all(v.dtype == torch.float32
               for v in b.predictor.state_dict().values())
    # Declared shape differs from the tensors.
    bad = dict(common, num_heads=4)
    veda_bundle.save(path, weights, table, keep_ratio=0.25, **bad)
    with pytest.raises(ValueError, match='do not match'):
        veda_bundle.load(path)
    # Not a bundle.
    from safetensors.torch import save_file
    save_file({'x': torch.zeros(2)}, path, metadata={'format': 'other'})
    with pytest.raises(ValueError, match='not a'):
        veda_bundle.read_metadata(path)


def test_random_bundle_is_uniform_least_padding():
    geos = [veda_geometry.geometry_from_latent_t(a, 37)
            for a in ('16:9', '1:1')]
    b = veda_bundle.random_bundle(2, 4, 128, geos, keep_ratio=0.1, seed=3)
    assert sorted(b.plans.plans) == sorted(g.name for g in geos)
    for g in geos:
        p = b.plans.select(g)
        assert p.shapes == [tiling.least_padding_shape(g.video_grid)]
    assert all(v.dtype == torch.bfloat16
               for v in b.predictor.state_dict().values())
