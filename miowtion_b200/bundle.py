"""Predictor bundle: one safetensors file holding the predictor's weights and
the tile plans it was trained against.

File format `miowtion-veda-predictor-v1` (the reference's exporter,
miowtion/veda/bundle.py), so files move both ways between the two:

Tensors. The predictor's state dict under bare keys (`layers.{i}.proj_q`,
`layers.{i}.proj_k`, ...), all stored in one dtype: float32, bfloat16 or
float8_e4m3fn. A float8 tensor `name` is stored as e4m3 values of
`weight / scale` and travels with `name.__scale`, float32 [H]: per leading
index (head), max |weight| / 448 (448 = largest finite e4m3), never below
the smallest normal float32.

String metadata. `format`; `num_layers`, `num_heads`, `head_dim`,
`second_order_rank` (decimal integers); `count_term` ('1' / '0');
`tile_conditions` ('true' / 'false'); `dtype` (the storage dtype's name;
missing in old files, which are float32); `source`, `source_weights`,
`step`; `plans`, one JSON object mapping each geometry name (sorted) to its
plan's JSON; the budgets as `<p>_budget_kind` ('ratio' / 'tiles') and
`<p>_budget_value` (Python repr of a float) for p = 'target' and, with
tiled conditioning references, p = 'ref'; `keep_ratio` repeats a ratio
target budget (older readers know only that key).

Loading is strict: the tensors must fill exactly the parameters of the
predictor the metadata describes. float8 and bfloat16 files load as
bfloat16 parameters, float32 files as float32 (the scoring kernels read
fp32 whatever the parameter dtype).
"""

from __future__ import annotations

import dataclasses
import json
from collections.abc import Mapping, Sequence

import torch
from safetensors import safe_open
from safetensors.torch import save_file

from miowtion_b200 import geometry as veda_geometry
from miowtion_b200 import mask as veda_mask
from miowtion_b200 import plan as veda_plan
from miowtion_b200 import predictor as veda_predictor
from miowtion_b200 import tiling

FORMAT = 'miowtion-veda-predictor-v1'

DTYPES = {'float32': torch.float32, 'bfloat16': torch.bfloat16,
          'float8_e4m3fn': torch.float8_e4m3fn}
_DTYPE_NAMES = {dt: name for name, dt in DTYPES.items()}

_TRAINER_PREFIX = 'predictor.'  # how a training checkpoint names them
_SCALE = '.__scale'
_E4M3_LARGEST = 448.0


# -- tensor codecs -------------------------------------------------------

def _per_head(scale: torch.Tensor, like: torch.Tensor) -> torch.Tensor:
    """[H] -> broadcastable against [H, ...]."""
    return scale.reshape((-1,) + (1,) * (like.dim() - 1))


def _encode(weights: Mapping[str, torch.Tensor],
            dtype: torch.dtype) -> dict[str, torch.Tensor]:
    """Parameters -> the tensors stored for them in `dtype`."""
    stored = {}
    for name, weight in weights.items():
        w = weight.detach()
        if dtype is not torch.float8_e4m3fn:
            stored[name] = w.to(dtype).contiguous()
            continue
        w = w.float()
        amax = w.abs().flatten(1).amax(1) if w.dim() > 1 else w.abs()
        scale = (amax / _E4M3_LARGEST).clamp_min(
            torch.finfo(torch.float32).tiny)
        stored[name] = (w / _per_head(scale, w)).to(dtype).contiguous()
        stored[name + _SCALE] = scale.contiguous()
    return stored


def _decode(stored: Mapping[str, torch.Tensor], dtype: torch.dtype,
            where: str) -> tuple[dict[str, torch.Tensor], torch.dtype]:
    """Stored tensors -> (parameters, the dtype they load as)."""
    if dtype is not torch.float8_e4m3fn:
        return dict(stored), dtype
    params = {}
    missing = []
    for name, values in stored.items():
        if name.endswith(_SCALE):
            continue
        scale = stored.get(name + _SCALE)
        if scale is None:
            missing.append(name)
            continue
        params[name] = (values.float() * _per_head(scale, values)).to(
            torch.bfloat16)
    if missing:
        raise ValueError(f'{where}: fp8 tensors without a {_SCALE} scale: '
                         f'{sorted(missing)}')
    return params, torch.bfloat16


# -- budgets in the metadata ---------------------------------------------

def _budget_fields(which: str, ratio: float | None,
                   tiles: float | None) -> dict[str, str]:
    given = [(kind, val) for kind, val in (('ratio', ratio),
                                           ('tiles', tiles))
             if val is not None]
    if len(given) != 1:
        raise ValueError(f'set exactly one of {which}_ratio / '
                         f'{which}_tiles')
    kind, value = given[0]
    veda_mask.Budget(**{kind: value})  # rejects out-of-range values
    return {f'{which}_budget_kind': kind,
            f'{which}_budget_value': repr(float(value))}


def _budget_from(meta: Mapping[str, str],
                 which: str) -> veda_mask.Budget | None:
    kind = meta.get(f'{which}_budget_kind')
    if kind is None:
        return None
    value = meta.get(f'{which}_budget_value')
    if kind not in ('ratio', 'tiles') or value is None:
        raise ValueError(f'invalid {which} budget metadata: kind={kind!r}, '
                         f'value={value!r}')
    return veda_mask.Budget(**{kind: float(value)})


# -- the bundle ------------------------------------------------------------

@dataclasses.dataclass
class Bundle:
    """A loaded bundle."""

    predictor: veda_predictor.TileScorePredictor
    plans: veda_plan.PlanTable
    target_budget: veda_mask.Budget
    ref_budget: veda_mask.Budget | None
    tile_conditions: bool
    keep_ratio: float | None
    metadata: dict[str, str]


def _bare_keys(weights: Mapping[str, torch.Tensor]
               ) -> dict[str, torch.Tensor]:
    """Drops the trainer's 'predictor.' prefix (all keys or none)."""
    flags = {k.startswith(_TRAINER_PREFIX) for k in weights}
    if len(flags) > 1:
        raise ValueError('weights mix prefixed and bare keys')
    if flags == {True}:
        return {k[len(_TRAINER_PREFIX):]: v for k, v in weights.items()}
    return dict(weights)


def save(path: str, weights: dict[str, torch.Tensor],
         plans: veda_plan.PlanTable, *, num_layers: int, num_heads: int,
         head_dim: int, keep_ratio: float | None = None,
         keep_tiles: float | None = None,
         ref_keep_ratio: float | None = None,
         ref_keep_tiles: float | None = None,
         tile_conditions: bool = False, source: str,
         source_weights: str, step: int,
         dtype: torch.dtype = torch.bfloat16,
         second_order_rank: int = 0, count_term: bool = False) -> None:
    """Writes a bundle. Exactly one target budget (`keep_ratio` or
    `keep_tiles`); a reference budget exactly when `tile_conditions`.

    Raises:
        ValueError: No weights, prefixed and bare keys mixed, a storage
            dtype outside DTYPES, an empty plan table, or budgets that break
            the rules above.
    """
    if not weights:
        raise ValueError('no predictor weights to save')
    meta = _budget_fields('target', keep_ratio, keep_tiles)
    with_ref = (ref_keep_ratio, ref_keep_tiles) != (None, None)
    if with_ref != tile_conditions:
        raise ValueError('a reference budget requires tile_conditions'
                         if with_ref else
                         'tile_conditions requires a reference budget')
    if with_ref:
        meta.update(_budget_fields('ref', ref_keep_ratio, ref_keep_tiles))
    if dtype not in _DTYPE_NAMES:
        raise ValueError(f'unsupported storage dtype {dtype}; expected one '
                         f'of {sorted(DTYPES)}')
    params = _bare_keys(weights)
    if not plans.plans:
        raise ValueError('bundle without plans; pass the run\'s plan table')
    meta.update(
        format=FORMAT, num_layers=str(num_layers), num_heads=str(num_heads),
        head_dim=str(head_dim), dtype=_DTYPE_NAMES[dtype],
        tile_conditions=str(bool(tile_conditions)).lower(), source=source,
        source_weights=source_weights, step=str(step),
        second_order_rank=str(second_order_rank),
        count_term=str(int(bool(count_term))),
        plans=json.dumps({g: plans.plans[g].to_json()
                          for g in sorted(plans.plans)}))
    if keep_ratio is not None:
        meta['keep_ratio'] = repr(float(keep_ratio))
    stored = _encode(params, dtype)
    save_file({k: v.cpu() for k, v in stored.items()}, path, metadata=meta)


def read_metadata(path: str) -> dict[str, str]:
    """The string metadata alone (no tensor is read).

    Raises:
        ValueError: If the file is not a bundle of this format.
    """
    with safe_open(path, framework='pt', device='cpu') as f:
        meta = dict(f.metadata() or {})
    if meta.get('format') != FORMAT:
        raise ValueError(f'{path}: not a {FORMAT} bundle (format '
                         f'{meta.get("format")!r})')
    return meta


def load(path: str, device: torch.device | str = 'cpu') -> Bundle:
    """Loads a bundle strictly.

    Raises:
        ValueError: Not a bundle of this format, an unknown storage dtype,
            an fp8 tensor without its scale, tensors that do not fill the
            declared predictor exactly, no target budget, or tiled
            references without a reference budget.
    """
    meta = read_metadata(path)
    dtype_name = meta.get('dtype', 'float32')
    if dtype_name not in DTYPES:
        raise ValueError(f'{path}: unknown storage dtype {dtype_name!r}')
    with safe_open(path, framework='pt', device='cpu') as f:
        stored = {k: f.get_tensor(k) for k in f.keys()}
    params, param_dtype = _decode(stored, DTYPES[dtype_name], path)
    shape = (int(meta['num_layers']), int(meta['num_heads']),
             int(meta['head_dim']))
    # Parameters take the stored precision before the state is copied in,
    # so a bf16 file never sits in fp32 parameters.
    predictor = veda_predictor.TileScorePredictor(
        *shape, second_order_rank=int(meta.get('second_order_rank', 0)),
        count_term=meta.get('count_term', '0') == '1').to(param_dtype)
    try:
        predictor.load_state_dict(params, strict=True)
    except RuntimeError as err:
        raise ValueError(
            f'{path}: predictor weights do not match the {shape[0]} layers '
            f'x {shape[1]} heads x {shape[2]} the metadata declares: '
            f'{err}') from err
    target = _budget_from(meta, 'target')
    if target is None and 'keep_ratio' in meta:
        target = veda_mask.Budget(ratio=float(meta['keep_ratio']))
    if target is None:
        raise ValueError(f'{path}: bundle has no target budget')
    ref = _budget_from(meta, 'ref')
    tiled_refs = meta.get('tile_conditions', 'false') == 'true'
    if tiled_refs and ref is None:
        raise ValueError(f'{path}: tiled references need a ref budget')
    table = veda_plan.PlanTable(veda_plan.TilePlan.from_json(p)
                                for p in json.loads(meta['plans']).values())
    return Bundle(predictor.to(device).eval(), table, target, ref,
                  tiled_refs, target.ratio, meta)


def random_bundle(num_layers: int, num_heads: int, head_dim: int,
                  geometries: Sequence[veda_geometry.Geometry],
                  keep_ratio: float, seed: int = 0,
                  device: torch.device | str = 'cpu') -> Bundle:
    """A bf16 predictor with weights drawn from N(0, INIT_STD) by a
    generator seeded with `seed`, and one uniform least-padding plan per
    geometry: a stand-in for benchmarks, whose cost depends on the budget
    and the tile shapes rather than on the scores."""
    predictor = veda_predictor.TileScorePredictor(num_layers, num_heads,
                                                  head_dim)
    gen = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for param in predictor.parameters():
            param.copy_(torch.randn(param.shape, generator=gen) *
                        veda_predictor.INIT_STD)
    table = veda_plan.PlanTable(
        veda_plan.TilePlan.uniform(g, tiling.least_padding_shape(
            g.video_grid), num_layers, num_heads) for g in geometries)
    return Bundle(predictor.to(device, torch.bfloat16).eval(), table,
                  veda_mask.Budget(ratio=keep_ratio), None, False,
                  keep_ratio, {'source': 'random', 'seed': str(seed)})
