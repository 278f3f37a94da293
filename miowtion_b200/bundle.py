"""Predictor bundle: one safetensors file with the live predictor weights and
every tile plan the predictor was trained against.

The on-disk format is the reference's `miowtion-veda-predictor-v1`
(`miowtion/veda/bundle.py:1-330`), so a bundle exported by the reference
loads here and one written here loads there:

- tensors: the predictor's state dict with bare keys (`layers.{i}.proj_q`,
  `layers.{i}.proj_k`), stored as float32, bfloat16 or float8_e4m3fn;
- an fp8 tensor `name` carries `name.__scale`, fp32 [H]: per head, amax
  divided by 448 (the largest finite e4m3 value), at least the smallest
  normal float32, with weight ~= value * scale;
- `__metadata__` (str -> str): `format`, `num_layers`, `num_heads`,
  `head_dim`, `dtype`, `tile_conditions` ('true' / 'false'), `source`,
  `source_weights`, `step`, `second_order_rank`, `count_term` ('1' / '0'),
  `plans` (one JSON object, geometry name -> plan JSON, in name order),
  `target_budget_kind` / `target_budget_value` ('ratio' or 'tiles', the
  value as Python's repr of a float), optionally `ref_budget_kind` /
  `ref_budget_value`, and the legacy `keep_ratio` for ratio budgets.

Loading is strict: every stored tensor must land on a parameter of the
predictor the metadata describes. fp8 and bf16 bundles come back as bf16
parameters (the scoring kernel reads them as fp32 whatever they are stored
in); float32 bundles stay float32.
"""

from __future__ import annotations

import dataclasses
import json
from collections.abc import Sequence

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

_PREFIX = 'predictor.'
_SCALE_SUFFIX = '.__scale'
_E4M3_MAX = 448.0
# A bundle without a `dtype` key predates it and holds float32 tensors.
_LEGACY_DTYPE = 'float32'


def _quantize_fp8(weight: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """[H, ...] weights -> (e4m3 values, fp32 per-head scale) with
    weight ~= values * scale (bundle.py:69-85)."""
    w = weight.float()
    reduce_dims = tuple(range(1, w.dim()))
    scale = (w.abs().amax(dim=reduce_dims) / _E4M3_MAX).clamp(
        min=torch.finfo(torch.float32).tiny)
    shaped = scale.view(-1, *([1] * len(reduce_dims)))
    return (w / shaped).to(torch.float8_e4m3fn).contiguous(), \
        scale.contiguous()


def _dequantize_fp8(values: torch.Tensor, scale: torch.Tensor,
                    dtype: torch.dtype) -> torch.Tensor:
    shaped = scale.view(-1, *([1] * (values.dim() - 1)))
    return (values.float() * shaped).to(dtype)


@dataclasses.dataclass
class Bundle:
    """A loaded bundle (bundle.py:96-120)."""

    predictor: veda_predictor.TileScorePredictor
    plans: veda_plan.PlanTable
    target_budget: veda_mask.Budget
    ref_budget: veda_mask.Budget | None
    tile_conditions: bool
    keep_ratio: float | None
    metadata: dict[str, str]


def _budget_entries(prefix: str, ratio: float | None,
                    tiles: float | None) -> dict[str, str]:
    if (ratio is None) == (tiles is None):
        raise ValueError(f'set exactly one of {prefix}_ratio / {prefix}_tiles')
    kind, value = ('tiles', tiles) if tiles is not None else ('ratio', ratio)
    veda_mask.Budget(**{kind: value})  # validates the value
    return {f'{prefix}_budget_kind': kind,
            f'{prefix}_budget_value': repr(float(value))}


def _parse_budget(metadata: dict[str, str], prefix: str,
                  legacy_ratio: str | None = None) -> veda_mask.Budget | None:
    kind = metadata.get(f'{prefix}_budget_kind')
    value = metadata.get(f'{prefix}_budget_value')
    if kind is None:
        if legacy_ratio is not None and legacy_ratio in metadata:
            return veda_mask.Budget(ratio=float(metadata[legacy_ratio]))
        return None
    if kind not in ('ratio', 'tiles') or value is None:
        raise ValueError(f'invalid {prefix} budget metadata: kind={kind!r}, '
                         f'value={value!r}')
    return veda_mask.Budget(**{kind: float(value)})


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
    """Writes a bundle (bundle.py:151-249); same arguments and errors.

    Raises:
        ValueError: No weights, prefixed and bare keys mixed, an unsupported
            storage dtype, no plans, a budget given twice or not at all, or a
            reference budget without `tile_conditions` (and the converse).
    """
    if not weights:
        raise ValueError('no predictor weights to save')
    metadata_budgets = _budget_entries('target', keep_ratio, keep_tiles)
    has_ref = ref_keep_ratio is not None or ref_keep_tiles is not None
    if has_ref and not tile_conditions:
        raise ValueError('a reference budget requires tile_conditions')
    if tile_conditions and not has_ref:
        raise ValueError('tile_conditions requires a reference budget')
    if has_ref:
        metadata_budgets.update(
            _budget_entries('ref', ref_keep_ratio, ref_keep_tiles))
    dtype_name = {v: k for k, v in DTYPES.items()}.get(dtype)
    if dtype_name is None:
        raise ValueError(f'unsupported storage dtype {dtype}; '
                         f'expected one of {sorted(DTYPES)}')
    n_prefixed = sum(k.startswith(_PREFIX) for k in weights)
    if n_prefixed and n_prefixed != len(weights):
        raise ValueError('weights mix prefixed and bare keys')
    bare = {(k[len(_PREFIX):] if n_prefixed else k): v
            for k, v in weights.items()}
    tensors = {}
    for key, value in bare.items():
        if dtype is torch.float8_e4m3fn:
            tensors[key], tensors[key + _SCALE_SUFFIX] = _quantize_fp8(value)
        else:
            tensors[key] = value.detach().to(dtype).contiguous()
    if not plans.plans:
        raise ValueError('bundle without plans; pass the run\'s plan table')
    metadata = {
        'format': FORMAT,
        'num_layers': str(num_layers),
        'num_heads': str(num_heads),
        'head_dim': str(head_dim),
        'dtype': dtype_name,
        'tile_conditions': 'true' if tile_conditions else 'false',
        'source': source,
        'source_weights': source_weights,
        'step': str(step),
        'second_order_rank': str(second_order_rank),
        'count_term': '1' if count_term else '0',
        'plans': json.dumps({name: plans.plans[name].to_json()
                             for name in sorted(plans.plans)}),
    }
    metadata.update(metadata_budgets)
    if keep_ratio is not None:
        metadata['keep_ratio'] = repr(float(keep_ratio))
    save_file({k: v.cpu() for k, v in tensors.items()}, path,
              metadata=metadata)


def read_metadata(path: str) -> dict[str, str]:
    """The string metadata alone, no tensor read (bundle.py:252-263).

    Raises:
        ValueError: If the file is not a bundle of this format.
    """
    with safe_open(path, framework='pt', device='cpu') as f:
        metadata = dict(f.metadata() or {})
    if metadata.get('format') != FORMAT:
        raise ValueError(f'{path}: not a {FORMAT} bundle '
                         f'(format {metadata.get("format")!r})')
    return metadata


def load(path: str, device: torch.device | str = 'cpu') -> Bundle:
    """Loads a bundle strictly (bundle.py:266-330).

    Raises:
        ValueError: Not a bundle of this format, an unknown storage dtype, an
            fp8 tensor without its scale, tensors that do not match the
            predictor the metadata declares, no target budget, or tiled
            references without a reference budget.
        NotImplementedError: A predictor with a second-order head or a count
            term (no B200 scoring kernel for those).
    """
    metadata = read_metadata(path)
    with safe_open(path, framework='pt', device='cpu') as f:
        tensors = {k: f.get_tensor(k) for k in f.keys()}
    stored = metadata.get('dtype', _LEGACY_DTYPE)
    if stored not in DTYPES:
        raise ValueError(f'{path}: unknown storage dtype {stored!r}')
    model = veda_predictor.TileScorePredictor(
        int(metadata['num_layers']), int(metadata['num_heads']),
        int(metadata['head_dim']),
        second_order_rank=int(metadata.get('second_order_rank', 0)),
        count_term=metadata.get('count_term', '0') == '1')
    resident = DTYPES[stored]
    if resident is torch.float8_e4m3fn:
        resident = torch.bfloat16
        scales = {k[:-len(_SCALE_SUFFIX)]: v for k, v in tensors.items()
                  if k.endswith(_SCALE_SUFFIX)}
        values = {k: v for k, v in tensors.items()
                  if not k.endswith(_SCALE_SUFFIX)}
        unscaled = sorted(set(values) - set(scales))
        if unscaled:
            raise ValueError(f'{path}: fp8 tensors without a '
                             f'{_SCALE_SUFFIX} scale: {unscaled}')
        tensors = {k: _dequantize_fp8(v, scales[k], resident)
                   for k, v in values.items()}
    # Cast the module first: loading into fp32 parameters would upcast a
    # bf16 file and hold twice the memory it was exported to save.
    model = model.to(resident)
    declared = (f'{metadata["num_layers"]} layers x {metadata["num_heads"]} '
                f'heads x {metadata["head_dim"]}')
    try:
        model.load_state_dict(tensors, strict=True)
    except RuntimeError as error:
        raise ValueError(f'{path}: predictor weights do not match the '
                         f'{declared} the metadata declares: {error}') from error
    plans = veda_plan.PlanTable(
        [veda_plan.TilePlan.from_json(p)
         for p in json.loads(metadata['plans']).values()])
    target = _parse_budget(metadata, 'target', legacy_ratio='keep_ratio')
    if target is None:
        raise ValueError(f'{path}: bundle has no target budget')
    ref = _parse_budget(metadata, 'ref')
    tile_conditions = metadata.get('tile_conditions', 'false') == 'true'
    if tile_conditions and ref is None:
        raise ValueError(f'{path}: tiled references need a ref budget')
    return Bundle(predictor=model.to(device).eval(), plans=plans,
                  target_budget=target, ref_budget=ref,
                  tile_conditions=tile_conditions, keep_ratio=target.ratio,
                  metadata=metadata)


def random_bundle(num_layers: int, num_heads: int, head_dim: int,
                  geometries: Sequence[veda_geometry.Geometry],
                  keep_ratio: float, seed: int = 0,
                  device: torch.device | str = 'cpu') -> Bundle:
    """A randomly initialised bf16 predictor with a uniform least-padding
    plan per geometry, for benchmarks (bundle.py:333-369). The cost of a
    Veda step depends on the budget and the tile shapes, not on the scores."""
    with torch.random.fork_rng(devices=[]):
        torch.manual_seed(seed)
        predictor = veda_predictor.TileScorePredictor(num_layers, num_heads,
                                                      head_dim)
    plans = veda_plan.PlanTable([
        veda_plan.TilePlan.uniform(
            g, tiling.least_padding_shape(g.video_grid), num_layers,
            num_heads) for g in geometries])
    return Bundle(predictor=predictor.to(device, torch.bfloat16).eval(),
                  plans=plans, target_budget=veda_mask.Budget(ratio=keep_ratio),
                  ref_budget=None, tile_conditions=False,
                  keep_ratio=keep_ratio,
                  metadata={'source': 'random', 'seed': str(seed)})
