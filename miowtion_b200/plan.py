"""Tile plans: the tile shape each (layer, head) uses on one video geometry.

A plan is stored as one JSON object, the format of the reference's released
plans (miowtion/veda/plan.py:81-106, plans/released/*.json):

    geometry    geometry name "<W>x<H>_t<latent frames>", e.g. "16x9_t37"
    grid        [t, h, w], the latent video grid of that geometry
    shapes      the tile shapes in use, as "<t>x<h>x<w>" strings (128 tokens)
    head_shape  per layer, per head: an index into `shapes`
    provenance  a free-form object (search settings, derivations)

Rules this module enforces or implements (same behaviour as the reference):

- a layer uses at most two distinct shapes (each shape is one group of
  heads, one launch of the attention kernels);
- the heads of a layer form one group per shape, groups in the order of the
  shape index, heads ascending inside a group (plan.py:28-33, :68-79);
- H<->W symmetry: the plan of geometry "WxH_tN" serves "HxW_tN" with every
  tile shape and the grid transposed. `mirrored()` names the result after the
  mirrored geometry and requires its grid to be the exact transpose (canvas
  rounding may break the symmetry); `transposed()` keeps the name with a
  "_T" suffix and requires nothing;
- selecting a plan for a geometry (PlanTable.select): an exact name match;
  otherwise the nearest latent_t of the same aspect (ties to the shorter
  clip); otherwise, when the aspect has no plan at all, the nearest plan of
  the mirrored aspect or its transpose, whichever needs fewer padded tiles
  on this grid (the untransposed one on a tie). Plans are never
  interpolated.
"""

from __future__ import annotations

import dataclasses
import json
import os
import pathlib
from collections.abc import Iterable

import torch

from miowtion_b200 import geometry as veda_geometry
from miowtion_b200 import tiling

MAX_SHAPES_PER_LAYER = 2


@dataclasses.dataclass(frozen=True)
class HeadGroup:
    """The heads of one layer that share a tile shape."""

    shape: tiling.TileShape
    heads: torch.Tensor  # [H'] int64, ascending


def _aspect_key(geometry_name: str) -> str:
    """'16x9_t37' -> '16x9'."""
    return geometry_name.partition('_t')[0]


def _latent_t(plan: 'TilePlan') -> int:
    return plan.grid[0]


@dataclasses.dataclass
class TilePlan:
    """Tile shapes of every (layer, head) for one geometry."""

    geometry: str
    grid: tuple[int, int, int]
    shapes: list[tiling.TileShape]
    head_shape: list[list[int]]
    provenance: dict = dataclasses.field(default_factory=dict)

    def __post_init__(self):
        self.grid = tuple(int(g) for g in self.grid)
        for layer, row in enumerate(self.head_shape):
            distinct = len(set(row))
            if distinct > MAX_SHAPES_PER_LAYER:
                raise ValueError(
                    f'layer {layer} mixes {distinct} tile shapes; a layer '
                    f'may use at most {MAX_SHAPES_PER_LAYER}')
        self._group_cache: dict = {}

    # -- queries -----------------------------------------------------------

    @property
    def num_layers(self) -> int:
        return len(self.head_shape)

    def _shape_ids(self, layer: int) -> list[int]:
        return sorted(set(self.head_shape[layer]))

    def layer_shapes(self, layer: int) -> list[tiling.TileShape]:
        """The shapes layer `layer` uses, by shape index."""
        return [self.shapes[i] for i in self._shape_ids(layer)]

    def head_groups(self, layer: int,
                    device: torch.device | str) -> list[HeadGroup]:
        """One group per shape of the layer, built once per device."""
        key = (layer, str(device))
        groups = self._group_cache.get(key)
        if groups is None:
            row = self.head_shape[layer]
            groups = []
            for sid in self._shape_ids(layer):
                members = [h for h, s in enumerate(row) if s == sid]
                groups.append(HeadGroup(
                    self.shapes[sid],
                    torch.tensor(members, dtype=torch.int64, device=device)))
            self._group_cache[key] = groups
        return groups

    # -- JSON --------------------------------------------------------------

    def to_json(self) -> dict:
        return dict(geometry=self.geometry, grid=list(self.grid),
                    shapes=[str(s) for s in self.shapes],
                    head_shape=[list(r) for r in self.head_shape],
                    provenance=self.provenance)

    @classmethod
    def from_json(cls, data: dict) -> 'TilePlan':
        return cls(data['geometry'], tuple(data['grid']),
                   [tiling.TileShape.parse(s) for s in data['shapes']],
                   [list(r) for r in data['head_shape']],
                   data.get('provenance', {}))

    def save(self, path: str) -> None:
        """Writes the JSON next to `path` first, then renames it into place,
        so a reader never sees a half-written plan."""
        target = pathlib.Path(path)
        partial = target.with_name(target.name + '.tmp')
        partial.write_text(json.dumps(self.to_json(), indent=1))
        os.replace(partial, target)

    @classmethod
    def load(cls, path: str) -> 'TilePlan':
        return cls.from_json(json.loads(pathlib.Path(path).read_text()))

    # -- derived plans -----------------------------------------------------

    @classmethod
    def uniform(cls, geometry: veda_geometry.Geometry,
                shape: tiling.TileShape, num_layers: int,
                num_heads: int) -> 'TilePlan':
        """Every head of every layer on one shape."""
        rows = [[0] * num_heads for _ in range(num_layers)]
        return cls(geometry.name, tuple(geometry.video_grid), [shape], rows,
                   {'source': 'uniform'})

    def _hw_swapped(self, name: str, note: str) -> 'TilePlan':
        """This plan with H and W exchanged in the grid and every shape,
        under `name`, recording this plan's name as provenance[note]."""
        t, h, w = self.grid
        return TilePlan(name, (t, w, h),
                        [s.transposed() for s in self.shapes],
                        [list(r) for r in self.head_shape],
                        {**self.provenance, note: self.geometry})

    def mirrored(self) -> 'TilePlan':
        """The plan of the H<->W mirrored geometry ('9x16_t37' for
        '16x9_t37').

        Raises:
            ValueError: If the mirrored geometry's grid is not this grid
                transposed.
        """
        aspect, _, latent_t = self.geometry.partition('_t')
        width, _, height = aspect.partition('x')
        other = veda_geometry.geometry_from_latent_t(f'{height}:{width}',
                                                     int(latent_t))
        swapped = self._hw_swapped(other.name, 'mirrored_from')
        if tuple(other.video_grid) != swapped.grid:
            raise ValueError(
                f'{other.name} has grid {tuple(other.video_grid)}, not the '
                f'transpose of {self.geometry}\'s {self.grid}')
        return swapped

    def transposed(self) -> 'TilePlan':
        """The H<->W transpose, named '<geometry>_T'."""
        return self._hw_swapped(self.geometry + '_T', 'transposed_from')


class PlanTable:
    """Searched plans by geometry name, with the selection rule above."""

    def __init__(self, plans: Iterable[TilePlan]):
        self.plans = {p.geometry: p for p in plans}

    @classmethod
    def load_dir(cls, directory: str) -> 'PlanTable':
        """Every '*.json' plan in a directory, in file-name order.

        Raises:
            FileNotFoundError: If the directory holds no plan.
        """
        files = sorted(pathlib.Path(directory).glob('*.json'))
        if not files:
            raise FileNotFoundError(f'no plans in {directory}')
        return cls(TilePlan.load(str(f)) for f in files)

    def _of_aspect(self, key: str) -> list[TilePlan]:
        return [p for p in self.plans.values()
                if _aspect_key(p.geometry) == key]

    def select(self, geometry: veda_geometry.Geometry) -> TilePlan:
        """The plan serving `geometry`.

        Raises:
            KeyError: If neither the aspect nor its mirror has a plan.
        """
        exact = self.plans.get(geometry.name)
        if exact is not None:
            return exact
        width, _, height = geometry.aspect.partition(':')
        want_t = geometry.latent_t

        own = self._of_aspect(f'{width}x{height}')
        if own:
            # Nearest clip length; the shorter clip wins a tie.
            return min(own, key=lambda p: (abs(_latent_t(p) - want_t),
                                           _latent_t(p)))
        flipped = self._of_aspect(f'{height}x{width}')
        if not flipped:
            raise KeyError(f'no plan for {geometry.name}')
        base = min(flipped, key=lambda p: abs(_latent_t(p) - want_t))
        grid = geometry.video_grid
        candidates = (base, base.transposed())  # a tie keeps `base`
        return min(candidates,
                   key=lambda p: sum(s.num_tiles(grid) for s in p.shapes))
