"""Tile plans: which tile shape every (layer, head) uses on one geometry.

Mirror of the reference's `miowtion/veda/plan.py`: the JSON format of its
released plans (`plans/released/*.json`), the head grouping, the mirrored and
transposed plans and the plan table's selection rule. Plan search itself is
the reference's (`veda/search.py`); plans come from it or are built uniform.
"""

from __future__ import annotations

import dataclasses
import glob
import json
import os
from collections.abc import Sequence

import torch

from miowtion_b200 import geometry as veda_geometry
from miowtion_b200 import tiling


@dataclasses.dataclass(frozen=True)
class HeadGroup:
    """Heads of one layer that share a tile shape (plan.py:28-33)."""

    shape: tiling.TileShape
    heads: torch.Tensor  # [H'] int64


@dataclasses.dataclass
class TilePlan:
    """Per-(layer, head) tile shapes for one geometry (plan.py:36-144)."""

    geometry: str
    grid: tuple[int, int, int]
    shapes: list[tiling.TileShape]
    head_shape: list[list[int]]
    provenance: dict = dataclasses.field(default_factory=dict)

    def __post_init__(self):
        for layer, row in enumerate(self.head_shape):
            if len(set(row)) > 2:
                raise ValueError(f'layer {layer} uses {len(set(row))} shapes; '
                                 'at most 2 per layer are allowed')
        self._groups = {}

    @property
    def num_layers(self) -> int:
        return len(self.head_shape)

    def layer_shapes(self, layer: int) -> list[tiling.TileShape]:
        return [self.shapes[i] for i in sorted(set(self.head_shape[layer]))]

    def head_groups(self, layer: int,
                    device: torch.device | str) -> list[HeadGroup]:
        """Groups of heads sharing a shape (cached per layer and device)."""
        key = (layer, str(device))
        if key not in self._groups:
            row = torch.tensor(self.head_shape[layer])
            self._groups[key] = [
                HeadGroup(self.shapes[i],
                          torch.nonzero(row == i).view(-1).to(device))
                for i in sorted(set(self.head_shape[layer]))]
        return self._groups[key]

    def to_json(self) -> dict:
        return {'geometry': self.geometry, 'grid': list(self.grid),
                'shapes': [str(s) for s in self.shapes],
                'head_shape': self.head_shape,
                'provenance': self.provenance}

    @classmethod
    def from_json(cls, data: dict) -> TilePlan:
        return cls(geometry=data['geometry'], grid=tuple(data['grid']),
                   shapes=[tiling.TileShape.parse(s) for s in data['shapes']],
                   head_shape=[list(r) for r in data['head_shape']],
                   provenance=data.get('provenance', {}))

    def save(self, path: str) -> None:
        tmp = path + '.tmp'
        with open(tmp, 'w') as f:
            json.dump(self.to_json(), f, indent=1)
        os.replace(tmp, path)

    @classmethod
    def load(cls, path: str) -> TilePlan:
        with open(path) as f:
            return cls.from_json(json.load(f))

    @classmethod
    def uniform(cls, geometry: veda_geometry.Geometry,
                shape: tiling.TileShape, num_layers: int,
                num_heads: int) -> TilePlan:
        """Every head uses one shape (plan.py:108-114)."""
        return cls(geometry.name, tuple(geometry.video_grid), [shape],
                   [[0] * num_heads for _ in range(num_layers)],
                   {'source': 'uniform'})

    def mirrored(self) -> TilePlan:
        """The plan of the H<->W mirrored geometry (plan.py:116-138), e.g.
        9x16_t37 from 16x9_t37: shapes and grid transposed, the mirrored
        geometry's name, `mirrored_from` added to the provenance.

        Raises:
            ValueError: If the mirrored geometry's grid is not this grid
                transposed (the canvas rounding differs).
        """
        aspect, latent_t = self.geometry.split('_t')
        w, h = aspect.split('x')
        mirror = veda_geometry.geometry_from_latent_t(f'{h}:{w}',
                                                      int(latent_t))
        t, grid_h, grid_w = self.grid
        if tuple(mirror.video_grid) != (t, grid_w, grid_h):
            raise ValueError(f'{mirror.name} grid {mirror.video_grid} is not '
                             f'the transpose of {self.geometry} {self.grid}')
        return TilePlan(mirror.name, (t, grid_w, grid_h),
                        [s.transposed() for s in self.shapes],
                        [list(r) for r in self.head_shape],
                        {**self.provenance, 'mirrored_from': self.geometry})

    def transposed(self) -> TilePlan:
        """H<->W transposed plan named '<geometry>_T' (plan.py:140-146)."""
        t, h, w = self.grid
        return TilePlan(self.geometry + '_T', (t, w, h),
                        [s.transposed() for s in self.shapes],
                        [list(r) for r in self.head_shape],
                        {**self.provenance, 'transposed_from': self.geometry})


class PlanTable:
    """All searched plans, keyed by geometry name (plan.py:149-188)."""

    def __init__(self, plans: Sequence[TilePlan]):
        self.plans = {p.geometry: p for p in plans}

    @classmethod
    def load_dir(cls, directory: str) -> PlanTable:
        """Every `*.json` plan of a directory, in name order.

        Raises:
            FileNotFoundError: If the directory holds no plan.
        """
        paths = sorted(glob.glob(os.path.join(directory, '*.json')))
        if not paths:
            raise FileNotFoundError(f'no plans in {directory}')
        return cls([TilePlan.load(p) for p in paths])

    def select(self, geometry: veda_geometry.Geometry) -> TilePlan:
        """The plan for a geometry, by the reference's rule (plan.py:160-188):

        1. the geometry's own plan, if searched;
        2. else the plan of the same aspect with the nearest latent_t (ties
           to the shorter one; no interpolation);
        3. else, only when no plan of this aspect exists, the mirrored
           aspect's nearest plan or its transpose, whichever pads the
           target grid less (the untransposed one on a tie).

        Raises:
            KeyError: If neither this aspect nor its mirror has a plan.
        """
        if geometry.name in self.plans:
            return self.plans[geometry.name]

        def aspect_of(p: TilePlan) -> str:
            return p.geometry.split('_t')[0]

        key = geometry.aspect.replace(':', 'x')
        same = [p for p in self.plans.values() if aspect_of(p) == key]
        if same:
            return min(same, key=lambda p: (abs(p.grid[0] - geometry.latent_t),
                                            p.grid[0]))
        w, h = geometry.aspect.split(':')
        mirror = [p for p in self.plans.values()
                  if aspect_of(p) == f'{h}x{w}']
        if not mirror:
            raise KeyError(f'no plan for {geometry.name}')
        nearest = min(mirror, key=lambda p: abs(p.grid[0] - geometry.latent_t))
        grid = geometry.video_grid

        def padded_tiles(p: TilePlan) -> int:
            return sum(s.num_tiles(grid) for s in p.shapes)

        return min((nearest, nearest.transposed()), key=padded_tiles)
