"""Tile plans: which tile shape every (layer, head) uses on one geometry.

Mirror of the reference's `miowtion/veda/plan.py` data format (the JSON of
`plans/**.json`) and its head grouping. Plan search is out of scope here;
plans come from the reference's search or are built uniform.
"""

from __future__ import annotations

import dataclasses
import json
import os

import torch

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
    def uniform(cls, geometry: str, grid: tuple[int, int, int],
                shape: tiling.TileShape, num_layers: int,
                num_heads: int) -> TilePlan:
        """Every head uses one shape (baseline / bootstrap plan)."""
        return cls(geometry, tuple(grid), [shape],
                   [[0] * num_heads for _ in range(num_layers)],
                   {'source': 'uniform'})
