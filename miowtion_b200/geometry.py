"""Request geometry: pixel canvas, frame count and the token grid.

A tile plan is valid only for the exact token grid a request produces, so the
rounding rules that turn (aspect, duration) into a grid are part of the plan
format. These follow the reference's `miowtion/h3/geometry.py:13-169`:

- canvas: short edge 768 px scaled by the aspect, area capped at 768 x 1344
  px (both sides scaled by the square root of the excess), each side rounded
  to the nearest multiple of 32 (at least 32);
- frames: counts snap up to the next 17n + 5; latent_t = 5n + 2;
- grid: (latent_t, height / 16 / 2, width / 16 / 2) after the VAE's x16
  spatial stride and the 1x2x2 patch;
- name: '<w>x<h>_t<latent_t>', e.g. '16x9_t37'.
"""

from __future__ import annotations

import dataclasses
import math

FPS = 24
BASE_SHORT_EDGE = 768
MAX_PIXELS = BASE_SHORT_EDGE * 1344
CANVAS_MULTIPLE = 32
MIN_ASPECT_RATIO = 0.25
MAX_ASPECT_RATIO = 4.0
VAE_SPATIAL_STRIDE = 16
PATCH_HW = 2
AUDIO_LATENT_HZ = 40.0
AUDIO_CHANNELS = 2
MAX_DURATION_SECONDS = 15.0


def _round_to(value: float, multiple: int) -> int:
    # Python's round (half to even), as the reference's rule uses.
    return max(multiple, int(round(float(value) / multiple)) * multiple)


def resolve_canvas(aspect_w: int, aspect_h: int,
                   short_edge: int = BASE_SHORT_EDGE) -> tuple[int, int]:
    """(width, height) in pixels, multiples of 32 (geometry.py:30-58).

    Raises:
        ValueError: If the ratio is outside [1:4, 4:1].
    """
    ratio = float(aspect_w) / float(aspect_h)
    if not MIN_ASPECT_RATIO <= ratio <= MAX_ASPECT_RATIO:
        raise ValueError(f'aspect ratio {aspect_w}:{aspect_h} out of range')
    if ratio >= 1.0:
        width, height = float(short_edge) * ratio, float(short_edge)
    else:
        width, height = float(short_edge), float(short_edge) / ratio
    if width * height > MAX_PIXELS:
        shrink = math.sqrt(float(MAX_PIXELS) / (width * height))
        width, height = width * shrink, height * shrink
    return (_round_to(width, CANVAS_MULTIPLE),
            _round_to(height, CANVAS_MULTIPLE))


def align_frame_count(frame_count: int) -> int:
    """The smallest 17n + 5 at or above the count; 1 for none (:61-65)."""
    if frame_count <= 0:
        return 1
    return int(frame_count) + (5 - int(frame_count)) % 17


def video_latent_t(frame_count: int) -> int:
    """Latent frames of a 17n + 5 frame count: 5n + 2 (:68-71)."""
    if frame_count <= 5:
        return 2
    return (int(frame_count) - 5) // 17 * 5 + 2


def frame_count_from_latent_t(latent_t: int) -> int:
    """Inverse of `video_latent_t` (:74-77).

    Raises:
        ValueError: If latent_t is not 5n + 2.
    """
    if latent_t < 2 or (latent_t - 2) % 5:
        raise ValueError(f'latent_t {latent_t} is not of the form 5n+2')
    return 17 * ((latent_t - 2) // 5) + 5


def audio_latent_t(duration_seconds: float) -> int:
    return int(round(float(duration_seconds) * AUDIO_LATENT_HZ))


@dataclasses.dataclass(frozen=True)
class Geometry:
    """A resolved target geometry (geometry.py:84-134)."""

    aspect: str
    width: int
    height: int
    frame_count: int
    latent_t: int
    latent_h: int
    latent_w: int
    audio_t: int

    @property
    def duration_seconds(self) -> float:
        return self.frame_count / FPS

    @property
    def video_grid(self) -> tuple[int, int, int]:
        """Token grid (T, H, W) after the 1x2x2 patch."""
        return (self.latent_t, self.latent_h // PATCH_HW,
                self.latent_w // PATCH_HW)

    @property
    def num_video_tokens(self) -> int:
        t, h, w = self.video_grid
        return t * h * w

    @property
    def num_audio_rows(self) -> int:
        return AUDIO_CHANNELS * self.audio_t

    @property
    def name(self) -> str:
        return f'{self.aspect.replace(":", "x")}_t{self.latent_t}'


def resolve_geometry(aspect: str, duration_seconds: float,
                     short_edge: int = BASE_SHORT_EDGE) -> Geometry:
    """(aspect 'w:h', requested seconds) -> geometry (geometry.py:137-153)."""
    aspect_w, aspect_h = (int(v) for v in aspect.split(':'))
    width, height = resolve_canvas(aspect_w, aspect_h, short_edge)
    frames = align_frame_count(int(round(float(duration_seconds) * FPS)))
    return Geometry(aspect=aspect, width=width, height=height,
                    frame_count=frames, latent_t=video_latent_t(frames),
                    latent_h=height // VAE_SPATIAL_STRIDE,
                    latent_w=width // VAE_SPATIAL_STRIDE,
                    audio_t=audio_latent_t(frames / FPS))


def geometry_from_latent_t(aspect: str, latent_t: int,
                           short_edge: int = BASE_SHORT_EDGE) -> Geometry:
    """The geometry whose duration is exactly frame_count / FPS (:156-160)."""
    frames = frame_count_from_latent_t(latent_t)
    return resolve_geometry(aspect, frames / FPS, short_edge)


def latent_t_ladder(min_seconds: float = 5.0,
                    max_seconds: float = MAX_DURATION_SECONDS) -> list[int]:
    """Every latent_t whose duration lies in [min, max] seconds (:163-169)."""
    ladder = []
    latent_t = 2
    while frame_count_from_latent_t(latent_t) / FPS <= max_seconds:
        if frame_count_from_latent_t(latent_t) / FPS >= min_seconds:
            ladder.append(latent_t)
        latent_t += 5
    return ladder
