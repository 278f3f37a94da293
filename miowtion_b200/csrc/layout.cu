// a1: the tile permutation of a packed sequence, built on the device.
//
// Semantics of miowtion/veda/tiling.py:122-136 (span_tiles) and :214-275
// (build_tile_layout): each tiled span is cut into (st, sh, sw) boxes in
// (h-block, w-block, t-block) order; the real rows of a box, in t,h,w
// row-major order, form the tile's prefix; every uncovered real row of
// [0, used) is "global" and fills 128-row tiles in sequence order after all
// video tiles.
//
// The reference builds this with argsort / nonzero on the host. Here every
// slot is computed in closed form: a stable compaction of the rows of a box
// that fall inside the grid is the row-major order of the sub-box
// [0, vt) x [0, vh) x [0, vw), so slot `pos` of a tile maps to
// (pos / (vh*vw), (pos / vw) % vh, pos % vw) inside it.
#include "common.cuh"

namespace veda {

constexpr int kMaxSpans = 8;

struct LayoutParams {
  int n_spans;
  int64_t span_start[kMaxSpans];
  int grid[kMaxSpans][3];
  int shape[kMaxSpans][3];
  int64_t tile_begin[kMaxSpans + 1];  // first tile of each span; [n] = n_video
  // uncovered intervals of [0, used): global rows in order
  int n_gaps;
  int64_t gap_start[kMaxSpans + 1];
  int64_t gap_cum[kMaxSpans + 2];  // global rows before gap i
  int64_t n_tiles;
};

__global__ void build_layout_kernel(LayoutParams p, int64_t* perm,
                                    int32_t* valid_count) {
  const int64_t slot = static_cast<int64_t>(blockIdx.x) * blockDim.x +
                       threadIdx.x;
  if (slot >= p.n_tiles * kTile) return;
  const int64_t tile = slot / kTile;
  const int pos = static_cast<int>(slot % kTile);
  const int64_t n_video = p.tile_begin[p.n_spans];
  int64_t row = -1;
  int count = 0;
  if (tile < n_video) {
    int s = 0;
    while (s + 1 < p.n_spans && tile >= p.tile_begin[s + 1]) ++s;
    const int64_t lt = tile - p.tile_begin[s];
    const int T = p.grid[s][0], H = p.grid[s][1], W = p.grid[s][2];
    const int st = p.shape[s][0], sh = p.shape[s][1], sw = p.shape[s][2];
    const int nbt = (T + st - 1) / st, nbw = (W + sw - 1) / sw;
    const int bt = static_cast<int>(lt % nbt);
    const int bw = static_cast<int>((lt / nbt) % nbw);
    const int bh = static_cast<int>(lt / (static_cast<int64_t>(nbt) * nbw));
    const int t0 = bt * st, h0 = bh * sh, w0 = bw * sw;
    const int vt = min(st, T - t0), vh = min(sh, H - h0), vw = min(sw, W - w0);
    count = vt * vh * vw;
    if (pos < count) {
      const int dt = pos / (vh * vw);
      const int dh = (pos / vw) % vh;
      const int dw = pos % vw;
      row = p.span_start[s] +
            (static_cast<int64_t>(t0 + dt) * H + (h0 + dh)) * W + (w0 + dw);
    }
  } else {
    const int64_t total = p.gap_cum[p.n_gaps];
    const int64_t g0 = (tile - n_video) * kTile;
    const int64_t rest = total - g0;
    count = rest >= kTile ? kTile : (rest > 0 ? static_cast<int>(rest) : 0);
    const int64_t g = g0 + pos;
    if (g < total) {
      int i = 0;
      while (i + 1 < p.n_gaps && g >= p.gap_cum[i + 1]) ++i;
      row = p.gap_start[i] + (g - p.gap_cum[i]);
    }
  }
  perm[slot] = row;
  if (pos == 0) valid_count[tile] = count;
}

// The same tiles in box order: slot `pos` of a video tile is position
// (pos / (sh*sw), (pos / sw) % sh, pos % sw) of its (st, sh, sw) box, the
// order a 5D TMA box of the packed tensor lands in shared memory; slots
// outside the grid hold -1. Global tiles keep the prefix order of `perm`.
// key_mask[slot / 32] has bit (slot % 32) set for every real row.
__global__ void build_box_layout_kernel(LayoutParams p, int64_t* box_perm,
                                        uint32_t* key_mask) {
  const int64_t slot = static_cast<int64_t>(blockIdx.x) * blockDim.x +
                       threadIdx.x;
  const int64_t n_slots = p.n_tiles * kTile;
  // n_slots is a multiple of 128, so whole warps are in or out of range.
  if (slot - (threadIdx.x & 31) >= n_slots) return;
  int64_t row = -1;
  if (slot < n_slots) {
    const int64_t tile = slot / kTile;
    const int pos = static_cast<int>(slot % kTile);
    const int64_t n_video = p.tile_begin[p.n_spans];
    if (tile < n_video) {
      int s = 0;
      while (s + 1 < p.n_spans && tile >= p.tile_begin[s + 1]) ++s;
      const int64_t lt = tile - p.tile_begin[s];
      const int T = p.grid[s][0], H = p.grid[s][1], W = p.grid[s][2];
      const int st = p.shape[s][0], sh = p.shape[s][1], sw = p.shape[s][2];
      const int nbt = (T + st - 1) / st, nbw = (W + sw - 1) / sw;
      const int bt = static_cast<int>(lt % nbt);
      const int bw = static_cast<int>((lt / nbt) % nbw);
      const int bh = static_cast<int>(lt / (static_cast<int64_t>(nbt) * nbw));
      const int t = bt * st + pos / (sh * sw);
      const int h = bh * sh + (pos / sw) % sh;
      const int w = bw * sw + pos % sw;
      if (t < T && h < H && w < W)
        row = p.span_start[s] + (static_cast<int64_t>(t) * H + h) * W + w;
    } else {
      const int64_t total = p.gap_cum[p.n_gaps];
      const int64_t g = (tile - n_video) * kTile + pos;
      if (g < total) {
        int i = 0;
        while (i + 1 < p.n_gaps && g >= p.gap_cum[i + 1]) ++i;
        row = p.gap_start[i] + (g - p.gap_cum[i]);
      }
    }
    box_perm[slot] = row;
  }
  const unsigned bits = __ballot_sync(0xffffffffu, row >= 0);
  if ((threadIdx.x & 31) == 0 && slot < n_slots) key_mask[slot / 32] = bits;
}

// Fills LayoutParams from the spans (host side of both layout entry points).
int layout_params(const veda_span_t* spans, int32_t n_spans, int64_t used,
                  int64_t seq_len, int64_t n_tiles, LayoutParams* out) {
  VEDA_REQUIRE(spans != nullptr && n_spans >= 1,
               "at least the target span must be tiled");
  VEDA_REQUIRE(n_spans <= kMaxSpans, "at most 8 tiled spans are supported");
  VEDA_REQUIRE(used >= 0 && used <= seq_len, "need 0 <= used <= seq_len");
  LayoutParams p{};
  p.n_spans = n_spans;
  int64_t prev_stop = 0, tiles = 0;
  p.n_gaps = 0;
  p.gap_cum[0] = 0;
  for (int s = 0; s < n_spans; ++s) {
    const veda_span_t& sp = spans[s];
    int64_t rows = 1, vol = 1;
    for (int a = 0; a < 3; ++a) {
      VEDA_REQUIRE(sp.grid[a] > 0 && sp.shape[a] > 0,
                   "span grid and tile shape must be positive");
      rows *= sp.grid[a];
      vol *= sp.shape[a];
      p.grid[s][a] = sp.grid[a];
      p.shape[s][a] = sp.shape[a];
    }
    VEDA_REQUIRE(vol == kTile, "tile shape does not hold 128 tokens");
    VEDA_REQUIRE(sp.start >= prev_stop && sp.start + rows <= used,
                 "span overlaps the previous one or exceeds used");
    if (sp.start > prev_stop) {
      p.gap_start[p.n_gaps] = prev_stop;
      p.gap_cum[p.n_gaps + 1] = p.gap_cum[p.n_gaps] + (sp.start - prev_stop);
      ++p.n_gaps;
    }
    p.span_start[s] = sp.start;
    p.tile_begin[s] = tiles;
    int64_t n = 1;
    for (int a = 0; a < 3; ++a)
      n *= (sp.grid[a] + sp.shape[a] - 1) / sp.shape[a];
    tiles += n;
    prev_stop = sp.start + rows;
  }
  p.tile_begin[n_spans] = tiles;
  if (used > prev_stop) {
    p.gap_start[p.n_gaps] = prev_stop;
    p.gap_cum[p.n_gaps + 1] = p.gap_cum[p.n_gaps] + (used - prev_stop);
    ++p.n_gaps;
  }
  const int64_t n_global = (p.gap_cum[p.n_gaps] + kTile - 1) / kTile;
  VEDA_REQUIRE(n_tiles == tiles + n_global,
               "n_tiles does not match the spans and global rows");
  p.n_tiles = n_tiles;
  *out = p;
  return VEDA_OK;
}

}  // namespace veda

using namespace veda;

extern "C" int veda_build_layout(const veda_span_t* spans, int32_t n_spans,
                                 int64_t used, int64_t seq_len,
                                 int64_t n_tiles, int64_t* perm,
                                 int32_t* valid_count, void* stream) {
  LayoutParams p{};
  int rc = layout_params(spans, n_spans, used, seq_len, n_tiles, &p);
  if (rc != VEDA_OK) return rc;
  VEDA_REQUIRE(perm != nullptr && valid_count != nullptr,
               "perm and valid_count are required");
  const int64_t slots = n_tiles * kTile;
  if (slots == 0) return VEDA_OK;
  const int threads = 256;
  const int64_t blocks = (slots + threads - 1) / threads;
  build_layout_kernel<<<static_cast<unsigned>(blocks), threads, 0,
                        as_stream(stream)>>>(p, perm, valid_count);
  return check_launch("build_layout_kernel");
}

extern "C" int veda_build_box_layout(const veda_span_t* spans,
                                     int32_t n_spans, int64_t used,
                                     int64_t seq_len, int64_t n_tiles,
                                     int64_t* box_perm, uint32_t* key_mask,
                                     void* stream) {
  LayoutParams p{};
  int rc = layout_params(spans, n_spans, used, seq_len, n_tiles, &p);
  if (rc != VEDA_OK) return rc;
  VEDA_REQUIRE(box_perm != nullptr && key_mask != nullptr,
               "box_perm and key_mask are required");
  const int64_t slots = n_tiles * kTile;
  if (slots == 0) return VEDA_OK;
  const int threads = 256;
  const int64_t blocks = (slots + threads - 1) / threads;
  build_box_layout_kernel<<<static_cast<unsigned>(blocks), threads, 0,
                            as_stream(stream)>>>(p, box_perm, key_mask);
  return check_launch("build_box_layout_kernel");
}
