// a5-a8: budgeted top-k per query tile, the block mask and the full/partial
// index lists (and their transposes for the backward pass).
//
// Semantics:
//   miowtion/veda/mask.py:200-285 select_video_blocks (rule 'topk'):
//     per column block, empty key tiles score -inf, the query tile's own tile
//     +inf (only inside its block); keep the `k_lo + bresenham[row]` best
//     columns whose score is > -inf.
//   mask.py:79-93 bresenham_extra: row r keeps one more iff
//     floor((r+1) f) > floor(r f), evaluated in fp64 like the reference.
//   mask.py:288-317 dense_block_mask: global key columns are kept wherever
//     the key tile is non-empty, global query rows keep every non-empty tile.
//   miowtion/kernels/fa4.py:266-296 index_lists: members of (mask & full) and
//     (mask & ~full), ascending, optionally followed by the non-members in
//     ascending order (the reference's stable argsort puts them there).
//
// Top-k is an exact radix select on order-preserving 32-bit keys: one warp
// per (head, row) finds the k-th largest key bit by bit (32 warp-wide
// counts), then keeps every key above it and the lowest-numbered columns
// equal to it. Ties therefore rank the lower column first (torch.topk leaves
// tie order unspecified).
#include <math.h>

#include "common.cuh"

namespace veda {

namespace {

constexpr int kMaxBlocks = 2;
constexpr int kSelectWarps = 4;
constexpr int kMaxCols = 8192;

__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

const uint32_t kNegInfKey = 0x007FFFFFu;  // order_key(-inf)

struct Block {
  int start, stop, k_lo, k_hi, keeps_all;
  double frac;
};

struct SelectParams {
  const float* scores;
  int64_t ld;          // row stride of scores
  int n_heads;
  int64_t n_rows;      // selected video rows R
  const int64_t* rows;
  const int32_t* valid_count;
  int n_tiles;
  int n_video;
  Block blocks[kMaxBlocks];
  int n_blocks;
  int global_rows;
  int64_t n_rows_out;  // R (+ n - n_video with global rows)
  uint8_t* mask;
  int32_t *part_cnt, *part_idx, *full_cnt, *full_idx;
  int fill_tails;
  int64_t* sel_index;
  uint8_t* sel_keep;
  int sel_k;           // K = sum of block widths in the selection output
};

// Number of keys in [0, n) (this lane's strided share) that are >= thr.
__device__ __forceinline__ int count_ge(const uint32_t* keys, int n,
                                        uint32_t thr, int lane) {
  int c = 0;
  for (int i = lane; i < n; i += 32) c += keys[i] >= thr;
  return __reduce_add_sync(0xffffffffu, c);
}

// Largest key T with #(keys >= T) >= k (the k-th largest key), k >= 1.
__device__ uint32_t kth_largest(const uint32_t* keys, int n, int k,
                                int lane) {
  uint32_t t = 0;
  for (int bit = 31; bit >= 0; --bit) {
    const uint32_t cand = t | (1u << bit);
    if (count_ge(keys, n, cand, lane) >= k) t = cand;
  }
  return t;
}

// The same with this lane's keys (columns lane + 32 j, j < kPerLane) held
// in registers: the 32 passes read no shared memory. Absent columns hold 0,
// below every real key (order_key(-inf) > 0), so they never count.
template <int kPerLane>
__device__ uint32_t kth_largest_reg(const uint32_t (&kr)[kPerLane], int k) {
  uint32_t t = 0;
  for (int bit = 31; bit >= 0; --bit) {
    const uint32_t cand = t | (1u << bit);
    int c = 0;
#pragma unroll
    for (int j = 0; j < kPerLane; ++j) c += kr[j] >= cand;
    if (__reduce_add_sync(0xffffffffu, c) >= k) t = cand;
  }
  return t;
}

// Marks in `member` (one byte per column of the block) the `take` largest
// keys, ties to the lowest column. keys > thr are all members, then the
// first (take - #greater) columns with key == thr.
__device__ void mark_top(const uint32_t* keys, int n, uint32_t thr, int take,
                         bool exclude_thr, uint8_t* member, int lane) {
  int greater = 0;
  for (int i = lane; i < n; i += 32) greater += keys[i] > thr;
  greater = __reduce_add_sync(0xffffffffu, greater);
  int need = exclude_thr ? 0 : take - greater;
  for (int base = 0; base < n; base += 32) {
    const int i = base + lane;
    const uint32_t key = i < n ? keys[i] : 0u;
    const bool gt = i < n && key > thr;
    const bool eq = i < n && key == thr;
    const uint32_t eq_mask = __ballot_sync(0xffffffffu, eq);
    const int before = __popc(eq_mask & ((1u << lane) - 1u));
    const bool take_eq = eq && before < need;
    if (i < n) member[i] = (gt || take_eq) ? 1 : 0;
    need -= min(need, __popc(eq_mask));
  }
}

__device__ __forceinline__ bool extra_row(int64_t r, double frac) {
  return floor(static_cast<double>(r + 1) * frac) >
         floor(static_cast<double>(r) * frac);
}

// Writes the lists of one row from per-column membership bytes. `member`
// covers all n columns; full[c] says whether the key tile is full.
__device__ void write_lists(const uint8_t* member, const int32_t* valid_count,
                            int n, int32_t* pc, int32_t* pi, int32_t* fc,
                            int32_t* fi, bool tails, uint8_t* mask_row,
                            int lane) {
  int n_full = 0, n_part = 0;
  for (int base = 0; base < n; base += 32) {
    const int c = base + lane;
    const bool m = c < n && member[c];
    const bool full = c < n && valid_count[c] == kTile;
    n_full += __popc(__ballot_sync(0xffffffffu, m && full));
    n_part += __popc(__ballot_sync(0xffffffffu, m && !full));
  }
  int run_f = 0, run_p = 0, run_nf = 0, run_np = 0;
  const uint32_t below = (1u << lane) - 1u;
  for (int base = 0; base < n; base += 32) {
    const int c = base + lane;
    const bool in = c < n;
    const bool m = in && member[c];
    const bool full = in && valid_count[c] == kTile;
    const bool mf = m && full, mp = m && !full;
    const uint32_t bf = __ballot_sync(0xffffffffu, mf);
    const uint32_t bp = __ballot_sync(0xffffffffu, mp);
    if (mf && fi) fi[run_f + __popc(bf & below)] = c;
    if (mp && pi) pi[run_p + __popc(bp & below)] = c;
    if (tails) {
      const uint32_t bnf = __ballot_sync(0xffffffffu, in && !mf);
      const uint32_t bnp = __ballot_sync(0xffffffffu, in && !mp);
      if (in && !mf && fi) fi[n_full + run_nf + __popc(bnf & below)] = c;
      if (in && !mp && pi) pi[n_part + run_np + __popc(bnp & below)] = c;
      run_nf += __popc(bnf);
      run_np += __popc(bnp);
    }
    run_f += __popc(bf);
    run_p += __popc(bp);
    if (in && mask_row) mask_row[c] = m ? 1 : 0;
  }
  if (lane == 0) {
    if (fc) *fc = n_full;
    if (pc) *pc = n_part;
  }
}

// kRegKeys: keys per lane kept in registers for the radix select (blocks of
// up to 32 * kRegKeys columns; wider blocks select from shared memory).
template <int kRegKeys>
__global__ void __launch_bounds__(kSelectWarps * 32)
    select_kernel(SelectParams p) {
  extern __shared__ uint8_t sel_smem[];
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int64_t item = static_cast<int64_t>(blockIdx.x) * kSelectWarps + warp;
  if (item >= static_cast<int64_t>(p.n_heads) * p.n_rows_out) return;
  const int h = static_cast<int>(item / p.n_rows_out);
  const int64_t i = item % p.n_rows_out;
  const int n = p.n_tiles;
  // per warp: keys[kMaxCols] u32 + member[n] bytes
  const int stride = n * 4 + ((n + 15) & ~15);
  uint32_t* keys = reinterpret_cast<uint32_t*>(sel_smem + warp * stride);
  uint8_t* member = sel_smem + warp * stride + n * 4;

  const bool global = i >= p.n_rows;
  if (global) {
    for (int c = lane; c < n; c += 32) member[c] = p.valid_count[c] > 0;
  } else {
    const int64_t t = p.rows != nullptr ? p.rows[i] : i;
    const float* srow =
        p.scores + (static_cast<int64_t>(h) * p.n_rows + i) * p.ld;
    int64_t sel_off = 0;
    for (int b = 0; b < p.n_blocks; ++b) {
      const Block blk = p.blocks[b];
      const int w = blk.stop - blk.start;
      if (blk.keeps_all) {
        for (int c = lane; c < w; c += 32)
          member[blk.start + c] = p.valid_count[blk.start + c] > 0;
        if (p.sel_index != nullptr) {
          const int64_t base =
              (static_cast<int64_t>(h) * p.n_rows + i) * p.sel_k + sel_off;
          for (int c = lane; c < w; c += 32) {
            p.sel_index[base + c] = blk.start + c;
            p.sel_keep[base + c] = p.valid_count[blk.start + c] > 0;
          }
        }
        sel_off += w;
        continue;
      }
      // The keys also stay in registers when the block is narrow enough.
      uint32_t kr[kRegKeys];
#pragma unroll
      for (int j = 0; j < kRegKeys; ++j) kr[j] = 0u;
      for (int c = lane; c < w; c += 32) {
        const int col = blk.start + c;
        float v = srow[col];
        if (p.valid_count[col] == 0) v = -INFINITY;
        if (col == t) v = INFINITY;  // own tile, only inside its block
        keys[c] = order_key(v);
      }
      if (w <= 32 * kRegKeys) {
#pragma unroll
        for (int j = 0; j < kRegKeys; ++j)
          if (lane + 32 * j < w) kr[j] = keys[lane + 32 * j];
      }
      __syncwarp();
      int allowed = blk.k_lo + (extra_row(t, blk.frac) ? 1 : 0);
      allowed = min(allowed, blk.k_hi);
      const uint32_t thr = w <= 32 * kRegKeys
                               ? kth_largest_reg<kRegKeys>(kr, allowed)
                               : kth_largest(keys, w, allowed, lane);
      // -inf columns are never kept (mask.py:281-282).
      mark_top(keys, w, thr, allowed, thr == kNegInfKey, member + blk.start,
               lane);
      if (p.sel_index != nullptr) {
        // Reference rank order of the top k_hi: value descending, ties by
        // column ascending; keep = rank < allowed and value > -inf.
        const uint32_t thr_hi = kth_largest(keys, w, blk.k_hi, lane);
        int greater = 0;
        for (int c = lane; c < w; c += 32) greater += keys[c] > thr_hi;
        greater = __reduce_add_sync(0xffffffffu, greater);
        int need_eq = blk.k_hi - greater;
        const int64_t base =
            (static_cast<int64_t>(h) * p.n_rows + i) * p.sel_k + sel_off;
        for (int c0 = 0; c0 < w; c0 += 32) {
          const int c = c0 + lane;
          const uint32_t key = c < w ? keys[c] : 0u;
          const bool eq = c < w && key == thr_hi;
          const uint32_t eq_mask = __ballot_sync(0xffffffffu, eq);
          const int eq_before = __popc(eq_mask & ((1u << lane) - 1u));
          const bool in_top = c < w && (key > thr_hi || (eq && eq_before <
                                                          need_eq));
          need_eq -= min(need_eq, __popc(eq_mask));
          if (in_top) {
            // rank = #(key' > key) + #(key' == key, c' < c)
            int rank = 0;
            for (int c2 = 0; c2 < w; ++c2) {
              const uint32_t k2 = keys[c2];
              rank += (k2 > key) || (k2 == key && c2 < c);
            }
            p.sel_index[base + rank] = blk.start + c;
            p.sel_keep[base + rank] =
                (rank < allowed) && (key != kNegInfKey) ? 1 : 0;
          }
        }
        sel_off += blk.k_hi;
      }
      __syncwarp();
    }
    for (int c = p.n_video + lane; c < n; c += 32)
      member[c] = p.valid_count[c] > 0;
  }
  __syncwarp();
  const int64_t row_out = static_cast<int64_t>(h) * p.n_rows_out + i;
  write_lists(member, p.valid_count, n,
              p.part_cnt ? p.part_cnt + row_out : nullptr,
              p.part_idx ? p.part_idx + row_out * n : nullptr,
              p.full_cnt ? p.full_cnt + row_out : nullptr,
              p.full_idx ? p.full_idx + row_out * n : nullptr,
              p.fill_tails != 0,
              p.mask ? p.mask + row_out * n : nullptr, lane);
}

// Lists of an arbitrary mask. Forward: one warp per (head, row).
__global__ void __launch_bounds__(kSelectWarps * 32)
    lists_rows_kernel(const uint8_t* mask, int n_heads, int64_t n_rows,
                      int n_cols, const int32_t* valid_count, int32_t* pc,
                      int32_t* pi, int32_t* fc, int32_t* fi, int tails) {
  extern __shared__ uint8_t sel_smem[];
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int64_t item = static_cast<int64_t>(blockIdx.x) * kSelectWarps + warp;
  if (item >= static_cast<int64_t>(n_heads) * n_rows) return;
  uint8_t* member = sel_smem + warp * ((n_cols + 15) & ~15);
  const uint8_t* row = mask + item * n_cols;
  for (int c = lane; c < n_cols; c += 32)
    member[c] = row[c] && valid_count[c] > 0;
  __syncwarp();
  write_lists(member, valid_count, n_cols, pc ? pc + item : nullptr,
              pi ? pi + item * n_cols : nullptr, fc ? fc + item : nullptr,
              fi ? fi + item * n_cols : nullptr, tails != 0, nullptr, lane);
}

// Transposed lists: for key tile c, the query tiles r with mask[r, c]; all of
// them go to the full list when the key tile is full, else to the partial
// list. One warp per (head, 32 key tiles): lane j owns key tile c0 + j and
// reads the mask one 32-byte row segment at a time (coalesced).
__global__ void __launch_bounds__(32)
    lists_cols_kernel(const uint8_t* mask, int n_heads, int64_t n_rows,
                      int n_cols, const int32_t* valid_count, int32_t* pc,
                      int32_t* pi, int32_t* fc, int32_t* fi, int tails) {
  const int lane = threadIdx.x;
  const int col_blocks = (n_cols + 31) / 32;
  const int h = blockIdx.x / col_blocks;
  const int c = (blockIdx.x % col_blocks) * 32 + lane;
  const bool in = c < n_cols;
  const int vc = in ? valid_count[c] : 0;
  const bool ok = vc > 0;
  const bool full = vc == kTile;
  const uint8_t* m = mask + static_cast<int64_t>(h) * n_rows * n_cols;
  const int64_t out_row = static_cast<int64_t>(h) * n_cols + c;
  int32_t* mine = full ? (fi ? fi + out_row * n_rows : nullptr)
                       : (pi ? pi + out_row * n_rows : nullptr);
  int32_t* other = full ? (pi ? pi + out_row * n_rows : nullptr)
                        : (fi ? fi + out_row * n_rows : nullptr);
  int cnt = 0;
  for (int64_t r = 0; r < n_rows; ++r) {
    const bool member = in && ok && m[r * n_cols + c];
    if (member) {
      if (mine) mine[cnt] = static_cast<int32_t>(r);
      ++cnt;
    }
  }
  if (in && tails) {
    int pos = cnt;
    for (int64_t r = 0; r < n_rows; ++r) {
      const bool member = ok && m[r * n_cols + c];
      if (!member && mine) mine[pos++] = static_cast<int32_t>(r);
      if (other) other[r] = static_cast<int32_t>(r);
    }
  }
  if (in) {
    if (full) {
      if (fc) fc[out_row] = cnt;
      if (pc) pc[out_row] = 0;
    } else {
      if (pc) pc[out_row] = cnt;
      if (fc) fc[out_row] = 0;
    }
  }
}

}  // namespace

}  // namespace veda

using namespace veda;

extern "C" int veda_block_select(
    const float* scores, int64_t ld_scores, int32_t n_heads, int64_t n_rows,
    const int64_t* rows, const int32_t* valid_count, int64_t n_tiles,
    int64_t n_video, const veda_column_block_t* blocks, int32_t n_blocks,
    int32_t global_rows, uint8_t* mask, int32_t* part_cnt, int32_t* part_idx,
    int32_t* full_cnt, int32_t* full_idx, int32_t fill_tails,
    int64_t* sel_index, uint8_t* sel_keep, void* stream) {
  VEDA_REQUIRE(valid_count != nullptr, "valid_count is required");
  VEDA_REQUIRE(n_heads >= 1, "bad number of heads");
  VEDA_REQUIRE(n_tiles >= 1 && n_tiles <= kMaxCols,
               "n_tiles must be in [1, 8192]");
  VEDA_REQUIRE(n_video >= 0 && n_video <= n_tiles, "bad n_video");
  VEDA_REQUIRE(n_blocks >= 1 && n_blocks <= kMaxBlocks,
               "one or two column blocks are supported");
  VEDA_REQUIRE(n_rows >= 0 && (n_rows == 0 || scores != nullptr),
               "scores are required");
  VEDA_REQUIRE(ld_scores >= n_video, "ld_scores must cover the video columns");
  VEDA_REQUIRE(!global_rows || n_rows == n_video,
               "global_rows needs a selection of all video rows");
  VEDA_REQUIRE((sel_index == nullptr) == (sel_keep == nullptr),
               "sel_index and sel_keep go together");
  SelectParams p{};
  p.scores = scores;
  p.ld = ld_scores;
  p.n_heads = n_heads;
  p.n_rows = n_rows;
  p.rows = rows;
  p.valid_count = valid_count;
  p.n_tiles = static_cast<int>(n_tiles);
  p.n_video = static_cast<int>(n_video);
  p.n_blocks = n_blocks;
  int prev = 0, sel_k = 0;
  for (int b = 0; b < n_blocks; ++b) {
    const veda_column_block_t& c = blocks[b];
    VEDA_REQUIRE(c.start == prev && c.stop > c.start && c.stop <= n_video,
                 "column blocks must tile [0, n_video) in order");
    const int w = c.stop - c.start;
    VEDA_REQUIRE(c.keeps_all ||
                     (c.k_lo >= 1 && c.k_lo <= c.k_hi && c.k_hi <= w),
                 "need 1 <= k_lo <= k_hi <= block width");
    VEDA_REQUIRE(c.frac >= 0.0 && c.frac <= 1.0, "frac must be in [0, 1]");
    p.blocks[b] = Block{c.start, c.stop, c.k_lo, c.k_hi, c.keeps_all, c.frac};
    sel_k += c.keeps_all ? w : c.k_hi;
    prev = c.stop;
  }
  VEDA_REQUIRE(prev == n_video, "column blocks must end at n_video");
  if (rows == nullptr)
    VEDA_REQUIRE(n_rows <= n_video, "more rows than video tiles");
  p.global_rows = global_rows;
  p.n_rows_out = n_rows + (global_rows ? n_tiles - n_video : 0);
  p.mask = mask;
  p.part_cnt = part_cnt;
  p.part_idx = part_idx;
  p.full_cnt = full_cnt;
  p.full_idx = full_idx;
  p.fill_tails = fill_tails;
  p.sel_index = sel_index;
  p.sel_keep = sel_keep;
  p.sel_k = sel_k;
  const int64_t items = static_cast<int64_t>(n_heads) * p.n_rows_out;
  if (items == 0) return VEDA_OK;
  const int stride = static_cast<int>(n_tiles * 4 + ((n_tiles + 15) & ~15));
  const int smem = kSelectWarps * stride;
  const unsigned grid =
      static_cast<unsigned>((items + kSelectWarps - 1) / kSelectWarps);
  auto launch = [&](auto kernel) -> int {
    if (smem > 48 * 1024)
      VEDA_CUDA(cudaFuncSetAttribute(
          kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    kernel<<<grid, kSelectWarps * 32, smem, as_stream(stream)>>>(p);
    return check_launch("select_kernel");
  };
  if (n_video <= 256) return launch(select_kernel<8>);
  if (n_video <= 512) return launch(select_kernel<16>);
  return launch(select_kernel<32>);
}

extern "C" int veda_index_lists(const uint8_t* mask, int32_t n_heads,
                                int64_t n_rows, int64_t n_cols,
                                const int32_t* valid_count, int32_t transpose,
                                int32_t* part_cnt, int32_t* part_idx,
                                int32_t* full_cnt, int32_t* full_idx,
                                int32_t fill_tails, void* stream) {
  VEDA_REQUIRE(mask != nullptr && valid_count != nullptr,
               "mask and valid_count are required");
  VEDA_REQUIRE(n_heads >= 1 && n_rows >= 0 && n_cols >= 1 &&
                   n_cols <= kMaxCols,
               "bad mask shape");
  if (n_rows == 0) return VEDA_OK;
  if (!transpose) {
    const int64_t items = static_cast<int64_t>(n_heads) * n_rows;
    const int smem = kSelectWarps * static_cast<int>((n_cols + 15) & ~15);
    lists_rows_kernel<<<static_cast<unsigned>((items + kSelectWarps - 1) /
                                              kSelectWarps),
                        kSelectWarps * 32, smem, as_stream(stream)>>>(
        mask, n_heads, n_rows, static_cast<int>(n_cols), valid_count,
        part_cnt, part_idx, full_cnt, full_idx, fill_tails);
    return check_launch("lists_rows_kernel");
  }
  const int64_t blocks = static_cast<int64_t>(n_heads) * ((n_cols + 31) / 32);
  lists_cols_kernel<<<static_cast<unsigned>(blocks), 32, 0,
                      as_stream(stream)>>>(
      mask, n_heads, n_rows, static_cast<int>(n_cols), valid_count, part_cnt,
      part_idx, full_cnt, full_idx, fill_tails);
  return check_launch("lists_cols_kernel");
}
