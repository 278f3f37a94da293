// a2/a3/a12/a14: permutation into tile order with fused pooling, the inverse
// permutation, and the LSE gather. HBM-bound byte movement.
//
// One CTA per (tile, head): 256 threads, each owning 8 consecutive head-dim
// columns (one 16-byte vector) of 8 rows, so every half-warp moves one whole
// 256-byte row per instruction (fully coalesced reads and writes). Pooling
// (semantics of miowtion/veda/predictor.py:82-168) reduces in registers,
// then across the 16 row groups with one shuffle and a shared-memory pass.
#include "common.cuh"

namespace veda {

namespace {

constexpr int kPoolThreads = 256;
constexpr int kRowsPerThread = kTile / (kPoolThreads / 16);  // 8

__device__ __forceinline__ void bf16x8_to_float(const uint4& v, float* f) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

struct GatherParams {
  const __nv_bfloat16* x;
  int64_t x_stride_s, x_stride_h;
  const int64_t* perm;  // nullptr: identity (x already tile-ordered)
  const int32_t* valid_count;
  const int64_t* heads;  // nullptr: head h
  __nv_bfloat16* out;    // nullptr: pool only
  int64_t out_stride_n, out_stride_h;
  // out holds shared-memory images of the tiles instead of rows: tile
  // (h, tile) is 32 KB at (h * n_tiles + tile) * 32 KB, two 64-column halves
  // of 128 rows x 128 bytes, the 16-byte chunks of row r in the order of the
  // 128-byte swizzle (chunk c at position c ^ (r % 8)), exactly what a TMA
  // load of the two boxes with 128-byte swizzle writes to shared memory.
  int image;
  float* feats;  // [H', n, 3D] or nullptr
  float* sq;     // [H', n, D] or nullptr
  float* var;    // [H', n, D] or nullptr
  int64_t n_tiles;
};

// kMode: 0 gather only, 1 also mean/max/min, 2 also the second moments.
// Separate instantiations keep the gather and the first-moment pooling at
// the registers they need (the second moments hold every row's values for a
// second pass), so more CTAs per SM keep loads in flight.
template <int kMode>
__global__ void __launch_bounds__(kPoolThreads, kMode == 2 ? 1 : 4)
    gather_pool_kernel(GatherParams p, int64_t n_tiles) {
  // Tiles vary fastest across the grid: the CTAs in flight write one head's
  // tiles contiguously (measured faster than all heads of a tile at once).
  const int64_t tile = blockIdx.x % n_tiles;
  const int h = static_cast<int>(blockIdx.x / n_tiles);
  const int tid = threadIdx.x;
  const int c8 = tid & 15;   // column group: columns [8*c8, 8*c8 + 8)
  const int rg = tid >> 4;   // row group: rows rg + 16*i
  const int64_t head = p.heads != nullptr ? p.heads[h] : h;
  const int count = p.valid_count[tile];

  uint4 vals[kRowsPerThread];
#pragma unroll
  for (int i = 0; i < kRowsPerThread; ++i) {
    const int r = rg + 16 * i;
    const int64_t slot = tile * kTile + r;
    // Tile-ordered input keeps its padding rows (zero by contract) in the
    // sums exactly like predictor.pool_tiles; a gather reads real rows only.
    int64_t src = slot;
    bool valid = true;
    if (p.perm != nullptr) {
      src = p.perm[slot];
      valid = src >= 0;
    }
    vals[i] = make_uint4(0, 0, 0, 0);
    if (valid)
      vals[i] = __ldg(reinterpret_cast<const uint4*>(
          p.x + src * p.x_stride_s + head * p.x_stride_h + 8 * c8));
  }
  if (p.out != nullptr && p.image) {
    __nv_bfloat16* img = p.out + (static_cast<int64_t>(h) * p.n_tiles + tile) *
                                     (kTile * kHeadDim) +
                         (c8 >> 3) * (kTile * 64);
#pragma unroll
    for (int i = 0; i < kRowsPerThread; ++i) {
      const int r = rg + 16 * i;
      *reinterpret_cast<uint4*>(img + r * 64 + (((c8 & 7) ^ (r & 7)) * 8)) =
          vals[i];
    }
  } else if (p.out != nullptr) {
#pragma unroll
    for (int i = 0; i < kRowsPerThread; ++i) {
      const int64_t slot = tile * kTile + rg + 16 * i;
      *reinterpret_cast<uint4*>(p.out + slot * p.out_stride_n +
                                h * p.out_stride_h + 8 * c8) = vals[i];
    }
  }
  if constexpr (kMode == 0) {
    return;
  } else {

  __shared__ float red[3][kPoolThreads / 32][kHeadDim];
  __shared__ float mean_s[kHeadDim];
  const int warp = tid >> 5;
  const int lane = tid & 31;

  float sum[8], mx[8], mn[8];
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    sum[c] = 0.f;
    mx[c] = -INFINITY;
    mn[c] = INFINITY;
  }
#pragma unroll
  for (int i = 0; i < kRowsPerThread; ++i) {
    const int r = rg + 16 * i;
    float f[8];
    bf16x8_to_float(vals[i], f);
    const bool valid = r < count;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      sum[c] += f[c];  // padding rows hold 0
      if (valid) {
        mx[c] = fmaxf(mx[c], f[c]);
        mn[c] = fminf(mn[c], f[c]);
      }
    }
  }
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    sum[c] += __shfl_xor_sync(0xffffffffu, sum[c], 16);
    mx[c] = fmaxf(mx[c], __shfl_xor_sync(0xffffffffu, mx[c], 16));
    mn[c] = fminf(mn[c], __shfl_xor_sync(0xffffffffu, mn[c], 16));
  }
  if (lane < 16) {
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      red[0][warp][8 * c8 + c] = sum[c];
      red[1][warp][8 * c8 + c] = mx[c];
      red[2][warp][8 * c8 + c] = mn[c];
    }
  }
  __syncthreads();
  const float denom = static_cast<float>(max(count, 1));
  if (tid < kHeadDim) {
    float s = 0.f, a = -INFINITY, b = INFINITY;
#pragma unroll
    for (int w = 0; w < kPoolThreads / 32; ++w) {
      s += red[0][w][tid];
      a = fmaxf(a, red[1][w][tid]);
      b = fminf(b, red[2][w][tid]);
    }
    const float mean = s / denom;
    mean_s[tid] = mean;
    if (p.feats != nullptr) {
      float* f = p.feats + (static_cast<int64_t>(h) * p.n_tiles + tile) *
                               (3 * kHeadDim);
      const bool empty = count == 0;
      f[tid] = empty ? 0.f : mean;
      f[kHeadDim + tid] = empty ? 0.f : a;
      f[2 * kHeadDim + tid] = empty ? 0.f : b;
    }
  }
  if constexpr (kMode == 2) {
  __syncthreads();
  // Second moments from the rows still held in registers; the centred one
  // is two-pass (predictor.py:133-168 explains why not E[x^2] - E[x]^2).
  float m8[8], s2[8], v2[8];
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    m8[c] = mean_s[8 * c8 + c];
    s2[c] = 0.f;
    v2[c] = 0.f;
  }
#pragma unroll
  for (int i = 0; i < kRowsPerThread; ++i) {
    const int r = rg + 16 * i;
    if (r >= count) continue;
    float f[8];
    bf16x8_to_float(vals[i], f);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      s2[c] += f[c] * f[c];
      const float d = f[c] - m8[c];
      v2[c] += d * d;
    }
  }
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    s2[c] += __shfl_xor_sync(0xffffffffu, s2[c], 16);
    v2[c] += __shfl_xor_sync(0xffffffffu, v2[c], 16);
  }
  __syncthreads();
  if (lane < 16) {
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      red[0][warp][8 * c8 + c] = s2[c];
      red[1][warp][8 * c8 + c] = v2[c];
    }
  }
  __syncthreads();
  if (tid < kHeadDim) {
    float a = 0.f, b = 0.f;
#pragma unroll
    for (int w = 0; w < kPoolThreads / 32; ++w) {
      a += red[0][w][tid];
      b += red[1][w][tid];
    }
    const int64_t base = (static_cast<int64_t>(h) * p.n_tiles + tile) *
                         kHeadDim + tid;
    const bool empty = count == 0;
    if (p.sq != nullptr) p.sq[base] = empty ? 0.f : a / denom;
    if (p.var != nullptr) p.var[base] = empty ? 0.f : b / denom;
  }
  }  // kMode == 2
  }  // kMode > 0
}

struct ScatterParams {
  const __nv_bfloat16* tiled;
  int64_t t_stride_n, t_stride_h;
  const int64_t* perm;
  const int64_t* heads;
  __nv_bfloat16* out;
  int64_t out_stride_s, out_stride_h;
};

__global__ void __launch_bounds__(kPoolThreads)
    scatter_kernel(ScatterParams p, int64_t n_tiles) {
  const int64_t tile = blockIdx.x % n_tiles;
  const int h = static_cast<int>(blockIdx.x / n_tiles);
  const int tid = threadIdx.x;
  const int c8 = tid & 15;
  const int rg = tid >> 4;
  const int64_t head = p.heads != nullptr ? p.heads[h] : h;
  uint4 vals[kRowsPerThread];
  int64_t dst[kRowsPerThread];
#pragma unroll
  for (int i = 0; i < kRowsPerThread; ++i) {
    const int64_t slot = tile * kTile + rg + 16 * i;
    dst[i] = p.perm[slot];
    vals[i] = __ldg(reinterpret_cast<const uint4*>(
        p.tiled + slot * p.t_stride_n + h * p.t_stride_h + 8 * c8));
  }
#pragma unroll
  for (int i = 0; i < kRowsPerThread; ++i) {
    if (dst[i] < 0) continue;
    *reinterpret_cast<uint4*>(p.out + dst[i] * p.out_stride_s +
                              head * p.out_stride_h + 8 * c8) = vals[i];
  }
}

__global__ void gather_lse_kernel(const float* lse, int64_t ls, int64_t lh,
                                  const int64_t* perm, int64_t n_slots,
                                  const int64_t* heads, int n_heads,
                                  float* out) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x +
                    threadIdx.x;
  if (i >= n_slots * n_heads) return;
  const int64_t slot = i / n_heads;
  const int h = static_cast<int>(i % n_heads);
  const int64_t src = perm[slot];
  out[i] = src >= 0 ? lse[src * ls + heads[h] * lh] : 0.f;
}

int launch_gather(const GatherParams& p, int64_t n_tiles, int32_t n_heads,
                  void* stream) {
  VEDA_REQUIRE(n_tiles * n_heads < (int64_t(1) << 31), "too many tiles");
  const unsigned grid = static_cast<unsigned>(n_tiles * n_heads);
  if (p.sq != nullptr || p.var != nullptr)
    gather_pool_kernel<2><<<grid, kPoolThreads, 0, as_stream(stream)>>>(
        p, n_tiles);
  else if (p.feats != nullptr)
    gather_pool_kernel<1><<<grid, kPoolThreads, 0, as_stream(stream)>>>(
        p, n_tiles);
  else
    gather_pool_kernel<0><<<grid, kPoolThreads, 0, as_stream(stream)>>>(
        p, n_tiles);
  return check_launch("gather_pool_kernel");
}

// Head-block exchange layout for the head-parallel all-to-all. The
// strided side holds, per row, `blocks` segments of w bytes at
// row * row_bytes + b * block_bytes + offset; the packed side holds them as
// [block][row][w]. pack copies strided -> packed, unpack the reverse.
// 16-byte vectors (all sizes are multiples of 16), grid-stride.
__global__ void head_blocks_kernel(const uint4* __restrict__ src,
                                   uint4* __restrict__ dst, int64_t rows,
                                   int blocks, int64_t w16, int64_t row16,
                                   int64_t block16, int64_t off16, int pack) {
  const int64_t total = rows * blocks * w16;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x +
                   threadIdx.x;
       i < total; i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t j = i % w16;
    const int64_t r = (i / w16) % rows;
    const int64_t b = i / (w16 * rows);
    const int64_t strided = r * row16 + b * block16 + off16 + j;
    if (pack)
      dst[i] = src[strided];
    else
      dst[strided] = src[i];
  }
}

int check_rows(const void* p, int64_t stride_row, int64_t stride_head,
               const char* name) {
  if (reinterpret_cast<uintptr_t>(p) % 16 != 0 || stride_row % 8 != 0 ||
      stride_head % 8 != 0)
    return set_error(VEDA_ERR_INVALID,
                     std::string(name) +
                         " must be 16-byte aligned with row/head strides "
                         "that are multiples of 8 elements");
  return VEDA_OK;
}

}  // namespace

}  // namespace veda

using namespace veda;

extern "C" int veda_gather_pool(const void* x, int64_t x_stride_s,
                                int64_t x_stride_h, const int64_t* perm,
                                const int32_t* valid_count, int64_t n_tiles,
                                const int64_t* heads, int32_t n_heads,
                                void* out, int64_t out_stride_n,
                                int64_t out_stride_h, float* feats, float* sq,
                                float* var, void* stream) {
  VEDA_REQUIRE(x != nullptr && valid_count != nullptr,
               "x and valid_count are required");
  VEDA_REQUIRE(n_heads >= 1 && n_heads <= 65535, "bad number of heads");
  VEDA_REQUIRE(perm != nullptr || heads == nullptr,
               "heads needs a permutation (identity pooling uses all heads)");
  VEDA_REQUIRE(out != nullptr || feats != nullptr || sq != nullptr ||
                   var != nullptr,
               "nothing to compute");
  int rc = check_rows(x, x_stride_s, x_stride_h, "x");
  if (rc != VEDA_OK) return rc;
  if (out != nullptr) {
    rc = check_rows(out, out_stride_n, out_stride_h, "out");
    if (rc != VEDA_OK) return rc;
  }
  if (n_tiles == 0) return VEDA_OK;
  GatherParams p{};
  p.x = static_cast<const __nv_bfloat16*>(x);
  p.x_stride_s = x_stride_s;
  p.x_stride_h = x_stride_h;
  p.perm = perm;
  p.valid_count = valid_count;
  p.heads = heads;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_stride_n = out_stride_n;
  p.out_stride_h = out_stride_h;
  p.feats = feats;
  p.sq = sq;
  p.var = var;
  p.n_tiles = n_tiles;
  VEDA_REQUIRE(n_tiles * n_heads < (int64_t(1) << 31), "too many tiles");
  return launch_gather(p, n_tiles, n_heads, stream);
}

extern "C" int veda_gather_pool_images(const void* x, int64_t x_stride_s,
                                       int64_t x_stride_h,
                                       const int64_t* perm,
                                       const int32_t* valid_count,
                                       int64_t n_tiles, const int64_t* heads,
                                       int32_t n_heads, void* image,
                                       float* feats, void* stream) {
  VEDA_REQUIRE(x != nullptr && perm != nullptr && valid_count != nullptr &&
                   heads != nullptr && image != nullptr,
               "x, perm, valid_count, heads and image are required");
  VEDA_REQUIRE(n_heads >= 1 && n_heads <= 65535, "bad number of heads");
  VEDA_REQUIRE(reinterpret_cast<uintptr_t>(image) % 16 == 0,
               "image must be 16-byte aligned");
  int rc = check_rows(x, x_stride_s, x_stride_h, "x");
  if (rc != VEDA_OK) return rc;
  if (n_tiles == 0) return VEDA_OK;
  GatherParams p{};
  p.x = static_cast<const __nv_bfloat16*>(x);
  p.x_stride_s = x_stride_s;
  p.x_stride_h = x_stride_h;
  p.perm = perm;
  p.valid_count = valid_count;
  p.heads = heads;
  p.out = static_cast<__nv_bfloat16*>(image);
  p.image = 1;
  p.feats = feats;
  p.n_tiles = n_tiles;
  VEDA_REQUIRE(n_tiles * n_heads < (int64_t(1) << 31), "too many tiles");
  return launch_gather(p, n_tiles, n_heads, stream);
}

extern "C" int veda_scatter(const void* tiled, int64_t t_stride_n,
                            int64_t t_stride_h, const int64_t* perm,
                            int64_t n_tiles, const int64_t* heads,
                            int32_t n_heads, void* out, int64_t out_stride_s,
                            int64_t out_stride_h, void* stream) {
  VEDA_REQUIRE(tiled != nullptr && perm != nullptr && out != nullptr,
               "tiled, perm and out are required");
  VEDA_REQUIRE(n_heads >= 1 && n_heads <= 65535, "bad number of heads");
  int rc = check_rows(tiled, t_stride_n, t_stride_h, "tiled");
  if (rc != VEDA_OK) return rc;
  rc = check_rows(out, out_stride_s, out_stride_h, "out");
  if (rc != VEDA_OK) return rc;
  if (n_tiles == 0) return VEDA_OK;
  ScatterParams p{};
  p.tiled = static_cast<const __nv_bfloat16*>(tiled);
  p.t_stride_n = t_stride_n;
  p.t_stride_h = t_stride_h;
  p.perm = perm;
  p.heads = heads;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_stride_s = out_stride_s;
  p.out_stride_h = out_stride_h;
  VEDA_REQUIRE(n_tiles * n_heads < (int64_t(1) << 31), "too many tiles");
  scatter_kernel<<<static_cast<unsigned>(n_tiles * n_heads), kPoolThreads, 0,
                   as_stream(stream)>>>(p, n_tiles);
  return check_launch("scatter_kernel");
}

extern "C" int veda_gather_lse(const float* lse, int64_t l_stride_s,
                               int64_t l_stride_h, const int64_t* perm,
                               int64_t n_tiles, const int64_t* heads,
                               int32_t n_heads, float* out, void* stream) {
  VEDA_REQUIRE(lse != nullptr && perm != nullptr && heads != nullptr &&
                   out != nullptr,
               "lse, perm, heads and out are required");
  VEDA_REQUIRE(n_heads >= 1, "bad number of heads");
  const int64_t total = n_tiles * kTile * n_heads;
  if (total == 0) return VEDA_OK;
  const int threads = 256;
  gather_lse_kernel<<<static_cast<unsigned>((total + threads - 1) / threads),
                      threads, 0, as_stream(stream)>>>(
      lse, l_stride_s, l_stride_h, perm, n_tiles * kTile, heads, n_heads, out);
  return check_launch("gather_lse_kernel");
}

extern "C" int veda_head_blocks(const void* src, void* dst, int64_t rows,
                                int32_t blocks, int64_t seg_bytes,
                                int64_t row_bytes, int64_t block_bytes,
                                int64_t offset_bytes, int32_t pack,
                                void* stream) {
  VEDA_REQUIRE(src != nullptr && dst != nullptr && src != dst,
               "src and dst must be distinct buffers");
  VEDA_REQUIRE(rows >= 0 && blocks >= 1 && seg_bytes >= 16,
               "bad shape");
  VEDA_REQUIRE(seg_bytes % 16 == 0 && row_bytes % 16 == 0 &&
                   block_bytes % 16 == 0 && offset_bytes % 16 == 0,
               "sizes and offsets must be multiples of 16 bytes");
  VEDA_REQUIRE(offset_bytes >= 0 && offset_bytes + seg_bytes <= block_bytes &&
                   static_cast<int64_t>(blocks) * block_bytes <= row_bytes,
               "segments must lie inside their blocks and rows");
  VEDA_REQUIRE(reinterpret_cast<uintptr_t>(src) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(dst) % 16 == 0,
               "src and dst must be 16-byte aligned");
  const int64_t total = rows * blocks * (seg_bytes / 16);
  if (total == 0) return VEDA_OK;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int threads = 256;
  const int64_t want = (total + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(sms) * 8;
  head_blocks_kernel<<<static_cast<unsigned>(want < cap ? want : cap),
                       threads, 0, as_stream(stream)>>>(
      static_cast<const uint4*>(src), static_cast<uint4*>(dst), rows, blocks,
      seg_bytes / 16, row_bytes / 16, block_bytes / 16, offset_bytes / 16,
      pack);
  return check_launch("head_blocks_kernel");
}
