// a13: teacher block heat on tcgen05.
//
// Semantics (miowtion/veda/heatmap.py:36-99; the reference's fused Triton
// kernel miowtion/kernels/block_heat_triton.py:93-137 computes the same):
// for query tile r of `q_tiles` and key tile t, with s = q.k rounded to bf16
// (what the reference's bf16 bmm returns), scale = 1/sqrt(D) and the dense
// teacher's natural-log LSE L of each query row,
//   reduce max:  heat[h, r, t] = exp(max over valid rows i and valid keys j
//                                    of s_ij * scale - L_i)
//   reduce sum:  heat[h, r, t] = sum over valid rows i and valid keys j of
//                                    exp(s_ij * scale - L_i)
// with 0 where the tile has no valid row or key. Valid rows and keys are the
// prefix valid_count[tile] of each tile.
//
// Structure: a persistent kernel, one CTA per SM, items (head, query tile)
// with a stride of the grid (every item has n_tiles blocks, so the split is
// even). Q of the item stays in shared memory; key tiles stream through a
// 4-slot ring; S = Q K^T (8 SS MMAs, M=N=128, K=16) goes to one of four TMEM
// buffers (512 columns), so the tensor core runs up to four blocks ahead of
// the reduction. Warp w (0-15) reduces rows 32(w%4) .. +31 (its TMEM lanes)
// over keys 32(w/4) .. +31 to one partial per block; four such warps per
// SMSP hide one another's latencies. For reduce='sum' (one exponential per
// score, so the MUFU's 16 ex2 a clock per SM bound it) a quarter of the
// exponentials run on the FMA pipes (exp2_poly.cuh). Warp 16 issues TMA,
// warp 17 the MMAs (converged, elected lane), and warp 18 combines each
// block's sixteen partials into its heat, off the other two warps' paths.
// All waits are bounded (common.cuh).
#include <math.h>

#include "common.cuh"
#include "exp2_poly.cuh"

namespace veda {

namespace {

constexpr int kWarps = 16;  // reduction warps
constexpr int kProducerWarp = kWarps;
constexpr int kMmaWarp = kWarps + 1;
constexpr int kWriterWarp = kWarps + 2;
constexpr int kHeatThreads = 32 * (kWarps + 3);
// Of each warp's 32 columns, those whose exponential (reduce='sum') runs on
// the FMA pipes.
constexpr int kPolyCols = 8;
constexpr int kSBufs = 4;
constexpr int kRing = 4;
constexpr uint32_t kTileBytes = 32768;
constexpr uint32_t kHalfBytes = 16384;
constexpr uint32_t kTileUnits = kTileBytes >> 4;
constexpr float kLog2e = 1.4426950408889634f;
constexpr int kHeatSmem = (2 + kRing) * kTileBytes + 1024 + 1024;

enum Bar {
  kQFull = 0,                  // [2] per Q buffer (item parity)
  kQEmpty = 2,                 // [2] the item's last QK finished
  kKFull = 4,                  // [kRing]
  kKEmpty = kKFull + kRing,    // [kRing]
  kSFull = kKEmpty + kRing,    // [kSBufs]
  kSFree = kSFull + kSBufs,    // [kSBufs] the warps read S, wrote partials
  kPartFree = kSFree + kSBufs,  // [kSBufs] the writer read the partials
  kDrain = kPartFree + kSBufs,
  kNumBars
};

struct HeatParams {
  int n_heads;
  int n_tiles;          // key tiles
  int n_q;              // supervised query tiles
  int n_items;          // n_heads * n_q
  const int32_t* valid_count;
  const int64_t* q_tiles;
  const float* lse;
  int64_t lse_sr, lse_sh;
  float* heat;          // [H][n_q][n_tiles]
  int sum;              // 0: max, 1: sum
  float scale_log2;     // scale * log2(e)
  unsigned int* status;
};

__device__ __forceinline__ bool wait_all(uint64_t* bar, uint32_t parity,
                                         volatile int* abort,
                                         unsigned int* status) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort, status));
}

__device__ __forceinline__ float round_bf16(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

__global__ void __launch_bounds__(kHeatThreads, 1)
    heat_kernel(const __grid_constant__ CUtensorMap map_q,
                const __grid_constant__ CUtensorMap map_k, HeatParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* s_q = smem;                      // [2]
  uint8_t* s_k = smem + 2 * kTileBytes;     // [kRing]
  float* s_part = reinterpret_cast<float*>(smem + (2 + kRing) * kTileBytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_part + kSBufs * kWarps);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tid = threadIdx.x;
  const int warp = tid / 32;
  const int lane = tid % 32;
  const int n = p.n_tiles;
  if (tid == 0) {
    for (int b = 0; b < kNumBars; ++b)
      mbar_init(&bars[b], (b >= kSFree && b < kSFree + kSBufs) ? kWarps : 1);
    *abort = 0;
    fence_barrier_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kProducerWarp) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      prefetch_tensor_map(&map_q);
      prefetch_tensor_map(&map_k);
    }
    int b = 0, ka = 0, q_loads = 0;
    bool run = true;
    for (int it = blockIdx.x; run && it < p.n_items; it += gridDim.x, ++ka) {
      const int h = it / p.n_q;
      const int qt = static_cast<int>(p.q_tiles[it % p.n_q]);
      const int qb = ka & 1;
      if (ka >= 2 && !wait_all(&bars[kQEmpty + qb], ((ka >> 1) & 1) ^ 1,
                               abort, p.status))
        break;
      if (lane == 0) {
        uint8_t* dst = s_q + qb * kTileBytes;
        mbar_arrive_expect_tx(&bars[kQFull + qb], kTileBytes);
        tma_load_3d(dst, &map_q, &bars[kQFull + qb], 0, h, qt * kTile);
        tma_load_3d(dst + kHalfBytes, &map_q, &bars[kQFull + qb], 64, h,
                    qt * kTile);
      }
      __syncwarp();
      q_loads = ka + 1;
      for (int t = 0; t < n; ++t, ++b) {
        const int slot = b % kRing;
        if (b >= kRing && !wait_all(&bars[kKEmpty + slot],
                                    ((b / kRing) - 1) & 1, abort, p.status)) {
          run = false;
          break;
        }
        if (lane == 0) {
          uint8_t* dst = s_k + slot * kTileBytes;
          mbar_arrive_expect_tx(&bars[kKFull + slot], kTileBytes);
          tma_load_3d(dst, &map_k, &bars[kKFull + slot], 0, h, t * kTile);
          tma_load_3d(dst + kHalfBytes, &map_k, &bars[kKFull + slot], 64, h,
                      t * kTile);
        }
        __syncwarp();
      }
    }
    if (lane == 0 && *abort) {
      volatile int never = 0;
      for (int k = q_loads - 2; k < q_loads; ++k)
        if (k >= 0)
          mbar_wait(&bars[kQFull + (k & 1)], (k >> 1) & 1, &never, nullptr);
      for (int k = b - kRing; k < b; ++k)
        if (k >= 0)
          mbar_wait(&bars[kKFull + k % kRing], (k / kRing) & 1, &never,
                    nullptr);
    }
  } else if (warp == kWriterWarp) {
    // ---------------- heat writer ----------------
    // Walks the same blocks as the other roles: block w of this CTA is key
    // tile t of item it.
    int64_t w = 0;
    bool run = true;
    for (int it = blockIdx.x; run && it < p.n_items; it += gridDim.x) {
      for (int t = 0; t < n; ++t, ++w) {
        const int sb = static_cast<int>(w % kSBufs);
        if (!wait_all(&bars[kSFree + sb], (w / kSBufs) & 1, abort,
                      p.status)) {
          run = false;
          break;
        }
        if (lane == 0) {
          float v;
          if (p.sum) {
            v = 0.f;
#pragma unroll
            for (int i = 0; i < kWarps; ++i) v += s_part[sb * kWarps + i];
          } else {
            v = -INFINITY;
#pragma unroll
            for (int i = 0; i < kWarps; ++i)
              v = fmaxf(v, s_part[sb * kWarps + i]);
            v = ex2_approx(v);  // partials are in log2 units
          }
          p.heat[static_cast<int64_t>(it) * n + t] = v;
          mbar_arrive(&bars[kPartFree + sb]);
        }
        __syncwarp();
      }
    }
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issuer ----------------
    constexpr uint32_t idesc = idesc_bf16(128, 128, false, false);
    const uint32_t q_lo = sw128_desc_lo(smem_u32(s_q), 16);
    const uint32_t k_lo = sw128_desc_lo(smem_u32(s_k), 16);
    int b = 0, ka = 0;
    bool run = true;
    for (int it = blockIdx.x; run && it < p.n_items; it += gridDim.x, ++ka) {
      const int qb = ka & 1;
      if (!wait_all(&bars[kQFull + qb], (ka >> 1) & 1, abort, p.status))
        break;
      for (int t = 0; t < n; ++t, ++b) {
        const int sb = b % kSBufs;
        const int slot = b % kRing;
        // S buffer sb is free once block b - kSBufs's partials are read.
        if (b >= kSBufs && !wait_all(&bars[kPartFree + sb],
                                     ((b / kSBufs) - 1) & 1, abort,
                                     p.status)) {
          run = false;
          break;
        }
        if (!wait_all(&bars[kKFull + slot], (b / kRing) & 1, abort,
                      p.status)) {
          run = false;
          break;
        }
        tc_fence_after();
        const uint32_t a = q_lo + qb * kTileUnits;
        const uint32_t bk = k_lo + slot * kTileUnits;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * (kHalfBytes >> 4) + (kk & 3) * 2;
          umma_ss_warp(tmem + sb * 128, a + off, bk + off, idesc, kk > 0);
        }
        umma_commit_warp(&bars[kSFull + sb]);
        umma_commit_warp(&bars[kKEmpty + slot]);
        if (t == n - 1) umma_commit_warp(&bars[kQEmpty + qb]);
      }
    }
    if (*abort) {
      volatile int never = 0;
      umma_commit_warp(&bars[kDrain]);
      mbar_wait(&bars[kDrain], 0, &never, nullptr);
    }
  } else {
    // ---------------- reduction warps 0-15 ----------------
    const int kq = warp / 4;  // keys 32 kq .. 32 kq + 31 of each block
    const int quarter = warp % 4;
    const int row = quarter * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    int b = 0;
    bool ok = true;
    for (int it = blockIdx.x; ok && it < p.n_items; it += gridDim.x) {
      const int h = it / p.n_q;
      const int qt = static_cast<int>(p.q_tiles[it % p.n_q]);
      const bool row_ok = row < p.valid_count[qt];
      const float l2 =
          row_ok ? p.lse[(static_cast<int64_t>(qt) * kTile + row) * p.lse_sr +
                         h * p.lse_sh] *
                       kLog2e
                 : 0.f;
      const float2 scale2 = make_float2(p.scale_log2, p.scale_log2);
      const float2 neg_l2 = make_float2(-l2, -l2);
      int kvalid_next = p.valid_count[0];
      for (int t = 0; t < n; ++t, ++b) {
        const int kvalid = kvalid_next;
        if (t + 1 < n) kvalid_next = p.valid_count[t + 1];
        const int sb = b % kSBufs;
        if (!wait_all(&bars[kSFull + sb], (b / kSBufs) & 1, abort,
                      p.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t r[32];
        tmem_ld32(tmem + sb * 128 + kq * 32 + lane_base, r);
        tmem_wait_ld();
        const int nk = kvalid - kq * 32;  // valid keys among these 32
        float v;
        if (p.sum) {
          // Keys past the valid prefix (partial tiles only) score -inf.
          if (nk < 32) {
#pragma unroll
            for (int c = 0; c < 32; ++c)
              if (c >= nk) r[c] = __float_as_uint(-INFINITY);
          }
          float2 acc = make_float2(0.f, 0.f);
#pragma unroll
          for (int c = 0; c < 32; c += 2) {
            // Scores rounded to bf16 (the reference's bmm output dtype).
            const float2 sr = __bfloat1622float2(__floats2bfloat162_rn(
                __uint_as_float(r[c]), __uint_as_float(r[c + 1])));
            const float2 x = __ffma2_rn(sr, scale2, neg_l2);
            const float2 e = c >= 32 - kPolyCols
                                 ? exp2_poly2(x)
                                 : make_float2(ex2_approx(x.x),
                                               ex2_approx(x.y));
            acc = __fadd2_rn(acc, e);
          }
          v = row_ok ? acc.x + acc.y : 0.f;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1)
            v += __shfl_xor_sync(0xffffffffu, v, o);
        } else {
          float m = -INFINITY;
#pragma unroll
          for (int c = 0; c < 32; ++c)
            if (c < nk) m = fmaxf(m, __uint_as_float(r[c]));
          // Rounding is monotone: the max of the rounded scores is the
          // rounded max.
          v = (row_ok && m > -INFINITY)
                  ? fmaf(round_bf16(m), p.scale_log2, -l2)
                  : -INFINITY;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1)
            v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
        }
        if (lane == 0) s_part[sb * kWarps + warp] = v;
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[kSFree + sb]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

}  // namespace veda

using namespace veda;

extern "C" int veda_teacher_heat(const void* q, int64_t q_stride_n,
                                 int64_t q_stride_h, const void* k,
                                 int64_t k_stride_n, int64_t k_stride_h,
                                 const float* lse, int64_t lse_stride_row,
                                 int64_t lse_stride_h, int32_t n_heads,
                                 int64_t n_tiles, const int32_t* valid_count,
                                 const int64_t* q_tiles, int64_t n_q,
                                 int32_t reduce_sum, float* heat,
                                 float softmax_scale, void* stream) {
  int rc = require_sm100("veda_teacher_heat");
  if (rc != VEDA_OK) return rc;
  VEDA_REQUIRE(q && k && lse && valid_count && heat && (q_tiles || n_q == 0),
               "q, k, lse, valid_count, q_tiles and heat are required");
  VEDA_REQUIRE(n_heads >= 1 && n_tiles >= 1 && n_q >= 0, "bad shape");
  VEDA_REQUIRE(n_q * n_heads < (int64_t(1) << 30) && n_tiles < (1 << 20),
               "too many tiles");
  VEDA_REQUIRE(softmax_scale > 0.f, "softmax_scale must be positive");
  if (n_q == 0) return VEDA_OK;
  CUtensorMap mq, mk;
  rc = make_tile_map(&mq, q, n_tiles * kTile, n_heads, q_stride_n, q_stride_h,
                     "q");
  if (rc == VEDA_OK)
    rc = make_tile_map(&mk, k, n_tiles * kTile, n_heads, k_stride_n,
                       k_stride_h, "k");
  if (rc != VEDA_OK) return rc;
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    VEDA_CUDA(cudaGetDevice(&dev));
    VEDA_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount,
                                     dev));
    VEDA_CUDA(cudaFuncSetAttribute(
        heat_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kHeatSmem));
  }
  HeatParams p{};
  p.n_heads = n_heads;
  p.n_tiles = static_cast<int>(n_tiles);
  p.n_q = static_cast<int>(n_q);
  p.n_items = static_cast<int>(n_q * n_heads);
  p.valid_count = valid_count;
  p.q_tiles = q_tiles;
  p.lse = lse;
  p.lse_sr = lse_stride_row;
  p.lse_sh = lse_stride_h;
  p.heat = heat;
  p.sum = reduce_sum ? 1 : 0;
  p.scale_log2 = softmax_scale * kLog2e;
  p.status = device_status_ptr();
  const int grid = p.n_items < sms ? p.n_items : sms;
  heat_kernel<<<grid, kHeatThreads, kHeatSmem, as_stream(stream)>>>(mq, mk, p);
  return check_launch("heat_kernel");
}
