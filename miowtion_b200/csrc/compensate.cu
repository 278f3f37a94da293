// (f) Zero-order compensation next to the sparse kernel
// (miowtion/kernels/compensation_triton.py:1-245; torch form
// miowtion/veda/attention.py:591-689).
//
// Every key tile the mask dropped is replaced by one virtual key at its
// centroid, mean_j k_j, carrying the value sum_j v_j and weighted by its
// real row count B_t. With the reference exponent taken as the sparse
// kernel's own log-sum-exp L (over the kept keys), the kept denominator is
// exactly 1 and each query row becomes
//
//   out = (o_kept + sum_dropped p_t vsum_t) / (1 + sum_dropped p_t B_t),
//   p_t = exp(q . kmean_t * scale - L)
//
// (L = 0 for a row whose L is not finite, as the reference does).
//
// Two kernels:
//  1. `comp_summary_kernel` (HBM-bound): per (key tile, head) the mean of k
//     and the sum of v over the tile's real rows, in fp32, stored as bf16
//     (the Triton form's precision) in a [n_pad, H, 128] workspace whose
//     rows n_tiles .. n_pad are zero.
//  2. `comp_kernel` (tcgen05): per (query tile, head), walk the centroids
//     in chunks of 128 tiles: S = Q . KC^T (SS MMA into one of three TMEM
//     S buffers), eight compute warps turn S into p (0 where the tile was
//     kept or is empty) and accumulate the weighted denominator, P goes
//     back over S in TMEM as bf16, and O += P . VC (TS MMA). The epilogue
//     combines O with o_kept. Persistent, one CTA per SM, 13 warps:
//     8 compute, a Q / key-centroid TMA warp, a value-sum TMA warp, an S
//     issuer (up to three chunks ahead), a P.V issuer, and a prep warp that
//     builds the next item's per-tile weights (row counts, 0 for the tiles
//     the forward's index lists kept) and LSE in shared memory.
#include "common.cuh"

namespace veda {

namespace {

constexpr int kCompWarps = 8;                   // compute warps
constexpr int kCompProducer = kCompWarps;       // TMA: Q, key centroids
constexpr int kCompSIssuer = kCompWarps + 1;    // S MMAs, TMEM owner
constexpr int kCompVProducer = kCompWarps + 2;  // TMA: value sums
constexpr int kCompPvIssuer = kCompWarps + 3;   // P.V MMAs
constexpr int kCompPrep = kCompWarps + 4;  // weights and LSE of the next item
constexpr int kCompThreads = 32 * (kCompWarps + 5);
constexpr uint32_t kTileBytes = 32768;
constexpr uint32_t kHalfBytes = 16384;
constexpr uint32_t kTileUnits = kTileBytes >> 4;
constexpr int kSBufs = 3;                // S / P buffers in TMEM
constexpr uint32_t kCompTmemCols = 512;  // S[3] 0..383, O 384..511
// Key tiles: their row counts and two items' weights sit in shared memory.
constexpr int kMaxTiles = 5120;

enum CompBar {
  kQFull = 0,
  kQEmpty,
  kKcFull,   // [2]
  kKcEmpty = kKcFull + 2,
  kVcFull = kKcEmpty + 2,
  kVcEmpty = kVcFull + 2,
  kSFull = kVcEmpty + 2,       // [3]
  kPFull = kSFull + kSBufs,    // [3], 8 warps
  kPvDone = kPFull + kSBufs,   // [3]
  kODone = kPvDone + kSBufs,
  kOFree,  // 8 warps
  kWFull,  // [2] weights and LSE of an item ready (prep warp)
  kWEmpty = kWFull + 2,  // [2] the compute warps are done with them (8)
  kDrainS = kWEmpty + 2,
  kDrainPv,
  kCompBars
};

struct CompParams {
  const __nv_bfloat16* o_kept;
  int64_t ok_sn, ok_sh;
  const float* lse;  // [H, n_q * 128] natural log
  int64_t lse_sh;
  const int32_t* valid_count;
  const int32_t *part_cnt, *part_idx, *full_cnt, *full_idx;
  int64_t ld_idx;
  __nv_bfloat16* out;
  int64_t out_sn, out_sh;
  int n_heads, n_q_tiles, n_kv_tiles, n_chunks, n_items;
  float scale_log2;
  unsigned int* status;
};

__device__ __forceinline__ bool wait_all(uint64_t* bar, uint32_t parity,
                                         volatile int* abort,
                                         unsigned int* status) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort, status));
}

__device__ __forceinline__ void arrive_warp(uint64_t* bar) {
  tc_fence_before();
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
}

// Named barrier of the eight compute warps.
__device__ __forceinline__ void compute_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(32 * kCompWarps) : "memory");
}

__device__ __forceinline__ void load_tile(uint8_t* dst,
                                          const CUtensorMap* map,
                                          uint64_t* bar, int h, int row0) {
  mbar_arrive_expect_tx(bar, kTileBytes);
  tma_load_3d(dst, map, bar, 0, h, row0);
  tma_load_3d(dst + kHalfBytes, map, bar, 64, h, row0);
}

// Grid (n_pad, H), 256 threads: thread t sums 8 columns (one 16-byte
// vector) of rows t/16, t/16 + 16, ...; the 16 row groups are combined in
// shared memory.
__global__ void __launch_bounds__(256)
    comp_summary_kernel(const __nv_bfloat16* __restrict__ k, int64_t ks,
                        int64_t kh, const __nv_bfloat16* __restrict__ v,
                        int64_t vs, int64_t vh,
                        const int32_t* __restrict__ valid_count, int n_tiles,
                        __nv_bfloat16* __restrict__ kc,
                        __nv_bfloat16* __restrict__ vc) {
  const int tile = blockIdx.x, h = blockIdx.y, n_heads = gridDim.y;
  const int rg = threadIdx.x / 16, c8 = threadIdx.x % 16;
  const int count = tile < n_tiles ? valid_count[tile] : 0;
  float sk[8] = {0.f}, sv[8] = {0.f};
  for (int i = rg; i < count; i += 16) {
    const int64_t row = static_cast<int64_t>(tile) * kTile + i;
    const uint4 a = *reinterpret_cast<const uint4*>(k + row * ks + h * kh +
                                                    c8 * 8);
    const uint4 b = *reinterpret_cast<const uint4*>(v + row * vs + h * vh +
                                                    c8 * 8);
    const __nv_bfloat162* pa = reinterpret_cast<const __nv_bfloat162*>(&a);
    const __nv_bfloat162* pb = reinterpret_cast<const __nv_bfloat162*>(&b);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 fa = __bfloat1622float2(pa[e]);
      const float2 fb = __bfloat1622float2(pb[e]);
      sk[2 * e] += fa.x;
      sk[2 * e + 1] += fa.y;
      sv[2 * e] += fb.x;
      sv[2 * e + 1] += fb.y;
    }
  }
  __shared__ float s_k[16][kHeadDim], s_v[16][kHeadDim];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    s_k[rg][c8 * 8 + e] = sk[e];
    s_v[rg][c8 * 8 + e] = sv[e];
  }
  __syncthreads();
  if (threadIdx.x < kHeadDim) {
    const int d = threadIdx.x;
    float a = 0.f, b = 0.f;
    for (int g = 0; g < 16; ++g) {
      a += s_k[g][d];
      b += s_v[g][d];
    }
    const int64_t o = (static_cast<int64_t>(tile) * n_heads + h) * kHeadDim +
                      d;
    kc[o] = __float2bfloat16_rn(count > 0 ? a / static_cast<float>(count)
                                          : 0.f);
    vc[o] = __float2bfloat16_rn(b);
  }
}

// Thirteen warps: per SMSP at most four, so at most 128 registers each.
__global__ void __maxnreg__(128)
    comp_kernel(const __grid_constant__ CUtensorMap map_q,
                const __grid_constant__ CUtensorMap map_kc,
                const __grid_constant__ CUtensorMap map_vc,
                const CompParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* s_q = smem;
  uint8_t* s_kc = s_q + kTileBytes;       // [2]
  uint8_t* s_vc = s_kc + 2 * kTileBytes;  // [2]
  const int n_pad = p.n_chunks * kTile;
  // Weight of every key tile for a query tile: its real row count if
  // dropped, 0 if kept, empty or past the last tile. [2 items][n_pad],
  // 1024-byte aligned (read as float4).
  float* s_w = reinterpret_cast<float*>(s_vc + 2 * kTileBytes);
  float* s_cnt = s_w + 2 * n_pad;     // [n_pad] real row counts
  float* s_den = s_cnt + n_pad;       // [2 items][2 halves][128 rows]
  float* s_lse = s_den + 4 * kTile;   // [2 items][128 rows], log2 units
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_lse + 2 * kTile);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kCompBars);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    for (int b = 0; b < kCompBars; ++b) {
      const bool by_compute = (b >= kPFull && b < kPFull + kSBufs) ||
                              b == kOFree || b == kWEmpty || b == kWEmpty + 1;
      mbar_init(&bars[b], by_compute ? kCompWarps : 1);
    }
    *abort = 0;
    fence_barrier_init();
  }
  if (warp == kCompSIssuer) {
    tmem_alloc(tmem_slot, kCompTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int nc = p.n_chunks;

  if (warp == kCompProducer) {
    // ---------------- TMA producer: Q and key centroids ----------------
    if (lane == 0) {
      prefetch_tensor_map(&map_q);
      prefetch_tensor_map(&map_kc);
    }
    int g = 0, it = 0;
    bool ok = true;
    for (int item = blockIdx.x; ok && item < p.n_items;
         item += gridDim.x, ++it) {
      const int r = item / p.n_heads, h = item % p.n_heads;
      if (it > 0 &&
          !wait_all(&bars[kQEmpty], (it - 1) & 1, abort, p.status)) {
        ok = false;
        break;
      }
      if (lane == 0) load_tile(s_q, &map_q, &bars[kQFull], h, r * kTile);
      __syncwarp();
      for (int c = 0; c < nc; ++c, ++g) {
        const int s = g & 1;
        if (g >= 2 && !wait_all(&bars[kKcEmpty + s], ((g >> 1) - 1) & 1,
                                abort, p.status)) {
          ok = false;
          break;
        }
        if (lane == 0)
          load_tile(s_kc + s * kTileBytes, &map_kc, &bars[kKcFull + s], h,
                    c * kTile);
        __syncwarp();
      }
    }
    if (lane == 0 && *abort) {
      // Let the copies in flight land before the CTA exits.
      volatile int never = 0;
      for (int b = g - 2; b < g; ++b)
        if (b >= 0)
          mbar_wait(&bars[kKcFull + (b & 1)], (b >> 1) & 1, &never, nullptr);
      if (it > 0) mbar_wait(&bars[kQFull], (it - 1) & 1, &never, nullptr);
    }
  } else if (warp == kCompVProducer) {
    // ---------------- TMA producer: value sums ----------------
    // Its own warp, so that a value load waiting for a P.V MMA never holds
    // up the key loads.
    if (lane == 0) prefetch_tensor_map(&map_vc);
    int g = 0;
    bool ok = true;
    for (int item = blockIdx.x; ok && item < p.n_items; item += gridDim.x) {
      const int h = item % p.n_heads;
      for (int c = 0; c < nc; ++c, ++g) {
        const int s = g & 1;
        if (g >= 2 && !wait_all(&bars[kVcEmpty + s], ((g >> 1) - 1) & 1,
                                abort, p.status)) {
          ok = false;
          break;
        }
        if (lane == 0)
          load_tile(s_vc + s * kTileBytes, &map_vc, &bars[kVcFull + s], h,
                    c * kTile);
        __syncwarp();
      }
    }
    if (lane == 0 && *abort) {
      volatile int never = 0;
      for (int b = g - 2; b < g; ++b)
        if (b >= 0)
          mbar_wait(&bars[kVcFull + (b & 1)], (b >> 1) & 1, &never, nullptr);
    }
  } else if (warp == kCompSIssuer) {
    // ---------------- S = Q . KC^T, up to three chunks ahead ----------------
    constexpr uint32_t idesc_s = idesc_bf16(128, 128, false, false);
    const uint32_t q_lo = sw128_desc_lo(smem_u32(s_q), 16);
    const uint32_t kc_lo = sw128_desc_lo(smem_u32(s_kc), 16);
    int g = 0, it = 0;
    bool ok = true;
    for (int item = blockIdx.x; ok && item < p.n_items;
         item += gridDim.x, ++it) {
      if (!wait_all(&bars[kQFull], it & 1, abort, p.status)) break;
      for (int c = 0; c < nc; ++c, ++g) {
        const int s = g & 1, sb = g % kSBufs;
        // S buffer sb held P of chunk g - 3: its P.V must have read it.
        if (!wait_all(&bars[kKcFull + s], (g >> 1) & 1, abort, p.status) ||
            (g >= kSBufs &&
             !wait_all(&bars[kPvDone + sb], (g / kSBufs - 1) & 1, abort,
                       p.status))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t bk = kc_lo + s * kTileUnits;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * (kHalfBytes >> 4) + (kk & 3) * 2;
          umma_ss_warp(tmem + sb * 128, q_lo + off, bk + off, idesc_s,
                       kk > 0 ? 1u : 0u);
        }
        umma_commit_warp(&bars[kKcEmpty + s]);
        umma_commit_warp(&bars[kSFull + sb]);
        if (c == nc - 1) umma_commit_warp(&bars[kQEmpty]);
      }
    }
    if (*abort) {
      volatile int never = 0;
      umma_commit_warp(&bars[kDrainS]);
      mbar_wait(&bars[kDrainS], 0, &never, nullptr);
    }
  } else if (warp == kCompPvIssuer) {
    // ---------------- O (+)= P . VC ----------------
    constexpr uint32_t idesc_pv = idesc_bf16(128, 128, false, true);
    const uint32_t vc_lo = sw128_desc_lo(smem_u32(s_vc), kHalfBytes);
    const uint32_t t_o = tmem + kSBufs * 128;
    int g = 0, it = 0;
    bool ok = true;
    for (int item = blockIdx.x; ok && item < p.n_items;
         item += gridDim.x, ++it) {
      for (int c = 0; c < nc; ++c, ++g) {
        const int s = g & 1, sb = g % kSBufs;
        // The item's first P.V overwrites O: the epilogue must have read
        // the previous item's.
        if ((c == 0 && it > 0 &&
             !wait_all(&bars[kOFree], (it - 1) & 1, abort, p.status)) ||
            !wait_all(&bars[kVcFull + s], (g >> 1) & 1, abort, p.status) ||
            !wait_all(&bars[kPFull + sb], (g / kSBufs) & 1, abort,
                      p.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t t_p = tmem + sb * 128;
        const uint32_t bv = vc_lo + s * kTileUnits;
        // P of keys 16kk .. 16kk + 15: half kk / 4 holds its 64 keys packed
        // in its first 32 columns.
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_ts_warp(t_o, t_p + (kk >> 2) * 64 + (kk & 3) * 8,
                       bv + kk * 128, idesc_pv, (kk > 0 || c > 0) ? 1u : 0u);
        umma_commit_warp(&bars[kVcEmpty + s]);
        umma_commit_warp(&bars[kPvDone + sb]);
        if (c == nc - 1) umma_commit_warp(&bars[kODone]);
      }
    }
    if (*abort) {
      volatile int never = 0;
      umma_commit_warp(&bars[kDrainPv]);
      mbar_wait(&bars[kDrainPv], 0, &never, nullptr);
    }
  } else if (warp == kCompPrep) {
    // ---------------- prep: weights and LSE, one item ahead ----------------
    for (int t = lane; t < n_pad; t += 32)
      s_cnt[t] = t < p.n_kv_tiles ? static_cast<float>(p.valid_count[t])
                                  : 0.f;
    __syncwarp();
    int it = 0;
    for (int item = blockIdx.x; item < p.n_items; item += gridDim.x, ++it) {
      const int r = item / p.n_heads, h = item % p.n_heads;
      const int b = it & 1;
      if (it >= 2 && !wait_all(&bars[kWEmpty + b], ((it >> 1) - 1) & 1,
                               abort, p.status))
        break;
      float* w = s_w + b * n_pad;
      for (int t = 4 * lane; t < n_pad; t += 128)
        *reinterpret_cast<float4*>(w + t) =
            *reinterpret_cast<const float4*>(s_cnt + t);
      __syncwarp();
      const int64_t li = static_cast<int64_t>(h) * p.n_q_tiles + r;
      const int np = p.part_cnt[li], nf = p.full_cnt[li];
      for (int e = lane; e < np + nf; e += 32) {
        const int t = e < np ? p.part_idx[li * p.ld_idx + e]
                             : p.full_idx[li * p.ld_idx + (e - np)];
        if (t >= 0 && t < p.n_kv_tiles) w[t] = 0.f;
      }
      for (int i = lane; i < kTile; i += 32) {
        const float l = p.lse[h * p.lse_sh + static_cast<int64_t>(r) * kTile +
                              i];
        s_lse[b * kTile + i] = isfinite(l) ? l * 1.4426950408889634f : 0.f;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[kWFull + b]);
    }
  } else {
    // ---------------- compute warps 0-7 ----------------
    const int quarter = warp % 4, half = warp / 4;
    const int row = quarter * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    int g = 0, it = 0;
    bool ok = true;
    for (int item = blockIdx.x; ok && item < p.n_items;
         item += gridDim.x, ++it) {
      const int r = item / p.n_heads, h = item % p.n_heads;
      const int wb = it & 1;
      const int64_t q_row = static_cast<int64_t>(r) * kTile + row;
      const __nv_bfloat16* src = p.o_kept + q_row * p.ok_sn + h * p.ok_sh +
                                 half * 64;
      // This row's o_kept (one 128-byte line) is read in the epilogue:
      // bring it into L2 now.
      asm volatile("prefetch.global.L2 [%0];" ::"l"(src));
      if (!wait_all(&bars[kWFull + wb], (it >> 1) & 1, abort, p.status)) {
        ok = false;
        break;
      }
      const float l2 = s_lse[wb * kTile + row];
      // Four partial sums keep the denominator's FMA chain short.
      float den4[4] = {0.f, 0.f, 0.f, 0.f};
      for (int c = 0; c < nc; ++c, ++g) {
        const int sb = g % kSBufs;
        if (!wait_all(&bars[kSFull + sb], (g / kSBufs) & 1, abort,
                      p.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float* w_s = s_w + wb * n_pad + c * kTile + half * 64;
        const uint32_t t_s = tmem + sb * 128 + half * 64 + lane_base;
#pragma unroll 1
        for (int sub = 0; sub < 2; ++sub) {
          uint32_t x[32], pk[16];
          tmem_ld32(t_s + sub * 32, x);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float4 w =
                *reinterpret_cast<const float4*>(w_s + sub * 32 + 4 * i);
            const float wv[4] = {w.x, w.y, w.z, w.w};
            float e[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              e[j] = ex2_approx(
                  fmaf(__uint_as_float(x[4 * i + j]), p.scale_log2, -l2));
              e[j] = wv[j] > 0.f ? e[j] : 0.f;
              den4[j] = fmaf(e[j], wv[j], den4[j]);
            }
            pk[2 * i] = pack_bf16(e[0], e[1]);
            pk[2 * i + 1] = pack_bf16(e[2], e[3]);
          }
          // P of these 32 keys over the first half of this warp's S
          // columns (keys 64 half + k in column 64 half + k / 2).
          tmem_st16(t_s + sub * 16, pk);
        }
        tmem_wait_st();
        arrive_warp(&bars[kPFull + sb]);
      }
      if (!ok) break;
      uint4 okept[8];
#pragma unroll
      for (int v8 = 0; v8 < 8; ++v8)
        okept[v8] = *reinterpret_cast<const uint4*>(src + v8 * 8);
      // This item's weights and LSE are no longer read.
      arrive_warp(&bars[kWEmpty + wb]);
      // Epilogue: the two column halves' denominators, then O.
      float* den_x = s_den + wb * 2 * kTile;
      den_x[half * kTile + row] = (den4[0] + den4[1]) + (den4[2] + den4[3]);
      compute_sync();
      const float inv = 1.f / (1.f + den_x[row] + den_x[kTile + row]);
      if (!wait_all(&bars[kODone], it & 1, abort, p.status)) break;
      tc_fence_after();
      __nv_bfloat16* dst = p.out + q_row * p.out_sn + h * p.out_sh +
                           half * 64;
#pragma unroll
      for (int part = 0; part < 2; ++part) {
        uint32_t o[32];
        tmem_ld32(tmem + kSBufs * 128 + half * 64 + part * 32 + lane_base, o);
        tmem_wait_ld();
        if (part == 1) arrive_warp(&bars[kOFree]);
#pragma unroll
        for (int v8 = 0; v8 < 4; ++v8) {
          const __nv_bfloat162* pa =
              reinterpret_cast<const __nv_bfloat162*>(&okept[part * 4 + v8]);
          uint4 res;
          uint32_t* pr = reinterpret_cast<uint32_t*>(&res);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __bfloat1622float2(pa[e]);
            pr[e] = pack_bf16((f.x + __uint_as_float(o[v8 * 8 + 2 * e])) * inv,
                              (f.y + __uint_as_float(o[v8 * 8 + 2 * e + 1])) *
                                  inv);
          }
          *reinterpret_cast<uint4*>(dst + part * 32 + v8 * 8) = res;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kCompSIssuer) {
    tc_fence_after();
    tmem_dealloc(tmem, kCompTmemCols);
  }
}

size_t comp_smem_bytes(int64_t n_kv_tiles) {
  const int64_t n_pad = (n_kv_tiles + kTile - 1) / kTile * kTile;
  return 1024 + 5 * kTileBytes + 3 * n_pad * sizeof(float) +
         6 * kTile * sizeof(float) + kCompBars * sizeof(uint64_t) + 16;
}

}  // namespace

}  // namespace veda

using namespace veda;

extern "C" int64_t veda_compensate_workspace(int32_t n_heads,
                                             int64_t n_kv_tiles) {
  const int64_t n_pad = (n_kv_tiles + kTile - 1) / kTile * kTile;
  return 2 * n_pad * n_heads * kHeadDim * 2;
}

extern "C" int veda_compensate(
    const void* o_kept, int64_t ok_stride_n, int64_t ok_stride_h,
    const float* lse_kept, const void* q, int64_t q_stride_n,
    int64_t q_stride_h, const void* k, int64_t k_stride_n, int64_t k_stride_h,
    const void* v, int64_t v_stride_n, int64_t v_stride_h, int32_t n_heads,
    int64_t n_q_tiles, int64_t n_kv_tiles, const int32_t* valid_count,
    const int32_t* part_cnt, const int32_t* part_idx, const int32_t* full_cnt,
    const int32_t* full_idx, int64_t ld_idx, void* out, int64_t out_stride_n,
    int64_t out_stride_h, float softmax_scale, void* workspace,
    int64_t workspace_bytes, void* stream) {
  int rc = require_sm100("veda_compensate");
  if (rc != VEDA_OK) return rc;
  VEDA_REQUIRE(o_kept && lse_kept && q && k && v && valid_count && part_cnt &&
                   part_idx && full_cnt && full_idx && out,
               "o_kept, lse_kept, q, k, v, valid_count, the four lists and "
               "out are required");
  VEDA_REQUIRE(n_heads >= 1 && n_heads <= 65535 && n_q_tiles >= 0 &&
                   n_kv_tiles >= 1 && n_kv_tiles <= kMaxTiles,
               "bad shape (at most 5120 key tiles)");
  VEDA_REQUIRE(ld_idx >= n_kv_tiles, "ld_idx must be >= n_kv_tiles");
  VEDA_REQUIRE(n_q_tiles * n_heads < (int64_t(1) << 30), "too many tiles");
  VEDA_REQUIRE(softmax_scale > 0.f, "softmax_scale must be positive");
  VEDA_REQUIRE(reinterpret_cast<uintptr_t>(out) % 16 == 0 &&
                   out_stride_n % 8 == 0 && out_stride_h % 8 == 0 &&
                   reinterpret_cast<uintptr_t>(o_kept) % 16 == 0 &&
                   ok_stride_n % 8 == 0 && ok_stride_h % 8 == 0 &&
                   reinterpret_cast<uintptr_t>(k) % 16 == 0 &&
                   k_stride_n % 8 == 0 && k_stride_h % 8 == 0 &&
                   reinterpret_cast<uintptr_t>(v) % 16 == 0 &&
                   v_stride_n % 8 == 0 && v_stride_h % 8 == 0,
               "o_kept, out, k and v must be 16-byte aligned with strides "
               "multiple of 8");
  VEDA_REQUIRE(workspace != nullptr &&
                   workspace_bytes >=
                       veda_compensate_workspace(n_heads, n_kv_tiles) &&
                   reinterpret_cast<uintptr_t>(workspace) % 16 == 0,
               "workspace too small (veda_compensate_workspace) or "
               "misaligned");
  const int64_t n_pad = (n_kv_tiles + kTile - 1) / kTile * kTile;
  __nv_bfloat16* kc = static_cast<__nv_bfloat16*>(workspace);
  __nv_bfloat16* vc = kc + n_pad * n_heads * kHeadDim;
  cudaStream_t s = as_stream(stream);
  comp_summary_kernel<<<dim3(static_cast<unsigned>(n_pad),
                             static_cast<unsigned>(n_heads)),
                        256, 0, s>>>(
      static_cast<const __nv_bfloat16*>(k), k_stride_n, k_stride_h,
      static_cast<const __nv_bfloat16*>(v), v_stride_n, v_stride_h,
      valid_count, static_cast<int>(n_kv_tiles), kc, vc);
  rc = check_launch("comp_summary_kernel");
  if (rc != VEDA_OK || n_q_tiles == 0) return rc;
  CUtensorMap mq, mkc, mvc;
  rc = make_tile_map(&mq, q, n_q_tiles * kTile, n_heads, q_stride_n,
                     q_stride_h, "q");
  if (rc == VEDA_OK)
    rc = make_tile_map(&mkc, kc, n_pad, n_heads, n_heads * kHeadDim,
                       kHeadDim, "key centroids");
  if (rc == VEDA_OK)
    rc = make_tile_map(&mvc, vc, n_pad, n_heads, n_heads * kHeadDim,
                       kHeadDim, "value sums");
  if (rc != VEDA_OK) return rc;
  CompParams p{};
  p.o_kept = static_cast<const __nv_bfloat16*>(o_kept);
  p.ok_sn = ok_stride_n;
  p.ok_sh = ok_stride_h;
  p.lse = lse_kept;
  p.lse_sh = n_q_tiles * kTile;
  p.valid_count = valid_count;
  p.part_cnt = part_cnt;
  p.part_idx = part_idx;
  p.full_cnt = full_cnt;
  p.full_idx = full_idx;
  p.ld_idx = ld_idx;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_sn = out_stride_n;
  p.out_sh = out_stride_h;
  p.n_heads = n_heads;
  p.n_q_tiles = static_cast<int>(n_q_tiles);
  p.n_kv_tiles = static_cast<int>(n_kv_tiles);
  p.n_chunks = static_cast<int>(n_pad / kTile);
  p.n_items = static_cast<int>(n_q_tiles * n_heads);
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  p.status = device_status_ptr();
  static int sms = 0;
  static size_t configured = 0;
  const size_t smem = comp_smem_bytes(n_kv_tiles);
  if (sms == 0) {
    int dev = 0;
    VEDA_CUDA(cudaGetDevice(&dev));
    VEDA_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount,
                                     dev));
  }
  if (smem > configured) {
    VEDA_CUDA(cudaFuncSetAttribute(comp_kernel,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(comp_smem_bytes(
                                       kMaxTiles))));
    configured = comp_smem_bytes(kMaxTiles);
  }
  const int grid = p.n_items < sms ? p.n_items : sms;
  comp_kernel<<<grid, kCompThreads, smem, s>>>(mq, mkc, mvc, p);
  return check_launch("comp_kernel");
}
