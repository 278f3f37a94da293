// a9/a11: block-sparse (and dense) attention forward on tcgen05.
//
// Semantics (miowtion/kernels/reference.py:1-10, :23-56): a query row of tile
// i attends to the valid prefix of every key tile listed for i; rows with no
// key output 0 (lse -inf). Lists are the reference's BlockSparseTensors
// (miowtion/kernels/fa4.py:266-296); the walk order is the SM100 one of the
// reference backend, partial list then full list, each from its end
// (fa4_sm8x/block_sparse_utils.py:813-853), which only affects the fp32
// summation order.
//
// One CTA per (head, query tile), two CTAs per SM, 6 warps:
//   warps 0-3  softmax + epilogue; thread t owns query row t (TMEM lane t)
//   warp 4     TMA producer: Q once, then K and V of each listed key tile
//   warp 5     TMEM allocator and the single-thread tcgen05.mma issuer
// Per listed key tile j:
//   S = Q K^T          tcgen05.mma, A/B K-major from 128B-swizzled smem,
//                      fp32 accumulator in TMEM columns [0, 128)
//   P = exp2(S*c - m)  softmax warps: tcgen05.ld S, mask the key tile's
//                      padding suffix, online max with lazy rescaling (only
//                      when the running max grows by more than 2^8), write
//                      P as bf16 pairs back over S (columns [0, 64))
//   O += P V           tcgen05.mma with A = P from TMEM, B = V MN-major from
//                      smem, accumulator in TMEM columns [128, 256)
// The two co-resident CTAs interleave: one CTA's exponentials overlap the
// other's MMAs. All mbarrier waits are bounded (common.cuh).
#include <math.h>

#include "common.cuh"

namespace veda {

namespace {

constexpr int kFwdThreads = 192;
constexpr uint32_t kTileBytes = 32768;  // 128 x 128 bf16
constexpr uint32_t kHalfBytes = 16384;  // 128 x 64 bf16 (one TMA box)
constexpr uint32_t kTmemCols = 256;
constexpr int kSmemBytes = 3 * kTileBytes + 256 + 1024;

enum Bar {
  kQFull = 0,
  kKFull,
  kKEmpty,
  kVFull,
  kVEmpty,
  kSFull,
  kPFull0,  // P columns for keys 0-63 written
  kPFull1,  // P columns for keys 64-127 written
  kODone,
  kDrain,
  kNumBars
};

struct FwdParams {
  int n_heads;
  int n_q_tiles;
  int n_kv_tiles;
  const int32_t* valid_count;
  const int32_t* part_cnt;
  const int32_t* part_idx;
  const int32_t* full_cnt;
  const int32_t* full_idx;
  int64_t ld_idx;
  __nv_bfloat16* out;
  int64_t out_stride_n, out_stride_h;
  float* lse;
  int64_t lse_stride_row, lse_stride_h;
  float scale_log2;
  int dense;     // dense mode: every key tile [0, n_kv_tiles), keys < used
  int64_t used;  // dense mode only
  unsigned int* status;
};

// Key tile of step j and the number of valid keys in it (128 when full).
struct Step {
  int kv;
  int valid;
};

__device__ __forceinline__ Step block_at(const FwdParams& p, int j, int pc,
                                         int fc, int64_t list_off) {
  Step s;
  if (p.dense) {
    s.kv = j;
    const int64_t rest = p.used - static_cast<int64_t>(j) * kTile;
    s.valid = rest < kTile ? static_cast<int>(rest) : kTile;
  } else if (j < pc) {
    s.kv = p.part_idx[list_off + (pc - 1 - j)];
    s.valid = p.valid_count[s.kv];
  } else {
    s.kv = p.full_idx[list_off + (fc - 1 - (j - pc))];
    s.valid = kTile;
  }
  return s;
}

// Columns of each 128-key block whose exponential runs on the FMA pipes.
constexpr int kPolyCols = 32;

__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Max of 128 values as a shallow tree of three-input max instructions.
__device__ __forceinline__ float row_max128(const float* s) {
  float m[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) m[i] = s[i];
#pragma unroll
  for (int c = 8; c < 120; c += 16)
#pragma unroll
    for (int i = 0; i < 8; ++i) m[i] = max3(m[i], s[c + i], s[c + 8 + i]);
#pragma unroll
  for (int i = 0; i < 8; ++i) m[i] = fmaxf(m[i], s[120 + i]);
  return max3(max3(m[0], m[1], m[2]), max3(m[3], m[4], m[5]),
              fmaxf(m[6], m[7]));
}

// 2^x on the FMA pipes for a pair of values: x = n + f with n = rint(x),
// f in [-1/2, 1/2]; 2^f from the degree-3 minimax polynomial fitted by
// csrc/fit_exp2_poly.py (max relative error 7.5e-5); 2^n added to the
// exponent field. Arguments below -125 (masked keys) give ~0.
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23: rounds to integers
  x.x = fmaxf(x.x, -125.0f);
  x.y = fmaxf(x.y, -125.0f);
  const float2 t = __fadd2_rn(x, make_float2(kRound, kRound));
  const float2 n = __fadd2_rn(t, make_float2(-kRound, -kRound));
  const float2 f = __ffma2_rn(n, make_float2(-1.0f, -1.0f), x);
  float2 q = __ffma2_rn(f, make_float2(0x1.c3f76p-5f, 0x1.c3f76p-5f),
                        make_float2(0x1.f0de1ap-3f, 0x1.f0de1ap-3f));
  q = __ffma2_rn(q, f, make_float2(0x1.62f31ap-1f, 0x1.62f31ap-1f));
  q = __ffma2_rn(q, f, make_float2(0x1.fff692p-1f, 0x1.fff692p-1f));
  // The integer n sits in the low mantissa bits of t; n << 23 scales by 2^n.
  const int bx = __float_as_int(q.x) + (__float_as_int(t.x) << 23);
  const int by = __float_as_int(q.y) + (__float_as_int(t.y) << 23);
  return make_float2(__int_as_float(bx), __int_as_float(by));
}

// O *= alpha for this thread's row (its TMEM lane), 16 columns at a time.
__device__ __forceinline__ void rescale_o(uint32_t t_row, float alpha) {
#pragma unroll 1
  for (int c = 0; c < 8; ++c) {
    uint32_t o[16];
    tmem_ld16(t_row + c * 16, o);
    tmem_wait_ld();
#pragma unroll
    for (int i = 0; i < 16; ++i)
      o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
    tmem_st16(t_row + c * 16, o);
  }
  tmem_wait_st();
}

__global__ void __launch_bounds__(kFwdThreads, 2)
    bsa_fwd_kernel(const __grid_constant__ CUtensorMap map_q,
                   const __grid_constant__ CUtensorMap map_k,
                   const __grid_constant__ CUtensorMap map_v, FwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* s_q = smem;
  uint8_t* s_k = smem + kTileBytes;
  uint8_t* s_v = smem + 2 * kTileBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 3 * kTileBytes);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tid = threadIdx.x;
  const int warp = tid / 32;
  const int lane = tid % 32;
  const int bid = blockIdx.x;
  const int h = bid / p.n_q_tiles;
  // Heaviest query tiles (the dense global rows, last in tile order) first.
  const int qt = p.n_q_tiles - 1 - bid % p.n_q_tiles;

  int pc = 0, fc = 0;
  int64_t list_off = 0;
  if (p.dense) {
    fc = p.n_kv_tiles;
  } else {
    const int64_t row = static_cast<int64_t>(h) * p.n_q_tiles + qt;
    pc = p.part_cnt[row];
    fc = p.full_cnt[row];
    list_off = row * p.ld_idx;
  }
  const int n_steps = pc + fc;

  if (tid == 0) {
    for (int b = 0; b < kNumBars; ++b)
      mbar_init(&bars[b], (b == kPFull0 || b == kPFull1) ? 128 : 1);
    *abort = 0;
    fence_barrier_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_s = tmem;        // S / P
  const uint32_t t_o = tmem + 128;  // O

  if (warp == 4) {
    // ---------------- TMA producer ----------------
    if (lane == 0 && n_steps > 0) {
      prefetch_tensor_map(&map_q);
      prefetch_tensor_map(&map_k);
      prefetch_tensor_map(&map_v);
      const int q_row = qt * kTile;
      mbar_arrive_expect_tx(&bars[kQFull], kTileBytes);
      tma_load_3d(s_q, &map_q, &bars[kQFull], 0, h, q_row);
      tma_load_3d(s_q + kHalfBytes, &map_q, &bars[kQFull], 64, h, q_row);
      int k_issued = 0, v_issued = 0;
      for (int j = 0; j < n_steps; ++j) {
        const int kv_row = block_at(p, j, pc, fc, list_off).kv * kTile;
        if (j > 0 && !mbar_wait(&bars[kKEmpty], (j - 1) & 1, abort, p.status))
          break;
        mbar_arrive_expect_tx(&bars[kKFull], kTileBytes);
        tma_load_3d(s_k, &map_k, &bars[kKFull], 0, h, kv_row);
        tma_load_3d(s_k + kHalfBytes, &map_k, &bars[kKFull], 64, h, kv_row);
        ++k_issued;
        if (j > 0 && !mbar_wait(&bars[kVEmpty], (j - 1) & 1, abort, p.status))
          break;
        mbar_arrive_expect_tx(&bars[kVFull], kTileBytes);
        tma_load_3d(s_v, &map_v, &bars[kVFull], 0, h, kv_row);
        tma_load_3d(s_v + kHalfBytes, &map_v, &bars[kVFull], 64, h, kv_row);
        ++v_issued;
      }
      if (*abort) {
        // Let the copies already in flight land before the CTA retires: at
        // most one per buffer is outstanding, the last one issued.
        volatile int never = 0;
        mbar_wait(&bars[kQFull], 0, &never, nullptr);
        if (k_issued > 0)
          mbar_wait(&bars[kKFull], (k_issued - 1) & 1, &never, nullptr);
        if (v_issued > 0)
          mbar_wait(&bars[kVFull], (v_issued - 1) & 1, &never, nullptr);
      }
    }
  } else if (warp == 5) {
    // ---------------- tcgen05.mma issuer ----------------
    if (lane == 0 && n_steps > 0) {
      constexpr uint32_t idesc_qk = idesc_bf16(128, 128, false, false);
      constexpr uint32_t idesc_pv = idesc_bf16(128, 128, false, true);
      const uint32_t a_q = smem_u32(s_q);
      const uint32_t a_k = smem_u32(s_k);
      const uint32_t a_v = smem_u32(s_v);
      bool ok = mbar_wait(&bars[kQFull], 0, abort, p.status);
      for (int j = 0; ok && j < n_steps; ++j) {
        if (!mbar_wait(&bars[kKFull], j & 1, abort, p.status)) break;
        if (j > 0 && !mbar_wait(&bars[kODone], (j - 1) & 1, abort, p.status))
          break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * kHalfBytes + (kk & 3) * 32;
          umma_ss(t_s, sw128_desc(a_q + off, 16), sw128_desc(a_k + off, 16),
                  idesc_qk, kk > 0);
        }
        umma_commit(&bars[kSFull]);
        umma_commit(&bars[kKEmpty]);
        if (!mbar_wait(&bars[kVFull], j & 1, abort, p.status)) break;
        // PV in two halves of 64 keys, each as soon as its P is written.
        if (!mbar_wait(&bars[kPFull0], j & 1, abort, p.status)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_ts(t_o, t_s + kk * 8, sw128_desc(a_v + kk * 2048, kHalfBytes),
                  idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
        if (!mbar_wait(&bars[kPFull1], j & 1, abort, p.status)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 4; kk < 8; ++kk)
          umma_ts(t_o, t_s + kk * 8, sw128_desc(a_v + kk * 2048, kHalfBytes),
                  idesc_pv, 1u);
        umma_commit(&bars[kODone]);
        umma_commit(&bars[kVEmpty]);
      }
      if (*abort) {
        volatile int never = 0;
        umma_commit(&bars[kDrain]);
        mbar_wait(&bars[kDrain], 0, &never, nullptr);
      }
    }
  } else {
    // ---------------- softmax + epilogue (warps 0-3) ----------------
    const int row = tid;  // TMEM lane and query row within the tile
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    float m_ref = -INFINITY;  // running max, already in log2 units
    float l = 0.f;
    bool ok = true;
    // The list entry of the next step is loaded one step ahead so its
    // global-memory latency overlaps the current step.
    Step next = n_steps > 0 ? block_at(p, 0, pc, fc, list_off) : Step{0, 0};
    for (int j = 0; j < n_steps; ++j) {
      const Step st = next;
      if (j + 1 < n_steps) next = block_at(p, j + 1, pc, fc, list_off);
      // Waits and breaks stay warp-uniform: tcgen05.ld/st are warp-wide.
      if (!__all_sync(0xffffffffu,
                      mbar_wait(&bars[kSFull], j & 1, abort, p.status))) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t r[128];
      tmem_ld32(t_s + lane_base + 0, r);
      tmem_ld32(t_s + lane_base + 32, r + 32);
      tmem_ld32(t_s + lane_base + 64, r + 64);
      tmem_ld32(t_s + lane_base + 96, r + 96);
      tmem_wait_ld();
      float* s = reinterpret_cast<float*>(r);
      if (st.valid < kTile) {
#pragma unroll
        for (int c = 0; c < 128; ++c)
          if (c >= st.valid) s[c] = -INFINITY;
      }
      const float mb = row_max128(s) * p.scale_log2;
      // Lazy rescaling: the reference max moves only when a row's max grows
      // by more than 2^8, so P <= 256 and O is rarely touched.
      bool rescale = false;
      float alpha = 1.0f;
      if (j == 0) {
        m_ref = mb;
      } else {
        const bool grow = mb > m_ref + 8.0f;
        rescale = __any_sync(0xffffffffu, grow);
        if (rescale) {
          const float m_new = grow ? mb : m_ref;
          alpha = ex2_approx(m_ref - m_new);
          m_ref = m_new;
        }
      }
      const float2 scale2 = make_float2(p.scale_log2, p.scale_log2);
      const float2 neg_m2 = make_float2(-m_ref, -m_ref);
      float2 sum_a = make_float2(0.f, 0.f), sum_b = make_float2(0.f, 0.f);
      // Keys 0-63: exponentials on the MUFU.
#pragma unroll
      for (int c = 0; c < 64; c += 4) {
        const float2 x0 = __ffma2_rn(make_float2(s[c], s[c + 1]), scale2,
                                     neg_m2);
        const float2 x1 = __ffma2_rn(make_float2(s[c + 2], s[c + 3]), scale2,
                                     neg_m2);
        const float2 e0 = make_float2(ex2_approx(x0.x), ex2_approx(x0.y));
        const float2 e1 = make_float2(ex2_approx(x1.x), ex2_approx(x1.y));
        sum_a = __fadd2_rn(sum_a, e0);
        sum_b = __fadd2_rn(sum_b, e1);
        r[c / 2] = pack_bf16(e0.x, e0.y);
        r[c / 2 + 1] = pack_bf16(e1.x, e1.y);
      }
      if (rescale) {
        // O holds steps < j: wait for PV(j-1), then scale it (PV(j) cannot
        // start before this thread arrives on kPFull0 below).
        if (!__all_sync(0xffffffffu, mbar_wait(&bars[kODone], (j - 1) & 1,
                                               abort, p.status))) {
          ok = false;
          break;
        }
        tc_fence_after();
        rescale_o(t_o + lane_base, alpha);
        l *= alpha;
      }
      tmem_st32(t_s + lane_base + 0, r);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars[kPFull0]);
      // Keys 64-127: P never overwrites S columns 64-127, so they are read
      // again from TMEM instead of staying live in registers since the max.
      tmem_ld32(t_s + lane_base + 64, r + 64);
      tmem_ld32(t_s + lane_base + 96, r + 96);
      tmem_wait_ld();
      if (st.valid < kTile) {
#pragma unroll
        for (int c = 64; c < 128; ++c)
          if (c >= st.valid) s[c] = -INFINITY;
      }
      // The first 32 on the MUFU, the last kPolyCols on the FMA pipes
      // (exp2_poly2), which balances the two units.
#pragma unroll
      for (int c = 64; c < 128; c += 4) {
        const float2 x0 = __ffma2_rn(make_float2(s[c], s[c + 1]), scale2,
                                     neg_m2);
        const float2 x1 = __ffma2_rn(make_float2(s[c + 2], s[c + 3]), scale2,
                                     neg_m2);
        float2 e0, e1;
        if (c >= 128 - kPolyCols) {
          e0 = exp2_poly2(x0);
          e1 = exp2_poly2(x1);
        } else {
          e0 = make_float2(ex2_approx(x0.x), ex2_approx(x0.y));
          e1 = make_float2(ex2_approx(x1.x), ex2_approx(x1.y));
        }
        sum_a = __fadd2_rn(sum_a, e0);
        sum_b = __fadd2_rn(sum_b, e1);
        r[c / 2] = pack_bf16(e0.x, e0.y);
        r[c / 2 + 1] = pack_bf16(e1.x, e1.y);
      }
      tmem_st32(t_s + lane_base + 32, r + 32);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars[kPFull1]);
      const float2 sum2 = __fadd2_rn(sum_a, sum_b);
      l += sum2.x + sum2.y;
    }
    // ---------------- epilogue ----------------
    if (ok && n_steps > 0)
      ok = mbar_wait(&bars[kODone], (n_steps - 1) & 1, abort, p.status);
    ok = __all_sync(0xffffffffu, ok);
    const int64_t q_row = static_cast<int64_t>(qt) * kTile + row;
    // Dense mode: rows >= used keep the zeros written before the launch.
    const bool write = !p.dense || q_row < p.used;
    if (ok) {
      __nv_bfloat16* dst = p.out + q_row * p.out_stride_n + h * p.out_stride_h;
      if (n_steps > 0) tc_fence_after();
      const float inv_l = n_steps > 0 ? 1.0f / l : 0.f;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        if (n_steps > 0) {
          tmem_ld32(t_o + lane_base + c * 32, o);  // warp-wide, unpredicated
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0u;
        }
        uint32_t packed[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          packed[i] = pack_bf16(__uint_as_float(o[2 * i]) * inv_l,
                                __uint_as_float(o[2 * i + 1]) * inv_l);
        if (write) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            d4[i] = make_uint4(packed[4 * i], packed[4 * i + 1],
                               packed[4 * i + 2], packed[4 * i + 3]);
        }
      }
      if (p.lse != nullptr && write) {
        const float lse = n_steps > 0
                              ? (m_ref + lg2_approx(l)) * 0.69314718055994531f
                              : -INFINITY;
        p.lse[q_row * p.lse_stride_row + h * p.lse_stride_h] = lse;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

__global__ void zero_rows_kernel(__nv_bfloat16* out, int64_t stride_s,
                                 int64_t stride_h, float* lse, int64_t ls,
                                 int64_t lh, int64_t row0, int64_t n_rows,
                                 int n_heads) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x +
                    threadIdx.x;
  const int64_t per_row = static_cast<int64_t>(n_heads) * (kHeadDim / 8);
  if (i >= n_rows * per_row) return;
  const int64_t r = row0 + i / per_row;
  const int h = static_cast<int>((i % per_row) / (kHeadDim / 8));
  const int c8 = static_cast<int>(i % (kHeadDim / 8));
  *reinterpret_cast<uint4*>(out + r * stride_s + h * stride_h + 8 * c8) =
      make_uint4(0, 0, 0, 0);
  if (lse != nullptr && c8 == 0) lse[r * ls + h * lh] = 0.f;
}

int launch_fwd(const CUtensorMap& mq, const CUtensorMap& mk,
               const CUtensorMap& mv, const FwdParams& p, int64_t grid,
               cudaStream_t stream) {
  static bool configured = false;
  if (!configured) {
    VEDA_CUDA(cudaFuncSetAttribute(bsa_fwd_kernel,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   kSmemBytes));
    configured = true;
  }
  if (grid == 0) return VEDA_OK;
  bsa_fwd_kernel<<<static_cast<unsigned>(grid), kFwdThreads, kSmemBytes,
                   stream>>>(mq, mk, mv, p);
  return check_launch("bsa_fwd_kernel");
}

}  // namespace

}  // namespace veda

using namespace veda;

extern "C" int veda_bsa_fwd(const void* q, int64_t q_stride_n,
                            int64_t q_stride_h, const void* k,
                            int64_t k_stride_n, int64_t k_stride_h,
                            const void* v, int64_t v_stride_n,
                            int64_t v_stride_h, int32_t n_heads,
                            int64_t n_q_tiles, int64_t n_kv_tiles,
                            const int32_t* valid_count,
                            const int32_t* part_cnt, const int32_t* part_idx,
                            const int32_t* full_cnt, const int32_t* full_idx,
                            int64_t ld_idx, void* out, int64_t out_stride_n,
                            int64_t out_stride_h, float* lse,
                            float softmax_scale, void* stream) {
  int rc = require_sm100("veda_bsa_fwd");
  if (rc != VEDA_OK) return rc;
  VEDA_REQUIRE(q && k && v && out && valid_count && part_cnt && part_idx &&
                   full_cnt && full_idx,
               "q, k, v, out, valid_count and the four lists are required");
  VEDA_REQUIRE(n_heads >= 1 && n_q_tiles >= 0 && n_kv_tiles >= 1,
               "bad shape");
  VEDA_REQUIRE(ld_idx >= n_kv_tiles, "ld_idx must be >= n_kv_tiles");
  VEDA_REQUIRE(n_q_tiles * n_heads < (int64_t(1) << 31), "grid too large");
  VEDA_REQUIRE(softmax_scale > 0.f, "softmax_scale must be positive");
  VEDA_REQUIRE(reinterpret_cast<uintptr_t>(out) % 16 == 0 &&
                   out_stride_n % 8 == 0 && out_stride_h % 8 == 0,
               "out must be 16-byte aligned with strides multiple of 8");
  CUtensorMap mq, mk, mv;
  rc = make_tile_map(&mq, q, n_q_tiles * kTile, n_heads, q_stride_n,
                     q_stride_h, "q");
  if (rc == VEDA_OK)
    rc = make_tile_map(&mk, k, n_kv_tiles * kTile, n_heads, k_stride_n,
                       k_stride_h, "k");
  if (rc == VEDA_OK)
    rc = make_tile_map(&mv, v, n_kv_tiles * kTile, n_heads, v_stride_n,
                       v_stride_h, "v");
  if (rc != VEDA_OK) return rc;
  FwdParams p{};
  p.n_heads = n_heads;
  p.n_q_tiles = static_cast<int>(n_q_tiles);
  p.n_kv_tiles = static_cast<int>(n_kv_tiles);
  p.valid_count = valid_count;
  p.part_cnt = part_cnt;
  p.part_idx = part_idx;
  p.full_cnt = full_cnt;
  p.full_idx = full_idx;
  p.ld_idx = ld_idx;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_stride_n = out_stride_n;
  p.out_stride_h = out_stride_h;
  p.lse = lse;
  p.lse_stride_row = 1;
  p.lse_stride_h = n_q_tiles * kTile;
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  p.dense = 0;
  p.used = 0;
  p.status = device_status_ptr();
  return launch_fwd(mq, mk, mv, p, n_q_tiles * n_heads, as_stream(stream));
}

extern "C" int veda_dense_fwd(const void* q, const void* k, const void* v,
                              int64_t stride_s, int64_t stride_h,
                              int64_t seq_len, int64_t used, int32_t n_heads,
                              void* out, int64_t out_stride_s,
                              int64_t out_stride_h, float* lse,
                              int64_t lse_stride_s, int64_t lse_stride_h,
                              float softmax_scale, void* stream) {
  int rc = require_sm100("veda_dense_fwd");
  if (rc != VEDA_OK) return rc;
  VEDA_REQUIRE(q && k && v && out, "q, k, v and out are required");
  VEDA_REQUIRE(n_heads >= 1 && seq_len >= 0 && used >= 0 && used <= seq_len,
               "need 0 <= used <= seq_len");
  VEDA_REQUIRE(softmax_scale > 0.f, "softmax_scale must be positive");
  VEDA_REQUIRE(reinterpret_cast<uintptr_t>(out) % 16 == 0 &&
                   out_stride_s % 8 == 0 && out_stride_h % 8 == 0,
               "out must be 16-byte aligned with strides multiple of 8");
  const int64_t tiles = (used + kTile - 1) / kTile;
  VEDA_REQUIRE(tiles * n_heads < (int64_t(1) << 31), "grid too large");
  if (seq_len > used) {
    const int64_t n = (seq_len - used) * n_heads * (kHeadDim / 8);
    zero_rows_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0,
                       as_stream(stream)>>>(
        static_cast<__nv_bfloat16*>(out), out_stride_s, out_stride_h, lse,
        lse_stride_s, lse_stride_h, used, seq_len - used, n_heads);
    rc = check_launch("zero_rows_kernel");
    if (rc != VEDA_OK) return rc;
  }
  if (tiles == 0) return VEDA_OK;
  CUtensorMap mq, mk, mv;
  rc = make_tile_map(&mq, q, seq_len, n_heads, stride_s, stride_h, "q");
  if (rc == VEDA_OK)
    rc = make_tile_map(&mk, k, seq_len, n_heads, stride_s, stride_h, "k");
  if (rc == VEDA_OK)
    rc = make_tile_map(&mv, v, seq_len, n_heads, stride_s, stride_h, "v");
  if (rc != VEDA_OK) return rc;
  FwdParams p{};
  p.n_heads = n_heads;
  p.n_q_tiles = static_cast<int>(tiles);
  p.n_kv_tiles = static_cast<int>(tiles);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_stride_n = out_stride_s;
  p.out_stride_h = out_stride_h;
  p.lse = lse;
  p.lse_stride_row = lse_stride_s;
  p.lse_stride_h = lse_stride_h;
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  p.dense = 1;
  p.used = used;
  p.status = device_status_ptr();
  return launch_fwd(mq, mk, mv, p, tiles * n_heads, as_stream(stream));
}
