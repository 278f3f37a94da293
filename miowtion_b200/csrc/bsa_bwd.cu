// a10: block-sparse attention backward on tcgen05.
//
// Semantics: the gradients of the block-sparse forward (bsa_fwd.cu,
// miowtion/kernels/reference.py:23-56) with respect to q, k and v, as the
// reference's FA4 backward computes them through autograd
// (miowtion/kernels/fa4.py:337-359; its test compares with autograd through
// the reference, tests/gpu/test_kernels_gpu.py:200-250). With the forward's
// natural-log LSE L and D_i = rowsum(dO_i * O_i):
//     P  = exp(S * scale - L)     (S = Q K^T; keys past a tile's valid prefix
//                                  are masked, P = 0)
//     dP = dO V^T,  dS = P * (dP - D)
//     dQ = scale dS K,  dK = scale dS^T Q,  dV = P^T dO
// Every row of a listed query tile (padding rows included, as autograd
// through the reference treats them) contributes.
//
// Three launches, no atomics (results are deterministic):
//   prep    D and L * log2(e) per query row into the workspace (HBM bound);
//   dq      query-major over the forward lists: per block S and dP (SS MMAs),
//           dS written back over S in TMEM as bf16, dQ += dS K (TS MMA);
//   dkdv    key-major over the transposed lists: per block S^T = K Q^T and
//           dP^T = V dO^T, P^T and dS^T written back over them, then
//           dV += P^T dO and dK += dS^T Q (TS MMAs); K and V stay in shared
//           memory for the whole key tile.
// Both main kernels are persistent (one CTA per SM taking items from a
// global counter, heaviest rows first within a head), with 8 compute warps (warp w: TMEM lanes
// 32(w%4).., columns 64(w/4)..), a TMA producer warp and a converged MMA
// warp. The walk of each list is the forward's: partial list then full list,
// each from its end. All waits are bounded (common.cuh).
#include <math.h>

#include "common.cuh"

namespace veda {

namespace {

constexpr int kBwdThreads = 320;
constexpr int kProducer = 8;
constexpr int kMma = 9;
constexpr uint32_t kTileBytes = 32768;  // 128 x 128 bf16
constexpr uint32_t kHalfBytes = 16384;  // 128 x 64 bf16 (one TMA box)
constexpr uint32_t kTileUnits = kTileBytes >> 4;
constexpr uint32_t kTmemCols = 512;
constexpr int kListCap = 1024;
constexpr float kLog2e = 1.4426950408889634f;

// One set of block lists: for each head and list row, `part` then `full`
// entries (the reference's BlockSparseTensors, miowtion/kernels/fa4.py:
// 266-296).
struct ListSet {
  int n_rows;
  const int32_t* part_cnt;
  const int32_t* part_idx;
  const int32_t* full_cnt;
  const int32_t* full_idx;
  int64_t ld;
};

struct BwdParams {
  int n_heads;
  int n_q_tiles;
  int n_kv_tiles;
  const int32_t* valid_count;
  ListSet lists;        // forward lists (dq) or transposed lists (dkdv)
  const float* delta;   // [H][n_q_tiles * 128]
  const float* lse2;    // [H][n_q_tiles * 128], LSE * log2(e)
  __nv_bfloat16* grad;  // dq (dq kernel) or dk (dkdv kernel)
  int64_t grad_sn, grad_sh;
  __nv_bfloat16* grad2;  // dv (dkdv kernel)
  int64_t grad2_sn, grad2_sh;
  float scale;
  float scale_log2;
  unsigned int* counter;  // the item counter, zero at launch
  unsigned int* status;
};

__device__ __forceinline__ bool wait_all(uint64_t* bar, uint32_t parity,
                                         volatile int* abort,
                                         unsigned int* status) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort, status));
}

// Work items are handed out dynamically: the producer warp of each CTA takes
// the next item index from a global counter and publishes it in a shared
// queue, which the MMA warp and the compute warps read in the same order.
// All CTAs then work on neighbouring items at any time (the tiles they load
// stay in L2) and load balances itself, however unequal the lists are.
constexpr int kQueue = 8;
constexpr int kQueueReaders = 9;  // the MMA warp and 8 compute warps

struct ItemQueue {
  volatile int* slots;   // [kQueue] item indices, -1 = end
  uint64_t* full;        // [kQueue] published (producer)
  uint64_t* empty;       // [kQueue] read by every reader
  unsigned int* counter;
  int n_items;
  volatile int* abort;
  unsigned int* status;
};

// The items (head, list row) one CTA takes, heaviest rows (the last ones:
// the global tiles) first within a head, and their blocks. Every role walks
// the same sequence, so they agree on barrier phases without talking.
struct ListStream {
  const ListSet* L;
  const ItemQueue* Q;
  bool producer;
  int q;  // queue position
  int n_items, it;
  int h, row, pc, fc, len, j, blk, ka;
  int64_t off;
  bool ok;  // false after an expired wait

  // The next item index from the queue (warp-collective); -1 at the end.
  __device__ int pull() {
    const int slot = q % kQueue;
    const uint32_t phase = (q / kQueue) & 1;
    int item = -1;
    if (producer) {
      if (q >= kQueue && !wait_all(&Q->empty[slot], phase ^ 1, Q->abort,
                                   Q->status)) {
        ok = false;
        return -1;
      }
      if ((threadIdx.x & 31) == 0) {
        item = static_cast<int>(atomicAdd(Q->counter, 1u));
        if (item >= Q->n_items) item = -1;
        Q->slots[slot] = item;
        mbar_arrive(&Q->full[slot]);
      }
      item = __shfl_sync(0xffffffffu, item, 0);
    } else {
      if (!wait_all(&Q->full[slot], phase, Q->abort, Q->status)) {
        ok = false;
        return -1;
      }
      item = Q->slots[slot];
      __syncwarp();
      if ((threadIdx.x & 31) == 0) mbar_arrive(&Q->empty[slot]);
    }
    ++q;
    return item;
  }
  __device__ void set_item(int item) {
    if (item < 0) {
      it = n_items;
      return;
    }
    it = item;
    h = it / L->n_rows;
    row = L->n_rows - 1 - it % L->n_rows;
    const int64_t r = static_cast<int64_t>(h) * L->n_rows + row;
    off = r * L->ld;
    pc = L->part_cnt[r];
    fc = L->full_cnt[r];
    len = pc + fc;
    j = 0;
    if (len > 0) ++ka;
  }
  __device__ void init(const ListSet* ls, const ItemQueue* queue,
                       bool is_producer, bool keep_empty) {
    L = ls;
    Q = queue;
    producer = is_producer;
    q = 0;
    n_items = queue->n_items;
    blk = 0;
    ka = -1;
    ok = true;
    set_item(pull());
    if (!keep_empty) skip_empty();
  }
  __device__ void skip_empty() {
    while (it < n_items && len == 0) set_item(pull());
  }
  __device__ void next_item(bool keep_empty) {
    set_item(pull());
    if (!keep_empty) skip_empty();
  }
  __device__ bool valid() const { return it < n_items; }
  // Entry jj of the current item's walk: part list, then full list, each
  // from its end.
  __device__ int entry(int jj) const {
    return jj < pc ? L->part_idx[off + (pc - 1 - jj)]
                   : L->full_idx[off + (fc - 1 - (jj - pc))];
  }
  __device__ void next_block() {
    ++blk;
    if (++j < len) return;
    next_item(false);
  }
};

__device__ __forceinline__ void arrive_warp(uint64_t* bar) {
  tc_fence_before();
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
}

// TMA load of one 128 x 128 bf16 tile (two 64-column boxes).
__device__ __forceinline__ void load_tile(uint8_t* dst, const CUtensorMap* map,
                                          uint64_t* bar, int h, int tile) {
  tma_load_3d(dst, map, bar, 0, h, tile * kTile);
  tma_load_3d(dst + kHalfBytes, map, bar, 64, h, tile * kTile);
}

// The A operand columns of key (or query) step kk: the compute warps write
// the packed bf16 of columns 0-63 over TMEM columns 0-31 and of columns
// 64-127 over columns 64-95.
__device__ __forceinline__ uint32_t packed_col(int kk) {
  return kk < 4 ? kk * 8 : 64 + (kk - 4) * 8;
}

// Writes a 64-column bf16 row segment (32 words) to global memory.
__device__ __forceinline__ void store_row64(__nv_bfloat16* dst,
                                            const uint32_t* w) {
  uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int i = 0; i < 8; ++i)
    d4[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
}

// Reads 64 fp32 TMEM columns of this thread's lane, scales them and packs
// them to bf16 pairs.
__device__ __forceinline__ void tmem_row64_bf16(uint32_t taddr, float scale,
                                                uint32_t* w) {
  uint32_t o[32];
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    tmem_ld32(taddr + c * 32, o);
    tmem_wait_ld();
#pragma unroll
    for (int i = 0; i < 16; ++i)
      w[c * 16 + i] = pack_bf16(__uint_as_float(o[2 * i]) * scale,
                                __uint_as_float(o[2 * i + 1]) * scale);
  }
}

// ---------------------------------------------------------------------------
// prep: D = rowsum(dO * O) and L * log2(e), one warp per (row, head).
// ---------------------------------------------------------------------------
__global__ void bwd_prep_kernel(const __nv_bfloat16* out, int64_t o_sn,
                                int64_t o_sh, const __nv_bfloat16* dout,
                                int64_t d_sn, int64_t d_sh, const float* lse,
                                int64_t l_sr, int64_t l_sh, int64_t rows,
                                int heads, float* delta, float* lse2) {
  const int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x +
                     threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (w >= rows * heads) return;
  const int64_t r = w / heads;
  const int h = static_cast<int>(w % heads);
  const uint2 a = *reinterpret_cast<const uint2*>(out + r * o_sn + h * o_sh +
                                                  lane * 4);
  const uint2 b = *reinterpret_cast<const uint2*>(dout + r * d_sn +
                                                  h * d_sh + lane * 4);
  const __nv_bfloat162* a2 = reinterpret_cast<const __nv_bfloat162*>(&a);
  const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&b);
  float acc = 0.f;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float2 x = __bfloat1622float2(a2[i]);
    const float2 y = __bfloat1622float2(b2[i]);
    acc = fmaf(x.x, y.x, fmaf(x.y, y.y, acc));
  }
#pragma unroll
  for (int s = 16; s > 0; s >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, s);
  if (lane == 0) {
    delta[static_cast<int64_t>(h) * rows + r] = acc;
    lse2[static_cast<int64_t>(h) * rows + r] =
        lse[r * l_sr + h * l_sh] * kLog2e;
  }
}

// ---------------------------------------------------------------------------
// dq: query-major. Each block's 128 key columns run as two halves of 64 so
// that one half's elementwise work overlaps the other half's MMAs. TMEM, per
// half h: S [128h, 128h+64) (dS over its columns 0-15 and 32-47), dP
// [128h+64, 128h+128); dQ [256,384).
// ---------------------------------------------------------------------------
enum DqBar {
  kQFull = 0,      // Q and dO of the item landed
  kQEmpty,         // the item's last S and dP MMAs finished
  kKvFull,         // [2] K and V of the block landed (stage = block parity)
  kKvEmpty = kKvFull + 2,  // [2] the block's MMAs finished reading them
  kSdFull = kKvEmpty + 2,  // [2 halves] S and dP of the block's half
  kDsFull = kSdFull + 2,   // [2 halves] dS written (8 warps)
  kDqDone = kDsFull + 2,   // the item's last dQ MMA finished
  kDqFree,         // the epilogue has read dQ (8 warps)
  kDqDrain,
  kDqItemFull,                       // [kQueue]
  kDqItemEmpty = kDqItemFull + kQueue,  // [kQueue]
  kDqNumBars = kDqItemEmpty + kQueue
};
constexpr int kDqSmem = 6 * kTileBytes + kListCap * 4 + 512 + 1024;

__global__ void __launch_bounds__(kBwdThreads, 1)
    bsa_bwd_dq_kernel(const __grid_constant__ CUtensorMap map_q,
                      const __grid_constant__ CUtensorMap map_do,
                      const __grid_constant__ CUtensorMap map_k,
                      const __grid_constant__ CUtensorMap map_v, BwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* s_q = smem;
  uint8_t* s_do = smem + kTileBytes;
  uint8_t* s_kv = smem + 2 * kTileBytes;  // [2 stages] x (K, V)
  int32_t* s_list = reinterpret_cast<int32_t*>(smem + 6 * kTileBytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_list + kListCap);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kDqNumBars);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const ItemQueue queue{reinterpret_cast<volatile int*>(tmem_slot + 2),
                        bars + kDqItemFull, bars + kDqItemEmpty, p.counter,
                        p.n_heads * p.lists.n_rows, abort, p.status};

  const int tid = threadIdx.x;
  const int warp = tid / 32;
  const int lane = tid % 32;
  if (tid == 0) {
    for (int b = 0; b < kDqNumBars; ++b)
      mbar_init(&bars[b], (b == kDsFull || b == kDsFull + 1 || b == kDqFree)
                              ? 8
                          : (b >= kDqItemEmpty) ? kQueueReaders
                                                : 1);
    *abort = 0;
    fence_barrier_init();
  }
  if (warp == kMma) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kProducer) {
    if (lane == 0) {
      prefetch_tensor_map(&map_q);
      prefetch_tensor_map(&map_do);
      prefetch_tensor_map(&map_k);
      prefetch_tensor_map(&map_v);
    }
    ListStream st;
    st.init(&p.lists, &queue, true, false);
    int q_loads = 0, kv_loads = 0;
    while (st.valid()) {
      if (st.j == 0) {
        if (st.len <= kListCap)
          for (int jj = lane; jj < st.len; jj += 32) s_list[jj] = st.entry(jj);
        __syncwarp();
        if (st.ka > 0 && !wait_all(&bars[kQEmpty], (st.ka - 1) & 1, abort,
                                   p.status))
          break;
        if (lane == 0) {
          mbar_arrive_expect_tx(&bars[kQFull], 2 * kTileBytes);
          load_tile(s_q, &map_q, &bars[kQFull], st.h, st.row);
          load_tile(s_do, &map_do, &bars[kQFull], st.h, st.row);
        }
        __syncwarp();
        q_loads = st.ka + 1;
      }
      const int kv = st.len <= kListCap ? s_list[st.j] : st.entry(st.j);
      const int stage = st.blk & 1;
      if (st.blk >= 2 && !wait_all(&bars[kKvEmpty + stage],
                                   ((st.blk >> 1) - 1) & 1, abort, p.status))
        break;
      if (lane == 0) {
        uint8_t* dst = s_kv + stage * 2 * kTileBytes;
        mbar_arrive_expect_tx(&bars[kKvFull + stage], 2 * kTileBytes);
        load_tile(dst, &map_k, &bars[kKvFull + stage], st.h, kv);
        load_tile(dst + kTileBytes, &map_v, &bars[kKvFull + stage], st.h, kv);
      }
      __syncwarp();
      kv_loads = st.blk + 1;
      st.next_block();
    }
    if (lane == 0 && *abort) {
      volatile int never = 0;
      if (q_loads > 0)
        mbar_wait(&bars[kQFull], (q_loads - 1) & 1, &never, nullptr);
      for (int b = kv_loads - 2; b < kv_loads; ++b)
        if (b >= 0)
          mbar_wait(&bars[kKvFull + (b & 1)], (b >> 1) & 1, &never, nullptr);
    }
  } else if (warp == kMma) {
    // Per block j, halves a (keys 0-63) and b (64-127):
    //   S_a, dP_a, S_b, dP_b of block 0 of the item, then for each j
    //   dQ += half a of j; S_a, dP_a of j + 1;
    //   dQ += half b of j; S_b, dP_b of j + 1.
    constexpr uint32_t idesc_sd = idesc_bf16(128, 64, false, false);
    constexpr uint32_t idesc_bmn = idesc_bf16(128, 128, false, true);
    const uint32_t q_lo = sw128_desc_lo(smem_u32(s_q), 16);
    const uint32_t do_lo = sw128_desc_lo(smem_u32(s_do), 16);
    const uint32_t kv_lo = sw128_desc_lo(smem_u32(s_kv), 16);
    const uint32_t kvmn_lo = sw128_desc_lo(smem_u32(s_kv), kHalfBytes);
    const uint32_t t_dq = tmem + 256;
    // S and dP of key half h of the tiles in stage `stage` (key rows
    // 64h .. 64h + 63: 8 KB into each 64-column box).
    auto issue_sd = [&](int stage, int h) {
      const uint32_t k_lo = kv_lo + stage * 2 * kTileUnits + h * (8192 >> 4);
      const uint32_t v_lo = k_lo + kTileUnits;
      const uint32_t t_s = tmem + h * 128, t_dp = t_s + 64;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t off = (kk >> 2) * (kHalfBytes >> 4) + (kk & 3) * 2;
        umma_ss_warp(t_s, q_lo + off, k_lo + off, idesc_sd, kk > 0);
      }
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t off = (kk >> 2) * (kHalfBytes >> 4) + (kk & 3) * 2;
        umma_ss_warp(t_dp, do_lo + off, v_lo + off, idesc_sd, kk > 0);
      }
      umma_commit_warp(&bars[kSdFull + h]);
    };
    // dQ += dS K over half h's 64 keys (4 K-steps; dS of keys 16kk' ..
    // lies in columns 32(kk'/2) + 8(kk'%2) of the half's S).
    auto issue_dq = [&](int stage, int h, bool first) {
      const uint32_t kmn = kvmn_lo + stage * 2 * kTileUnits;
      const uint32_t t_a = tmem + h * 128;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        umma_ts_warp(t_dq, t_a + (kk >> 1) * 32 + (kk & 1) * 8,
                     kmn + (4 * h + kk) * 128, idesc_bmn,
                     (kk > 0 || h > 0 || !first) ? 1u : 0u);
    };
    ListStream st;
    st.init(&p.lists, &queue, false, false);
    bool run = true;
    while (run && st.valid()) {
      const int ka = st.ka, len = st.len;
      const int blk0 = st.blk;
      if (!wait_all(&bars[kQFull], ka & 1, abort, p.status) ||
          !wait_all(&bars[kKvFull + (blk0 & 1)], (blk0 >> 1) & 1, abort,
                    p.status))
        break;
      tc_fence_after();
      issue_sd(blk0 & 1, 0);
      issue_sd(blk0 & 1, 1);
      if (len == 1) umma_commit_warp(&bars[kQEmpty]);
      for (int j = 0; j < len; ++j) {
        const int blk = blk0 + j;
        const int stage = blk & 1;
        const bool first = j == 0, last = j == len - 1;
        // The item's first dQ overwrites dQ: the epilogue must have read it.
        if (first && ka > 0 &&
            !wait_all(&bars[kDqFree], (ka - 1) & 1, abort, p.status)) {
          run = false;
          break;
        }
        if (!wait_all(&bars[kDsFull + 0], blk & 1, abort, p.status)) {
          run = false;
          break;
        }
        tc_fence_after();
        issue_dq(stage, 0, first);
        if (!last) {
          if (!wait_all(&bars[kKvFull + ((blk + 1) & 1)],
                        ((blk + 1) >> 1) & 1, abort, p.status)) {
            run = false;
            break;
          }
          tc_fence_after();
          issue_sd((blk + 1) & 1, 0);
        }
        if (!wait_all(&bars[kDsFull + 1], blk & 1, abort, p.status)) {
          run = false;
          break;
        }
        tc_fence_after();
        issue_dq(stage, 1, first);
        umma_commit_warp(&bars[kKvEmpty + stage]);
        if (!last) {
          issue_sd((blk + 1) & 1, 1);
          if (j + 1 == len - 1) umma_commit_warp(&bars[kQEmpty]);
        } else {
          umma_commit_warp(&bars[kDqDone]);
        }
      }
      if (!run) break;
      for (int j = 0; j < len; ++j) st.next_block();
    }
    if (*abort) {
      volatile int never = 0;
      umma_commit_warp(&bars[kDqDrain]);
      mbar_wait(&bars[kDqDrain], 0, &never, nullptr);
    }
  } else {
    // ---------------- compute warps 0-7 ----------------
    const int half = warp / 4;
    const int quarter = warp % 4;
    const int row = quarter * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const int64_t n_rows_q = static_cast<int64_t>(p.n_q_tiles) * kTile;
    ListStream st;
    st.init(&p.lists, &queue, false, true);
    bool ok = true;
    while (ok && st.valid()) {
      const int h = st.h, qt = st.row, len = st.len, ka = st.ka;
      const int64_t q_row = static_cast<int64_t>(qt) * kTile + row;
      __nv_bfloat16* dst =
          p.grad + q_row * p.grad_sn + h * p.grad_sh + half * 64;
      if (len == 0) {
        uint32_t z[32] = {0};
        store_row64(dst, z);
        st.next_item(true);
        continue;
      }
      const float l2 = p.lse2[h * n_rows_q + q_row];
      const float dlt = p.delta[h * n_rows_q + q_row];
      // Warp (wq, quarter) takes keys 32 wq .. 32 wq + 31 of each half.
      const int wq = half;
      for (int j = 0; j < len && ok; ++j) {
        const int blk = st.blk;
        const int valid = j < st.pc ? p.valid_count[st.entry(j)] : kTile;
        st.j += 1;
        st.blk += 1;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          if (!wait_all(&bars[kSdFull + hh], blk & 1, abort, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int key0 = hh * 64 + wq * 32;  // key column of the block
          const uint32_t t_s = tmem + hh * 128 + wq * 32 + lane_base;
          uint32_t s[32], dp[32];
          tmem_ld32(t_s, s);
          tmem_ld32(t_s + 64, dp);
          tmem_wait_ld();
          uint32_t w[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            float d2[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int cc = 2 * i + e;
              float pr = ex2_approx(
                  fmaf(__uint_as_float(s[cc]), p.scale_log2, -l2));
              if (key0 + cc >= valid) pr = 0.f;
              d2[e] = pr * (__uint_as_float(dp[cc]) - dlt);
            }
            w[i] = pack_bf16(d2[0], d2[1]);
          }
          // dS of these 32 keys over the first 16 of this warp's own 32
          // columns of S.
          tmem_st16(t_s, w);
          tmem_wait_st();
          arrive_warp(&bars[kDsFull + hh]);
        }
      }
      if (!ok) break;
      if (!wait_all(&bars[kDqDone], ka & 1, abort, p.status)) break;
      tc_fence_after();
      uint32_t w[32];
      tmem_row64_bf16(tmem + 256 + half * 64 + lane_base, p.scale, w);
      arrive_warp(&bars[kDqFree]);
      store_row64(dst, w);
      st.next_item(true);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMma) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// dkdv: key-major. Each block's 128 query columns run as two halves of 64
// so that one half's elementwise work overlaps the other half's MMAs.
// TMEM, per half h: S^T [128h, 128h+64) (P^T over its columns 0-15 and
// 32-47), dP^T [128h+64, 128h+128) (dS^T likewise); dV [256,384),
// dK [384,512).
// ---------------------------------------------------------------------------
enum KvBar {
  kKtFull = 0,     // K and V of the key tile landed
  kKtEmpty,        // the item's last S^T and dP^T MMAs finished
  kQdFull,         // [2] Q, dO, L and D of the block landed (block parity)
  kQdEmpty = kQdFull + 2,  // [2] the block's MMAs finished reading them
  kStFull = kQdEmpty + 2,  // [2 halves] S^T and dP^T of the block's half
  kPdsFull = kStFull + 2,  // [2 halves] P^T and dS^T written (8 warps)
  kKvDone = kPdsFull + 2,  // the item's last dV/dK MMAs finished
  kKvFree,         // the epilogue has read dV and dK (8 warps)
  kKvDrain,
  kKvItemFull,                       // [kQueue]
  kKvItemEmpty = kKvItemFull + kQueue,  // [kQueue]
  kKvNumBars = kKvItemEmpty + kQueue
};
// K, V, then [2 stages] x (Q, dO), then [2 stages] x (L, D) vectors.
constexpr int kKvSmem = 6 * kTileBytes + 2 * 1024 + kListCap * 4 + 512 + 1024;

__global__ void __launch_bounds__(kBwdThreads, 1)
    bsa_bwd_dkdv_kernel(const __grid_constant__ CUtensorMap map_q,
                        const __grid_constant__ CUtensorMap map_do,
                        const __grid_constant__ CUtensorMap map_k,
                        const __grid_constant__ CUtensorMap map_v,
                        BwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* s_k = smem;
  uint8_t* s_v = smem + kTileBytes;
  uint8_t* s_qd = smem + 2 * kTileBytes;  // [2 stages] x (Q, dO)
  float* s_vec = reinterpret_cast<float*>(smem + 6 * kTileBytes);  // [2][L|D]
  int32_t* s_list = reinterpret_cast<int32_t*>(s_vec + 512);
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_list + kListCap);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kKvNumBars);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const ItemQueue queue{reinterpret_cast<volatile int*>(tmem_slot + 2),
                        bars + kKvItemFull, bars + kKvItemEmpty, p.counter,
                        p.n_heads * p.lists.n_rows, abort, p.status};

  const int tid = threadIdx.x;
  const int warp = tid / 32;
  const int lane = tid % 32;
  const int64_t n_rows_q = static_cast<int64_t>(p.n_q_tiles) * kTile;
  if (tid == 0) {
    for (int b = 0; b < kKvNumBars; ++b)
      mbar_init(&bars[b], (b == kPdsFull || b == kPdsFull + 1 || b == kKvFree)
                              ? 8
                          : (b >= kKvItemEmpty) ? kQueueReaders
                                                : 1);
    *abort = 0;
    fence_barrier_init();
  }
  if (warp == kMma) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kProducer) {
    if (lane == 0) {
      prefetch_tensor_map(&map_q);
      prefetch_tensor_map(&map_do);
      prefetch_tensor_map(&map_k);
      prefetch_tensor_map(&map_v);
    }
    ListStream st;
    st.init(&p.lists, &queue, true, false);
    int kt_loads = 0, qd_loads = 0;
    while (st.valid()) {
      if (st.j == 0) {
        if (st.len <= kListCap)
          for (int jj = lane; jj < st.len; jj += 32) s_list[jj] = st.entry(jj);
        __syncwarp();
        if (st.ka > 0 && !wait_all(&bars[kKtEmpty], (st.ka - 1) & 1, abort,
                                   p.status))
          break;
        if (lane == 0) {
          mbar_arrive_expect_tx(&bars[kKtFull], 2 * kTileBytes);
          load_tile(s_k, &map_k, &bars[kKtFull], st.h, st.row);
          load_tile(s_v, &map_v, &bars[kKtFull], st.h, st.row);
        }
        __syncwarp();
        kt_loads = st.ka + 1;
      }
      const int qi = st.len <= kListCap ? s_list[st.j] : st.entry(st.j);
      const int stage = st.blk & 1;
      if (st.blk >= 2 && !wait_all(&bars[kQdEmpty + stage],
                                   ((st.blk >> 1) - 1) & 1, abort, p.status))
        break;
      if (lane == 0) {
        uint8_t* dst = s_qd + stage * 2 * kTileBytes;
        const int64_t base = static_cast<int64_t>(st.h) * n_rows_q +
                             static_cast<int64_t>(qi) * kTile;
        mbar_arrive_expect_tx(&bars[kQdFull + stage], 2 * kTileBytes + 1024);
        load_tile(dst, &map_q, &bars[kQdFull + stage], st.h, qi);
        load_tile(dst + kTileBytes, &map_do, &bars[kQdFull + stage], st.h, qi);
        bulk_load(s_vec + stage * 256, p.lse2 + base, 512,
                  &bars[kQdFull + stage]);
        bulk_load(s_vec + stage * 256 + 128, p.delta + base, 512,
                  &bars[kQdFull + stage]);
      }
      __syncwarp();
      qd_loads = st.blk + 1;
      st.next_block();
    }
    if (lane == 0 && *abort) {
      volatile int never = 0;
      if (kt_loads > 0)
        mbar_wait(&bars[kKtFull], (kt_loads - 1) & 1, &never, nullptr);
      for (int b = qd_loads - 2; b < qd_loads; ++b)
        if (b >= 0)
          mbar_wait(&bars[kQdFull + (b & 1)], (b >> 1) & 1, &never, nullptr);
    }
  } else if (warp == kMma) {
    // Per block j, halves a (queries 0-63) and b (64-127):
    //   S^T_a, dP^T_a, S^T_b, dP^T_b of block 0 of the item, then for each j
    //   dV, dK += half a of j; S^T_a, dP^T_a of j + 1;
    //   dV, dK += half b of j; S^T_b, dP^T_b of j + 1,
    // so the tensor core has the other half's MMAs while the compute warps
    // turn one half's S^T, dP^T into P^T, dS^T.
    constexpr uint32_t idesc_st = idesc_bf16(128, 64, false, false);
    constexpr uint32_t idesc_bmn = idesc_bf16(128, 128, false, true);
    const uint32_t k_lo = sw128_desc_lo(smem_u32(s_k), 16);
    const uint32_t v_lo = sw128_desc_lo(smem_u32(s_v), 16);
    const uint32_t qd_lo = sw128_desc_lo(smem_u32(s_qd), 16);
    const uint32_t qdmn_lo = sw128_desc_lo(smem_u32(s_qd), kHalfBytes);
    const uint32_t t_dv = tmem + 256, t_dk = tmem + 384;
    // S^T and dP^T of half h of the block in stage `stage` (query rows
    // 64h .. 64h + 63 of the Q and dO tiles: 8 KB into each 64-column box).
    auto issue_st = [&](int stage, int h) {
      const uint32_t q_lo = qd_lo + stage * 2 * kTileUnits + h * (8192 >> 4);
      const uint32_t do_lo = q_lo + kTileUnits;
      const uint32_t t_s = tmem + h * 128, t_dp = t_s + 64;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t off = (kk >> 2) * (kHalfBytes >> 4) + (kk & 3) * 2;
        umma_ss_warp(t_s, k_lo + off, q_lo + off, idesc_st, kk > 0);
      }
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t off = (kk >> 2) * (kHalfBytes >> 4) + (kk & 3) * 2;
        umma_ss_warp(t_dp, v_lo + off, do_lo + off, idesc_st, kk > 0);
      }
      umma_commit_warp(&bars[kStFull + h]);
    };
    // dV += P^T dO and dK += dS^T Q over half h's 64 queries (4 K-steps
    // each; P^T of queries 16kk' .. lies in columns 32(kk'/2) + 8(kk'%2)).
    auto issue_acc = [&](int stage, int h, bool first) {
      const uint32_t qmn = qdmn_lo + stage * 2 * kTileUnits;
      const uint32_t domn = qmn + kTileUnits;
      const uint32_t t_p = tmem + h * 128, t_ds = t_p + 64;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        umma_ts_warp(t_dv, t_p + (kk >> 1) * 32 + (kk & 1) * 8,
                     domn + (4 * h + kk) * 128, idesc_bmn,
                     (kk > 0 || h > 0 || !first) ? 1u : 0u);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        umma_ts_warp(t_dk, t_ds + (kk >> 1) * 32 + (kk & 1) * 8,
                     qmn + (4 * h + kk) * 128, idesc_bmn,
                     (kk > 0 || h > 0 || !first) ? 1u : 0u);
    };
    ListStream st;
    st.init(&p.lists, &queue, false, false);
    bool run = true;
    while (run && st.valid()) {
      const int ka = st.ka, len = st.len;
      const int blk0 = st.blk;
      if (!wait_all(&bars[kKtFull], ka & 1, abort, p.status) ||
          !wait_all(&bars[kQdFull + (blk0 & 1)], (blk0 >> 1) & 1, abort,
                    p.status))
        break;
      tc_fence_after();
      issue_st(blk0 & 1, 0);
      issue_st(blk0 & 1, 1);
      if (len == 1) umma_commit_warp(&bars[kKtEmpty]);
      for (int j = 0; j < len; ++j) {
        const int blk = blk0 + j;
        const int stage = blk & 1;
        const bool first = j == 0, last = j == len - 1;
        // The item's first dV/dK overwrite the accumulators, which the
        // epilogue must have read.
        if (first && ka > 0 &&
            !wait_all(&bars[kKvFree], (ka - 1) & 1, abort, p.status)) {
          run = false;
          break;
        }
        if (!wait_all(&bars[kPdsFull + 0], blk & 1, abort, p.status)) {
          run = false;
          break;
        }
        tc_fence_after();
        issue_acc(stage, 0, first);
        if (!last) {
          if (!wait_all(&bars[kQdFull + ((blk + 1) & 1)],
                        ((blk + 1) >> 1) & 1, abort, p.status)) {
            run = false;
            break;
          }
          tc_fence_after();
          issue_st((blk + 1) & 1, 0);
        }
        if (!wait_all(&bars[kPdsFull + 1], blk & 1, abort, p.status)) {
          run = false;
          break;
        }
        tc_fence_after();
        issue_acc(stage, 1, first);
        umma_commit_warp(&bars[kQdEmpty + stage]);
        if (!last) {
          issue_st((blk + 1) & 1, 1);
          if (j + 1 == len - 1) umma_commit_warp(&bars[kKtEmpty]);
        } else {
          umma_commit_warp(&bars[kKvDone]);
        }
      }
      if (!run) break;
      for (int j = 0; j < len; ++j) st.next_block();
    }
    if (*abort) {
      volatile int never = 0;
      umma_commit_warp(&bars[kKvDrain]);
      mbar_wait(&bars[kKvDrain], 0, &never, nullptr);
    }
  } else {
    // ---------------- compute warps 0-7 ----------------
    const int half = warp / 4;
    const int quarter = warp % 4;
    const int row = quarter * 32 + lane;  // key row of the tile
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    ListStream st;
    st.init(&p.lists, &queue, false, true);
    bool ok = true;
    while (ok && st.valid()) {
      const int h = st.h, kt = st.row, len = st.len, ka = st.ka;
      const int64_t k_row = static_cast<int64_t>(kt) * kTile + row;
      __nv_bfloat16* dk_dst =
          p.grad + k_row * p.grad_sn + h * p.grad_sh + half * 64;
      __nv_bfloat16* dv_dst =
          p.grad2 + k_row * p.grad2_sn + h * p.grad2_sh + half * 64;
      if (len == 0) {
        uint32_t z[32] = {0};
        store_row64(dk_dst, z);
        store_row64(dv_dst, z);
        st.next_item(true);
        continue;
      }
      // Keys past the tile's valid prefix take no part: P = dS = 0.
      const bool key_ok = row < p.valid_count[kt];
      // Warp (wq, quarter) takes queries 32 wq .. 32 wq + 31 of each half.
      const int wq = half;
      for (int j = 0; j < len && ok; ++j) {
        const int blk = st.blk;
        st.j += 1;
        st.blk += 1;
        const float* vl = s_vec + (blk & 1) * 256;  // L*log2e, then D
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          if (!wait_all(&bars[kStFull + h], blk & 1, abort, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int q0 = h * 64 + wq * 32;  // query column of the block
          const uint32_t t_s = tmem + h * 128 + wq * 32 + lane_base;
          const uint32_t t_dp = t_s + 64;
          uint32_t s[32], dp[32];
          tmem_ld32(t_s, s);
          tmem_ld32(t_dp, dp);
          tmem_wait_ld();
          uint32_t wp[16], wd[16];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float4 l4 = *reinterpret_cast<const float4*>(vl + q0 + 4 * i);
            const float4 d4 =
                *reinterpret_cast<const float4*>(vl + 128 + q0 + 4 * i);
            const float lv[4] = {l4.x, l4.y, l4.z, l4.w};
            const float dv[4] = {d4.x, d4.y, d4.z, d4.w};
            float pr[4], ds[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int cc = 4 * i + e;
              pr[e] = key_ok ? ex2_approx(fmaf(__uint_as_float(s[cc]),
                                               p.scale_log2, -lv[e]))
                             : 0.f;
              ds[e] = pr[e] * (__uint_as_float(dp[cc]) - dv[e]);
            }
            wp[2 * i] = pack_bf16(pr[0], pr[1]);
            wp[2 * i + 1] = pack_bf16(pr[2], pr[3]);
            wd[2 * i] = pack_bf16(ds[0], ds[1]);
            wd[2 * i + 1] = pack_bf16(ds[2], ds[3]);
          }
          // P^T and dS^T of these 32 queries over the first 16 of this
          // warp's own 32 columns of S^T and dP^T.
          tmem_st16(t_s, wp);
          tmem_st16(t_dp, wd);
          tmem_wait_st();
          arrive_warp(&bars[kPdsFull + h]);
        }
      }
      if (!ok) break;
      if (!wait_all(&bars[kKvDone], ka & 1, abort, p.status)) break;
      tc_fence_after();
      uint32_t wv[32], wk[32];
      tmem_row64_bf16(tmem + 256 + half * 64 + lane_base, 1.0f, wv);
      tmem_row64_bf16(tmem + 384 + half * 64 + lane_base, p.scale, wk);
      arrive_warp(&bars[kKvFree]);
      store_row64(dv_dst, wv);
      store_row64(dk_dst, wk);
      st.next_item(true);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMma) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

int sm_count() {
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) !=
            cudaSuccess)
      sms = 148;
  }
  return sms;
}

}  // namespace

}  // namespace veda

using namespace veda;

extern "C" int64_t veda_bsa_bwd_workspace(int32_t n_heads,
                                          int64_t n_q_tiles) {
  if (n_heads < 1 || n_q_tiles < 0) return -1;
  // D and LSE*log2(e) per query row, then the two kernels' item counters.
  return 2 * static_cast<int64_t>(n_heads) * n_q_tiles * kTile *
             static_cast<int64_t>(sizeof(float)) +
         16;
}

extern "C" int veda_bsa_bwd(
    const void* q, int64_t q_stride_n, int64_t q_stride_h, const void* k,
    int64_t k_stride_n, int64_t k_stride_h, const void* v, int64_t v_stride_n,
    int64_t v_stride_h, const void* out, int64_t out_stride_n,
    int64_t out_stride_h, const void* dout, int64_t dout_stride_n,
    int64_t dout_stride_h, const float* lse, int64_t lse_stride_row,
    int64_t lse_stride_h, int32_t n_heads, int64_t n_q_tiles,
    int64_t n_kv_tiles, const int32_t* valid_count, const int32_t* part_cnt,
    const int32_t* part_idx, const int32_t* full_cnt, const int32_t* full_idx,
    int64_t ld_idx, const int32_t* t_part_cnt, const int32_t* t_part_idx,
    const int32_t* t_full_cnt, const int32_t* t_full_idx, int64_t ld_t_idx,
    void* dq, int64_t dq_stride_n, int64_t dq_stride_h, void* dk,
    int64_t dk_stride_n, int64_t dk_stride_h, void* dv, int64_t dv_stride_n,
    int64_t dv_stride_h, float softmax_scale, void* workspace,
    size_t workspace_bytes, void* stream) {
  int rc = require_sm100("veda_bsa_bwd");
  if (rc != VEDA_OK) return rc;
  VEDA_REQUIRE(q && k && v && out && dout && lse && valid_count && part_cnt &&
                   part_idx && full_cnt && full_idx && t_part_cnt &&
                   t_part_idx && t_full_cnt && t_full_idx && dq && dk && dv &&
                   workspace,
               "every tensor argument is required");
  VEDA_REQUIRE(n_heads >= 1 && n_q_tiles >= 0 && n_kv_tiles >= 1,
               "bad shape");
  VEDA_REQUIRE(ld_idx >= n_kv_tiles && ld_t_idx >= n_q_tiles,
               "list leading dimensions too small");
  VEDA_REQUIRE(n_q_tiles * n_heads < (int64_t(1) << 30) &&
                   n_kv_tiles * n_heads < (int64_t(1) << 30),
               "too many tiles");
  VEDA_REQUIRE(softmax_scale > 0.f, "softmax_scale must be positive");
  const int64_t need = veda_bsa_bwd_workspace(n_heads, n_q_tiles);
  VEDA_REQUIRE(static_cast<int64_t>(workspace_bytes) >= need,
               "workspace too small");
  VEDA_REQUIRE(reinterpret_cast<uintptr_t>(workspace) % 16 == 0,
               "workspace must be 16-byte aligned");
  auto aligned = [](const void* ptr, int64_t sn, int64_t sh) {
    return reinterpret_cast<uintptr_t>(ptr) % 16 == 0 && sn % 8 == 0 &&
           sh % 8 == 0;
  };
  VEDA_REQUIRE(aligned(out, out_stride_n, out_stride_h) &&
                   aligned(dout, dout_stride_n, dout_stride_h) &&
                   aligned(dq, dq_stride_n, dq_stride_h) &&
                   aligned(dk, dk_stride_n, dk_stride_h) &&
                   aligned(dv, dv_stride_n, dv_stride_h),
               "out, dout, dq, dk, dv must be 16-byte aligned with strides "
               "multiple of 8");
  const int64_t rows = n_q_tiles * kTile;
  float* delta = static_cast<float*>(workspace);
  float* lse2 = delta + static_cast<size_t>(n_heads) * rows;
  unsigned int* counters = reinterpret_cast<unsigned int*>(
      lse2 + static_cast<size_t>(n_heads) * rows);
  cudaStream_t s = as_stream(stream);
  VEDA_CUDA(cudaMemsetAsync(counters, 0, 2 * sizeof(unsigned int), s));
  if (n_q_tiles > 0) {
    const int64_t warps = rows * n_heads;
    bwd_prep_kernel<<<static_cast<unsigned>((warps * 32 + 255) / 256), 256, 0,
                      s>>>(static_cast<const __nv_bfloat16*>(out),
                           out_stride_n, out_stride_h,
                           static_cast<const __nv_bfloat16*>(dout),
                           dout_stride_n, dout_stride_h, lse, lse_stride_row,
                           lse_stride_h, rows, n_heads, delta, lse2);
    rc = check_launch("bwd_prep_kernel");
    if (rc != VEDA_OK) return rc;
  }
  CUtensorMap mq, mdo, mk, mv;
  rc = make_tile_map(&mq, q, rows, n_heads, q_stride_n, q_stride_h, "q");
  if (rc == VEDA_OK)
    rc = make_tile_map(&mdo, dout, rows, n_heads, dout_stride_n,
                       dout_stride_h, "dout");
  if (rc == VEDA_OK)
    rc = make_tile_map(&mk, k, n_kv_tiles * kTile, n_heads, k_stride_n,
                       k_stride_h, "k");
  if (rc == VEDA_OK)
    rc = make_tile_map(&mv, v, n_kv_tiles * kTile, n_heads, v_stride_n,
                       v_stride_h, "v");
  if (rc != VEDA_OK) return rc;
  static bool attrs = false;
  if (!attrs) {
    VEDA_CUDA(cudaFuncSetAttribute(bsa_bwd_dq_kernel,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   kDqSmem));
    VEDA_CUDA(cudaFuncSetAttribute(bsa_bwd_dkdv_kernel,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   kKvSmem));
    attrs = true;
  }
  BwdParams p{};
  p.n_heads = n_heads;
  p.n_q_tiles = static_cast<int>(n_q_tiles);
  p.n_kv_tiles = static_cast<int>(n_kv_tiles);
  p.valid_count = valid_count;
  p.delta = delta;
  p.lse2 = lse2;
  p.scale = softmax_scale;
  p.scale_log2 = softmax_scale * kLog2e;
  p.status = device_status_ptr();
  const int sms = sm_count();
  if (n_q_tiles > 0) {
    BwdParams pq = p;
    pq.lists = ListSet{static_cast<int>(n_q_tiles), part_cnt, part_idx,
                       full_cnt, full_idx, ld_idx};
    pq.counter = counters;
    pq.grad = static_cast<__nv_bfloat16*>(dq);
    pq.grad_sn = dq_stride_n;
    pq.grad_sh = dq_stride_h;
    const int64_t items = n_q_tiles * n_heads;
    const int grid = static_cast<int>(items < sms ? items : sms);
    bsa_bwd_dq_kernel<<<grid, kBwdThreads, kDqSmem, s>>>(mq, mdo, mk, mv, pq);
    rc = check_launch("bsa_bwd_dq_kernel");
    if (rc != VEDA_OK) return rc;
  }
  BwdParams pk = p;
  pk.lists = ListSet{static_cast<int>(n_kv_tiles), t_part_cnt, t_part_idx,
                     t_full_cnt, t_full_idx, ld_t_idx};
  pk.counter = counters + 1;
  pk.grad = static_cast<__nv_bfloat16*>(dk);
  pk.grad_sn = dk_stride_n;
  pk.grad_sh = dk_stride_h;
  pk.grad2 = static_cast<__nv_bfloat16*>(dv);
  pk.grad2_sn = dv_stride_n;
  pk.grad2_sh = dv_stride_h;
  const int64_t items = n_kv_tiles * n_heads;
  const int grid = static_cast<int>(items < sms ? items : sms);
  bsa_bwd_dkdv_kernel<<<grid, kBwdThreads, kKvSmem, s>>>(mq, mdo, mk, mv, pk);
  return check_launch("bsa_bwd_dkdv_kernel");
}
