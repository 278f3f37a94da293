// a9/a11: block-sparse (and dense) attention forward on tcgen05.
//
// Semantics (miowtion/kernels/reference.py:1-10, :23-56): a query row of tile
// i attends to the valid prefix of every key tile listed for i; rows with no
// key output 0 (lse -inf). Lists are the reference's BlockSparseTensors
// (miowtion/kernels/fa4.py:266-296); each list is walked in the reference
// backend's SM100 order, partial list then full list, each from its end
// (fa4_sm8x/block_sparse_utils.py:813-853); the order only changes the fp32
// summation order.
//
// Structure: a persistent kernel, one CTA per SM, walking work items (head,
// query tile) with a stride of the grid. One query tile is in flight at a
// time; the blocks of consecutive items form one sequence (b = 0, 1, ...),
// and tensor memory holds three S buffers (block b uses S[b % 3]) and O:
//     TMEM columns [  0,128) S0   [128,256) S1   [256,384) S2   [384,512) O
// so the tensor core computes S(b+1) and S(b+2) while the softmax works on
// S(b), and the softmax never waits for a QK.
//   warps 0-15 softmax and epilogue. Warp w serves query rows 32(w%4) ..
//              32(w%4)+31 (its TMEM lanes) and keys 32(w/4) .. 32(w/4)+31 of
//              every block; the four warps of a row range exchange partial
//              row maxima through shared memory (named barrier). Each warp
//              writes its P (bf16 pairs) over the first 16 columns of its
//              own 32 columns of S. Four warps per SMSP hide one another's
//              latencies.
//   warp 16    TMA producer: Q of each item (two buffers), K(b) and V(b)
//              through two 2-slot rings, each tile with a record of its block
//              for the warp that consumes it.
//   warp 17    QK issuer and TMEM owner: S(b) = Q K(b)^T once K(b) landed
//              and S[b % 3] is free (PV(b-3) finished).
//   warp 18    PV issuer: O += P(b) V(b) as the softmax writes P(b).
// Both issuers run converged with the elected lane issuing. Split this way,
// neither waits on the other's dependencies: the QK stream runs ahead while
// the PV stream waits for the softmax, and the tensor core takes MMAs from
// both. Each block runs
//     S = Q K^T          8 SS MMAs (M=N=128, K=16), 128B-swizzled K-major
//     P = exp2(S*c - m)  online softmax, lazy rescaling (the max moves only
//                        when it grows by more than 2^8), a quarter of the
//                        exponentials on an FMA polynomial
//     O += P V           8 TS MMAs (A = P from TMEM, B = V MN-major), the
//                        first four once keys 0-63 have P, the others once
//                        keys 64-127 have.
// The softmax learns a block's valid key count two blocks ahead (partial
// tiles only; full ones have 128) so that no list read stalls it.
// All mbarrier waits are bounded (common.cuh).
#include <math.h>

#include "common.cuh"
#include "exp2_poly.cuh"

namespace veda {

namespace {

// Warp roles: the softmax warps (16 in one group, 8 in two groups), then
// the TMA producer, the QK issuer (TMEM owner) and the PV issuer.
template <bool kDual>
struct Roles {
  static constexpr int kSoftmax = kDual ? 8 : 16;
  static constexpr int kProducer = kSoftmax;
  static constexpr int kQk = kSoftmax + 1;
  static constexpr int kPv = kSoftmax + 2;
  static constexpr int kThreads = 32 * (kSoftmax + 3);
};
constexpr int kSoftmaxWarps = Roles<false>::kSoftmax;
constexpr int kRing = 2;  // per K and V ring
constexpr uint32_t kTileBytes = 32768;  // 128 x 128 bf16
constexpr uint32_t kHalfBytes = 16384;  // 128 x 64 bf16 (one TMA box)
constexpr uint32_t kTmemCols = 512;
// The key tiles of the producer's current item in walk order (longer lists
// are read from global memory).
constexpr int kListCap = 1024;
// Exchange between the four warps of a row: partial maxima [block parity][4
// key quarters][128 rows] and partial sums [4 key quarters][128 rows]; for
// the fused heat, the partial sums of each block [block parity][4][128] and
// the rows' log-sum-exp [128].
constexpr int kExchangeFloats = 2 * 4 * 128 + 4 * 128 + 2 * 4 * 128 + 128;
constexpr int kSmemBytes = (2 + 2 * kRing) * kTileBytes + kListCap * 4 +
                           kExchangeFloats * 4 + 512 + 1024;

// Of each warp's 32 columns, those whose exponential runs on the FMA pipes.
// A quarter balances the MUFU (ex2 at 16 a clock per SM) against the FMA
// pipes: measured on B200 with four such warps per SMSP, 8 of 32 columns
// gives the shortest P computation (0, 16 and 32 are slower).
constexpr int kPolyCols = 8;

constexpr int kSBufs = 3;

// Video spans the packed mode reads in place (one 5D tensor map each).
constexpr int kMaxPackedSpans = 2;

enum Bar {
  kQFull = 0,       // [2] per Q buffer (item parity)
  kQEmpty = 2,      // [2] the item's last QK finished reading Q
  kKFull = 4,       // [kRing] K tile (and its record) landed
  kKEmpty = 6,      // [kRing] its QK finished
  kVFull = 8,       // [kRing] V tile (and its record) landed
  kVEmpty = 10,     // [kRing] its PV finished
  kSFull = 12,      // [3] per S buffer
  kPFull0 = 15,     // [3] P of keys 0-63 written (warps 0-7)
  kPFull1 = 18,     // [3] P of keys 64-127 written (warps 8-15)
  kPVDone = 21,     // [3] the block's PV finished (per S buffer)
  kODone = 24,      // the item's last PV finished
  kOFree = 25,      // the epilogue has read O (16 warps)
  kDrainQk = 26,    // MMAs in flight after an abort, per issuer
  kDrainPv = 27,
  kHeatIn = 28,     // fused heat: an item's row maxima / sums stored (16)
  kHeatOut = 29,    // fused heat: the item's heat written (16)
  kRefPub = 30,     // [4] two groups: block b's reference published (4)
  kVFull3 = 34,     // [3] two groups: the 3-slot V ring, tile landed
  kVEmpty3 = 37,    // [3] two groups: the 3-slot V ring, its PV finished
  kNumBars = 40
};
// Block records live after the barriers (and the TMEM slot / abort word).
constexpr int kRecOffset = 44;  // in 8-byte units from the barriers

struct FwdParams {
  int n_heads;
  int n_q_tiles;
  int n_kv_tiles;
  int n_items;
  // Optional work order: CTA c walks slots c, c + G, c + 2G, ... of
  // item_order ([n_slots / G][G], G = the grid), each slot an item
  // h * n_q_tiles + qt or -1 for none. Without it a CTA walks items c,
  // c + G, ... with each head's query tiles in reverse (the dense global
  // rows first).
  const int32_t* item_order;
  int n_slots;
  int order_ctas;    // G, the grid a work order is laid out for
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
  // Fused teacher heat (the kHeat kernel): heat [H, n_q, n_kv] at
  // h * heat_sh + qt * heat_sq + kv; per CTA a [n_kv][128] scratch of each
  // (block, row): the bf16-rounded raw score maximum (max mode) or the
  // log2 of the row's exponential sum over the block (sum mode).
  float* heat;
  int64_t heat_sh, heat_sq;
  float* heat_scratch;
  int heat_sum;
  // Packed mode (veda_bsa_fwd_packed): the output goes to row
  // box_perm[slot], head head_ids[h], of the packed [S, H, D] tensor, and
  // query tiles are read in place (box_q); key and value tiles either from
  // tile-ordered copies or in place too (box_kv). Read in place, a video
  // tile is a box of the packed tensor through a 5D map, one per span
  // (maps.x[1 + s]), and a global tile comes from the gathered copies of
  // the global tiles (maps.x[0], head h); partial key tiles are masked by
  // key_mask words (the box order is not a prefix).
  int packed;
  int box_kv;
  int total_heads;  // heads of the packed tensors
  int n_video;
  int n_spans;
  int span_begin[kMaxPackedSpans + 1];
  int span_nbt[kMaxPackedSpans], span_nbw[kMaxPackedSpans];
  int span_shape[kMaxPackedSpans][3];
  // Key and value tiles as shared-memory images (veda_gather_tile_images):
  // tile (h, kv) is 32 KB at (h * n_kv_tiles + kv) * 32 KB, loaded with one
  // bulk copy. nullptr: through the tensor maps.
  const uint8_t* k_img;
  const uint8_t* v_img;
  const int64_t* head_ids;
  const int64_t* box_perm;
  const uint32_t* key_mask;
  unsigned int* status;
};

// Tensor maps of q, k and v: [0] the tile-ordered tensors (or, in packed
// mode, the global tiles), [1 + s] the box map of span s (packed mode).
struct FwdMaps {
  CUtensorMap q[1 + kMaxPackedSpans];
  CUtensorMap k[1 + kMaxPackedSpans];
  CUtensorMap v[1 + kMaxPackedSpans];
};

// TMA coordinates of tile `tile` of one tensor (head h of the item, hg its
// packed head): the map index (0: tile order or global tiles, 1 + s: box map
// of span s) and the coordinates after the head-dim one.
struct TileCoords {
  int map, c1, c2, c3, c4;
};

__device__ __forceinline__ TileCoords tile_coords(const FwdParams& p, int h,
                                                  int hg, int tile,
                                                  bool boxed) {
  TileCoords c;
  if (boxed && tile < p.n_video) {
    const int s = (p.n_spans > 1 && tile >= p.span_begin[1]) ? 1 : 0;
    const int lt = tile - p.span_begin[s];
    const int nbt = p.span_nbt[s];
    const int rest = lt / nbt;
    const int bh = rest / p.span_nbw[s];
    c.map = 1 + s;
    c.c1 = hg;
    c.c2 = (rest - bh * p.span_nbw[s]) * p.span_shape[s][2];  // w0
    c.c3 = bh * p.span_shape[s][1];                          // h0
    c.c4 = (lt - rest * nbt) * p.span_shape[s][0];           // t0
  } else {
    c.map = 0;
    c.c1 = h;
    c.c2 = (tile - (boxed ? p.n_video : 0)) * kTile;
    c.c3 = c.c4 = 0;
  }
  return c;
}

// Issues the two 64-column TMA boxes of tile `tile` of one tensor (head h
// of the item, hg its packed head) into dst, completing on bar.
__device__ __forceinline__ void load_tile(uint8_t* dst,
                                          const CUtensorMap* maps,
                                          uint64_t* bar, const FwdParams& p,
                                          int h, int hg, int tile,
                                          bool boxed) {
  const TileCoords c = tile_coords(p, h, hg, tile, boxed);
  if (c.map > 0) {
    tma_load_5d(dst, &maps[c.map], bar, 0, c.c1, c.c2, c.c3, c.c4);
    tma_load_5d(dst + kHalfBytes, &maps[c.map], bar, 64, c.c1, c.c2, c.c3,
                c.c4);
  } else {
    tma_load_3d(dst, &maps[0], bar, 0, c.c1, c.c2);
    tma_load_3d(dst + kHalfBytes, &maps[0], bar, 64, c.c1, c.c2);
  }
}

// Heat of the key tiles jj = first, first + step, ... < len of one query
// tile, from the scratch value v of each (key tile, row): over the tile's
// 128 rows, the sum of 2^(v - lse2[row]) (sum mode, v the log2 of the
// row's exponential sum over the block against the row's reference) or
// 2^(max of v c - lse2[row]) (max mode, v the raw score maximum). One warp
// per key tile, lane l reading rows l, l + 32, l + 64, l + 96; four key
// tiles per round, so that each lane has 16 loads in flight.
template <typename KvOf>
__device__ __forceinline__ void reduce_heat(const float* hs,
                                            const float* lse2, int first,
                                            int step, int len, bool sum,
                                            float scale_log2, float* dst,
                                            KvOf kv_of, int lane) {
  for (int j0 = first; j0 < len; j0 += 4 * step) {
    float v[4][4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int jj = j0 + u * step;
#pragma unroll
      for (int i = 0; i < 4; ++i)
        v[u][i] = jj < len ? hs[jj * kTile + lane + 32 * i] : 0.f;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int jj = j0 + u * step;
      float acc = sum ? 0.f : -INFINITY;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float l2 = lse2[lane + 32 * i];
        acc = sum ? acc + ex2_approx(v[u][i] - l2)
                  : fmaxf(acc, fmaf(v[u][i], scale_log2, -l2));
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        const float o2 = __shfl_xor_sync(0xffffffffu, acc, off);
        acc = sum ? acc + o2 : fmaxf(acc, o2);
      }
      if (lane == 0 && jj < len) dst[kv_of(jj)] = sum ? acc : ex2_approx(acc);
    }
  }
}

// One key block of a slot's stream.
struct Block {
  int h, qt;   // work item
  int kv;      // key tile
  int valid;   // valid key rows of the tile (128 when full)
  int blk;     // running block number of the slot (barrier phases)
  int ka;      // running number of non-empty items of the slot
  bool first, second, last;
};

// The work items of one slot, item by item and block by block. Every role
// walks the same sequence, so they agree on barrier phases without talking.
struct Stream {
  int it, stride;
  int h, qt, pc, fc, len;
  int64_t off;
  int j, blk, ka;
  // List lengths of item it + stride, loaded one item ahead so that their
  // latency overlaps the current item.
  int npc, nfc;

  bool pad;  // the slot holds no item (work order padding)

  // Row (h * n_q_tiles + qt) of slot `slot`, or -1.
  __device__ int64_t row_of(const FwdParams& p, int slot) const {
    if (p.item_order != nullptr) return p.item_order[slot];
    // Heaviest query tiles (the dense global rows, last in tile order)
    // first.
    return static_cast<int64_t>(slot / p.n_q_tiles) * p.n_q_tiles +
           (p.n_q_tiles - 1 - slot % p.n_q_tiles);
  }

  __device__ void fetch(const FwdParams& p, int slot) {
    npc = 0;
    nfc = 0;
    if (slot >= p.n_slots) return;
    const int64_t row = row_of(p, slot);
    if (row < 0) return;
    if (p.dense) {
      nfc = p.n_kv_tiles;
      return;
    }
    npc = p.part_cnt[row];
    nfc = p.full_cnt[row];
  }

  __device__ void load_item(const FwdParams& p) {
    const int64_t row = row_of(p, it);
    pad = row < 0;
    h = pad ? 0 : static_cast<int>(row / p.n_q_tiles);
    qt = pad ? 0 : static_cast<int>(row % p.n_q_tiles);
    off = p.dense ? 0 : (pad ? 0 : row * p.ld_idx);
    pc = npc;
    fc = nfc;
    len = pc + fc;
    j = 0;
    fetch(p, it + stride);
  }

  // Moves past padding slots (never items, not even empty ones).
  __device__ void skip_pads(const FwdParams& p) {
    while (it < p.n_slots && pad) {
      it += stride;
      if (it < p.n_slots) load_item(p);
    }
  }

  // Positions on the first item (on the first non-empty one unless
  // `keep_empty`, which the softmax uses to write the empty items' rows).
  __device__ void init(const FwdParams& p, int first, int step,
                       bool keep_empty) {
    it = first;
    stride = step;
    blk = 0;
    ka = -1;
    pad = false;
    if (it < p.n_slots) {
      fetch(p, it);
      load_item(p);
      skip_pads(p);
      if (it < p.n_slots && len > 0) ka = 0;
      if (!keep_empty) skip_empty(p);
    }
  }

  __device__ void skip_empty(const FwdParams& p) {
    while (it < p.n_slots && len == 0) {
      it += stride;
      if (it < p.n_slots) {
        load_item(p);
        skip_pads(p);
        if (it < p.n_slots && len > 0) ++ka;
      }
    }
  }

  __device__ void next_item(const FwdParams& p, bool keep_empty) {
    it += stride;
    if (it < p.n_slots) {
      load_item(p);
      skip_pads(p);
      if (it < p.n_slots && len > 0) ++ka;
      if (!keep_empty) skip_empty(p);
    }
  }

  __device__ bool valid(const FwdParams& p) const { return it < p.n_slots; }

  // The current block without its key tile (no memory access).
  __device__ Block flags() const {
    Block b{};
    b.h = h;
    b.qt = qt;
    b.blk = blk;
    b.ka = ka;
    b.first = j == 0;
    b.second = j == 1;
    b.last = j == len - 1;
    return b;
  }

  // Key tile of block jj of the current item, read from global memory.
  __device__ int kv_global(const FwdParams& p, int jj) const {
    if (p.dense) return jj;
    return jj < pc ? p.part_idx[off + (pc - 1 - jj)]
                   : p.full_idx[off + (fc - 1 - (jj - pc))];
  }

  // Next block; at the end of an item, the next (non-empty) item.
  __device__ void next_block(const FwdParams& p) {
    ++blk;
    if (++j < len) return;
    next_item(p, false);
  }
};

__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Max of 32 values as a shallow tree of three-input max instructions.
__device__ __forceinline__ float row_max32(const float* s) {
  float m[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) m[i] = max3(s[i], s[8 + i], s[16 + i]);
#pragma unroll
  for (int i = 0; i < 8; ++i) m[i] = fmaxf(m[i], s[24 + i]);
  return max3(max3(m[0], m[1], m[2]), max3(m[3], m[4], m[5]),
              fmaxf(m[6], m[7]));
}

// O *= alpha for 32 columns of this thread's row (its TMEM lane).
__device__ __forceinline__ void rescale_o32(uint32_t t_row, float alpha) {
  uint32_t o[32];
  tmem_ld32(t_row, o);
  tmem_wait_ld();
#pragma unroll
  for (int i = 0; i < 32; ++i)
    o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
  tmem_st32(t_row, o);
  tmem_wait_st();
}

// O *= alpha for 16 columns of this thread's row (fewer live registers,
// for the rare rescale of the two-group softmax).
__device__ __forceinline__ void rescale_o16(uint32_t t_row, float alpha) {
  uint32_t o[16];
  tmem_ld16(t_row, o);
  tmem_wait_ld();
#pragma unroll
  for (int i = 0; i < 16; ++i)
    o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
  tmem_st16(t_row, o);
  tmem_wait_st();
}

// P for this warp's 32 keys: x = s*c - m, exp2 on the MUFU (or, for the last
// kPolyCols columns, on the FMA pipes), bf16 pairs into r[c/2]. Returns the
// (fp32) sum of the exponentials.
__device__ __forceinline__ float2 p32(uint32_t* r, const float* s,
                                      float2 scale2, float2 neg_m2) {
  float2 sum_a = make_float2(0.f, 0.f), sum_b = make_float2(0.f, 0.f);
#pragma unroll
  for (int c = 0; c < 32; c += 4) {
    const float2 x0 = __ffma2_rn(make_float2(s[c], s[c + 1]), scale2, neg_m2);
    const float2 x1 =
        __ffma2_rn(make_float2(s[c + 2], s[c + 3]), scale2, neg_m2);
    float2 e0, e1;
    if (c >= 32 - kPolyCols) {
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
  return __fadd2_rn(sum_a, sum_b);
}

// Named barrier for the four warps of a row range (128 threads; ids 1-4, 0
// is __syncthreads).
__device__ __forceinline__ void row_sync(int id) {
  asm volatile("bar.sync %0, 128;" ::"r"(id) : "memory");
}

// Two-group softmax: the two warps (one per group) of a row range, 64
// threads (ids 1-4).
__device__ __forceinline__ void quarter_sync(int id) {
  asm volatile("bar.sync %0, 64;" ::"r"(id) : "memory");
}

// Warp-uniform wait: tcgen05.ld/st after it are warp-wide instructions.
__device__ __forceinline__ bool wait_all(uint64_t* bar, uint32_t parity,
                                         volatile int* abort,
                                         unsigned int* status) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort, status));
}

// The record of a block, written by the producer before the block's K copy
// and published by that ring slot's full barrier, so the MMA warp needs no
// walk of the work stream. With ka the item's number among the CTA's
// non-empty items: bit 0 end of the stream, bit 1 first block of the item,
// bit 2 last block, bit 3 ka & 1 (its Q buffer, and the parity of the O
// barriers' phase), bit 4 (ka >> 1) & 1 (the parity of the Q buffer's
// phase), bit 5 ka >= 1 (O held an earlier item).
constexpr uint32_t kRecEnd = 1, kRecFirst = 2, kRecLast = 4, kRecItem = 8,
                   kRecQPhase = 16, kRecLater = 32, kRecSecond = 64;

__device__ __forceinline__ uint32_t block_record(const Block& b) {
  return (b.first ? kRecFirst : 0u) | (b.second ? kRecSecond : 0u) |
         (b.last ? kRecLast : 0u) |
         ((b.ka & 1) ? kRecItem : 0u) | (((b.ka >> 1) & 1) ? kRecQPhase : 0u) |
         (b.ka >= 1 ? kRecLater : 0u);
}

// kDual: the two-group softmax (see the comment at the softmax role).
template <bool kHeat, bool kDual>
__global__ void __launch_bounds__(Roles<kDual>::kThreads, 1)
    bsa_fwd_kernel(const __grid_constant__ FwdMaps maps, FwdParams p) {
  static_assert(!(kHeat && kDual), "the fused heat uses the one-group path");
  // Shared memory holds six 32 KB tiles. One group: Q double-buffered
  // (the next item's Q loads while the current item runs), K and V rings of
  // two. Two groups: one Q buffer and a V ring of three, since V(b) can
  // only start loading when PV(b - ring) has finished and a tile takes
  // longer to land than one PV lasts (measured: with two slots the PV
  // waited for V in most blocks).
  constexpr int kQBufs = kDual ? 1 : 2;
  constexpr int kRingV = kDual ? 3 : 2;
  constexpr int kVFullB = kDual ? kVFull3 : kVFull;
  constexpr int kVEmptyB = kDual ? kVEmpty3 : kVEmpty;
  static_assert(kQBufs + kRing + kRingV == 6, "six tiles of shared memory");
  constexpr uint32_t kSB = static_cast<uint32_t>(kSBufs);
  constexpr int kSoftmaxN = Roles<kDual>::kSoftmax;
  constexpr int kProducerWarp = Roles<kDual>::kProducer;
  constexpr int kMmaWarp = Roles<kDual>::kQk;
  constexpr int kPvWarp = Roles<kDual>::kPv;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* s_q = smem;                           // [kQBufs] x 32 KB
  uint8_t* s_k = smem + kQBufs * kTileBytes;     // [kRing] x 32 KB
  uint8_t* s_v = s_k + kRing * kTileBytes;       // [kRingV] x 32 KB
  int32_t* s_list =
      reinterpret_cast<int32_t*>(smem + (2 + 2 * kRing) * kTileBytes);
  float* s_xchg = reinterpret_cast<float*>(s_list + kListCap);
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_xchg + kExchangeFloats);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  static_assert(kNumBars + 1 <= kRecOffset,
                "barriers overlap the block records");
  static_assert(kRecOffset * 8 + (kRing + 3) * 4 <= 512, "barrier area");
  // Block records beside the K and the V ring slots.
  volatile uint32_t* k_rec =
      reinterpret_cast<volatile uint32_t*>(bars + kRecOffset);
  volatile uint32_t* v_rec = k_rec + kRing;

  const int tid = threadIdx.x;
  const int warp = tid / 32;
  const int lane = tid % 32;

  if (tid == 0) {
    for (int b = 0; b < kNumBars; ++b) {
      uint32_t count = 1;
      // P halves: 8 warps (one group), or P of the whole block: the 4
      // warps of one group (two groups).
      if (b >= kPFull0 && b < kPFull1 + kSBufs)
        count = kDual ? 4 : kSoftmaxN / 2;
      if (b >= kRefPub && b < kRefPub + 4) count = 4;
      if (b == kOFree || b == kHeatIn || b == kHeatOut) count = kSoftmaxN;
      mbar_init(&bars[b], count);
    }
    *abort = 0;
    fence_barrier_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kProducerWarp) {
    // ---------------- TMA producer (one warp) ----------------
    // K(b) through the K ring, V(b) through the V ring, V two blocks behind
    // K (the PV of a block trails its QK by the softmax); Q of an item
    // before its first K; end records after the last tiles. The whole warp
    // walks the stream (it copies each item's list to shared memory) and
    // waits converged; lane 0 issues the copies.
    if (lane < 3 * (1 + kMaxPackedSpans)) {
      const int m = lane % (1 + kMaxPackedSpans);
      const bool boxed = lane < 1 + kMaxPackedSpans ? p.packed : p.box_kv;
      const bool used = boxed ? (m == 0 ? p.n_video < p.n_q_tiles
                                        : m <= p.n_spans)
                              : m == 0;
      const CUtensorMap* base = lane < 1 + kMaxPackedSpans ? maps.q
                                : lane < 2 * (1 + kMaxPackedSpans) ? maps.k
                                                                 : maps.v;
      if (used) prefetch_tensor_map(&base[m]);
    }
    Stream st;
    st.init(p, blockIdx.x, gridDim.x, false);
    int nk = 0, nv = 0;  // K and V tiles loaded
    int q_issued = 0;    // items whose Q was loaded
    // Key tile, head (local and packed) and record of blocks b - 1 and
    // b - 2; the packed head of the current item.
    int kv1 = 0, h1 = 0, kv2 = 0, h2 = 0, g1 = 0, g2 = 0, hg = 0;
    uint32_t r1 = 0, r2 = 0;
    bool run = true;
    // Waits for a free slot of a ring (n tiles loaded so far); -1 on abort.
    auto slot_of = [&](int n, int empty_bar, int ring) -> int {
      const int slot = n % ring;
      if (n >= ring && !wait_all(&bars[empty_bar + slot],
                                 ((n / ring) - 1) & 1, abort, p.status))
        return -1;
      return slot;
    };
    auto load = [&](const CUtensorMap* map, const uint8_t* img,
                    uint8_t* ring, int full_bar, int slot, int h, int g,
                    int kv) {
      uint8_t* dst = ring + slot * kTileBytes;
      mbar_arrive_expect_tx(&bars[full_bar + slot], kTileBytes);
      if (img != nullptr)
        bulk_load(dst,
                  img + (static_cast<int64_t>(h) * p.n_kv_tiles + kv) *
                            static_cast<int64_t>(kTileBytes),
                  kTileBytes, &bars[full_bar + slot]);
      else
        load_tile(dst, map, &bars[full_bar + slot], p, h, g, kv, p.box_kv);
    };
    auto load_v = [&](int h, int g, int kv, uint32_t rec) -> bool {
      const int slot = slot_of(nv, kVEmptyB, kRingV);
      if (slot < 0) return false;
      if (lane == 0) {
        v_rec[slot] = rec;
        load(maps.v, p.v_img, s_v, kVFullB, slot, h, g, kv);
      }
      __syncwarp();
      ++nv;
      return true;
    };
    while (st.valid(p)) {
      const Block b = st.flags();
      if (b.first) {
        if (!p.dense && st.len <= kListCap)
          for (int jj = lane; jj < st.len; jj += 32)
            s_list[jj] = st.kv_global(p, jj);
        __syncwarp();
        hg = p.packed ? static_cast<int>(p.head_ids[b.h]) : b.h;
        // The Q buffer frees after the last QK of the item two back (one
        // group) or one back (two groups, one buffer).
        const int qb = kDual ? 0 : b.ka & 1;
        const bool qwait = kDual ? b.ka >= 1 : b.ka >= 2;
        const uint32_t qpar = kDual ? (b.ka - 1) & 1 : ((b.ka >> 1) & 1) ^ 1;
        if (qwait && !wait_all(&bars[kQEmpty + qb], qpar, abort, p.status)) {
          run = false;
          break;
        }
        if (lane == 0) {
          uint8_t* dst = s_q + qb * kTileBytes;
          mbar_arrive_expect_tx(&bars[kQFull + qb], kTileBytes);
          load_tile(dst, maps.q, &bars[kQFull + qb], p, b.h, hg, b.qt,
                    p.packed);
        }
        __syncwarp();
        q_issued = b.ka + 1;
      }
      const int kv = p.dense ? st.j
                             : (st.len <= kListCap ? s_list[st.j]
                                                   : st.kv_global(p, st.j));
      const uint32_t rec = block_record(b);
      const int slot = slot_of(nk, kKEmpty, kRing);
      if (slot < 0) {
        run = false;
        break;
      }
      if (lane == 0) {
        k_rec[slot] = rec;
        load(maps.k, p.k_img, s_k, kKFull, slot, b.h, hg, kv);
      }
      __syncwarp();
      ++nk;
      if (nk >= 3 && !load_v(h2, g2, kv2, r2)) {
        run = false;
        break;
      }
      kv2 = kv1;
      h2 = h1;
      g2 = g1;
      r2 = r1;
      kv1 = kv;
      h1 = b.h;
      g1 = hg;
      r1 = rec;
      st.next_block(p);
    }
    if (run) {
      // The last V tiles, then an end record in each ring (completing the
      // slot's full barrier without a copy).
      if (nk >= 2) run = load_v(h2, g2, kv2, r2);
      if (run && nk >= 1) run = load_v(h1, g1, kv1, r1);
      int slot = run ? slot_of(nk, kKEmpty, kRing) : -1;
      if (slot >= 0) {
        if (lane == 0) {
          k_rec[slot] = kRecEnd;
          mbar_arrive(&bars[kKFull + slot]);
        }
        __syncwarp();
        slot = slot_of(nv, kVEmptyB, kRingV);
        if (slot >= 0) {
          if (lane == 0) {
            v_rec[slot] = kRecEnd;
            mbar_arrive(&bars[kVFullB + slot]);
          }
          __syncwarp();
        }
      }
    }
    if (lane == 0 && *abort) {
      // Let the copies already in flight land before the CTA retires.
      volatile int never = 0;
      for (int ka = q_issued - kQBufs; ka < q_issued; ++ka)
        if (ka >= 0)
          mbar_wait(&bars[kQFull + (kDual ? 0 : ka & 1)],
                    kDual ? ka & 1 : (ka >> 1) & 1, &never, nullptr);
      for (int k = nk - kRing; k < nk; ++k)
        if (k >= 0)
          mbar_wait(&bars[kKFull + k % kRing], (k / kRing) & 1, &never,
                    nullptr);
      for (int k = nv - kRingV; k < nv; ++k)
        if (k >= 0)
          mbar_wait(&bars[kVFullB + k % kRingV], (k / kRingV) & 1, &never,
                    nullptr);
    }
  } else if (warp == kMmaWarp) {
    // ---------------- QK issuer ----------------
    constexpr uint32_t idesc_qk = idesc_bf16(128, 128, false, false);
    // Descriptor low halves; per step only a constant is added (16-byte
    // units): K-major steps advance 32 B inside a 128-B swizzle row and
    // jump to the second 64-column box after four steps.
    const uint32_t q_lo = sw128_desc_lo(smem_u32(s_q), 16);
    const uint32_t k_lo = sw128_desc_lo(smem_u32(s_k), 16);
    constexpr uint32_t kTileUnits = kTileBytes >> 4;
    for (uint32_t b = 0;; ++b) {
      const int slot = b % kRing;
      if (!wait_all(&bars[kKFull + slot], (b / kRing) & 1, abort, p.status))
        break;
      const uint32_t rec = k_rec[slot];
      if (rec & kRecEnd) break;
      const uint32_t sb = b % kSB;
      // One group: Q buffer ka & 1, phase (ka >> 1) & 1; two groups: the one
      // buffer, phase ka & 1.
      const uint32_t qb = kDual ? 0u : ((rec & kRecItem) ? 1u : 0u);
      const uint32_t qphase = kDual ? ((rec & kRecItem) ? 1u : 0u)
                                    : ((rec & kRecQPhase) ? 1u : 0u);
      // S[sb] held P of block b - kSB: its PV must have finished.
      if (b >= kSB && !wait_all(&bars[kPVDone + sb],
                                ((b / kSB) - 1) & 1, abort, p.status))
        break;
      if ((rec & kRecFirst) &&
          !wait_all(&bars[kQFull + qb], qphase, abort, p.status))
        break;
      tc_fence_after();
      const uint32_t a = q_lo + qb * kTileUnits;
      const uint32_t b_ = k_lo + slot * kTileUnits;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t off = (kk >> 2) * (kHalfBytes >> 4) + (kk & 3) * 2;
        umma_ss_warp(tmem + sb * 128, a + off, b_ + off, idesc_qk,
                     kk > 0 ? 1u : 0u);
      }
      umma_commit_warp(&bars[kSFull + sb]);
      umma_commit_warp(&bars[kKEmpty + slot]);
      if (rec & kRecLast) umma_commit_warp(&bars[kQEmpty + qb]);
    }
    if (*abort) {
      // Let the MMAs in flight finish before TMEM is released.
      volatile int never = 0;
      umma_commit_warp(&bars[kDrainQk]);
      mbar_wait(&bars[kDrainQk], 0, &never, nullptr);
    }
  } else if (warp == kPvWarp) {
    // ---------------- PV issuer ----------------
    constexpr uint32_t idesc_pv = idesc_bf16(128, 128, false, true);
    // V steps advance 16 key rows (2 KB) in the MN-major V tile.
    const uint32_t v_lo = sw128_desc_lo(smem_u32(s_v), kHalfBytes);
    constexpr uint32_t kTileUnits = kTileBytes >> 4;
    const uint32_t t_o0 = tmem + kSB * 128;
    for (uint32_t b = 0;; ++b) {
      const int slot = b % kRingV;
      if (!wait_all(&bars[kVFullB + slot], (b / kRingV) & 1, abort,
                    p.status))
        break;
      const uint32_t rec = v_rec[slot];
      if (rec & kRecEnd) break;
      const uint32_t sb = b % kSB;
      const uint32_t spar = (b / kSB) & 1;
      const bool first = rec & kRecFirst;
      const uint32_t t_o = t_o0;
      const bool fresh = first;
      // The item's first PV overwrites O: the epilogue must have read the
      // previous item's.
      if (first && (rec & kRecLater) &&
          !wait_all(&bars[kOFree], (rec & kRecItem) ? 0u : 1u, abort,
                    p.status))
        break;
      if (!wait_all(&bars[kPFull0 + sb], spar, abort, p.status)) break;
      tc_fence_after();
      const uint32_t bv = v_lo + slot * kTileUnits;
      // Two groups: P of the block is in columns [0, 64) of S[sb], keys
      // 0-63 (kPFull0) then 64-127 (kPFull1).
      const uint32_t t_p = tmem + sb * 128;
      // P of key step kk (16 keys, 8 columns): one group, the first 16
      // columns of its key quarter's 32; two groups, columns 8 kk.
      auto p_col = [](int kk) -> uint32_t {
        return kDual ? kk * 8 : (kk >> 1) * 32 + (kk & 1) * 8;
      };
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        umma_ts_warp(t_o, t_p + p_col(kk), bv + kk * 128, idesc_pv,
                     (kk > 0 || !fresh) ? 1u : 0u);
      if (!wait_all(&bars[kPFull1 + sb], spar, abort, p.status)) break;
      tc_fence_after();
#pragma unroll
      for (int kk = 4; kk < 8; ++kk)
        umma_ts_warp(t_o, t_p + p_col(kk), bv + kk * 128, idesc_pv, 1u);
      umma_commit_warp(&bars[kVEmptyB + slot]);
      umma_commit_warp(&bars[kPVDone + sb]);
      if (rec & kRecLast) umma_commit_warp(&bars[kODone]);
    }
    if (*abort) {
      volatile int never = 0;
      umma_commit_warp(&bars[kDrainPv]);
      mbar_wait(&bars[kDrainPv], 0, &never, nullptr);
    }
  } else if constexpr (kDual) {
    // -------------- softmax + epilogue, two groups (warps 0-7) -------------
    // Group g = warp / 4 takes the blocks whose running number blk has
    // parity g, so the two groups work on consecutive blocks at once: while
    // one loads S and stores P, the other computes exponentials. Warp w
    // serves query row 32 (w % 4) + lane (its TMEM lane) over all 128 keys
    // of its blocks, so no maxima cross warps inside a group. Both groups
    // feed the one accumulator O with P against one running reference per
    // row, handed from block to block through shared memory: block b's
    // group publishes the reference it used (xref[b % 4], barrier
    // kRefPub + b % 4), and block b + 1's group starts from it. A block
    // takes its own maximum as the reference on the item's first block and
    // when a row's maximum passes the reference by more than 8 (log2
    // units); O is then rescaled once the PV of block b - 1 has finished
    // (the PV of block b waits for P(b), which comes after). Each group
    // keeps its row sum relative to the reference of its latest block; the
    // epilogue brings both to the final (largest) reference.
    const int grp = warp / 4;
    const int quarter = warp % 4;
    const int row = quarter * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    float* xref = s_xchg;          // [4][128]
    float* xm = s_xchg + 4 * 128;  // [item parity][grp][128]
    float* xl = xm + 2 * 2 * 128;  // [item parity][grp][128]
    static_assert(4 * 128 + 2 * (2 * 2 * 128) <= kExchangeFloats,
                  "exchange area");
    const int quarter_bar = 1 + quarter;  // the two warps of a row range
    const uint32_t t_o = tmem + kSB * 128 + lane_base;
    const float2 scale2 = make_float2(p.scale_log2, p.scale_log2);
    Stream st;
    st.init(p, blockIdx.x, gridDim.x, true);
    auto part_kv = [&](int jj) -> int {
      return p.part_idx[st.off + (st.pc - 1 - jj)];
    };
    // Valid keys [32 q32, 32 q32 + 32) of a prefix tile with `valid` real
    // rows, as a bit mask.
    auto count_word = [](int valid, int q32) -> uint32_t {
      const int n = valid - q32 * 32;
      return n >= 32 ? ~0u : (n <= 0 ? 0u : (1u << n) - 1u);
    };
    // Valid keys of block jj of the current item: the tile's real rows,
    // or -1 - kv with the packed mode's box masks.
    auto block_valid = [&](int jj) -> int {
      if (p.dense) {
        const int64_t rest = p.used - static_cast<int64_t>(jj) * kTile;
        return rest < kTile ? static_cast<int>(rest) : kTile;
      }
      if (jj >= st.pc) return kTile;
      const int kv = part_kv(jj);
      return p.key_mask != nullptr ? -1 - kv : p.valid_count[kv];
    };
    auto mask_chunk = [&](uint32_t* x, int q32, int valid) {
      if (valid != kTile) {
        const uint32_t word = valid < 0 ? p.key_mask[(-1 - valid) * 4 + q32]
                                        : count_word(valid, q32);
        float* f = reinterpret_cast<float*>(x);
#pragma unroll
        for (int c = 0; c < 32; ++c)
          if (!((word >> c) & 1u)) f[c] = -INFINITY;
      }
    };
    int items = 0;
    bool ok = true;
    while (ok && st.valid(p)) {
      const int h = st.h, qt = st.qt, len = st.len, ka = st.ka;
      const int blk0 = st.blk;
      const int j0 = (blk0 & 1) == grp ? 0 : 1;  // this group's first block
      float m_last = -INFINITY;  // reference of this group's latest block
      float l = 0.f;             // this group's row sum, against m_last
      // Output row of this thread's query row (packed mode: from the box
      // layout, loaded here so that the epilogue does not wait for it).
      const int64_t slot_row = static_cast<int64_t>(qt) * kTile + row;
      int64_t out_off = -1;  // element offset of the row's output; -1: none
      if (p.packed) {
        const int64_t r = p.box_perm[slot_row];
        const int64_t hg = p.head_ids[h];
        // A head outside the tensors reads zeros (TMA bounds) and writes
        // nothing.
        if (r >= 0 && hg >= 0 && hg < p.total_heads)
          out_off = r * p.out_stride_n + hg * p.out_stride_h;
      } else if (!p.dense || slot_row < p.used) {
        // Dense mode: rows >= used keep the zeros written before the launch.
        out_off = slot_row * p.out_stride_n + h * p.out_stride_h;
      }
      int vnext = j0 < len ? block_valid(j0) : kTile;
      for (int j = j0; j < len; j += 2) {
        const int valid = vnext;
        // The next block's valid count loads while this block computes.
        if (j + 2 < len) vnext = block_valid(j + 2);
        const uint32_t blk = static_cast<uint32_t>(blk0 + j);
        const uint32_t sb = blk % kSB;
        if (!wait_all(&bars[kSFull + sb], (blk / kSB) & 1, abort,
                      p.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t t_s = tmem + sb * 128 + lane_base;
        // All 128 scores of the row in one round trip to tensor memory.
        uint32_t x[4][32];
#pragma unroll
        for (int q32 = 0; q32 < 4; ++q32) tmem_ld32(t_s + q32 * 32, x[q32]);
        tmem_wait_ld();
        float mx = -INFINITY;
#pragma unroll
        for (int q32 = 0; q32 < 4; ++q32) {
          mask_chunk(x[q32], q32, valid);
          mx = fmaxf(mx, row_max32(reinterpret_cast<float*>(x[q32])));
        }
        const float mb = mx * p.scale_log2;
        float m_use = mb;  // the item's first block: its own maximum
        bool rescale = false;
        float alpha = 1.0f;
        if (j > 0) {
          // The reference after block blk - 1 (the other group's).
          const uint32_t pb = blk - 1;
          if (!wait_all(&bars[kRefPub + (pb & 3)], (pb >> 2) & 1, abort,
                        p.status)) {
            ok = false;
            break;
          }
          const float m_prev = xref[(pb & 3) * 128 + row];
          const bool grow = mb > m_prev + 8.0f;
          rescale = __any_sync(0xffffffffu, grow);
          m_use = grow ? mb : m_prev;
          if (rescale) alpha = ex2_approx(m_prev - m_use);
        }
        // Publish this block's reference before its exponentials.
        xref[(blk & 3) * 128 + row] = m_use;
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[kRefPub + (blk & 3)]);
        if (rescale) {
          // O holds the PV of every block before blk once the PV of blk - 1
          // has finished; the PV of blk waits for this block's P.
          const uint32_t pb = blk - 1;
          if (!wait_all(&bars[kPVDone + pb % kSB], (pb / kSB) & 1, abort,
                        p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll 1
          for (int q16 = 0; q16 < 8; ++q16)
            rescale_o16(t_o + q16 * 16, alpha);
        }
        // P = 2^(s c - m_use), packed in place over the first 16 words of
        // each chunk, stored and released in two halves (keys 0-63, then
        // 64-127) so the first PVs start before the second half's
        // exponentials. P of key 2i, 2i + 1 goes to column i of S[sb].
        const float2 negm2 = make_float2(-m_use, -m_use);
        float2 sums[4];
#pragma unroll
        for (int half = 0; half < 2; ++half) {
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            const int q32 = half * 2 + q;
            sums[q32] = p32(x[q32], reinterpret_cast<float*>(x[q32]), scale2,
                            negm2);
            tmem_st16(t_s + q32 * 16, x[q32]);
          }
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0)
            mbar_arrive(&bars[(half == 0 ? kPFull0 : kPFull1) + sb]);
        }
        // This group's row sum follows the reference.
        if (m_use != m_last) l *= ex2_approx(m_last - m_use);
        m_last = m_use;
        l += ((sums[0].x + sums[0].y) + (sums[1].x + sums[1].y)) +
             ((sums[2].x + sums[2].y) + (sums[3].x + sums[3].y));
      }
      if (!ok) break;
      st.j = len;
      st.blk = blk0 + len;
      // ---------------- epilogue of the item ----------------
      const int ip = items & 1;
      xm[(ip * 2 + grp) * 128 + row] = m_last;
      xl[(ip * 2 + grp) * 128 + row] = l;
      quarter_sync(quarter_bar);
      const float m0 = xm[(ip * 2) * 128 + row];
      const float m1 = xm[(ip * 2 + 1) * 128 + row];
      const float l0 = xl[(ip * 2) * 128 + row];
      const float l1 = xl[(ip * 2 + 1) * 128 + row];
      // The final reference is the larger one (references only grow).
      const float m = fmaxf(m0, m1);
      const float l_row = (l0 > 0.f ? l0 * ex2_approx(m0 - m) : 0.f) +
                          (l1 > 0.f ? l1 * ex2_approx(m1 - m) : 0.f);
      if (len > 0 && !wait_all(&bars[kODone], ka & 1, abort, p.status)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const float inv_l = len > 0 ? 1.0f / l_row : 0.f;
      // This warp writes output columns [64 grp, 64 grp + 64) of its row.
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int col = grp * 64 + half * 32;
        uint32_t o[32];
        if (len > 0) {
          tmem_ld32(t_o + col, o);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0u;
        }
        if (out_off >= 0) {
          uint4* d4 = reinterpret_cast<uint4*>(p.out + out_off + col);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            d4[i] = make_uint4(
                pack_bf16(__uint_as_float(o[8 * i]) * inv_l,
                          __uint_as_float(o[8 * i + 1]) * inv_l),
                pack_bf16(__uint_as_float(o[8 * i + 2]) * inv_l,
                          __uint_as_float(o[8 * i + 3]) * inv_l),
                pack_bf16(__uint_as_float(o[8 * i + 4]) * inv_l,
                          __uint_as_float(o[8 * i + 5]) * inv_l),
                pack_bf16(__uint_as_float(o[8 * i + 6]) * inv_l,
                          __uint_as_float(o[8 * i + 7]) * inv_l));
        }
      }
      if (len > 0) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[kOFree]);  // O may be overwritten
      }
      if (grp == 0 && p.lse != nullptr && out_off >= 0)
        p.lse[slot_row * p.lse_stride_row + h * p.lse_stride_h] =
            len > 0 ? (m + lg2_approx(l_row)) * 0.69314718055994531f
                    : -INFINITY;
      ++items;
      st.next_item(p, true);
    }
  } else {
    // ---------------- softmax + epilogue (warps 0-15) ----------------
    const int kq = warp / 4;       // keys [32 kq, 32 kq + 32) of a block
    const int quarter = warp % 4;  // TMEM lane quarter
    const int row = quarter * 32 + lane;  // query row of the tile
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    float* xmax = s_xchg;            // [block parity][key quarter][row]
    float* xsum = s_xchg + 2 * 512;  // [key quarter][row]
    float* xbs = xsum + 512;         // [block parity][key quarter][row]
    float* s_hl = xbs + 2 * 512;     // [row] log2-sum-exp (fused heat)
    // Fused heat: this CTA's scratch, the previous block's partial sum and
    // the reference maximum it used, and the items whose heat was written.
    float* hs = nullptr;
    if constexpr (kHeat)
      hs = p.heat_scratch +
           static_cast<int64_t>(blockIdx.x) * p.n_kv_tiles * kTile;
    float bsum_prev = 0.f, mref_prev = 0.f;
    int heat_items = 0;
    const uint32_t t_o = tmem + kSBufs * 128 + kq * 32 + lane_base;
    Stream st;
    st.init(p, blockIdx.x, gridDim.x, true);
    // Valid key count of block jj of the current item: partial tiles from
    // valid_count (part list first, walked from its end), full ones 128.
    auto part_kv = [&](int jj) -> int {
      return p.part_idx[st.off + (st.pc - 1 - jj)];
    };
    // Valid keys among this warp's 32 of a key tile, as a bit mask: the
    // first `valid - 32 kq` of a prefix tile, or the packed mode's box mask.
    auto count_word = [&](int valid) -> uint32_t {
      const int n = valid - kq * 32;
      return n >= 32 ? ~0u : (n <= 0 ? 0u : (1u << n) - 1u);
    };
    auto tile_word = [&](int kv) -> uint32_t {
      return p.key_mask != nullptr ? p.key_mask[kv * 4 + kq]
                                   : count_word(p.valid_count[kv]);
    };
    auto dense_word = [&](int jj) -> uint32_t {
      const int64_t rest = p.used - static_cast<int64_t>(jj) * kTile;
      return count_word(rest < kTile ? static_cast<int>(rest) : kTile);
    };
    bool ok = true;
    while (ok && st.valid(p)) {
      const int h = st.h, qt = st.qt, len = st.len, ka = st.ka, pc = st.pc;
      float m_ref = -INFINITY;  // running max, in log2 units
      float l = 0.f;            // this warp's part of the row sum
      // Output row of this thread's query row (packed mode: from the box
      // layout, loaded here so that the epilogue does not wait for it).
      const int64_t slot_row = static_cast<int64_t>(qt) * kTile + row;
      int64_t out_off = -1;  // element offset of the row's output; -1: none
      if (p.packed) {
        const int64_t r = p.box_perm[slot_row];
        const int64_t hg = p.head_ids[h];
        // A head outside the tensors reads zeros (TMA bounds) and writes
        // nothing.
        if (r >= 0 && hg >= 0 && hg < p.total_heads)
          out_off = r * p.out_stride_n + hg * p.out_stride_h;
      } else if (!p.dense || slot_row < p.used) {
        // Dense mode: rows >= used keep the zeros written before the launch.
        out_off = slot_row * p.out_stride_n + h * p.out_stride_h;
      }
      // Pipeline: v0 = key mask word of block j, v1 of block j + 1 (load in
      // flight), k2 = key tile of block j + 2 if it is partial.
      uint32_t v0 = ~0u, v1 = ~0u;
      int k2 = 0;
      if (p.dense) {
        v0 = dense_word(0);
        v1 = dense_word(1);
      } else {
        if (pc > 0) v0 = tile_word(part_kv(0));
        if (pc > 1) v1 = tile_word(part_kv(1));
        if (pc > 2) k2 = part_kv(2);
      }
      for (int j = 0; j < len; ++j) {
        const uint32_t kmask = v0;
        v0 = v1;
        if (p.dense) {
          v1 = dense_word(j + 2);
        } else {
          v1 = j + 2 < pc ? tile_word(k2) : ~0u;
          if (j + 3 < pc) k2 = part_kv(j + 3);
        }
        const int blk = st.blk;
        st.j += 1;
        st.blk += 1;
        const uint32_t sb = static_cast<uint32_t>(blk) % kSBufs;
        const uint32_t spar = (static_cast<uint32_t>(blk) / kSBufs) & 1;
        const int xb = blk & 1;
        if (!wait_all(&bars[kSFull + sb], spar, abort, p.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t t_s = tmem + sb * 128 + kq * 32 + lane_base;
        uint32_t r[32];
        tmem_ld32(t_s, r);
        tmem_wait_ld();
        float* sc = reinterpret_cast<float*>(r);
        if (kmask != ~0u) {
#pragma unroll
          for (int c = 0; c < 32; ++c)
            if (!((kmask >> c) & 1u)) sc[c] = -INFINITY;
        }
        const float pm = row_max32(sc);
        float* xm = xmax + xb * 512 + row;
        xm[kq * 128] = pm;
        if constexpr (kHeat) {
          // The previous block's partial sum travels with this block's max.
          if (p.heat_sum && j > 0) xbs[(xb ^ 1) * 512 + kq * 128 + row] =
              bsum_prev;
        }
        row_sync(1 + quarter);
        const float raw_max = max3(fmaxf(xm[0], xm[128]), xm[256], xm[384]);
        const float mb = raw_max * p.scale_log2;
        if constexpr (kHeat) {
          if (kq == 0) {
            if (!p.heat_sum) {
              // The reference rounds every score to bf16 before its max;
              // rounding is monotonic, so rounding the max is the same.
              hs[j * kTile + row] = __bfloat162float(__float2bfloat16_rn(
                  raw_max));
            } else if (j > 0) {
              const float* xs = xbs + (xb ^ 1) * 512 + row;
              hs[(j - 1) * kTile + row] =
                  mref_prev +
                  lg2_approx((xs[0] + xs[128]) + (xs[256] + xs[384]));
            }
          }
        }
        bool rescale = false;
        float alpha = 1.0f;
        if (j == 0) {
          m_ref = mb;
        } else {
          // The four warps of a row see the same maxima: same decision.
          const bool grow = mb > m_ref + 8.0f;
          rescale = __any_sync(0xffffffffu, grow);
          if (rescale) {
            const float m_new = grow ? mb : m_ref;
            alpha = ex2_approx(m_ref - m_new);
            m_ref = m_new;
          }
        }
        const float2 sum = p32(r, sc, make_float2(p.scale_log2, p.scale_log2),
                               make_float2(-m_ref, -m_ref));
        if (rescale) {
          // O holds PV of the previous block once that PV has finished.
          const uint32_t pb = static_cast<uint32_t>(blk - 1);
          if (!wait_all(&bars[kPVDone + pb % kSBufs], (pb / kSBufs) & 1,
                        abort, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          rescale_o32(t_o, alpha);
          l *= alpha;
        }
        tmem_st16(t_s, r);  // P over the first 16 of this warp's columns
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[(kq < 2 ? kPFull0 : kPFull1) + sb]);
        l += sum.x + sum.y;
        if constexpr (kHeat) {
          bsum_prev = sum.x + sum.y;
          mref_prev = m_ref;
        }
      }
      if (!ok) break;
      // ---------------- epilogue of the item ----------------
      float l_row = 0.f;
      if (len > 0) {
        xsum[kq * 128 + row] = l;
        const int last_par = (st.blk - 1) & 1;
        if constexpr (kHeat) {
          if (p.heat_sum) xbs[last_par * 512 + kq * 128 + row] = bsum_prev;
        }
        row_sync(1 + quarter);
        l_row = (xsum[row] + xsum[128 + row]) + (xsum[256 + row] + xsum[384 + row]);
        if constexpr (kHeat) {
          if (kq == 0) {
            if (p.heat_sum) {
              const float* xs = xbs + last_par * 512 + row;
              hs[(len - 1) * kTile + row] =
                  mref_prev +
                  lg2_approx((xs[0] + xs[128]) + (xs[256] + xs[384]));
            }
            // Padding query rows carry no heat.
            s_hl[row] = row < p.valid_count[qt]
                            ? m_ref + lg2_approx(l_row)
                            : INFINITY;
          }
        }
        if (!wait_all(&bars[kODone], ka & 1, abort, p.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      const int64_t q_row = slot_row;
      const bool write = out_off >= 0;
      const float inv_l = len > 0 ? 1.0f / l_row : 0.f;
      uint32_t o[32];
      if (len > 0) {
        tmem_ld32(t_o, o);  // warp-wide, unpredicated
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[kOFree]);  // O may be overwritten
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = 0u;
      }
      if (write) {
        uint4* d4 = reinterpret_cast<uint4*>(p.out + out_off + kq * 32);
#pragma unroll
        for (int i = 0; i < 4; ++i)
          d4[i] = make_uint4(
              pack_bf16(__uint_as_float(o[8 * i]) * inv_l,
                        __uint_as_float(o[8 * i + 1]) * inv_l),
              pack_bf16(__uint_as_float(o[8 * i + 2]) * inv_l,
                        __uint_as_float(o[8 * i + 3]) * inv_l),
              pack_bf16(__uint_as_float(o[8 * i + 4]) * inv_l,
                        __uint_as_float(o[8 * i + 5]) * inv_l),
              pack_bf16(__uint_as_float(o[8 * i + 6]) * inv_l,
                        __uint_as_float(o[8 * i + 7]) * inv_l));
      }
      if (kq == 0 && p.lse != nullptr && write) {
        const float lse =
            len > 0 ? (m_ref + lg2_approx(l_row)) * 0.69314718055994531f
                    : -INFINITY;
        p.lse[q_row * p.lse_stride_row + h * p.lse_stride_h] = lse;
      }
      if constexpr (kHeat) {
        if (len > 0) {
          // Every row's maxima or sums and log-sum-exp are stored: warp w
          // reduces blocks w, w + 16, ... over the 128 rows.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars[kHeatIn]);
          if (!wait_all(&bars[kHeatIn], heat_items & 1, abort, p.status)) {
            ok = false;
            break;
          }
          float* dst = p.heat + h * p.heat_sh + qt * p.heat_sq;
          reduce_heat(hs, s_hl, warp, kSoftmaxWarps, len, p.heat_sum != 0,
                      p.scale_log2, dst,
                      [&](int jj) { return st.kv_global(p, jj); }, lane);
          // The scratch and the LSE rows are free for the next item.
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars[kHeatOut]);
          if (!wait_all(&bars[kHeatOut], heat_items & 1, abort, p.status)) {
            ok = false;
            break;
          }
          ++heat_items;
        }
      }
      st.next_item(p, true);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Dense forward over query-tile pairs (dense mode, and the fused dense + heat
// pass, whose keep-all lists are the same for every query tile).
//
// Every query tile attends to the same key tiles here, so a CTA takes two
// query tiles of one head (a pair) and streams each key/value tile once for
// both: per key block, QK of tile A and of tile B read the one K tile, PV of
// each reads the one V tile. Tensor memory holds an S buffer and an O
// accumulator per tile (S_A 0-127, S_B 128-255, O_A 256-383, O_B 384-511);
// softmax group g (warps 4g .. 4g + 3) owns tile g, one query row per thread
// over all 128 keys, with the online softmax and lazy rescaling of the
// sparse kernel. Per key block the shared memory traffic is half the
// one-tile kernel's K/V copies plus the operand reads: 128 KB per tile
// block instead of 160 KB. Warps: 8 softmax, a TMA producer (Q_A and Q_B per
// item into the two Q buffers, K and V through 2-slot rings, V two blocks
// behind K), a QK issuer (TMEM owner) and a PV issuer. All roles walk the
// same items (head, pair) with a stride of the grid and the same blocks, so
// they agree on barrier phases. All waits are bounded.
namespace pair {

constexpr int kWarps = 11;
constexpr int kProducer = 8, kQk = 9, kPv = 10;
enum PairBar {
  kQFullP = 0,   // Q_A and Q_B landed (one barrier, 64 KB)
  kQEmptyP = 1,  // the item's last QKs finished reading Q_A and Q_B
  kKFullP = 2,   // [2]
  kKEmptyP = 4,  // [2] both QKs of the block finished
  kVFullP = 6,   // [2]
  kVEmptyP = 8,  // [2] both PVs of the block finished
  kSFullP = 10,  // [2] per tile
  kPFullP = 12,  // [2] per tile: P written (4 warps)
  kPVDoneP = 14, // [2] per tile
  kODoneP = 16,  // the item's last PVs finished
  kOFreeP = 17,  // the epilogue read O_A and O_B (8 warps)
  kDrainQkP = 18,
  kDrainPvP = 19,
  kPHalfP = 20,  // [2] per tile: P of keys 64-127 written (4 warps)
  kNumBarsP = 22
};

// Length and key tile j of item (h, query tile qa): every key tile in dense
// mode, else the query tile's lists (partial list then full list, each
// from its end).
struct PairKeys {
  int len, pc, fc;
  int64_t off;
  __device__ void load(const FwdParams& p, int h, int qa) {
    if (p.dense) {
      len = p.n_kv_tiles;
      pc = fc = 0;
      off = 0;
      return;
    }
    const int64_t row = static_cast<int64_t>(h) * p.n_q_tiles + qa;
    pc = p.part_cnt[row];
    fc = p.full_cnt[row];
    len = pc + fc;
    off = row * p.ld_idx;
  }
  __device__ int kv(const FwdParams& p, int j) const {
    if (p.dense) return j;
    return j < pc ? p.part_idx[off + (pc - 1 - j)]
                  : p.full_idx[off + (fc - 1 - (j - pc))];
  }
  // Valid keys of block j (a prefix of the tile).
  __device__ int valid(const FwdParams& p, int j) const {
    if (p.dense) {
      const int64_t rest = p.used - static_cast<int64_t>(j) * kTile;
      return rest < kTile ? static_cast<int>(rest) : kTile;
    }
    return j < pc ? p.valid_count[kv(p, j)] : kTile;
  }
};

}  // namespace pair

template <bool kHeat>
__global__ void __launch_bounds__(32 * pair::kWarps, 1)
    pair_fwd_kernel(const __grid_constant__ FwdMaps maps, FwdParams p) {
  using namespace pair;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* s_q = smem;                   // [2] x 32 KB: Q_A, Q_B
  uint8_t* s_k = smem + 2 * kTileBytes;  // [kRing] x 32 KB
  uint8_t* s_v = s_k + kRing * kTileBytes;
  int32_t* s_list =
      reinterpret_cast<int32_t*>(smem + (2 + 2 * kRing) * kTileBytes);
  float* s_hl = reinterpret_cast<float*>(s_list + kListCap);  // [2][128]
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_hl + kExchangeFloats);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBarsP);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tid = threadIdx.x;
  const int warp = tid / 32;
  const int lane = tid % 32;
  const int n_pairs = (p.n_q_tiles + 1) / 2;
  const int n_items = p.n_heads * n_pairs;

  if (tid == 0) {
    for (int b = 0; b < kNumBarsP; ++b) {
      uint32_t count = 1;
      if (b == kPFullP || b == kPFullP + 1 || b == kPHalfP ||
          b == kPHalfP + 1)
        count = 4;
      if (b == kOFreeP) count = 8;
      mbar_init(&bars[b], count);
    }
    *abort = 0;
    fence_barrier_init();
  }
  if (warp == kQk) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kProducer) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      prefetch_tensor_map(&maps.q[0]);
      prefetch_tensor_map(&maps.k[0]);
      prefetch_tensor_map(&maps.v[0]);
    }
    int nk = 0, nv = 0, ka = 0;
    int kv1 = 0, kv2 = 0, h1 = 0, h2 = 0;  // V lags K by two blocks
    bool run = true;
    auto slot_of = [&](int n, int empty_bar) -> int {
      const int slot = n % kRing;
      if (n >= kRing && !wait_all(&bars[empty_bar + slot],
                                  ((n / kRing) - 1) & 1, abort, p.status))
        return -1;
      return slot;
    };
    auto load_v = [&](int h, int kv) -> bool {
      const int slot = slot_of(nv, kVEmptyP);
      if (slot < 0) return false;
      if (lane == 0) {
        mbar_arrive_expect_tx(&bars[kVFullP + slot], kTileBytes);
        load_tile(s_v + slot * kTileBytes, maps.v, &bars[kVFullP + slot], p,
                  h, h, kv, false);
      }
      __syncwarp();
      ++nv;
      return true;
    };
    for (int it = blockIdx.x; run && it < n_items; it += gridDim.x) {
      const int h = it / n_pairs, qa = 2 * (it % n_pairs);
      PairKeys keys;
      keys.load(p, h, qa);
      if (keys.len == 0) continue;
      if (!p.dense && keys.len <= kListCap) {
        __syncwarp();
        for (int jj = lane; jj < keys.len; jj += 32) s_list[jj] = keys.kv(p, jj);
        __syncwarp();
      }
      if (ka >= 1) {
        // The previous item's last two V tiles first (its PVs need them),
        // then its last QKs must finish before Q_A and Q_B are replaced.
        if (nk - nv >= 2) run = load_v(h2, kv2);
        if (run && nk - nv >= 1) run = load_v(h1, kv1);
        if (!run) break;
        if (!wait_all(&bars[kQEmptyP], (ka - 1) & 1, abort, p.status)) {
          run = false;
          break;
        }
      }
      if (lane == 0) {
        mbar_arrive_expect_tx(&bars[kQFullP], 2 * kTileBytes);
        load_tile(s_q, maps.q, &bars[kQFullP], p, h, h, qa, false);
        // A missing tile B (odd tile count) reads the map's zero fill.
        load_tile(s_q + kTileBytes, maps.q, &bars[kQFullP], p, h, h, qa + 1,
                  false);
      }
      __syncwarp();
      for (int j = 0; j < keys.len; ++j) {
        const int kv = p.dense ? j
                               : (keys.len <= kListCap ? s_list[j]
                                                       : keys.kv(p, j));
        const int slot = slot_of(nk, kKEmptyP);
        if (slot < 0) {
          run = false;
          break;
        }
        if (lane == 0) {
          mbar_arrive_expect_tx(&bars[kKFullP + slot], kTileBytes);
          load_tile(s_k + slot * kTileBytes, maps.k, &bars[kKFullP + slot],
                    p, h, h, kv, false);
        }
        __syncwarp();
        ++nk;
        if (nk - nv > 2 && !load_v(h2, kv2)) {
          run = false;
          break;
        }
        kv2 = kv1;
        h2 = h1;
        kv1 = kv;
        h1 = h;
      }
      ++ka;
    }
    if (run) {
      if (nk - nv >= 2) run = load_v(h2, kv2);
      if (run && nk - nv >= 1) run = load_v(h1, kv1);
    }
    if (lane == 0 && *abort) {
      // Let the copies in flight land before the CTA retires.
      volatile int never = 0;
      if (ka >= 1) mbar_wait(&bars[kQFullP], (ka - 1) & 1, &never, nullptr);
      for (int k = nk - kRing; k < nk; ++k)
        if (k >= 0)
          mbar_wait(&bars[kKFullP + k % kRing], (k / kRing) & 1, &never,
                    nullptr);
      for (int k = nv - kRing; k < nv; ++k)
        if (k >= 0)
          mbar_wait(&bars[kVFullP + k % kRing], (k / kRing) & 1, &never,
                    nullptr);
    }
  } else if (warp == kQk) {
    // ---------------- QK issuer ----------------
    constexpr uint32_t idesc_qk = idesc_bf16(128, 128, false, false);
    const uint32_t q_lo = sw128_desc_lo(smem_u32(s_q), 16);
    const uint32_t k_lo = sw128_desc_lo(smem_u32(s_k), 16);
    constexpr uint32_t kTileUnits = kTileBytes >> 4;
    uint32_t b = 0;
    int ka = 0;
    bool ok = true;
    for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x) {
      PairKeys keys;
      keys.load(p, it / n_pairs, 2 * (it % n_pairs));
      if (keys.len == 0) continue;
      for (int j = 0; j < keys.len; ++j, ++b) {
        const int slot = b % kRing;
        if (!wait_all(&bars[kKFullP + slot], (b / kRing) & 1, abort,
                      p.status) ||
            (j == 0 && !wait_all(&bars[kQFullP], ka & 1, abort, p.status))) {
          ok = false;
          break;
        }
        for (int g = 0; g < 2; ++g) {
          // S_g held P_g of the previous block until its PV finished.
          if (b >= 1 && !wait_all(&bars[kPVDoneP + g], (b - 1) & 1, abort,
                                  p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = q_lo + g * kTileUnits;
          const uint32_t bk = k_lo + slot * kTileUnits;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t off = (kk >> 2) * (kHalfBytes >> 4) + (kk & 3) * 2;
            umma_ss_warp(tmem + g * 128, a + off, bk + off, idesc_qk,
                         kk > 0 ? 1u : 0u);
          }
          umma_commit_warp(&bars[kSFullP + g]);
        }
        if (!ok) break;
        umma_commit_warp(&bars[kKEmptyP + slot]);
        if (j == keys.len - 1) umma_commit_warp(&bars[kQEmptyP]);
      }
      ++ka;
    }
    if (*abort) {
      volatile int never = 0;
      umma_commit_warp(&bars[kDrainQkP]);
      mbar_wait(&bars[kDrainQkP], 0, &never, nullptr);
    }
  } else if (warp == kPv) {
    // ---------------- PV issuer ----------------
    constexpr uint32_t idesc_pv = idesc_bf16(128, 128, false, true);
    const uint32_t v_lo = sw128_desc_lo(smem_u32(s_v), kHalfBytes);
    constexpr uint32_t kTileUnits = kTileBytes >> 4;
    uint32_t b = 0;
    int ka = 0;
    bool ok = true;
    for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x) {
      PairKeys keys;
      keys.load(p, it / n_pairs, 2 * (it % n_pairs));
      if (keys.len == 0) continue;
      for (int j = 0; j < keys.len; ++j, ++b) {
        const int slot = b % kRing;
        if (!wait_all(&bars[kVFullP + slot], (b / kRing) & 1, abort,
                      p.status) ||
            (j == 0 && ka >= 1 &&
             !wait_all(&bars[kOFreeP], (ka - 1) & 1, abort, p.status))) {
          ok = false;
          break;
        }
        const uint32_t bv = v_lo + slot * kTileUnits;
        for (int g = 0; g < 2; ++g) {
          // P of key step kk (16 keys) is in columns 8 kk of S_g; the
          // keys 0-63 half is written first.
          if (!wait_all(&bars[kPFullP + g], b & 1, abort, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_ts_warp(tmem + 256 + g * 128, tmem + g * 128 + kk * 8,
                         bv + kk * 128, idesc_pv,
                         (kk > 0 || j > 0) ? 1u : 0u);
          if (!wait_all(&bars[kPHalfP + g], b & 1, abort, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int kk = 4; kk < 8; ++kk)
            umma_ts_warp(tmem + 256 + g * 128, tmem + g * 128 + kk * 8,
                         bv + kk * 128, idesc_pv, 1u);
          umma_commit_warp(&bars[kPVDoneP + g]);
        }
        if (!ok) break;
        umma_commit_warp(&bars[kVEmptyP + slot]);
        if (j == keys.len - 1) umma_commit_warp(&bars[kODoneP]);
      }
      ++ka;
    }
    if (*abort) {
      volatile int never = 0;
      umma_commit_warp(&bars[kDrainPvP]);
      mbar_wait(&bars[kDrainPvP], 0, &never, nullptr);
    }
  } else {
    // ---------------- softmax + epilogue (warps 0-7) ----------------
    const int grp = warp / 4;  // tile of the pair
    const int quarter = warp % 4;
    const int row = quarter * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t t_s = tmem + grp * 128 + lane_base;
    const uint32_t t_o = tmem + 256 + grp * 128 + lane_base;
    const float2 scale2 = make_float2(p.scale_log2, p.scale_log2);
    float* hs = nullptr;  // this CTA's heat scratch for this tile
    if constexpr (kHeat)
      hs = p.heat_scratch +
           (static_cast<int64_t>(blockIdx.x) * 2 + grp) * p.n_kv_tiles *
               kTile;
    uint32_t b = 0;
    int ka = 0;
    bool ok = true;
    for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x) {
      const int h = it / n_pairs;
      const int qa = 2 * (it % n_pairs);
      const int qt = qa + grp;
      PairKeys keys;
      keys.load(p, h, qa);
      const int len = keys.len;
      float m_ref = -INFINITY, l = 0.f;
      for (int j = 0; j < len; ++j, ++b) {
        const int valid = keys.valid(p, j);
        if (!wait_all(&bars[kSFullP + grp], b & 1, abort, p.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t x[4][32];
#pragma unroll
        for (int q32 = 0; q32 < 4; ++q32) tmem_ld32(t_s + q32 * 32, x[q32]);
        tmem_wait_ld();
        float mx = -INFINITY;
#pragma unroll
        for (int q32 = 0; q32 < 4; ++q32) {
          if (valid < kTile) {
            const int n = valid - q32 * 32;
            const uint32_t word =
                n >= 32 ? ~0u : (n <= 0 ? 0u : (1u << n) - 1u);
            float* f = reinterpret_cast<float*>(x[q32]);
#pragma unroll
            for (int c = 0; c < 32; ++c)
              if (!((word >> c) & 1u)) f[c] = -INFINITY;
          }
          mx = fmaxf(mx, row_max32(reinterpret_cast<float*>(x[q32])));
        }
        const float mb = mx * p.scale_log2;
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
        if (rescale) {
          // O_g holds the previous blocks once the PV of blk - 1 finished;
          // it is rescaled before this block's P is released.
          if (!wait_all(&bars[kPVDoneP + grp], (b - 1) & 1, abort,
                        p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll 1
          for (int q16 = 0; q16 < 8; ++q16)
            rescale_o16(t_o + q16 * 16, alpha);
          l *= alpha;
        }
        // P in two halves (keys 0-63, then 64-127), each released as soon
        // as it is stored, so the first PVs start before the second half's
        // exponentials.
        const float2 negm2 = make_float2(-m_ref, -m_ref);
        float2 sums[4];
#pragma unroll
        for (int half = 0; half < 2; ++half) {
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            const int q32 = half * 2 + q;
            sums[q32] = p32(x[q32], reinterpret_cast<float*>(x[q32]), scale2,
                            negm2);
            tmem_st16(t_s + q32 * 16, x[q32]);
          }
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0)
            mbar_arrive(&bars[(half == 0 ? kPFullP : kPHalfP) + grp]);
        }
        const float bsum = ((sums[0].x + sums[0].y) + (sums[1].x + sums[1].y)) +
                           ((sums[2].x + sums[2].y) + (sums[3].x + sums[3].y));
        if constexpr (kHeat) {
          // Max mode: the raw score maximum rounded to bf16 (the reference
          // rounds every score; rounding is monotonic). Sum mode: log2 of
          // the block's exponential sum against the row's reference.
          hs[j * kTile + row] =
              p.heat_sum ? m_ref + lg2_approx(bsum)
                         : __bfloat162float(__float2bfloat16_rn(mx));
        }
        l += bsum;
      }
      if (!ok) break;
      // ---------------- epilogue of the tile ----------------
      const int64_t slot_row = static_cast<int64_t>(qt) * kTile + row;
      const bool real_tile = qt < p.n_q_tiles;
      const bool write = real_tile && (!p.dense || slot_row < p.used);
      const float inv_l = len > 0 ? 1.0f / l : 0.f;
      if (len > 0) {
        if (!wait_all(&bars[kODoneP], ka & 1, abort, p.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        if (len > 0) {
          tmem_ld32(t_o + c * 32, o);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0u;
        }
        if (write) {
          uint4* d4 = reinterpret_cast<uint4*>(
              p.out + slot_row * p.out_stride_n + h * p.out_stride_h +
              c * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            d4[i] = make_uint4(
                pack_bf16(__uint_as_float(o[8 * i]) * inv_l,
                          __uint_as_float(o[8 * i + 1]) * inv_l),
                pack_bf16(__uint_as_float(o[8 * i + 2]) * inv_l,
                          __uint_as_float(o[8 * i + 3]) * inv_l),
                pack_bf16(__uint_as_float(o[8 * i + 4]) * inv_l,
                          __uint_as_float(o[8 * i + 5]) * inv_l),
                pack_bf16(__uint_as_float(o[8 * i + 6]) * inv_l,
                          __uint_as_float(o[8 * i + 7]) * inv_l));
        }
      }
      if (len > 0) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[kOFreeP]);
      }
      const float lse2 = len > 0 ? m_ref + lg2_approx(l) : -INFINITY;
      if (write && p.lse != nullptr)
        p.lse[slot_row * p.lse_stride_row + h * p.lse_stride_h] =
            lse2 * 0.69314718055994531f;
      if constexpr (kHeat) {
        if (len > 0 && real_tile) {
          // Padding query rows carry no heat.
          s_hl[grp * kTile + row] =
              row < p.valid_count[qt] ? lse2 : INFINITY;
          row_sync(1 + grp);  // the tile's 4 warps: rows and scratch stored
          float* dst = p.heat + h * p.heat_sh + qt * p.heat_sq;
          reduce_heat(hs, s_hl + grp * kTile, quarter, 4, len,
                      p.heat_sum != 0, p.scale_log2, dst,
                      [&](int jj) { return keys.kv(p, jj); }, lane);
          row_sync(1 + grp);  // the scratch is free for the next item
        }
      }
      if (len > 0) ++ka;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kQk) {
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

int sm_count() {
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) !=
            cudaSuccess)
      sms = 0;
  }
  return sms;
}

// Which softmax the non-fused forward runs: the two-group one (default) or
// the one-group one (veda_set_fwd_groups).
int g_fwd_groups = 2;

template <bool kHeat, bool kDual>
int launch_fwd_variant(const FwdMaps& maps, const FwdParams& p,
                       cudaStream_t stream) {
  static bool configured = false;
  const int sms = sm_count();
  if (sms == 0) return set_error(VEDA_ERR_CUDA, "no CUDA device");
  if (!configured) {
    VEDA_CUDA(cudaFuncSetAttribute(bsa_fwd_kernel<kHeat, kDual>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   kSmemBytes));
    configured = true;
  }
  if (p.n_items == 0) return VEDA_OK;
  // SMs left free for kernels that overlap this one (collectives).
  const int cap = sms - sm_reserve() > 0 ? sms - sm_reserve() : 1;
  int grid = p.n_items < cap ? p.n_items : cap;
  if (p.item_order != nullptr) {
    // A work order is laid out for its own number of CTAs.
    grid = p.order_ctas;
    if (grid > sms)
      return set_error(VEDA_ERR_INVALID, "the work order has more CTAs than "
                                         "the device has SMs");
  }
  bsa_fwd_kernel<kHeat, kDual>
      <<<grid, Roles<kDual>::kThreads, kSmemBytes, stream>>>(
      maps, p);
  return check_launch("bsa_fwd_kernel");
}

// The pair kernel: dense mode and the fused dense + heat pass.
template <bool kHeat>
int launch_pair(const FwdMaps& maps, const FwdParams& p,
                cudaStream_t stream) {
  static bool configured = false;
  const int sms = sm_count();
  if (sms == 0) return set_error(VEDA_ERR_CUDA, "no CUDA device");
  if (!configured) {
    VEDA_CUDA(cudaFuncSetAttribute(pair_fwd_kernel<kHeat>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   kSmemBytes));
    configured = true;
  }
  const int items = p.n_heads * ((p.n_q_tiles + 1) / 2);
  if (items == 0) return VEDA_OK;
  const int cap = sms - sm_reserve() > 0 ? sms - sm_reserve() : 1;
  const int grid = items < cap ? items : cap;
  pair_fwd_kernel<kHeat><<<grid, 32 * pair::kWarps, kSmemBytes, stream>>>(
      maps, p);
  return check_launch("pair_fwd_kernel");
}

template <bool kHeat>
int launch_fwd(const FwdMaps& maps, const FwdParams& p, cudaStream_t stream) {
  if constexpr (kHeat) {
    return g_fwd_groups == 2 ? launch_pair<true>(maps, p, stream)
                             : launch_fwd_variant<true, false>(maps, p,
                                                               stream);
  } else {
    if (g_fwd_groups == 2 && p.dense)
      return launch_pair<false>(maps, p, stream);
    return g_fwd_groups == 2 ? launch_fwd_variant<false, true>(maps, p, stream)
                             : launch_fwd_variant<false, false>(maps, p,
                                                                stream);
  }
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
  VEDA_REQUIRE(n_q_tiles * n_heads < (int64_t(1) << 30), "too many tiles");
  VEDA_REQUIRE(softmax_scale > 0.f, "softmax_scale must be positive");
  VEDA_REQUIRE(reinterpret_cast<uintptr_t>(out) % 16 == 0 &&
                   out_stride_n % 8 == 0 && out_stride_h % 8 == 0,
               "out must be 16-byte aligned with strides multiple of 8");
  FwdMaps maps{};
  CUtensorMap &mq = maps.q[0], &mk = maps.k[0], &mv = maps.v[0];
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
  p.n_items = static_cast<int>(n_q_tiles * n_heads);
  p.n_slots = p.n_items;
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
  return launch_fwd<false>(maps, p, as_stream(stream));
}

extern "C" int64_t veda_bsa_fwd_heat_workspace(int64_t n_kv_tiles) {
  // Two [n_kv_tiles][128] scratches per SM: the pair kernel's two tiles.
  return 2 * static_cast<int64_t>(sm_count()) * n_kv_tiles * kTile *
         static_cast<int64_t>(sizeof(float));
}

extern "C" int veda_bsa_fwd_heat(
    const void* q, int64_t q_stride_n, int64_t q_stride_h, const void* k,
    int64_t k_stride_n, int64_t k_stride_h, const void* v, int64_t v_stride_n,
    int64_t v_stride_h, int32_t n_heads, int64_t n_tiles,
    const int32_t* valid_count, const int32_t* part_cnt,
    const int32_t* part_idx, const int32_t* full_cnt, const int32_t* full_idx,
    int64_t ld_idx, void* out, int64_t out_stride_n, int64_t out_stride_h,
    float* lse, int32_t reduce_sum, float* heat, float softmax_scale,
    void* workspace, int64_t workspace_bytes, void* stream) {
  int rc = require_sm100("veda_bsa_fwd_heat");
  if (rc != VEDA_OK) return rc;
  VEDA_REQUIRE(q && k && v && out && valid_count && part_cnt && part_idx &&
                   full_cnt && full_idx && heat,
               "q, k, v, out, valid_count, the four lists and heat are "
               "required");
  VEDA_REQUIRE(n_heads >= 1 && n_tiles >= 1, "bad shape");
  VEDA_REQUIRE(ld_idx >= n_tiles, "ld_idx must be >= n_tiles");
  VEDA_REQUIRE(n_tiles * n_heads < (int64_t(1) << 30), "too many tiles");
  VEDA_REQUIRE(softmax_scale > 0.f, "softmax_scale must be positive");
  VEDA_REQUIRE(reinterpret_cast<uintptr_t>(out) % 16 == 0 &&
                   out_stride_n % 8 == 0 && out_stride_h % 8 == 0,
               "out must be 16-byte aligned with strides multiple of 8");
  VEDA_REQUIRE(workspace != nullptr &&
                   workspace_bytes >= veda_bsa_fwd_heat_workspace(n_tiles),
               "workspace too small (veda_bsa_fwd_heat_workspace)");
  FwdMaps maps{};
  CUtensorMap &mq = maps.q[0], &mk = maps.k[0], &mv = maps.v[0];
  rc = make_tile_map(&mq, q, n_tiles * kTile, n_heads, q_stride_n,
                     q_stride_h, "q");
  if (rc == VEDA_OK)
    rc = make_tile_map(&mk, k, n_tiles * kTile, n_heads, k_stride_n,
                       k_stride_h, "k");
  if (rc == VEDA_OK)
    rc = make_tile_map(&mv, v, n_tiles * kTile, n_heads, v_stride_n,
                       v_stride_h, "v");
  if (rc != VEDA_OK) return rc;
  FwdParams p{};
  p.n_heads = n_heads;
  p.n_q_tiles = static_cast<int>(n_tiles);
  p.n_kv_tiles = static_cast<int>(n_tiles);
  p.n_items = static_cast<int>(n_tiles * n_heads);
  p.n_slots = p.n_items;
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
  p.lse_stride_h = n_tiles * kTile;
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  p.heat = heat;
  p.heat_sh = n_tiles * n_tiles;
  p.heat_sq = n_tiles;
  p.heat_scratch = static_cast<float*>(workspace);
  p.heat_sum = reduce_sum != 0;
  p.status = device_status_ptr();
  return launch_fwd<true>(maps, p, as_stream(stream));
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
  VEDA_REQUIRE(tiles * n_heads < (int64_t(1) << 30), "too many tiles");
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
  FwdMaps maps{};
  CUtensorMap &mq = maps.q[0], &mk = maps.k[0], &mv = maps.v[0];
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
  p.n_items = static_cast<int>(tiles * n_heads);
  p.n_slots = p.n_items;
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
  return launch_fwd<false>(maps, p, as_stream(stream));
}

extern "C" int veda_bsa_fwd_packed(
    const void* q, const void* k, const void* v, int64_t stride_s,
    int64_t stride_h, int64_t seq_len, int32_t total_heads,
    int32_t kv_tile_order, int64_t kv_stride_n, int64_t kv_stride_h,
    const void* q_glob, const void* k_glob, const void* v_glob,
    int64_t glob_stride_n, int64_t glob_stride_h, const veda_span_t* spans,
    int32_t n_spans, int64_t n_tiles, int64_t n_video, const int64_t* heads,
    int32_t n_heads, const int64_t* box_perm, const uint32_t* key_mask,
    const int32_t* valid_count, const int32_t* part_cnt,
    const int32_t* part_idx, const int32_t* full_cnt,
    const int32_t* full_idx, int64_t ld_idx, void* out, int64_t out_stride_s,
    int64_t out_stride_h, float softmax_scale, const int32_t* item_order,
    int32_t order_ctas, int64_t order_slots, void* stream) {
  int rc = require_sm100("veda_bsa_fwd_packed");
  if (rc != VEDA_OK) return rc;
  VEDA_REQUIRE(q && k && v && out && heads && box_perm && part_cnt &&
                   part_idx && full_cnt && full_idx && spans,
               "q, k, v, out, heads, box_perm, spans and the four lists are "
               "required");
  VEDA_REQUIRE(kv_tile_order ? valid_count != nullptr : key_mask != nullptr,
               "tile-ordered k/v need valid_count; packed k/v need key_mask");
  VEDA_REQUIRE(n_spans >= 1 && n_spans <= kMaxPackedSpans,
               "the packed forward reads at most 2 tiled spans in place");
  VEDA_REQUIRE(n_heads >= 1 && total_heads >= n_heads && seq_len >= 1,
               "bad shape");
  VEDA_REQUIRE(n_video >= 1 && n_tiles >= n_video, "bad tile counts");
  VEDA_REQUIRE(n_tiles == n_video ||
                   (q_glob && (kv_tile_order || (k_glob && v_glob))),
               "the layout has global tiles: their gathered copies are "
               "required");
  VEDA_REQUIRE(ld_idx >= n_tiles, "ld_idx must be >= n_tiles");
  VEDA_REQUIRE(n_tiles * n_heads < (int64_t(1) << 30), "too many tiles");
  VEDA_REQUIRE(softmax_scale > 0.f, "softmax_scale must be positive");
  VEDA_REQUIRE(reinterpret_cast<uintptr_t>(out) % 16 == 0 &&
                   out_stride_s % 8 == 0 && out_stride_h % 8 == 0,
               "out must be 16-byte aligned with strides multiple of 8");
  FwdMaps maps{};
  FwdParams p{};
  int64_t tiles = 0;
  for (int s = 0; s < n_spans; ++s) {
    const veda_span_t& sp = spans[s];
    int64_t vol = 1, n = 1;
    for (int a = 0; a < 3; ++a) {
      VEDA_REQUIRE(sp.grid[a] > 0 && sp.shape[a] > 0,
                   "span grid and tile shape must be positive");
      vol *= sp.shape[a];
      n *= (sp.grid[a] + sp.shape[a] - 1) / sp.shape[a];
      p.span_shape[s][a] = sp.shape[a];
    }
    VEDA_REQUIRE(vol == kTile, "tile shape does not hold 128 tokens");
    VEDA_REQUIRE(sp.start >= 0 && sp.start + static_cast<int64_t>(sp.grid[0]) *
                                                  sp.grid[1] * sp.grid[2] <=
                                              seq_len,
                 "span exceeds the sequence");
    p.span_begin[s] = static_cast<int>(tiles);
    p.span_nbt[s] = (sp.grid[0] + sp.shape[0] - 1) / sp.shape[0];
    p.span_nbw[s] = (sp.grid[2] + sp.shape[2] - 1) / sp.shape[2];
    const char* names[3] = {"q span", "k span", "v span"};
    const void* bases[3] = {q, k, v};
    CUtensorMap* dst[3] = {&maps.q[1 + s], &maps.k[1 + s], &maps.v[1 + s]};
    for (int t = 0; t < (kv_tile_order ? 1 : 3); ++t) {
      const void* base = static_cast<const __nv_bfloat16*>(bases[t]) +
                         sp.start * stride_s;
      rc = make_box_map(dst[t], base, sp.grid, sp.shape, total_heads,
                        stride_s, stride_h, names[t]);
      if (rc != VEDA_OK) return rc;
    }
    tiles += n;
  }
  VEDA_REQUIRE(tiles == n_video, "n_video does not match the spans");
  p.span_begin[n_spans] = static_cast<int>(tiles);
  const int64_t n_global = n_tiles - n_video;
  if (n_global > 0) {
    rc = make_tile_map(&maps.q[0], q_glob, n_global * kTile, n_heads,
                       glob_stride_n, glob_stride_h, "q_glob");
    if (rc == VEDA_OK && !kv_tile_order)
      rc = make_tile_map(&maps.k[0], k_glob, n_global * kTile, n_heads,
                         glob_stride_n, glob_stride_h, "k_glob");
    if (rc == VEDA_OK && !kv_tile_order)
      rc = make_tile_map(&maps.v[0], v_glob, n_global * kTile, n_heads,
                         glob_stride_n, glob_stride_h, "v_glob");
    if (rc != VEDA_OK) return rc;
  }
  if (kv_tile_order == 2) {
    VEDA_REQUIRE(reinterpret_cast<uintptr_t>(k) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(v) % 16 == 0,
                 "tile images must be 16-byte aligned");
    p.k_img = static_cast<const uint8_t*>(k);
    p.v_img = static_cast<const uint8_t*>(v);
  } else if (kv_tile_order) {
    rc = make_tile_map(&maps.k[0], k, n_tiles * kTile, n_heads, kv_stride_n,
                       kv_stride_h, "k");
    if (rc == VEDA_OK)
      rc = make_tile_map(&maps.v[0], v, n_tiles * kTile, n_heads,
                         kv_stride_n, kv_stride_h, "v");
    if (rc != VEDA_OK) return rc;
  }
  p.n_heads = n_heads;
  p.n_q_tiles = static_cast<int>(n_tiles);
  p.n_kv_tiles = static_cast<int>(n_tiles);
  p.n_items = static_cast<int>(n_tiles * n_heads);
  p.n_slots = p.n_items;
  p.valid_count = kv_tile_order ? valid_count : nullptr;
  p.part_cnt = part_cnt;
  p.part_idx = part_idx;
  p.full_cnt = full_cnt;
  p.full_idx = full_idx;
  p.ld_idx = ld_idx;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_stride_n = out_stride_s;
  p.out_stride_h = out_stride_h;
  p.lse = nullptr;
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  p.dense = 0;
  p.used = 0;
  if (item_order != nullptr) {
    VEDA_REQUIRE(order_ctas >= 1 && order_slots >= order_ctas &&
                     order_slots % order_ctas == 0 &&
                     order_slots < (int64_t(1) << 31),
                 "the work order must be [rounds, order_ctas] slots");
    p.item_order = item_order;
    p.order_ctas = order_ctas;
    p.n_slots = static_cast<int>(order_slots);
  }
  p.packed = 1;
  p.box_kv = kv_tile_order ? 0 : 1;
  p.total_heads = total_heads;
  p.n_video = static_cast<int>(n_video);
  p.n_spans = n_spans;
  p.head_ids = heads;
  p.box_perm = box_perm;
  p.key_mask = kv_tile_order ? nullptr : key_mask;
  p.status = device_status_ptr();
  return launch_fwd<false>(maps, p, as_stream(stream));
}

extern "C" int veda_set_fwd_groups(int32_t groups) {
  VEDA_REQUIRE(groups == 1 || groups == 2,
               "the forward's softmax runs in 1 or 2 groups");
  g_fwd_groups = groups;
  return VEDA_OK;
}
