// Shared host/device helpers of the Veda B200 library: error reporting,
// bounded mbarrier waits, TMA and tcgen05 (UMMA / TMEM) wrappers for sm_100a.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdint.h>

#include <string>

#include "veda_b200.h"

namespace veda {

// ---------------------------------------------------------------------------
// host-side error handling
// ---------------------------------------------------------------------------

int set_error(int code, const std::string& msg);
int check_cuda(cudaError_t err, const char* what);
int check_launch(const char* what);

#define VEDA_REQUIRE(cond, msg)                                   \
  do {                                                            \
    if (!(cond)) return ::veda::set_error(VEDA_ERR_INVALID, msg); \
  } while (0)

#define VEDA_CUDA(call)                                            \
  do {                                                             \
    int rc_ = ::veda::check_cuda((call), #call);                   \
    if (rc_ != VEDA_OK) return rc_;                                \
  } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Returns VEDA_OK when the current device is an sm_100 part.
int require_sm100(const char* op);

// Device status word written by kernels whose bounded waits expire.
unsigned int* device_status_ptr();

// SMs the persistent attention forward leaves free (veda_set_sm_reserve).
int sm_reserve();

// 3D bf16 tensor map over a [rows, heads, 128] tensor with a (64, 1, 128)
// box and 128-byte swizzle: coordinates are (d0 in {0, 64}, head, row0).
int make_tile_map(CUtensorMap* map, const void* base, int64_t rows,
                  int64_t heads, int64_t stride_row, int64_t stride_head,
                  const char* name);

// 5D bf16 tensor map over the (T, Hh, W) grid of a span of a packed
// [rows, heads, 128] tensor (base = the span's first row): dimensions
// (d, head, w, h, t), box (64, 1, sw, sh, st) with 128-byte swizzle, so a
// box lands in shared memory exactly like a (64, 1, 128) box of tile-ordered
// rows, its rows in the tile's (t, h, w) row-major order. Coordinates are
// (d0 in {0, 64}, head, w0, h0, t0); rows outside the grid read as zero.
int make_box_map(CUtensorMap* map, const void* base, const int grid[3],
                 const int shape[3], int64_t heads, int64_t stride_row,
                 int64_t stride_head, const char* name);

constexpr int kTile = 128;
constexpr int kHeadDim = 128;

// ---------------------------------------------------------------------------
// device helpers
// ---------------------------------------------------------------------------

constexpr unsigned long long kWaitTimeoutNs = 4000000000ull;  // 4 s

__device__ __forceinline__ uint64_t global_timer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{ .reg .b64 st; mbarrier.arrive.shared::cta.b64 st, [%0]; }" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar,
                                                      uint32_t bytes) {
  asm volatile(
      "{ .reg .b64 st; mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], "
      "%1; }" ::"r"(smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; "
      "selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Records the first error code of the launch in the device status word.
__device__ __forceinline__ void raise_status(unsigned int* status,
                                             unsigned int code) {
  if (status != nullptr) atomicCAS(status, 0u, code);
}

// Waits for the phase of `bar` with the given parity. Gives up when another
// role of the CTA already gave up (*abort != 0) or after `limit_ns`
// (kWaitTimeoutNs unless a caller asks for less), which it records in *abort
// and in the device status word. Returns true when the phase completed.
__device__ __forceinline__ bool mbar_wait(
    uint64_t* bar, uint32_t parity, volatile int* abort, unsigned int* status,
    unsigned long long limit_ns = kWaitTimeoutNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
    if (global_timer() - t0 > limit_ns) {
      *abort = 1;
      raise_status(status, VEDA_ERR_TIMEOUT);
      return false;
    }
  }
}

// TMA: 3D tiled bulk tensor load into shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map,
                                            uint64_t* bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::"
      "bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0),
      "r"(c1), "r"(c2)
      : "memory");
}

// TMA: 5D tiled bulk tensor load (a box of the packed tensor, see
// make_box_map), completing on `bar`.
__device__ __forceinline__ void tma_load_5d(void* dst, const CUtensorMap* map,
                                            uint64_t* bar, int c0, int c1,
                                            int c2, int c3, int c4) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.mbarrier::complete_tx::"
      "bytes [%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0),
      "r"(c1), "r"(c2), "r"(c3), "r"(c4)
      : "memory");
}

// TMA: contiguous bulk copy global -> shared (both addresses 16-byte aligned,
// bytes a multiple of 16), completing on `bar`.
__device__ __forceinline__ void bulk_load(void* dst, const void* src,
                                          uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void prefetch_tensor_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map))
               : "memory");
}

// --- tcgen05 (5th-generation tensor core, tensor memory) -----------------

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile(
      "tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
          smem_u32(dst_smem)),
      "r"(ncols)
      : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::
                   : "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(
                   taddr),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] . B[smem]^T-or-B, kind::f16 (bf16 in, fp32 accumulate).
__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t a_desc,
                                        uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0; "
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] . B[smem], kind::f16.
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem,
                                        uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0; "
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p; }" ::"r"(
          d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives on `bar` once every tcgen05 operation issued so far by this thread
// has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
      "[%0];" ::"r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 32 consecutive 32-bit columns of this thread's lane (warp w of a warpgroup
// reaches lanes 32w..32w+31; taddr carries the lane base in bits 31:16).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
      "%30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]),
        "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]),
        "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]),
        "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]),
        "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
      "%30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]),
      "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]),
      "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
      "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]),
      "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]),
      "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]),
      "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// The same descriptor split into 32-bit halves, so that issue loops add a
// per-step offset (in 16-byte units) to the low half with one instruction:
// the start address occupies the low 14 bits and never carries out of them
// inside shared memory. The high half (SBO 1024 B, version 1, SWIZZLE_128B)
// is the same for every operand here.
__device__ __forceinline__ uint32_t sw128_desc_lo(uint32_t smem_addr,
                                                  uint32_t lbo_bytes) {
  return ((smem_addr >> 4) & 0x3FFF) | (((lbo_bytes >> 4) & 0x3FFF) << 16);
}
constexpr uint32_t kSw128DescHi = (1024u >> 4) | (1u << 14) | (2u << 29);

// Warp-collective issue: every lane of the warp executes these (converged),
// and the lane that elect.sync picks issues the instruction. An issue loop
// written this way keeps the warp converged between MMA groups; a loop run
// by one lane inside `if (lane == 0)` pays ~100 cycles of tensor-core idle
// for every branch or barrier wait between groups (measured on B200).
//
// D[tmem] (+)= A[smem] . B[smem], descriptors given as low halves.
__device__ __forceinline__ void umma_ss_warp(uint32_t d_tmem, uint32_t a_lo,
                                             uint32_t b_lo, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p, e; .reg .b64 da, db; .reg .b32 rx; "
      "elect.sync rx|e, 0xFFFFFFFF; mov.b64 da, {%1, %5}; "
      "mov.b64 db, {%2, %5}; setp.ne.b32 p, %4, 0; "
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %3, p; }" ::"r"(
          d_tmem),
      "r"(a_lo), "r"(b_lo), "r"(idesc), "r"(accumulate), "r"(kSw128DescHi)
      : "memory");
}

// D[tmem] (+)= A[tmem] . B[smem], B descriptor given as its low half.
__device__ __forceinline__ void umma_ts_warp(uint32_t d_tmem, uint32_t a_tmem,
                                             uint32_t b_lo, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p, e; .reg .b64 db; .reg .b32 rx; "
      "elect.sync rx|e, 0xFFFFFFFF; mov.b64 db, {%2, %5}; "
      "setp.ne.b32 p, %4, 0; "
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], db, %3, p; }" ::"r"(
          d_tmem),
      "r"(a_tmem), "r"(b_lo), "r"(idesc), "r"(accumulate), "r"(kSw128DescHi)
      : "memory");
}

// tcgen05.commit from the elected lane: `bar` completes one arrival when
// every MMA this warp issued before has completed.
__device__ __forceinline__ void umma_commit_warp(uint64_t* bar) {
  asm volatile(
      "{ .reg .pred e; .reg .b32 rx; elect.sync rx|e, 0xFFFFFFFF; "
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster."
      "b64 [%0]; }" ::"r"(smem_u32(bar))
      : "memory");
}

// Shared-memory matrix descriptor (tcgen05 "SM100" format, version 1) of a
// 128-byte-swizzled operand. K-major: rows of 64 bf16, 8-row atoms 1024 B
// apart (SBO). MN-major: 64-element MN chunks `lbo` bytes apart, 8-row K
// groups 1024 B apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t smem_addr,
                                               uint32_t lbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= static_cast<uint64_t>((1024u >> 4) & 0x3FFF) << 32;
  d |= 1ull << 46;  // descriptor version for tcgen05
  d |= 2ull << 61;  // SWIZZLE_128B
  return d;
}

// Instruction descriptor of kind::f16 with bf16 A/B, fp32 D.
__host__ __device__ constexpr uint32_t idesc_bf16(int m, int n, bool a_mn,
                                                   bool b_mn) {
  return (1u << 4)                    // D format: f32
         | (1u << 7)                  // A format: bf16
         | (1u << 10)                 // B format: bf16
         | ((a_mn ? 1u : 0u) << 15)   // A major
         | ((b_mn ? 1u : 0u) << 16)   // B major
         | (static_cast<uint32_t>(n >> 3) << 17)
         | (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm volatile("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float lg2_approx(float x) {
  float y;
  asm volatile("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ bool elect_one_sync() {
  uint32_t pred = 0;
  asm volatile(
      "{ .reg .b32 rx; .reg .pred px; elect.sync rx|px, 0xFFFFFFFF; "
      "selp.b32 %0, 1, 0, px; }"
      : "=r"(pred));
  return pred != 0;
}

}  // namespace veda
