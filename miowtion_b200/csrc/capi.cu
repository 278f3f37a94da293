// Library state of the C ABI: thread-local error messages, the device status
// word, device checks, tensor-map encoding, and the UMMA layout probe.
#include <stdio.h>
#include <string.h>

#include <atomic>
#include <mutex>
#include <string>

#include "common.cuh"

namespace veda {

namespace {
thread_local int g_last_code = VEDA_OK;
thread_local std::string g_last_msg;
}  // namespace

int set_error(int code, const std::string& msg) {
  g_last_code = code;
  g_last_msg = msg;
  return code;
}

int check_cuda(cudaError_t err, const char* what) {
  if (err == cudaSuccess) return VEDA_OK;
  return set_error(VEDA_ERR_CUDA, std::string(what) + ": " +
                                      cudaGetErrorString(err));
}

int check_launch(const char* what) {
  return check_cuda(cudaGetLastError(), what);
}

// Status word kernels raise when a bounded wait expires; one per device
// context, zero-initialised at module load.
__device__ unsigned int g_device_status = 0;

unsigned int* device_status_ptr() {
  // cudaGetSymbolAddress is cheap after the first call, but is cached per
  // device to keep it off the launch path.
  static std::mutex mu;
  static unsigned int* cache[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_status) != cudaSuccess)
      return nullptr;
    cache[dev] = static_cast<unsigned int*>(p);
  }
  return cache[dev];
}

namespace {
std::atomic<int> g_sm_reserve{0};
}  // namespace

int sm_reserve() { return g_sm_reserve.load(std::memory_order_relaxed); }

int require_sm100(const char* op) {
  int dev = 0;
  VEDA_CUDA(cudaGetDevice(&dev));
  int major = 0, minor = 0;
  VEDA_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor,
                                   dev));
  VEDA_CUDA(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor,
                                   dev));
  if (major != 10 || minor != 0) {
    char buf[160];
    snprintf(buf, sizeof(buf),
             "%s needs sm_100a (B200); device %d is sm_%d%d, which has no "
             "tcgen05 tensor cores this library was built for",
             op, dev, major, minor);
    return set_error(VEDA_ERR_UNSUPPORTED, buf);
  }
  return VEDA_OK;
}

namespace {
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p,
                                cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}
}  // namespace

int make_tile_map(CUtensorMap* map, const void* base, int64_t rows,
                  int64_t heads, int64_t stride_row, int64_t stride_head,
                  const char* name) {
  auto fn = encode_fn();
  if (fn == nullptr)
    return set_error(VEDA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const auto addr = reinterpret_cast<uintptr_t>(base);
  if (addr % 16 != 0 || (stride_row * 2) % 16 != 0 ||
      (heads > 1 && (stride_head * 2) % 16 != 0))
    return set_error(VEDA_ERR_INVALID,
                     std::string(name) +
                         ": base address and row/head strides must be "
                         "16-byte aligned for TMA");
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(kHeadDim),
                        static_cast<cuuint64_t>(heads),
                        static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[2] = {
      static_cast<cuuint64_t>((heads > 1 ? stride_head : kHeadDim) * 2),
      static_cast<cuuint64_t>(stride_row * 2)};
  cuuint32_t box[3] = {64, 1, static_cast<cuuint32_t>(kTile)};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                  const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[200];
    snprintf(buf, sizeof(buf),
             "%s: cuTensorMapEncodeTiled failed (%d) for rows=%lld "
             "heads=%lld strides=(%lld,%lld)",
             name, static_cast<int>(r), static_cast<long long>(rows),
             static_cast<long long>(heads), static_cast<long long>(stride_row),
             static_cast<long long>(stride_head));
    return set_error(VEDA_ERR_INVALID, buf);
  }
  return VEDA_OK;
}

int make_box_map(CUtensorMap* map, const void* base, const int grid[3],
                 const int shape[3], int64_t heads, int64_t stride_row,
                 int64_t stride_head, const char* name) {
  auto fn = encode_fn();
  if (fn == nullptr)
    return set_error(VEDA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const auto addr = reinterpret_cast<uintptr_t>(base);
  if (addr % 16 != 0 || (stride_row * 2) % 16 != 0 ||
      (stride_head * 2) % 16 != 0)
    return set_error(VEDA_ERR_INVALID,
                     std::string(name) +
                         ": base address and row/head strides must be "
                         "16-byte aligned for TMA");
  const int T = grid[0], Hh = grid[1], W = grid[2];
  cuuint64_t dims[5] = {static_cast<cuuint64_t>(kHeadDim),
                        static_cast<cuuint64_t>(heads),
                        static_cast<cuuint64_t>(W),
                        static_cast<cuuint64_t>(Hh),
                        static_cast<cuuint64_t>(T)};
  cuuint64_t strides[4] = {
      static_cast<cuuint64_t>(stride_head * 2),
      static_cast<cuuint64_t>(stride_row * 2),
      static_cast<cuuint64_t>(stride_row * 2) * static_cast<cuuint64_t>(W),
      static_cast<cuuint64_t>(stride_row * 2) * static_cast<cuuint64_t>(W) *
          static_cast<cuuint64_t>(Hh)};
  cuuint32_t box[5] = {64, 1, static_cast<cuuint32_t>(shape[2]),
                       static_cast<cuuint32_t>(shape[1]),
                       static_cast<cuuint32_t>(shape[0])};
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5,
                  const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[200];
    snprintf(buf, sizeof(buf),
             "%s: cuTensorMapEncodeTiled failed (%d) for grid=(%d,%d,%d) "
             "box=(%d,%d,%d) heads=%lld",
             name, static_cast<int>(r), T, Hh, W, shape[0], shape[1],
             shape[2], static_cast<long long>(heads));
    return set_error(VEDA_ERR_INVALID, buf);
  }
  return VEDA_OK;
}

// ---------------------------------------------------------------------------
// UMMA layout probe: one 128x128x128 MMA, operands as the attention kernels
// stage them (TMA with 128-byte swizzle; P through tensor memory).
// ---------------------------------------------------------------------------

__global__ void __launch_bounds__(128, 1)
    probe_umma_kernel(const __grid_constant__ CUtensorMap map_a,
                      const __grid_constant__ CUtensorMap map_b,
                      const __nv_bfloat16* a, float* d, int mode,
                      unsigned int* status) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sa = smem;            // 32 KB
  uint8_t* sb = smem + 32768;    // 32 KB
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 65536);
  uint32_t* tbase_smem = reinterpret_cast<uint32_t*>(smem + 65536 + 64);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + 65536 + 128);
  const int tid = threadIdx.x;
  const int warp = tid / 32;

  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    *abort = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (warp == 0) {
    tmem_alloc(tbase_smem, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tbase_smem;
  const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;

  if (tid == 0) {
    if (mode == 0) {
      mbar_arrive_expect_tx(&bars[0], 65536);
      tma_load_3d(sa, &map_a, &bars[0], 0, 0, 0);
      tma_load_3d(sa + 16384, &map_a, &bars[0], 64, 0, 0);
    } else {
      mbar_arrive_expect_tx(&bars[0], 32768);
    }
    tma_load_3d(sb, &map_b, &bars[0], 0, 0, 0);
    tma_load_3d(sb + 16384, &map_b, &bars[0], 64, 0, 0);
  }
  if (mode == 1) {
    // Row `tid` of a, packed two bf16 per 32-bit column, into columns
    // [256, 320) of this thread's lane.
    const uint32_t* row = reinterpret_cast<const uint32_t*>(a + tid * 128);
    uint32_t buf[32];
    for (int half = 0; half < 2; ++half) {
      for (int i = 0; i < 32; ++i) buf[i] = row[half * 32 + i];
      tmem_st32(tbase + lane_base + 256 + half * 32, buf);
    }
    tmem_wait_st();
  }
  tc_fence_before();
  __syncthreads();
  if (tid == 0) {
    tc_fence_after();
    if (mbar_wait(&bars[0], 0, abort, status)) {
      const uint32_t sa_addr = smem_u32(sa);
      const uint32_t sb_addr = smem_u32(sb);
      for (int kk = 0; kk < 8; ++kk) {
        if (mode == 0) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          umma_ss(tbase, sw128_desc(sa_addr + off, 16),
                  sw128_desc(sb_addr + off, 16),
                  idesc_bf16(128, 128, false, false), kk > 0);
        } else {
          umma_ts(tbase, tbase + 256 + kk * 8,
                  sw128_desc(sb_addr + kk * 2048, 16384),
                  idesc_bf16(128, 128, false, true), kk > 0);
        }
      }
    }
    umma_commit(&bars[1]);
  }
  __syncwarp();
  if (mbar_wait(&bars[1], 0, abort, status)) {
    tc_fence_after();
    uint32_t r[32];
    for (int c = 0; c < 4; ++c) {
      tmem_ld32(tbase + lane_base + c * 32, r);
      tmem_wait_ld();
      for (int i = 0; i < 32; ++i)
        d[tid * 128 + c * 32 + i] = __uint_as_float(r[i]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

// Two warps wait on mbarriers that nothing completes: warp 0 with the given
// limit, warp 1 with the library's, leaving on warp 0's abort flag.
__global__ void __launch_bounds__(64, 1)
    expire_wait_kernel(unsigned long long limit_ns, int32_t* completed,
                       unsigned int* status) {
  __shared__ uint64_t bars[2];
  __shared__ int abort_flag;
  const int warp = threadIdx.x / 32;
  if (threadIdx.x == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  volatile int* abort = &abort_flag;
  const bool ok = warp == 0
                      ? mbar_wait(&bars[0], 0, abort, status, limit_ns)
                      : mbar_wait(&bars[1], 0, abort, status);
  if (threadIdx.x % 32 == 0) completed[warp] = ok ? 1 : 0;
}

}  // namespace veda

using namespace veda;

extern "C" int veda_last_error(char* buf, size_t size) {
  if (buf != nullptr && size > 0) {
    strncpy(buf, g_last_msg.c_str(), size - 1);
    buf[size - 1] = '\0';
  }
  return g_last_code;
}

extern "C" int veda_device_status(int32_t* status, int32_t reset) {
  unsigned int* p = device_status_ptr();
  if (p == nullptr) return set_error(VEDA_ERR_CUDA, "no device status word");
  VEDA_CUDA(cudaDeviceSynchronize());
  unsigned int v = 0;
  VEDA_CUDA(cudaMemcpy(&v, p, sizeof(v), cudaMemcpyDeviceToHost));
  if (status != nullptr) *status = static_cast<int32_t>(v);
  if (reset) VEDA_CUDA(cudaMemset(p, 0, sizeof(unsigned int)));
  return VEDA_OK;
}

extern "C" int veda_set_sm_reserve(int32_t n) {
  VEDA_REQUIRE(n >= 0 && n <= 128, "the SM reserve must lie in [0, 128]");
  g_sm_reserve.store(n, std::memory_order_relaxed);
  return VEDA_OK;
}

extern "C" int veda_supported_device(void) {
  return require_sm100("veda") == VEDA_OK ? 1 : 0;
}

extern "C" int veda_probe_umma(const void* a, const void* b, float* d,
                               int32_t mode, void* stream) {
  int rc = require_sm100("veda_probe_umma");
  if (rc != VEDA_OK) return rc;
  VEDA_REQUIRE(mode == 0 || mode == 1, "mode must be 0 or 1");
  CUtensorMap ma, mb;
  rc = make_tile_map(&ma, a, 128, 1, 128, 128, "probe a");
  if (rc != VEDA_OK) return rc;
  rc = make_tile_map(&mb, b, 128, 1, 128, 128, "probe b");
  if (rc != VEDA_OK) return rc;
  const int smem = 65536 + 256 + 1024;
  VEDA_CUDA(cudaFuncSetAttribute(probe_umma_kernel,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 smem));
  probe_umma_kernel<<<1, 128, smem, as_stream(stream)>>>(
      ma, mb, static_cast<const __nv_bfloat16*>(a), d, mode,
      device_status_ptr());
  return check_launch("probe_umma_kernel");
}

extern "C" int veda_expire_wait(int64_t limit_ns, int32_t* completed,
                                void* stream) {
  int rc = require_sm100("veda_expire_wait");
  if (rc != VEDA_OK) return rc;
  VEDA_REQUIRE(limit_ns >= 1000000 &&
                   limit_ns <= static_cast<int64_t>(kWaitTimeoutNs),
               "limit_ns must lie in [1 ms, 4 s]");
  VEDA_REQUIRE(completed != nullptr, "completed[2] is required");
  unsigned int* status = device_status_ptr();
  if (status == nullptr) return set_error(VEDA_ERR_CUDA, "no device status word");
  expire_wait_kernel<<<1, 64, 0, as_stream(stream)>>>(
      static_cast<unsigned long long>(limit_ns), completed, status);
  return check_launch("expire_wait_kernel");
}
