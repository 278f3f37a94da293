// a4: tile-predictor logits in fp32 (miowtion/veda/predictor.py:251-255,
// :299-338):
//   q_hat = feats_q @ proj_q[h] + mean_q,  k_hat = feats_k @ proj_k[h] + mean_k
//   logits = q_hat . k_hat^T / sqrt(D)
// Two SIMT fp32 GEMM kernels with shared-memory tiles. The work is small
// (~4 GFLOP at the H3 shape) and must stay fp32 because the scores are only
// used through their ranking.
#include <math.h>
#include <stdio.h>

#include <mutex>

#include "common.cuh"

namespace veda {

namespace {

constexpr int kFeat = 3 * kHeadDim;  // 384
constexpr int kEmbRows = 64;
constexpr int kEmbK = 16;

// out[h, i, :] = feats[h, i, :] @ proj[heads[h]] + feats[h, i, :D]
// grid (ceil(n/64), H', 2): z selects the q or the k side.
struct EmbedParams {
  const float* feats[2];
  const float* proj[2];
  float* out[2];
  int64_t n[2];
  const int64_t* heads;
};

__global__ void __launch_bounds__(256) embed_kernel(EmbedParams p) {
  const bool k_side = blockIdx.z != 0;
  const int h = blockIdx.y;
  const int64_t n = k_side ? p.n[1] : p.n[0];
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * kEmbRows;
  if (row0 >= n) return;
  const int64_t head = p.heads[h];
  const float* feats = (k_side ? p.feats[1] : p.feats[0]) +
                       static_cast<int64_t>(h) * n * kFeat;
  const float* proj = (k_side ? p.proj[1] : p.proj[0]) +
                      head * kFeat * kHeadDim;
  float* out = (k_side ? p.out[1] : p.out[0]) +
               static_cast<int64_t>(h) * n * kHeadDim;

  // Two buffers: chunk c + 1 is loaded into registers while chunk c is
  // multiplied from shared memory.
  __shared__ __align__(16) float a_s[2][kEmbK][kEmbRows + 4];  // transposed feats chunk
  __shared__ __align__(16) float b_s[2][kEmbK][kHeadDim];
  const int tid = threadIdx.x;
  const int tr = tid / 32;  // rows tr*8 .. +8
  const int tc = tid % 32;  // cols tc*4 .. +4
  constexpr int kA = kEmbRows * kEmbK / 256;  // feats values per thread
  constexpr int kB = kEmbK * kHeadDim / 256;  // proj values per thread
  float ra[kA], rb[kB];
  auto fetch = [&](int k0) {
#pragma unroll
    for (int i = 0; i < kA; ++i) {
      const int e = tid + 256 * i;
      const int64_t row = row0 + e / kEmbK;
      ra[i] = row < n ? feats[row * kFeat + k0 + e % kEmbK] : 0.f;
    }
#pragma unroll
    for (int i = 0; i < kB; ++i) {
      const int e = tid + 256 * i;
      rb[i] = proj[static_cast<int64_t>(k0 + e / kHeadDim) * kHeadDim +
                   e % kHeadDim];
    }
  };
  auto stash = [&](int buf) {
#pragma unroll
    for (int i = 0; i < kA; ++i) {
      const int e = tid + 256 * i;
      a_s[buf][e % kEmbK][e / kEmbK] = ra[i];
    }
#pragma unroll
    for (int i = 0; i < kB; ++i) {
      const int e = tid + 256 * i;
      b_s[buf][e / kHeadDim][e % kHeadDim] = rb[i];
    }
  };
  // Column pairs accumulate with packed fp32x2 FMAs (two independent fp32
  // FMAs per instruction, rounded as fmaf rounds).
  float2 acc[8][2];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 2; ++j) acc[i][j] = make_float2(0.f, 0.f);

  fetch(0);
  constexpr int kChunks = kFeat / kEmbK;
  for (int c = 0; c < kChunks; ++c) {
    const int buf = c & 1;
    stash(buf);
    __syncthreads();
    if (c + 1 < kChunks) fetch((c + 1) * kEmbK);
#pragma unroll 8
    for (int k = 0; k < kEmbK; ++k) {
      float a[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) a[i] = a_s[buf][k][tr * 8 + i];
      const float4 b4 = *reinterpret_cast<const float4*>(&b_s[buf][k][tc * 4]);
      const float2 b01 = make_float2(b4.x, b4.y), b23 = make_float2(b4.z, b4.w);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float2 ai = make_float2(a[i], a[i]);
        acc[i][0] = __ffma2_rn(ai, b01, acc[i][0]);
        acc[i][1] = __ffma2_rn(ai, b23, acc[i][1]);
      }
    }
    // The next stash writes the other buffer; the one after writes this
    // buffer again, behind the next iteration's barrier.
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t row = row0 + tr * 8 + i;
    if (row >= n) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = tc * 4 + j;
      const float v = (j & 1) ? acc[i][j >> 1].y : acc[i][j >> 1].x;
      out[row * kHeadDim + c] = v + feats[row * kFeat + c];
    }
  }
}

// logits[h, i, j] = q_hat[h, i, :] . k_hat[h, j, :] / sqrt(D)
// grid (ceil(n_k/128), ceil(n_q/128), H'); 256 threads in a 16 x 16 grid,
// 8 x 8 outputs each: rows 4 ti + x and 64 + 4 ti + x, columns 4 tj + y and
// 64 + 4 tj + y (x, y < 4), so each thread reads its 8 query and 8 key
// values of a k step as four 16-byte shared-memory loads for 32 paired
// FMAs. Every output sums its 128 products in k order with fused
// multiply-adds, as a one-output-per-thread loop would.
constexpr int kLogitTile = 128;
constexpr int kLogitK = 16;

__global__ void __launch_bounds__(256)
    logits_kernel(const float* q_hat, const float* k_hat, int64_t n_q,
                  int64_t n_k, float sqrt_d, float* logits) {
  const int h = blockIdx.z;
  const int64_t i0 = static_cast<int64_t>(blockIdx.y) * kLogitTile;
  const int64_t j0 = static_cast<int64_t>(blockIdx.x) * kLogitTile;
  const float* qh = q_hat + static_cast<int64_t>(h) * n_q * kHeadDim;
  const float* kh = k_hat + static_cast<int64_t>(h) * n_k * kHeadDim;
  // Two buffers of a 16-wide k chunk, transposed ([k][row]): chunk c + 1
  // is loaded into registers while chunk c is multiplied.
  __shared__ __align__(16) float q_s[2][kLogitK][kLogitTile + 4];
  __shared__ __align__(16) float k_s[2][kLogitK][kLogitTile + 4];
  const int tid = threadIdx.x;
  const int ti = tid / 16, tj = tid % 16;
  float2 acc[8][4];  // [row][column pair]
#pragma unroll
  for (int x = 0; x < 8; ++x)
#pragma unroll
    for (int y = 0; y < 4; ++y) acc[x][y] = make_float2(0.f, 0.f);
  // 128 rows x 16 k of each side: 8 values per thread, 16 threads per row
  // (64 contiguous bytes).
  float rq[8], rk[8];
  auto fetch = [&](int d0) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int e = tid + 256 * i;
      const int r = e / kLogitK, d = e % kLogitK;
      rq[i] = (i0 + r < n_q) ? qh[(i0 + r) * kHeadDim + d0 + d] : 0.f;
      rk[i] = (j0 + r < n_k) ? kh[(j0 + r) * kHeadDim + d0 + d] : 0.f;
    }
  };
  fetch(0);
  constexpr int kChunks = kHeadDim / kLogitK;
  for (int c = 0; c < kChunks; ++c) {
    const int buf = c & 1;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int e = tid + 256 * i;
      q_s[buf][e % kLogitK][e / kLogitK] = rq[i];
      k_s[buf][e % kLogitK][e / kLogitK] = rk[i];
    }
    __syncthreads();
    if (c + 1 < kChunks) fetch((c + 1) * kLogitK);
#pragma unroll 4
    for (int d = 0; d < kLogitK; ++d) {
      const float4 a_lo = *reinterpret_cast<const float4*>(&q_s[buf][d][ti * 4]);
      const float4 a_hi =
          *reinterpret_cast<const float4*>(&q_s[buf][d][64 + ti * 4]);
      const float4 b_lo = *reinterpret_cast<const float4*>(&k_s[buf][d][tj * 4]);
      const float4 b_hi =
          *reinterpret_cast<const float4*>(&k_s[buf][d][64 + tj * 4]);
      const float a[8] = {a_lo.x, a_lo.y, a_lo.z, a_lo.w,
                          a_hi.x, a_hi.y, a_hi.z, a_hi.w};
      const float2 b[4] = {make_float2(b_lo.x, b_lo.y),
                           make_float2(b_lo.z, b_lo.w),
                           make_float2(b_hi.x, b_hi.y),
                           make_float2(b_hi.z, b_hi.w)};
#pragma unroll
      for (int x = 0; x < 8; ++x) {
        const float2 ax = make_float2(a[x], a[x]);
#pragma unroll
        for (int y = 0; y < 4; ++y) acc[x][y] = __ffma2_rn(ax, b[y], acc[x][y]);
      }
    }
    // The next iteration's stash writes the other buffer; this one is
    // written again only behind the barrier after that.
  }
  float* out = logits + static_cast<int64_t>(h) * n_q * n_k;
#pragma unroll
  for (int x = 0; x < 8; ++x) {
    const int64_t i = i0 + (x < 4 ? ti * 4 + x : 64 + ti * 4 + (x - 4));
    if (i >= n_q) continue;
#pragma unroll
    for (int y = 0; y < 8; ++y) {
      const int64_t j = j0 + (y < 4 ? tj * 4 + y : 64 + tj * 4 + (y - 4));
      // Divided, not multiplied by the reciprocal, as the reference does.
      const float2 v2 = acc[x][y >> 1];
      const float v = (y & 1) ? v2.y : v2.x;
      if (j < n_k) out[i * n_k + j] = __fdiv_rn(v, sqrt_d);
    }
  }
}

}  // namespace

}  // namespace veda

using namespace veda;

// Tile counts above this are rejected before any size arithmetic, so that
// n_heads (<= 65535) x (n_q + n_k) x 128 x 4 bytes stays far below 2^63.
constexpr int64_t kMaxPredictTiles = int64_t{1} << 31;

static bool predict_sizes_ok(int32_t n_heads, int64_t n_q, int64_t n_k) {
  return n_heads >= 1 && n_heads <= 65535 && n_q >= 0 && n_k >= 0 &&
         n_q <= kMaxPredictTiles && n_k <= kMaxPredictTiles;
}

extern "C" int64_t veda_predict_workspace(int32_t n_heads, int64_t n_q,
                                          int64_t n_k) {
  if (!predict_sizes_ok(n_heads, n_q, n_k)) return -1;
  return static_cast<int64_t>(n_heads) * (n_q + n_k) * kHeadDim *
         static_cast<int64_t>(sizeof(float));
}

extern "C" int veda_predict_logits(const float* feats_q, const float* feats_k,
                                   const float* proj_q, const float* proj_k,
                                   const int64_t* heads, int32_t n_heads,
                                   int64_t n_q, int64_t n_k, float* logits,
                                   void* workspace, int64_t workspace_bytes,
                                   void* stream) {
  VEDA_REQUIRE(feats_q && feats_k && proj_q && proj_k && heads && logits,
               "all tensors are required");
  VEDA_REQUIRE(n_heads >= 1 && n_heads <= 65535, "bad number of heads");
  VEDA_REQUIRE(n_q >= 0 && n_k >= 0, "bad tile counts");
  VEDA_REQUIRE(n_q <= kMaxPredictTiles && n_k <= kMaxPredictTiles,
               "tile counts above 2^31");
  VEDA_REQUIRE(workspace != nullptr &&
                   workspace_bytes >= veda_predict_workspace(n_heads, n_q, n_k),
               "workspace is smaller than veda_predict_workspace()");
  if (n_q == 0 || n_k == 0) return VEDA_OK;
  float* q_hat = static_cast<float*>(workspace);
  float* k_hat = q_hat + static_cast<int64_t>(n_heads) * n_q * kHeadDim;
  EmbedParams p{};
  p.feats[0] = feats_q;
  p.feats[1] = feats_k;
  p.proj[0] = proj_q;
  p.proj[1] = proj_k;
  p.out[0] = q_hat;
  p.out[1] = k_hat;
  p.n[0] = n_q;
  p.n[1] = n_k;
  p.heads = heads;
  const int64_t nmax = n_q > n_k ? n_q : n_k;
  dim3 g1(static_cast<unsigned>((nmax + kEmbRows - 1) / kEmbRows),
          static_cast<unsigned>(n_heads), 2);
  embed_kernel<<<g1, 256, 0, as_stream(stream)>>>(p);
  int rc = check_launch("embed_kernel");
  if (rc != VEDA_OK) return rc;
  dim3 g2(static_cast<unsigned>((n_k + kLogitTile - 1) / kLogitTile),
          static_cast<unsigned>((n_q + kLogitTile - 1) / kLogitTile),
          static_cast<unsigned>(n_heads));
  logits_kernel<<<g2, 256, 0, as_stream(stream)>>>(
      q_hat, k_hat, n_q, n_k, sqrtf(static_cast<float>(kHeadDim)), logits);
  return check_launch("logits_kernel");
}

// ---------------------------------------------------------------------------
// veda_predict_logits_noalloc: the same computation with no workspace
// argument, for callers that cannot allocate device memory themselves.
//
// Its scratch (q_hat and k_hat of one call) is this fixed file-scope array,
// which every GPU that loads the library holds until the process exits. The
// array's name in host code is only a host-side stand-in: the device address
// is obtained once per device with cudaGetSymbolAddress (with that device
// current) on the first call made on it, and passed to the kernels. The
// address is cached for the life of the process, so the entry point must not
// be used across a cudaDeviceReset (or any other teardown of the device's
// primary context), after which the module loads again at a new address.
// ---------------------------------------------------------------------------

namespace veda {
namespace {

constexpr int64_t kNoAllocScratchFloats = VEDA_PREDICT_NOALLOC_MAX_FLOATS;

static __device__ __align__(256) float g_predict_scratch[kNoAllocScratchFloats];

std::mutex g_scratch_mu;
float* g_scratch_ptr[64] = {};

// Device address of g_predict_scratch on the current device.
int scratch_on_current_device(float** out) {
  int dev = 0;
  VEDA_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64)
    return set_error(VEDA_ERR_UNSUPPORTED, "device ordinal above 63");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&p, g_predict_scratch);
    if (err != cudaSuccess)
      return check_cuda(err, "cudaGetSymbolAddress(g_predict_scratch)");
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[dev];
  return VEDA_OK;
}

}  // namespace
}  // namespace veda

extern "C" int veda_predict_logits_noalloc(
    const float* feats_q, const float* feats_k, const float* proj_q,
    const float* proj_k, const int64_t* heads, int32_t n_heads, int64_t n_q,
    int64_t n_k, float* logits, void* stream) {
  VEDA_REQUIRE(n_heads >= 1 && n_heads <= 65535, "bad number of heads");
  VEDA_REQUIRE(n_q >= 0 && n_k >= 0, "bad tile counts");
  // Bounded first, so the product below cannot wrap.
  VEDA_REQUIRE(n_q <= kMaxPredictTiles && n_k <= kMaxPredictTiles,
               "tile counts above 2^31");
  const int64_t need = static_cast<int64_t>(n_heads) * (n_q + n_k) * kHeadDim;
  if (need > kNoAllocScratchFloats) {
    char buf[256];
    snprintf(buf, sizeof(buf),
             "veda_predict_logits_noalloc: %lld heads x (%lld + %lld) tiles "
             "need %lld scratch floats, above its fixed %lld (32 MiB); call "
             "it on fewer heads at a time, or use veda_predict_logits with a "
             "workspace",
             static_cast<long long>(n_heads), static_cast<long long>(n_q),
             static_cast<long long>(n_k), static_cast<long long>(need),
             static_cast<long long>(kNoAllocScratchFloats));
    return set_error(VEDA_ERR_INVALID, buf);
  }
  float* scratch = nullptr;
  const int rc = scratch_on_current_device(&scratch);
  if (rc != VEDA_OK) return rc;
  // The embed kernel writes every q_hat / k_hat element the logits kernel
  // reads, so nothing left from an earlier call needs clearing.
  return veda_predict_logits(feats_q, feats_k, proj_q, proj_k, heads, n_heads,
                             n_q, n_k, logits, scratch,
                             kNoAllocScratchFloats *
                                 static_cast<int64_t>(sizeof(float)),
                             stream);
}
