// Tile-search oracle error (miowtion/veda/search.py:86-127): the relative
// MSE of the sparse output of sampled query tiles against the dense output,
// per head,
//
//   rel_mse[h] = sum_rows ||o_sparse - o_dense||^2 / sum_rows ||o_dense||^2
//
// over the real rows of the sampled tiles (differences and squares in fp32
// of the bf16 outputs, as the reference's `.float()` arithmetic).
//
// HBM-bound: every sampled row of both outputs is read once (2 x 256 bytes
// per row and head). One CTA per (sampled tile, head) reduces its 128 rows
// to an (error, norm) pair in a fixed order; a second kernel sums the pairs
// of each head in tile order in fp64, so the result is deterministic.
#include "common.cuh"

namespace veda {

namespace {

constexpr int kMseThreads = 256;  // 8 warps x 16 rows each

__device__ __forceinline__ void bf16x4(const uint2& v, float* f) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
  const float2 a = __bfloat1622float2(h[0]);
  const float2 b = __bfloat1622float2(h[1]);
  f[0] = a.x;
  f[1] = a.y;
  f[2] = b.x;
  f[3] = b.y;
}

// Grid (n_rows, n_heads). Block (r, h): sampled tile r (slots r*128 ...
// r*128 + 127 of o_sparse), head h of o_sparse and head heads[h] of o_dense.
__global__ void __launch_bounds__(kMseThreads)
    rel_mse_tiles_kernel(const __nv_bfloat16* __restrict__ sparse,
                         int64_t ss, int64_t sh,
                         const __nv_bfloat16* __restrict__ dense, int64_t ds,
                         int64_t dh, const int64_t* __restrict__ seq_row,
                         const int64_t* __restrict__ heads,
                         float2* __restrict__ partial, int n_rows) {
  const int r = blockIdx.x;
  const int h = blockIdx.y;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int64_t hd = heads[h];
  float err = 0.f, norm = 0.f;
  for (int i = warp; i < kTile; i += kMseThreads / 32) {
    const int64_t slot = static_cast<int64_t>(r) * kTile + i;
    const int64_t src = seq_row[slot];
    if (src < 0) continue;  // padding slot: not a real row
    const uint2 a = *reinterpret_cast<const uint2*>(sparse + slot * ss +
                                                    h * sh + lane * 4);
    const uint2 b = *reinterpret_cast<const uint2*>(dense + src * ds +
                                                    hd * dh + lane * 4);
    float fa[4], fb[4];
    bf16x4(a, fa);
    bf16x4(b, fb);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float d = fa[e] - fb[e];
      err = fmaf(d, d, err);
      norm = fmaf(fb[e], fb[e], norm);
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    err += __shfl_xor_sync(0xffffffffu, err, off);
    norm += __shfl_xor_sync(0xffffffffu, norm, off);
  }
  __shared__ float2 s_part[kMseThreads / 32];
  if (lane == 0) s_part[warp] = make_float2(err, norm);
  __syncthreads();
  if (threadIdx.x == 0) {
    float2 t = s_part[0];
    for (int w = 1; w < kMseThreads / 32; ++w) {
      t.x += s_part[w].x;
      t.y += s_part[w].y;
    }
    partial[static_cast<int64_t>(h) * n_rows + r] = t;
  }
}

// One CTA per head: the head's tile pairs summed in tile order (fp64).
__global__ void rel_mse_heads_kernel(const float2* __restrict__ partial,
                                     int n_rows, float* __restrict__ out) {
  const int h = blockIdx.x;
  __shared__ double s_err[256], s_norm[256];
  double err = 0.0, norm = 0.0;
  // Thread t sums tiles t, t + 256, ...; then a fixed-shape tree.
  for (int r = threadIdx.x; r < n_rows; r += blockDim.x) {
    const float2 p = partial[static_cast<int64_t>(h) * n_rows + r];
    err += p.x;
    norm += p.y;
  }
  s_err[threadIdx.x] = err;
  s_norm[threadIdx.x] = norm;
  __syncthreads();
  for (int stride = blockDim.x / 2; stride > 0; stride >>= 1) {
    if (threadIdx.x < stride) {
      s_err[threadIdx.x] += s_err[threadIdx.x + stride];
      s_norm[threadIdx.x] += s_norm[threadIdx.x + stride];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const float tiny = 1.17549435e-38f;  // smallest normal float32
    const float e = static_cast<float>(s_err[0]);
    const float n = static_cast<float>(s_norm[0]);
    out[h] = e / fmaxf(n, tiny);
  }
}

}  // namespace

}  // namespace veda

using namespace veda;

extern "C" int64_t veda_rel_mse_workspace(int64_t n_rows, int32_t n_heads) {
  return n_rows * n_heads * static_cast<int64_t>(sizeof(float2));
}

extern "C" int veda_rel_mse(const void* o_sparse, int64_t s_stride_n,
                            int64_t s_stride_h, const void* o_dense,
                            int64_t d_stride_s, int64_t d_stride_h,
                            const int64_t* seq_row, const int64_t* heads,
                            int64_t n_rows, int32_t n_heads, float* rel_mse,
                            void* workspace, int64_t workspace_bytes,
                            void* stream) {
  VEDA_REQUIRE(o_sparse != nullptr && o_dense != nullptr &&
                   seq_row != nullptr && heads != nullptr &&
                   rel_mse != nullptr,
               "o_sparse, o_dense, seq_row, heads and rel_mse are required");
  VEDA_REQUIRE(n_heads >= 1 && n_heads <= 65535, "bad number of heads");
  VEDA_REQUIRE(n_rows >= 0 && n_rows <= (1LL << 31) - 1,
               "bad number of sampled tiles");
  VEDA_REQUIRE(reinterpret_cast<uintptr_t>(o_sparse) % 8 == 0 &&
                   reinterpret_cast<uintptr_t>(o_dense) % 8 == 0 &&
                   s_stride_n % 4 == 0 && s_stride_h % 4 == 0 &&
                   d_stride_s % 4 == 0 && d_stride_h % 4 == 0,
               "outputs must be 8-byte aligned with strides that are "
               "multiples of 4 elements");
  VEDA_REQUIRE(workspace_bytes >= veda_rel_mse_workspace(n_rows, n_heads) &&
                   (n_rows == 0 || workspace != nullptr),
               "workspace too small (veda_rel_mse_workspace)");
  float2* partial = static_cast<float2*>(workspace);
  cudaStream_t s = as_stream(stream);
  if (n_rows > 0) {
    rel_mse_tiles_kernel<<<dim3(static_cast<unsigned>(n_rows),
                                static_cast<unsigned>(n_heads)),
                           kMseThreads, 0, s>>>(
        static_cast<const __nv_bfloat16*>(o_sparse), s_stride_n, s_stride_h,
        static_cast<const __nv_bfloat16*>(o_dense), d_stride_s, d_stride_h,
        seq_row, heads, partial, static_cast<int>(n_rows));
    const int rc = check_launch("rel_mse_tiles_kernel");
    if (rc != VEDA_OK) return rc;
  }
  rel_mse_heads_kernel<<<static_cast<unsigned>(n_heads), 256, 0, s>>>(
      partial, static_cast<int>(n_rows), rel_mse);
  return check_launch("rel_mse_heads_kernel");
}
