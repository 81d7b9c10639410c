// layernorm.cu -- LayerNorm over the channel axis, one warp per row.
//
// Restates LAYERNORM_WGSL (src/webgpu/kernels/layernorm.ts:309-389): f32 sum
// and sum of squares of the row, var = max(E[x^2] - mean^2, 0),
// rstd = 1/sqrt(var + eps), y = (x - mean) * rstd * gamma + beta, stored in the
// profile scalar.  The reference spends a 256-lane workgroup per row; here a
// warp holds the whole 1024-channel row in registers (128-bit loads, shuffle
// reductions, one read and one write of the row: the HBM minimum).
#include "pk_common.cuh"
#include "pk_internal.h"

namespace pk {

// Fast path: channels == 1024.  f16 rows: 4 x 16-byte loads per lane;
// f32 rows: 8 x 16-byte loads per lane.
template <typename T>
__global__ void __launch_bounds__(256) layernorm1024_kernel(const T* __restrict__ x, const float* __restrict__ gamma,
                                                            const float* __restrict__ beta, float eps,
                                                            T* __restrict__ y, int64_t rows) {
  constexpr int VEC = 16 / sizeof(T);        // elements per 16-byte load
  constexpr int LOADS = 1024 / (32 * VEC);   // loads per lane
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const uint4* src = reinterpret_cast<const uint4*>(x + row * 1024);
  float v[LOADS][VEC];
  float sum = 0.0f, sq = 0.0f;
#pragma unroll
  for (int i = 0; i < LOADS; ++i) {
    const uint4 raw = __ldg(src + i * 32 + lane);
    if constexpr (sizeof(T) == 2) {
      const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __half22float2(h[j]);
        v[i][2 * j] = f.x;
        v[i][2 * j + 1] = f.y;
      }
    } else {
      const float* f = reinterpret_cast<const float*>(&raw);
#pragma unroll
      for (int j = 0; j < 4; ++j) v[i][j] = f[j];
    }
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      sum += v[i][j];
      sq = fmaf(v[i][j], v[i][j], sq);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    sum += __shfl_xor_sync(0xffffffffu, sum, o);
    sq += __shfl_xor_sync(0xffffffffu, sq, o);
  }
  const float inv = 1.0f / 1024.0f;
  const float mean = sum * inv;
  const float var = fmaxf(sq * inv - mean * mean, 0.0f);
  const float rstd = 1.0f / sqrtf(var + eps);
  uint4* dst = reinterpret_cast<uint4*>(y + row * 1024);
#pragma unroll
  for (int i = 0; i < LOADS; ++i) {
    const int c0 = (i * 32 + lane) * VEC;
    float o[VEC];
#pragma unroll
    for (int j = 0; j < VEC; ++j) o[j] = fmaf((v[i][j] - mean) * rstd, __ldg(gamma + c0 + j), __ldg(beta + c0 + j));
    uint4 raw;
    if constexpr (sizeof(T) == 2) {
      __half2* h = reinterpret_cast<__half2*>(&raw);
#pragma unroll
      for (int j = 0; j < 4; ++j) h[j] = __floats2half2_rn(o[2 * j], o[2 * j + 1]);
    } else {
      float* f = reinterpret_cast<float*>(&raw);
#pragma unroll
      for (int j = 0; j < 4; ++j) f[j] = o[j];
    }
    dst[i * 32 + lane] = raw;
  }
}

// Generic path: any channel count, one 256-thread block per row.
template <typename T>
__global__ void __launch_bounds__(256) layernorm_generic_kernel(const T* __restrict__ x, const float* __restrict__ gamma,
                                                                const float* __restrict__ beta, float eps,
                                                                T* __restrict__ y, int64_t channels) {
  __shared__ float red[2][8];
  const int64_t row = blockIdx.x;
  float sum = 0.0f, sq = 0.0f;
  for (int64_t c = threadIdx.x; c < channels; c += 256) {
    const float v = (float)x[row * channels + c];
    sum += v;
    sq = fmaf(v, v, sq);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    sum += __shfl_xor_sync(0xffffffffu, sum, o);
    sq += __shfl_xor_sync(0xffffffffu, sq, o);
  }
  if ((threadIdx.x & 31) == 0) {
    red[0][threadIdx.x >> 5] = sum;
    red[1][threadIdx.x >> 5] = sq;
  }
  __syncthreads();
  sum = 0.0f;
  sq = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    sum += red[0][i];
    sq += red[1][i];
  }
  const float inv = 1.0f / (float)channels;
  const float mean = sum * inv;
  const float var = fmaxf(sq * inv - mean * mean, 0.0f);
  const float rstd = 1.0f / sqrtf(var + eps);
  for (int64_t c = threadIdx.x; c < channels; c += 256) {
    const float v = (float)x[row * channels + c];
    y[row * channels + c] = (T)fmaf((v - mean) * rstd, gamma[c], beta[c]);
  }
}

int launch_layernorm(int precision, int64_t rows, int64_t channels, const void* x, const float* gamma,
                     const float* beta, float eps, void* y, cudaStream_t stream) {
  const bool aligned = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15) == 0;
  if (channels == 1024 && aligned) {
    const unsigned blocks = (unsigned)((rows + 7) / 8);
    if (precision == PK_FP16)
      layernorm1024_kernel<__half><<<blocks, 256, 0, stream>>>(static_cast<const __half*>(x), gamma, beta, eps,
                                                              static_cast<__half*>(y), rows);
    else
      layernorm1024_kernel<float><<<blocks, 256, 0, stream>>>(static_cast<const float*>(x), gamma, beta, eps,
                                                             static_cast<float*>(y), rows);
  } else {
    if (precision == PK_FP16)
      layernorm_generic_kernel<__half><<<(unsigned)rows, 256, 0, stream>>>(
          static_cast<const __half*>(x), gamma, beta, eps, static_cast<__half*>(y), channels);
    else
      layernorm_generic_kernel<float><<<(unsigned)rows, 256, 0, stream>>>(
          static_cast<const float*>(x), gamma, beta, eps, static_cast<float*>(y), channels);
  }
  return cuda_error(cudaGetLastError(), "layernorm launch");
}

}  // namespace pk
