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

// Fast path: channels == 1024.  One warp per row, all of the row's 128-bit
// loads issued before reducing (f16: 4 per lane, f32: 8); gamma/beta are
// 128-bit L1-resident loads.  A small register footprint keeps every row of
// a batch-32 launch resident at once (one wave), so HBM latency overlaps
// across the whole launch.  One HBM read and one write of each row.
template <typename T>
constexpr int ln_rows() { return sizeof(T) == 2 ? 2 : 1; }

template <typename T>
__device__ __forceinline__ void unpack16(const uint4& raw, float* v) {
  if constexpr (sizeof(T) == 2) {
    const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __half22float2(h[j]);
      v[2 * j] = f.x;
      v[2 * j + 1] = f.y;
    }
  } else {
    const float* f = reinterpret_cast<const float*>(&raw);
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = f[j];
  }
}

template <typename T>
__global__ void __launch_bounds__(256) layernorm1024_kernel(const T* __restrict__ x, const float* __restrict__ gamma,
                                                            const float* __restrict__ beta, float eps,
                                                            T* __restrict__ y, int64_t rows) {
  constexpr int VEC = 16 / sizeof(T);        // elements per 16-byte load
  constexpr int LOADS = 1024 / (32 * VEC);   // loads per lane per row
  const int lane = threadIdx.x & 31;
  constexpr int LN_ROWS = ln_rows<T>();
  const int64_t row0 = ((int64_t)blockIdx.x * 8 + (threadIdx.x >> 5)) * LN_ROWS;
  if (row0 >= rows) return;
  uint4 raw[LN_ROWS][LOADS];
#pragma unroll
  for (int r = 0; r < LN_ROWS; ++r) {
    if (row0 + r < rows) {
      const uint4* src = reinterpret_cast<const uint4*>(x + (row0 + r) * 1024);
#pragma unroll
      for (int i = 0; i < LOADS; ++i) raw[r][i] = __ldg(src + i * 32 + lane);
    }
  }
#pragma unroll
  for (int r = 0; r < LN_ROWS; ++r) {
    if (row0 + r >= rows) break;
    float v[LOADS][VEC];
    float sum = 0.0f, sq = 0.0f;
#pragma unroll
    for (int i = 0; i < LOADS; ++i) {
      unpack16<T>(raw[r][i], v[i]);
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
    uint4* dst = reinterpret_cast<uint4*>(y + (row0 + r) * 1024);
#pragma unroll
    for (int i = 0; i < LOADS; ++i) {
      const int c0 = (i * 32 + lane) * VEC;
      float o[VEC];
#pragma unroll
      for (int j = 0; j < VEC; j += 4) {
        const float4 gg = __ldg(reinterpret_cast<const float4*>(gamma + c0 + j));
        const float4 bb = __ldg(reinterpret_cast<const float4*>(beta + c0 + j));
        o[j] = fmaf((v[i][j] - mean) * rstd, gg.x, bb.x);
        o[j + 1] = fmaf((v[i][j + 1] - mean) * rstd, gg.y, bb.y);
        o[j + 2] = fmaf((v[i][j + 2] - mean) * rstd, gg.z, bb.z);
        o[j + 3] = fmaf((v[i][j + 3] - mean) * rstd, gg.w, bb.w);
      }
      uint4 out;
      if constexpr (sizeof(T) == 2) {
        __half2* h = reinterpret_cast<__half2*>(&out);
#pragma unroll
        for (int j = 0; j < 4; ++j) h[j] = __floats2half2_rn(o[2 * j], o[2 * j + 1]);
      } else {
        float* f = reinterpret_cast<float*>(&out);
#pragma unroll
        for (int j = 0; j < 4; ++j) f[j] = o[j];
      }
      dst[i * 32 + lane] = out;
    }
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
  const bool params_aligned = ((reinterpret_cast<uintptr_t>(gamma) | reinterpret_cast<uintptr_t>(beta)) & 15) == 0;
  if (channels == 1024 && aligned && params_aligned) {
    const int per_block = 8 * (precision == PK_FP16 ? ln_rows<__half>() : ln_rows<float>());
    const unsigned blocks = (unsigned)((rows + per_block - 1) / per_block);
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
