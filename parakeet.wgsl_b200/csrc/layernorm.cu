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

// Fast path: channels == 1024.  One warp per row, the row's 128-bit loads
// (f16: 4 per lane, f32: 8) all issued before reducing; gamma and beta are
// staged once per CTA in shared memory (while the rows are in flight), so
// the only global traffic is one read and one write of each row.  Small
// CTAs and a small register footprint keep every row of a batch-32 launch
// resident at once, so load latency overlaps across the whole launch.
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

constexpr int LN_WARPS = 8;

template <typename T>
__global__ void __launch_bounds__(LN_WARPS * 32) layernorm1024_kernel(const T* __restrict__ x,
                                                                    const float* __restrict__ gamma,
                                                                    const float* __restrict__ beta, float eps,
                                                                    T* __restrict__ y, int64_t rows) {
  pdl_entry();
  constexpr int VEC = 16 / sizeof(T);        // elements per 16-byte load
  constexpr int LOADS = 1024 / (32 * VEC);   // loads per lane per row
  __shared__ __align__(16) float s_gamma[1024], s_beta[1024];
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * LN_WARPS + (threadIdx.x >> 5);
  uint4 raw[LOADS];
  if (row < rows) {
    const uint4* src = reinterpret_cast<const uint4*>(x + row * 1024);
#pragma unroll
    for (int i = 0; i < LOADS; ++i) raw[i] = __ldg(src + i * 32 + lane);
  }
  for (int c = threadIdx.x * 4; c < 1024; c += LN_WARPS * 32 * 4) {
    *reinterpret_cast<float4*>(s_gamma + c) = __ldg(reinterpret_cast<const float4*>(gamma + c));
    *reinterpret_cast<float4*>(s_beta + c) = __ldg(reinterpret_cast<const float4*>(beta + c));
  }
  __syncthreads();
  if (row >= rows) return;
  float v[LOADS][VEC];
  float sum = 0.0f, sq = 0.0f;
#pragma unroll
  for (int i = 0; i < LOADS; ++i) {
    unpack16<T>(raw[i], v[i]);
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
    for (int j = 0; j < VEC; j += 4) {
      const float4 gg = *reinterpret_cast<const float4*>(s_gamma + c0 + j);
      const float4 bb = *reinterpret_cast<const float4*>(s_beta + c0 + j);
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

// Row statistics and normalization of one warp's 1024-wide row held as
// v[LOADS][VEC] (lane's chunks i*32 + lane), gamma/beta from shared memory.
template <int LOADS, int VEC>
__device__ __forceinline__ void ln_row(float (&v)[LOADS][VEC], const float* s_gamma, const float* s_beta, float eps,
                                       int lane) {
  float sum = 0.0f, sq = 0.0f;
#pragma unroll
  for (int i = 0; i < LOADS; ++i)
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      sum += v[i][j];
      sq = fmaf(v[i][j], v[i][j], sq);
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
#pragma unroll
  for (int i = 0; i < LOADS; ++i) {
    const int c0 = (i * 32 + lane) * VEC;
#pragma unroll
    for (int j = 0; j < VEC; j += 4) {
      const float4 gg = *reinterpret_cast<const float4*>(s_gamma + c0 + j);
      const float4 bb = *reinterpret_cast<const float4*>(s_beta + c0 + j);
      v[i][j] = fmaf((v[i][j] - mean) * rstd, gg.x, bb.x);
      v[i][j + 1] = fmaf((v[i][j + 1] - mean) * rstd, gg.y, bb.y);
      v[i][j + 2] = fmaf((v[i][j + 2] - mean) * rstd, gg.z, bb.z);
      v[i][j + 3] = fmaf((v[i][j + 3] - mean) * rstd, gg.w, bb.w);
    }
  }
}

// Pack VEC floats into 16 bytes of T; with ROUND, v is also replaced by the
// values as stored (what a reader of the stored row sees).
template <typename T, int VEC>
__device__ __forceinline__ uint4 pack16(float (&v)[VEC]) {
  uint4 out;
  if constexpr (sizeof(T) == 2) {
    __half2* h = reinterpret_cast<__half2*>(&out);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      h[j] = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
      const float2 f = __half22float2(h[j]);
      v[2 * j] = f.x;
      v[2 * j + 1] = f.y;
    }
  } else {
    float* f = reinterpret_cast<float*>(&out);
#pragma unroll
    for (int j = 0; j < 4; ++j) f[j] = v[j];
  }
  return out;
}

// Two LayerNorms in sequence on the same rows: y1 = LN(x; g1, b1) is stored
// (rounded to T), then y2 = LN(y1 as stored; g2, b2).  The encoder ends
// every layer with norm_out and starts the next with norm_feed_forward1 on
// its output (encoder.ts:1869-2138), so this reads each row once instead of
// twice.  y2 may alias x: a warp holds its whole row before storing.
template <typename T>
__global__ void __launch_bounds__(LN_WARPS * 32) layernorm1024_dual_kernel(
    const T* x, const float* __restrict__ g1, const float* __restrict__ b1, const float* __restrict__ g2,
    const float* __restrict__ b2, float eps, T* __restrict__ y1, T* y2, int64_t rows) {
  pdl_entry();
  constexpr int VEC = 16 / sizeof(T);
  constexpr int LOADS = 1024 / (32 * VEC);
  __shared__ __align__(16) float s_g1[1024], s_b1[1024], s_g2[1024], s_b2[1024];
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * LN_WARPS + (threadIdx.x >> 5);
  uint4 raw[LOADS];
  if (row < rows) {
    const uint4* src = reinterpret_cast<const uint4*>(x + row * 1024);
#pragma unroll
    for (int i = 0; i < LOADS; ++i) raw[i] = src[i * 32 + lane];
  }
  for (int c = threadIdx.x * 4; c < 1024; c += LN_WARPS * 32 * 4) {
    *reinterpret_cast<float4*>(s_g1 + c) = __ldg(reinterpret_cast<const float4*>(g1 + c));
    *reinterpret_cast<float4*>(s_b1 + c) = __ldg(reinterpret_cast<const float4*>(b1 + c));
    *reinterpret_cast<float4*>(s_g2 + c) = __ldg(reinterpret_cast<const float4*>(g2 + c));
    *reinterpret_cast<float4*>(s_b2 + c) = __ldg(reinterpret_cast<const float4*>(b2 + c));
  }
  __syncthreads();
  if (row >= rows) return;
  float v[LOADS][VEC];
#pragma unroll
  for (int i = 0; i < LOADS; ++i) unpack16<T>(raw[i], v[i]);
  ln_row<LOADS, VEC>(v, s_g1, s_b1, eps, lane);
  uint4* d1 = reinterpret_cast<uint4*>(y1 + row * 1024);
#pragma unroll
  for (int i = 0; i < LOADS; ++i) d1[i * 32 + lane] = pack16<T, VEC>(v[i]);
  ln_row<LOADS, VEC>(v, s_g2, s_b2, eps, lane);
  uint4* d2 = reinterpret_cast<uint4*>(y2 + row * 1024);
#pragma unroll
  for (int i = 0; i < LOADS; ++i) d2[i * 32 + lane] = pack16<T, VEC>(v[i]);
}

// Generic path: any channel count, one 256-thread block per row.
template <typename T>
__global__ void __launch_bounds__(256) layernorm_generic_kernel(const T* __restrict__ x, const float* __restrict__ gamma,
                                                                const float* __restrict__ beta, float eps,
                                                                T* __restrict__ y, int64_t channels) {
  pdl_entry();
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
  if (precision == PK_FP16 && g_reference_arith)
    return launch_ref_layernorm(rows, channels, x, gamma, beta, eps, y, stream);
  const bool aligned = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15) == 0;
  const bool params_aligned = ((reinterpret_cast<uintptr_t>(gamma) | reinterpret_cast<uintptr_t>(beta)) & 15) == 0;
  if (channels == 1024 && aligned && params_aligned) {
    const unsigned blocks = (unsigned)((rows + LN_WARPS - 1) / LN_WARPS);
    if (precision == PK_FP16)
      launch_kernel(layernorm1024_kernel<__half>, blocks, LN_WARPS * 32, 0, stream, 
          static_cast<const __half*>(x), gamma, beta, eps, static_cast<__half*>(y), rows);
    else
      launch_kernel(layernorm1024_kernel<float>, blocks, LN_WARPS * 32, 0, stream, 
          static_cast<const float*>(x), gamma, beta, eps, static_cast<float*>(y), rows);
  } else {
    if (precision == PK_FP16)
      launch_kernel(layernorm_generic_kernel<__half>, (unsigned)rows, 256, 0, stream, 
          static_cast<const __half*>(x), gamma, beta, eps, static_cast<__half*>(y), channels);
    else
      launch_kernel(layernorm_generic_kernel<float>, (unsigned)rows, 256, 0, stream, 
          static_cast<const float*>(x), gamma, beta, eps, static_cast<float*>(y), channels);
  }
  return cuda_error(cudaGetLastError(), "layernorm launch");
}

int launch_layernorm_dual(int precision, int64_t rows, const void* x, const float* g1, const float* b1,
                          const float* g2, const float* b2, float eps, void* y1, void* y2, cudaStream_t stream) {
  if (precision == PK_FP16 && g_reference_arith) {
    const int st = launch_ref_layernorm(rows, 1024, x, g1, b1, eps, y1, stream);
    return st != PK_OK ? st : launch_ref_layernorm(rows, 1024, y1, g2, b2, eps, y2, stream);
  }
  const uintptr_t any = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y1) |
                        reinterpret_cast<uintptr_t>(y2) | reinterpret_cast<uintptr_t>(g1) |
                        reinterpret_cast<uintptr_t>(b1) | reinterpret_cast<uintptr_t>(g2) |
                        reinterpret_cast<uintptr_t>(b2);
  if ((any & 15) != 0) {  // unaligned: two single LayerNorms in stream order
    int st = launch_layernorm(precision, rows, 1024, x, g1, b1, eps, y1, stream);
    return st != PK_OK ? st : launch_layernorm(precision, rows, 1024, y1, g2, b2, eps, y2, stream);
  }
  const unsigned blocks = (unsigned)((rows + LN_WARPS - 1) / LN_WARPS);
  if (precision == PK_FP16)
    launch_kernel(layernorm1024_dual_kernel<__half>, blocks, LN_WARPS * 32, 0, stream, 
        static_cast<const __half*>(x), g1, b1, g2, b2, eps, static_cast<__half*>(y1), static_cast<__half*>(y2), rows);
  else
    launch_kernel(layernorm1024_dual_kernel<float>, blocks, LN_WARPS * 32, 0, stream, 
        static_cast<const float*>(x), g1, b1, g2, b2, eps, static_cast<float*>(y1), static_cast<float*>(y2), rows);
  return cuda_error(cudaGetLastError(), "layernorm dual launch");
}

}  // namespace pk
