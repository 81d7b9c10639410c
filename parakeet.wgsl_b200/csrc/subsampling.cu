// subsampling.cu -- dw-striding subsampling front end (8x in time and frequency).
//
// Restates the reference's three subsampling shaders
// (src/webgpu/kernels/subsampling.ts):
//   * FUSED_CONV0_DEPTHWISE2_WGSL (:1092-1268): conv0 3x3 stride 2 pad 1 from
//     the f32 feature-major log-mel [B, 128, 1501] to 256 channels, ReLU,
//     rounded to the profile scalar, rows >= ceil(L/2) zero; then depthwise
//     3x3 stride 2 + bias into channel-last [B, 376, 32, 256], rows >=
//     ceil(ceil(L/2)/2) zero;
//   * DEPTHWISE_WGSL (:1270-1372): depthwise 3x3 stride 2 + bias over
//     channel-last input with valid-length masking;
//   * SUBSAMPLING_TIME_MASK_WGSL (:1374-1425): zero frames past the valid
//     length (the pointwise-6 bias re-introduces non-zero padding,
//     src/webgpu/encoder.ts:2370-2377).
// The pointwise 1x1 convolutions and the flatten projection run through the
// palette GEMM.  Arithmetic order (fma chains from the bias, ky outer, kx
// inner, skipped taps outside the valid area) follows the shaders.
#include "pk_common.cuh"
#include "pk_internal.h"

namespace pk {

constexpr int SUB_IH = 1501, SUB_IW = 128, SUB_CH = 751, SUB_CW = 64, SUB_OH = 376, SUB_OW = 32, SUB_C = 256;

__device__ __forceinline__ int sub_len(int raw, int steps) {
  for (int s = 0; s < steps; ++s) raw = (raw + 1) >> 1;
  return raw;
}

template <typename T>
__device__ __forceinline__ float ldf(const T* p) {
  return (float)*p;
}

// One CTA: window b, two output rows (2*blockIdx.y, +1), 16 channels
// (blockIdx.x).  conv0 rows 4y-1 .. 4y+3 are computed once into shared memory
// (as the rounded profile scalar, held in f32) and reused by the depthwise.
template <typename T>
__global__ void __launch_bounds__(256) conv0_dw2_kernel(const float* __restrict__ fbank, const T* __restrict__ w0,
                                                        const float* __restrict__ b0, const T* __restrict__ wd,
                                                        const float* __restrict__ bd,
                                                        const uint32_t* __restrict__ feature_lengths,
                                                        T* __restrict__ out) {
  constexpr int CG = 16;        // channels per CTA
  constexpr int ROWS0 = 5;      // conv0 rows per CTA
  constexpr int IN_ROWS = 11;   // input time samples per CTA
  __shared__ float in_tile[IN_ROWS][SUB_IW + 1];
  __shared__ float c0_tile[ROWS0][SUB_CW][CG + 1];
  __shared__ float w0s[9][CG], wds[9][CG], b0s[CG], bds[CG];
  const int b = blockIdx.z;
  const int oy0 = blockIdx.y * 2;
  const int cbase = blockIdx.x * CG;
  const int raw = (int)feature_lengths[b];
  const int vin = sub_len(raw, 1), vout = sub_len(raw, 2);
  const int y0_first = 2 * oy0 - 1;      // first conv0 row
  const int iy_first = 2 * y0_first - 1; // first input time sample
  for (int i = threadIdx.x; i < 9 * CG; i += 256) {
    w0s[i / CG][i % CG] = ldf(w0 + (i / CG) * SUB_C + cbase + i % CG);
    wds[i / CG][i % CG] = ldf(wd + (i / CG) * SUB_C + cbase + i % CG);
  }
  if (threadIdx.x < CG) {
    b0s[threadIdx.x] = b0[cbase + threadIdx.x];
    bds[threadIdx.x] = bd[cbase + threadIdx.x];
  }
  for (int i = threadIdx.x; i < IN_ROWS * SUB_IW; i += 256) {
    const int r = i % IN_ROWS, x = i / IN_ROWS;  // consecutive threads walk time (contiguous)
    const int iy = iy_first + r;
    in_tile[r][x] = (iy >= 0 && iy < SUB_IH) ? fbank[((size_t)b * SUB_IW + x) * SUB_IH + iy] : 0.0f;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < ROWS0 * SUB_CW * CG; i += 256) {
    const int c = i % CG, x = (i / CG) % SUB_CW, r = i / (CG * SUB_CW);
    const int y = y0_first + r;
    float v = 0.0f;
    if (y >= 0 && y < SUB_CH && y < vin) {
      float sum = b0s[c];
#pragma unroll
      for (int ky = 0; ky < 3; ++ky) {
        const int iy = y * 2 + ky - 1;
        if (iy < 0 || iy >= SUB_IH) continue;
#pragma unroll
        for (int kx = 0; kx < 3; ++kx) {
          const int ix = x * 2 + kx - 1;
          if (ix < 0 || ix >= SUB_IW) continue;
          sum = fmaf(w0s[ky * 3 + kx][c], in_tile[iy - iy_first][ix], sum);
        }
      }
      v = (float)(T)fmaxf(sum, 0.0f);  // rounded to the profile scalar
    }
    c0_tile[r][x][c] = v;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 2 * SUB_OW * CG; i += 256) {
    const int c = i % CG, ox = (i / CG) % SUB_OW, ry = i / (CG * SUB_OW);
    const int oy = oy0 + ry;
    const size_t oi = (((size_t)b * SUB_OH + oy) * SUB_OW + ox) * SUB_C + cbase + c;
    if (oy >= vout) {
      out[oi] = (T)0.0f;
      continue;
    }
    float sum = bds[c];
#pragma unroll
    for (int ky = 0; ky < 3; ++ky) {
      const int iy = oy * 2 + ky - 1;
      if (iy < 0 || iy >= SUB_CH || iy >= vin) continue;
#pragma unroll
      for (int kx = 0; kx < 3; ++kx) {
        const int ix = ox * 2 + kx - 1;
        if (ix < 0 || ix >= SUB_CW) continue;
        sum = fmaf(c0_tile[iy - y0_first][ix][c], wds[ky * 3 + kx][c], sum);
      }
    }
    out[oi] = (T)sum;
  }
}

// Depthwise 3x3 stride 2 pad 1 + bias, channel-last; one thread per output
// element.
template <typename T>
__global__ void depthwise_kernel(const T* __restrict__ in, const T* __restrict__ w, const float* __restrict__ bias,
                                 const uint32_t* __restrict__ feature_lengths, T* __restrict__ out, int batch, int ih,
                                 int iw, int channels, int steps) {
  const int oh = (ih - 1) / 2 + 1, ow = (iw - 1) / 2 + 1;
  const int64_t total = (int64_t)batch * oh * ow * channels;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int c = (int)(i % channels);
  const int ox = (int)((i / channels) % ow);
  const int oy = (int)((i / ((int64_t)channels * ow)) % oh);
  const int b = (int)(i / ((int64_t)channels * ow * oh));
  const int raw = (int)feature_lengths[b];
  const int vin = sub_len(raw, steps - 1), vout = sub_len(raw, steps);
  if (oy >= vout) {
    out[i] = (T)0.0f;
    return;
  }
  float sum = bias[c];
#pragma unroll
  for (int ky = 0; ky < 3; ++ky) {
    const int iy = oy * 2 + ky - 1;
    if (iy < 0 || iy >= ih || iy >= vin) continue;
#pragma unroll
    for (int kx = 0; kx < 3; ++kx) {
      const int ix = ox * 2 + kx - 1;
      if (ix < 0 || ix >= iw) continue;
      sum = fmaf(ldf(in + (((int64_t)b * ih + iy) * iw + ix) * channels + c), ldf(w + (ky * 3 + kx) * channels + c),
                 sum);
    }
  }
  out[i] = (T)sum;
}

template <typename T>
__global__ void time_mask_kernel(T* __restrict__ values, const uint32_t* __restrict__ feature_lengths, int height,
                                 int row_elems, int steps) {
  const int frame = blockIdx.x, b = blockIdx.y;
  if (frame < sub_len((int)feature_lengths[b], steps)) return;
  T* row = values + ((size_t)b * height + frame) * row_elems;
  for (int i = threadIdx.x; i < row_elems; i += blockDim.x) row[i] = (T)0.0f;
}

int launch_subsampling_conv0_dw2(int precision, int batch, const float* features, const void* conv0_w,
                                 const float* conv0_b, const void* dw_w, const float* dw_b,
                                 const uint32_t* feature_lengths, void* out, cudaStream_t stream) {
  const dim3 grid(SUB_C / 16, SUB_OH / 2, batch);
  if (precision == PK_FP16)
    conv0_dw2_kernel<__half><<<grid, 256, 0, stream>>>(features, static_cast<const __half*>(conv0_w), conv0_b,
                                                       static_cast<const __half*>(dw_w), dw_b, feature_lengths,
                                                       static_cast<__half*>(out));
  else
    conv0_dw2_kernel<float><<<grid, 256, 0, stream>>>(features, static_cast<const float*>(conv0_w), conv0_b,
                                                      static_cast<const float*>(dw_w), dw_b, feature_lengths,
                                                      static_cast<float*>(out));
  return cuda_error(cudaGetLastError(), "subsampling conv0+dw2 launch");
}

int launch_subsampling_depthwise(int precision, int batch, int ih, int iw, int channels, const void* input,
                                 const void* w, const float* b, const uint32_t* feature_lengths, int steps,
                                 void* out, cudaStream_t stream) {
  const int oh = (ih - 1) / 2 + 1, ow = (iw - 1) / 2 + 1;
  const int64_t total = (int64_t)batch * oh * ow * channels;
  const unsigned blocks = (unsigned)((total + 255) / 256);
  if (precision == PK_FP16)
    depthwise_kernel<__half><<<blocks, 256, 0, stream>>>(static_cast<const __half*>(input),
                                                         static_cast<const __half*>(w), b, feature_lengths,
                                                         static_cast<__half*>(out), batch, ih, iw, channels, steps);
  else
    depthwise_kernel<float><<<blocks, 256, 0, stream>>>(static_cast<const float*>(input),
                                                        static_cast<const float*>(w), b, feature_lengths,
                                                        static_cast<float*>(out), batch, ih, iw, channels, steps);
  return cuda_error(cudaGetLastError(), "subsampling depthwise launch");
}

int launch_subsampling_time_mask(int precision, int batch, int height, int width, int channels, void* values,
                                 const uint32_t* feature_lengths, int steps, cudaStream_t stream) {
  const dim3 grid(height, batch);
  if (precision == PK_FP16)
    time_mask_kernel<__half><<<grid, 256, 0, stream>>>(static_cast<__half*>(values), feature_lengths, height,
                                                       width * channels, steps);
  else
    time_mask_kernel<float><<<grid, 256, 0, stream>>>(static_cast<float*>(values), feature_lengths, height,
                                                      width * channels, steps);
  return cuda_error(cudaGetLastError(), "subsampling time mask launch");
}

}  // namespace pk
