// conformer_conv.cu -- fused GLU + depthwise k9 conv + folded BatchNorm + SiLU.
//
// Restates CONFORMER_CONV_WGSL (src/webgpu/kernels/conformer-conv.ts:471-575):
//   glu[t, c]  = g[t, c] * sigmoid(g[t, 1024 + c]), zero for t outside
//                [0, min(T, valid)) (sigmoid clamps its input to [-20, 20]);
//   s[t, c]    = fma chain over k = 0..8 of glu[t + k - 4, c] * w[k, c];
//   a          = s * scale[c] + shift[c]   (BN folded, model/convert.py:1705-1735);
//   y[t, c]    = a * sigmoid(a), for every frame t < T.
// Each thread owns one 16-byte channel vector of one window and walks a frame
// range with a 9-frame register window, so every input row is read once per
// frame range (HBM-bound: read 2048 + write 1024 values per frame).
#include "pk_common.cuh"
#include "pk_internal.h"

namespace pk {

constexpr int CONV_C = 1024;
constexpr int CONV_K = 9;
constexpr int CONV_FRAME_CHUNK = 16;  // frames per thread (halo of 8 re-read from L2)

template <typename T>
__device__ __forceinline__ void load_vec(const T* p, float* v);
template <>
__device__ __forceinline__ void load_vec<__half>(const __half* p, float* v) {
  const uint4 raw = __ldg(reinterpret_cast<const uint4*>(p));
  const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __half22float2(h[j]);
    v[2 * j] = f.x;
    v[2 * j + 1] = f.y;
  }
}
template <>
__device__ __forceinline__ void load_vec<float>(const float* p, float* v) {
  const float4 f = __ldg(reinterpret_cast<const float4*>(p));
  v[0] = f.x;
  v[1] = f.y;
  v[2] = f.z;
  v[3] = f.w;
}
template <typename T>
__device__ __forceinline__ void store_vec(T* p, const float* v);
template <>
__device__ __forceinline__ void store_vec<__half>(__half* p, const float* v) {
  uint4 raw;
  __half2* h = reinterpret_cast<__half2*>(&raw);
#pragma unroll
  for (int j = 0; j < 4; ++j) h[j] = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
  *reinterpret_cast<uint4*>(p) = raw;
}
template <>
__device__ __forceinline__ void store_vec<float>(float* p, const float* v) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
}

template <typename T>
__global__ void __launch_bounds__(128) conformer_conv_kernel(const T* __restrict__ g, const T* __restrict__ dw,
                                                             const float* __restrict__ scale,
                                                             const float* __restrict__ shift,
                                                             const uint32_t* __restrict__ valid_lengths,
                                                             T* __restrict__ out, int batch, int frames) {
  constexpr int VEC = 16 / sizeof(T);
  constexpr int CV = CONV_C / VEC;  // channel vectors per frame
  const int cv = blockIdx.x * blockDim.x + threadIdx.x;
  const int b = blockIdx.z;
  if (cv >= CV || b >= batch) return;
  const int t0 = blockIdx.y * CONV_FRAME_CHUNK;
  const int t1 = min(frames, t0 + CONV_FRAME_CHUNK);
  if (t0 >= t1) return;
  const int valid = min((int)valid_lengths[b], frames);
  const int c0 = cv * VEC;
  float w[CONV_K][VEC];
#pragma unroll
  for (int k = 0; k < CONV_K; ++k) load_vec<T>(dw + k * CONV_C + c0, w[k]);
  float sc[VEC], sh[VEC];
#pragma unroll
  for (int j = 0; j < VEC; ++j) {
    sc[j] = __ldg(scale + c0 + j);
    sh[j] = __ldg(shift + c0 + j);
  }
  float win[CONV_K][VEC];  // GLU values of frames t-4 .. t+4
  auto glu_at = [&](int tt, float* dst) {
    if (tt >= 0 && tt < frames && tt < valid) {
      const T* row = g + ((size_t)b * frames + tt) * (2 * CONV_C);
      float v[VEC], gt[VEC];
      load_vec<T>(row + c0, v);
      load_vec<T>(row + CONV_C + c0, gt);
#pragma unroll
      for (int j = 0; j < VEC; ++j) dst[j] = v[j] * sigmoid_ref(gt[j]);
    } else {
#pragma unroll
      for (int j = 0; j < VEC; ++j) dst[j] = 0.0f;
    }
  };
#pragma unroll
  for (int k = 0; k < CONV_K - 1; ++k) glu_at(t0 - 4 + k, win[k + 1]);
  for (int t = t0; t < t1; ++t) {
#pragma unroll
    for (int k = 0; k < CONV_K - 1; ++k)
#pragma unroll
      for (int j = 0; j < VEC; ++j) win[k][j] = win[k + 1][j];
    glu_at(t + 4, win[CONV_K - 1]);
    float y[VEC];
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      float s = 0.0f;
#pragma unroll
      for (int k = 0; k < CONV_K; ++k) s = fmaf(win[k][j], w[k][j], s);
      const float a = fmaf(s, sc[j], sh[j]);
      y[j] = a * sigmoid_ref(a);
    }
    store_vec<T>(out + ((size_t)b * frames + t) * CONV_C + c0, y);
  }
}

int launch_conformer_conv(int precision, int batch, int frames, const void* pointwise, const void* dw,
                          const float* scale, const float* shift, const uint32_t* valid_lengths, void* out,
                          cudaStream_t stream) {
  const int vec = precision == PK_FP16 ? 8 : 4;
  const int cvs = CONV_C / vec;
  const dim3 block(128);
  const dim3 grid((cvs + 127) / 128, (frames + CONV_FRAME_CHUNK - 1) / CONV_FRAME_CHUNK, batch);
  if (precision == PK_FP16)
    conformer_conv_kernel<__half><<<grid, block, 0, stream>>>(
        static_cast<const __half*>(pointwise), static_cast<const __half*>(dw), scale, shift, valid_lengths,
        static_cast<__half*>(out), batch, frames);
  else
    conformer_conv_kernel<float><<<grid, block, 0, stream>>>(
        static_cast<const float*>(pointwise), static_cast<const float*>(dw), scale, shift, valid_lengths,
        static_cast<float*>(out), batch, frames);
  return cuda_error(cudaGetLastError(), "conformer_conv launch");
}

}  // namespace pk
