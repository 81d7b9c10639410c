// conformer_conv.cu -- fused GLU + depthwise k9 conv + folded BatchNorm + SiLU.
//
// Restates CONFORMER_CONV_WGSL (src/webgpu/kernels/conformer-conv.ts:471-575):
//   glu[t, c]  = g[t, c] * sigmoid(g[t, 1024 + c]), zero for t outside
//                [0, min(T, valid)) (sigmoid clamps its input to [-20, 20]);
//   s[t, c]    = fma chain over k = 0..8 of glu[t + k - 4, c] * w[k, c];
//   a          = s * scale[c] + shift[c]   (BN folded, model/convert.py:1705-1735);
//   y[t, c]    = a * sigmoid(a), for every frame t < T.
// One CTA = (window, 32 frames, 128 channels): the 40-frame GLU halo tile is
// computed once into shared memory from 128-bit loads of the pointwise output,
// then every output vector is a 9-tap register FMA chain.  Each input element
// is read from HBM once (plus the 8-frame halo, from L2); HBM-bound.
#include "pk_common.cuh"
#include "pk_internal.h"

namespace pk {

constexpr int CONV_C = 1024;
constexpr int CONV_K = 9;
constexpr int CONV_TF = 32;                  // frames per CTA
constexpr int CONV_TC = 128;                 // channels per CTA
constexpr int CONV_ROWS = CONV_TF + CONV_K - 1;
constexpr int CONV_THREADS = 256;

__device__ __forceinline__ float fast_sigmoid(float v) {
  const float b = fminf(fmaxf(v, -20.0f), 20.0f);
  return __fdividef(1.0f, 1.0f + __expf(-b));
}

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
// 16 bytes already in registers -> floats.
template <typename T>
__device__ __forceinline__ void unpack_vec(const uint4& raw, float* v) {
  if constexpr (sizeof(T) == 2) {
    const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __half22float2(h[j]);
      v[2 * j] = f.x;
      v[2 * j + 1] = f.y;
    }
  } else {
    v[0] = __uint_as_float(raw.x);
    v[1] = __uint_as_float(raw.y);
    v[2] = __uint_as_float(raw.z);
    v[3] = __uint_as_float(raw.w);
  }
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
__global__ void __launch_bounds__(CONV_THREADS, 2) conformer_conv_kernel(
    const T* __restrict__ g, const T* __restrict__ dw, const float* __restrict__ scale,
    const float* __restrict__ shift, const uint32_t* __restrict__ valid_lengths, T* __restrict__ out, int frames) {
  constexpr int VEC = 16 / sizeof(T);          // channels per 16-byte vector
  constexpr int NV = CONV_TC / VEC;            // vectors per tile row
  constexpr int GROUPS = CONV_THREADS / NV;    // frame groups
  constexpr int FPT = CONV_TF / GROUPS;        // frames per thread
  __shared__ __align__(16) float glu[CONV_ROWS][CONV_TC];
  const int c0 = blockIdx.x * CONV_TC, t0 = blockIdx.y * CONV_TF, b = blockIdx.z;
  const int tid = threadIdx.x;
  const int valid = min((int)valid_lengths[b], frames);
  // ---- GLU halo tile: all of this thread's 128-bit loads are issued before
  // any GLU math so their latencies overlap.
  constexpr int ITEMS = (CONV_ROWS * NV + CONV_THREADS - 1) / CONV_THREADS;
  uint4 vraw[ITEMS], graw[ITEMS];
#pragma unroll
  for (int it = 0; it < ITEMS; ++it) {
    const int i = tid + it * CONV_THREADS;
    const int r = i / NV, v = i % NV;
    const int t = t0 - CONV_K / 2 + r;
    vraw[it] = graw[it] = make_uint4(0, 0, 0, 0);
    if (i < CONV_ROWS * NV && t >= 0 && t < valid) {
      const T* row = g + ((size_t)b * frames + t) * (2 * CONV_C) + c0 + v * VEC;
      vraw[it] = __ldg(reinterpret_cast<const uint4*>(row));
      graw[it] = __ldg(reinterpret_cast<const uint4*>(row + CONV_C));
    }
  }
#pragma unroll
  for (int it = 0; it < ITEMS; ++it) {
    const int i = tid + it * CONV_THREADS;
    if (i >= CONV_ROWS * NV) break;
    const int r = i / NV, v = i % NV;
    float val[VEC], gate[VEC];
    unpack_vec<T>(vraw[it], val);
    unpack_vec<T>(graw[it], gate);
#pragma unroll
    for (int j = 0; j < VEC; ++j) val[j] *= fast_sigmoid(gate[j]);  // zero rows stay zero
#pragma unroll
    for (int j = 0; j < VEC; j += 4)
      *reinterpret_cast<float4*>(&glu[r][v * VEC + j]) = make_float4(val[j], val[j + 1], val[j + 2], val[j + 3]);
  }
  // ---- this thread's channel vector: taps, scale, shift in registers
  const int v = tid % NV, grp = tid / NV;
  const int c = c0 + v * VEC;
  float w[CONV_K][VEC];
#pragma unroll
  for (int k = 0; k < CONV_K; ++k) load_vec<T>(dw + k * CONV_C + c, w[k]);
  float sc[VEC], sh[VEC];
#pragma unroll
  for (int j = 0; j < VEC; j += 4) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(scale + c + j));
    const float4 s = __ldg(reinterpret_cast<const float4*>(shift + c + j));
    sc[j] = a.x, sc[j + 1] = a.y, sc[j + 2] = a.z, sc[j + 3] = a.w;
    sh[j] = s.x, sh[j + 1] = s.y, sh[j + 2] = s.z, sh[j + 3] = s.w;
  }
  __syncthreads();
#pragma unroll
  for (int f = 0; f < FPT; ++f) {
    const int tl = grp + f * GROUPS;  // frame within the tile
    const int t = t0 + tl;
    if (t >= frames) break;
    float y[VEC];
#pragma unroll
    for (int j = 0; j < VEC; ++j) y[j] = 0.0f;
#pragma unroll
    for (int k = 0; k < CONV_K; ++k) {
      float x[VEC];
#pragma unroll
      for (int j = 0; j < VEC; j += 4) {
        const float4 q = *reinterpret_cast<const float4*>(&glu[tl + k][v * VEC + j]);
        x[j] = q.x, x[j + 1] = q.y, x[j + 2] = q.z, x[j + 3] = q.w;
      }
#pragma unroll
      for (int j = 0; j < VEC; ++j) y[j] = fmaf(x[j], w[k][j], y[j]);
    }
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      const float a = fmaf(y[j], sc[j], sh[j]);
      y[j] = a * fast_sigmoid(a);
    }
    store_vec<T>(out + ((size_t)b * frames + t) * CONV_C + c, y);
  }
}

int launch_conformer_conv(int precision, int batch, int frames, const void* pointwise, const void* dw,
                          const float* scale, const float* shift, const uint32_t* valid_lengths, void* out,
                          cudaStream_t stream) {
  const dim3 grid(CONV_C / CONV_TC, (frames + CONV_TF - 1) / CONV_TF, batch);
  if (precision == PK_FP16)
    conformer_conv_kernel<__half><<<grid, CONV_THREADS, 0, stream>>>(
        static_cast<const __half*>(pointwise), static_cast<const __half*>(dw), scale, shift, valid_lengths,
        static_cast<__half*>(out), frames);
  else
    conformer_conv_kernel<float><<<grid, CONV_THREADS, 0, stream>>>(
        static_cast<const float*>(pointwise), static_cast<const float*>(dw), scale, shift, valid_lengths,
        static_cast<float*>(out), frames);
  return cuda_error(cudaGetLastError(), "conformer_conv launch");
}

}  // namespace pk
