// conformer_conv.cu -- fused GLU + depthwise k9 conv + folded BatchNorm + SiLU.
//
// Restates CONFORMER_CONV_WGSL (src/webgpu/kernels/conformer-conv.ts:471-575):
//   glu[t, c]  = g[t, c] * sigmoid(g[t, 1024 + c]), zero for t outside
//                [0, min(T, valid)) (sigmoid clamps its input to [-20, 20]);
//   s[t, c]    = fma chain over k = 0..8 of glu[t + k - 4, c] * w[k, c];
//   a          = s * scale[c] + shift[c]   (BN folded, model/convert.py:1705-1735);
//   y[t, c]    = a * sigmoid(a), for every frame t < T.
// One CTA = (window, 64 frames, 128 channels): the 72-frame GLU halo tile is
// computed once into shared memory from 128-bit loads of the pointwise output,
// then each thread slides the 9-tap window down 8 frames of 4 channels.  Each
// input element is read from HBM once (plus the 8-frame halo, from L2).
#include "pk_common.cuh"
#include "pk_internal.h"

namespace pk {

constexpr int CONV_C = 1024;
constexpr int CONV_K = 9;
constexpr int CONV_TF = 64;                  // frames per CTA
constexpr int CONV_TC = 128;                 // channels per CTA
constexpr int CONV_ROWS = CONV_TF + CONV_K - 1;
constexpr int CONV_THREADS = 512;
constexpr int CONV_CPT = 2;                  // channels per thread in the depthwise phase
constexpr int CONV_FPT = CONV_TF / (CONV_THREADS / (CONV_TC / CONV_CPT));  // 8 consecutive frames per thread
constexpr int CONV_SMEM = CONV_ROWS * CONV_TC * 4;                  // 36 KB GLU tile

__device__ __forceinline__ float fast_sigmoid(float v) {
  const float b = fminf(fmaxf(v, -20.0f), 20.0f);
  return __fdividef(1.0f, 1.0f + __expf(-b));
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

// Store 4 consecutive channels.
template <typename T>
__device__ __forceinline__ void store4(T* p, const float* v);
template <>
__device__ __forceinline__ void store4<__half>(__half* p, const float* v) {
  const __half2 a = __floats2half2_rn(v[0], v[1]), b = __floats2half2_rn(v[2], v[3]);
  uint2 raw;
  raw.x = *reinterpret_cast<const uint32_t*>(&a);
  raw.y = *reinterpret_cast<const uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = raw;
}
template <>
__device__ __forceinline__ void store4<float>(float* p, const float* v) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
}
// Two consecutive channels.
template <typename T>
__device__ __forceinline__ void load2(const T* p, float* v);
template <>
__device__ __forceinline__ void load2<__half>(const __half* p, float* v) {
  const float2 a = __half22float2(__ldg(reinterpret_cast<const __half2*>(p)));
  v[0] = a.x, v[1] = a.y;
}
template <>
__device__ __forceinline__ void load2<float>(const float* p, float* v) {
  const float2 f = __ldg(reinterpret_cast<const float2*>(p));
  v[0] = f.x, v[1] = f.y;
}
template <typename T>
__device__ __forceinline__ void store2(T* p, const float* v);
template <>
__device__ __forceinline__ void store2<__half>(__half* p, const float* v) {
  *reinterpret_cast<__half2*>(p) = __floats2half2_rn(v[0], v[1]);
}
template <>
__device__ __forceinline__ void store2<float>(float* p, const float* v) {
  *reinterpret_cast<float2*>(p) = make_float2(v[0], v[1]);
}
template <typename T>
__device__ __forceinline__ void load4(const T* p, float* v);
template <>
__device__ __forceinline__ void load4<__half>(const __half* p, float* v) {
  const uint2 raw = __ldg(reinterpret_cast<const uint2*>(p));
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
  v[0] = a.x, v[1] = a.y, v[2] = b.x, v[3] = b.y;
}
template <>
__device__ __forceinline__ void load4<float>(const float* p, float* v) {
  const float4 f = __ldg(reinterpret_cast<const float4*>(p));
  v[0] = f.x, v[1] = f.y, v[2] = f.z, v[3] = f.w;
}

// One CTA = (window, CONV_TF frames, CONV_TC channels).  Phase 1: the GLU of
// the (CONV_TF + 8)-frame halo tile goes to shared memory (f32), every
// 128-bit load issued before any GLU math.  Phase 2: thread (u, sg) owns
// channels 2u, 2u+1 and frames sg*CONV_FPT ..: it slides the 9-tap window
// down its frames, so each of its CONV_FPT + 8 rows is read from shared
// memory once (a warp reads 256 contiguous bytes of one row: conflict-free)
// and reused by up to 9 outputs.  512 threads with two channels each (not
// 256 with four) keep the register count low enough for two CTAs -- 32
// warps -- per SM.
template <typename T>
__global__ void __launch_bounds__(CONV_THREADS, 2) conformer_conv_kernel(
    const T* __restrict__ g, const T* __restrict__ dw, const float* __restrict__ scale,
    const float* __restrict__ shift, const uint32_t* __restrict__ valid_lengths, T* __restrict__ out, int frames) {
  pdl_entry();
  constexpr int VEC = 16 / sizeof(T);          // channels per 16-byte global vector
  constexpr int NV = CONV_TC / VEC;            // vectors per tile row
  constexpr int ITEMS = (CONV_ROWS * NV + CONV_THREADS - 1) / CONV_THREADS;
  extern __shared__ __align__(16) float glu[];  // [CONV_ROWS][CONV_TC]
  const int c0 = blockIdx.x * CONV_TC, t0 = blockIdx.y * CONV_TF, b = blockIdx.z;
  const int tid = threadIdx.x;
  const int valid = min((int)valid_lengths[b], frames);
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
      *reinterpret_cast<float4*>(&glu[r * CONV_TC + v * VEC + j]) =
          make_float4(val[j], val[j + 1], val[j + 2], val[j + 3]);
  }
  const int u = tid % (CONV_TC / CONV_CPT), sg = tid / (CONV_TC / CONV_CPT);
  const int c = c0 + CONV_CPT * u;
  static_assert(CONV_CPT == 2, "a thread's channel pair shares each paired FMA");
  float2 w[CONV_K];
#pragma unroll
  for (int k = 0; k < CONV_K; ++k) {
    float wk[2];
    load2<T>(dw + k * CONV_C + c, wk);
    w[k] = make_float2(wk[0], wk[1]);
  }
  const float2 sc = __ldg(reinterpret_cast<const float2*>(scale + c));
  const float2 sh = __ldg(reinterpret_cast<const float2*>(shift + c));
  __syncthreads();
  const int f0 = sg * CONV_FPT;  // first frame of this thread within the tile
  float2 acc[CONV_FPT];
#pragma unroll
  for (int f = 0; f < CONV_FPT; ++f) acc[f] = make_float2(0.0f, 0.0f);
  // Row f0 + r feeds output frames f0 + r - k for taps k (fma in tap order),
  // both channels in one paired FMA (each lane exactly fmaf).
#pragma unroll
  for (int r = 0; r < CONV_FPT + CONV_K - 1; ++r) {
    const float2 q = *reinterpret_cast<const float2*>(&glu[(f0 + r) * CONV_TC + CONV_CPT * u]);
#pragma unroll
    for (int k = 0; k < CONV_K; ++k) {
      const int f = r - k;
      if (f >= 0 && f < CONV_FPT) acc[f] = ffma2(q, w[k], acc[f]);
    }
  }
#pragma unroll
  for (int f = 0; f < CONV_FPT; ++f) {
    const int t = t0 + f0 + f;
    if (t >= frames) break;
    const float2 a = ffma2(acc[f], sc, sh);
    const float y[CONV_CPT] = {a.x * fast_sigmoid(a.x), a.y * fast_sigmoid(a.y)};
    store2<T>(out + ((size_t)b * frames + t) * CONV_C + c, y);
  }
}

int launch_conformer_conv(int precision, int batch, int frames, const void* pointwise, const void* dw,
                          const float* scale, const float* shift, const uint32_t* valid_lengths, void* out,
                          cudaStream_t stream) {
  if (precision == PK_FP16 && g_reference_arith)
    return launch_ref_conformer_conv(batch, frames, pointwise, dw, scale, shift, valid_lengths, out, stream);
  const dim3 grid(CONV_C / CONV_TC, (frames + CONV_TF - 1) / CONV_TF, batch);
  if (precision == PK_FP16)
    launch_kernel(conformer_conv_kernel<__half>, grid, CONV_THREADS, CONV_SMEM, stream, 
        static_cast<const __half*>(pointwise), static_cast<const __half*>(dw), scale, shift, valid_lengths,
        static_cast<__half*>(out), frames);
  else
    launch_kernel(conformer_conv_kernel<float>, grid, CONV_THREADS, CONV_SMEM, stream, 
        static_cast<const float*>(pointwise), static_cast<const float*>(dw), scale, shift, valid_lengths,
        static_cast<float*>(out), frames);
  return cuda_error(cudaGetLastError(), "conformer_conv launch");
}

}  // namespace pk
