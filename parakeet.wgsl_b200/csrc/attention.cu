// attention.cu -- fused relative-position multi-head self-attention.
//
// Restates RELATIVE_ATTENTION_WGSL (src/webgpu/kernels/attention.ts:418-728)
// for 8 heads of 128 channels:
//   s_ij = (sum over 32 vec4 of fma((q_i+u).x, k_j.x), fma((q_i+v).x,
//           p[T-1-i+j].x), ... interleaved per component) * 1/sqrt(128)
//   keys j >= valid get -3.402823466e38; f32 softmax over keys;
//   ctx_i = fma chain over j of prob_ij * v_j; rows i >= valid are zero.
// qkv [B*T, 3072] (q | k | v per row), projected positions in the
// head-vector-position-vec4 layout [8][32][2T-1][4] (model/convert.py:
// 1195-1228), bias_u / bias_v f32 [8, 128].
// One CTA = (query block of QB queries, head, window).  Scores stay on chip
// (no O(T^2) tensor in HBM).  Requires T <= 192 like the reference
// (attention.ts:224-228).
#include "pk_common.cuh"
#include "pk_internal.h"

namespace pk {

constexpr int ATT_QB = 8;        // queries per CTA
constexpr int ATT_MAXT = 192;
constexpr int ATT_THREADS = 256;

template <typename T>
__device__ __forceinline__ void ld4(const T* p, float* v);
template <>
__device__ __forceinline__ void ld4<__half>(const __half* p, float* v) {
  const uint2 raw = __ldg(reinterpret_cast<const uint2*>(p));
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
  v[0] = a.x;
  v[1] = a.y;
  v[2] = b.x;
  v[3] = b.y;
}
template <>
__device__ __forceinline__ void ld4<float>(const float* p, float* v) {
  const float4 f = __ldg(reinterpret_cast<const float4*>(p));
  v[0] = f.x;
  v[1] = f.y;
  v[2] = f.z;
  v[3] = f.w;
}

template <typename T>
__global__ void __launch_bounds__(ATT_THREADS) rel_attention_simt_kernel(
    const T* __restrict__ qkv, const T* __restrict__ positions, const float* __restrict__ bias_u,
    const float* __restrict__ bias_v, const uint32_t* __restrict__ valid_lengths, T* __restrict__ context,
    int frames) {
  pdl_entry();
  __shared__ float qu[ATT_QB][128], qv[ATT_QB][128];
  __shared__ float probs[ATT_QB][ATT_MAXT];
  const int q0 = blockIdx.x * ATT_QB, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x;
  const int valid = min((int)valid_lengths[b], frames);
  const int P = 2 * frames - 1;
  const size_t row0 = (size_t)b * frames;
  for (int i = tid; i < ATT_QB * 128; i += ATT_THREADS) {
    const int qs = i / 128, d = i % 128, q = q0 + qs;
    float v = 0.0f;
    if (q < frames) v = (float)qkv[(row0 + q) * 3072 + h * 128 + d];
    qu[qs][d] = v + bias_u[h * 128 + d];
    qv[qs][d] = v + bias_v[h * 128 + d];
  }
  __syncthreads();
  // Scores: thread j owns key j for all queries of the block.
  const int j = tid;
  if (j < frames) {
    float s[ATT_QB];
#pragma unroll
    for (int qs = 0; qs < ATT_QB; ++qs) s[qs] = 0.0f;
    if (j < valid) {
      const T* krow = qkv + (row0 + j) * 3072 + 1024 + h * 128;
      for (int vec = 0; vec < 32; ++vec) {
        float k4[4];
        ld4<T>(krow + vec * 4, k4);
        const T* pbase = positions + ((size_t)(h * 32 + vec) * P) * 4;
#pragma unroll
        for (int qs = 0; qs < ATT_QB; ++qs) {
          const int q = q0 + qs;
          if (q < valid) {
            float p4[4];
            ld4<T>(pbase + (size_t)(frames - 1 - q + j) * 4, p4);
            float r = s[qs];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              r = fmaf(qu[qs][vec * 4 + c], k4[c], r);
              r = fmaf(qv[qs][vec * 4 + c], p4[c], r);
            }
            s[qs] = r;
          }
        }
      }
    }
    const float scale = 0.08838834764831845f;  // 1 / sqrt(128)
#pragma unroll
    for (int qs = 0; qs < ATT_QB; ++qs) probs[qs][j] = j < valid ? s[qs] * scale : -3.402823466e+38f;
  }
  __syncthreads();
  // Softmax: warp w normalizes query w's row.
  const int warp = tid >> 5, lane = tid & 31;
  if (warp < ATT_QB && q0 + warp < valid) {
    float mx = -3.402823466e+38f;
    for (int jj = lane; jj < frames; jj += 32) mx = fmaxf(mx, probs[warp][jj]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.0f;
    for (int jj = lane; jj < frames; jj += 32) {
      const float e = jj < valid ? expf(probs[warp][jj] - mx) : 0.0f;
      probs[warp][jj] = e;
      sum += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float inv = 1.0f / sum;
    for (int jj = lane; jj < frames; jj += 32) probs[warp][jj] *= inv;
  }
  __syncthreads();
  // Context: thread -> (query slot, 4-channel vector).
  for (int i = tid; i < ATT_QB * 32; i += ATT_THREADS) {
    const int qs = i / 32, vec = i % 32, q = q0 + qs;
    if (q >= frames) continue;
    float o[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (q < valid) {
      const T* vcol = qkv + row0 * 3072 + 2048 + h * 128 + vec * 4;
      for (int jj = 0; jj < valid; ++jj) {
        float v4[4];
        ld4<T>(vcol + (size_t)jj * 3072, v4);
        const float p = probs[qs][jj];
#pragma unroll
        for (int c = 0; c < 4; ++c) o[c] = fmaf(p, v4[c], o[c]);
      }
    }
    T* dst = context + (row0 + q) * 1024 + h * 128 + vec * 4;
#pragma unroll
    for (int c = 0; c < 4; ++c) dst[c] = (T)o[c];
  }
}


int launch_rel_attention(const DeviceCtx& dev, int precision, int batch, int frames, const void* qkv,
                         const void* positions, const float* bias_u, const float* bias_v,
                         const uint32_t* valid_lengths, void* context, cudaStream_t stream,
                         const void* positions_rowmajor) {
  if (precision == PK_FP16 && g_reference_arith)
    return launch_ref_attention(batch, frames, qkv, positions, bias_u, bias_v, valid_lengths, context, stream);
  if (precision == PK_FP16 && g_attention_route == 3)
    return launch_rel_attention_umma(dev, batch, frames, qkv, positions, bias_u, bias_v, valid_lengths, context,
                                     stream);
  if (precision == PK_FP16 && g_attention_route == 0 &&
      rel_attention_umma_supported(dev, frames, qkv, positions_rowmajor, context))
    return launch_rel_attention_umma(dev, batch, frames, qkv, positions_rowmajor, bias_u, bias_v, valid_lengths,
                                     context, stream);
  if (precision == PK_FP16 && g_attention_route != 1)
    return launch_rel_attention_tc(batch, frames, qkv, positions_rowmajor ? positions_rowmajor : positions, bias_u,
                                   bias_v, valid_lengths, context, stream, positions_rowmajor != nullptr);
  const dim3 grid((frames + ATT_QB - 1) / ATT_QB, 8, batch);
  if (precision == PK_FP16)
    launch_kernel(rel_attention_simt_kernel<__half>, grid, ATT_THREADS, 0, stream, 
        static_cast<const __half*>(qkv), static_cast<const __half*>(positions), bias_u, bias_v, valid_lengths,
        static_cast<__half*>(context), frames);
  else
    launch_kernel(rel_attention_simt_kernel<float>, grid, ATT_THREADS, 0, stream, 
        static_cast<const float*>(qkv), static_cast<const float*>(positions), bias_u, bias_v, valid_lengths,
        static_cast<float*>(context), frames);
  return cuda_error(cudaGetLastError(), "rel_attention launch");
}

}  // namespace pk
