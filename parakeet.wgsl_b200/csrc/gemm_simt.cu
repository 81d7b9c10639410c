// gemm_simt.cu -- fused palette-dequantizing GEMM on the CUDA cores.
//
// Used for the FP32 package (fp32 activations, fp32 LUT, fp32 accumulate) and
// for FP16 shapes the tensor-core kernel does not tile (N % 128 != 0 or
// K % 64 != 0).  Restates the reference's FP32 SIMT GEMM
// (f32SubgroupGemmWgsl, src/webgpu/kernels/gemm.ts:2356-2599): every output is
// one fmaf chain in increasing k, so FP32 results are bit-identical to the
// oracle's FP32 mode.  Weights are decoded from their packed codes straight
// into shared memory per K-tile (never expanded to HBM).
//
// Reference-algorithm route (pk_debug_set_gemm_route(5) or
// pk_debug_set_reference_arithmetic, FP16 only): the accumulator is rounded
// to f16 after every fma, in increasing k -- the
// f16 vec4 accumulators of f16SubgroupGemmWgsl / f16PortableGemmWgsl
// (gemm.ts:1445-1502), each step taken as an f32 fma then one rounding to
// f16, as the CPU restatement states it; the epilogue rounds each step as
// written, with the correctly rounded f32 exp.  A parity route, not a fast
// path.
#include <algorithm>

#include "pk_common.cuh"
#include "pk_internal.h"

namespace pk {

constexpr int SG_BM = 64;   // tokens per CTA
constexpr int SG_BN = 128;  // output features per CTA
constexpr int SG_BK = 32;
constexpr int SG_THREADS = 256;

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }
template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }

template <typename T, int BITS, bool ACC16 = false>
__global__ void __launch_bounds__(SG_THREADS) simt_palette_gemm_kernel(
    const T* __restrict__ a, const uint32_t* __restrict__ codes, const T* __restrict__ palette,
    const float* __restrict__ bias, const T* __restrict__ residual, T* __restrict__ out, int rows, int inner,
    int columns, int groups, int group_cols, int act, int has_residual, float res_scale) {
  pdl_entry();
  constexpr int CPG = BITS == 5 ? 32 : 16, WPG = BITS == 5 ? 5 : 3, E = 1 << BITS;
  __shared__ float As[SG_BK][SG_BM + 4];
  __shared__ float Ws[SG_BK][SG_BN + 4];
  __shared__ float lut[3 * 64];
  const int tid = threadIdx.x;
  const int m0 = blockIdx.y * SG_BM, n0 = blockIdx.x * SG_BN;
  for (int i = tid; i < groups * E; i += SG_THREADS) lut[i] = to_f<T>(palette[i]);
  const int ty = tid / 16, tx = tid % 16;  // 4 tokens x 8 features per thread
  float acc[4][8];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;
  __syncthreads();

  constexpr int GROUPS_PER_ROW = SG_BN / CPG;
  for (int k0 = 0; k0 < inner; k0 += SG_BK) {
    // Activations, transposed into As[k][m].
    for (int i = tid; i < SG_BM * SG_BK; i += SG_THREADS) {
      const int m = i / SG_BK, k = i % SG_BK;
      const int gm = m0 + m, gk = k0 + k;
      As[k][m] = (gm < rows && gk < inner) ? to_f<T>(a[(size_t)gm * inner + gk]) : 0.0f;
    }
    // Decode the [SG_BK x SG_BN] weight tile group by group.
    for (int g = tid; g < SG_BK * GROUPS_PER_ROW; g += SG_THREADS) {
      const int k = g / GROUPS_PER_ROW, ng = g % GROUPS_PER_ROW;
      const int gk = k0 + k, col = n0 + ng * CPG;
      if (gk < inner && col < columns) {
        const size_t group_index = ((size_t)gk * columns + col) / CPG;
        uint32_t w[WPG];
#pragma unroll
        for (int j = 0; j < WPG; ++j) w[j] = codes[group_index * WPG + j];
        const float* lg = lut + min(col / group_cols, groups - 1) * E;
#pragma unroll
        for (int c = 0; c < CPG; ++c) {
          const int bit = c * BITS, word = bit >> 5, sh = bit & 31;
          uint32_t v = w[word] >> sh;
          if (sh + BITS > 32) v |= w[word + 1] << (32 - sh);
          Ws[k][ng * CPG + c] = lg[v & (E - 1)];
        }
      } else {
#pragma unroll
        for (int c = 0; c < CPG; ++c) Ws[k][ng * CPG + c] = 0.0f;
      }
    }
    __syncthreads();
#pragma unroll 8
    for (int k = 0; k < SG_BK; ++k) {
      float av[4], wv[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = As[k][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 8; ++j) wv[j] = Ws[k][tx * 8 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          acc[i][j] = fmaf(av[i], wv[j], acc[i][j]);
          if constexpr (ACC16) acc[i][j] = __half2float(__float2half_rn(acc[i][j]));
        }
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty * 4 + i;
    if (m >= rows) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int n = n0 + tx * 8 + j;
      if (n >= columns) continue;
      float v = acc[i][j];
      const size_t idx = (size_t)m * columns + n;
      if constexpr (ACC16) {  // the reference epilogue, each step rounded as written
        if (bias) v = __fadd_rn(v, bias[n]);
        if (act == PK_ACT_SILU) {
          const float b = fminf(fmaxf(v, -20.0f), 20.0f);
          v = __fdiv_rn(v, __fadd_rn(1.0f, __double2float_rn(exp(-(double)b))));
        } else if (act == PK_ACT_RELU) {
          v = fmaxf(v, 0.0f);
        }
        if (has_residual) v = __fadd_rn(to_f<T>(residual[idx]), __fmul_rn(res_scale, v));
      } else {
        if (bias) v += bias[n];
        if (act == PK_ACT_SILU) v = silu_ref(v);
        else if (act == PK_ACT_RELU) v = fmaxf(v, 0.0f);
        if (has_residual) v = to_f<T>(residual[idx]) + res_scale * v;
      }
      out[idx] = from_f<T>(v);
    }
  }
}

int launch_gemm_simt(const DeviceCtx& dev, const GemmArgs& g, cudaStream_t stream) {
  (void)dev;
  const dim3 grid((unsigned)((g.columns + SG_BN - 1) / SG_BN), (unsigned)((g.rows + SG_BM - 1) / SG_BM));
  if (grid.y > 65535u) return set_error(PK_E_SHAPE, "SIMT GEMM: too many rows (%lld)", (long long)g.rows);
  const int rows = (int)g.rows, inner = (int)g.inner, columns = (int)g.columns, gc = (int)g.group_cols;
  if (g.precision == PK_FP32) {
    auto* a = static_cast<const float*>(g.a);
    auto* pal = static_cast<const float*>(g.palette);
    auto* res = static_cast<const float*>(g.residual);
    auto* c = static_cast<float*>(g.c);
    if (g.bits == 5)
      launch_kernel(simt_palette_gemm_kernel<float, 5>, grid, SG_THREADS, 0, stream, 
          a, g.codes, pal, g.bias, res, c, rows, inner, columns, g.groups, gc, g.act, g.has_residual,
          g.residual_scale);
    else
      launch_kernel(simt_palette_gemm_kernel<float, 6>, grid, SG_THREADS, 0, stream, 
          a, g.codes, pal, g.bias, res, c, rows, inner, columns, g.groups, gc, g.act, g.has_residual,
          g.residual_scale);
  } else {
    auto* a = static_cast<const __half*>(g.a);
    auto* pal = static_cast<const __half*>(g.palette);
    auto* res = static_cast<const __half*>(g.residual);
    auto* c = static_cast<__half*>(g.c);
    const bool acc16 = gemm_acc16();
    auto kernel = g.bits == 5 ? (acc16 ? simt_palette_gemm_kernel<__half, 5, true> : simt_palette_gemm_kernel<__half, 5>)
                              : (acc16 ? simt_palette_gemm_kernel<__half, 6, true> : simt_palette_gemm_kernel<__half, 6>);
    launch_kernel(kernel, grid, SG_THREADS, 0, stream, a, g.codes, pal, g.bias, res, c, rows, inner, columns,
                  g.groups, gc, g.act, g.has_residual, g.residual_scale);
  }
  return cuda_error(cudaGetLastError(), "simt_palette_gemm launch");
}

}  // namespace pk
