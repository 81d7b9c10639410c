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
// Register-tiled: a CTA of 256 threads owns BM tokens x 128 features (BM =
// 128, or 64 when the grid would not fill the SMs); a thread holds BM/16 x 8
// accumulators and reads its operands as 16-byte shared-memory vectors.  K
// advances 16 at a time through two shared-memory buffers: while one tile's
// products run, cp.async copies the next tile's activation rows and packed
// code words into the other buffer, whose weights are then decoded through
// the LUT.  Each thread still walks k in increasing order for each of its
// outputs, so the fma chain per output is the reference's.
//
// Reference-algorithm route (pk_debug_set_gemm_route(5) or
// pk_debug_set_reference_arithmetic, FP16 only): the accumulator is rounded
// to f16 after every fma, in increasing k -- the f16 vec4 accumulators of
// f16SubgroupGemmWgsl / f16PortableGemmWgsl (gemm.ts:1445-1502), each step
// taken as an f32 fma then one rounding to f16, as the CPU restatement states
// it; the epilogue rounds each step as written, with the correctly rounded
// f32 exp.  A parity route, not a fast path.
#include <algorithm>

#include "pk_common.cuh"
#include "pk_internal.h"

namespace pk {

constexpr int SG_BN = 128;  // output features per CTA
constexpr int SG_BK = 16;   // k per shared-memory tile
constexpr int SG_THREADS = 256;
constexpr int SG_PAD = 4;   // floats of padding per shared-memory row

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

// Shared-memory tiles of one k-step of 16: the activations row-major as they
// arrive ([token][k], copied by cp.async while the previous step's products
// run), the raw packed-code words of the 16 k rows, and the decoded weights
// [k][feature] as f32.
template <typename T, int BITS, int BM>
struct SimtTiles {
  static constexpr int AK = sizeof(T) == 4 ? SG_BK + 4 : SG_BK + 8;  // row pitch (16-byte multiple)
  static constexpr int CW = SG_BN * BITS / 32;                       // code words per k row of the tile
  T a[2][BM][AK];
  uint32_t codes[2][SG_BK][CW];
  float w[2][SG_BK][SG_BN + SG_PAD];
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Issues the cp.async copies of k-tile `k0` into buffer `b`: activation rows
// (16-byte pieces when the activations are 16-byte aligned, else 4-byte;
// rows past M zero-filled) and the tile's code words (4-byte pieces; words of
// features past N zero-filled).
template <typename T, int BITS, int BM, bool VEC>
__device__ __forceinline__ void simt_issue(SimtTiles<T, BITS, BM>& t, int b, const T* __restrict__ a,
                                           const uint32_t* __restrict__ codes, int rows, int inner, int columns,
                                           int m0, int n0, int k0) {
  using S = SimtTiles<T, BITS, BM>;
  constexpr int CPG = BITS == 5 ? 32 : 16, WPG = BITS == 5 ? 5 : 3;
  constexpr int PIECE = VEC ? 16 : 4;                   // bytes per copy
  constexpr int PER_ROW = SG_BK * (int)sizeof(T) / PIECE;
  for (int i = threadIdx.x; i < BM * PER_ROW; i += SG_THREADS) {
    const int r = i / PER_ROW, piece = i % PER_ROW;
    const int gm = min(m0 + r, rows - 1);
    const T* src = a + (size_t)gm * inner + k0 + piece * (PIECE / (int)sizeof(T));
    const uint32_t dst = smem_addr(&t.a[b][r][piece * (PIECE / (int)sizeof(T))]);
    if constexpr (VEC)
      cp_async16(dst, src, m0 + r < rows ? 16u : 0u);
    else
      cp_async4(dst, src, m0 + r < rows ? 4u : 0u);
  }
  for (int i = threadIdx.x; i < SG_BK * S::CW; i += SG_THREADS) {
    const int k = i / S::CW, word = i % S::CW;
    const int col = n0 + (word / WPG) * CPG;  // first feature of this word's group
    const size_t at = ((size_t)(k0 + k) * columns + n0) / CPG * WPG + word;
    cp_async4(smem_addr(&t.codes[b][k][word]), col < columns ? codes + at : codes, col < columns ? 4u : 0u);
  }
  cp_async_commit();
}

// Codes C0 .. C0 + 7 of a packed group (constant word indices, so the words
// stay in registers) through the LUT.
template <int BITS, int C0>
__device__ __forceinline__ void decode8(const uint32_t (&w)[BITS == 5 ? 5 : 3], const float* lg, float (&v)[8]) {
  constexpr int E = 1 << BITS;
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const int bit = (C0 + c) * BITS, word = bit >> 5, sh = bit & 31;
    uint32_t x = w[word] >> sh;
    if (sh + BITS > 32) x |= w[word + 1] << (32 - sh);
    v[c] = lg[x & (E - 1)];
  }
}

// Decodes buffer `b`'s code words into its f32 weight tile: thread -> k row
// tid / 16, features (tid % 16) * 8 .. + 7.
template <typename T, int BITS, int BM>
__device__ __forceinline__ void simt_decode(SimtTiles<T, BITS, BM>& t, int b, const float* lut, int columns, int n0,
                                            int groups, int group_cols) {
  constexpr int CPG = BITS == 5 ? 32 : 16, WPG = BITS == 5 ? 5 : 3, E = 1 << BITS;
  const int k = threadIdx.x / 16, seg = (threadIdx.x % 16) * 8, col = n0 + seg;
  float v[8];
  if (col < columns) {
    uint32_t w[WPG];
#pragma unroll
    for (int j = 0; j < WPG; ++j) w[j] = t.codes[b][k][(seg / CPG) * WPG + j];
    const float* lg = lut + min(col / group_cols, groups - 1) * E;
    switch ((seg % CPG) / 8) {  // first code of the 8 inside its group
      case 0: decode8<BITS, 0>(w, lg, v); break;
      case 1: decode8<BITS, 8>(w, lg, v); break;
      case 2: if constexpr (BITS == 5) decode8<BITS, 16>(w, lg, v); break;
      default: if constexpr (BITS == 5) decode8<BITS, 24>(w, lg, v); break;
    }
  } else {
#pragma unroll
    for (int c = 0; c < 8; ++c) v[c] = 0.0f;
  }
  *reinterpret_cast<float4*>(&t.w[b][k][seg]) = make_float4(v[0], v[1], v[2], v[3]);
  *reinterpret_cast<float4*>(&t.w[b][k][seg + 4]) = make_float4(v[4], v[5], v[6], v[7]);
}

// Four consecutive k of one activation row as f32.
__device__ __forceinline__ float4 load4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 load4(const __half* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
  const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
  return make_float4(lo.x, lo.y, hi.x, hi.y);
}

template <typename T, int BITS, bool ACC16, int BM, bool VEC>
__global__ void __launch_bounds__(SG_THREADS, 2) simt_palette_gemm_kernel(
    const T* __restrict__ a, const uint32_t* __restrict__ codes, const T* __restrict__ palette,
    const float* __restrict__ bias, const T* __restrict__ residual, T* __restrict__ out, int rows, int inner,
    int columns, int groups, int group_cols, int act, int has_residual, float res_scale) {
  pdl_entry();
  constexpr int E = 1 << BITS;
  constexpr int TM = BM / 16, TN = 8;
  __shared__ __align__(16) SimtTiles<T, BITS, BM> t;
  __shared__ float lut[3 * 64];
  const int tid = threadIdx.x;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * SG_BN;
  simt_issue<T, BITS, BM, VEC>(t, 0, a, codes, rows, inner, columns, m0, n0, 0);
  for (int i = tid; i < groups * E; i += SG_THREADS) lut[i] = to_f<T>(palette[i]);
  // This thread's outputs: rows ty*4 + {0..3} (and 64 + ty*4 + {0..3} when
  // BM = 128), columns tx*4 + {0..3} and 64 + tx*4 + {0..3}.
  const int ty = tid / 16, tx = tid % 16;
  // Accumulator pairs (features j, j+1): the FP32 chains run two outputs per
  // paired FMA (fma.rn.f32x2, each lane exactly fmaf, still in increasing k).
  float2 acc[TM][TN / 2];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN / 2; ++j) acc[i][j] = make_float2(0.0f, 0.0f);
  cp_async_wait_all();
  __syncthreads();  // tile 0 and the LUT
  simt_decode<T, BITS, BM>(t, 0, lut, columns, n0, groups, group_cols);
  __syncthreads();
  const int tiles = inner / SG_BK;
  for (int kt = 0; kt < tiles; ++kt) {
    const int cur = kt & 1;
    if (kt + 1 < tiles) simt_issue<T, BITS, BM, VEC>(t, cur ^ 1, a, codes, rows, inner, columns, m0, n0, (kt + 1) * SG_BK);
#pragma unroll
    for (int k4 = 0; k4 < SG_BK; k4 += 4) {
      float av[TM][4];
#pragma unroll
      for (int i = 0; i < TM; ++i) {
        const int r = i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4;
        const float4 q = load4(&t.a[cur][r][k4]);
        av[i][0] = q.x, av[i][1] = q.y, av[i][2] = q.z, av[i][3] = q.w;
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 w0 = *reinterpret_cast<const float4*>(&t.w[cur][k4 + q][tx * 4]);
        const float4 w1 = *reinterpret_cast<const float4*>(&t.w[cur][k4 + q][64 + tx * 4]);
        const float2 wv[TN / 2] = {make_float2(w0.x, w0.y), make_float2(w0.z, w0.w), make_float2(w1.x, w1.y),
                                   make_float2(w1.z, w1.w)};
#pragma unroll
        for (int i = 0; i < TM; ++i)
#pragma unroll
          for (int j = 0; j < TN / 2; ++j) {
            if constexpr (ACC16) {
              acc[i][j].x = __half2float(__float2half_rn(fmaf(av[i][q], wv[j].x, acc[i][j].x)));
              acc[i][j].y = __half2float(__float2half_rn(fmaf(av[i][q], wv[j].y, acc[i][j].y)));
            } else {
              acc[i][j] = ffma2(make_float2(av[i][q], av[i][q]), wv[j], acc[i][j]);
            }
          }
      }
    }
    if (kt + 1 < tiles) {
      cp_async_wait_all();
      __syncthreads();  // the next tile's words have landed for every thread
      simt_decode<T, BITS, BM>(t, cur ^ 1, lut, columns, n0, groups, group_cols);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const int m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
    if (m >= rows) continue;
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      const int n = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + j - 4);
      if (n >= columns) continue;
      float v = (j & 1) ? acc[i][j / 2].y : acc[i][j / 2].x;
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

template <typename T, int BM>
static cudaError_t launch_simt(const GemmArgs& g, dim3 grid, cudaStream_t stream, bool acc16) {
  auto* a = static_cast<const T*>(g.a);
  auto* pal = static_cast<const T*>(g.palette);
  auto* res = static_cast<const T*>(g.residual);
  auto* c = static_cast<T*>(g.c);
  const int rows = (int)g.rows, inner = (int)g.inner, columns = (int)g.columns, gc = (int)g.group_cols;
  const bool vec = (reinterpret_cast<uintptr_t>(g.a) & 15) == 0;
  void (*kernel)(const T*, const uint32_t*, const T*, const float*, const T*, T*, int, int, int, int, int, int, int,
                 float);
  if (g.bits == 5)
    kernel = acc16 ? (vec ? simt_palette_gemm_kernel<T, 5, true, BM, true> : simt_palette_gemm_kernel<T, 5, true, BM, false>)
                   : (vec ? simt_palette_gemm_kernel<T, 5, false, BM, true> : simt_palette_gemm_kernel<T, 5, false, BM, false>);
  else
    kernel = acc16 ? (vec ? simt_palette_gemm_kernel<T, 6, true, BM, true> : simt_palette_gemm_kernel<T, 6, true, BM, false>)
                   : (vec ? simt_palette_gemm_kernel<T, 6, false, BM, true> : simt_palette_gemm_kernel<T, 6, false, BM, false>);
  return launch_kernel(kernel, grid, SG_THREADS, 0, stream, a, g.codes, pal, g.bias, res, c, rows, inner, columns,
                       g.groups, gc, g.act, g.has_residual, g.residual_scale);
}

int launch_gemm_simt(const DeviceCtx& dev, const GemmArgs& g, cudaStream_t stream) {
  if (g.inner % SG_BK != 0) return set_error(PK_E_SHAPE, "SIMT GEMM: K must be a multiple of %d", SG_BK);
  const unsigned n_tiles = (unsigned)((g.columns + SG_BN - 1) / SG_BN);
  // 128-token tiles when they fill the SMs, else 64.
  const bool big = (uint64_t)((g.rows + 127) / 128) * n_tiles >= (uint64_t)dev.sm_count;
  const int bm = big ? 128 : 64;
  const dim3 grid(n_tiles, (unsigned)((g.rows + bm - 1) / bm));
  if (grid.y > 65535u) return set_error(PK_E_SHAPE, "SIMT GEMM: too many rows (%lld)", (long long)g.rows);
  const bool acc16 = g.precision == PK_FP16 && gemm_acc16();
  cudaError_t e;
  if (g.precision == PK_FP32)
    e = big ? launch_simt<float, 128>(g, grid, stream, false) : launch_simt<float, 64>(g, grid, stream, false);
  else
    e = big ? launch_simt<__half, 128>(g, grid, stream, acc16) : launch_simt<__half, 64>(g, grid, stream, acc16);
  return cuda_error(e, "simt_palette_gemm launch");
}

}  // namespace pk
