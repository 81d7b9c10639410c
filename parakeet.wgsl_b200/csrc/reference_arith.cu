// reference_arith.cu -- CUDA-core replays of the reference shaders' FP16
// arithmetic, for parity runs only (pk_debug_set_reference_arithmetic).
//
// The production kernels compute the same functions with tensor cores, fp32
// accumulation and reordered reductions.  These kernels instead take every
// rounding step in the order the reference's shaders and the CPU restatement
// take them, so a whole encoder run can be compared with the restatement's
// reference mode value for value:
//   * LayerNorm (layernorm.ts:344-387): per row a sequential f32 sum and
//     fma sum of squares, var = max(E[x^2] - mean^2, 0), rstd = 1/sqrt(var +
//     eps), y = fma((x - mean) * rstd, gamma, beta);
//   * relative-position attention (attention.ts:485-727): per query an fma
//     chain over the 128 channels interleaving (q+u).k and (q+v).p, times
//     1/sqrt(128), masked keys at -FLT_MAX, softmax with sequential f32 sums,
//     context as an fma chain in increasing key order;
//   * the fused conformer conv (conformer-conv.ts:505-574): GLU, 9-tap fma
//     chain, folded BN as one fma, SiLU;
//   * the subsampling front end (subsampling.ts:1115-1372): conv0 3x3 s2 as an
//     fma chain from its bias, ReLU, rounded to f16, depthwise 3x3 s2 from its
//     bias (conv0 values are recomputed per depthwise tap instead of staged:
//     the same arithmetic, no scratch buffer).
// Every a*b+c is an explicit __fmaf_rn or two rounded operations (nvcc would
// otherwise contract), and exp is the correctly rounded f32 value taken from
// the double-precision function -- the shaders' exp is backend-defined, and
// the CPU restatement uses the same correctly rounded value.
#include <cuda_fp16.h>

#include <cfloat>
#include <cmath>

#include "pk_common.cuh"
#include "pk_internal.h"

namespace pk {

int g_reference_arith = 0;

namespace {

constexpr int RA_THREADS = 128;

__device__ __forceinline__ float h2f(__half v) { return __half2float(v); }
__device__ __forceinline__ float exp_cr(float x) { return __double2float_rn(exp((double)x)); }
__device__ __forceinline__ float sigmoid_cr(float v) {
  const float b = fminf(fmaxf(v, -20.0f), 20.0f);
  return __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_cr(-b)));
}
__device__ __forceinline__ int sub_len(int raw, int steps) {
  for (int s = 0; s < steps; ++s) raw = (raw + 1) / 2;
  return raw;
}

__global__ void ref_layernorm_kernel(const __half* __restrict__ x, const float* __restrict__ gamma,
                                     const float* __restrict__ beta, float eps, __half* __restrict__ y,
                                     int64_t rows, int channels) {
  pdl_entry();
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  const __half* xr = x + r * channels;
  float sum = 0.0f, square = 0.0f;
  for (int c = 0; c < channels; ++c) {
    const float v = h2f(xr[c]);
    sum = __fadd_rn(sum, v);
    square = __fmaf_rn(v, v, square);
  }
  const float inv = __fdiv_rn(1.0f, (float)channels);
  const float mean = __fmul_rn(sum, inv);
  const float var = fmaxf(__fsub_rn(__fmul_rn(square, inv), __fmul_rn(mean, mean)), 0.0f);
  const float rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
  for (int c = 0; c < channels; ++c) {
    const float nrm = __fmul_rn(__fsub_rn(h2f(xr[c]), mean), rstd);
    y[r * channels + c] = __float2half_rn(__fmaf_rn(nrm, gamma[c], beta[c]));
  }
}

// One thread per (window, head, query).  Scores live in a per-thread array.
__global__ void ref_attention_kernel(const __half* __restrict__ qkv, const __half* __restrict__ positions,
                                     const float* __restrict__ bias_u, const float* __restrict__ bias_v,
                                     const uint32_t* __restrict__ valid_lengths, __half* __restrict__ context,
                                     int batch, int frames, float scale) {
  pdl_entry();
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= batch * 8 * frames) return;
  const int i = idx % frames, h = (idx / frames) % 8, b = idx / (8 * frames);
  constexpr int H = 1024, D = 128;
  const int P = 2 * frames - 1;
  const int valid = min((int)valid_lengths[b], frames);
  const int64_t row = (int64_t)b * frames + i;
  __half* out = context + row * H + h * D;
  if (i >= valid) {
    for (int d = 0; d < D; ++d) out[d] = __float2half_rn(0.0f);
    return;
  }
  float qu[D], qv[D], sc[192];
  for (int d = 0; d < D; ++d) {
    const float q = h2f(qkv[row * 3 * H + h * D + d]);
    qu[d] = __fadd_rn(q, bias_u[h * D + d]);
    qv[d] = __fadd_rn(q, bias_v[h * D + d]);
  }
  float mx = -FLT_MAX;
  for (int j = 0; j < frames; ++j) {
    if (j >= valid) {
      sc[j] = -FLT_MAX;
      continue;
    }
    const __half* k = qkv + ((int64_t)b * frames + j) * 3 * H + H + h * D;
    const int rel = frames - 1 - i + j;
    float s = 0.0f;
    for (int d = 0; d < D; ++d) {
      const float pp = h2f(positions[(((int64_t)h * 32 + d / 4) * P + rel) * 4 + d % 4]);
      s = __fmaf_rn(qu[d], h2f(k[d]), s);
      s = __fmaf_rn(qv[d], pp, s);
    }
    s = __fmul_rn(s, scale);
    sc[j] = s;
    mx = mx < s ? s : mx;
  }
  float sum = 0.0f;
  for (int j = 0; j < valid; ++j) {
    sc[j] = exp_cr(__fsub_rn(sc[j], mx));
    sum = __fadd_rn(sum, sc[j]);
  }
  const float inv = __fdiv_rn(1.0f, sum);
  for (int j = 0; j < valid; ++j) sc[j] = __fmul_rn(sc[j], inv);
  for (int d = 0; d < D; ++d) {
    float o = 0.0f;
    for (int j = 0; j < valid; ++j) o = __fmaf_rn(sc[j], h2f(qkv[((int64_t)b * frames + j) * 3 * H + 2 * H + h * D + d]), o);
    out[d] = __float2half_rn(o);
  }
}

__global__ void ref_conformer_conv_kernel(const __half* __restrict__ pointwise, const __half* __restrict__ dw,
                                          const float* __restrict__ scale, const float* __restrict__ shift,
                                          const uint32_t* __restrict__ valid_lengths, __half* __restrict__ out,
                                          int batch, int frames) {
  pdl_entry();
  constexpr int C = 1024;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)batch * frames * C) return;
  const int c = (int)(idx % C), t = (int)((idx / C) % frames), b = (int)(idx / ((int64_t)C * frames));
  const int64_t valid = valid_lengths[b];
  float sum = 0.0f;
  for (int k = 0; k < 9; ++k) {
    const int tt = t + k - 4;
    float glu = 0.0f;
    if (tt >= 0 && tt < frames && tt < valid) {
      const int64_t row = (int64_t)b * frames + tt;
      glu = __fmul_rn(h2f(pointwise[row * 2 * C + c]), sigmoid_cr(h2f(pointwise[row * 2 * C + C + c])));
    }
    sum = __fmaf_rn(glu, h2f(dw[k * C + c]), sum);
  }
  const float affine = __fmaf_rn(sum, scale[c], shift[c]);
  out[idx] = __float2half_rn(__fmul_rn(affine, sigmoid_cr(affine)));
}

// conv0 (3x3, stride 2, pad 1, 1 -> 256 channels) at conv0 row `iy`, column
// `ix`, channel c, exactly as the shader: bias + fma chain, ReLU, f16.
__device__ __forceinline__ float conv0_value(const float* __restrict__ fb, const __half* __restrict__ w0,
                                             const float* __restrict__ b0, int iy, int ix, int c) {
  constexpr int IH = 1501, IW = 128, C = 256;
  float sum = b0[c];
  for (int ky = 0; ky < 3; ++ky) {
    const int fy = iy * 2 + ky - 1;
    if (fy < 0 || fy >= IH) continue;
    for (int kx = 0; kx < 3; ++kx) {
      const int fx = ix * 2 + kx - 1;
      if (fx < 0 || fx >= IW) continue;
      sum = __fmaf_rn(h2f(w0[(ky * 3 + kx) * C + c]), fb[(int64_t)fx * IH + fy], sum);
    }
  }
  return h2f(__float2half_rn(fmaxf(sum, 0.0f)));
}

__global__ void ref_conv0_dw2_kernel(const float* __restrict__ features, const __half* __restrict__ w0,
                                     const float* __restrict__ b0, const __half* __restrict__ wd,
                                     const float* __restrict__ bd, const uint32_t* __restrict__ feature_lengths,
                                     __half* __restrict__ out, int batch) {
  pdl_entry();
  constexpr int CH = 751, CW = 64, OH = 376, OW = 32, C = 256;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)batch * OH * OW * C) return;
  const int c = (int)(idx % C), x = (int)((idx / C) % OW), y = (int)((idx / (C * OW)) % OH);
  const int b = (int)(idx / ((int64_t)C * OW * OH));
  const int vin = sub_len((int)feature_lengths[b], 1), vout = sub_len((int)feature_lengths[b], 2);
  if (y >= vout) {
    out[idx] = __float2half_rn(0.0f);
    return;
  }
  const float* fb = features + (int64_t)b * 128 * 1501;
  float sum = bd[c];
  for (int ky = 0; ky < 3; ++ky) {
    const int iy = y * 2 + ky - 1;
    if (iy < 0 || iy >= CH || iy >= vin) continue;
    for (int kx = 0; kx < 3; ++kx) {
      const int ix = x * 2 + kx - 1;
      if (ix < 0 || ix >= CW) continue;
      sum = __fmaf_rn(conv0_value(fb, w0, b0, iy, ix, c), h2f(wd[(ky * 3 + kx) * C + c]), sum);
    }
  }
  out[idx] = __float2half_rn(sum);
}

__global__ void ref_depthwise_kernel(const __half* __restrict__ input, const __half* __restrict__ w,
                                     const float* __restrict__ bias, const uint32_t* __restrict__ feature_lengths,
                                     __half* __restrict__ out, int batch, int ih, int iw, int channels, int steps) {
  pdl_entry();
  const int oh = (ih + 2 - 3) / 2 + 1, ow = (iw + 2 - 3) / 2 + 1;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)batch * oh * ow * channels) return;
  const int c = (int)(idx % channels), x = (int)((idx / channels) % ow), y = (int)((idx / ((int64_t)channels * ow)) % oh);
  const int b = (int)(idx / ((int64_t)channels * ow * oh));
  const int vin = sub_len((int)feature_lengths[b], steps - 1), vout = sub_len((int)feature_lengths[b], steps);
  if (y >= vout) {
    out[idx] = __float2half_rn(0.0f);
    return;
  }
  float sum = bias[c];
  for (int ky = 0; ky < 3; ++ky) {
    const int iy = y * 2 + ky - 1;
    if (iy < 0 || iy >= ih || iy >= vin) continue;
    for (int kx = 0; kx < 3; ++kx) {
      const int ix = x * 2 + kx - 1;
      if (ix < 0 || ix >= iw) continue;
      sum = __fmaf_rn(h2f(input[(((int64_t)b * ih + iy) * iw + ix) * channels + c]),
                      h2f(w[(ky * 3 + kx) * channels + c]), sum);
    }
  }
  out[idx] = __float2half_rn(sum);
}

unsigned int blocks_for(int64_t n) { return (unsigned int)((n + RA_THREADS - 1) / RA_THREADS); }

}  // namespace

int launch_ref_layernorm(int64_t rows, int64_t channels, const void* x, const float* gamma, const float* beta,
                         float eps, void* y, cudaStream_t stream) {
  launch_kernel(ref_layernorm_kernel, blocks_for(rows), RA_THREADS, 0, stream, static_cast<const __half*>(x), gamma,
                beta, eps, static_cast<__half*>(y), rows, (int)channels);
  return cuda_error(cudaGetLastError(), "reference-arithmetic layernorm launch");
}

int launch_ref_attention(int batch, int frames, const void* qkv, const void* positions, const float* bias_u,
                         const float* bias_v, const uint32_t* valid_lengths, void* context, cudaStream_t stream) {
  const float scale = (float)(1.0 / std::sqrt(128.0));
  launch_kernel(ref_attention_kernel, blocks_for((int64_t)batch * 8 * frames), RA_THREADS, 0, stream,
                static_cast<const __half*>(qkv), static_cast<const __half*>(positions), bias_u, bias_v, valid_lengths,
                static_cast<__half*>(context), batch, frames, scale);
  return cuda_error(cudaGetLastError(), "reference-arithmetic attention launch");
}

int launch_ref_conformer_conv(int batch, int frames, const void* pointwise, const void* dw, const float* scale,
                              const float* shift, const uint32_t* valid_lengths, void* out, cudaStream_t stream) {
  launch_kernel(ref_conformer_conv_kernel, blocks_for((int64_t)batch * frames * 1024), RA_THREADS, 0, stream,
                static_cast<const __half*>(pointwise), static_cast<const __half*>(dw), scale, shift, valid_lengths,
                static_cast<__half*>(out), batch, frames);
  return cuda_error(cudaGetLastError(), "reference-arithmetic conformer conv launch");
}

int launch_ref_conv0_dw2(int batch, const float* features, const void* conv0_w, const float* conv0_b,
                         const void* dw_w, const float* dw_b, const uint32_t* feature_lengths, void* out,
                         cudaStream_t stream) {
  launch_kernel(ref_conv0_dw2_kernel, blocks_for((int64_t)batch * 376 * 32 * 256), RA_THREADS, 0, stream, features,
                static_cast<const __half*>(conv0_w), conv0_b, static_cast<const __half*>(dw_w), dw_b, feature_lengths,
                static_cast<__half*>(out), batch);
  return cuda_error(cudaGetLastError(), "reference-arithmetic conv0/depthwise launch");
}

int launch_ref_depthwise(int batch, int ih, int iw, int channels, const void* input, const void* w, const float* b,
                         const uint32_t* feature_lengths, int steps, void* out, cudaStream_t stream) {
  const int oh = (ih + 2 - 3) / 2 + 1, ow = (iw + 2 - 3) / 2 + 1;
  launch_kernel(ref_depthwise_kernel, blocks_for((int64_t)batch * oh * ow * channels), RA_THREADS, 0, stream,
                static_cast<const __half*>(input), static_cast<const __half*>(w), b, feature_lengths,
                static_cast<__half*>(out), batch, ih, iw, channels, steps);
  return cuda_error(cudaGetLastError(), "reference-arithmetic depthwise launch");
}

}  // namespace pk

extern "C" int pk_debug_set_reference_arithmetic(int enable) {
  pk::g_reference_arith = enable ? 1 : 0;
  return PK_OK;
}
