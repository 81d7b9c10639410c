// capi.cu -- extern "C" entry points of libpk_b200.so for the operator layer.
//
// Each entry point validates its arguments the way the reference's operator
// classes do (synchronous errors before any GPU work: requireGemmShape /
// requireRuntimeWeight / validatePalettePair in src/webgpu/kernels/gemm.ts:
// 971-1161 and src/model/runtime-plan.ts:529-588, requireTransientDescriptor in
// src/model/palette-expander.ts:336-402), then launches its kernel on the
// caller's stream.  There is no CPU fallback: a missing or failing kernel is
// an error.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <set>
#include <string>
#include <utility>

#include "pk_internal.h"

namespace pk {

static thread_local std::string t_last_error;
int g_gemm_route = 0;
int g_gemm_tile = 0;
int g_attention_route = 0;
int g_decoder_route = 0;

int set_error(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return code;
}

int cuda_error(cudaError_t err, const char* what) {
  if (err == cudaSuccess) return PK_OK;
  if (err == cudaErrorMemoryAllocation)
    return set_error(PK_E_OOM, "%s: %s", what, cudaGetErrorString(err));
  return set_error(PK_E_CUDA, "%s: %s", what, cudaGetErrorString(err));
}

int set_max_dynamic_smem(const void* kernel, int bytes) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_error(e, "cudaGetDevice");
  std::lock_guard<std::mutex> lock(mu);
  if (done.count({kernel, dev})) return PK_OK;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(max dynamic shared memory)");
  done.insert({kernel, dev});
  return PK_OK;
}

int validate_gemm(const GemmArgs& g) {
  if (!g.a || !g.codes || !g.palette || !g.c) return set_error(PK_E_INVALID, "GEMM operand pointer is null");
  if (g.precision != PK_FP16 && g.precision != PK_FP32)
    return set_error(PK_E_INVALID, "unknown precision %d", g.precision);
  if (g.rows <= 0 || g.inner <= 0 || g.inner % 32 != 0 || g.columns <= 0 || g.columns % 8 != 0)
    return set_error(PK_E_SHAPE, "Unsupported GEMM shape: M=%lld K=%lld N=%lld (needs K%%32==0, N%%8==0)",
                     (long long)g.rows, (long long)g.inner, (long long)g.columns);
  if (g.rows > ((int64_t)1 << 31) / 8 || g.inner > (1 << 20) || g.columns > (1 << 20))
    return set_error(PK_E_SHAPE, "GEMM shape exceeds the supported range");
  if (g.bits != 5 && g.bits != 6) return set_error(PK_E_LAYOUT, "palette bits must be 5 or 6, got %d", g.bits);
  const int cpg = g.bits == 5 ? 32 : 16;
  if (g.columns % cpg != 0)
    return set_error(PK_E_LAYOUT, "palette codes are not group aligned (N=%lld, %d codes per group)",
                     (long long)g.columns, cpg);
  if (g.groups <= 0 || g.group_cols <= 0 || g.group_cols * g.groups != g.columns || g.group_cols % cpg != 0)
    return set_error(PK_E_LAYOUT, "palette does not partition output columns (G=%d, group columns=%lld)", g.groups,
                     (long long)g.group_cols);
  if ((g.groups << g.bits) > 192)
    return set_error(PK_E_LAYOUT, "palette has %d entries; at most 192 are supported", g.groups << g.bits);
  if (g.bias && g.has_residual) return set_error(PK_E_SIGNATURE, "cannot fuse bias and residual together");
  if (g.has_residual && !g.residual) return set_error(PK_E_INVALID, "residual requested but pointer is null");
  if (g.act < PK_ACT_NONE || g.act > PK_ACT_RELU) return set_error(PK_E_INVALID, "unknown activation %d", g.act);
  return PK_OK;
}

static inline cudaStream_t as_stream(pk_stream s) { return static_cast<cudaStream_t>(s); }

}  // namespace pk

using namespace pk;

extern "C" {

int pk_last_error(char* buffer, size_t length) {
  if (!buffer || length == 0) return PK_E_INVALID;
  std::snprintf(buffer, length, "%s", t_last_error.c_str());
  return PK_OK;
}

int pk_version(void) { return 1; }

int pk_device_open(int ordinal, pk_device** out) {
  if (!out) return set_error(PK_E_INVALID, "out is null");
  *out = nullptr;
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess) return cuda_error(e, "cudaGetDeviceCount");
  if (ordinal < 0 || ordinal >= count) return set_error(PK_E_INVALID, "device ordinal %d out of range", ordinal);
  if ((e = cudaSetDevice(ordinal)) != cudaSuccess) return cuda_error(e, "cudaSetDevice");
  cudaDeviceProp prop;
  if ((e = cudaGetDeviceProperties(&prop, ordinal)) != cudaSuccess) return cuda_error(e, "cudaGetDeviceProperties");
  if (prop.major != 10) return set_error(PK_E_INVALID, "device %d is sm_%d%d; libpk_b200 targets sm_100a", ordinal,
                                         prop.major, prop.minor);
  auto* d = new pk_device();
  d->ctx.ordinal = ordinal;
  d->ctx.sm_count = prop.multiProcessorCount;
  d->ctx.max_smem_optin = (int)prop.sharedMemPerBlockOptin;
  cudaDriverEntryPointQueryResult q;
  void* fn = nullptr;
  e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn) {
    delete d;
    return set_error(PK_E_CUDA, "cuTensorMapEncodeTiled is unavailable");
  }
  d->ctx.encode_tiled = fn;
  if ((e = cudaMalloc(&d->ctx.status, sizeof(unsigned int))) != cudaSuccess) {
    delete d;
    return cuda_error(e, "cudaMalloc(status)");
  }
  cudaMemset(d->ctx.status, 0, sizeof(unsigned int));
  if ((e = cudaMalloc(&d->ctx.tdt_exchange, kTdtExchangeBytes)) != cudaSuccess) {
    cudaFree(d->ctx.status);
    delete d;
    return cuda_error(e, "cudaMalloc(decoder exchange)");
  }
  *out = d;
  return PK_OK;
}

int pk_device_close(pk_device* device) {
  if (!device) return PK_OK;
  if (!device->closed) {
    cudaSetDevice(device->ctx.ordinal);
    cudaFree(device->ctx.status);
    cudaFree(device->ctx.tdt_exchange);
    device->closed = true;
  }
  delete device;
  return PK_OK;
}

int pk_device_status(pk_device* device, uint32_t* status_bits) {
  if (!device || !status_bits) return set_error(PK_E_INVALID, "null argument");
  cudaSetDevice(device->ctx.ordinal);
  unsigned int v = 0;
  cudaError_t e = cudaMemcpy(&v, device->ctx.status, sizeof(v), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_error(e, "reading device status");
  cudaMemset(device->ctx.status, 0, sizeof(unsigned int));
  *status_bits = v;
  return v ? set_error(PK_E_TIMEOUT, "a bounded device wait expired (status bits 0x%x)", v) : PK_OK;
}

int pk_palette_expand(pk_device* device, const pk_palette_desc* d, pk_stream stream) {
  if (!device || !d) return set_error(PK_E_INVALID, "null argument");
  if (!d->codes || !d->palette || !d->target) return set_error(PK_E_INVALID, "palette expansion pointer is null");
  if (d->precision != PK_FP16 && d->precision != PK_FP32) return set_error(PK_E_INVALID, "unknown precision");
  if (d->bits != 5 && d->bits != 6) return set_error(PK_E_LAYOUT, "palette bits must be 5 or 6");
  const int cpg = d->bits == 5 ? 32 : 16;
  const int64_t scalars = d->inner * d->columns;
  if (d->inner <= 0 || d->columns <= 0 || scalars % cpg != 0 || d->palette_groups <= 0 ||
      d->palette_group_columns <= 0 || d->columns % d->palette_group_columns != 0 ||
      d->palette_group_columns * d->palette_groups != d->columns)
    return set_error(PK_E_LAYOUT, "invalid transient palette geometry");
  if (d->layout == PK_LAYOUT_ROW_MAJOR) {
    if (d->bits == 6) return set_error(PK_E_LAYOUT, "The fixed runtime has no row-major palette6 matrix");
  } else if (d->layout == PK_LAYOUT_TILE_MAJOR) {
    const int64_t tile = d->precision == PK_FP16 ? 256 : 128;
    if (d->inner % 32 != 0 || d->columns % tile != 0) return set_error(PK_E_LAYOUT, "invalid tile-major geometry");
  } else {
    return set_error(PK_E_LAYOUT, "unknown expanded layout %d", d->layout);
  }
  cudaSetDevice(device->ctx.ordinal);
  return launch_palette_expand(*d, as_stream(stream));
}

int pk_palette_gemm(pk_device* device, const pk_gemm_desc* d, pk_stream stream) {
  if (!device || !d) return set_error(PK_E_INVALID, "null argument");
  GemmArgs g;
  g.precision = d->precision;
  g.rows = d->rows;
  g.inner = d->inner;
  g.columns = d->columns;
  g.bits = d->bits;
  g.groups = d->palette_groups;
  g.group_cols = d->palette_group_columns;
  g.act = d->activation;
  g.has_residual = d->has_residual;
  g.residual_scale = d->residual_scale;
  g.bias = d->bias;
  g.residual = d->residual;
  g.a = d->a;
  g.codes = d->codes;
  g.palette = d->palette;
  g.c = d->c;
  int st = validate_gemm(g);
  if (st != PK_OK) return st;
  cudaSetDevice(device->ctx.ordinal);
  const bool tc = gemm_tc_supported(g);
  if (g_gemm_route >= 2 && g_gemm_route <= 4 && !tc) return set_error(PK_E_SHAPE, "tensor-core GEMM forced but shape unsupported");
  if (tc && !gemm_route_simt()) return launch_gemm_tc(device->ctx, g, as_stream(stream));
  return launch_gemm_simt(device->ctx, g, as_stream(stream));
}

// Test hook: 0 automatic, 1 SIMT only, 2 tensor cores only, 3 tensor cores
// with single-CTA tiles only, 4 tensor cores with CTA-pair tiles wherever N
// is a multiple of 256, 5 SIMT with FP16 accumulating in f16 (the
// reference's own algorithm; a parity route).
int pk_debug_set_gemm_route(int route) {
  if (route < 0 || route > 5) return set_error(PK_E_INVALID, "route must be 0..5");
  g_gemm_route = route;
  return PK_OK;
}

// Test hook: 0 automatic; 128/192/256 a single-CTA token tile; -256/-384/-512
// a CTA-pair token tile (pairs only where N is a multiple of 256).
int pk_debug_set_gemm_tile(int tile) {
  switch (tile) {
    case 0: case 128: case 192: case 256: case -256: case -384: case -512:
      g_gemm_tile = tile;
      return PK_OK;
    default:
      return set_error(PK_E_INVALID, "tile must be 0, 128, 192, 256, -256, -384 or -512");
  }
}

int pk_debug_set_attention_route(int route) {
  if (route < 0 || route > 3) return set_error(PK_E_INVALID, "route must be 0, 1, 2 or 3");
  g_attention_route = route;
  return PK_OK;
}

int pk_layernorm(pk_device* device, int precision, int64_t rows, int64_t channels, const void* x, const float* gamma,
                 const float* beta, float epsilon, void* y, pk_stream stream) {
  if (!device || !x || !gamma || !beta || !y) return set_error(PK_E_INVALID, "null argument");
  if (precision != PK_FP16 && precision != PK_FP32) return set_error(PK_E_INVALID, "unknown precision");
  if (rows <= 0 || channels <= 0 || channels % 4 != 0 || rows > (int64_t)1 << 31)
    return set_error(PK_E_SHAPE, "LayerNorm rows must be positive and channels a positive multiple of 4");
  cudaSetDevice(device->ctx.ordinal);
  return launch_layernorm(precision, rows, channels, x, gamma, beta, epsilon, y, as_stream(stream));
}

int pk_rel_attention(pk_device* device, int precision, int batch, int frames, const void* qkv, const void* positions,
                     const float* bias_u, const float* bias_v, const uint32_t* valid_lengths, void* context,
                     pk_stream stream) {
  if (!device || !qkv || !positions || !bias_u || !bias_v || !valid_lengths || !context)
    return set_error(PK_E_INVALID, "null argument");
  if (precision != PK_FP16 && precision != PK_FP32) return set_error(PK_E_INVALID, "unknown precision");
  if (batch <= 0 || frames <= 0 || frames > 192 || batch > 65535)
    return set_error(PK_E_SHAPE, "Unsupported attention shape (batch=%d, frames=%d; frames must be in [1, 192])",
                     batch, frames);
  cudaSetDevice(device->ctx.ordinal);
  return launch_rel_attention(device->ctx, precision, batch, frames, qkv, positions, bias_u, bias_v, valid_lengths,
                              context, as_stream(stream));
}

int pk_logmel(pk_device* device, int batch, int sample_count, const float* samples, const uint32_t* valid_samples,
              float* features, pk_stream stream) {
  if (!device || !samples || !valid_samples || !features) return set_error(PK_E_INVALID, "null argument");
  if (batch <= 0 || batch > 65535) return set_error(PK_E_SHAPE, "batchSize must be in [1, 65535]");
  if (sample_count < 160 || sample_count > 240000)
    return set_error(PK_E_SHAPE, "sampleCount must be in [160, 240000] (hop 160, at most 1501 frames)");
  cudaSetDevice(device->ctx.ordinal);
  return launch_logmel(batch, sample_count, samples, valid_samples, features, as_stream(stream));
}

int pk_tdt_decode(pk_device* device, const pk_tdt_desc* d, pk_stream stream) {
  if (!device || !d) return set_error(PK_E_INVALID, "null argument");
  if (d->precision != PK_FP16 && d->precision != PK_FP32) return set_error(PK_E_INVALID, "unknown precision");
  if (d->batch <= 0 || d->batch > 16383) return set_error(PK_E_SHAPE, "Invalid TDT decoder batchSize");
  if (d->frames <= 0 || d->frames > (1 << 20)) return set_error(PK_E_SHAPE, "Invalid TDT decoder frames");
  if (d->max_tokens <= 0 || (int64_t)d->max_tokens * d->batch > ((int64_t)1 << 31))
    return set_error(PK_E_SHAPE, "Invalid TDT decoder maxTokens");
  const void* ptrs[] = {d->encoder_projected, d->encoded_lengths, d->decode_starts, d->decode_ends,
                        d->flush_finals, d->embedding, d->lstm_weight0, d->lstm_bias0, d->lstm_weight1,
                        d->lstm_bias1, d->projector_weight, d->projector_bias, d->head_weight, d->head_bias,
                        d->tokens, d->token_frames, d->token_durations, d->metadata};
  for (const void* q : ptrs)
    if (!q) return set_error(PK_E_INVALID, "TDT decoder pointer is null");
  const void* aligned16[] = {d->encoder_projected, d->embedding, d->lstm_weight0, d->lstm_weight1,
                             d->projector_weight, d->head_weight};
  for (const void* q : aligned16)
    if (reinterpret_cast<uintptr_t>(q) & 15)
      return set_error(PK_E_LAYOUT, "TDT decoder weights and encoder input must be 16-byte aligned");
  cudaSetDevice(device->ctx.ordinal);
  if (g_decoder_route != 1) {
    const int st = launch_tdt_resident(device->ctx, *d, as_stream(stream));
    if (st != PK_E_SHAPE || g_decoder_route == 2) return st;
  }
  return launch_tdt_decode(device->ctx, *d, as_stream(stream));
}

int pk_debug_set_decoder_route(int route) {
  if (route < 0 || route > 2) return set_error(PK_E_INVALID, "decoder route must be 0, 1 or 2");
  g_decoder_route = route;
  return PK_OK;
}

int pk_conformer_conv(pk_device* device, int precision, int batch, int frames, const void* pointwise,
                      const void* dw_weights, const float* bn_scale, const float* bn_shift,
                      const uint32_t* valid_lengths, void* out, pk_stream stream) {
  if (!device || !pointwise || !dw_weights || !bn_scale || !bn_shift || !valid_lengths || !out)
    return set_error(PK_E_INVALID, "null argument");
  if (precision != PK_FP16 && precision != PK_FP32) return set_error(PK_E_INVALID, "unknown precision");
  if (batch <= 0 || frames <= 0 || batch > 65535 || frames > (1 << 20))
    return set_error(PK_E_SHAPE, "batchSize and frames must be positive integers");
  cudaSetDevice(device->ctx.ordinal);
  return launch_conformer_conv(precision, batch, frames, pointwise, dw_weights, bn_scale, bn_shift, valid_lengths,
                               out, as_stream(stream));
}

int pk_subsampling_conv0_dw2(pk_device* device, int precision, int batch, const float* features, const void* conv0_w,
                             const float* conv0_b, const void* dw_w, const float* dw_b,
                             const uint32_t* feature_lengths, void* out, pk_stream stream) {
  if (!device || !features || !conv0_w || !conv0_b || !dw_w || !dw_b || !feature_lengths || !out)
    return set_error(PK_E_INVALID, "null argument");
  if (precision != PK_FP16 && precision != PK_FP32) return set_error(PK_E_INVALID, "unknown precision");
  if (batch <= 0 || batch > 65535) return set_error(PK_E_SHAPE, "batch must be in [1, 65535]");
  cudaSetDevice(device->ctx.ordinal);
  return launch_subsampling_conv0_dw2(precision, batch, features, conv0_w, conv0_b, dw_w, dw_b, feature_lengths, out,
                                      as_stream(stream));
}

int pk_subsampling_depthwise(pk_device* device, int precision, int batch, int in_height, int in_width, int channels,
                             const void* input, const void* weights, const float* bias,
                             const uint32_t* feature_lengths, int steps, void* out, pk_stream stream) {
  if (!device || !input || !weights || !bias || !feature_lengths || !out)
    return set_error(PK_E_INVALID, "null argument");
  if (precision != PK_FP16 && precision != PK_FP32) return set_error(PK_E_INVALID, "unknown precision");
  if (batch <= 0 || in_height <= 0 || in_width <= 0 || channels <= 0 || steps < 1 || steps > 8)
    return set_error(PK_E_SHAPE, "invalid depthwise subsampling geometry");
  cudaSetDevice(device->ctx.ordinal);
  return launch_subsampling_depthwise(precision, batch, in_height, in_width, channels, input, weights, bias,
                                      feature_lengths, steps, out, as_stream(stream));
}

int pk_subsampling_time_mask(pk_device* device, int precision, int batch, int height, int width, int channels,
                             void* values, const uint32_t* feature_lengths, int steps, pk_stream stream) {
  if (!device || !values || !feature_lengths) return set_error(PK_E_INVALID, "null argument");
  if (precision != PK_FP16 && precision != PK_FP32) return set_error(PK_E_INVALID, "unknown precision");
  if (batch <= 0 || height <= 0 || width <= 0 || channels <= 0 || steps < 0 || steps > 8 || height > 65535 ||
      batch > 65535)
    return set_error(PK_E_SHAPE, "invalid time-mask geometry");
  cudaSetDevice(device->ctx.ordinal);
  return launch_subsampling_time_mask(precision, batch, height, width, channels, values, feature_lengths, steps,
                                      as_stream(stream));
}

}  // extern "C"
