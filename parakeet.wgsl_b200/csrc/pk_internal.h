// pk_internal.h -- host-side declarations shared by the libpk_b200 sources.
#pragma once

#include <cuda_runtime.h>
#include <cstdint>
#include <string>

#include "../../include/pk_b200.h"

namespace pk {

// Per-device context (the pk_device handle's payload).
struct DeviceCtx {
  int ordinal = 0;
  int sm_count = 148;
  int max_smem_optin = 0;
  unsigned int* status = nullptr;  // device word; kernels OR PK_STATUS_* bits into it
  void* encode_tiled = nullptr;    // cuTensorMapEncodeTiled
  void* tdt_exchange = nullptr;    // resident decoder's cross-CTA exchange area (kTdtExchangeBytes)
};

// Bytes of the resident TDT decoder's exchange area (hidden / projection
// vectors, argmax partials and the grid-barrier counter for up to 40 windows),
// allocated with the device handle.
constexpr size_t kTdtExchangeBytes = 12ull * 1024 * 1024;

// Thread-local error reporting.
int set_error(int code, const char* fmt, ...);
int cuda_error(cudaError_t err, const char* what);

// Launch with programmatic stream serialization: the kernel may be scheduled
// while the previous kernel of the stream finishes its last CTAs, and waits
// for it in pdl_entry() (pk_common.cuh) -- which every kernel of this
// library calls before touching shared buffers.  In a captured graph this
// becomes a programmatic dependency edge.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                                 Args... args) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

struct GemmArgs {
  int precision = PK_FP16;
  int64_t rows = 0, inner = 0, columns = 0;
  int bits = 5;
  int groups = 1;
  int64_t group_cols = 0;
  int act = PK_ACT_NONE;
  int has_residual = 0;
  float residual_scale = 1.0f;
  const float* bias = nullptr;
  const void* residual = nullptr;
  const void* a = nullptr;
  const uint32_t* codes = nullptr;
  const void* palette = nullptr;
  void* c = nullptr;
  // Optional time mask fused into the tensor-core epilogues: output row r
  // (frame f = (r / mask_group) % mask_frames of window (r / mask_group) /
  // mask_frames) is stored as zero when f >= mask_lengths[window].
  const uint32_t* mask_lengths = nullptr;
  int mask_group = 1, mask_frames = 1;
  bool* mask_applied = nullptr;  // set by the tensor-core launcher: whether the mask was fused
};

// Raises a kernel's dynamic shared-memory limit on the current device, once
// per (kernel, device) (returns pk_status).
int set_max_dynamic_smem(const void* kernel, int bytes);

// Validation shared by every GEMM entry point (returns pk_status).
int validate_gemm(const GemmArgs& g);

// Kernel launchers (return pk_status; errors recorded with set_error).
int launch_gemm_tc(const DeviceCtx& dev, const GemmArgs& g, cudaStream_t stream, int forced_bn = 0);
int launch_gemm_simt(const DeviceCtx& dev, const GemmArgs& g, cudaStream_t stream);
bool gemm_tc_supported(const GemmArgs& g);
int launch_palette_expand(const pk_palette_desc& d, cudaStream_t stream);
int launch_layernorm(int precision, int64_t rows, int64_t channels, const void* x, const float* gamma,
                     const float* beta, float eps, void* y, cudaStream_t stream);
// Two LayerNorms on 1024-wide rows: y1 = LN(x; g1, b1), y2 = LN(y1; g2, b2).
int launch_layernorm_dual(int precision, int64_t rows, const void* x, const float* g1, const float* b1,
                          const float* g2, const float* b2, float eps, void* y1, void* y2, cudaStream_t stream);
// positions_rowmajor (optional): the same positions re-laid out [8][2T-1][128]
// by launch_positions_rowmajor, used by the tensor-core kernel when given.
int launch_rel_attention(const DeviceCtx& dev, int precision, int batch, int frames, const void* qkv,
                         const void* positions, const float* bias_u, const float* bias_v,
                         const uint32_t* valid_lengths, void* context, cudaStream_t stream,
                         const void* positions_rowmajor = nullptr);
int launch_rel_attention_tc(int batch, int frames, const void* qkv, const void* positions, const float* bias_u,
                            const float* bias_v, const uint32_t* valid_lengths, void* context, cudaStream_t stream,
                            bool positions_rowmajor);
int launch_positions_rowmajor(const void* pkg, void* rm, int frames, cudaStream_t stream);
// tcgen05 attention (FP16, frames <= 192, positions row-major [8][2T-1][128]).
bool rel_attention_umma_supported(const DeviceCtx& dev, int frames, const void* qkv, const void* positions_rowmajor,
                                  const void* context);
int launch_rel_attention_umma(const DeviceCtx& dev, int batch, int frames, const void* qkv,
                              const void* positions_rowmajor, const float* bias_u, const float* bias_v,
                              const uint32_t* valid_lengths, void* context, cudaStream_t stream);
int launch_conformer_conv(int precision, int batch, int frames, const void* pointwise, const void* dw,
                          const float* scale, const float* shift, const uint32_t* valid_lengths, void* out,
                          cudaStream_t stream);
int launch_subsampling_conv0_dw2(int precision, int batch, const float* features, const void* conv0_w,
                                 const float* conv0_b, const void* dw_w, const float* dw_b,
                                 const uint32_t* feature_lengths, void* out, cudaStream_t stream);
int launch_subsampling_depthwise(int precision, int batch, int ih, int iw, int channels, const void* input,
                                 const void* w, const float* b, const uint32_t* feature_lengths, int steps,
                                 void* out, cudaStream_t stream);
int launch_subsampling_time_mask(int precision, int batch, int height, int width, int channels, void* values,
                                 const uint32_t* feature_lengths, int steps, cudaStream_t stream);

int launch_tdt_decode(const DeviceCtx& dev, const pk_tdt_desc& d, cudaStream_t stream);
// Resident FP16 decoder (all windows in lockstep on 128 co-resident CTAs);
// returns PK_E_SHAPE when it does not apply (then the cluster kernel runs).
int launch_tdt_resident(const DeviceCtx& dev, const pk_tdt_desc& d, cudaStream_t stream);
// Test knob: 0 = automatic, 1 = cluster kernel only, 2 = resident kernel only.
extern int g_decoder_route;
int launch_logmel(int batch, int sample_count, const float* samples, const uint32_t* valid_samples, float* features,
                  cudaStream_t stream);

// Debug / test knob: 0 = automatic kernel choice, 1 = force the SIMT GEMM,
// 2 = force the tensor-core GEMM (fails if the shape is unsupported), 3/4 =
// tensor cores with single-CTA / CTA-pair tiles, 5 = the SIMT GEMM with FP16
// accumulating in f16 (the reference's algorithm, for parity runs).
extern int g_gemm_route;
// Parity knob (pk_debug_set_reference_arithmetic): FP16 operators replay the
// reference shaders' arithmetic on the CUDA cores (reference_arith.cu).
extern int g_reference_arith;
inline bool gemm_route_simt() { return g_gemm_route == 1 || g_gemm_route == 5 || g_reference_arith; }
inline bool gemm_acc16() { return g_gemm_route == 5 || g_reference_arith; }
int launch_ref_layernorm(int64_t rows, int64_t channels, const void* x, const float* gamma, const float* beta,
                         float eps, void* y, cudaStream_t stream);
int launch_ref_attention(int batch, int frames, const void* qkv, const void* positions, const float* bias_u,
                         const float* bias_v, const uint32_t* valid_lengths, void* context, cudaStream_t stream);
int launch_ref_conformer_conv(int batch, int frames, const void* pointwise, const void* dw, const float* scale,
                              const float* shift, const uint32_t* valid_lengths, void* out, cudaStream_t stream);
int launch_ref_conv0_dw2(int batch, const float* features, const void* conv0_w, const float* conv0_b,
                         const void* dw_w, const float* dw_b, const uint32_t* feature_lengths, void* out,
                         cudaStream_t stream);
int launch_ref_depthwise(int batch, int ih, int iw, int channels, const void* input, const void* w, const float* b,
                         const uint32_t* feature_lengths, int steps, void* out, cudaStream_t stream);
extern int g_gemm_tile;
// Debug / test knob: 0 = automatic (FP16: the tcgen05 kernel when row-major
// positions are at hand, else the mma.sync kernel), 1 = CUDA-core attention,
// 2 = the mma.sync kernel, 3 = the tcgen05 kernel with `positions` already
// row-major [8][2T-1][128].
extern int g_attention_route;

}  // namespace pk

// Payload of the opaque pk_device handle.
struct pk_device {
  pk::DeviceCtx ctx;
  bool closed = false;
};
