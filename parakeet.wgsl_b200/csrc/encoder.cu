// encoder.cu -- model package residency and the fixed-shape encoder graph.
//
// pk_weights mirrors ParakeetGpuPackage (src/model/package.ts:45-52): named
// tensors with dtype, logical shape and layout, resident on one device.
// pk_encoder mirrors ParakeetEncoderGraph (src/webgpu/encoder.ts:1299-1862):
//   subsampling (encoder.ts:2140-2430) -> 24 Macaron Conformer layers, each
//   the 15 logical dispatches of createEncoderLayerDispatches
//   (encoder.ts:1869-2138) over two rotating [B*188, 1024] slots
//   (planEncoderLayerArena, encoder.ts:538-565) -> projector 1024 -> 640 +
//   bias (encoder.ts:1489-1509).
// The reference submits 26 command buffers and drains the queue between them
// (webgpu-engine.ts:970-1000); here the whole device-side forward for a given
// active batch is captured once into a CUDA graph and replayed.  Palette
// weights stay packed in HBM (15.2 MB per layer); every GEMM decodes on chip.
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "pk_internal.h"

namespace {

struct DevTensor {
  int dtype = 0;
  std::vector<int64_t> shape;
  std::string layout;
  void* ptr = nullptr;
  size_t bytes = 0;
};

constexpr int kFeatureBins = 128;
constexpr int kFeatureFrames = 1501;
constexpr int kFrames = 188;
constexpr int kHidden = 1024;
constexpr int kProjected = 640;
constexpr int kLayers = 24;
constexpr int kBatchCapacity = 40;  // PARAKEET_ENCODER_BATCH_CAPACITY (encoder.ts:68)

int sub_len(int raw, int steps) {
  for (int s = 0; s < steps; ++s) raw = (raw + 1) / 2;
  return raw;
}

}  // namespace

struct pk_weights {
  pk_device* device = nullptr;
  std::unordered_map<std::string, DevTensor> tensors;
  void* block = nullptr;
};

struct MatrixRef {
  const uint32_t* codes = nullptr;
  const void* palette = nullptr;
  int bits = 5, groups = 1;
  int64_t inner = 0, columns = 0;
};

struct LayerRefs {
  const float *ln_ff1_w, *ln_ff1_b, *ln_att_w, *ln_att_b, *ln_conv_w, *ln_conv_b, *ln_ff2_w, *ln_ff2_b, *ln_out_w,
      *ln_out_b;
  MatrixRef ff1_l1, ff1_l2, qkv, o_proj, pw1, pw2, ff2_l1, ff2_l2;
  const void* positions;
  const void* positions_rm = nullptr;  // FP16: [8][375][128] copy for the tensor-core attention
  const float *bias_u, *bias_v;
  const void* dw;
  const float *bn_scale, *bn_shift;
};

struct pk_encoder {
  pk_device* device = nullptr;
  pk_weights* weights = nullptr;
  int precision = PK_FP16;
  int capacity = 0;
  size_t scalar = 2;
  // arena
  float* features = nullptr;
  uint32_t* feature_lengths = nullptr;
  uint32_t* encoder_lengths = nullptr;
  // Pinned staging of the per-batch lengths: a ring of kLengthSlots buffers of
  // [2 * capacity], each reused only after the event recorded behind its
  // uploads has completed, so a caller may queue the next batch before the
  // previous one has started on the GPU.
  static constexpr int kLengthSlots = 4;
  uint32_t* host_lengths = nullptr;  // pinned [kLengthSlots][2 * capacity]
  cudaEvent_t length_uploaded[kLengthSlots] = {};
  int length_slot = 0;
  void* slots[2] = {nullptr, nullptr};
  void* big = nullptr;       // [cap*188, 4096]
  void* projected = nullptr; // [cap*188, 640]
  void* s376 = nullptr;      // [cap, 376, 32, 256]
  void* p376 = nullptr;
  void* s188 = nullptr;      // [cap, 188, 16, 256]
  void* p188 = nullptr;
  void* positions_rm = nullptr;  // FP16: every layer's positions, row-major per head
  std::vector<void*> checkpoints;  // optional per-layer outputs
  bool keep_checkpoints = false;
  // model references
  std::vector<LayerRefs> layers;
  const void *conv0_w, *dw2_w, *dw5_w;
  const float *conv0_b, *dw2_b, *pw3_b, *dw5_b, *pw6_b, *flat_b, *proj_b;
  MatrixRef pw3, pw6, flat, proj;
  int final_slot = 0;
  std::map<int, cudaGraphExec_t> graphs;
  cudaStream_t capture_stream = nullptr;
};

using namespace pk;

namespace {

int lookup(pk_weights* w, const std::string& name, DevTensor** out) {
  auto it = w->tensors.find(name);
  if (it == w->tensors.end()) return set_error(PK_E_NOT_FOUND, "Missing model tensor %s", name.c_str());
  *out = &it->second;
  return PK_OK;
}

int require(pk_weights* w, const std::string& name, int dtype, std::vector<int64_t> shape, const char* layout,
            const void** ptr) {
  DevTensor* t;
  int st = lookup(w, name, &t);
  if (st) return st;
  if (t->dtype != dtype || t->shape != shape || (layout && t->layout != layout))
    return set_error(PK_E_LAYOUT, "%s has an unexpected dtype/shape/layout (%s)", name.c_str(), t->layout.c_str());
  *ptr = t->ptr;
  return PK_OK;
}

int require_f32(pk_weights* w, const std::string& name, int64_t n, const char* layout, const float** ptr) {
  const void* p;
  int st = require(w, name, PK_DTYPE_F32, {n}, layout, &p);
  *ptr = static_cast<const float*>(p);
  return st;
}

// matrixTensor (src/webgpu/encoder.ts:2458-2512): packed codes with layout
// k-by-output-row-major-palette{5,6}-lsb-u32 and a [G, 2^bits] palette in the
// profile scalar with layout output-group-by-palette-lut.
int require_matrix(pk_weights* w, const std::string& name, int64_t inner, int64_t columns, int precision,
                   MatrixRef* m) {
  DevTensor* t;
  int st = lookup(w, name, &t);
  if (st) return st;
  int bits = 0;
  if (t->layout == "k-by-output-row-major-palette5-lsb-u32") bits = 5;
  else if (t->layout == "k-by-output-row-major-palette6-lsb-u32") bits = 6;
  else return set_error(PK_E_LAYOUT, "%s has an unsupported weight format %s", name.c_str(), t->layout.c_str());
  const int cpg = bits == 5 ? 32 : 16, wpg = bits == 5 ? 5 : 3;
  if (t->dtype != PK_DTYPE_U32 || t->shape != std::vector<int64_t>{inner, columns} ||
      t->bytes != (size_t)(inner * columns / cpg * wpg * 4))
    return set_error(PK_E_LAYOUT, "%s has invalid packed palette indices", name.c_str());
  DevTensor* p;
  if ((st = lookup(w, name + ".palette", &p))) return st;
  const int pdtype = precision == PK_FP16 ? PK_DTYPE_F16 : PK_DTYPE_F32;
  if (p->dtype != pdtype || p->shape.size() != 2 || p->shape[1] != (1 << bits) ||
      p->layout != "output-group-by-palette-lut" || p->shape[0] <= 0 || columns % p->shape[0] != 0)
    return set_error(PK_E_LAYOUT, "%s.palette has invalid palette storage", name.c_str());
  m->codes = static_cast<const uint32_t*>(t->ptr);
  m->palette = p->ptr;
  m->bits = bits;
  m->groups = (int)p->shape[0];
  m->inner = inner;
  m->columns = columns;
  return PK_OK;
}

// `mask`: the subsampling time mask (rows of mask_group outputs per frame,
// 188 frames per window, encoder lengths on the device), fused into the
// single-CTA tensor-core epilogue when that kernel runs; *masked says whether
// it was, else the caller masks.
int gemm(pk_encoder* e, const MatrixRef& m, int64_t rows, const void* a, void* c, int act, const float* bias,
         const void* residual, float res_scale, cudaStream_t s, const uint32_t* mask = nullptr, int mask_group = 1,
         bool* masked = nullptr) {
  GemmArgs g;
  g.precision = e->precision;
  g.rows = rows;
  g.inner = m.inner;
  g.columns = m.columns;
  g.bits = m.bits;
  g.groups = m.groups;
  g.group_cols = m.columns / m.groups;
  g.act = act;
  g.has_residual = residual != nullptr;
  g.residual_scale = res_scale;
  g.bias = bias;
  g.residual = residual;
  g.a = a;
  g.codes = m.codes;
  g.palette = m.palette;
  g.c = c;
  int st = validate_gemm(g);
  if (st) return st;
  if (masked) *masked = false;
  if (gemm_tc_supported(g) && !gemm_route_simt()) {
    g.mask_lengths = mask;
    g.mask_group = mask_group;
    g.mask_frames = kFrames;
    g.mask_applied = masked;
    return launch_gemm_tc(e->device->ctx, g, s);
  }
  return launch_gemm_simt(e->device->ctx, g, s);
}

#define PK_TRY(x)              \
  do {                         \
    const int _st = (x);       \
    if (_st != PK_OK) return _st; \
  } while (0)

// Device-side forward for `batch` active windows (everything after the input
// uploads).  Records into stream `s` (a capturing stream when building the
// graph).
int record_forward(pk_encoder* e, int batch, cudaStream_t s) {
  const int prec = e->precision;
  const int64_t rows = (int64_t)batch * kFrames;
  // Subsampling front end (encoder.ts:2300-2419), whole batch at once.
  PK_TRY(launch_subsampling_conv0_dw2(prec, batch, e->features, e->conv0_w, e->conv0_b, e->dw2_w, e->dw2_b,
                                      e->feature_lengths, e->s376, s));
  PK_TRY(gemm(e, e->pw3, (int64_t)batch * 376 * 32, e->s376, e->p376, PK_ACT_RELU, e->pw3_b, nullptr, 1.0f, s));
  PK_TRY(launch_subsampling_depthwise(prec, batch, 376, 32, 256, e->p376, e->dw5_w, e->dw5_b, e->feature_lengths, 3,
                                      e->s188, s));
  // Frames past each window's encoder length are zeroed in the pointwise-6
  // epilogue (the tensor-core path), else by the separate mask kernel.
  bool masked = false;
  PK_TRY(gemm(e, e->pw6, (int64_t)batch * 188 * 16, e->s188, e->p188, PK_ACT_RELU, e->pw6_b, nullptr, 1.0f, s,
              e->encoder_lengths, 16, &masked));
  if (!masked) PK_TRY(launch_subsampling_time_mask(prec, batch, 188, 16, 256, e->p188, e->feature_lengths, 3, s));
  PK_TRY(gemm(e, e->flat, rows, e->p188, e->slots[0], PK_ACT_NONE, e->flat_b, nullptr, 1.0f, s));
  if (e->keep_checkpoints)
    PK_TRY(cuda_error(cudaMemcpyAsync(e->checkpoints[0], e->slots[0], rows * kHidden * e->scalar,
                                      cudaMemcpyDeviceToDevice, s),
                      "checkpoint copy"));
  // Conformer layers (encoder.ts:1869-2138).
  char* big = static_cast<char*>(e->big);
  void* ff = big;                                               // [rows, 4096]
  void* qkv = big;                                              // [rows, 3072]
  void* ctx = big + (size_t)rows * 3072 * e->scalar;            // [rows, 1024]
  void* pw = big;                                               // [rows, 2048]
  void* conv = big + (size_t)rows * 2048 * e->scalar;           // [rows, 1024]
  int in_slot = 0;
  for (int l = 0; l < kLayers; ++l) {
    const LayerRefs& L = e->layers[l];
    void* x = e->slots[in_slot];
    void* y = e->slots[in_slot ^ 1];  // alternate == postFeedForward1 == output slot
    void* scratch = x;               // moduleScratch aliases the input slot
    // norm_feed_forward1 of every layer after the first ran fused with the
    // previous layer's norm_out (below).
    if (l == 0) PK_TRY(launch_layernorm(prec, rows, kHidden, x, L.ln_ff1_w, L.ln_ff1_b, 1e-5f, y, s));
    PK_TRY(gemm(e, L.ff1_l1, rows, y, ff, PK_ACT_SILU, nullptr, nullptr, 1.0f, s));
    PK_TRY(gemm(e, L.ff1_l2, rows, ff, y, PK_ACT_NONE, nullptr, x, 0.5f, s));
    PK_TRY(launch_layernorm(prec, rows, kHidden, y, L.ln_att_w, L.ln_att_b, 1e-5f, scratch, s));
    PK_TRY(gemm(e, L.qkv, rows, scratch, qkv, PK_ACT_NONE, nullptr, nullptr, 1.0f, s));
    PK_TRY(launch_rel_attention(e->device->ctx, prec, batch, kFrames, qkv, L.positions, L.bias_u, L.bias_v,
                                e->encoder_lengths, ctx, s, L.positions_rm));
    PK_TRY(gemm(e, L.o_proj, rows, ctx, scratch, PK_ACT_NONE, nullptr, y, 1.0f, s));
    PK_TRY(launch_layernorm(prec, rows, kHidden, scratch, L.ln_conv_w, L.ln_conv_b, 1e-5f, y, s));
    PK_TRY(gemm(e, L.pw1, rows, y, pw, PK_ACT_NONE, nullptr, nullptr, 1.0f, s));
    PK_TRY(launch_conformer_conv(prec, batch, kFrames, pw, L.dw, L.bn_scale, L.bn_shift, e->encoder_lengths, conv, s));
    PK_TRY(gemm(e, L.pw2, rows, conv, y, PK_ACT_NONE, nullptr, scratch, 1.0f, s));
    PK_TRY(launch_layernorm(prec, rows, kHidden, y, L.ln_ff2_w, L.ln_ff2_b, 1e-5f, scratch, s));
    PK_TRY(gemm(e, L.ff2_l1, rows, scratch, ff, PK_ACT_SILU, nullptr, nullptr, 1.0f, s));
    PK_TRY(gemm(e, L.ff2_l2, rows, ff, scratch, PK_ACT_NONE, nullptr, y, 0.5f, s));
    if (l + 1 < kLayers) {
      // norm_out into y (the layer output), then the next layer's
      // norm_feed_forward1 of it into the next layer's alternate slot, which
      // is this layer's scratch slot (read by the same warp first).
      const LayerRefs& N = e->layers[l + 1];
      PK_TRY(launch_layernorm_dual(prec, rows, scratch, L.ln_out_w, L.ln_out_b, N.ln_ff1_w, N.ln_ff1_b, 1e-5f, y,
                                   scratch, s));
    } else {
      PK_TRY(launch_layernorm(prec, rows, kHidden, scratch, L.ln_out_w, L.ln_out_b, 1e-5f, y, s));
    }
    in_slot ^= 1;
    if (e->keep_checkpoints)
      PK_TRY(cuda_error(cudaMemcpyAsync(e->checkpoints[l + 1], y, rows * kHidden * e->scalar,
                                        cudaMemcpyDeviceToDevice, s),
                        "checkpoint copy"));
  }
  e->final_slot = in_slot;
  PK_TRY(gemm(e, e->proj, rows, e->slots[in_slot], e->projected, PK_ACT_NONE, e->proj_b, nullptr, 1.0f, s));
  return PK_OK;
}

void free_encoder(pk_encoder* e) {
  for (auto& kv : e->graphs) cudaGraphExecDestroy(kv.second);
  e->graphs.clear();
  void* bufs[] = {e->features, e->feature_lengths, e->encoder_lengths, e->slots[0], e->slots[1], e->big,
                  e->projected, e->s376, e->p376, e->s188, e->p188, e->positions_rm};
  for (void* b : bufs)
    if (b) cudaFree(b);
  for (void* b : e->checkpoints)
    if (b) cudaFree(b);
  if (e->host_lengths) cudaFreeHost(e->host_lengths);
  for (cudaEvent_t ev : e->length_uploaded)
    if (ev) cudaEventDestroy(ev);
  if (e->capture_stream) cudaStreamDestroy(e->capture_stream);
}

}  // namespace

extern "C" {

int pk_weights_upload(pk_device* device, const pk_tensor_desc* tensors, int count, pk_weights** out) {
  if (!device || !out || (count > 0 && !tensors)) return set_error(PK_E_INVALID, "null argument");
  *out = nullptr;
  cudaSetDevice(device->ctx.ordinal);
  size_t total = 0;
  for (int i = 0; i < count; ++i) {
    const pk_tensor_desc& t = tensors[i];
    if (!t.name || !t.data || t.ndim < 1 || t.ndim > 4 || t.dtype < PK_DTYPE_F16 || t.dtype > PK_DTYPE_U32)
      return set_error(PK_E_INVALID, "tensor %d has an invalid descriptor", i);
    int64_t elems = 1;
    for (int d = 0; d < t.ndim; ++d) elems *= t.shape[d];
    const size_t esize = t.dtype == PK_DTYPE_F16 ? 2 : 4;
    const bool packed = t.dtype == PK_DTYPE_U32 && t.layout && std::strstr(t.layout, "palette");
    if (!packed && (size_t)elems * esize != t.bytes)
      return set_error(PK_E_LAYOUT, "%s byte length %zu does not match its shape", t.name, t.bytes);
    total += (t.bytes + 255) / 256 * 256;  // RUNTIME_STORAGE_ALIGNMENT (runtime-plan.ts:10)
  }
  auto* w = new pk_weights();
  w->device = device;
  cudaError_t e = cudaMalloc(&w->block, total ? total : 256);
  if (e != cudaSuccess) {
    delete w;
    return cuda_error(e, "cudaMalloc(weights)");
  }
  size_t off = 0;
  for (int i = 0; i < count; ++i) {
    const pk_tensor_desc& t = tensors[i];
    DevTensor d;
    d.dtype = t.dtype;
    d.shape.assign(t.shape, t.shape + t.ndim);
    d.layout = t.layout ? t.layout : "";
    d.ptr = static_cast<char*>(w->block) + off;
    d.bytes = t.bytes;
    e = cudaMemcpy(d.ptr, t.data, t.bytes, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
      cudaFree(w->block);
      delete w;
      return cuda_error(e, "cudaMemcpy(weights)");
    }
    off += (t.bytes + 255) / 256 * 256;
    w->tensors[t.name] = d;
  }
  *out = w;
  return PK_OK;
}

int pk_weights_release(pk_weights* weights) {
  if (!weights) return PK_OK;
  cudaSetDevice(weights->device->ctx.ordinal);
  cudaFree(weights->block);
  delete weights;
  return PK_OK;
}

int pk_encoder_create(pk_device* device, pk_weights* weights, int precision, int batch_capacity, pk_encoder** out) {
  if (!device || !weights || !out) return set_error(PK_E_INVALID, "null argument");
  *out = nullptr;
  if (precision != PK_FP16 && precision != PK_FP32) return set_error(PK_E_INVALID, "unknown precision");
  if (batch_capacity <= 0 || batch_capacity > kBatchCapacity)
    return set_error(PK_E_SHAPE, "Encoder batch capacity must be in [1, %d]", kBatchCapacity);
  cudaSetDevice(device->ctx.ordinal);
  std::unique_ptr<pk_encoder> e(new pk_encoder());
  e->device = device;
  e->weights = weights;
  e->precision = precision;
  e->capacity = batch_capacity;
  e->scalar = precision == PK_FP16 ? 2 : 4;
  const int sdt = precision == PK_FP16 ? PK_DTYPE_F16 : PK_DTYPE_F32;
  pk_weights* w = weights;
  // Model tensors, validated like requiredTensor / matrixTensor / channelTensor.
  const void* p;
  PK_TRY(require(w, "encoder.subsampling.layers.0.weight", sdt, {3, 3, 256}, "kh-kw-output-channel-vec4", &e->conv0_w));
  PK_TRY(require_f32(w, "encoder.subsampling.layers.0.bias", 256, "output-channel", &e->conv0_b));
  PK_TRY(require(w, "encoder.subsampling.layers.2.weight", sdt, {3, 3, 256}, "kh-kw-channel-vec4", &e->dw2_w));
  PK_TRY(require_f32(w, "encoder.subsampling.layers.2.bias", 256, "output-channel", &e->dw2_b));
  PK_TRY(require_matrix(w, "encoder.subsampling.layers.3.weight", 256, 256, precision, &e->pw3));
  PK_TRY(require_f32(w, "encoder.subsampling.layers.3.bias", 256, "output-channel", &e->pw3_b));
  PK_TRY(require(w, "encoder.subsampling.layers.5.weight", sdt, {3, 3, 256}, "kh-kw-channel-vec4", &e->dw5_w));
  PK_TRY(require_f32(w, "encoder.subsampling.layers.5.bias", 256, "output-channel", &e->dw5_b));
  PK_TRY(require_matrix(w, "encoder.subsampling.layers.6.weight", 256, 256, precision, &e->pw6));
  PK_TRY(require_f32(w, "encoder.subsampling.layers.6.bias", 256, "output-channel", &e->pw6_b));
  PK_TRY(require_matrix(w, "encoder.subsampling.linear.weight", 4096, kHidden, precision, &e->flat));
  PK_TRY(require_f32(w, "encoder.subsampling.linear.bias", kHidden, "output-channel", &e->flat_b));
  PK_TRY(require_matrix(w, "encoder_projector.weight", kHidden, kProjected, precision, &e->proj));
  PK_TRY(require_f32(w, "encoder_projector.bias", kProjected, "output-channel", &e->proj_b));
  e->layers.resize(kLayers);
  for (int l = 0; l < kLayers; ++l) {
    const std::string pre = "encoder.layers." + std::to_string(l) + ".";
    LayerRefs& L = e->layers[l];
    PK_TRY(require_f32(w, pre + "norm_feed_forward1.weight", kHidden, "channel", &L.ln_ff1_w));
    PK_TRY(require_f32(w, pre + "norm_feed_forward1.bias", kHidden, "channel", &L.ln_ff1_b));
    PK_TRY(require_f32(w, pre + "norm_self_att.weight", kHidden, "channel", &L.ln_att_w));
    PK_TRY(require_f32(w, pre + "norm_self_att.bias", kHidden, "channel", &L.ln_att_b));
    PK_TRY(require_f32(w, pre + "norm_conv.weight", kHidden, "channel", &L.ln_conv_w));
    PK_TRY(require_f32(w, pre + "norm_conv.bias", kHidden, "channel", &L.ln_conv_b));
    PK_TRY(require_f32(w, pre + "norm_feed_forward2.weight", kHidden, "channel", &L.ln_ff2_w));
    PK_TRY(require_f32(w, pre + "norm_feed_forward2.bias", kHidden, "channel", &L.ln_ff2_b));
    PK_TRY(require_f32(w, pre + "norm_out.weight", kHidden, "channel", &L.ln_out_w));
    PK_TRY(require_f32(w, pre + "norm_out.bias", kHidden, "channel", &L.ln_out_b));
    PK_TRY(require_matrix(w, pre + "feed_forward1.linear1.weight", kHidden, 4096, precision, &L.ff1_l1));
    PK_TRY(require_matrix(w, pre + "feed_forward1.linear2.weight", 4096, kHidden, precision, &L.ff1_l2));
    PK_TRY(require_matrix(w, pre + "self_attn.qkv.weight", kHidden, 3 * kHidden, precision, &L.qkv));
    PK_TRY(require_matrix(w, pre + "self_attn.o_proj.weight", kHidden, kHidden, precision, &L.o_proj));
    PK_TRY(require_matrix(w, pre + "conv.pointwise_conv1.weight", kHidden, 2 * kHidden, precision, &L.pw1));
    PK_TRY(require_matrix(w, pre + "conv.pointwise_conv2.weight", kHidden, kHidden, precision, &L.pw2));
    PK_TRY(require_matrix(w, pre + "feed_forward2.linear1.weight", kHidden, 4096, precision, &L.ff2_l1));
    PK_TRY(require_matrix(w, pre + "feed_forward2.linear2.weight", 4096, kHidden, precision, &L.ff2_l2));
    PK_TRY(require(w, pre + "self_attn.projected_positions", sdt, {375, kHidden}, "head-vector-position-vec4",
                   &L.positions));
    PK_TRY(require(w, pre + "self_attn.bias_u", PK_DTYPE_F32, {8, 128}, "head-by-channel", &p));
    L.bias_u = static_cast<const float*>(p);
    PK_TRY(require(w, pre + "self_attn.bias_v", PK_DTYPE_F32, {8, 128}, "head-by-channel", &p));
    L.bias_v = static_cast<const float*>(p);
    PK_TRY(require(w, pre + "conv.depthwise_conv.weight", sdt, {9, kHidden}, "kernel-channel-vec4", &L.dw));
    PK_TRY(require_f32(w, pre + "conv.norm.scale", kHidden, "channel", &L.bn_scale));
    PK_TRY(require_f32(w, pre + "conv.norm.shift", kHidden, "channel", &L.bn_shift));
  }
  // Activation arena: the whole batch goes through subsampling at once (the
  // reference microbatches by 3 to fit browser buffer limits).
  const size_t cap = (size_t)batch_capacity, rows = cap * kFrames, sc = e->scalar;
  struct Alloc {
    void** ptr;
    size_t bytes;
  } allocs[] = {
      {reinterpret_cast<void**>(&e->features), cap * kFeatureBins * kFeatureFrames * sizeof(float)},
      {reinterpret_cast<void**>(&e->feature_lengths), cap * sizeof(uint32_t)},
      {reinterpret_cast<void**>(&e->encoder_lengths), cap * sizeof(uint32_t)},
      {&e->slots[0], rows * kHidden * sc},
      {&e->slots[1], rows * kHidden * sc},
      {&e->big, rows * 4096 * sc},
      {&e->projected, rows * kProjected * sc},
      {&e->s376, cap * 376 * 32 * 256 * sc},
      {&e->p376, cap * 376 * 32 * 256 * sc},
      {&e->s188, cap * 188 * 16 * 256 * sc},
      {&e->p188, cap * 188 * 16 * 256 * sc},
  };
  for (auto& a : allocs) {
    cudaError_t err = cudaMalloc(a.ptr, a.bytes);
    if (err != cudaSuccess) {
      free_encoder(e.get());
      return cuda_error(err, "cudaMalloc(encoder arena)");
    }
  }
  cudaError_t err = cudaMallocHost(&e->host_lengths, pk_encoder::kLengthSlots * 2 * cap * sizeof(uint32_t));
  for (int i = 0; i < pk_encoder::kLengthSlots && err == cudaSuccess; ++i)
    err = cudaEventCreateWithFlags(&e->length_uploaded[i], cudaEventDisableTiming);
  if (err == cudaSuccess) err = cudaStreamCreateWithFlags(&e->capture_stream, cudaStreamNonBlocking);
  if (err != cudaSuccess) {
    free_encoder(e.get());
    return cuda_error(err, "encoder host staging");
  }
  if (e->precision == PK_FP16) {
    // The tensor-core attention reads each head's positions as contiguous
    // 256-byte rows: re-lay the package's head-vector-position-vec4 tensors
    // out once ([8][375][128] per layer).
    const size_t per_layer = (size_t)8 * (2 * kFrames - 1) * 128 * sizeof(uint16_t);
    err = cudaMalloc(&e->positions_rm, per_layer * kLayers);
    for (int l = 0; l < kLayers && err == cudaSuccess; ++l) {
      void* dst = static_cast<char*>(e->positions_rm) + per_layer * l;
      if (launch_positions_rowmajor(e->layers[l].positions, dst, kFrames, e->capture_stream) != PK_OK) {
        free_encoder(e.get());
        return PK_E_CUDA;
      }
      e->layers[l].positions_rm = dst;
    }
    if (err == cudaSuccess) err = cudaStreamSynchronize(e->capture_stream);
    if (err != cudaSuccess) {
      free_encoder(e.get());
      return cuda_error(err, "encoder positions re-layout");
    }
  }
  *out = e.release();
  return PK_OK;
}

// Enables per-layer output capture (encodeDiagnosticB1Checkpoints analogue).
int pk_encoder_set_checkpoints(pk_encoder* e, int enable) {
  if (!e) return set_error(PK_E_INVALID, "null encoder");
  cudaSetDevice(e->device->ctx.ordinal);
  if (enable && e->checkpoints.empty()) {
    const size_t bytes = (size_t)e->capacity * kFrames * kHidden * e->scalar;
    for (int i = 0; i <= kLayers; ++i) {
      void* p = nullptr;
      cudaError_t err = cudaMalloc(&p, bytes);
      if (err != cudaSuccess) return cuda_error(err, "cudaMalloc(checkpoints)");
      e->checkpoints.push_back(p);
    }
  }
  if ((bool)enable != e->keep_checkpoints) {
    for (auto& kv : e->graphs) cudaGraphExecDestroy(kv.second);
    e->graphs.clear();
  }
  e->keep_checkpoints = enable != 0;
  return PK_OK;
}

int pk_encoder_forward(pk_encoder* e, const float* features, int features_on_device, const uint32_t* feature_lengths,
                       int batch, void* projected_out, int out_on_device, uint32_t* encoded_lengths,
                       pk_stream stream) {
  if (!e || !features || !feature_lengths || !projected_out) return set_error(PK_E_INVALID, "null argument");
  if (batch <= 0 || batch > e->capacity)
    return set_error(PK_E_SHAPE, "Encoder active batch must be in [1, %d]", e->capacity);
  for (int i = 0; i < batch; ++i)
    if (feature_lengths[i] < 1 || feature_lengths[i] > (uint32_t)kFeatureFrames)
      return set_error(PK_E_SHAPE, "Feature length %d must be in [1, %d]", i, kFeatureFrames);
  cudaSetDevice(e->device->ctx.ordinal);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // Lengths: raw feature frames and the derived three-times stride-2 encoder
  // lengths (deriveEncoderValidLengths, encoder.ts:441-479).
  const int slot = e->length_slot;
  e->length_slot = (slot + 1) % pk_encoder::kLengthSlots;
  PK_TRY(cuda_error(cudaEventSynchronize(e->length_uploaded[slot]), "length staging slot"));
  uint32_t* staged = e->host_lengths + (size_t)slot * 2 * e->capacity;
  for (int i = 0; i < batch; ++i) {
    staged[i] = feature_lengths[i];
    staged[e->capacity + i] = (uint32_t)sub_len((int)feature_lengths[i], 3);
  }
  if (encoded_lengths)
    for (int i = 0; i < batch; ++i) encoded_lengths[i] = staged[e->capacity + i];
  PK_TRY(cuda_error(cudaMemcpyAsync(e->feature_lengths, staged, batch * sizeof(uint32_t), cudaMemcpyHostToDevice, s),
                    "upload feature lengths"));
  PK_TRY(cuda_error(cudaMemcpyAsync(e->encoder_lengths, staged + e->capacity, batch * sizeof(uint32_t),
                                    cudaMemcpyHostToDevice, s),
                    "upload encoder lengths"));
  PK_TRY(cuda_error(cudaEventRecord(e->length_uploaded[slot], s), "record length upload"));
  const size_t feat_bytes = (size_t)batch * kFeatureBins * kFeatureFrames * sizeof(float);
  PK_TRY(cuda_error(cudaMemcpyAsync(e->features, features, feat_bytes,
                                    features_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, s),
                    "upload features"));
  auto it = e->graphs.find(batch);
  if (it == e->graphs.end()) {
    // Capture the device-side forward once per active batch size.
    cudaGraph_t graph;
    PK_TRY(cuda_error(cudaStreamBeginCapture(e->capture_stream, cudaStreamCaptureModeThreadLocal), "begin capture"));
    const int st = record_forward(e, batch, e->capture_stream);
    cudaError_t ce = cudaStreamEndCapture(e->capture_stream, &graph);
    if (st != PK_OK) {
      if (ce == cudaSuccess) cudaGraphDestroy(graph);
      return st;
    }
    PK_TRY(cuda_error(ce, "end capture"));
    cudaGraphExec_t exec;
    ce = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    PK_TRY(cuda_error(ce, "graph instantiate"));
    it = e->graphs.emplace(batch, exec).first;
  }
  PK_TRY(cuda_error(cudaGraphLaunch(it->second, s), "graph launch"));
  const size_t out_bytes = (size_t)batch * kFrames * kProjected * e->scalar;
  PK_TRY(cuda_error(cudaMemcpyAsync(projected_out, e->projected, out_bytes,
                                    out_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, s),
                    "download projected output"));
  if (!out_on_device) PK_TRY(cuda_error(cudaStreamSynchronize(s), "synchronize"));
  return PK_OK;
}

int pk_encoder_checkpoint(pk_encoder* e, int layer, void* out, pk_stream stream) {
  if (!e || !out) return set_error(PK_E_INVALID, "null argument");
  if (!e->keep_checkpoints) return set_error(PK_E_INVALID, "checkpoints are disabled (pk_encoder_set_checkpoints)");
  if (layer < -1 || layer >= kLayers) return set_error(PK_E_SHAPE, "layer must be in [-1, %d]", kLayers - 1);
  cudaSetDevice(e->device->ctx.ordinal);
  const size_t bytes = (size_t)e->capacity * kFrames * kHidden * e->scalar;
  return cuda_error(cudaMemcpyAsync(out, e->checkpoints[layer + 1], bytes, cudaMemcpyDeviceToDevice,
                                    static_cast<cudaStream_t>(stream)),
                    "checkpoint copy");
}

int pk_encoder_destroy(pk_encoder* e) {
  if (!e) return PK_OK;
  cudaSetDevice(e->device->ctx.ordinal);
  cudaDeviceSynchronize();
  free_encoder(e);
  delete e;
  return PK_OK;
}

}  // extern "C"
