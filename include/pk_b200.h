/*
 * pk_b200.h -- C ABI of libpk_b200.so, the B200 (sm_100a) engine for the
 * FastConformer encoder hot path of parakeet.wgsl.
 *
 * Every entry point returns a pk_status (0 = OK, negative = error) and records
 * a per-thread message readable with pk_last_error().  All pointers named
 * "device" are CUDA device pointers owned by the caller; streams are
 * cudaStream_t passed as void* (NULL = the legacy default stream).  Handles are
 * opaque.  No entry point takes or returns a framework type.
 *
 * Each declaration cites the reference interface it replaces
 * (narcotic-sh/parakeet.wgsl v1.0.1, path:line).
 */
#ifndef PK_B200_H
#define PK_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes.  The reference throws synchronous Error / RangeError from
 * createDispatch/encode (src/webgpu/kernels/gemm.ts:971-1161, :434-436); these
 * are their C equivalents. */
typedef enum pk_status {
  PK_OK = 0,
  PK_E_INVALID = -1,   /* null handle / argument out of range            */
  PK_E_SHAPE = -2,     /* RangeError: unsupported shape                  */
  PK_E_LAYOUT = -3,    /* Error: invalid packed palette / tensor layout  */
  PK_E_SIGNATURE = -4, /* Error: not a fixed production GEMM signature   */
  PK_E_CUDA = -5,      /* CUDA runtime error                             */
  PK_E_OOM = -6,       /* device allocation failed                       */
  PK_E_TIMEOUT = -7,   /* a bounded device wait expired                  */
  PK_E_DESTROYED = -8, /* handle used after destroy                      */
  PK_E_NOT_FOUND = -9  /* model tensor missing (ParakeetGpuPackage.tensor) */
} pk_status;

/* Execution precision: the reference's FP16 / FP32 packages
 * (src/webgpu/capabilities.ts, ParakeetExecutionProfile.precision). */
enum { PK_FP16 = 0, PK_FP32 = 1 };
/* GemmActivation (src/webgpu/kernels/gemm.ts:148). */
enum { PK_ACT_NONE = 0, PK_ACT_SILU = 1, PK_ACT_RELU = 2 };
/* Expanded palette target layouts (src/model/runtime-plan.ts:26-33):
 * k-by-output-row-major-{f16,f32} and n{256,128}-k32-tile-major-{f16,f32}. */
enum { PK_LAYOUT_ROW_MAJOR = 0, PK_LAYOUT_TILE_MAJOR = 1 };
/* Tensor element types (ParakeetTensorRecord.dtype). */
enum { PK_DTYPE_F16 = 0, PK_DTYPE_F32 = 1, PK_DTYPE_U32 = 2 };

typedef struct pk_device pk_device;
typedef struct pk_weights pk_weights;
typedef struct pk_encoder pk_encoder;
typedef void* pk_stream;

/* Copies the calling thread's last error message (NUL-terminated). */
int pk_last_error(char* buffer, size_t length);
int pk_version(void);

/* Opens CUDA device `ordinal`.  Replaces the WebGPU adapter/device request in
 * createRawWebGpuParakeetEngine (src/runtime/webgpu-engine.ts:1062-1120). */
int pk_device_open(int ordinal, pk_device** out);
int pk_device_close(pk_device* device);
/* Reads and clears the device status word (bits 0..5: a bounded wait inside a
 * kernel expired -- 0 TMA/mbarrier, 1 MMA, 2 decode, 3 epilogue, 4 unwind
 * drain, 5 grid barrier).  Replaces the uncapturederror listener / throwGpuError
 * (src/runtime/webgpu-engine.ts:274, :959).  Synchronizes the device. */
int pk_device_status(pk_device* device, uint32_t* status_bits);

/* ---------------------------------------------------------------- operators
 * Palette expansion, bit-exact with paletteDequantWgslForScalar
 * (src/model/palette-expander.ts:478-587) and the index map
 * runtimeGemmTileMajorScalarIndex (src/model/runtime-plan.ts:454-490).
 * Replaces PaletteWeightExpander.createPooledDispatch + encode
 * (src/model/palette-expander.ts:234-309). */
typedef struct pk_palette_desc {
  int precision;             /* PK_FP16 (f16 palette/target) or PK_FP32 */
  int bits;                  /* 5 or 6 */
  int64_t inner;             /* K */
  int64_t columns;           /* N */
  int palette_groups;        /* G: palette is [G, 2^bits] */
  int64_t palette_group_columns; /* N / G */
  int layout;                /* PK_LAYOUT_ROW_MAJOR or PK_LAYOUT_TILE_MAJOR */
  const uint32_t* codes;     /* device [K*N/codes_per_group, words_per_group] */
  const void* palette;       /* device [G, 2^bits] f16 or f32 */
  void* target;              /* device [K*N] f16 or f32 */
} pk_palette_desc;
int pk_palette_expand(pk_device* device, const pk_palette_desc* desc, pk_stream stream);

/* Fused palette-dequantizing GEMM: C = epilogue(A . W), W decoded from its
 * packed codes on chip (never written to HBM).  Mirrors GemmDescriptor
 * (src/webgpu/kernels/gemm.ts:358-373) and the epilogues
 * specializedBias/Activation/Residual (:2006-2044, :2847-2869); replaces
 * F16GemmKernel/F32GemmKernel.createDispatch + GemmDispatch.encode
 * (:483-855, :2974-3340, :400-470).  Bias and residual are exclusive. */
typedef struct pk_gemm_desc {
  int precision;             /* PK_FP16: A/C/residual f16, LUT f16; PK_FP32: all f32 */
  int64_t rows;              /* M (active rows) */
  int64_t inner;             /* K */
  int64_t columns;           /* N */
  int bits;                  /* 5 or 6 */
  int palette_groups;        /* G */
  int64_t palette_group_columns; /* N / G */
  int activation;            /* PK_ACT_* */
  int has_residual;          /* residual = residual + scale * value */
  float residual_scale;
  const float* bias;         /* device f32 [N] or NULL */
  const void* residual;      /* device [M, N] or NULL */
  const void* a;             /* device [M, K] */
  const uint32_t* codes;     /* device packed k-by-output-row-major codes */
  const void* palette;       /* device [G, 2^bits] */
  void* c;                   /* device [M, N] */
} pk_gemm_desc;
int pk_palette_gemm(pk_device* device, const pk_gemm_desc* desc, pk_stream stream);

/* LayerNorm over `channels` per row (src/webgpu/kernels/layernorm.ts:309-389);
 * replaces LayerNormKernel.createDispatch + encode (:73-240). */
int pk_layernorm(pk_device* device, int precision, int64_t rows, int64_t channels, const void* x,
                 const float* gamma, const float* beta, float epsilon, void* y, pk_stream stream);

/* Fused relative-position MHSA, 8 heads x 128 (src/webgpu/kernels/attention.ts:
 * 418-728); replaces RelativeAttentionKernel.createDispatch + encode
 * (:105-321).  qkv [B*T, 3072]; positions head-vector-position-vec4
 * [8][32][2T-1][4]; bias_u/v f32 [8,128]; valid_lengths u32 [B] (device);
 * context [B*T, 1024].  Requires 1 <= T <= 192. */
int pk_rel_attention(pk_device* device, int precision, int batch, int frames, const void* qkv,
                     const void* positions, const float* bias_u, const float* bias_v,
                     const uint32_t* valid_lengths, void* context, pk_stream stream);

/* Allocation-free FP16 relative-position attention.  No counterpart in the
 * reference: it exists for callers that may not allocate device memory (a
 * host with its own fixed device pool, a process under a scheduler-set memory
 * cap, a harness that must see every allocation up front), which cannot open a
 * pk_device either.  It takes no handle and runs on the calling thread's
 * current device.  Arguments mean what they mean for pk_rel_attention (package
 * position layout, 1 <= frames <= 192; qkv, positions and context 16-byte
 * aligned).  The positions are re-laid out into a fixed 784,640-byte scratch
 * array that the library holds on every GPU that loads it; no cudaMalloc,
 * cudaFree or allocating library call is made.  Calls whose GPU work overlaps
 * race on that array: serialise them.  The first call on a device resolves
 * the array's address; make it before any stream capture.  wait_status
 * (host, optional): when given, the call waits for the stream and stores the
 * kernel's status bits (0 = every bounded wait completed; non-zero returns
 * PK_E_TIMEOUT). */
int pk_rel_attention_noalloc(int batch, int frames, const void* qkv, const void* positions,
                             const float* bias_u, const float* bias_v, const uint32_t* valid_lengths,
                             void* context, uint32_t* wait_status, pk_stream stream);

/* Fused GLU + depthwise k9 + folded BN + SiLU (src/webgpu/kernels/
 * conformer-conv.ts:471-575); replaces FusedConformerConvKernel
 * (:174-351).  pointwise [B*T, 2048]; dw [9, 1024]; scale/shift f32 [1024];
 * out [B*T, 1024]. */
int pk_conformer_conv(pk_device* device, int precision, int batch, int frames, const void* pointwise,
                      const void* dw_weights, const float* bn_scale, const float* bn_shift,
                      const uint32_t* valid_lengths, void* out, pk_stream stream);

/* Subsampling kernels (src/webgpu/kernels/subsampling.ts): fused conv0 +
 * depthwise2 (:1092-1268; FusedSubsamplingConv0Depthwise2Kernel :620),
 * depthwise (:1270-1372; DepthwiseSubsamplingKernel :438) and time mask
 * (:1374-1425; SubsamplingTimeMaskKernel :250).  feature_lengths are the raw
 * feature-frame lengths (device u32 [B]). */
int pk_subsampling_conv0_dw2(pk_device* device, int precision, int batch, const float* features,
                             const void* conv0_w, const float* conv0_b, const void* dw_w,
                             const float* dw_b, const uint32_t* feature_lengths, void* out,
                             pk_stream stream);
int pk_subsampling_depthwise(pk_device* device, int precision, int batch, int in_height, int in_width,
                             int channels, const void* input, const void* weights, const float* bias,
                             const uint32_t* feature_lengths, int steps, void* out, pk_stream stream);
int pk_subsampling_time_mask(pk_device* device, int precision, int batch, int height, int width,
                             int channels, void* values, const uint32_t* feature_lengths, int steps,
                             pk_stream stream);

/* Log-mel front end: the reference's native front end, parakeet_fbank_
 * compute_item (src/cpp/fbank/parakeet_fbank.cpp:596-653; wrapper
 * ParakeetFbankWasm, src/audio/fbank-wasm.ts:158), for a whole batch at once.
 * samples: device f32 [batch, sample_count] (16 kHz PCM, the physical window
 * arena, 160 <= sample_count <= 240000); valid_samples: device u32 [batch]
 * (values above sample_count are treated as sample_count); features: device
 * f32 [batch, 128, sample_count / 160 + 1] feature-major, normalized over the
 * floor(valid / 160) valid frames and zero beyond them -- the encoder's input
 * layout.  The reference's raw-frame reuse between overlapping windows only
 * skips recomputing identical frames and has no counterpart.  The first call
 * on a device uploads constant tables; make it before any stream capture. */
int pk_logmel(pk_device* device, int batch, int sample_count, const float* samples,
              const uint32_t* valid_samples, float* features, pk_stream stream);

/* Persistent greedy TDT decoder (prediction net: 2-layer LSTM 640 + projector;
 * joint: relu(encoder + predictor) -> head 640 x 1032 = 1025 tokens (blank
 * 1024) + 5 durations {0..4}).  Mirrors TdtDecoderDescriptor (src/webgpu/
 * kernels/tdt-decoder.ts:54-82) with the decoder tensors of the package
 * (requireDecoderWeights, :367-420); replaces PersistentTdtDecoderKernel.create
 * + createDispatch + TdtDecoderDispatch.encode (:155-330, :84-149).  All
 * pointers are device pointers; weights and the encoder input are f16
 * (PK_FP16) or f32 (PK_FP32), biases f32; weight, embedding and encoder
 * pointers 16-byte aligned.  The decoder state lives on chip, so the
 * reference's state / predictorScratch arena slices have no counterpart.
 * The resident FP16 kernel exchanges vectors through one area owned by the
 * pk_device (each launch first rebuilds the layer-0 token table there from
 * the call's weights and resets the grid-barrier counter): decoder calls
 * on one pk_device must not overlap on the GPU -- issue them on one stream,
 * or open one pk_device per stream. */
typedef struct pk_tdt_desc {
  int precision;                      /* PK_FP16 or PK_FP32 */
  int batch;                          /* windows */
  int frames;                         /* encoder frames per window (stride of encoder_projected) */
  int max_tokens;                     /* output capacity per window */
  const void* encoder_projected;      /* [batch, frames, 640] (after encoder_projector) */
  const uint32_t* encoded_lengths;    /* u32 [batch] */
  const uint32_t* decode_starts;      /* u32 [batch]: first frame each decoder consumes */
  const uint32_t* decode_ends;        /* u32 [batch]: exclusive frame bound */
  const uint32_t* flush_finals;       /* u32 [batch]: nonzero runs the bounded end-of-stream flush */
  const void* embedding;              /* decoder.embedding.weight [1025, 640] */
  const void* lstm_weight0;           /* decoder.lstm.weight_l0 [1280, 2560] (input-hidden-k-by-ifgo) */
  const float* lstm_bias0;            /* decoder.lstm.bias_l0 [2560] */
  const void* lstm_weight1;           /* decoder.lstm.weight_l1 [1280, 2560] */
  const float* lstm_bias1;            /* decoder.lstm.bias_l1 [2560] */
  const void* projector_weight;       /* decoder.decoder_projector.weight [640, 640] (k-by-output) */
  const float* projector_bias;        /* decoder.decoder_projector.bias [640] */
  const void* head_weight;            /* joint.head.weight [640, 1032] (k-by-output, padded) */
  const float* head_bias;             /* joint.head.bias [1032] */
  uint32_t* tokens;                   /* u32 [batch, max_tokens] */
  uint32_t* token_frames;             /* u32 [batch, max_tokens]: encoder frame of each emission */
  uint32_t* token_durations;          /* u32 [batch, max_tokens] */
  uint32_t* metadata;                 /* u32 [2 * batch]: token counts, then status flags (1 = overflow) */
} pk_tdt_desc;
int pk_tdt_decode(pk_device* device, const pk_tdt_desc* desc, pk_stream stream);

/* ------------------------------------------------------------ model + graph
 * One named tensor of a weight package (ParakeetTensorRecord,
 * src/model/manifest.ts; runtime layouts src/model/runtime-plan.ts:26-37). */
typedef struct pk_tensor_desc {
  const char* name;          /* e.g. "encoder.layers.0.self_attn.qkv.weight" */
  int dtype;                 /* PK_DTYPE_* */
  int ndim;
  int64_t shape[4];          /* logical shape */
  const char* layout;        /* e.g. "k-by-output-row-major-palette5-lsb-u32" */
  const void* data;          /* host pointer */
  size_t bytes;
} pk_tensor_desc;
/* Uploads a package to the device.  Replaces ParakeetGpuPackage
 * (src/model/package.ts:45-52) plus the runtime plan (runtime-plan.ts:144-340). */
int pk_weights_upload(pk_device* device, const pk_tensor_desc* tensors, int count, pk_weights** out);
int pk_weights_release(pk_weights* weights);

/* Builds the fixed-shape 24-layer encoder graph for up to batch_capacity 15 s
 * windows (<= 40).  Replaces ParakeetEncoderGraph.create
 * (src/webgpu/encoder.ts:1299-1535). */
int pk_encoder_create(pk_device* device, pk_weights* weights, int precision, int batch_capacity,
                      pk_encoder** out);
/* Runs subsampling, 24 Conformer layers and the projector for `batch`
 * windows.  features: f32 [batch, 128, 1501] feature-major; feature_lengths:
 * host u32 [batch] in [1, 1501]; projected_out: [batch*188, 640] in the
 * profile scalar; encoded_lengths (host, optional): u32 [batch].
 * features_on_device / out_on_device select device or host buffers (host
 * buffers are copied inside the call).  Replaces encodeSubmissionChunks +
 * decoderInput (src/webgpu/encoder.ts:1711-1743, :1821). */
int pk_encoder_forward(pk_encoder* encoder, const float* features, int features_on_device,
                       const uint32_t* feature_lengths, int batch, void* projected_out, int out_on_device,
                       uint32_t* encoded_lengths, pk_stream stream);
/* Diagnostic per-layer capture, the analogue of encodeDiagnosticB1Checkpoints
 * (src/webgpu/encoder.ts:1751-1819, plan :621-688): after
 * pk_encoder_set_checkpoints(encoder, 1) every forward also keeps the
 * subsampling output and each layer's output; pk_encoder_checkpoint copies
 * the [capacity*188, 1024] buffer of `layer` (-1 = subsampling) into `out`
 * (device). */
int pk_encoder_set_checkpoints(pk_encoder* encoder, int enable);
int pk_encoder_checkpoint(pk_encoder* encoder, int layer, void* out, pk_stream stream);
int pk_encoder_destroy(pk_encoder* encoder);

/* ---- Overlap merge of decoded windows (host code; no GPU) ----------------
 * Replaces IncrementalStitchAccumulator (src/runtime/stitch.ts:135-213) for
 * token streams without word pieces: append / snapshot with the same merge
 * (mergeTokenStreams :247-359 -- disjoint, longest contiguous run, LCS,
 * midpoint), the same trace and enforceMonotonicTokenTimes (:230-262).
 * A token is int64[4] (token_id, start_sample, end_sample, duration_frames),
 * a trace entry int64[5] (left window index, right window index, method 0
 * disjoint / 1 contiguous / 2 lcs / 3 midpoint, overlap start and end
 * sample).  Errors: PK_E_INVALID with the reference's RangeError messages
 * (validateWindow, :715-775; out-of-order windows).  One accumulator must not
 * be used from two threads at once. */
typedef struct pk_stitch pk_stitch;
enum { PK_STITCH_COLLECT_TRACE = 1, PK_STITCH_RECORD_RUN = 2 };
int pk_stitch_create(int flags, pk_stitch** out);
int pk_stitch_destroy(pk_stitch* stitch);
/* window: int64[3] (index, start_sample, end_sample), the logical emission
 * range; tokens: int64[count][4] sorted by start_sample (append, :146-179). */
int pk_stitch_append(pk_stitch* stitch, const int64_t* window, const int64_t* tokens, int64_t count);
/* globalizeTdtTokens (stitch.ts:69-99) + append: window int64[4] (index,
 * emission start, emission end, timestamp offset sample); the decoder's
 * per-emission token ids, window-local encoder frames and durations. */
int pk_stitch_append_tdt(pk_stitch* stitch, const int64_t* window, const int32_t* token_ids,
                         const int32_t* frames, const int32_t* durations, int64_t count);
/* A contiguous run of windows merged on its own by an accumulator created with
 * PK_STITCH_RECORD_RUN (no reference counterpart: the reference merges on one
 * thread).  window_meta int64[windows][4] (index, start, end, token count),
 * window_tokens the windows' own tokens, merged the run's merged stream,
 * trace its internal trace; guard / local_ok from pk_stitch_read_run. */
typedef struct pk_stitch_run {
  const int64_t* window_meta;
  int64_t windows;
  const int64_t* window_tokens;
  const int64_t* merged;
  int64_t tokens;
  const int64_t* trace;
  int64_t trace_entries;
  int64_t guard;
  int local_ok;
} pk_stitch_run;
/* Appends a run: spliced in at its first seam when that is exact (an empty
 * stream, a one-window run, or the run's locality conditions hold and the
 * stream joined ends before the run's guard sample), otherwise window by
 * window.  Either way the result equals appending the run's windows. */
int pk_stitch_extend(pk_stitch* stitch, const pk_stitch_run* run);
/* counts: int64[4] = merged tokens, trace entries, recorded windows,
 * recorded window tokens. */
int pk_stitch_counts(const pk_stitch* stitch, int64_t* counts);
/* Copies the merged tokens (clamp != 0: snapshot's monotonic clamp) and the
 * trace; either pointer may be null. */
int pk_stitch_read(const pk_stitch* stitch, int clamp, int64_t* tokens, int64_t* trace);
/* The recorded run: window_meta int64[windows][4], window_tokens, and
 * conditions int64[2] = (guard sample, local_ok). */
int pk_stitch_read_run(const pk_stitch* stitch, int64_t* window_meta, int64_t* window_tokens, int64_t* conditions);

/* Test hook (no reference counterpart): selects the GEMM kernel for later
 * pk_palette_gemm / encoder launches in this process.  0 = automatic
 * (tensor cores where the shape tiles, else CUDA cores), 1 = CUDA-core
 * kernel only, 2 = tensor-core kernel only (unsupported shapes fail),
 * 3 = as 2 but single-CTA tiles only, 4 = as 2 but CTA-pair tiles
 * (cta_group::2) wherever N is a multiple of 256, 5 = CUDA-core kernel with
 * FP16 GEMMs accumulating in f16 in increasing K (each step an f32 fma
 * rounded to f16): the reference's own accumulation
 * (src/webgpu/kernels/gemm.ts:1445-1502), for parity runs only. */
int pk_debug_set_gemm_route(int route);
/* Test hook (no reference counterpart): while enabled, every FP16 operator --
 * GEMM, LayerNorm, attention, conformer conv, subsampling -- and the encoder
 * graphs recorded afterwards run CUDA-core kernels that replay the reference
 * shaders' arithmetic step by step: f16 accumulation in increasing K in the
 * GEMMs (gemm.ts:1445-1502), sequential f32 reductions (layernorm.ts:344-387,
 * attention.ts:485-727), the conv and subsampling fma chains
 * (conformer-conv.ts:505-574, subsampling.ts:1115-1372), every product and sum
 * rounded as written and exp taken as the correctly rounded f32 value.  For
 * parity runs against the CPU restatement; slow. */
int pk_debug_set_reference_arithmetic(int enable);
/* Test hook (no reference counterpart): forces the tensor-core GEMM token
 * tile for later launches in this process.  0 = automatic (cost model),
 * 128 / 192 / 256 = single-CTA tile, -256 / -384 / -512 = CTA-pair tile
 * (used where N is a multiple of 256, else the 256-token single-CTA tile). */
int pk_debug_set_gemm_tile(int tile);
/* Test hook (no reference counterpart): 0 = automatic (FP16: the tcgen05
 * attention where positions are held row-major -- the encoder -- else the
 * mma.sync tensor-core kernel), 1 = CUDA-core attention kernel, 2 = the
 * mma.sync kernel, 3 = the tcgen05 kernel reading `positions` of
 * pk_rel_attention as row-major [8][2T-1][128] instead of the package layout. */
int pk_debug_set_attention_route(int route);

/* Test hook (no reference counterpart): selects the TDT decoder kernel for
 * later pk_tdt_decode calls in this process.  0 = automatic (the resident
 * kernel -- FP16, at most 40 windows, weights held across 128 co-resident
 * CTAs -- where it applies, else the cluster-per-window kernel), 1 = the
 * cluster kernel only, 2 = the resident kernel only (PK_E_SHAPE where it does
 * not apply). */
int pk_debug_set_decoder_route(int route);

/* Test hook (no reference counterpart; the reference's device-loss path is the
 * uncapturederror listener, src/runtime/webgpu-engine.ts:274): makes one of
 * the library's bounded device waits run out, with a limit of `limit_ms`
 * (1..2000) instead of the 4 s production limit, and synchronizes `stream`.
 * kind 0: an mbarrier wait whose producer arrives (completes; no status bit);
 * 1: an mbarrier wait that nothing completes (status bit 0);
 * 2: a grid barrier of a two-CTA cooperative launch that both CTAs reach;
 * 3: the same barrier with one CTA returning before it (status bit 5).
 * Returns PK_OK once the probe kernel has finished; a wait that ran out shows
 * up as PK_E_TIMEOUT from the next pk_device_status, as in production.  The
 * probe traps, faults and hangs nothing: the context stays usable. */
int pk_debug_wait_probe(pk_device* device, int kind, uint32_t limit_ms, pk_stream stream);

#ifdef __cplusplus
}
#endif
#endif /* PK_B200_H */
