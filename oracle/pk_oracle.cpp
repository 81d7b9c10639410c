// pk_oracle.cpp -- CPU restatement of parakeet.wgsl's encoder shader math.
//
// TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA library in
// parakeet.wgsl_b200/csrc; it is never linked into, loaded by or called from the
// product path.  Only tests/, __graft_entry__.smoke() and bench.py's CPU
// baseline legs may load it.
//
// Every function restates the arithmetic of one WGSL shader emitted by the
// reference (narcotic-sh/parakeet.wgsl v1.0.1); the citation beside each one is
// the reference file:line it follows.  Pinning:
//   * palette bit packing / expansion and the tile-major index map are pinned
//     bit-exactly against the reference's own known-answer tests
//     (model/tests/test_convert.py:447-511, test/model/palette-expander.test.ts:
//     147-247) through the fixtures in tests/golden/;
//   * GEMM, LayerNorm, attention, conformer-conv and subsampling numerics are
//     PARITY UNPINNED: the reference's tests pin shader text, not outputs, and
//     its WGSL cannot execute without a browser WebGPU stack.
//
// Precision modes (argument `acc_mode` of the GEMM):
//   0 = reference algorithm: FP16 packages accumulate in f16 in increasing-K
//       order (gemm.ts:1445-1502); each f16 FMA is emulated as an f32 fmaf
//       followed by rounding to f16 (a double rounding that differs from a
//       fused f16 FMA in rare midpoint cases; WGSL leaves f16 fma fusion to the
//       backend anyway).  FP32 packages use an fp32 fmaf chain in increasing K
//       (gemm.ts:2396-2436).
//   1 = wide: f32 accumulation for both packages (what the tensor-core path
//       computes), used to bound the GPU's error tightly.
// Compiled with -ffp-contract=off so every a*b+c below is written as either an
// explicit fmaf or two rounded operations, exactly as stated.

#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>
#include <algorithm>

typedef _Float16 half_t;

static inline float h2f(uint16_t bits) {
  half_t h;
  std::memcpy(&h, &bits, 2);
  return (float)h;
}
static inline uint16_t f2h(float v) {
  half_t h = (half_t)v;  // round-to-nearest-even
  uint16_t bits;
  std::memcpy(&bits, &h, 2);
  return bits;
}
static inline float round_h(float v) { return (float)(half_t)v; }

// Load element i of a profile-scalar buffer (prec 0 = f16 bits, 1 = f32).
static inline float ld(const void* p, int prec, size_t i) {
  return prec == 0 ? h2f(((const uint16_t*)p)[i]) : ((const float*)p)[i];
}
static inline void st(void* p, int prec, size_t i, float v) {
  if (prec == 0) ((uint16_t*)p)[i] = f2h(v);
  else ((float*)p)[i] = v;
}

extern "C" {

int or_version(void) { return 1; }

// ---------------------------------------------------------------------------
// Palette codes.
// One code group = 32 (5-bit) or 16 (6-bit) consecutive scalars of the
// k-by-output row-major [K, N] matrix, packed LSB-first into 5 or 3 u32 words
// (model/convert.py:2130-2157).  Code i occupies bits [i*b, i*b+b) of the
// group's little-endian bit stream and may straddle two words
// (src/model/palette-expander.ts:500-511).
// ---------------------------------------------------------------------------
static inline uint32_t code_at(const uint32_t* words, int bits, int i) {
  const int bit = i * bits;
  const int w = bit >> 5, s = bit & 31;
  uint64_t v = words[w];
  if (s + bits > 32) v |= (uint64_t)words[w + 1] << 32;
  return (uint32_t)(v >> s) & ((1u << bits) - 1u);
}

// Unpack the raw code of every scalar of a [K, N] matrix (test helper).
void or_unpack_codes(const uint32_t* packed, int bits, int64_t scalars, uint8_t* codes) {
  const int per = bits == 5 ? 32 : 16, words = bits == 5 ? 5 : 3;
  for (int64_t g = 0; g < scalars / per; ++g)
    for (int i = 0; i < per; ++i) codes[g * per + i] = (uint8_t)code_at(packed + g * words, bits, i);
}

// Pack codes LSB-first (restates model/convert.py:2130-2157).
void or_pack_codes(const uint8_t* codes, int bits, int64_t scalars, uint32_t* packed) {
  const int per = bits == 5 ? 32 : 16, words = bits == 5 ? 5 : 3;
  std::memset(packed, 0, sizeof(uint32_t) * (size_t)(scalars / per) * words);
  for (int64_t g = 0; g < scalars / per; ++g) {
    uint32_t* out = packed + g * words;
    for (int i = 0; i < per; ++i) {
      const uint32_t c = codes[g * per + i];
      const int bit = i * bits, w = bit >> 5, s = bit & 31;
      out[w] |= c << s;
      if (s + bits > 32) out[w + 1] |= c >> (32 - s);
    }
  }
}

// runtimeGemmTileMajorScalarIndexForColumns (src/model/runtime-plan.ts:454-490):
// ((n_tile * k_tiles + k_tile) * 32 + k % 32) * T + n % T.
int64_t or_tile_major_index(int64_t scalar, int64_t inner, int64_t columns, int64_t tile_cols) {
  const int64_t k = scalar / columns, n = scalar % columns;
  const int64_t n_tile = n / tile_cols, k_tile = k / 32, k_tiles = inner / 32;
  return ((n_tile * k_tiles + k_tile) * 32 + k % 32) * tile_cols + n % tile_cols;
}

// paletteDequantWgslForScalar (src/model/palette-expander.ts:478-587).
// palette group of a code group = min(col / group_cols, groups - 1) evaluated
// at the group's first scalar (:543-549, :581-582).  layout 0 = row-major
// target, 1 = tile-major target with T = 256 (f16) or 128 (f32).
void or_palette_expand(const uint32_t* codes, const void* palette, int prec, int bits,
                       int64_t inner, int64_t columns, int groups, int64_t group_cols,
                       int layout, void* target) {
  const int per = bits == 5 ? 32 : 16, words = bits == 5 ? 5 : 3;
  const int entries = 1 << bits;
  const int64_t scalars = inner * columns;
  const int64_t tile_cols = prec == 0 ? 256 : 128;
#pragma omp parallel for schedule(static)
  for (int64_t g = 0; g < scalars / per; ++g) {
    const int64_t base = g * per;
    const int64_t col = base % columns;
    const int64_t pg = std::min<int64_t>(col / group_cols, groups - 1);
    for (int i = 0; i < per; ++i) {
      const uint32_t c = code_at(codes + g * words, bits, i);
      const int64_t dst = layout == 0 ? base + i : or_tile_major_index(base + i, inner, columns, tile_cols);
      const size_t src = (size_t)(pg * entries + c);
      if (prec == 0) ((uint16_t*)target)[dst] = ((const uint16_t*)palette)[src];
      else ((float*)target)[dst] = ((const float*)palette)[src];
    }
  }
}

// ---------------------------------------------------------------------------
// Palette GEMM: C = epilogue(A . W) with W expanded from its palette.
// f16 package: f16SubgroupGemmWgsl (src/webgpu/kernels/gemm.ts:1362-1716) --
//   vec4<f16> accumulators, fma in increasing K; epilogue in f32 with
//   specializedBias/Activation/Residual (:2006-2044), store f16.
// f32 package: f32SubgroupGemmWgsl (:2356-2599), fp32 fma chain, epilogue
//   fp32SpecializedBias/Residual (:2847-2869), store f32.
// act: 0 none, 1 SiLU v/(1+exp(-clamp(v,-20,20))), 2 ReLU max(v,0).
// Residual: value = residual + scale * value (bias and residual exclusive).
// ---------------------------------------------------------------------------
// The shaders' f32 exp is backend-defined to a few ulp; this restatement
// uses the correctly rounded f32 value (the double-precision exp rounded
// once), as the CUDA reference-arithmetic kernels do.
static inline float exp_f32(float x) { return (float)std::exp((double)x); }

static inline float epilogue(float v, const float* bias, int64_t n, int act) {
  if (bias) v += bias[n];
  if (act == 1) {
    const float b = std::min(std::max(v, -20.0f), 20.0f);
    v = v / (1.0f + exp_f32(-b));
  } else if (act == 2) {
    v = std::max(v, 0.0f);
  }
  return v;
}

void or_palette_gemm(int prec, int acc_mode, int64_t rows, int64_t inner, int64_t columns,
                     const void* a, const uint32_t* codes, const void* palette, int bits,
                     int groups, int64_t group_cols, const float* bias, const void* residual,
                     float residual_scale, int act, void* c) {
  // Dense f32 copy of the expanded weight [K, N] (values are exact: f16 or f32).
  std::vector<float> w((size_t)(inner * columns));
  {
    const int per = bits == 5 ? 32 : 16, words = bits == 5 ? 5 : 3;
    const int entries = 1 << bits;
#pragma omp parallel for schedule(static)
    for (int64_t g = 0; g < inner * columns / per; ++g) {
      const int64_t base = g * per;
      const int64_t pg = std::min<int64_t>((base % columns) / group_cols, groups - 1);
      for (int i = 0; i < per; ++i) {
        const uint32_t code = code_at(codes + g * words, bits, i);
        w[(size_t)(base + i)] = ld(palette, prec, (size_t)(pg * entries + code));
      }
    }
  }
  const bool round16 = prec == 0 && acc_mode == 0;
  const int64_t RB = 8, CB = 256;
  const int64_t row_blocks = (rows + RB - 1) / RB, col_blocks = (columns + CB - 1) / CB;
#pragma omp parallel for schedule(dynamic, 1) collapse(2)
  for (int64_t rb = 0; rb < row_blocks; ++rb) {
    for (int64_t cb = 0; cb < col_blocks; ++cb) {
      const int64_t r0 = rb * RB, r1 = std::min(rows, r0 + RB);
      const int64_t c0 = cb * CB, c1 = std::min(columns, c0 + CB);
      const int64_t nc = c1 - c0;
      float acc[8][256];
      for (int64_t r = 0; r < r1 - r0; ++r)
        for (int64_t j = 0; j < nc; ++j) acc[r][j] = 0.0f;
      for (int64_t k = 0; k < inner; ++k) {
        const float* wk = &w[(size_t)(k * columns + c0)];
        for (int64_t r = 0; r < r1 - r0; ++r) {
          const float av = ld(a, prec, (size_t)((r0 + r) * inner + k));
          float* ar = acc[r];
          if (round16) {
            for (int64_t j = 0; j < nc; ++j) ar[j] = round_h(std::fma(av, wk[j], ar[j]));
          } else {
            for (int64_t j = 0; j < nc; ++j) ar[j] = std::fma(av, wk[j], ar[j]);
          }
        }
      }
      for (int64_t r = 0; r < r1 - r0; ++r) {
        for (int64_t j = 0; j < nc; ++j) {
          const int64_t idx = (r0 + r) * columns + c0 + j;
          float v = epilogue(acc[r][j], bias, c0 + j, act);
          if (residual) {
            const float sv = residual_scale * v;  // exact for the 0.5 / 1 scales in use
            v = ld(residual, prec, (size_t)idx) + sv;
          }
          st(c, prec, (size_t)idx, v);
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// LayerNorm (src/webgpu/kernels/layernorm.ts:309-389): per row f32 sum and
// sum of squares, var = max(E[x^2] - mean^2, 0), y = (x - mean) * rsqrt(var +
// eps) * gamma + beta, stored in the profile scalar.
// ---------------------------------------------------------------------------
void or_layernorm(int prec, int64_t rows, int64_t channels, const void* x, const float* gamma,
                  const float* beta, float eps, void* y) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    float sum = 0.0f, square = 0.0f;
    for (int64_t c = 0; c < channels; ++c) {
      const float v = ld(x, prec, (size_t)(r * channels + c));
      sum += v;
      square = std::fma(v, v, square);
    }
    const float inv = 1.0f / (float)channels;
    const float mean = sum * inv;
    const float var = std::max(square * inv - mean * mean, 0.0f);
    const float rstd = 1.0f / std::sqrt(var + eps);
    for (int64_t c = 0; c < channels; ++c) {
      const float v = ld(x, prec, (size_t)(r * channels + c));
      const float nrm = (v - mean) * rstd;
      st(y, prec, (size_t)(r * channels + c), std::fma(nrm, gamma[c], beta[c]));
    }
  }
}

// ---------------------------------------------------------------------------
// Relative-position MHSA (src/webgpu/kernels/attention.ts:418-728).
// qkv [B*T, 3072] (q | k | v), positions packed head-vector-position-vec4
// [8][32][2T-1][4] (model/convert.py:1195-1228), bias_u/v f32 [8,128].
// s_ij = sum over vec4 of fma((q+u), k) and fma((q+v), p[T-1-i+j]) interleaved
// per component (accumulate_score_vector, :455-471), times 1/sqrt(128); keys
// j >= valid get -3.402823466e38; f32 softmax; ctx = sum_j p_ij v_j (fma,
// increasing j); rows i >= valid are zero.
// ---------------------------------------------------------------------------
void or_rel_attention(int prec, int64_t batch, int64_t frames, const void* qkv,
                      const void* positions, const float* bias_u, const float* bias_v,
                      const uint32_t* valid_lengths, void* context) {
  const int H = 8, D = 128, HID = 1024;
  const int64_t P = 2 * frames - 1;
  const float scale = (float)(1.0 / std::sqrt(128.0));
#pragma omp parallel for schedule(dynamic, 1) collapse(2)
  for (int64_t b = 0; b < batch; ++b) {
    for (int h = 0; h < H; ++h) {
      const int64_t valid = std::min<int64_t>(valid_lengths[b], frames);
      std::vector<float> qu(D), qv(D), sc(frames);
      for (int64_t i = 0; i < frames; ++i) {
        const int64_t row = b * frames + i;
        if (i >= valid) {
          for (int d = 0; d < D; ++d) st(context, prec, (size_t)(row * HID + h * D + d), 0.0f);
          continue;
        }
        for (int d = 0; d < D; ++d) {
          const float q = ld(qkv, prec, (size_t)(row * 3 * HID + h * D + d));
          qu[d] = q + bias_u[h * D + d];
          qv[d] = q + bias_v[h * D + d];
        }
        float mx = -3.402823466e+38f;
        for (int64_t j = 0; j < frames; ++j) {
          if (j >= valid) { sc[j] = -3.402823466e+38f; continue; }
          const int64_t krow = b * frames + j;
          const int64_t rel = frames - 1 - i + j;
          float s = 0.0f;
          for (int vec = 0; vec < 32; ++vec) {
            for (int comp = 0; comp < 4; ++comp) {
              const int d = vec * 4 + comp;
              const float kk = ld(qkv, prec, (size_t)(krow * 3 * HID + HID + h * D + d));
              const float pp = ld(positions, prec, (size_t)((((int64_t)h * 32 + vec) * P + rel) * 4 + comp));
              s = std::fma(qu[d], kk, s);
              s = std::fma(qv[d], pp, s);
            }
          }
          s *= scale;
          sc[j] = s;
          mx = std::max(mx, s);
        }
        float sum = 0.0f;
        for (int64_t j = 0; j < valid; ++j) {
          sc[j] = exp_f32(sc[j] - mx);
          sum += sc[j];
        }
        const float inv = 1.0f / sum;
        for (int64_t j = 0; j < valid; ++j) sc[j] = sc[j] * inv;
        for (int d = 0; d < D; ++d) {
          float o = 0.0f;
          for (int64_t j = 0; j < valid; ++j)
            o = std::fma(sc[j], ld(qkv, prec, (size_t)((b * frames + j) * 3 * HID + 2 * HID + h * D + d)), o);
          st(context, prec, (size_t)(row * HID + h * D + d), o);
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Fused conformer convolution (src/webgpu/kernels/conformer-conv.ts:471-575):
// glu = value * sigmoid(gate) with sigmoid clamped to [-20,20], zero outside
// [0, min(T, valid)); dw k=9 same padding as an fma chain; affine = sum * scale
// + shift (folded BN, model/convert.py:1705-1735); y = affine * sigmoid(affine).
// Output rows are produced for every frame < T (no output mask).
// ---------------------------------------------------------------------------
static inline float sigmoid_clamped(float v) {
  const float b = std::min(std::max(v, -20.0f), 20.0f);
  return 1.0f / (1.0f + exp_f32(-b));
}

void or_conformer_conv(int prec, int64_t batch, int64_t frames, const void* pointwise,
                       const void* dw_weights, const float* bn_scale, const float* bn_shift,
                       const uint32_t* valid_lengths, void* out) {
  const int C = 1024, K = 9, R = 4;
#pragma omp parallel for schedule(static) collapse(2)
  for (int64_t b = 0; b < batch; ++b) {
    for (int64_t t = 0; t < frames; ++t) {
      const int64_t valid = valid_lengths[b];
      for (int c = 0; c < C; ++c) {
        float sum = 0.0f;
        for (int k = 0; k < K; ++k) {
          const int64_t tt = t + k - R;
          float glu = 0.0f;
          if (tt >= 0 && tt < frames && tt < valid) {
            const int64_t row = b * frames + tt;
            const float value = ld(pointwise, prec, (size_t)(row * 2 * C + c));
            const float gate = ld(pointwise, prec, (size_t)(row * 2 * C + C + c));
            glu = value * sigmoid_clamped(gate);
          }
          sum = std::fma(glu, ld(dw_weights, prec, (size_t)(k * C + c)), sum);
        }
        const float affine = std::fma(sum, bn_scale[c], bn_shift[c]);
        st(out, prec, (size_t)((b * frames + t) * C + c), affine * sigmoid_clamped(affine));
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Subsampling front end (src/webgpu/kernels/subsampling.ts:1092-1425).
// Valid lengths shrink by ceil(L/2) per stride-2 step (fused_subsampled_length).
// ---------------------------------------------------------------------------
static inline int64_t sub_len(int64_t raw, int steps) {
  for (int s = 0; s < steps; ++s) raw = (raw + 1) / 2;
  return raw;
}

// FUSED_CONV0_DEPTHWISE2_WGSL (:1092-1268).  fbank f32 [B,128,1501] feature-
// major; conv0 weights [3,3,256] (kh-kw-output-channel), conv0 bias f32;
// conv0 = ReLU(sum) rounded to the profile scalar; rows >= ceil(L/2) of conv0
// are zero; depthwise 3x3 s2 over conv0 plus bias; output rows >= ceil(L/4)
// zero.  Output [B, 376, 32, 256] channel-last.
void or_subsampling_conv0_dw2(int prec, int64_t batch, const float* fbank, const void* conv0_w,
                              const float* conv0_b, const void* dw_w, const float* dw_b,
                              const uint32_t* feature_lengths, void* out) {
  const int IH = 1501, IW = 128, CH = 751, CW = 64, OH = 376, OW = 32, C = 256;
  for (int64_t b = 0; b < batch; ++b) {
    const int64_t vin = sub_len(feature_lengths[b], 1), vout = sub_len(feature_lengths[b], 2);
    std::vector<float> conv0((size_t)CH * CW * C);
#pragma omp parallel for schedule(static)
    for (int y = 0; y < CH; ++y) {
      for (int x = 0; x < CW; ++x) {
        for (int c = 0; c < C; ++c) {
          float r = 0.0f;
          if (y < vin) {
            float sum = conv0_b[c];
            for (int ky = 0; ky < 3; ++ky) {
              const int iy = y * 2 + ky - 1;
              if (iy < 0 || iy >= IH) continue;
              for (int kx = 0; kx < 3; ++kx) {
                const int ix = x * 2 + kx - 1;
                if (ix < 0 || ix >= IW) continue;
                const float v = fbank[(b * IW + ix) * IH + iy];
                sum = std::fma(ld(conv0_w, prec, (size_t)((ky * 3 + kx) * C + c)), v, sum);
              }
            }
            r = std::max(sum, 0.0f);
            if (prec == 0) r = round_h(r);
          }
          conv0[((size_t)y * CW + x) * C + c] = r;
        }
      }
    }
#pragma omp parallel for schedule(static)
    for (int y = 0; y < OH; ++y) {
      for (int x = 0; x < OW; ++x) {
        for (int c = 0; c < C; ++c) {
          const size_t oi = (((size_t)b * OH + y) * OW + x) * C + c;
          if (y >= vout) { st(out, prec, oi, 0.0f); continue; }
          float sum = dw_b[c];
          for (int ky = 0; ky < 3; ++ky) {
            const int iy = y * 2 + ky - 1;
            if (iy < 0 || iy >= CH || iy >= vin) continue;
            for (int kx = 0; kx < 3; ++kx) {
              const int ix = x * 2 + kx - 1;
              if (ix < 0 || ix >= CW) continue;
              sum = std::fma(conv0[((size_t)iy * CW + ix) * C + c],
                             ld(dw_w, prec, (size_t)((ky * 3 + kx) * C + c)), sum);
            }
          }
          st(out, prec, oi, sum);
        }
      }
    }
  }
}

// DEPTHWISE_WGSL (:1270-1372): dw 3x3 s2 p1 + bias over channel-last input;
// input rows >= sub_len(L, steps-1) are skipped, output rows >= sub_len(L,
// steps) are zero.
void or_subsampling_depthwise(int prec, int64_t batch, int64_t ih, int64_t iw, int64_t channels,
                              const void* input, const void* w, const float* bias,
                              const uint32_t* feature_lengths, int steps, void* out) {
  const int64_t oh = (ih + 2 - 3) / 2 + 1, ow = (iw + 2 - 3) / 2 + 1;
#pragma omp parallel for schedule(static) collapse(2)
  for (int64_t b = 0; b < batch; ++b) {
    for (int64_t y = 0; y < oh; ++y) {
      const int64_t vin = sub_len(feature_lengths[b], steps - 1), vout = sub_len(feature_lengths[b], steps);
      for (int64_t x = 0; x < ow; ++x) {
        for (int64_t c = 0; c < channels; ++c) {
          const size_t oi = (size_t)(((b * oh + y) * ow + x) * channels + c);
          if (y >= vout) { st(out, prec, oi, 0.0f); continue; }
          float sum = bias[c];
          for (int ky = 0; ky < 3; ++ky) {
            const int64_t iy = y * 2 + ky - 1;
            if (iy < 0 || iy >= ih || iy >= vin) continue;
            for (int kx = 0; kx < 3; ++kx) {
              const int64_t ix = x * 2 + kx - 1;
              if (ix < 0 || ix >= iw) continue;
              sum = std::fma(ld(input, prec, (size_t)(((b * ih + iy) * iw + ix) * channels + c)),
                             ld(w, prec, (size_t)((ky * 3 + kx) * channels + c)), sum);
            }
          }
          st(out, prec, oi, sum);
        }
      }
    }
  }
}

// SUBSAMPLING_TIME_MASK_WGSL (:1374-1425): zero frames >= sub_len(L, steps).
void or_subsampling_time_mask(int prec, int64_t batch, int64_t height, int64_t width,
                              int64_t channels, void* values, const uint32_t* feature_lengths,
                              int steps) {
  for (int64_t b = 0; b < batch; ++b) {
    const int64_t v = sub_len(feature_lengths[b], steps);
    for (int64_t y = v; y < height; ++y)
      for (int64_t i = 0; i < width * channels; ++i)
        st(values, prec, (size_t)((b * height + y) * width * channels + i), 0.0f);
  }
}


// ---------------------------------------------------------------------------
// Persistent TDT greedy decoder (src/webgpu/kernels/tdt-decoder.ts:1076-2000,
// the subgroup shader; one sequence at a time -- the shader pairs two
// sequences per workgroup only to share weight loads, with no arithmetic
// shared between them).
//
// FP16 package (prec 0): every LSTM gate is two f16 FMA chains in increasing
// input index -- even indices starting from f16(bias), odd indices from 0 --
// summed in f16 (wgslLstmAccumulate / wgslLstmStore, :596-671); each chain
// input is f16(x).  The head is one f16 FMA chain per output starting from
// f16(bias) (wgslFp16PairedHeadBody, :1005-1057) that skips an input index
// whose f32 value is +0 as long as no -0 or NaN input has been seen.  The
// projection is an f32 FMA chain over f32(h1) and f32(weight) (:1435-1456).
// An f16 FMA is emulated with a single rounding: the product of two f16
// values and the sum with an f16 addend are formed exactly in double, then
// rounded once to f16 (a fused f16 FMA, as Apple GPUs and CUDA's HFMA2 do).
// FP32 package (prec 1): the same chains in f32 with fmaf (:682-700, :864-878).
// Gate nonlinearities: sigmoid(v) = 1/(1+exp(-clamp(v,+-20))), tanh of a value
// clamped to +-10 (:1310-1326); cell = fma(f, c, i*g), h = o*tanh(cell).
// Argmax: the largest score (NaN -> -FLT_MAX), lowest id on ties
// (choose_better, :1478-1486); tokens 0..1023 plus blank 1024, durations from
// outputs 1025..1029 (wgslHeadArgmaxAndReduce, :769-830).
// Control: tdt-decoder.ts:1702-1990 (main loop, at most 10 symbols per frame,
// then the bounded end-of-stream flush).
// ---------------------------------------------------------------------------
namespace tdt {
constexpr int H = 640, G = 2560, KIN = 1280, NOUT = 1032, BLANK = 1024, MAXSYM = 10;

// a*b + c and a + b for f16 operands, rounded once to f16.  The product of
// two f16 values is exact in f32; TwoSum gives the exact error of the f32 sum,
// which then rounds to odd (an inexact result with an even last bit moves one
// ulp toward the exact value); rounding that to f16 (11 bits, far fewer than
// f32's 24) is the correctly rounded f16 result.
static inline float sum_round_odd(float p, float c) {
  const float s = p + c;
  const float bp = s - c;
  const float err = (p - bp) + (c - (s - bp));
  uint32_t bits;
  std::memcpy(&bits, &s, 4);
  // Branch-free (so the loops vectorize): move only when inexact and even;
  // s != 0 whenever err != 0.
  const uint32_t move = (uint32_t)(err != 0.0f) & ~bits & 1u;
  const uint32_t away = (uint32_t)((err > 0.0f) == (s > 0.0f));
  bits += move * (away ? 1u : 0xffffffffu);
  float r;
  std::memcpy(&r, &bits, 4);
  return r;
}
static inline float hfma(float a, float b, float c) { return (float)(half_t)sum_round_odd(a * b, c); }
static inline float hadd(float a, float b) { return (float)(half_t)sum_round_odd(a, b); }
// The same operation through double (an exact sum), kept to cross-check.
static inline float hfma_double(float a, float b, float c) {
  return (float)(half_t)((double)a * (double)b + (double)c);
}
// exp / tanh are taken correctly rounded to f32 (the double-precision
// functions, rounded once); the shader's f32 versions are backend-defined to
// a few ulp, and the CUDA decoder uses the same correctly rounded values.
static inline float sig(float v) {
  const float b = std::min(std::max(v, -20.0f), 20.0f);
  return 1.0f / (1.0f + (float)std::exp((double)-b));
}
static inline float stanh(float v) { return (float)std::tanh((double)std::min(std::max(v, -10.0f), 10.0f)); }

struct Weights {
  int prec;
  const void *emb, *w0, *w1, *pw, *hw;
  const float *b0, *b1, *pb, *hb;
};

struct Seq {
  std::vector<float> h0, c0, h1, c1, proj;
  Seq() : h0(H, 0.f), c0(H, 0.f), h1(H, 0.f), c1(H, 0.f), proj(H, 0.f) {}
};

// One LSTM layer: gates from `x` (KIN inputs, only the first `limit` used),
// then the cell update of (h, c) in place.
static void lstm_layer(const Weights& W, const void* w, const float* bias, const float* x, int limit,
                       std::vector<float>& h, std::vector<float>& c) {
  std::vector<float> gate(G);
  const int p = W.prec;
  // Each thread owns a block of outputs and walks the inputs in increasing
  // order, so every output's two chains keep the shader's order.
#pragma omp parallel for schedule(static)
  for (int o0 = 0; o0 < G; o0 += 256) {
    float even[256], odd[256];
    for (int i = 0; i < 256; ++i) {
      even[i] = p == 0 ? round_h(bias[o0 + i]) : bias[o0 + i];
      odd[i] = 0.0f;
    }
    for (int k = 0; k < limit; k += 2) {
      if (p == 0) {
        const float xe = round_h(x[k]), xo = round_h(x[k + 1]);
        const uint16_t* re = (const uint16_t*)w + (size_t)k * G + o0;
        const uint16_t* ro = re + G;
        for (int i = 0; i < 256; ++i) {
          even[i] = hfma(xe, h2f(re[i]), even[i]);
          odd[i] = hfma(xo, h2f(ro[i]), odd[i]);
        }
      } else {
        const float* re = (const float*)w + (size_t)k * G + o0;
        const float* ro = re + G;
        for (int i = 0; i < 256; ++i) {
          even[i] = std::fma(x[k], re[i], even[i]);
          odd[i] = std::fma(x[k + 1], ro[i], odd[i]);
        }
      }
    }
    for (int i = 0; i < 256; ++i) gate[o0 + i] = p == 0 ? hadd(even[i], odd[i]) : even[i] + odd[i];
  }
  for (int ch = 0; ch < H; ++ch) {
    const float i = sig(gate[ch]), f = sig(gate[H + ch]), g = stanh(gate[2 * H + ch]), o = sig(gate[3 * H + ch]);
    const float cell = std::fma(f, c[ch], i * g);
    c[ch] = cell;
    h[ch] = o * stanh(cell);
  }
}

// prepare_predictor + commit (the committed state always equals the last
// candidate, so the state is advanced in place).
static void predict(const Weights& W, Seq& s, int token, bool initial) {
  std::vector<float> x(KIN, 0.0f);
  if (!initial) {
    for (int k = 0; k < H; ++k) x[k] = ld(W.emb, W.prec, (size_t)token * H + k);
    for (int k = 0; k < H; ++k) x[H + k] = s.h0[k];
    lstm_layer(W, W.w0, W.b0, x.data(), KIN, s.h0, s.c0);
  } else {
    lstm_layer(W, W.w0, W.b0, x.data(), 0, s.h0, s.c0);  // SOS: zero input and state
  }
  for (int k = 0; k < H; ++k) x[k] = s.h0[k];
  for (int k = 0; k < H; ++k) x[H + k] = s.h1[k];
  lstm_layer(W, W.w1, W.b1, x.data(), initial ? H : KIN, s.h1, s.c1);
  for (int o = 0; o < H; ++o) {
    float acc = W.pb[o];
    for (int k = 0; k < H; ++k) acc = std::fma(s.h1[k], ld(W.pw, W.prec, (size_t)k * H + o), acc);
    s.proj[o] = acc;
  }
}

static inline float sanitize(float v) { return v != v ? -3.402823466e38f : v; }
static inline bool better(float lv, uint32_t lid, float rv, uint32_t rid) {
  return rv > lv || (rv == lv && rid < lid);
}

static void joint(const Weights& W, const Seq& s, const void* enc_row, uint32_t* token, uint32_t* duration) {
  const int p = W.prec;
  std::vector<float> jin(H);
  for (int k = 0; k < H; ++k) jin[k] = std::max(ld(enc_row, p, k) + s.proj[k], 0.0f);
  std::vector<float> acc(NOUT);
  for (int o = 0; o < NOUT; ++o) acc[o] = p == 0 ? round_h(W.hb[o]) : W.hb[o];
  std::vector<char> skip(H);
  bool safe = true;
  for (int k = 0; k < H; ++k) {
    uint32_t bits;
    std::memcpy(&bits, &jin[k], 4);
    const bool nan = (bits & 0x7fffffffu) > 0x7f800000u;
    safe = safe && !(bits == 0x80000000u || nan);
    skip[k] = safe && bits == 0u;
  }
#pragma omp parallel for schedule(static)
  for (int o0 = 0; o0 < NOUT; o0 += 129) {  // 8 blocks of outputs, inputs in increasing order
    const int o1 = std::min(o0 + 129, NOUT);
    for (int k = 0; k < H; ++k) {
      if (skip[k]) continue;
      if (p == 0) {
        const float xk = round_h(jin[k]);
        for (int o = o0; o < o1; ++o) acc[o] = hfma(xk, ld(W.hw, 0, (size_t)k * NOUT + o), acc[o]);
      } else {
        for (int o = o0; o < o1; ++o) acc[o] = std::fma(jin[k], ld(W.hw, 1, (size_t)k * NOUT + o), acc[o]);
      }
    }
  }
  float tv = -3.402823466e38f, dv = -3.402823466e38f;
  uint32_t tid = 0xffffffffu, did = 0xffffffffu;
  for (uint32_t o = 0; o <= (uint32_t)BLANK; ++o)
    if (better(tv, tid, sanitize(acc[o]), o)) tv = sanitize(acc[o]), tid = o;
  for (uint32_t d = 0; d < 5; ++d)
    if (better(dv, did, sanitize(acc[BLANK + 1 + d]), d)) dv = sanitize(acc[BLANK + 1 + d]), did = d;
  *token = tid;
  *duration = did;
}
}  // namespace tdt

// Self-check of the f16 FMA emulation: how many of n seeded operand triples
// (f16 values over the whole finite range) round differently through
// round-to-odd f32 and through double.
int64_t or_hfma_selfcheck(int64_t n, uint64_t seed) {
  uint64_t x = seed | 1;
  auto next = [&]() {
    x ^= x << 13;
    x ^= x >> 7;
    x ^= x << 17;
    return x;
  };
  auto h = [&]() {
    uint16_t bits = (uint16_t)next();
    if ((bits & 0x7c00u) == 0x7c00u) bits &= 0xbbffu;  // no inf / NaN
    return h2f(bits);
  };
  int64_t bad = 0;
  for (int64_t i = 0; i < n; ++i) {
    const float a = h(), b = h(), c = h();
    const float r1 = tdt::hfma(a, b, c), r2 = tdt::hfma_double(a, b, c);
    if (std::memcmp(&r1, &r2, 4) != 0 && !(r1 != r1 && r2 != r2)) ++bad;
  }
  return bad;
}

// Decodes `batch` sequences.  enc: [batch, frames, 640] profile scalar;
// lengths/starts/ends/flush: u32 [batch]; outputs tokens / token_frames /
// token_durations u32 [batch, max_tokens]; metadata u32 [2*batch] = counts
// then status flags (bit 0 = more tokens than max_tokens).
void or_tdt_decode(int prec, int64_t batch, int64_t frames, int64_t max_tokens, const void* enc,
                   const uint32_t* lengths, const uint32_t* starts, const uint32_t* ends, const uint32_t* flush,
                   const void* embedding, const void* lstm0, const float* bias0, const void* lstm1,
                   const float* bias1, const void* proj_w, const float* proj_b, const void* head_w,
                   const float* head_b, uint32_t* tokens, uint32_t* token_frames, uint32_t* token_durations,
                   uint32_t* metadata) {
  using namespace tdt;
  const Weights W{prec, embedding, lstm0, lstm1, proj_w, head_w, bias0, bias1, proj_b, head_b};
  const size_t es = prec == 0 ? 2 : 4;
  for (int64_t b = 0; b < batch; ++b) {  // the chains inside each step run in parallel
    Seq s;
    uint32_t count = 0, status = 0, sym = 0;
    const uint32_t enc_len = std::min(std::min(lengths[b], (uint32_t)frames), ends[b]);
    uint32_t t = std::min(starts[b], enc_len);
    auto row = [&](uint32_t tt) {
      return static_cast<const void*>(static_cast<const char*>(enc) + ((size_t)b * frames + tt) * H * es);
    };
    auto emit = [&](uint32_t tok, uint32_t frame, uint32_t dur) {
      if (count < (uint32_t)max_tokens) {
        const size_t o = (size_t)b * max_tokens + count;
        tokens[o] = tok;
        token_frames[o] = frame;
        token_durations[o] = dur;
        ++count;
      } else {
        status |= 1u;
      }
    };
    if (t < enc_len) predict(W, s, 0, true);
    while (t < enc_len) {
      uint32_t tok, dur;
      joint(W, s, row(t), &tok, &dur);
      const bool nonblank = tok != (uint32_t)BLANK;
      if (nonblank) emit(tok, t, dur);
      sym += 1;
      if (dur != 0) {
        t += dur;
        sym = 0;
      } else if (!nonblank || sym >= (uint32_t)MAXSYM) {
        t += 1;
        sym = 0;
      }
      if (nonblank) predict(W, s, (int)tok, false);
    }
    if (flush[b] != 0 && starts[b] < enc_len) {
      uint32_t fsym = 0, blanks = 0, ft = t;
      const uint32_t len_c = std::min(lengths[b], (uint32_t)frames);
      while (fsym < (uint32_t)MAXSYM && blanks < 5) {
        const uint32_t v = fsym % 3;
        if (v == 0) t = std::min(ft, len_c - 1);
        else if (v == 1) t = std::min(enc_len - 1, (uint32_t)frames - 1);
        else t = std::min(std::max(enc_len, 2u) - 2, (uint32_t)frames - 1);
        uint32_t tok, dur;
        joint(W, s, row(t), &tok, &dur);
        const bool nonblank = tok != (uint32_t)BLANK;
        if (!nonblank) {
          blanks += 1;
        } else {
          blanks = 0;
          emit(tok, std::min(ft, enc_len - 1), dur);
        }
        ft = std::min(ft + std::max(1u, dur), enc_len);
        fsym += 1;
        if (nonblank) predict(W, s, (int)tok, false);
      }
    }
    metadata[b] = count;
    metadata[batch + b] = status;
  }
}


// ---------------------------------------------------------------------------
// Log-mel front end (src/cpp/fbank/parakeet_fbank.cpp): per window,
// floor(valid/160) frames of a centered 512-point STFT over a 400-sample
// Hann window (periodic = false, centered in the 512 frame), preemphasis 0.97
// applied in double inside each frame's samples (the first sample of the
// window kept), radix-2 decimation-in-time FFT in f32 on bit-reversed input
// with a twiddle-free first butterfly per block (:195-240), power in double,
// 128 Slaney mel filters (Slaney-normalized, f32 weights from double, :139-186)
// summed in double in bin order, log(energy + 2^-24) in double, then
// per-window per-bin normalization over the valid frames with an unbiased
// standard deviation (+1e-5), zero beyond them (:486-521).  The reference's
// raw-frame reuse between overlapping windows only skips recomputing frames
// whose result is identical, so every frame is computed here.
// ---------------------------------------------------------------------------
namespace lm {
constexpr int kFft = 512, kBins = 257, kWin = 400, kHop = 160, kMels = 128, kSr = 16000;
constexpr double kPi = 3.14159265358979323846264338327950288;

struct Tables {
  float hann[kFft];
  float tw_re[kFft / 2], tw_im[kFft / 2];
  int rev[kFft];
  float mel[kMels][kBins];
  int first[kMels], last[kMels];
  Tables() {
    for (int i = 0; i < kFft; ++i) hann[i] = 0.0f;
    for (int i = 0; i < kWin; ++i)
      hann[(kFft - kWin) / 2 + i] = (float)(0.5 * (1.0 - std::cos(2.0 * kPi * (double)i / (double)(kWin - 1))));
    for (int i = 0; i < kFft / 2; ++i) {
      const double ph = (-2.0 * kPi * (double)i) / (double)kFft;
      tw_re[i] = (float)std::cos(ph);
      tw_im[i] = (float)std::sin(ph);
    }
    for (int i = 0; i < kFft; ++i) {
      int r = 0;
      for (int b = 0; b < 9; ++b) r |= ((i >> b) & 1) << (8 - b);
      rev[i] = r;
    }
    auto to_mel = [](double f) {
      const double lin = 200.0 / 3.0, ft = 1000.0, mt = ft / lin, step = 0.06875177742094912;
      return f >= ft ? mt + std::log(f / ft) / step : f / lin;
    };
    auto to_hz = [](double m) {
      const double lin = 200.0 / 3.0, ft = 1000.0, mt = ft / lin, step = 0.06875177742094912;
      return m >= mt ? ft * std::exp(step * (m - mt)) : m * lin;
    };
    double freq[kBins], pts[kMels + 2];
    for (int b = 0; b < kBins; ++b) freq[b] = ((double)kSr * 0.5 * b) / (double)(kBins - 1);
    const double m0 = to_mel(0.0), m1 = to_mel(kSr * 0.5);
    for (int i = 0; i < kMels + 2; ++i) pts[i] = to_hz(m0 + (m1 - m0) * i / (kMels + 1));
    for (int m = 0; m < kMels; ++m) {
      const double norm = 2.0 / (pts[m + 2] - pts[m]);
      first[m] = -1;
      last[m] = -1;
      for (int b = 0; b < kBins; ++b) {
        const double down = (freq[b] - pts[m]) / (pts[m + 1] - pts[m]);
        const double up = (pts[m + 2] - freq[b]) / (pts[m + 2] - pts[m + 1]);
        double tri = down < up ? down : up;
        if (tri < 0.0) tri = 0.0;
        mel[m][b] = (float)(tri * norm);
        if (mel[m][b] > 0.0f) {
          if (first[m] < 0) first[m] = b;
          last[m] = b;
        }
      }
      if (first[m] < 0) first[m] = 0, last[m] = -1;
    }
  }
};

static const Tables& tables() {
  static const Tables t;
  return t;
}

// One frame's 128 raw log-mel values; `n` samples are real, the rest zero.
static void raw_frame(const float* x, int n, int frame, float* out /* [128], stride ostride */, int64_t ostride) {
  const Tables& T = tables();
  float re[kFft], im[kFft];
  for (int i = 0; i < kFft; ++i) re[i] = im[i] = 0.0f;
  const int center = frame * kHop;
  const int lo = std::max(0, center - kWin / 2), hi = std::min(n, center + kWin / 2);
  for (int src = lo; src < hi; ++src) {
    const double e = src == 0 ? (double)x[0] : (double)x[src] - (double)0.97f * (double)x[src - 1];
    const int fi = src - center + kFft / 2;
    re[T.rev[fi]] = (float)(e * (double)T.hann[fi]);
  }
  for (int len = 2; len <= kFft; len <<= 1) {
    const int half = len >> 1, step = kFft / len;
    for (int blk = 0; blk < kFft; blk += len) {
      {
        const float rr = re[blk + half], ri = im[blk + half], lr = re[blk], li = im[blk];
        re[blk] = lr + rr;
        im[blk] = li + ri;
        re[blk + half] = lr - rr;
        im[blk + half] = li - ri;
      }
      for (int j = 1; j < half; ++j) {
        const int l = blk + j, r = l + half, t = j * step;
        const float rr = re[r], ri = im[r];
        const float xr = T.tw_re[t] * rr - T.tw_im[t] * ri;
        const float xi = T.tw_re[t] * ri + T.tw_im[t] * rr;
        const float lr = re[l], li = im[l];
        re[l] = lr + xr;
        im[l] = li + xi;
        re[r] = lr - xr;
        im[r] = li - xi;
      }
    }
  }
  double pw[kBins];
  for (int b = 0; b < kBins; ++b) pw[b] = (double)re[b] * (double)re[b] + (double)im[b] * (double)im[b];
  for (int m = 0; m < kMels; ++m) {
    double en = 0.0;
    for (int b = T.first[m]; b <= T.last[m]; ++b) en += (double)T.mel[m][b] * pw[b];
    out[m * ostride] = (float)std::log(en + 1.0 / 16777216.0);
  }
}
}  // namespace lm

// samples f32 [batch, sample_count]; valid u32 [batch] (<= sample_count);
// features f32 [batch, 128, sample_count / 160 + 1] feature-major.
void or_logmel(int64_t batch, int64_t sample_count, const float* samples, const uint32_t* valid, float* features) {
  using namespace lm;
  const int64_t frames = sample_count / kHop + 1;
  tables();
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t b = 0; b < batch; ++b) {
    const int n = (int)valid[b];
    const int nf = n / kHop;
    float* f = features + (size_t)b * kMels * frames;
    const float* x = samples + (size_t)b * sample_count;
    for (int t = 0; t < nf; ++t) raw_frame(x, n, t, f + t, frames);
    for (int m = 0; m < kMels; ++m) {
      float* row = f + (size_t)m * frames;
      double sum = 0.0;
      for (int t = 0; t < nf; ++t) sum += (double)row[t];
      const double mean = nf > 0 ? sum / (double)nf : 0.0;
      double sq = 0.0;
      for (int t = 0; t < nf; ++t) {
        const double d = (double)row[t] - mean;
        sq += d * d;
      }
      const double sd = nf > 1 ? std::sqrt(sq / (double)(nf - 1)) : 0.0;
      const double inv = 1.0 / (sd + 1.0e-5);
      for (int t = 0; t < nf; ++t) row[t] = (float)(((double)row[t] - mean) * inv);
      for (int64_t t = nf; t < frames; ++t) row[t] = 0.0f;
    }
  }
}

// The tables the CUDA front end uploads: hann [512], twiddles re/im [256],
// mel filter bins first/count [128] and the packed nonzero weights.
int or_logmel_tables(float* hann, float* tw_re, float* tw_im, int* first, int* count, float* packed, int capacity) {
  const lm::Tables& T = lm::tables();
  std::memcpy(hann, T.hann, sizeof(T.hann));
  std::memcpy(tw_re, T.tw_re, sizeof(T.tw_re));
  std::memcpy(tw_im, T.tw_im, sizeof(T.tw_im));
  int n = 0;
  for (int m = 0; m < lm::kMels; ++m) {
    first[m] = T.first[m];
    count[m] = T.last[m] - T.first[m] + 1;
    for (int b = T.first[m]; b <= T.last[m]; ++b) {
      if (n < capacity) packed[n] = T.mel[m][b];
      ++n;
    }
  }
  return n;
}

}  // extern "C"
