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
static inline float epilogue(float v, const float* bias, int64_t n, int act) {
  if (bias) v += bias[n];
  if (act == 1) {
    const float b = std::min(std::max(v, -20.0f), 20.0f);
    v = v / (1.0f + std::exp(-b));
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
          sc[j] = std::exp(sc[j] - mx);
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
  return 1.0f / (1.0f + std::exp(-b));
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

}  // extern "C"
