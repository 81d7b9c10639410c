// subsampling.cu -- dw-striding subsampling front end (8x in time and frequency).
//
// Restates the reference's three subsampling shaders
// (src/webgpu/kernels/subsampling.ts):
//   * FUSED_CONV0_DEPTHWISE2_WGSL (:1092-1268): conv0 3x3 stride 2 pad 1 from
//     the f32 feature-major log-mel [B, 128, 1501] to 256 channels, ReLU,
//     rounded to the profile scalar, rows >= ceil(L/2) zero; then depthwise
//     3x3 stride 2 + bias into channel-last [B, 376, 32, 256], rows >=
//     ceil(ceil(L/2)/2) zero;
//   * DEPTHWISE_WGSL (:1270-1372): depthwise 3x3 stride 2 + bias over
//     channel-last input with valid-length masking;
//   * SUBSAMPLING_TIME_MASK_WGSL (:1374-1425): zero frames past the valid
//     length (the pointwise-6 bias re-introduces non-zero padding,
//     src/webgpu/encoder.ts:2370-2377).
// The pointwise 1x1 convolutions and the flatten projection run through the
// palette GEMM.  Arithmetic order (fma chains from the bias, ky outer, kx
// inner, skipped taps outside the valid area) follows the shaders.  Each
// thread owns 8 channels so taps live in registers and every shared-memory
// read feeds 8 FMAs.
#include "pk_common.cuh"
#include "pk_internal.h"

namespace pk {

constexpr int SUB_IH = 1501, SUB_IW = 128, SUB_CH = 751, SUB_CW = 64, SUB_OH = 376, SUB_OW = 32, SUB_C = 256;
constexpr int C0_CG = 32;        // channels per CTA
constexpr int C0_SR = 24;        // depthwise output rows per CTA (a strip)
constexpr int C0_STRIPS = (SUB_OH + C0_SR - 1) / C0_SR;
constexpr int C0_IN_ROWS = 4 * C0_SR + 3;  // input time samples a strip needs
constexpr int C0_IN_PITCH = SUB_IW + 1;
constexpr int C0_PITCH = C0_CG + 4;  // padded channel pitch of the conv0 ring (conflict-free 16-byte access)
// The input strip is padded to a multiple of 4 floats so the conv0 ring and
// the depthwise taps that follow it start on 16-byte boundaries (float4).
constexpr int C0_IN_FLOATS = (C0_IN_ROWS * C0_IN_PITCH + 3) / 4 * 4;
constexpr int C0_RING = 5;  // conv0 rows 2oy-1 .. 2oy+3 for two depthwise rows per pass
constexpr int C0_RING_FLOATS = C0_RING * SUB_CW * C0_PITCH;
constexpr int C0_SMEM = (C0_IN_FLOATS + C0_RING_FLOATS + 9 * C0_CG + C0_CG) * 4;
static_assert(C0_IN_FLOATS % 4 == 0 && C0_PITCH % 4 == 0 && C0_RING_FLOATS % 4 == 0,
              "conv0 ring must stay 16-byte aligned");

__device__ __forceinline__ int sub_len(int raw, int steps) {
  for (int s = 0; s < steps; ++s) raw = (raw + 1) >> 1;
  return raw;
}

// 8 consecutive profile scalars <-> floats.
template <typename T>
__device__ __forceinline__ void load8(const T* p, float* v);
template <>
__device__ __forceinline__ void load8<__half>(const __half* p, float* v) {
  const uint4 raw = __ldg(reinterpret_cast<const uint4*>(p));
  const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __half22float2(h[j]);
    v[2 * j] = f.x;
    v[2 * j + 1] = f.y;
  }
}
template <>
__device__ __forceinline__ void load8<float>(const float* p, float* v) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  const float4 b = __ldg(reinterpret_cast<const float4*>(p + 4));
  v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
}
template <typename T>
__device__ __forceinline__ void store8(T* p, const float* v);
template <>
__device__ __forceinline__ void store8<__half>(__half* p, const float* v) {
  uint4 raw;
  __half2* h = reinterpret_cast<__half2*>(&raw);
#pragma unroll
  for (int j = 0; j < 4; ++j) h[j] = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
  *reinterpret_cast<uint4*>(p) = raw;
}
template <>
__device__ __forceinline__ void store8<float>(float* p, const float* v) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
}

// D (+)= A . B on tensor cores, mma.m16n8k16 with f16 A/B and f32 D.
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_h2(__half lo, __half hi) {
  return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
}

// FP32 profile.  One CTA: window b, a strip of C0_SR depthwise output rows,
// 32 channels.  The strip's input time samples (4*SR+3 of them, all 128 mel
// bins) are staged once; conv0 rows are produced in order into a 5-row ring
// (f32): depthwise row oy needs conv0 rows 2oy-1 .. 2oy+1, and consecutive
// rows share one.
__global__ void __launch_bounds__(256, 2) conv0_dw2_f32_kernel(const float* __restrict__ fbank,
                                                               const float* __restrict__ w0,
                                                               const float* __restrict__ b0,
                                                               const float* __restrict__ wd,
                                                               const float* __restrict__ bd,
                                                               const uint32_t* __restrict__ feature_lengths,
                                                               float* __restrict__ out) {
  pdl_entry();
  extern __shared__ __align__(16) float sub_smem[];
  float* in_s = sub_smem;                                 // [C0_IN_ROWS][129]
  float* ring = sub_smem + C0_IN_FLOATS;                  // [5][64][C0_PITCH], 16-byte aligned
  float* wd_s = ring + C0_RING_FLOATS;                    // [9][32] depthwise taps
  float* bd_s = wd_s + 9 * C0_CG;                         // [32] depthwise bias
  const int b = blockIdx.z;
  const int oy0 = blockIdx.y * C0_SR;
  const int oy_end = min(oy0 + C0_SR, SUB_OH);
  const int cbase = blockIdx.x * C0_CG;
  const int tid = threadIdx.x;
  const int raw = (int)feature_lengths[b];
  const int vin = sub_len(raw, 1), vout = sub_len(raw, 2);
  const int y_first = 2 * oy0 - 1;       // first conv0 row of the strip
  const int iy_first = 2 * y_first - 1;  // first input time sample
  // Stage the strip's input with asynchronous 4-byte copies, all in flight at
  // once (zero-filled outside the utterance); consecutive threads walk time,
  // which is contiguous in the feature-major log-mel.
  for (int i = tid; i < C0_IN_ROWS * SUB_IW; i += 256) {
    const int r = i % C0_IN_ROWS, x = i / C0_IN_ROWS;
    const int iy = iy_first + r;
    const bool in_range = iy >= 0 && iy < SUB_IH;
    const float* src = fbank + ((size_t)b * SUB_IW + x) * SUB_IH + (in_range ? iy : 0);
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_addr(in_s + r * C0_IN_PITCH + x)),
                 "l"(src), "r"(in_range ? 4 : 0)
                 : "memory");
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  for (int i = tid; i < 9 * C0_CG; i += 256) wd_s[i] = wd[(i / C0_CG) * SUB_C + cbase + i % C0_CG];
  if (tid < C0_CG) bd_s[tid] = bd[cbase + tid];
  const int cg = tid >> 6;  // 8-channel group of this thread's conv0 outputs
  const int c = cbase + cg * 8;
  const int x = tid & 63;
  float w[9][8], bias[8];
#pragma unroll
  for (int k = 0; k < 9; ++k) load8<float>(w0 + k * SUB_C + c, w[k]);
#pragma unroll
  for (int j = 0; j < 8; ++j) bias[j] = __ldg(b0 + c + j);
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();

  // conv0 row y (3x3 stride 2 over the staged input) -> ring slot (y + 5) % 5.
  auto conv0_row = [&](int y) {
    float acc[8];
    if (y >= 0 && y < SUB_CH && y < vin) {
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = bias[j];
#pragma unroll
      for (int ky = 0; ky < 3; ++ky) {
        const int iy = y * 2 + ky - 1;
        if (iy < 0 || iy >= SUB_IH) continue;
#pragma unroll
        for (int kx = 0; kx < 3; ++kx) {
          const int ix = x * 2 + kx - 1;
          if (ix < 0 || ix >= SUB_IW) continue;
          const float v = in_s[(iy - iy_first) * C0_IN_PITCH + ix];
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[j] = fmaf(w[ky * 3 + kx][j], v, acc[j]);
        }
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = fmaxf(acc[j], 0.0f);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
    }
    float* dst = ring + (((y + C0_RING) % C0_RING) * SUB_CW + x) * C0_PITCH + cg * 8;
    *reinterpret_cast<float4*>(dst) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    *reinterpret_cast<float4*>(dst + 4) = make_float4(acc[4], acc[5], acc[6], acc[7]);
  };

  conv0_row(y_first);
  // Two depthwise rows per pass: conv0 rows 2oy .. 2oy+3, one barrier,
  // depthwise rows oy, oy+1 (all 256 threads), one barrier.
  const int y_last = 2 * oy_end - 1;  // last conv0 row this strip needs
#pragma unroll 1
  for (int oy = oy0; oy < oy_end; oy += 2) {
    for (int y = 2 * oy; y <= min(2 * oy + 3, y_last); ++y) conv0_row(y);
    __syncthreads();
    const int oyr = oy + (tid >> 7);  // depthwise: thread = (row, channel group, output x)
    if (oyr < oy_end) {
      const int dcg = (tid >> 5) & 3, ox = tid & 31;
      float acc[8];
      if (oyr >= vout) {
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = bd_s[dcg * 8 + j];
#pragma unroll
        for (int ky = 0; ky < 3; ++ky) {
          const int iy = oyr * 2 + ky - 1;
          if (iy < 0 || iy >= SUB_CH || iy >= vin) continue;
#pragma unroll
          for (int kx = 0; kx < 3; ++kx) {
            const int ix = ox * 2 + kx - 1;
            if (ix < 0 || ix >= SUB_CW) continue;
            const float* src = ring + (((iy + C0_RING) % C0_RING) * SUB_CW + ix) * C0_PITCH + dcg * 8;
            const float4 lo = *reinterpret_cast<const float4*>(src);
            const float4 hi = *reinterpret_cast<const float4*>(src + 4);
            const float* wk = wd_s + (ky * 3 + kx) * C0_CG + dcg * 8;
            const float4 wl = *reinterpret_cast<const float4*>(wk);
            const float4 wh = *reinterpret_cast<const float4*>(wk + 4);
            const float v[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
            const float ww[8] = {wl.x, wl.y, wl.z, wl.w, wh.x, wh.y, wh.z, wh.w};
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[j] = fmaf(v[j], ww[j], acc[j]);
          }
        }
      }
      store8<float>(out + (((size_t)b * SUB_OH + oyr) * SUB_OW + ox) * SUB_C + cbase + dcg * 8, acc);
    }
    __syncthreads();  // the next pass overwrites the slots of rows 2oy-1 .. 2oy+2
  }
}

// FP16 profile: same strip / channel tiling as the FP32 kernel.
//
// conv0 runs on tensor cores (mma.m16n8k16, f16 operands, f32 accumulate):
// rows = 16 positions of one conv0 row, n = 8 channels, k = the 9 taps as six
// pairs of horizontally adjacent input samples -- (ky, kx 0..1) and (ky, kx 2)
// with a zero-weight partner -- so every A-fragment register is one aligned
// 4-byte shared load.  The f32 features enter as f16 hi + lo parts (two MMAs
// into one f32 accumulator), so the products keep f32-level precision.
//
// Input planes: after the f32 strip is staged (mel bin c at float index
// c + 1 of its row, bins -1 and 128 zero), each 8-byte slot s -- bins 2s-1
// and 2s -- is rewritten in place as {hi(2s-1), hi(2s), lo(2s-1), lo(2s)}.
// The depthwise stage reads the conv0 ring as f16 (its values are rounded to
// f16 by the reference already): thread = (output x, 4 channels), taps in
// registers, one 8-byte load per tap; the 96-byte position pitch keeps the
// stride-2 loads of a half-warp (2 positions x 8 channel groups) on distinct
// banks.
constexpr int C0H_ROW_WORDS = 138;  // 4-byte words per plane row (130 used; 138 % 32 == 10: conflict-free)
constexpr int C0H_PLANE_BYTES = (C0_IN_ROWS * C0H_ROW_WORDS * 4 + 15) / 16 * 16;
constexpr int C0H_POS = 48;  // halves per conv0 position in the ring (32 channels + 16 padding)
constexpr int C0H_RING = 3;  // conv0 rows 2oy-1 .. 2oy+1 of one depthwise row
constexpr int C0H_RING_HALVES = C0H_RING * SUB_CW * C0H_POS;
constexpr int C0H_SMEM = C0H_PLANE_BYTES + C0H_RING_HALVES * 2 + 2 * C0_CG * 4;
static_assert(C0H_PLANE_BYTES % 16 == 0 && (C0H_RING_HALVES * 2) % 16 == 0, "FP16 conv0 layout alignment");

__device__ __forceinline__ uint2 lds64(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}

__global__ void __launch_bounds__(256, 3) conv0_dw2_f16_kernel(const float* __restrict__ fbank,
                                                               const __half* __restrict__ w0,
                                                               const float* __restrict__ b0,
                                                               const __half* __restrict__ wd,
                                                               const float* __restrict__ bd,
                                                               const uint32_t* __restrict__ feature_lengths,
                                                               __half* __restrict__ out) {
  pdl_entry();
  extern __shared__ __align__(16) float sub_smem[];
  float* plane = sub_smem;  // [C0_IN_ROWS][C0H_ROW_WORDS]
  __half* ring = reinterpret_cast<__half*>(reinterpret_cast<uint8_t*>(sub_smem) + C0H_PLANE_BYTES);
  float* bias0_s = reinterpret_cast<float*>(ring + C0H_RING_HALVES);  // [32] conv0 bias
  float* biasd_s = bias0_s + C0_CG;                                    // [32] depthwise bias
  const int b = blockIdx.z;
  const int oy0 = blockIdx.y * C0_SR;
  const int oy_end = min(oy0 + C0_SR, SUB_OH);
  const int cbase = blockIdx.x * C0_CG;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int raw = (int)feature_lengths[b];
  const int vin = sub_len(raw, 1), vout = sub_len(raw, 2);
  const int y_first = 2 * oy0 - 1;       // first conv0 row of the strip
  const int iy_first = 2 * y_first - 1;  // first input time sample
  // Stage the strip: 4-byte asynchronous copies, all in flight at once,
  // consecutive threads walking time (contiguous in the feature-major log-mel).
  // Item i = x * C0_IN_ROWS + r; (r, x) advance by the stride's quotient and
  // remainder instead of a division per item.
  constexpr int STEP_R = 256 % C0_IN_ROWS, STEP_X = 256 / C0_IN_ROWS;
  for (int i = tid, r = tid % C0_IN_ROWS, x = tid / C0_IN_ROWS; i < C0_IN_ROWS * SUB_IW; i += 256) {
    const int iy = iy_first + r;
    const bool in_range = iy >= 0 && iy < SUB_IH;
    const float* src = fbank + ((size_t)b * SUB_IW + x) * SUB_IH + (in_range ? iy : 0);
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_addr(plane + r * C0H_ROW_WORDS + x + 1)),
                 "l"(src), "r"(in_range ? 4 : 0)
                 : "memory");
    r += STEP_R;
    x += STEP_X;
    if (r >= C0_IN_ROWS) {
      r -= C0_IN_ROWS;
      ++x;
    }
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  for (int r = tid; r < C0_IN_ROWS; r += 256) {  // mel bins -1 and 128
    plane[r * C0H_ROW_WORDS] = 0.0f;
    plane[r * C0H_ROW_WORDS + SUB_IW + 1] = 0.0f;
  }
  if (tid < C0_CG) {
    bias0_s[tid] = b0[cbase + tid];
    biasd_s[tid] = bd[cbase + tid];
  }
  const int g = lane >> 2, t = lane & 3;
  // B fragments: lane (g, t) holds k = 2t, 2t+1 (pair t) and 2t+8, 2t+9
  // (pair t + 4) of channel cbase + 8 nt + g.  Pair p < 6: ky = p / 2; even p
  // = taps (ky, 0), (ky, 1); odd p = tap (ky, 2) and a zero weight.
  uint32_t bw[4][2];
#pragma unroll
  for (int nt = 0; nt < 4; ++nt) {
    const int ch = cbase + nt * 8 + g;
    auto wtap = [&](int p, int second) {
      if (p >= 6 || ((p & 1) && second)) return __float2half(0.0f);
      const int ky = p >> 1, kx = (p & 1) ? 2 : second;
      return w0[(ky * 3 + kx) * SUB_C + ch];
    };
    bw[nt][0] = pack_h2(wtap(t, 0), wtap(t, 1));
    bw[nt][1] = pack_h2(wtap(t + 4, 0), wtap(t + 4, 1));
  }
  // Depthwise: thread = (output x, channels 4 dq .. 4 dq + 3).
  const int ox = warp * 4 + (lane >> 3), dq = lane & 7;
  float2 wdr[9][2];  // channel pairs (4 dq, 4 dq + 1), (4 dq + 2, 4 dq + 3)
#pragma unroll
  for (int k = 0; k < 9; ++k)
#pragma unroll
    for (int j = 0; j < 2; ++j)
      wdr[k][j] = make_float2(__half2float(wd[k * SUB_C + cbase + 4 * dq + 2 * j]),
                              __half2float(wd[k * SUB_C + cbase + 4 * dq + 2 * j + 1]));
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();
  // In place: f32 pairs -> {hi pair, lo pair}; consecutive threads walk rows.
  for (int i = tid, r = tid % C0_IN_ROWS, sl = tid / C0_IN_ROWS; i < C0_IN_ROWS * (SUB_IW / 2 + 1); i += 256) {
    float2* slot = reinterpret_cast<float2*>(plane + r * C0H_ROW_WORDS) + sl;
    const float2 v = *slot;
    const __half2 hi = __floats2half2_rn(v.x, v.y);
    const float2 hf = __half22float2(hi);
    const __half2 lo = __floats2half2_rn(v.x - hf.x, v.y - hf.y);
    uint2 packed;
    packed.x = *reinterpret_cast<const uint32_t*>(&hi);
    packed.y = *reinterpret_cast<const uint32_t*>(&lo);
    *reinterpret_cast<uint2*>(slot) = packed;
    r += STEP_R;
    sl += STEP_X;
    if (r >= C0_IN_ROWS) {
      r -= C0_IN_ROWS;
      ++sl;
    }
  }
  __syncthreads();

  const uint32_t plane_addr = smem_addr(plane);
  // conv0 row y, output positions x0 .. x0+15, all 32 channels, by one warp
  // -> ring slot y % 3 (ReLU, rounded to f16; rows past the valid length are
  // zero).
  auto conv0_mma = [&](int y, int x0) {
    float acc[4][4];
    const bool live = y >= 0 && y < SUB_CH && y < vin;
    if (live) {
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const float2 bb = *reinterpret_cast<const float2*>(bias0_s + nt * 8 + 2 * t);
        acc[nt][0] = acc[nt][2] = bb.x;
        acc[nt][1] = acc[nt][3] = bb.y;
      }
      // Pair t at rows ky = t / 2, slot x + (t & 1); pair t + 4 (t < 2) at ky = 2.
      const int xa = x0 + g;
      const uint32_t row0 = plane_addr + (uint32_t)((2 * y - 1 - iy_first) * C0H_ROW_WORDS * 4);
      const uint32_t ra = row0 + (uint32_t)((t >> 1) * C0H_ROW_WORDS * 4 + (xa + (t & 1)) * 8);
      const uint2 pa = lds64(ra), pb = lds64(ra + 64);  // positions xa, xa + 8
      uint2 qa = make_uint2(0u, 0u), qb = make_uint2(0u, 0u);
      if (t < 2) {
        const uint32_t rq = row0 + (uint32_t)(2 * C0H_ROW_WORDS * 4 + (xa + t) * 8);
        qa = lds64(rq);
        qb = lds64(rq + 64);
      }
      const uint32_t ahi[4] = {pa.x, pb.x, qa.x, qb.x};
      const uint32_t alo[4] = {pa.y, pb.y, qa.y, qb.y};
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        mma_16816(acc[nt], ahi, bw[nt][0], bw[nt][1]);
        mma_16816(acc[nt], alo, bw[nt][0], bw[nt][1]);
      }
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[nt][e] = fmaxf(acc[nt][e], 0.0f);
    } else {
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[nt][e] = 0.0f;
    }
    __half* slot = ring + (y + C0H_RING) % C0H_RING * (SUB_CW * C0H_POS);
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      *reinterpret_cast<__half2*>(slot + (x0 + g) * C0H_POS + nt * 8 + 2 * t) =
          __floats2half2_rn(acc[nt][0], acc[nt][1]);
      *reinterpret_cast<__half2*>(slot + (x0 + g + 8) * C0H_POS + nt * 8 + 2 * t) =
          __floats2half2_rn(acc[nt][2], acc[nt][3]);
    }
  };

  if (warp < 4) conv0_mma(y_first, warp * 16);
  const int y_last = 2 * oy_end - 1;  // last conv0 row this strip needs
  // One depthwise row per pass: conv0 rows 2oy, 2oy+1 (8 warps = 2 rows x 4
  // position tiles), one barrier, the depthwise row, one barrier.
#pragma unroll 1
  for (int oy = oy0; oy < oy_end; ++oy) {
    const int y = 2 * oy + (warp >> 2);
    if (y <= y_last) conv0_mma(y, (warp & 3) * 16);
    __syncthreads();
    // Per channel an fma chain from the bias in tap order (ky outer, kx
    // inner), two channels per paired FMA.
    float2 acc01, acc23;
    if (oy >= vout) {
      acc01 = acc23 = make_float2(0.0f, 0.0f);
    } else {
      const float4 bq = *reinterpret_cast<const float4*>(biasd_s + 4 * dq);
      acc01 = make_float2(bq.x, bq.y);
      acc23 = make_float2(bq.z, bq.w);
#pragma unroll
      for (int ky = 0; ky < 3; ++ky) {
        const int iy = oy * 2 + ky - 1;
        if (iy < 0 || iy >= SUB_CH || iy >= vin) continue;
        const __half* rowp = ring + (iy % C0H_RING) * (SUB_CW * C0H_POS) + 4 * dq;
#pragma unroll
        for (int kx = 0; kx < 3; ++kx) {
          const int ix = ox * 2 + kx - 1;  // <= 63
          if (ix < 0) continue;
          const uint2 raw2 = *reinterpret_cast<const uint2*>(rowp + ix * C0H_POS);
          acc01 = ffma2(__half22float2(*reinterpret_cast<const __half2*>(&raw2.x)), wdr[ky * 3 + kx][0], acc01);
          acc23 = ffma2(__half22float2(*reinterpret_cast<const __half2*>(&raw2.y)), wdr[ky * 3 + kx][1], acc23);
        }
      }
    }
    const __half2 o01 = __floats2half2_rn(acc01.x, acc01.y), o23 = __floats2half2_rn(acc23.x, acc23.y);
    uint2 packed;
    packed.x = *reinterpret_cast<const uint32_t*>(&o01);
    packed.y = *reinterpret_cast<const uint32_t*>(&o23);
    *reinterpret_cast<uint2*>(out + (((size_t)b * SUB_OH + oy) * SUB_OW + ox) * SUB_C + cbase + 4 * dq) = packed;
    __syncthreads();  // the next pass overwrites the slots of rows 2oy-1, 2oy
  }
}

// Depthwise 3x3 stride 2 pad 1 + bias, channel-last; one thread per output
// pixel and 8 channels.
template <typename T>
__global__ void __launch_bounds__(256) depthwise_kernel(const T* __restrict__ in, const T* __restrict__ w,
                                                        const float* __restrict__ bias,
                                                        const uint32_t* __restrict__ feature_lengths,
                                                        T* __restrict__ out, int batch, int ih, int iw,
                                                        int channels, int steps) {
  pdl_entry();
  const int oh = (ih - 1) / 2 + 1, ow = (iw - 1) / 2 + 1;
  const int cv = channels / 8;
  const int64_t total = (int64_t)batch * oh * ow * cv;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int c = (int)(i % cv) * 8;
  const int ox = (int)((i / cv) % ow);
  const int oy = (int)((i / ((int64_t)cv * ow)) % oh);
  const int b = (int)(i / ((int64_t)cv * ow * oh));
  const int raw = (int)feature_lengths[b];
  const int vin = sub_len(raw, steps - 1), vout = sub_len(raw, steps);
  T* dst = out + (((int64_t)b * oh + oy) * ow + ox) * channels + c;
  float acc[8];
  if (oy >= vout) {
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
    store8<T>(dst, acc);
    return;
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = __ldg(bias + c + j);
  // Channel pairs share one paired FMA (each lane exactly fmaf).
  float2* acc2 = reinterpret_cast<float2*>(acc);
#pragma unroll
  for (int ky = 0; ky < 3; ++ky) {
    const int iy = oy * 2 + ky - 1;
    if (iy < 0 || iy >= ih || iy >= vin) continue;
#pragma unroll
    for (int kx = 0; kx < 3; ++kx) {
      const int ix = ox * 2 + kx - 1;
      if (ix < 0 || ix >= iw) continue;
      float v[8], wk[8];
      load8<T>(in + (((int64_t)b * ih + iy) * iw + ix) * channels + c, v);
      load8<T>(w + (ky * 3 + kx) * channels + c, wk);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        acc2[j] = ffma2(make_float2(v[2 * j], v[2 * j + 1]), make_float2(wk[2 * j], wk[2 * j + 1]), acc2[j]);
    }
  }
  store8<T>(dst, acc);
}

template <typename T>
__global__ void time_mask_kernel(T* __restrict__ values, const uint32_t* __restrict__ feature_lengths, int height,
                                 int row_elems, int steps) {
  pdl_entry();
  const int frame = blockIdx.x, b = blockIdx.y;
  if (frame < sub_len((int)feature_lengths[b], steps)) return;
  T* row = values + ((size_t)b * height + frame) * row_elems;
  for (int i = threadIdx.x; i < row_elems; i += blockDim.x) row[i] = (T)0.0f;
}

int launch_subsampling_conv0_dw2(int precision, int batch, const float* features, const void* conv0_w,
                                 const float* conv0_b, const void* dw_w, const float* dw_b,
                                 const uint32_t* feature_lengths, void* out, cudaStream_t stream) {
  if (precision == PK_FP16 && g_reference_arith)
    return launch_ref_conv0_dw2(batch, features, conv0_w, conv0_b, dw_w, dw_b, feature_lengths, out, stream);
  const dim3 grid(SUB_C / C0_CG, C0_STRIPS, batch);
  if (precision == PK_FP16) {
    int st = set_max_dynamic_smem(reinterpret_cast<const void*>(conv0_dw2_f16_kernel), C0H_SMEM);
    if (st != PK_OK) return st;
    launch_kernel(conv0_dw2_f16_kernel, grid, 256, C0H_SMEM, stream, features, static_cast<const __half*>(conv0_w),
                  conv0_b, static_cast<const __half*>(dw_w), dw_b, feature_lengths, static_cast<__half*>(out));
  } else {
    int st = set_max_dynamic_smem(reinterpret_cast<const void*>(conv0_dw2_f32_kernel), C0_SMEM);
    if (st != PK_OK) return st;
    launch_kernel(conv0_dw2_f32_kernel, grid, 256, C0_SMEM, stream, features, static_cast<const float*>(conv0_w),
                  conv0_b, static_cast<const float*>(dw_w), dw_b, feature_lengths, static_cast<float*>(out));
  }
  return cuda_error(cudaGetLastError(), "subsampling conv0+dw2 launch");
}

int launch_subsampling_depthwise(int precision, int batch, int ih, int iw, int channels, const void* input,
                                 const void* w, const float* b, const uint32_t* feature_lengths, int steps,
                                 void* out, cudaStream_t stream) {
  if (precision == PK_FP16 && g_reference_arith)
    return launch_ref_depthwise(batch, ih, iw, channels, input, w, b, feature_lengths, steps, out, stream);
  if (channels % 8 != 0) return set_error(PK_E_SHAPE, "depthwise subsampling needs channels %% 8 == 0");
  const int oh = (ih - 1) / 2 + 1, ow = (iw - 1) / 2 + 1;
  const int64_t total = (int64_t)batch * oh * ow * (channels / 8);
  const unsigned blocks = (unsigned)((total + 255) / 256);
  if (precision == PK_FP16)
    launch_kernel(depthwise_kernel<__half>, blocks, 256, 0, stream, static_cast<const __half*>(input),
                                                         static_cast<const __half*>(w), b, feature_lengths,
                                                         static_cast<__half*>(out), batch, ih, iw, channels, steps);
  else
    launch_kernel(depthwise_kernel<float>, blocks, 256, 0, stream, static_cast<const float*>(input),
                                                        static_cast<const float*>(w), b, feature_lengths,
                                                        static_cast<float*>(out), batch, ih, iw, channels, steps);
  return cuda_error(cudaGetLastError(), "subsampling depthwise launch");
}

int launch_subsampling_time_mask(int precision, int batch, int height, int width, int channels, void* values,
                                 const uint32_t* feature_lengths, int steps, cudaStream_t stream) {
  const dim3 grid(height, batch);
  if (precision == PK_FP16)
    launch_kernel(time_mask_kernel<__half>, grid, 256, 0, stream, static_cast<__half*>(values), feature_lengths, height,
                                                       width * channels, steps);
  else
    launch_kernel(time_mask_kernel<float>, grid, 256, 0, stream, static_cast<float*>(values), feature_lengths, height,
                                                      width * channels, steps);
  return cuda_error(cudaGetLastError(), "subsampling time mask launch");
}

}  // namespace pk
