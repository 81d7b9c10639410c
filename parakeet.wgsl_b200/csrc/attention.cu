// attention.cu -- fused relative-position multi-head self-attention.
//
// Restates RELATIVE_ATTENTION_WGSL (src/webgpu/kernels/attention.ts:418-728)
// for 8 heads of 128 channels:
//   s_ij = (sum over 32 vec4 of fma((q_i+u).x, k_j.x), fma((q_i+v).x,
//           p[T-1-i+j].x), ... interleaved per component) * 1/sqrt(128)
//   keys j >= valid get -3.402823466e38; f32 softmax over keys;
//   ctx_i = fma chain over j of prob_ij * v_j; rows i >= valid are zero.
// qkv [B*T, 3072] (q | k | v per row), projected positions in the
// head-vector-position-vec4 layout [8][32][2T-1][4] (model/convert.py:
// 1195-1228), bias_u / bias_v f32 [8, 128].
// One CTA = (query block of QB queries, head, window).  Scores stay on chip
// (no O(T^2) tensor in HBM).  Requires T <= 192 like the reference
// (attention.ts:224-228).
#include "pk_common.cuh"
#include "pk_internal.h"

namespace pk {

constexpr int ATT_QB = 8;        // queries per CTA
constexpr int ATT_MAXT = 192;
constexpr int ATT_THREADS = 256;

template <typename T>
__device__ __forceinline__ void ld4(const T* p, float* v);
template <>
__device__ __forceinline__ void ld4<__half>(const __half* p, float* v) {
  const uint2 raw = __ldg(reinterpret_cast<const uint2*>(p));
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
  v[0] = a.x;
  v[1] = a.y;
  v[2] = b.x;
  v[3] = b.y;
}
template <>
__device__ __forceinline__ void ld4<float>(const float* p, float* v) {
  const float4 f = __ldg(reinterpret_cast<const float4*>(p));
  v[0] = f.x;
  v[1] = f.y;
  v[2] = f.z;
  v[3] = f.w;
}

template <typename T>
__global__ void __launch_bounds__(ATT_THREADS) rel_attention_simt_kernel(
    const T* __restrict__ qkv, const T* __restrict__ positions, const float* __restrict__ bias_u,
    const float* __restrict__ bias_v, const uint32_t* __restrict__ valid_lengths, T* __restrict__ context,
    int frames) {
  __shared__ float qu[ATT_QB][128], qv[ATT_QB][128];
  __shared__ float probs[ATT_QB][ATT_MAXT];
  const int q0 = blockIdx.x * ATT_QB, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x;
  const int valid = min((int)valid_lengths[b], frames);
  const int P = 2 * frames - 1;
  const size_t row0 = (size_t)b * frames;
  for (int i = tid; i < ATT_QB * 128; i += ATT_THREADS) {
    const int qs = i / 128, d = i % 128, q = q0 + qs;
    float v = 0.0f;
    if (q < frames) v = (float)qkv[(row0 + q) * 3072 + h * 128 + d];
    qu[qs][d] = v + bias_u[h * 128 + d];
    qv[qs][d] = v + bias_v[h * 128 + d];
  }
  __syncthreads();
  // Scores: thread j owns key j for all queries of the block.
  const int j = tid;
  if (j < frames) {
    float s[ATT_QB];
#pragma unroll
    for (int qs = 0; qs < ATT_QB; ++qs) s[qs] = 0.0f;
    if (j < valid) {
      const T* krow = qkv + (row0 + j) * 3072 + 1024 + h * 128;
      for (int vec = 0; vec < 32; ++vec) {
        float k4[4];
        ld4<T>(krow + vec * 4, k4);
        const T* pbase = positions + ((size_t)(h * 32 + vec) * P) * 4;
#pragma unroll
        for (int qs = 0; qs < ATT_QB; ++qs) {
          const int q = q0 + qs;
          if (q < valid) {
            float p4[4];
            ld4<T>(pbase + (size_t)(frames - 1 - q + j) * 4, p4);
            float r = s[qs];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              r = fmaf(qu[qs][vec * 4 + c], k4[c], r);
              r = fmaf(qv[qs][vec * 4 + c], p4[c], r);
            }
            s[qs] = r;
          }
        }
      }
    }
    const float scale = 0.08838834764831845f;  // 1 / sqrt(128)
#pragma unroll
    for (int qs = 0; qs < ATT_QB; ++qs) probs[qs][j] = j < valid ? s[qs] * scale : -3.402823466e+38f;
  }
  __syncthreads();
  // Softmax: warp w normalizes query w's row.
  const int warp = tid >> 5, lane = tid & 31;
  if (warp < ATT_QB && q0 + warp < valid) {
    float mx = -3.402823466e+38f;
    for (int jj = lane; jj < frames; jj += 32) mx = fmaxf(mx, probs[warp][jj]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.0f;
    for (int jj = lane; jj < frames; jj += 32) {
      const float e = jj < valid ? expf(probs[warp][jj] - mx) : 0.0f;
      probs[warp][jj] = e;
      sum += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float inv = 1.0f / sum;
    for (int jj = lane; jj < frames; jj += 32) probs[warp][jj] *= inv;
  }
  __syncthreads();
  // Context: thread -> (query slot, 4-channel vector).
  for (int i = tid; i < ATT_QB * 32; i += ATT_THREADS) {
    const int qs = i / 32, vec = i % 32, q = q0 + qs;
    if (q >= frames) continue;
    float o[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (q < valid) {
      const T* vcol = qkv + row0 * 3072 + 2048 + h * 128 + vec * 4;
      for (int jj = 0; jj < valid; ++jj) {
        float v4[4];
        ld4<T>(vcol + (size_t)jj * 3072, v4);
        const float p = probs[qs][jj];
#pragma unroll
        for (int c = 0; c < 4; ++c) o[c] = fmaf(p, v4[c], o[c]);
      }
    }
    T* dst = context + (row0 + q) * 1024 + h * 128 + vec * 4;
#pragma unroll
    for (int c = 0; c < 4; ++c) dst[c] = (T)o[c];
  }
}

// ---------------------------------------------------------------------------
// FP16 package: tensor-core version (mma.sync m16n8k16, f16 operands, f32
// accumulation).  One CTA = (64 queries, head, window), 4 warps x 16 queries.
//   * K [192 x 128] and the band of projected positions the block needs
//     (rows T-64-q0 .. T-1-q0+191, 256 rows) are staged in shared memory;
//   * BD: each warp computes (q+v)[16 x 128] . P_band[208 rows]^T once into a
//     per-warp scratch; the relative shift becomes an index remap:
//     s_bd(i, j) = scratch[i][j + 15 - i];
//   * AC: (q+u) . K^T per 8-key tile, combined with the shifted BD, scaled,
//     masked and soft-maxed in registers (f32);
//   * PV: probabilities (f16, already normalized) . V, with V staged into the
//     positions' buffer (cp.async, overlapped with AC + softmax).
// (q+u) / (q+v) and the probabilities are rounded to f16 for the MMA; scores,
// softmax and accumulation stay f32.
// ---------------------------------------------------------------------------
constexpr int TA_QB = 64;
constexpr int TA_KEYS = 192;
constexpr int TA_STRIDE = 136;  // halves per shared row (128 + 8: conflict-free fragment loads)
constexpr int TA_PROWS = 256;
constexpr int TA_BDW = 208;     // BD columns per warp (26 n-tiles)
constexpr int TA_THREADS = 128;
constexpr int TA_SMEM = (TA_KEYS + TA_PROWS) * TA_STRIDE * 2 + 4 * 16 * TA_BDW * 4;

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                                  uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void cp_async16(uint32_t saddr, const void* gptr) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr), "l"(gptr) : "memory");
}

// A fragments of (q + bias) for 16 query rows starting at i0 (rows >= frames
// read as zero).  frag[ks] covers dims ks*16 .. ks*16+15.
__device__ __forceinline__ void load_q_frags(uint32_t (&frag)[8][4], const __half* __restrict__ qkv,
                                             const float* __restrict__ bias, size_t row0, int i0, int frames,
                                             int h, int g, int t) {
  const int r0 = i0 + g, r1 = i0 + g + 8;
  const __half* q0 = qkv + (row0 + (size_t)min(r0, frames - 1)) * 3072 + h * 128;
  const __half* q1 = qkv + (row0 + (size_t)min(r1, frames - 1)) * 3072 + h * 128;
  const float* bb = bias + h * 128;
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int d = ks * 16 + half * 8 + 2 * t;
      const float2 b2 = *reinterpret_cast<const float2*>(bb + d);
      float2 x0 = __half22float2(*reinterpret_cast<const __half2*>(q0 + d));
      float2 x1 = __half22float2(*reinterpret_cast<const __half2*>(q1 + d));
      if (r0 >= frames) x0 = make_float2(0.0f, 0.0f);
      if (r1 >= frames) x1 = make_float2(0.0f, 0.0f);
      frag[ks][half * 2 + 0] = pack_half2(x0.x + b2.x, x0.y + b2.y);
      frag[ks][half * 2 + 1] = pack_half2(x1.x + b2.x, x1.y + b2.y);
    }
  }
}

__global__ void __launch_bounds__(TA_THREADS) rel_attention_tc_kernel(
    const __half* __restrict__ qkv, const __half* __restrict__ positions, const float* __restrict__ bias_u,
    const float* __restrict__ bias_v, const uint32_t* __restrict__ valid_lengths, __half* __restrict__ context,
    int frames) {
  extern __shared__ __align__(16) uint8_t ta_smem[];
  __half* Ks = reinterpret_cast<__half*>(ta_smem);
  __half* PVs = Ks + TA_KEYS * TA_STRIDE;
  float* BDs = reinterpret_cast<float*>(PVs + TA_PROWS * TA_STRIDE);
  const int q0 = blockIdx.x * TA_QB, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int valid = min((int)valid_lengths[b], frames);
  const size_t row0 = (size_t)b * frames;
  const int P = 2 * frames - 1;
  const int qend = min(q0 + TA_QB, frames);
  if (q0 >= valid) {  // whole block masked: zero its context rows
    for (int i = tid; i < (qend - q0) * 16; i += TA_THREADS) {
      const int q = q0 + i / 16, c = (i % 16) * 8;
      *reinterpret_cast<uint4*>(context + (row0 + q) * 1024 + h * 128 + c) = make_uint4(0, 0, 0, 0);
    }
    return;
  }
  // ---- stage K rows (zero past T) and the positional band
  for (int i = tid; i < TA_KEYS * 16; i += TA_THREADS) {
    const int j = i >> 4, c = (i & 15) * 8;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (j < frames) v = *reinterpret_cast<const uint4*>(qkv + (row0 + j) * 3072 + 1024 + h * 128 + c);
    *reinterpret_cast<uint4*>(Ks + j * TA_STRIDE + c) = v;
  }
  const int band0 = frames - TA_QB - q0;  // relative index of band row 0
  for (int i = tid; i < TA_PROWS * 32; i += TA_THREADS) {
    const int r = i % TA_PROWS, vec = i / TA_PROWS, rel = band0 + r;
    uint2 v = make_uint2(0, 0);
    if (rel >= 0 && rel < P) v = *reinterpret_cast<const uint2*>(positions + ((size_t)(h * 32 + vec) * P + rel) * 4);
    *reinterpret_cast<uint2*>(PVs + r * TA_STRIDE + vec * 4) = v;
  }
  __syncthreads();

  const int i0 = q0 + warp * 16;
  const bool active = i0 < valid;
  float* bd = BDs + warp * 16 * TA_BDW;
  uint32_t qf[8][4];
  if (active) {
    // ---- BD band: (q+v) . P[band]^T -> scratch
    load_q_frags(qf, qkv, bias_v, row0, i0, frames, h, g, t);
    const int wb = 48 - 16 * warp;  // this warp's first band row
#pragma unroll 2
    for (int nt = 0; nt < TA_BDW / 8; ++nt) {
      float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      const __half* prow = PVs + (wb + nt * 8 + g) * TA_STRIDE + 2 * t;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(prow + ks * 16);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(prow + ks * 16 + 8);
        mma16816(acc, qf[ks], b0, b1);
      }
      bd[g * TA_BDW + nt * 8 + 2 * t] = acc[0];
      bd[g * TA_BDW + nt * 8 + 2 * t + 1] = acc[1];
      bd[(g + 8) * TA_BDW + nt * 8 + 2 * t] = acc[2];
      bd[(g + 8) * TA_BDW + nt * 8 + 2 * t + 1] = acc[3];
    }
  }
  __syncthreads();  // every warp is done with the positional band
  // ---- stage V into the band buffer (overlaps AC + softmax)
  for (int i = tid; i < TA_KEYS * 16; i += TA_THREADS) {
    const int j = i >> 4, c = (i & 15) * 8;
    const uint32_t dst = smem_addr(PVs + j * TA_STRIDE + c);
    if (j < valid) cp_async16(dst, qkv + (row0 + j) * 3072 + 2048 + h * 128 + c);
    else *reinterpret_cast<uint4*>(PVs + j * TA_STRIDE + c) = make_uint4(0, 0, 0, 0);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");

  float s[TA_KEYS / 8][4];
  uint32_t pf[TA_KEYS / 16][4];
  if (active) {
    // ---- AC scores + shifted BD, scale, mask, softmax
    load_q_frags(qf, qkv, bias_u, row0, i0, frames, h, g, t);
    const float scale = 0.08838834764831845f;  // 1 / sqrt(128)
    float mx0 = -3.402823466e+38f, mx1 = -3.402823466e+38f;
#pragma unroll
    for (int nt = 0; nt < TA_KEYS / 8; ++nt) {
      float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      const __half* krow = Ks + (nt * 8 + g) * TA_STRIDE + 2 * t;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(krow + ks * 16);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(krow + ks * 16 + 8);
        mma16816(acc, qf[ks], b0, b1);
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = g + (e >> 1) * 8;           // row within the warp's 16 queries
        const int j = nt * 8 + 2 * t + (e & 1);   // key
        float v = (acc[e] + bd[r * TA_BDW + j + 15 - r]) * scale;
        if (j >= valid) v = -3.402823466e+38f;
        s[nt][e] = v;
      }
      mx0 = fmaxf(mx0, fmaxf(s[nt][0], s[nt][1]));
      mx1 = fmaxf(mx1, fmaxf(s[nt][2], s[nt][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    float sum0 = 0.0f, sum1 = 0.0f;
#pragma unroll
    for (int nt = 0; nt < TA_KEYS / 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int j = nt * 8 + 2 * t + (e & 1);
        const float p = j < valid ? expf(s[nt][e] - (e < 2 ? mx0 : mx1)) : 0.0f;
        s[nt][e] = p;
        if (e < 2) sum0 += p;
        else sum1 += p;
      }
    }
    sum0 += __shfl_xor_sync(0xffffffffu, sum0, 1);
    sum0 += __shfl_xor_sync(0xffffffffu, sum0, 2);
    sum1 += __shfl_xor_sync(0xffffffffu, sum1, 1);
    sum1 += __shfl_xor_sync(0xffffffffu, sum1, 2);
    const float inv0 = 1.0f / sum0, inv1 = 1.0f / sum1;
#pragma unroll
    for (int kk = 0; kk < TA_KEYS / 16; ++kk) {
      pf[kk][0] = pack_half2(s[2 * kk][0] * inv0, s[2 * kk][1] * inv0);
      pf[kk][1] = pack_half2(s[2 * kk][2] * inv1, s[2 * kk][3] * inv1);
      pf[kk][2] = pack_half2(s[2 * kk + 1][0] * inv0, s[2 * kk + 1][1] * inv0);
      pf[kk][3] = pack_half2(s[2 * kk + 1][2] * inv1, s[2 * kk + 1][3] * inv1);
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();  // V staged
  if (!active) {
    // Rows of this warp are all past the valid length: zero them.
    for (int i = lane; i < 16 * 16; i += 32) {
      const int q = i0 + i / 16, c = (i % 16) * 8;
      if (q < frames)
        *reinterpret_cast<uint4*>(context + (row0 + q) * 1024 + h * 128 + c) = make_uint4(0, 0, 0, 0);
    }
    return;
  }
  // ---- PV
  float o[16][4];
#pragma unroll
  for (int dt = 0; dt < 16; ++dt)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[dt][e] = 0.0f;
  const int lr = lane & 7, lm = lane >> 3;  // ldmatrix row / matrix index
#pragma unroll
  for (int kk = 0; kk < TA_KEYS / 16; ++kk) {
#pragma unroll
    for (int dp = 0; dp < 8; ++dp) {  // pairs of 8-dim tiles
      const int key = kk * 16 + (lm & 1) * 8 + lr;
      const int dim = dp * 16 + (lm >> 1) * 8;
      uint32_t b00, b01, b10, b11;
      ldmatrix_x4_trans(smem_addr(PVs + key * TA_STRIDE + dim), b00, b01, b10, b11);
      mma16816(o[2 * dp], pf[kk], b00, b01);
      mma16816(o[2 * dp + 1], pf[kk], b10, b11);
    }
  }
  const int ra = i0 + g, rb = i0 + g + 8;
#pragma unroll
  for (int dt = 0; dt < 16; ++dt) {
    const int d = h * 128 + dt * 8 + 2 * t;
    if (ra < frames)
      *reinterpret_cast<uint32_t*>(context + (row0 + ra) * 1024 + d) =
          ra < valid ? pack_half2(o[dt][0], o[dt][1]) : 0u;
    if (rb < frames)
      *reinterpret_cast<uint32_t*>(context + (row0 + rb) * 1024 + d) =
          rb < valid ? pack_half2(o[dt][2], o[dt][3]) : 0u;
  }
}

int launch_rel_attention(const DeviceCtx& dev, int precision, int batch, int frames, const void* qkv,
                         const void* positions, const float* bias_u, const float* bias_v,
                         const uint32_t* valid_lengths, void* context, cudaStream_t stream) {
  if (precision == PK_FP16 && g_attention_route != 1) {
    static int configured[32] = {};
    if (dev.ordinal < 0 || dev.ordinal >= 32 || !configured[dev.ordinal]) {
      cudaError_t e =
          cudaFuncSetAttribute(rel_attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, TA_SMEM);
      if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(rel_attention_tc)");
      if (dev.ordinal >= 0 && dev.ordinal < 32) configured[dev.ordinal] = 1;
    }
    const dim3 grid((frames + TA_QB - 1) / TA_QB, 8, batch);
    rel_attention_tc_kernel<<<grid, TA_THREADS, TA_SMEM, stream>>>(
        static_cast<const __half*>(qkv), static_cast<const __half*>(positions), bias_u, bias_v, valid_lengths,
        static_cast<__half*>(context), frames);
    return cuda_error(cudaGetLastError(), "rel_attention_tc launch");
  }
  const dim3 grid((frames + ATT_QB - 1) / ATT_QB, 8, batch);
  if (precision == PK_FP16)
    rel_attention_simt_kernel<__half><<<grid, ATT_THREADS, 0, stream>>>(
        static_cast<const __half*>(qkv), static_cast<const __half*>(positions), bias_u, bias_v, valid_lengths,
        static_cast<__half*>(context), frames);
  else
    rel_attention_simt_kernel<float><<<grid, ATT_THREADS, 0, stream>>>(
        static_cast<const float*>(qkv), static_cast<const float*>(positions), bias_u, bias_v, valid_lengths,
        static_cast<float*>(context), frames);
  return cuda_error(cudaGetLastError(), "rel_attention launch");
}

}  // namespace pk
