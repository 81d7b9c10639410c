// attention_tc.cu -- FP16 relative-position MHSA on tensor cores (mma.sync).
//
// Same arithmetic contract as RELATIVE_ATTENTION_WGSL
// (src/webgpu/kernels/attention.ts:418-728):
//   s_ij = ((q_i+u).k_j + (q_i+v).p[T-1-i+j]) / sqrt(128), keys j >= valid
//   excluded, f32 softmax over keys, ctx_i = sum_j prob_ij v_j, rows i >= valid
//   zero.
// One CTA = (64 queries, head, window), 4 warps x 16 queries, keys processed
// in three 64-key chunks with an online (running max / sum) softmax:
//   per chunk the K rows, V rows and the band of projected positions the
//   chunk needs (rows T-64-q0+j0 .. +127) are staged with cp.async;
//   BD: each warp computes (q+v)[16x128] . P_band[80 rows]^T into a small
//   per-warp scratch and reads it back shifted, s_bd(i, j) =
//   scratch[i][j - j0 + 15 - i];
//   AC: (q+u) . K^T per 8-key tile, + shifted BD, scaled, masked;
//   PV: exp(s - running max) in f16 . V, accumulated in f32 registers.
// 88 KB of shared memory per CTA lets two CTAs share an SM, so one CTA's
// loads overlap the other's MMAs.  (q+u), (q+v) and the probabilities are
// rounded to f16 for the MMA; scores, softmax and accumulation are f32.
#include "pk_common.cuh"
#include "pk_internal.h"

namespace pk {

namespace {

constexpr int AQ = 64;        // queries per CTA
constexpr int AKC = 64;       // keys per chunk
constexpr int ANC = 3;        // chunks (192 keys >= T)
constexpr int AS = 136;       // halves per shared row (128 + 8: conflict-free fragment loads)
constexpr int APR = 128;      // positional band rows per chunk (64 + 63, padded)
constexpr int ABD = 80;       // BD columns per warp per chunk (16 + 63, padded)
constexpr int ATHREADS = 128;
constexpr int ASMEM = (2 * AKC + APR) * AS * 2 + 4 * 16 * ABD * 4;

// Not volatile: no side effects, so the compiler may interleave independent
// accumulator chains.
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// 2^x (hardware approximation, relative error ~2^-22); softmax runs in base
// 2 with log2(e) folded into the score scale.
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
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

// Four 8x8 b16 matrices, row addresses from lanes 8m..8m+7 for matrix m:
// thread (g, t) gets row g, columns 2t, 2t+1 of each -- the B fragment of
// mma.m16n8k16 .col when the rows are keys (positions) and the columns dims.
__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void cp_async16(uint32_t saddr, const void* gptr) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr), "l"(gptr) : "memory");
}
__device__ __forceinline__ void cp_async8(uint32_t saddr, const void* gptr) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(saddr), "l"(gptr) : "memory");
}

// A fragments of (q + bias) for 16 query rows starting at i0 (rows >= frames
// read as zero).  frag[ks] covers dims ks*16 .. ks*16+15.
__device__ __forceinline__ void q_frags(uint32_t (&frag)[8][4], const __half* __restrict__ qkv,
                                        const float* __restrict__ bias, size_t row0, int i0, int frames, int h,
                                        int g, int t) {
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

// ROWMAJOR: positions as [8 heads][2T-1][128] (row-contiguous, re-laid out
// once by the encoder); otherwise the package's head-vector-position-vec4
// layout [8*32 vectors][2T-1][4].
template <bool ROWMAJOR>
__global__ void __launch_bounds__(ATHREADS, 2) rel_attention_flash_kernel(
    const __half* __restrict__ qkv, const __half* __restrict__ positions, const float* __restrict__ bias_u,
    const float* __restrict__ bias_v, const uint32_t* __restrict__ valid_lengths, __half* __restrict__ context,
    int frames) {
  pdl_entry();
  extern __shared__ __align__(16) uint8_t fa_smem[];
  __half* Ks = reinterpret_cast<__half*>(fa_smem);   // [64][AS]
  __half* Vs = Ks + AKC * AS;                         // [64][AS]
  __half* Ps = Vs + AKC * AS;                         // [128][AS]
  float* BDs = reinterpret_cast<float*>(Ps + APR * AS);
  const int q0 = blockIdx.x * AQ, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int valid = min((int)valid_lengths[b], frames);
  const size_t row0 = (size_t)b * frames;
  const int P = 2 * frames - 1;
  const int qend = min(q0 + AQ, frames);
  if (q0 >= valid) {  // whole block masked: zero its context rows
    for (int i = tid; i < (qend - q0) * 16; i += ATHREADS) {
      const int q = q0 + i / 16, c = (i % 16) * 8;
      *reinterpret_cast<uint4*>(context + (row0 + q) * 1024 + h * 128 + c) = make_uint4(0, 0, 0, 0);
    }
    return;
  }
  const int i0 = q0 + warp * 16;
  const bool active = i0 < valid;
  float* bd = BDs + warp * 16 * ABD;
  uint32_t qu[8][4], qv[8][4];
  if (active) {
    q_frags(qu, qkv, bias_u, row0, i0, frames, h, g, t);
    q_frags(qv, qkv, bias_v, row0, i0, frames, h, g, t);
  }
  float o[16][4];
#pragma unroll
  for (int dt = 0; dt < 16; ++dt)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[dt][e] = 0.0f;
  float m0 = -3.402823466e+38f, m1 = -3.402823466e+38f, l0 = 0.0f, l1 = 0.0f;
  const float scale = 0.08838834764831845f * 1.4426950408889634f;  // log2(e) / sqrt(128): base-2 softmax
  const int nchunks = min(ANC, (valid + AKC - 1) / AKC);  // chunks that hold a valid key

  for (int kc = 0; kc < nchunks; ++kc) {
    const int j0 = kc * AKC;
    if (kc > 0) __syncthreads();  // previous chunk's K / V / band no longer read
    // ---- stage K and V rows (zero past T / past valid) and the band
    for (int i = tid; i < AKC * 16; i += ATHREADS) {
      const int jr = i >> 4, c = (i & 15) * 8, j = j0 + jr;
      const size_t src = (row0 + j) * 3072 + h * 128 + c;
      if (j < frames) cp_async16(smem_addr(Ks + jr * AS + c), qkv + src + 1024);
      else *reinterpret_cast<uint4*>(Ks + jr * AS + c) = make_uint4(0, 0, 0, 0);
      if (j < valid) cp_async16(smem_addr(Vs + jr * AS + c), qkv + src + 2048);
      else *reinterpret_cast<uint4*>(Vs + jr * AS + c) = make_uint4(0, 0, 0, 0);
    }
    const int band0 = frames - AQ - q0 + j0;  // relative index of band row 0
    if constexpr (ROWMAJOR) {
      for (int i = tid; i < APR * 16; i += ATHREADS) {
        const int r = i >> 4, c = (i & 15) * 8, rel = band0 + r;
        if (rel >= 0 && rel < P)
          cp_async16(smem_addr(Ps + r * AS + c), positions + ((size_t)h * P + rel) * 128 + c);
        else
          *reinterpret_cast<uint4*>(Ps + r * AS + c) = make_uint4(0, 0, 0, 0);
      }
    } else {
      for (int i = tid; i < APR * 32; i += ATHREADS) {
        const int r = i % APR, vec = i / APR, rel = band0 + r;
        if (rel >= 0 && rel < P)
          cp_async8(smem_addr(Ps + r * AS + vec * 4), positions + ((size_t)(h * 32 + vec) * P + rel) * 4);
        else
          *reinterpret_cast<uint2*>(Ps + r * AS + vec * 4) = make_uint2(0, 0);
      }
    }
    asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    if (!active) continue;

    // ---- BD for this warp's 16 queries x the chunk's 64 keys (+15 diagonal)
    // Two passes of five independent 8-column tiles, k-steps outermost, so
    // consecutive MMAs do not wait on one another's accumulators.
    const int wb = 48 - 16 * warp;  // this warp's first band row
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      float acc[5][4];
#pragma unroll
      for (int u = 0; u < 5; ++u)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[u][e] = 0.0f;
#pragma unroll
      for (int ks = 0; ks < 8; ks += 2) {
#pragma unroll
        for (int u = 0; u < 5; ++u) {
          uint32_t b0, b1, b2, b3;  // dims ks*16 + {0, 8, 16, 24} .. +7 of band rows (half*5+u)*8 ..
          ldmatrix_x4(smem_addr(Ps + (wb + (half * 5 + u) * 8 + (lane & 7)) * AS + ks * 16 + (lane >> 3) * 8), b0,
                      b1, b2, b3);
          mma16816(acc[u], qv[ks], b0, b1);
          mma16816(acc[u], qv[ks + 1], b2, b3);
        }
      }
#pragma unroll
      for (int u = 0; u < 5; ++u) {
        const int c = (half * 5 + u) * 8 + 2 * t;
        *reinterpret_cast<float2*>(bd + g * ABD + c) = make_float2(acc[u][0], acc[u][1]);
        *reinterpret_cast<float2*>(bd + (g + 8) * ABD + c) = make_float2(acc[u][2], acc[u][3]);
      }
    }
    __syncwarp();

    // ---- AC + shifted BD, scale, mask; chunk max
    float s[AKC / 8][4];
#pragma unroll
    for (int nt = 0; nt < AKC / 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[nt][e] = 0.0f;
#pragma unroll
    for (int ks = 0; ks < 8; ks += 2) {
#pragma unroll
      for (int nt = 0; nt < AKC / 8; ++nt) {
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(smem_addr(Ks + (nt * 8 + (lane & 7)) * AS + ks * 16 + (lane >> 3) * 8), b0, b1, b2, b3);
        mma16816(s[nt], qu[ks], b0, b1);
        mma16816(s[nt], qu[ks + 1], b2, b3);
      }
    }
    float cm0 = -3.402823466e+38f, cm1 = -3.402823466e+38f;
#pragma unroll
    for (int nt = 0; nt < AKC / 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = g + (e >> 1) * 8;          // row within the warp's 16 queries
        const int jl = nt * 8 + 2 * t + (e & 1); // key within the chunk
        float v = (s[nt][e] + bd[r * ABD + jl + 15 - r]) * scale;
        if (j0 + jl >= valid) v = -3.402823466e+38f;
        s[nt][e] = v;
      }
      cm0 = fmaxf(cm0, fmaxf(s[nt][0], s[nt][1]));
      cm1 = fmaxf(cm1, fmaxf(s[nt][2], s[nt][3]));
    }
    __syncwarp();  // scratch is rewritten by the next chunk's BD
    cm0 = fmaxf(cm0, __shfl_xor_sync(0xffffffffu, cm0, 1));
    cm0 = fmaxf(cm0, __shfl_xor_sync(0xffffffffu, cm0, 2));
    cm1 = fmaxf(cm1, __shfl_xor_sync(0xffffffffu, cm1, 1));
    cm1 = fmaxf(cm1, __shfl_xor_sync(0xffffffffu, cm1, 2));
    const float nm0 = fmaxf(m0, cm0), nm1 = fmaxf(m1, cm1);
    const float a0 = ex2(m0 - nm0), a1 = ex2(m1 - nm1);
    m0 = nm0;
    m1 = nm1;
    float sum0 = 0.0f, sum1 = 0.0f;
    uint32_t pf[AKC / 16][4];
#pragma unroll
    for (int nt = 0; nt < AKC / 8; ++nt) {
      float p[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int jl = nt * 8 + 2 * t + (e & 1);
        p[e] = j0 + jl < valid ? ex2(s[nt][e] - (e < 2 ? m0 : m1)) : 0.0f;
      }
      sum0 += p[0] + p[1];
      sum1 += p[2] + p[3];
      pf[nt >> 1][(nt & 1) * 2 + 0] = pack_half2(p[0], p[1]);
      pf[nt >> 1][(nt & 1) * 2 + 1] = pack_half2(p[2], p[3]);
    }
    sum0 += __shfl_xor_sync(0xffffffffu, sum0, 1);
    sum0 += __shfl_xor_sync(0xffffffffu, sum0, 2);
    sum1 += __shfl_xor_sync(0xffffffffu, sum1, 1);
    sum1 += __shfl_xor_sync(0xffffffffu, sum1, 2);
    l0 = l0 * a0 + sum0;
    l1 = l1 * a1 + sum1;
#pragma unroll
    for (int dt = 0; dt < 16; ++dt) {
      o[dt][0] *= a0;
      o[dt][1] *= a0;
      o[dt][2] *= a1;
      o[dt][3] *= a1;
    }
    // ---- PV
    const int lr = lane & 7, lm = lane >> 3;  // ldmatrix row / matrix index
#pragma unroll
    for (int kk = 0; kk < AKC / 16; ++kk) {
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {
        const int key = kk * 16 + (lm & 1) * 8 + lr;
        const int dim = dp * 16 + (lm >> 1) * 8;
        uint32_t b00, b01, b10, b11;
        ldmatrix_x4_trans(smem_addr(Vs + key * AS + dim), b00, b01, b10, b11);
        mma16816(o[2 * dp], pf[kk], b00, b01);
        mma16816(o[2 * dp + 1], pf[kk], b10, b11);
      }
    }
  }

  if (!active) {
    for (int i = lane; i < 16 * 16; i += 32) {
      const int q = i0 + i / 16, c = (i % 16) * 8;
      if (q < frames)
        *reinterpret_cast<uint4*>(context + (row0 + q) * 1024 + h * 128 + c) = make_uint4(0, 0, 0, 0);
    }
    return;
  }
  const float inv0 = 1.0f / l0, inv1 = 1.0f / l1;
  const int ra = i0 + g, rb = i0 + g + 8;
#pragma unroll
  for (int dt = 0; dt < 16; ++dt) {
    const int d = h * 128 + dt * 8 + 2 * t;
    if (ra < frames)
      *reinterpret_cast<uint32_t*>(context + (row0 + ra) * 1024 + d) =
          ra < valid ? pack_half2(o[dt][0] * inv0, o[dt][1] * inv0) : 0u;
    if (rb < frames)
      *reinterpret_cast<uint32_t*>(context + (row0 + rb) * 1024 + d) =
          rb < valid ? pack_half2(o[dt][2] * inv1, o[dt][3] * inv1) : 0u;
  }
}

}  // namespace

// positions [8*32][P][4] (package layout) -> [8][P][128].
__global__ void positions_rowmajor_kernel(const __half* __restrict__ pkg, __half* __restrict__ rm, int P) {
  pdl_entry();
  const int h = blockIdx.y, p = blockIdx.x, vec = threadIdx.x;
  *reinterpret_cast<uint2*>(rm + ((size_t)h * P + p) * 128 + vec * 4) =
      *reinterpret_cast<const uint2*>(pkg + ((size_t)(h * 32 + vec) * P + p) * 4);
}

int launch_positions_rowmajor(const void* pkg, void* rm, int frames, cudaStream_t stream) {
  const int P = 2 * frames - 1;
  return cuda_error(launch_kernel(positions_rowmajor_kernel, dim3(P, 8), dim3(32), 0, stream,
                                  static_cast<const __half*>(pkg), static_cast<__half*>(rm), P),
                    "positions_rowmajor launch");
}

int launch_rel_attention_tc(int batch, int frames, const void* qkv, const void* positions, const float* bias_u,
                            const float* bias_v, const uint32_t* valid_lengths, void* context, cudaStream_t stream,
                            bool positions_rowmajor) {
  const dim3 grid((frames + AQ - 1) / AQ, 8, batch);
  if (positions_rowmajor) {
    const int st = set_max_dynamic_smem(reinterpret_cast<const void*>(rel_attention_flash_kernel<true>), ASMEM);
    if (st != PK_OK) return st;
    launch_kernel(rel_attention_flash_kernel<true>, grid, ATHREADS, ASMEM, stream,
                  static_cast<const __half*>(qkv), static_cast<const __half*>(positions), bias_u, bias_v,
                  valid_lengths, static_cast<__half*>(context), frames);
    return cuda_error(cudaGetLastError(), "rel_attention_flash launch");
  }
  const int st = set_max_dynamic_smem(reinterpret_cast<const void*>(rel_attention_flash_kernel<false>), ASMEM);
  if (st != PK_OK) return st;
  launch_kernel(rel_attention_flash_kernel<false>, grid, ATHREADS, ASMEM, stream, 
      static_cast<const __half*>(qkv), static_cast<const __half*>(positions), bias_u, bias_v, valid_lengths,
      static_cast<__half*>(context), frames);
  return cuda_error(cudaGetLastError(), "rel_attention_flash launch");
}

}  // namespace pk
