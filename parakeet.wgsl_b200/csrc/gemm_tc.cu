// gemm_tc.cu -- fused palette-dequantizing GEMM on the sm_100a tensor cores.
//
// Computes C[M, N] = epilogue(A[M, K] . W[K, N]) for the FP16 package, where W
// arrives as the reference's bit-packed 5/6-bit palette codes
// (k-by-output-row-major-palette{5,6}-lsb-u32, src/model/runtime-plan.ts:352-368)
// plus a [G, 2^bits] f16 lookup table, and is decoded on chip: the dequantized
// weights never go to HBM (the reference expands them to a scratch buffer
// first, src/model/palette-expander.ts:478-587, then runs
// f16SubgroupGemmWgsl, src/webgpu/kernels/gemm.ts:1362-1716).
//
// Formulation (swapped): D^T = W^T . A^T, so the 128 MMA rows are output
// features and the MMA N dimension is BN tokens.
//   * MMA-A = decoded weights, [128 features x 64 k] per stage, MN-major with
//     128-byte swizzle, written to shared memory by 8 decoder warps from the
//     packed-code tile (TMA, no swizzle) through the LUT held in shared memory;
//   * MMA-B = activations, [BN tokens x 64 k] per stage, K-major, loaded by TMA
//     with 128-byte swizzle (rows past M are zero-filled by TMA);
//   * D = fp32 accumulators in TMEM, double buffered (2 x BN columns) so the
//     epilogue of one tile overlaps the main loop of the next.
// Persistent CTAs (one per SM) walk the tile list; warp roles:
//   warp 0 TMA producer, warp 1 MMA issuer (+TMEM owner), warps 2-9 decoders,
//   warps 10-13 epilogue.  The epilogue (bias / SiLU / ReLU / scaled residual,
//   f16 store) is a compile-time specialization, so no dead activation or
//   residual code is issued.
// Accumulation is fp32 (the reference accumulates in f16, gemm.ts:1445-1453),
// so results agree with the reference algorithm within the FP16 package
// tolerance and with the oracle's wide-accumulation mode to f16 rounding.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>

#include "pk_common.cuh"
#include "pk_internal.h"

namespace pk {

constexpr int TC_BM = 128;         // output features per tile (MMA M)
constexpr int TC_BK = 64;          // k per stage: one 128-byte swizzle row of f16
constexpr int TC_STAGES = 4;
constexpr int TC_DECODE_WARPS = 8;
constexpr int TC_FIRST_EPI_WARP = 2 + TC_DECODE_WARPS;  // 10: warps 10..13 cover TMEM lane quarters 2,3,0,1
constexpr int TC_THREADS = (TC_FIRST_EPI_WARP + 4) * 32;  // 448
// CTA-pair kernel: one more warp (14) issues the code-tile loads, so that
// activation and code boxes come from different threads (a thread's TMA
// boxes are serviced one after another, ~0.3 us each).
constexpr int TC2_CODE_WARP = TC_FIRST_EPI_WARP + 4;
// ... and a second epilogue warp per TMEM lane quadrant (warps 15-18) takes
// every other 32-column chunk, halving the accumulator drain that the next
// tile's first MMAs wait for.
constexpr int TC2_EPI_WARPS = 8;
constexpr int TC2_THREADS = (TC2_CODE_WARP + 1 + 4) * 32;  // 608
constexpr int TC_EPI_THREADS = 128;

// EPI_RESIDUAL adds res_scale * acc to a residual loaded in the epilogue;
// EPI_RESADD folds the residual into the accumulator instead (residual
// k-steps, see the kernels) and only scales: used whenever 1/res_scale is a
// power of two and no activation follows, so both kernels round alike.
enum { EPI_PLAIN = 0, EPI_BIAS = 1, EPI_RESIDUAL = 2, EPI_RESADD = 3 };

struct TcGemmParams {
  CUtensorMap tmap_a;       // activations [M, K] f16, box {64, BN}, 128B swizzle
  CUtensorMap tmap_codes;   // packed codes [K, N*bits/32] u32, box {128*bits/32, 64}
  const uint16_t* palette;  // f16 bits [G, 2^bits]
  const float* bias;
  const __half* residual;
  __half* out;
  unsigned int* status;
  int rows, inner, columns;
  int groups, group_cols;
  float res_scale;
  int m_tiles, n_tiles;
  CUtensorMap tmap_res;     // CTA-pair kernel: residual [M, N] f16, box {64, T/2}, 128B swizzle
  uint32_t res_inv_h;       // CTA-pair kernel: f16 bits of 1 / res_scale (a power of two)
  const uint32_t* mask_lengths;  // time mask (GemmArgs), or null
  int mask_group, mask_frames;
};

// Whether output row `row` passes the time mask (rows past the end read no
// length; they are not stored).
__device__ __forceinline__ bool mask_keeps(const TcGemmParams& p, int row) {
  if (row >= p.rows) return false;
  const int fr = row / p.mask_group;
  const int w = fr / p.mask_frames;
  return (uint32_t)(fr - w * p.mask_frames) < __ldg(p.mask_lengths + w);
}
// Bit e set: output row row0 + e is kept by the time mask.  Lane e evaluates
// row row0 + e; the warp must be converged.
__device__ __forceinline__ uint32_t mask_keep_bits(const TcGemmParams& p, int row0) {
  return __ballot_sync(0xffffffffu, mask_keeps(p, row0 + (int)(threadIdx.x & 31)));
}

template <int BN, int BITS>
struct TcLayout {
  static constexpr int CPG = BITS == 5 ? 32 : 16;         // codes per packed group
  static constexpr int WPG = BITS == 5 ? 5 : 3;           // u32 words per packed group
  static constexpr int WORDS_PER_ROW = TC_BM * BITS / 32; // 20 or 24 words per k row of a tile
  static constexpr int A_BYTES = BN * TC_BK * 2;
  static constexpr int W_BYTES = TC_BM * TC_BK * 2;
  static constexpr int CODE_BYTES = TC_BK * WORDS_PER_ROW * 4;
  static constexpr int OFF_A = 0;
  static constexpr int OFF_W = OFF_A + TC_STAGES * A_BYTES;
  static constexpr int OFF_C = OFF_W + TC_STAGES * W_BYTES;
  static constexpr int OFF_BAR = OFF_C + TC_STAGES * CODE_BYTES;
  static constexpr int NUM_BARS = 3 * TC_STAGES + 2 + 2 + 1;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;  // + alignment slack
  static constexpr uint32_t IDESC = umma_idesc_f16(TC_BM, BN, /*A MN-major*/ 1, /*B K-major*/ 0);
  // Two accumulators of BN fp32 columns; TMEM allocations are powers of two.
  static constexpr uint32_t TMEM_COLS = 2 * BN <= 256 ? 256 : 512;
  static_assert(A_BYTES % 1024 == 0 && W_BYTES % 1024 == 0, "stage buffers must keep 1024B alignment");
  static_assert(CODE_BYTES % 128 == 0, "code stage must keep 128B alignment");
};

// Byte offset of code I's LUT entry (code * 2) ORed with the palette group's
// byte offset `goff` (a multiple of 2^(BITS+1), so the OR is an add): one
// shift and one 3-input logic op per code.
template <int BITS, int I>
__device__ __forceinline__ uint32_t lut_offset(const uint32_t (&w)[BITS == 5 ? 5 : 3], uint32_t goff) {
  constexpr int bit = I * BITS, word = bit >> 5, sh = bit & 31;
  constexpr uint32_t mask2 = ((1u << BITS) - 1u) << 1;
  uint32_t x;
  if constexpr (sh + BITS > 32) {
    x = __funnelshift_r(w[word], w[word + 1], sh - 1);
  } else if constexpr (sh == 0) {
    x = w[word] << 1;
  } else {
    x = w[word] >> (sh - 1);
  }
  return (x & mask2) | goff;
}

template <int BITS, int I, int N>
struct DecodePairs {
  // Decode codes [I, N) of a group into packed f16 pairs.
  static __device__ __forceinline__ void run(const uint32_t (&w)[BITS == 5 ? 5 : 3], const uint8_t* lut,
                                             uint32_t goff, uint32_t* out) {
    if constexpr (I < N) {
      const uint32_t lo = *reinterpret_cast<const uint16_t*>(lut + lut_offset<BITS, I>(w, goff));
      const uint32_t hi = *reinterpret_cast<const uint16_t*>(lut + lut_offset<BITS, I + 1>(w, goff));
      out[I / 2] = __byte_perm(lo, hi, 0x5410);
      DecodePairs<BITS, I + 2, N>::run(w, lut, goff, out);
    }
  }
};

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}

// Store CPG weights (fixed k, consecutive features from feature-in-tile `f0`,
// f16 pairs) into the MN-major SW128 weight tile.
// Tile layout: atom(n_block, k_group) at n_block * 8192 + k_group * 1024;
// row (k % 8) at 128 B; 16-byte chunk c (features 8c..8c+7 of the 64-wide
// block) at physical chunk c ^ (k % 8).
template <int CPG>
__device__ __forceinline__ void store_group(const uint32_t (&packed)[CPG / 2], uint32_t w_stage, int k, int f0) {
  const int r = k & 7;
  const uint32_t row = w_stage + (uint32_t)((f0 >> 6) * 8192 + (k >> 3) * 1024 + r * 128);
  const int c0 = (f0 & 63) >> 3;
#pragma unroll
  for (int q = 0; q < CPG / 8; ++q) {
    const uint32_t chunk = (uint32_t)((c0 + q) ^ r);
    st_shared_v4(row + chunk * 16, packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
  }
}

// Decode one packed group (fixed k, CPG consecutive features starting at
// feature-in-tile `f0`) into the weight tile.
template <int BITS>
__device__ __forceinline__ void decode_group(const uint32_t* src, const uint8_t* lut, uint32_t goff,
                                             uint32_t w_stage, int k, int f0) {
  constexpr int WPG = BITS == 5 ? 5 : 3, CPG = BITS == 5 ? 32 : 16;
  uint32_t words[WPG];
#pragma unroll
  for (int j = 0; j < WPG; ++j) words[j] = src[j];
  uint32_t packed[CPG / 2];
  DecodePairs<BITS, 0, CPG>::run(words, lut, goff, packed);
  store_group<CPG>(packed, w_stage, k, f0);
}

// Identity block of the residual k-steps (CTA-pair kernel): weight (k, f) of
// this group is `inv` where f == fsel, else zero.
template <int CPG>
__device__ __forceinline__ void identity_group(uint32_t inv, int fsel, uint32_t w_stage, int k, int f0) {
  uint32_t packed[CPG / 2];
#pragma unroll
  for (int i = 0; i < CPG / 2; ++i)
    packed[i] = (f0 + 2 * i == fsel ? inv : 0u) | (f0 + 2 * i + 1 == fsel ? inv << 16 : 0u);
  store_group<CPG>(packed, w_stage, k, f0);
}

template <int ACT>
__device__ __forceinline__ float activate(float v) {
  if constexpr (ACT == PK_ACT_SILU) {
    // SiLU v * sigmoid(v) (gemm.ts:2018-2032 writes v / (1 + exp(-v)) with v
    // clamped inside exp) through sigmoid(v) = (1 + tanh(v/2)) / 2:
    // h + h * tanh(h), h = v/2, one special-function op per element (the
    // hardware tanh approximation, absolute error below 2^-10) where
    // exp + divide take two.  The special-function unit bounds this epilogue.
    const float h = 0.5f * v;
    float t;
    asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(h));
    return fmaf(h, t, h);
  } else if constexpr (ACT == PK_ACT_RELU) {
    return fmaxf(v, 0.0f);
  } else {
    return v;
  }
}

// Epilogue of `count` consecutive tokens of one output feature (one TMEM lane).
// Residual values are all loaded before the first store so their latencies
// overlap (the output never aliases the residual: the encoder ping-pongs
// between two slots).
template <int EPI, int ACT, int COUNT>
__device__ __forceinline__ void epilogue_run(const uint32_t (&r)[32], float bias_v, const __half* __restrict__ res,
                                             __half* __restrict__ out, int ld, float res_scale, int count,
                                             uint32_t keep) {
  __half rv[EPI == EPI_RESIDUAL ? 32 : 1];
  if constexpr (EPI == EPI_RESIDUAL) {
#pragma unroll
    for (int j = 0; j < COUNT; ++j)
      if (COUNT == 32 || j < count) rv[j] = __ldg(res + (size_t)j * ld);
  }
#pragma unroll
  for (int j = 0; j < COUNT; ++j) {
    if (COUNT == 32 || j < count) {
      float v = __uint_as_float(r[j]);
      if constexpr (EPI == EPI_BIAS) v += bias_v;
      v = activate<ACT>(v);
      if constexpr (EPI == EPI_RESIDUAL) v = __half2float(rv[j]) + res_scale * v;
      if constexpr (EPI == EPI_RESADD) v *= res_scale;
      out[(size_t)j * ld] = (keep >> j) & 1u ? __float2half_rn(v) : __float2half_rn(0.0f);
    }
  }
}

// CTA-pair epilogue value of one accumulator element.  The CTA-pair kernel
// only takes the folded residual (EPI_RESADD), which scales.
template <int EPI, int ACT>
__device__ __forceinline__ __half pair_epilogue_value(uint32_t r, float bias_v, float res_scale) {
  static_assert(EPI != EPI_RESIDUAL, "the CTA-pair kernel folds the residual");
  static_assert(EPI != EPI_RESADD || ACT == PK_ACT_NONE, "the folded residual admits no activation");
  float v = __uint_as_float(r);
  if constexpr (EPI == EPI_BIAS) v += bias_v;
  if constexpr (EPI == EPI_RESADD) v *= res_scale;
  return __float2half_rn(activate<ACT>(v));
}

// 32 accumulator columns of one output feature: columns e < split are tokens
// tok_a + e, the rest tokens tok_b + e - split (a chunk crosses at most one
// boundary between contiguous token runs); tokens >= rows are not stored.
// The common case -- one run, all in range -- stores without predicates.
template <int EPI, int ACT>
__device__ __forceinline__ void pair_epilogue_chunk(const uint32_t (&r)[32], float bias_v, float res_scale,
                                                    __half* __restrict__ col_out, int ld, int rows, int tok_a,
                                                    int split, int tok_b) {
  if (split == 32 && tok_a + 32 <= rows) {
    __half* out = col_out + (size_t)tok_a * ld;
#pragma unroll
    for (int e = 0; e < 32; ++e) out[(size_t)e * ld] = pair_epilogue_value<EPI, ACT>(r[e], bias_v, res_scale);
    return;
  }
#pragma unroll
  for (int e = 0; e < 32; ++e) {
    const int tok = e < split ? tok_a + e : tok_b + (e - split);
    if (tok < rows) col_out[(size_t)tok * ld] = pair_epilogue_value<EPI, ACT>(r[e], bias_v, res_scale);
  }
}

template <int BN, int BITS, int EPI, int ACT, bool MASK = false>
__global__ void __launch_bounds__(TC_THREADS, 1) tc_palette_gemm_kernel(const __grid_constant__ TcGemmParams p) {
  using L = TcLayout<BN, BITS>;
  __shared__ __align__(16) uint16_t s_lut[3 * 64];
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem + L::OFF_A;
  uint8_t* sW = smem + L::OFF_W;
  uint32_t* sCodes = reinterpret_cast<uint32_t*>(smem + L::OFF_C);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* full_tma = bars;
  uint64_t* full_dec = bars + TC_STAGES;
  uint64_t* empty = bars + 2 * TC_STAGES;
  uint64_t* tm_full = bars + 3 * TC_STAGES;
  uint64_t* tm_empty = tm_full + 2;
  uint64_t* drain = tm_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int lut_entries = p.groups << BITS;
  for (int i = threadIdx.x; i < lut_entries; i += blockDim.x) s_lut[i] = p.palette[i];
  if (threadIdx.x == 0) {
    for (int s = 0; s < TC_STAGES; ++s) {
      mbar_init(&full_tma[s], 1);
      mbar_init(&full_dec[s], TC_DECODE_WARPS);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tm_full[a], 1);
      mbar_init(&tm_empty[a], TC_EPI_THREADS / 32);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&p.tmap_a);
    tma_prefetch_desc(&p.tmap_codes);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, L::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_entry();  // activations / residual / output are touched only after this

  // EPI_RESADD: KR extra k-steps first with B = the residual tile (the
  // tile's 128 output features as K) and A = 1/res_scale times the identity,
  // so the accumulator starts at residual / res_scale.
  constexpr int KR = EPI == EPI_RESADD ? TC_BM / TC_BK : 0;
  const int kb_count = p.inner / TC_BK + KR;
  const int num_tiles = p.m_tiles * p.n_tiles;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int last_round[TC_STAGES];
#pragma unroll
      for (int s = 0; s < TC_STAGES; ++s) last_round[s] = -1;
      uint32_t it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int n_tile = tile % p.n_tiles, m_tile = tile / p.n_tiles;
        for (int kb = 0; kb < kb_count; ++kb, ++it) {
          const int s = it % TC_STAGES;
          const uint32_t round = it / TC_STAGES;
          if (round > 0 && !mbar_wait(&empty[s], (round - 1) & 1, abort_flag, p.status, PK_STATUS_TIMEOUT_TMA)) {
            ok = false;
            break;
          }
          if (kb < KR) {
            mbar_arrive_expect_tx(&full_tma[s], L::A_BYTES);
            tma_load_2d(sA + s * L::A_BYTES, &p.tmap_res, &full_tma[s], n_tile * TC_BM + kb * TC_BK, m_tile * BN);
            last_round[s] = (int)round;
            continue;
          }
          mbar_arrive_expect_tx(&full_tma[s], L::A_BYTES + L::CODE_BYTES);
          tma_load_2d(sA + s * L::A_BYTES, &p.tmap_a, &full_tma[s], (kb - KR) * TC_BK, m_tile * BN);
          tma_load_2d(sCodes + s * (L::CODE_BYTES / 4), &p.tmap_codes, &full_tma[s], n_tile * L::WORDS_PER_ROW,
                      (kb - KR) * TC_BK);
          last_round[s] = (int)round;
        }
      }
      // Unwind: every load this thread issued must have landed before exit.
      for (int s = 0; s < TC_STAGES; ++s)
        if (last_round[s] >= 0) mbar_wait_drain(&full_tma[s], (uint32_t)last_round[s] & 1, p.status);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      uint32_t it = 0;
      int tile_iter = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++tile_iter) {
        const int acc = tile_iter & 1;
        const uint32_t acc_round = (uint32_t)tile_iter >> 1;
        if (acc_round > 0 &&
            !mbar_wait(&tm_empty[acc], (acc_round - 1) & 1, abort_flag, p.status, PK_STATUS_TIMEOUT_MMA)) {
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < kb_count; ++kb, ++it) {
          const int s = it % TC_STAGES;
          const uint32_t round = it / TC_STAGES;
          if (!mbar_wait(&full_tma[s], round & 1, abort_flag, p.status, PK_STATUS_TIMEOUT_MMA) ||
              !mbar_wait(&full_dec[s], round & 1, abort_flag, p.status, PK_STATUS_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t w_addr = smem_addr(sW + s * L::W_BYTES);
          const uint32_t a_addr = smem_addr(sA + s * L::A_BYTES);
#pragma unroll
          for (int kk = 0; kk < TC_BK / 16; ++kk) {
            // A (weights, MN-major): two 8-row k groups per K=16 step, SBO = 1024 B
            // between k groups, LBO = 8192 B between 64-feature blocks.
            const uint64_t a_desc = umma_smem_desc(w_addr + kk * 2048, 8192, 1024, 2);
            // B (activations, K-major): advance 32 B (16 f16) inside the swizzle row.
            const uint64_t b_desc = umma_smem_desc(a_addr + kk * 32, 16, 1024, 2);
            tc_mma_f16(d_tmem, a_desc, b_desc, L::IDESC, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          tc_commit(&empty[s]);
        }
        if (!ok) break;
        tc_commit(&tm_full[acc]);
      }
      // Unwind: wait until every MMA issued by this thread has completed.
      tc_commit(drain);
      mbar_wait_drain(drain, 0, p.status);
    }
  } else if (warp < TC_FIRST_EPI_WARP) {
    // ------------------------------------------------------------ decoders
    // Warp dw owns k rows dw*8 .. dw*8+7 of each stage; lane = (k % 8) + 8 * g,
    // g picking the packed group(s) along the 128 features (conflict-free
    // word reads and 16-byte swizzled stores).
    const int dw = warp - 2;
    const int k = dw * 8 + (lane & 7);
    constexpr int GROUPS_PER_LANE = BITS == 5 ? 1 : 2;
    const uint8_t* lut = reinterpret_cast<const uint8_t*>(s_lut);
    uint32_t it = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      const int f_base = (tile % p.n_tiles) * TC_BM;
      uint32_t goff[GROUPS_PER_LANE];
      int f0[GROUPS_PER_LANE];
#pragma unroll
      for (int j = 0; j < GROUPS_PER_LANE; ++j) {
        f0[j] = ((lane >> 3) + 4 * j) * L::CPG;
        const int pg = min((f_base + f0[j]) / p.group_cols, p.groups - 1);
        goff[j] = (uint32_t)pg << (BITS + 1);
      }
      bool ok = true;
      for (int kb = 0; kb < kb_count; ++kb, ++it) {
        const int s = it % TC_STAGES;
        const uint32_t round = it / TC_STAGES;
        // Warp-uniform outcome: the arrive below is one lane's, after __syncwarp.
        if (!__all_sync(0xffffffffu, mbar_wait(&full_tma[s], round & 1, abort_flag, p.status,
                                               PK_STATUS_TIMEOUT_DECODE))) {
          ok = false;
          break;
        }
        const uint32_t w_stage = smem_addr(sW + s * L::W_BYTES);
        if (kb < KR) {
          // Residual feature kb*64 + k of the tile carries weight 1/res_scale.
#pragma unroll
          for (int j = 0; j < GROUPS_PER_LANE; ++j)
            identity_group<L::CPG>(p.res_inv_h, kb * TC_BK + k, w_stage, k, f0[j]);
        } else {
          const uint32_t* codes = sCodes + s * (L::CODE_BYTES / 4) + k * L::WORDS_PER_ROW;
#pragma unroll
          for (int j = 0; j < GROUPS_PER_LANE; ++j)
            decode_group<BITS>(codes + (f0[j] / L::CPG) * L::WPG, lut, goff[j], w_stage, k, f0[j]);
        }
        // Each lane makes its generic-proxy stores visible to the tensor core
        // (async proxy); the warp's lanes are ordered by __syncwarp, and one
        // lane's release-arrive covers the warp.
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&full_dec[s]);
      }
      if (!ok) break;
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    int tile_iter = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++tile_iter) {
      const int acc = tile_iter & 1;
      const uint32_t acc_round = (uint32_t)tile_iter >> 1;
      if (!__all_sync(0xffffffffu,
                      mbar_wait(&tm_full[acc], acc_round & 1, abort_flag, p.status, PK_STATUS_TIMEOUT_EPILOGUE)))
        break;
      tc_fence_after();
      const int n_tile = tile % p.n_tiles, m_tile = tile / p.n_tiles;
      const int n = n_tile * TC_BM + q * 32 + lane;
      const int m0 = m_tile * BN;
      const float bias_v = EPI == EPI_BIAS ? __ldg(p.bias + n) : 0.0f;
      const uint32_t t_base = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
      const int ld = p.columns;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        const int left = p.rows - (m0 + c);
        if (left <= 0) break;
        uint32_t r[32];
        tc_ld_32x32b_x32(t_base + (uint32_t)c, r);
        tc_wait_ld();
        const size_t base = (size_t)(m0 + c) * ld + n;
        const __half* res = EPI == EPI_RESIDUAL ? p.residual + base : nullptr;
        const uint32_t keep = MASK ? mask_keep_bits(p, m0 + c) : 0xffffffffu;
        if (left >= 32)
          epilogue_run<EPI, ACT, 32>(r, bias_v, res, p.out + base, ld, p.res_scale, 32, keep);
        else
          epilogue_run<EPI, ACT, 31>(r, bias_v, res, p.out + base, ld, p.res_scale, left, keep);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tm_empty[acc]);
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, L::TMEM_COLS);
  }
}

// ===========================================================================
// CTA-pair variant (cluster of 2, tcgen05 cta_group::2, MMA M = 256).
// A pair owns 256 output features x T tokens, T = NSUB x BN_MMA.  Each CTA
// decodes its own 128 features (MMA-A rows 128*rank ..) and TMA-loads a
// contiguous half of the token tile, T/2 rows; per stage the leader issues
// NSUB MMAs of N = BN_MMA against the same decoded weights, MMA j taking rows
// [j*BN_MMA/2, (j+1)*BN_MMA/2) of each CTA's half.  Decoding a weight stage
// once for up to 512 tokens halves the decode work per FLOP of the
// single-CTA kernel (whose MMA N, and so its token tile, stops at 256).
// D rows of each CTA land in its own TMEM, so both CTAs run their own
// epilogue; accumulators are double buffered when 2T columns fit in TMEM,
// single buffered otherwise.
// Barriers: the leader's full_b[s] collects both halves' TMA bytes,
// full_dec[s] both CTAs' decoders, tm_empty[a] both epilogues; each CTA's
// own full_c[s] (its code tile), empty[s] and tm_full[a] are signalled by the
// leader's MMA commits (one commit addressed to each CTA).  The peer signals
// the leader with 16-byte shared-to-shared bulk copies that complete as
// transaction bytes on the leader's barrier (bulk_signal_cluster): a
// release.cluster arrive would make every signalling warp wait on a memory
// barrier, which measured 1.6x slower than the single-CTA kernel.
// ===========================================================================
template <int BN_MMA, int NSUB, int BITS>
struct Tc2Layout {
  static constexpr int T = BN_MMA * NSUB;                  // tokens per pair tile
  static constexpr int CPG = BITS == 5 ? 32 : 16;
  static constexpr int WPG = BITS == 5 ? 5 : 3;
  static constexpr int WORDS_PER_ROW = TC_BM * BITS / 32;
  static constexpr int HALF_ROWS = T / 2;                  // tokens this CTA loads
  static constexpr int SUB_ROWS = BN_MMA / 2;              // rows of one MMA's B half
  static constexpr int A_BYTES = HALF_ROWS * TC_BK * 2;
  static constexpr int W_BYTES = TC_BM * TC_BK * 2;
  static constexpr int CODE_BYTES = TC_BK * WORDS_PER_ROW * 4;
  static constexpr int STAGE_BYTES = A_BYTES + W_BYTES + CODE_BYTES;
  static constexpr int STAGES = (227 * 1024 - 2048) / STAGE_BYTES > 6 ? 6 : (227 * 1024 - 2048) / STAGE_BYTES;
  static constexpr int OFF_A = 0;
  static constexpr int OFF_W = OFF_A + STAGES * A_BYTES;
  static constexpr int OFF_C = OFF_W + STAGES * W_BYTES;
  static constexpr int OFF_BAR = OFF_C + STAGES * CODE_BYTES;
  static constexpr int NUM_BARS = 5 * STAGES + 2 + 2 + 1;
  // misc: TMEM slot, abort flag, then the 16-byte signal payload, which a
  // bulk copy reads and writes and so must be 16-byte aligned.
  static constexpr int OFF_MISC = (OFF_BAR + NUM_BARS * 8 + 15) / 16 * 16;
  static constexpr int SMEM_BYTES = OFF_MISC + 32 + 1024;
  static constexpr int ACC_BUFS = 2 * T <= 512 ? 2 : 1;
  // A single accumulator of two MMA sub-tiles is released per sub-tile
  // (tm_empty[j]: sub-tile j drained), so the next tile's first stages can
  // start on sub-tile 0 while the epilogue still drains sub-tile 1.
  static constexpr bool SPLIT_RELEASE = ACC_BUFS == 1 && NSUB == 2;
  static_assert(!SPLIT_RELEASE || BN_MMA % 32 == 0, "sub-tiles end on epilogue chunk boundaries");
  static constexpr uint32_t IDESC = umma_idesc_f16(2 * TC_BM, BN_MMA, /*A MN-major*/ 1, /*B K-major*/ 0);
  static constexpr uint32_t TMEM_COLS = ACC_BUFS * T <= 256 ? 256 : 512;
  static_assert(STAGES >= 3, "pipeline too shallow");
  static_assert(OFF_MISC % 16 == 0 && OFF_C % 128 == 0 && CODE_BYTES % 128 == 0, "TMA / bulk-copy alignment");
  static_assert(SUB_ROWS % 8 == 0 && SUB_ROWS >= 32, "MMA halves in whole 8-row swizzle atoms");
  static_assert(T % 32 == 0, "epilogue chunks of 32 accumulator columns");
  static_assert(A_BYTES % 1024 == 0 && W_BYTES % 1024 == 0, "stage buffers must keep 1024B alignment");
  static_assert(ACC_BUFS * T <= 512, "TMEM holds 512 columns");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
};

template <int BN_MMA, int NSUB, int BITS, int EPI, int ACT>
__global__ void __launch_bounds__(TC2_THREADS, 1) tc2_palette_gemm_kernel(const __grid_constant__ TcGemmParams p) {
  using L = Tc2Layout<BN_MMA, NSUB, BITS>;
  constexpr int S = L::STAGES;
  constexpr int T = L::T;
  __shared__ __align__(16) uint16_t s_lut[3 * 64];
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem + L::OFF_A;
  uint8_t* sW = smem + L::OFF_W;
  uint32_t* sCodes = reinterpret_cast<uint32_t*>(smem + L::OFF_C);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* full_b = bars;              // leader: both B halves landed
  uint64_t* full_c = bars + S;          // own code tile landed
  uint64_t* full_dec = bars + 2 * S;    // leader: both CTAs decoded
  uint64_t* empty = bars + 3 * S;       // own: stage consumed by the pair MMA
  uint64_t* dec_local = bars + 4 * S;   // peer: own decoders done (relayed to full_dec)
  uint64_t* tm_full = bars + 5 * S;     // own: accumulator ready
  uint64_t* tm_empty = tm_full + 2;     // leader: both epilogues drained
  uint64_t* drain = tm_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);
  const uint32_t signal_payload = smem_addr(smem + L::OFF_MISC + 16);  // 16 bytes, contents unused
  constexpr uint32_t SIGNAL_BYTES = 16;

  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int lut_entries = p.groups << BITS;
  for (int i = threadIdx.x; i < lut_entries; i += blockDim.x) s_lut[i] = p.palette[i];
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_b[s], 1);
      mbar_init(&full_c[s], 1);
      mbar_init(&full_dec[s], TC_DECODE_WARPS);  // + SIGNAL_BYTES from the peer's relay
      mbar_init(&empty[s], 1);
      mbar_init(&dec_local[s], TC_DECODE_WARPS);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tm_full[a], 1);
      mbar_init(&tm_empty[a], TC2_EPI_WARPS);  // + SIGNAL_BYTES per peer epilogue warp
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&p.tmap_a);
    tma_prefetch_desc(&p.tmap_codes);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, L::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // barriers of both CTAs initialised before any remote signal
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Programmatic dependent launch: only the activation producer waits for
  // the previous kernel (pdl_wait below), before its first activation /
  // residual load; every other global access of this kernel (output stores)
  // follows those loads through the pipeline barriers.  Weights are not
  // written by kernels, so the code-tile producer does not wait.
  pdl_launch_dependents();

  // Residual GEMMs run KR extra k-steps first: B = the residual tile (the
  // pair's 256 output features as K), A = 1/res_scale times the identity
  // block of this CTA's features, so the accumulator starts at
  // residual / res_scale and the epilogue's res_scale * acc is
  // residual + res_scale * (A . W), exactly for a power-of-two scale.
  constexpr int KR = EPI == EPI_RESADD ? 2 * TC_BM / TC_BK : 0;
  const int kb_count = p.inner / TC_BK + KR;
  const int pair_n_tiles = p.n_tiles / 2;  // 256-feature tiles
  const int num_tiles = p.m_tiles * pair_n_tiles;
  const int pair = blockIdx.x >> 1, num_pairs = gridDim.x >> 1;

  if (warp == 0) {
    // ------------------------------------------------- activation producer (both CTAs)
    if (lane == 0) {
      int last_round[S];
#pragma unroll
      for (int s = 0; s < S; ++s) last_round[s] = -1;
      pdl_wait();
      uint32_t it = 0;
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += num_pairs) {
        const int np = tile % pair_n_tiles, m_tile = tile / pair_n_tiles;
        for (int kb = 0; kb < kb_count; ++kb, ++it) {
          const int s = it % S;
          const uint32_t round = it / S;
          if (round > 0 && !mbar_wait(&empty[s], (round - 1) & 1, abort_flag, p.status, PK_STATUS_TIMEOUT_TMA)) {
            ok = false;
            break;
          }
          if (leader) mbar_arrive_expect_tx(&full_b[s], 2 * L::A_BYTES);
          const uint32_t full_b_leader = mapa_shared(smem_addr(&full_b[s]), 0);
          const int y = m_tile * T + (int)rank * L::HALF_ROWS;
          if (kb < KR)
            tma_load_2d_pair(sA + s * L::A_BYTES, &p.tmap_res, full_b_leader, np * 2 * TC_BM + kb * TC_BK, y);
          else
            tma_load_2d_pair(sA + s * L::A_BYTES, &p.tmap_a, full_b_leader, (kb - KR) * TC_BK, y);
          last_round[s] = (int)round;
        }
      }
      // Unwind: the B halves are tracked by the leader's barriers, which its
      // MMA thread drains; the leader's producer also waits for its own.
      if (leader)
        for (int s = 0; s < S; ++s)
          if (last_round[s] >= 0) mbar_wait_drain(&full_b[s], (uint32_t)last_round[s] & 1, p.status);
    }
  } else if (warp == TC2_CODE_WARP) {
    // -------------------------------------------------- code-tile producer (both CTAs)
    // Weights are not written by kernels, so this warp does not wait for the
    // previous kernel: the first round's code tiles load (and decode) during
    // its tail.
    if (lane == 0) {
      int last_round[S];
#pragma unroll
      for (int s = 0; s < S; ++s) last_round[s] = -1;
      uint32_t it = 0;
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += num_pairs) {
        const int np = tile % pair_n_tiles;
        const int n_tile = np * 2 + (int)rank;  // this CTA's 128-feature tile
        for (int kb = 0; kb < kb_count; ++kb, ++it) {
          const int s = it % S;
          const uint32_t round = it / S;
          if (round > 0 && !mbar_wait(&empty[s], (round - 1) & 1, abort_flag, p.status, PK_STATUS_TIMEOUT_TMA)) {
            ok = false;
            break;
          }
          if (kb < KR) {
            mbar_arrive(&full_c[s]);  // no code tile: the decoders write an identity block
          } else {
            mbar_arrive_expect_tx(&full_c[s], L::CODE_BYTES);
            tma_load_2d(sCodes + s * (L::CODE_BYTES / 4), &p.tmap_codes, &full_c[s], n_tile * L::WORDS_PER_ROW,
                        (kb - KR) * TC_BK);
          }
          last_round[s] = (int)round;
        }
      }
      // Unwind: this CTA's code tiles must have landed.
      for (int s = 0; s < S; ++s)
        if (last_round[s] >= 0) mbar_wait_drain(&full_c[s], (uint32_t)last_round[s] & 1, p.status);
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---------------------------------------------------------- MMA issuer (leader)
      const uint32_t peer_base = mapa_shared(smem_addr(bars), 1);
      auto peer = [&](uint64_t* b) { return peer_base + (uint32_t)((b - bars) * 8); };
      uint32_t it = 0;
      int tile_iter = 0;
      bool ok = true;
      // MMAs of sub-tile j of stage s (four K=16 steps).
      auto issue_sub = [&](int s, int kb, int j, uint32_t d_tmem) {
        const uint32_t w_addr = smem_addr(sW + s * L::W_BYTES);
        const uint32_t a_addr = smem_addr(sA + s * L::A_BYTES);
#pragma unroll
        for (int kk = 0; kk < TC_BK / 16; ++kk) {
          const uint64_t a_desc = umma_smem_desc(w_addr + kk * 2048, 8192, 1024, 2);
          const uint64_t b_desc = umma_smem_desc(a_addr + j * L::SUB_ROWS * 128 + kk * 32, 16, 1024, 2);
          tc_mma_f16_pair(d_tmem + (uint32_t)(j * BN_MMA), a_desc, b_desc, L::IDESC, (kb > 0 || kk > 0) ? 1u : 0u);
        }
      };
      for (int tile = pair; tile < num_tiles && ok; tile += num_pairs, ++tile_iter) {
        const int acc = tile_iter % L::ACC_BUFS;
        const uint32_t acc_round = (uint32_t)(tile_iter / L::ACC_BUFS);
        // Split release: sub-tile 0's columns must be drained before this
        // tile's first MMA; sub-tile 1's MMAs of the first stages wait (their
        // stages held) until its columns are drained as well.
        bool sub1_free = true;
        int held = 0, held_kb0 = 0;  // stages it - held .. it - 1 hold sub-tile-1 MMAs, from k-step held_kb0
        const uint32_t ph = (uint32_t)(tile_iter - 1) & 1;
        if (L::SPLIT_RELEASE && tile_iter > 0) {
          if (!mbar_wait(&tm_empty[0], ph, abort_flag, p.status, PK_STATUS_TIMEOUT_MMA)) break;
          sub1_free = mbar_try_wait(&tm_empty[1], ph);
        } else if (acc_round > 0 &&
                   !mbar_wait(&tm_empty[acc], (acc_round - 1) & 1, abort_flag, p.status, PK_STATUS_TIMEOUT_MMA)) {
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * T);
        auto flush_held = [&]() {  // sub-tile 1 of the held stages, in k order, then release them
          for (int h = 0; h < held; ++h) {
            const uint32_t hit = it - (uint32_t)held + (uint32_t)h;
            issue_sub((int)(hit % S), held_kb0 + h, 1, d_tmem);
            tc_commit_pair(smem_addr(&empty[hit % S]));
            tc_commit_pair(peer(&empty[hit % S]));
          }
          held = 0;
        };
        for (int kb = 0; kb < kb_count; ++kb, ++it) {
          const int s = it % S;
          const uint32_t round = it / S;
          if (!mbar_wait(&full_b[s], round & 1, abort_flag, p.status, PK_STATUS_TIMEOUT_MMA) ||
              !mbar_wait(&full_dec[s], round & 1, abort_flag, p.status, PK_STATUS_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          if (!sub1_free) {
            sub1_free = mbar_try_wait(&tm_empty[1], ph);
            if (!sub1_free && held == S - 1) {  // the last free stage: wait for sub-tile 1's columns
              if (!mbar_wait(&tm_empty[1], ph, abort_flag, p.status, PK_STATUS_TIMEOUT_MMA)) {
                ok = false;
                break;
              }
              sub1_free = true;
            }
            tc_fence_after();
            if (sub1_free) {
              flush_held();
            } else {
              if (held == 0) held_kb0 = kb;
              issue_sub(s, kb, 0, d_tmem);
              ++held;
              continue;
            }
          }
          tc_fence_after();
          const uint32_t w_addr = smem_addr(sW + s * L::W_BYTES);
          const uint32_t a_addr = smem_addr(sA + s * L::A_BYTES);
#pragma unroll
          for (int kk = 0; kk < TC_BK / 16; ++kk) {
            const uint64_t a_desc = umma_smem_desc(w_addr + kk * 2048, 8192, 1024, 2);
#pragma unroll
            for (int j = 0; j < NSUB; ++j) {
              const uint64_t b_desc = umma_smem_desc(a_addr + j * L::SUB_ROWS * 128 + kk * 32, 16, 1024, 2);
              tc_mma_f16_pair(d_tmem + (uint32_t)(j * BN_MMA), a_desc, b_desc, L::IDESC,
                              (kb > 0 || kk > 0) ? 1u : 0u);
            }
          }
          tc_commit_pair(smem_addr(&empty[s]));
          tc_commit_pair(peer(&empty[s]));
        }
        if (ok && held > 0) {  // a tile shorter than the held stages
          if (!mbar_wait(&tm_empty[1], ph, abort_flag, p.status, PK_STATUS_TIMEOUT_MMA)) {
            ok = false;
          } else {
            tc_fence_after();
            flush_held();
          }
        }
        if (!ok) break;
        tc_commit_pair(smem_addr(&tm_full[acc]));
        tc_commit_pair(peer(&tm_full[acc]));
      }
      // The last epilogue signals: the peer's bulk-copy signals must land
      // before this CTA's shared memory is released.
      if constexpr (L::SPLIT_RELEASE) {
        if (tile_iter > 0)
          for (int j = 0; j < 2; ++j) mbar_wait_drain(&tm_empty[j], (uint32_t)(tile_iter - 1) & 1, p.status);
      } else {
        for (int a = 0; a < L::ACC_BUFS && tile_iter > a; ++a)
          mbar_wait_drain(&tm_empty[a], (uint32_t)((tile_iter - 1 - a) / L::ACC_BUFS) & 1, p.status);
      }
      tc_commit_pair(smem_addr(drain));
      mbar_wait_drain(drain, 0, p.status);
    } else if (lane == 0) {
      // ---------------------------------------------------------- peer relay
      // Once this CTA's decoder warps have arrived on dec_local[s], signal the
      // leader's full_dec[s].
      const uint32_t full_dec_leader = mapa_shared(smem_addr(full_dec), 0);
      const uint32_t payload_leader = mapa_shared(signal_payload, 0);
      uint32_t it = 0;
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += num_pairs) {
        for (int kb = 0; kb < kb_count; ++kb, ++it) {
          const int s = it % S;
          const uint32_t round = it / S;
          if (!mbar_wait(&dec_local[s], round & 1, abort_flag, p.status, PK_STATUS_TIMEOUT_DECODE)) {
            ok = false;
            break;
          }
          bulk_signal_cluster(payload_leader, signal_payload, SIGNAL_BYTES, full_dec_leader + (uint32_t)(s * 8));
        }
      }
    }
  } else if (warp < TC_FIRST_EPI_WARP) {
    // ------------------------------------------------------------ decoders (both CTAs)
    const int dw = warp - 2;
    const int k = dw * 8 + (lane & 7);
    constexpr int GROUPS_PER_LANE = BITS == 5 ? 1 : 2;
    const uint8_t* lut = reinterpret_cast<const uint8_t*>(s_lut);
    uint32_t it = 0;
    for (int tile = pair; tile < num_tiles; tile += num_pairs) {
      const int f_base = ((tile % pair_n_tiles) * 2 + (int)rank) * TC_BM;
      uint32_t goff[GROUPS_PER_LANE];
      int f0[GROUPS_PER_LANE];
#pragma unroll
      for (int j = 0; j < GROUPS_PER_LANE; ++j) {
        f0[j] = ((lane >> 3) + 4 * j) * L::CPG;
        const int pg = min((f_base + f0[j]) / p.group_cols, p.groups - 1);
        goff[j] = (uint32_t)pg << (BITS + 1);
      }
      bool ok = true;
      for (int kb = 0; kb < kb_count; ++kb, ++it) {
        const int s = it % S;
        const uint32_t round = it / S;
        if (!__all_sync(0xffffffffu, mbar_wait(&full_c[s], round & 1, abort_flag, p.status,
                                               PK_STATUS_TIMEOUT_DECODE))) {
          ok = false;
          break;
        }
        const uint32_t w_stage = smem_addr(sW + s * L::W_BYTES);
        if (kb < KR) {
          // Residual feature kb*64 + k of the pair is this CTA's feature
          // kb*64 + k - 128*rank.
          const int fsel = kb * TC_BK + k - (int)rank * TC_BM;
#pragma unroll
          for (int j = 0; j < GROUPS_PER_LANE; ++j) identity_group<L::CPG>(p.res_inv_h, fsel, w_stage, k, f0[j]);
        } else {
          const uint32_t* codes = sCodes + s * (L::CODE_BYTES / 4) + k * L::WORDS_PER_ROW;
#pragma unroll
          for (int j = 0; j < GROUPS_PER_LANE; ++j)
            decode_group<BITS>(codes + (f0[j] / L::CPG) * L::WPG, lut, goff[j], w_stage, k, f0[j]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (!leader)
            mbar_arrive(&dec_local[s]);
          else if (dw == 0)
            mbar_arrive_expect_tx(&full_dec[s], SIGNAL_BYTES);
          else
            mbar_arrive(&full_dec[s]);
        }
      }
      if (!ok) break;
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int q = warp & 3;
    const int eset = warp < TC2_CODE_WARP ? 0 : 1;  // chunks eset, eset + 2, ...
    const uint32_t tm_empty_leader = mapa_shared(smem_addr(tm_empty), 0);
    const uint32_t payload_leader = mapa_shared(signal_payload, 0);
    constexpr int NCH = T / 32;
    int tile_iter = 0;
    for (int tile = pair; tile < num_tiles; tile += num_pairs, ++tile_iter) {
      const int acc = tile_iter % L::ACC_BUFS;
      const uint32_t acc_round = (uint32_t)(tile_iter / L::ACC_BUFS);
      const int np = tile % pair_n_tiles, m_tile = tile / pair_n_tiles;
      const int n0 = (np * 2 + (int)rank) * TC_BM + q * 32;
      const int m0 = m_tile * T;
      const int ld = p.columns;
      if (!__all_sync(0xffffffffu,
                      mbar_wait(&tm_full[acc], acc_round & 1, abort_flag, p.status, PK_STATUS_TIMEOUT_EPILOGUE)))
        break;
      tc_fence_after();
      const int n = n0 + lane;
      const float bias_v = EPI == EPI_BIAS ? __ldg(p.bias + n) : 0.0f;
      const uint32_t t_base = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * T);
      // Column c of MMA j's accumulator is B row c of that MMA: row
      // j*SUB_ROWS + c of CTA 0's half (c < SUB_ROWS), else row
      // j*SUB_ROWS + c - SUB_ROWS of CTA 1's half (tokens from m0 + T/2):
      // runs of SUB_ROWS contiguous tokens, starting every SUB_ROWS columns.
      auto col_token = [&](int col) {
        const int j = col / BN_MMA, c = col - j * BN_MMA;
        return m0 + (c < L::SUB_ROWS ? j * L::SUB_ROWS + c : L::HALF_ROWS + j * L::SUB_ROWS + c - L::SUB_ROWS);
      };
      // Accumulator columns drained -> the leader's tm_empty[idx].
      auto signal_empty = [&](int idx) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (!leader)
            bulk_signal_cluster(payload_leader, signal_payload, SIGNAL_BYTES, tm_empty_leader + (uint32_t)(idx * 8));
          else if (q == 0 && eset == 0)
            mbar_arrive_expect_tx(&tm_empty[idx], TC2_EPI_WARPS * SIGNAL_BYTES);
          else
            mbar_arrive(&tm_empty[idx]);
        }
      };
#pragma unroll 2
      for (int ci = eset; ci < NCH; ci += 2) {
        const int col0 = ci * 32;
        const int split = min(32, (col0 / L::SUB_ROWS + 1) * L::SUB_ROWS - col0);
        const int tok_a = col_token(col0);
        const int tok_b = split < 32 ? col_token(col0 + split) : 0;
        uint32_t r[32];
        tc_ld_32x32b_x32(t_base + (uint32_t)col0, r);
        tc_wait_ld();
        // This warp's last chunk of sub-tile 0 read out of TMEM.
        if (L::SPLIT_RELEASE && col0 < BN_MMA && col0 + 64 >= BN_MMA) signal_empty(0);
        if (tok_a < p.rows || (split < 32 && tok_b < p.rows))
          pair_epilogue_chunk<EPI, ACT>(r, bias_v, p.res_scale, p.out + n, ld, p.rows, tok_a, split, tok_b);
      }
      signal_empty(L::SPLIT_RELEASE ? 1 : acc);
    }
  }

  __syncthreads();
  tc_fence_before();
  cluster_sync();  // the leader's MMAs are drained and both epilogues are done with TMEM
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, L::TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host
static bool encode_2d(const DeviceCtx& dev, CUtensorMap* map, CUtensorMapDataType dtype, const void* base,
                      uint64_t inner, uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                      CUtensorMapSwizzle swizzle) {
  auto fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(dev.encode_tiled);
  if (!fn) return false;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool gemm_tc_supported(const GemmArgs& g) {
  return g.precision == PK_FP16 && g.columns % TC_BM == 0 && g.inner % TC_BK == 0 && g.rows > 0 &&
         g.rows <= (int64_t)1 << 30 && (g.bits == 5 || g.bits == 6) && (g.groups << g.bits) <= 192 &&
         (reinterpret_cast<uintptr_t>(g.a) & 15) == 0 && (reinterpret_cast<uintptr_t>(g.codes) & 15) == 0;
}

template <int BN, int BITS, int EPI, int ACT, bool MASK>
static int launch_tc_kernel(const DeviceCtx& dev, const TcGemmParams& p, cudaStream_t stream) {
  using L = TcLayout<BN, BITS>;
  auto kernel = tc_palette_gemm_kernel<BN, BITS, EPI, ACT, MASK>;
  // Opt-in shared memory is a per-device function attribute; set it once per
  // device (a racing duplicate set is harmless).
  static bool configured[32] = {};
  if (dev.ordinal < 0 || dev.ordinal >= 32 || !configured[dev.ordinal]) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM_BYTES);
    if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(tc_palette_gemm)");
    if (dev.ordinal >= 0 && dev.ordinal < 32) configured[dev.ordinal] = true;
  }
  const int tiles = p.m_tiles * p.n_tiles;
  return cuda_error(launch_kernel(kernel, dim3(std::min(tiles, dev.sm_count)), dim3(TC_THREADS), L::SMEM_BYTES, stream, p),
                    "tc_palette_gemm launch");
}

// The time mask has its own instantiation of the bias + ReLU epilogue (the
// subsampling pointwise GEMMs); every other launch compiles without it.
template <int BN, int BITS, int EPI, int ACT>
static int launch_tc_spec(const DeviceCtx& dev, const TcGemmParams& p, cudaStream_t stream) {
  if constexpr (EPI == EPI_BIAS && ACT == PK_ACT_RELU)
    if (p.mask_lengths) return launch_tc_kernel<BN, BITS, EPI, ACT, true>(dev, p, stream);
  return launch_tc_kernel<BN, BITS, EPI, ACT, false>(dev, p, stream);
}

// Whether the residual is folded into the accumulator as residual / scale
// (EPI_RESADD): exact only when 1/scale is a power of two that f16 holds as a
// normal number; no activation may follow the residual (the encoder's
// residual GEMMs have none), and TMA needs a 16-byte aligned base.  The
// CTA-pair kernel only takes residuals that fold.
static bool residual_folds(const GemmArgs& g) {
  if (!g.has_residual || g.act != PK_ACT_NONE || (reinterpret_cast<uintptr_t>(g.residual) & 15) != 0) return false;
  int e = 0;
  const float m = std::frexp(g.residual_scale, &e);  // scale = m * 2^e, m in [0.5, 1)
  return m == 0.5f && e >= -13 && e <= 15;           // 1/scale = 2^(1-e) in [2^-14, 2^14]
}

static bool encode_residual(const DeviceCtx& dev, const GemmArgs& g, TcGemmParams& p, uint32_t box_rows) {
  p.res_inv_h = __half_as_ushort(__float2half_rn(1.0f / g.residual_scale));
  return encode_2d(dev, &p.tmap_res, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, g.residual, (uint64_t)g.columns,
                   (uint64_t)g.rows, (uint64_t)g.columns * 2, TC_BK, box_rows, CU_TENSOR_MAP_SWIZZLE_128B);
}

template <int BN, int BITS>
static int launch_tc(const DeviceCtx& dev, const GemmArgs& g, cudaStream_t stream) {
  using L = TcLayout<BN, BITS>;
  TcGemmParams p;
  if (!encode_2d(dev, &p.tmap_a, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, g.a, (uint64_t)g.inner, (uint64_t)g.rows,
                 (uint64_t)g.inner * 2, TC_BK, BN, CU_TENSOR_MAP_SWIZZLE_128B))
    return set_error(PK_E_CUDA, "cuTensorMapEncodeTiled failed for the activation operand");
  const uint64_t words_per_k = (uint64_t)g.columns * BITS / 32;
  if (!encode_2d(dev, &p.tmap_codes, CU_TENSOR_MAP_DATA_TYPE_UINT32, g.codes, words_per_k, (uint64_t)g.inner,
                 words_per_k * 4, L::WORDS_PER_ROW, TC_BK, CU_TENSOR_MAP_SWIZZLE_NONE))
    return set_error(PK_E_CUDA, "cuTensorMapEncodeTiled failed for the packed codes");
  p.palette = static_cast<const uint16_t*>(g.palette);
  p.bias = g.bias;
  p.residual = static_cast<const __half*>(g.residual);
  p.out = static_cast<__half*>(g.c);
  p.status = dev.status;
  p.rows = (int)g.rows;
  p.inner = (int)g.inner;
  p.columns = (int)g.columns;
  p.groups = g.groups;
  p.group_cols = (int)g.group_cols;
  p.res_scale = g.residual_scale;
  p.mask_lengths = g.mask_lengths;
  p.mask_group = g.mask_group > 0 ? g.mask_group : 1;
  p.mask_frames = g.mask_frames > 0 ? g.mask_frames : 1;
  p.m_tiles = (int)((g.rows + BN - 1) / BN);
  p.n_tiles = (int)(g.columns / TC_BM);
  const bool fold = residual_folds(g);
  if (fold && !encode_residual(dev, g, p, BN))
    return set_error(PK_E_CUDA, "cuTensorMapEncodeTiled failed for the residual operand");
  if (fold) return launch_tc_spec<BN, BITS, EPI_RESADD, PK_ACT_NONE>(dev, p, stream);
  const int epi = g.has_residual ? EPI_RESIDUAL : (g.bias ? EPI_BIAS : EPI_PLAIN);
  // The epilogues the encoder uses (gemm.ts:204-356): SiLU plain, plain,
  // folded residual, bias, bias + ReLU; the rest of the grid for general callers.
  switch (epi * 3 + g.act) {
    case EPI_PLAIN * 3 + PK_ACT_NONE: return launch_tc_spec<BN, BITS, EPI_PLAIN, PK_ACT_NONE>(dev, p, stream);
    case EPI_PLAIN * 3 + PK_ACT_SILU: return launch_tc_spec<BN, BITS, EPI_PLAIN, PK_ACT_SILU>(dev, p, stream);
    case EPI_PLAIN * 3 + PK_ACT_RELU: return launch_tc_spec<BN, BITS, EPI_PLAIN, PK_ACT_RELU>(dev, p, stream);
    case EPI_BIAS * 3 + PK_ACT_NONE: return launch_tc_spec<BN, BITS, EPI_BIAS, PK_ACT_NONE>(dev, p, stream);
    case EPI_BIAS * 3 + PK_ACT_SILU: return launch_tc_spec<BN, BITS, EPI_BIAS, PK_ACT_SILU>(dev, p, stream);
    case EPI_BIAS * 3 + PK_ACT_RELU: return launch_tc_spec<BN, BITS, EPI_BIAS, PK_ACT_RELU>(dev, p, stream);
    case EPI_RESIDUAL * 3 + PK_ACT_NONE: return launch_tc_spec<BN, BITS, EPI_RESIDUAL, PK_ACT_NONE>(dev, p, stream);
    case EPI_RESIDUAL * 3 + PK_ACT_SILU: return launch_tc_spec<BN, BITS, EPI_RESIDUAL, PK_ACT_SILU>(dev, p, stream);
    default: return launch_tc_spec<BN, BITS, EPI_RESIDUAL, PK_ACT_RELU>(dev, p, stream);
  }
}

template <int BN_MMA, int NSUB, int BITS, int EPI, int ACT>
static int launch_tc2_spec(const DeviceCtx& dev, const TcGemmParams& p, cudaStream_t stream) {
  using L = Tc2Layout<BN_MMA, NSUB, BITS>;
  auto kernel = tc2_palette_gemm_kernel<BN_MMA, NSUB, BITS, EPI, ACT>;
  // Per device: opt-in shared memory, then how many CTA pairs can be resident
  // at once (a pair needs two SMs of one GPC, so this can be below
  // sm_count / 2).
  static int max_pairs[32] = {};
  if (dev.ordinal < 0 || dev.ordinal >= 32) return set_error(PK_E_INVALID, "device ordinal out of range");
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see launch_kernel
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.blockDim = dim3(TC2_THREADS);
  cfg.dynamicSmemBytes = L::SMEM_BYTES;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;  // occupancy query with the cluster shape only
  if (!max_pairs[dev.ordinal]) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM_BYTES);
    if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(tc2_palette_gemm)");
    cfg.gridDim = dim3(2 * (dev.sm_count / 2));
    int clusters = 0;
    e = cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg);
    if (e != cudaSuccess) return cuda_error(e, "cudaOccupancyMaxActiveClusters(tc2_palette_gemm)");
    if (clusters <= 0) return set_error(PK_E_CUDA, "no CTA pair of the palette GEMM fits on this device");
    max_pairs[dev.ordinal] = std::min(clusters, dev.sm_count / 2);
  }
  const int pair_tiles = p.m_tiles * (p.n_tiles / 2);
  cfg.gridDim = dim3(2 * std::min(pair_tiles, max_pairs[dev.ordinal]));
  cfg.numAttrs = 2;
  return cuda_error(cudaLaunchKernelEx(&cfg, kernel, p), "tc2_palette_gemm launch");
}

template <int BN_MMA, int NSUB, int BITS>
static int launch_tc2(const DeviceCtx& dev, const GemmArgs& g, cudaStream_t stream) {
  using L = Tc2Layout<BN_MMA, NSUB, BITS>;
  TcGemmParams p;
  if (!encode_2d(dev, &p.tmap_a, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, g.a, (uint64_t)g.inner, (uint64_t)g.rows,
                 (uint64_t)g.inner * 2, TC_BK, L::HALF_ROWS, CU_TENSOR_MAP_SWIZZLE_128B))
    return set_error(PK_E_CUDA, "cuTensorMapEncodeTiled failed for the activation operand");
  const uint64_t words_per_k = (uint64_t)g.columns * BITS / 32;
  if (!encode_2d(dev, &p.tmap_codes, CU_TENSOR_MAP_DATA_TYPE_UINT32, g.codes, words_per_k, (uint64_t)g.inner,
                 words_per_k * 4, L::WORDS_PER_ROW, TC_BK, CU_TENSOR_MAP_SWIZZLE_NONE))
    return set_error(PK_E_CUDA, "cuTensorMapEncodeTiled failed for the packed codes");
  p.palette = static_cast<const uint16_t*>(g.palette);
  p.bias = g.bias;
  p.residual = static_cast<const __half*>(g.residual);
  p.out = static_cast<__half*>(g.c);
  p.status = dev.status;
  p.rows = (int)g.rows;
  p.inner = (int)g.inner;
  p.columns = (int)g.columns;
  p.groups = g.groups;
  p.group_cols = (int)g.group_cols;
  p.res_scale = g.residual_scale;
  p.mask_lengths = g.mask_lengths;
  p.mask_group = g.mask_group > 0 ? g.mask_group : 1;
  p.mask_frames = g.mask_frames > 0 ? g.mask_frames : 1;
  p.m_tiles = (int)((g.rows + L::T - 1) / L::T);
  p.n_tiles = (int)(g.columns / TC_BM);
  if (g.has_residual && !residual_folds(g)) return set_error(PK_E_INVALID, "CTA-pair GEMM: residual must fold");
  if (g.has_residual && !encode_residual(dev, g, p, L::HALF_ROWS))
    return set_error(PK_E_CUDA, "cuTensorMapEncodeTiled failed for the residual operand");
  const int epi = g.has_residual ? EPI_RESADD : (g.bias ? EPI_BIAS : EPI_PLAIN);
#define PK_TC2(E, A) launch_tc2_spec<BN_MMA, NSUB, BITS, E, A>(dev, p, stream)
  switch (epi * 3 + g.act) {
    case EPI_PLAIN * 3 + PK_ACT_NONE: return PK_TC2(EPI_PLAIN, PK_ACT_NONE);
    case EPI_PLAIN * 3 + PK_ACT_SILU: return PK_TC2(EPI_PLAIN, PK_ACT_SILU);
    case EPI_PLAIN * 3 + PK_ACT_RELU: return PK_TC2(EPI_PLAIN, PK_ACT_RELU);
    case EPI_BIAS * 3 + PK_ACT_NONE: return PK_TC2(EPI_BIAS, PK_ACT_NONE);
    case EPI_BIAS * 3 + PK_ACT_SILU: return PK_TC2(EPI_BIAS, PK_ACT_SILU);
    case EPI_BIAS * 3 + PK_ACT_RELU: return PK_TC2(EPI_BIAS, PK_ACT_RELU);
    case EPI_RESADD * 3 + PK_ACT_NONE: return PK_TC2(EPI_RESADD, PK_ACT_NONE);
    default: return set_error(PK_E_INVALID, "CTA-pair GEMM: residual with an activation");
  }
#undef PK_TC2
}


// Tile choice: minimise (waves of persistent CTAs or CTA pairs) x (time per
// tile), with times fitted to B200 measurements of the encoder's shapes.  A
// k-stage costs about the same whatever the token tile (the weight decode,
// not the MMA, sets its pace): ~0.70 us for a single-CTA tile, ~0.78 us for a
// CTA pair (twice the features, decoded in parallel), so larger token tiles
// win per FLOP until wave quantization or the epilogue bites.  Single-CTA
// tiles hide their epilogue behind the next tile (double-buffered TMEM,
// ~0.6 us left); pair tiles of 384 / 512 tokens fill TMEM and expose it
// (~5.1 / ~7.9 us).  Residual k-steps (no decode) count half a stage.  The
// 256-token pair tile measured no faster than the single-CTA one and is left
// to the test hook.  Returns the token tile, negated for the CTA-pair kernel.
static int choose_tile(const DeviceCtx& dev, const GemmArgs& g, bool allow_single, bool allow_pair) {
  if (g.rows <= 128 && allow_single) return 128;
  const int n_tiles = (int)(g.columns / TC_BM);
  const double kb = (double)(g.inner / TC_BK);
  const bool fold = residual_folds(g);
  int best = allow_single ? 256 : -384;
  double best_cost = 1e30;
  if (allow_single)
    for (int bn : {128, 192, 256}) {
      const int64_t tiles = (g.rows + bn - 1) / bn * n_tiles;
      const int64_t waves = (tiles + dev.sm_count - 1) / dev.sm_count;
      const double stages = kb + (fold ? 0.5 * TC_BM / TC_BK : 0.0);
      const double cost = (double)waves * (stages * 0.70 + 0.6);
      if (cost < best_cost - 1e-9) best_cost = cost, best = bn;
    }
  if (allow_pair)
    for (int t : {384, 512}) {
      const int64_t tiles = (g.rows + t - 1) / t * (n_tiles / 2);
      const int64_t waves = (tiles + dev.sm_count / 2 - 1) / (dev.sm_count / 2);
      const double stages = kb + (fold ? 0.5 * 2 * TC_BM / TC_BK : 0.0);
      const double cost = (double)waves * (stages * 0.78 + (t == 384 ? 5.1 : 7.9));
      if (cost < best_cost - 1e-9) best_cost = cost, best = -t;
    }
  return best;
}

int launch_gemm_tc(const DeviceCtx& dev, const GemmArgs& g, cudaStream_t stream, int forced_bn) {
  if (!gemm_tc_supported(g)) return set_error(PK_E_SHAPE, "shape not supported by the tensor-core GEMM");
  // Route 3 keeps to single-CTA tiles, route 4 to CTA pairs (where N tiles
  // by 256); otherwise the cost model picks.  A tile forced through
  // pk_debug_set_gemm_tile overrides both.
  const bool allow_pair =
      g_gemm_route != 3 && g.columns % (2 * TC_BM) == 0 && (!g.has_residual || residual_folds(g));
  const bool allow_single = g_gemm_route != 4 || !allow_pair;
  int bn = forced_bn ? forced_bn : g_gemm_tile ? g_gemm_tile : choose_tile(dev, g, allow_single, allow_pair);
  if (bn < 0 && !allow_pair) bn = 256;
  if (g.mask_lengths) {
    // The time mask rides on the single-CTA bias + ReLU epilogue only; the
    // caller masks separately otherwise.
    const bool fused = bn > 0 && g.bias && g.act == PK_ACT_RELU && !g.has_residual;
    if (g.mask_applied) *g.mask_applied = fused;
    if (!fused) {
      GemmArgs plain = g;
      plain.mask_lengths = nullptr;
      return launch_gemm_tc(dev, plain, stream, bn);
    }
  }
  const bool b5 = g.bits == 5;
  switch (bn) {
    case -512: return b5 ? launch_tc2<256, 2, 5>(dev, g, stream) : launch_tc2<256, 2, 6>(dev, g, stream);
    case -384: return b5 ? launch_tc2<192, 2, 5>(dev, g, stream) : launch_tc2<192, 2, 6>(dev, g, stream);
    case -256: return b5 ? launch_tc2<256, 1, 5>(dev, g, stream) : launch_tc2<256, 1, 6>(dev, g, stream);
    case 256: return b5 ? launch_tc<256, 5>(dev, g, stream) : launch_tc<256, 6>(dev, g, stream);
    case 192: return b5 ? launch_tc<192, 5>(dev, g, stream) : launch_tc<192, 6>(dev, g, stream);
    case 128: return b5 ? launch_tc<128, 5>(dev, g, stream) : launch_tc<128, 6>(dev, g, stream);
    default: return set_error(PK_E_INVALID, "unknown GEMM tile");
  }
}

}  // namespace pk
