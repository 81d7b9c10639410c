// attention_umma.cu -- FP16 relative-position MHSA on the sm_100a tensor cores
// (tcgen05.mma, accumulators in TMEM).
//
// Same arithmetic contract as RELATIVE_ATTENTION_WGSL
// (src/webgpu/kernels/attention.ts:418-728):
//   s_ij = ((q_i+u).k_j + (q_i+v).p[T-1-i+j]) / sqrt(128), keys j >= valid
//   excluded, f32 softmax over keys, ctx_i = sum_j prob_ij v_j, rows i >= valid
//   zero.
// A tile = (128 queries, head, window), windows of at most 192 frames:
//   S  = (Q+u) . K^T       M=128, N=192 keys          TMEM columns [0, 192)
//   BD = (Q+v) . Pband^T   M=128, N=320 band rows     TMEM columns [192, 512)
//        band row rr holds relative position T-128-q0+rr, so query row r and
//        key j read band row 127 - r + j;
//   softmax over the full key row (exact row max, base 2, f32), the
//   probabilities rounded to f16 into shared memory as the next MMA's A;
//   O  = P . V             M=128, N=128 dims, K=192   TMEM columns [0, 128)
// (Q+u), (Q+v) and the probabilities are rounded to f16 for the MMAs; scores,
// softmax and accumulation are f32 -- the rounding points of the mma.sync
// kernel in attention_tc.cu.
//
// Operands: Q, K, V and the positional band arrive by TMA with 128-byte
// swizzle through 3-D tensor maps, so rows past the window read as zero (K
// and the band K-major; V, read as [keys x dims], is the MN-major B of the
// last MMA); the threads turn Q into (Q+u) in place and (Q+v) beside it.  The
// band needs the positions re-laid out row-major [8][2T-1][128]
// (launch_positions_rowmajor), which the encoder does once.  The context
// leaves through a TMA store of the f16 tile staged in shared memory.
//
// The per-row shift of BD (row r reads its key j at column 127 - r + j) is a
// skewed read: each warp loads the 64 BD columns its 32 rows need for 32 keys;
// every thread parks its row's 64 values in shared memory and reads back the
// 32 it needs at its own offset (both directions conflict-free).
//
// Persistent CTAs, one per SM (shared memory ~225 KB, TMEM all 512 columns),
// walk the tiles; the next tile's operands load while this one finishes: the
// band once the scores are formed, Q and K once PV has consumed the
// probabilities and V.  The context is staged in a buffer of its own, so its
// TMA store overlaps the next tile (the store of tile i must have read the
// staging before tile i+1 writes it, a whole tile later).
// Threads: 8 warps; warp w reads TMEM lanes 32 (w % 4) .. +31 (query rows) and
// handles keys [96 (w / 4), +96) of them in the softmax and dims
// [64 (w / 4), +64) in the epilogue.  Thread 0 issues the TMA loads and MMAs.
#include <cuda.h>
#include <algorithm>
#include <cudaTypedefs.h>

#include "pk_common.cuh"
#include "pk_internal.h"

namespace pk {

namespace {

constexpr int UQ = 128;       // queries per CTA (MMA M)
constexpr int UKEYS = 192;    // key columns (windows of at most 192 frames)
constexpr int UBAND = 320;    // band rows: 127 + 192, a multiple of 16
constexpr int UTHREADS = 256;
// Shared-memory layout (bytes from a 1024-aligned base).
constexpr int U_QU = 0;                        // (Q+u): 2 dim blocks x 128 rows x 128 B
constexpr int U_QV = 32768;                    // (Q+v)
constexpr int U_P = 0;                         // probabilities: 3 key blocks x 128 rows x 128 B (after the MMAs)
constexpr int U_KV = 65536;                    // K (then V): 2 dim blocks x 192 rows x 128 B
constexpr int U_PB = U_KV + 2 * UKEYS * 128;   // positional band: 2 dim blocks x 320 rows x 128 B
constexpr int U_CTX = U_PB + 2 * UBAND * 128;  // context staging: 2 dim blocks x 128 rows x 128 B
// Row max [2][128] and row sum [2][128] live in the second half of the (Q+v)
// block: written after the S and BD MMAs have read (Q+v), past the end of the
// probabilities, and read before the next tile rebuilds (Q+v).
constexpr int U_RED = U_P + 3 * UQ * 128;
constexpr int U_BAR = U_CTX + 2 * UQ * 128;    // 6 mbarriers
constexpr int U_MISC = U_BAR + 64;             // TMEM slot, abort flag, barrier arm counts
constexpr int U_SMEM = U_MISC + 64 + 1024;     // + alignment slack
static_assert(U_PB % 1024 == 0 && U_CTX % 1024 == 0 && (UKEYS * 128) % 1024 == 0 && (UBAND / 2 * 128) % 1024 == 0,
              "swizzled operands must start on 1024-byte boundaries");
static_assert(U_RED >= U_QV && U_RED + 4 * UQ * 4 <= U_KV, "row statistics inside the (Q+v) block, after P");
static_assert(U_SMEM <= 232448, "shared memory budget");
static_assert(8 * 32 * 68 * 4 <= 2 * UBAND * 128, "per-thread shift scratch rows fit in the band region");

constexpr uint32_t IDESC_S = umma_idesc_f16(UQ, UKEYS, 0, 0);
constexpr uint32_t IDESC_BD = umma_idesc_f16(UQ, UBAND / 2, 0, 0);
constexpr uint32_t IDESC_PV = umma_idesc_f16(UQ, 128, 0, /*B = V, MN-major*/ 1);

struct UmmaAttnParams {
  CUtensorMap tmap_q;    // qkv [B][T][3072] f16, box {64, 128, 1}, 128B swizzle (rows past T read as zero)
  CUtensorMap tmap_kv;   // the same tensor, box {64, 192, 1}
  CUtensorMap tmap_pos;  // positions [8][2T-1][128] f16, box {64, 160, 1}
  CUtensorMap tmap_ctx;  // context [B][T][1024] f16, box {64, 128, 1} (rows past T are not written)
  const float* bias_u;
  const float* bias_v;
  const uint32_t* valid_lengths;
  __half* context;
  unsigned int* status;
  int frames;
  int batch;
};

__device__ __forceinline__ void sts128(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

__device__ __forceinline__ uint32_t pack_h2f(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Byte offset of 16-byte chunk `c` (of 8) in row `r` of a 128-row, 128-byte
// swizzled K-major block.
__device__ __forceinline__ uint32_t sw128(int r, int c) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

__global__ void __launch_bounds__(UTHREADS, 1) rel_attention_umma_kernel(const __grid_constant__ UmmaAttnParams p) {
  pdl_entry();
  extern __shared__ uint8_t u_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(u_raw) + 1023) & ~uintptr_t(1023));
  const int T = p.frames;
  const int qtiles = (T + UQ - 1) / UQ;
  const int num_tiles = qtiles * 8 * p.batch;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + U_BAR);
  // Each barrier completes once per tile (phase parity = tile iteration & 1).
  uint64_t* bar_q = bars;       // Q landed
  uint64_t* bar_k = bars + 1;   // K landed
  uint64_t* bar_pb = bars + 2;  // band landed
  uint64_t* bar_v = bars + 3;   // V landed
  uint64_t* bar_sb = bars + 4;  // S and BD MMAs done
  uint64_t* bar_o = bars + 5;   // PV MMAs done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + U_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + U_MISC + 4);
  float* red_max = reinterpret_cast<float*>(sm + U_RED);
  float* red_sum = red_max + 2 * UQ;

  if (tid == 0) {
    for (int i = 0; i < 6; ++i) {
      mbar_init(&bars[i], 1);
      reinterpret_cast<uint32_t*>(sm + U_MISC + 16)[i] = 0;
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // Tile t = (query tile, head, window), query tile fastest.
  auto tile_of = [&](int t, int& q0, int& h, int& b) {
    q0 = (t % qtiles) * UQ;
    h = (t / qtiles) % 8;
    b = t / (qtiles * 8);
  };
  // Loads and MMA commits are issued by thread 0, which counts each
  // barrier's arms for the unwind.
  uint32_t* arms = reinterpret_cast<uint32_t*>(sm + U_MISC + 16);  // thread 0 only
  auto load_q = [&](int t) {
    int q0, h, b;
    tile_of(t, q0, h, b);
    mbar_arrive_expect_tx(bar_q, 2 * UQ * 128);
    for (int kb = 0; kb < 2; ++kb) tma_load_3d(sm + U_QU + kb * UQ * 128, &p.tmap_q, bar_q, h * 128 + kb * 64, q0, b);
    ++arms[0];
  };
  auto load_kv = [&](int t, uint64_t* bar, int col0, int idx) {  // col0 1024: K, 2048: V
    int q0, h, b;
    tile_of(t, q0, h, b);
    mbar_arrive_expect_tx(bar, 2 * UKEYS * 128);
    for (int kb = 0; kb < 2; ++kb)
      tma_load_3d(sm + U_KV + kb * UKEYS * 128, &p.tmap_kv, bar, col0 + h * 128 + kb * 64, 0, b);
    ++arms[idx];
  };
  auto load_band = [&](int t) {
    int q0, h, b;
    tile_of(t, q0, h, b);
    const int band0 = T - UQ - q0;  // relative position of band row 0
    mbar_arrive_expect_tx(bar_pb, 2 * UBAND * 128);
    for (int kb = 0; kb < 2; ++kb)
      for (int half = 0; half < 2; ++half)
        tma_load_3d(sm + U_PB + kb * UBAND * 128 + half * (UBAND / 2) * 128, &p.tmap_pos, bar_pb, kb * 64,
                    band0 + half * (UBAND / 2), h);
    ++arms[2];
  };
  if (tid == 0 && (int)blockIdx.x < num_tiles) {
    tma_prefetch_desc(&p.tmap_q);
    tma_prefetch_desc(&p.tmap_kv);
    tma_prefetch_desc(&p.tmap_pos);
    tma_prefetch_desc(&p.tmap_ctx);
    load_q(blockIdx.x);
    load_kv(blockIdx.x, bar_k, 1024, 1);
    load_band(blockIdx.x);
  }

  const int qd = warp & 3, kh = warp >> 2;
  const int r = qd * 32 + lane;  // query row in the tile
  const uint32_t t_row = tmem_base + ((uint32_t)(qd * 32) << 16);
  const float scale = 0.08838834764831845f * 1.4426950408889634f;  // log2(e) / sqrt(128): base-2 softmax
  uint32_t it = 0;
#pragma unroll 1
  for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++it) {
    const uint32_t ph = it & 1;
    int q0, h, b;
    tile_of(t, q0, h, b);
    const int valid = min((int)p.valid_lengths[b], T);
    const int tn = t + (int)gridDim.x;
    const bool has_next = tn < num_tiles;
    // ---- (Q+u) in place and (Q+v) beside it, rounded to f16, in the same
    // swizzled K-major layout (rows past the window stay zero).  Each thread
    // keeps one 8-dim chunk column, so its biases load once per tile.
    bool ok;
    {
      const int c8 = tid & 15;
      float ub[8], vb[8];
      *reinterpret_cast<float4*>(ub) = __ldg(reinterpret_cast<const float4*>(p.bias_u + h * 128 + c8 * 8));
      *reinterpret_cast<float4*>(ub + 4) = __ldg(reinterpret_cast<const float4*>(p.bias_u + h * 128 + c8 * 8 + 4));
      *reinterpret_cast<float4*>(vb) = __ldg(reinterpret_cast<const float4*>(p.bias_v + h * 128 + c8 * 8));
      *reinterpret_cast<float4*>(vb + 4) = __ldg(reinterpret_cast<const float4*>(p.bias_v + h * 128 + c8 * 8 + 4));
      ok = mbar_wait(bar_q, ph, abort_flag, p.status, PK_STATUS_TIMEOUT_TMA);
#pragma unroll 4
      for (int rr = tid >> 4; rr < UQ && ok; rr += UTHREADS / 16) {
        const uint32_t off = (uint32_t)((c8 >> 3) * (UQ * 128)) + sw128(rr, c8 & 7);
        const uint4 raw = *reinterpret_cast<const uint4*>(sm + U_QU + off);
        const __half2* hv = reinterpret_cast<const __half2*>(&raw);
        const bool live = q0 + rr < T;
        uint32_t qu[4], qv[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 f = __half22float2(hv[k]);
          qu[k] = live ? pack_h2f(f.x + ub[2 * k], f.y + ub[2 * k + 1]) : 0u;
          qv[k] = live ? pack_h2f(f.x + vb[2 * k], f.y + vb[2 * k + 1]) : 0u;
        }
        sts128(smem_addr(sm + U_QU + off), qu[0], qu[1], qu[2], qu[3]);
        sts128(smem_addr(sm + U_QV + off), qv[0], qv[1], qv[2], qv[3]);
      }
    }
    fence_proxy_async_smem();  // the threads' writes become visible to the tensor core
    ok = __syncthreads_and(ok) != 0;
    if (!ok) break;
    // ---- BD = (Q+v) . band^T as soon as the band is in, then S = (Q+u) . K^T
    if (tid == 0) {
      const uint32_t qu = smem_addr(sm + U_QU), qv = smem_addr(sm + U_QV);
      const uint32_t kbase = smem_addr(sm + U_KV), pbase = smem_addr(sm + U_PB);
      if (mbar_wait(bar_pb, ph, abort_flag, p.status, PK_STATUS_TIMEOUT_TMA)) {
        tc_fence_after();
#pragma unroll
        for (int half = 0; half < 2; ++half)
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {  // 8 K=16 steps over the 128 dims
            const uint32_t ko = (uint32_t)((ks >> 2) * (UQ * 128) + (ks & 3) * 32);
            const uint32_t bo = (uint32_t)((ks >> 2) * UBAND * 128 + half * (UBAND / 2) * 128 + (ks & 3) * 32);
            tc_mma_f16(tmem_base + (uint32_t)(UKEYS + half * (UBAND / 2)), umma_smem_desc(qv + ko, 16, 1024, 2),
                       umma_smem_desc(pbase + bo, 16, 1024, 2), IDESC_BD, ks > 0 ? 1u : 0u);
          }
        if (mbar_wait(bar_k, ph, abort_flag, p.status, PK_STATUS_TIMEOUT_TMA)) {
          tc_fence_after();
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {
            const uint32_t ko = (uint32_t)((ks >> 2) * (UQ * 128) + (ks & 3) * 32);
            tc_mma_f16(tmem_base, umma_smem_desc(qu + ko, 16, 1024, 2),
                       umma_smem_desc(kbase + (uint32_t)((ks >> 2) * UKEYS * 128 + (ks & 3) * 32), 16, 1024, 2),
                       IDESC_S, ks > 0 ? 1u : 0u);
          }
        }
        tc_commit(bar_sb);  // also after a failed K wait: the BD MMAs must drain
        ++arms[4];
      }
    }
    ok = mbar_wait(bar_sb, ph, abort_flag, p.status, PK_STATUS_TIMEOUT_MMA);
    ok = __syncthreads_and(ok && *abort_flag == 0) != 0;  // thread 0's own flag covers a failed K wait
    if (!ok) break;
    tc_fence_after();
    if (tid == 0) load_kv(t, bar_v, 2048, 3);  // V replaces K, which the S MMAs have read
    {
    // ---- scores = (S + shifted BD) * scale, masked; written back over S.
    // Row r needs BD window entry 31 - lane + jj for key jc + jj: the thread
    // parks its 64 window values in its own scratch row (16-byte stores, row
    // pitch 68 floats: conflict-free both ways) and reads them back shifted.
    // The next chunk's TMEM loads are issued before this chunk's arithmetic.
    const uint32_t scr_row = smem_addr(sm + U_PB) + (uint32_t)((warp * 32 + lane) * 68 * 4);
    float mx = -3.402823466e+38f;
    uint32_t sa[32], sb[32], d0[32], d1[32];
    auto load_chunk = [&](int jc, uint32_t(&sv)[32]) {
      const uint32_t cb = (uint32_t)(UKEYS + 96 - 32 * qd + jc);  // band rows 96 - 32 qd + jc .. +63
      tc_ld_32x32b_x32(t_row + (uint32_t)jc, sv);
      tc_ld_32x32b_x32(t_row + cb, d0);
      tc_ld_32x32b_x32(t_row + cb + 32, d1);
    };
    auto score_chunk = [&](int c, uint32_t(&sv)[32], uint32_t(&next)[32]) {
      const int jc = kh * 96 + c * 32;
      tc_wait_ld();
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        sts128(scr_row + k * 16, d0[4 * k], d0[4 * k + 1], d0[4 * k + 2], d0[4 * k + 3]);
        sts128(scr_row + 128 + k * 16, d1[4 * k], d1[4 * k + 1], d1[4 * k + 2], d1[4 * k + 3]);
      }
      if (c < 2) load_chunk(jc + 32, next);
      const uint32_t rd = scr_row + (uint32_t)((31 - lane) * 4);
      if (jc + 32 <= valid) {
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) {
          float bd;
          asm volatile("ld.shared.f32 %0, [%1];" : "=f"(bd) : "r"(rd + jj * 4));
          const float v = (__uint_as_float(sv[jj]) + bd) * scale;
          mx = fmaxf(mx, v);
          sv[jj] = __float_as_uint(v);
        }
      } else {
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) {
          float bd;
          asm volatile("ld.shared.f32 %0, [%1];" : "=f"(bd) : "r"(rd + jj * 4));
          float v = (__uint_as_float(sv[jj]) + bd) * scale;
          if (jc + jj >= valid) v = -3.402823466e+38f;
          mx = fmaxf(mx, v);
          sv[jj] = __float_as_uint(v);
        }
      }
      tc_st_32x32b_x32(t_row + (uint32_t)jc, sv);
    };
    load_chunk(kh * 96, sa);
    score_chunk(0, sa, sb);
    score_chunk(1, sb, sa);
    score_chunk(2, sa, sb);
    tc_wait_st();
    red_max[kh * UQ + r] = mx;
    fence_proxy_async_smem();  // scratch writes ordered before the next band's TMA writes
    __syncthreads();
    if (tid == 0 && has_next) load_band(tn);  // the BD MMAs and the scratch are done with the band region
    mx = fmaxf(red_max[r], red_max[UQ + r]);
    // ---- probabilities (f16) into the A operand of the PV MMA; f32 row sums
    float sum = 0.0f;
    const uint32_t pbuf = smem_addr(sm + U_P);
    auto prob_chunk = [&](int c, uint32_t(&sv)[32], uint32_t(&next)[32]) {
      const int jc = kh * 96 + c * 32;
      tc_wait_ld();
      if (c < 2) tc_ld_32x32b_x32(t_row + (uint32_t)(jc + 32), next);
      uint32_t pk[16];
      if (jc + 32 <= valid) {
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float p0 = ex2f(__uint_as_float(sv[2 * e]) - mx);
          const float p1 = ex2f(__uint_as_float(sv[2 * e + 1]) - mx);
          sum += p0 + p1;
          pk[e] = pack_h2f(p0, p1);
        }
      } else {
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const int j = jc + 2 * e;
          const float p0 = j < valid ? ex2f(__uint_as_float(sv[2 * e]) - mx) : 0.0f;
          const float p1 = j + 1 < valid ? ex2f(__uint_as_float(sv[2 * e + 1]) - mx) : 0.0f;
          sum += p0 + p1;
          pk[e] = pack_h2f(p0, p1);
        }
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int key0 = jc + 8 * q;
        sts128(pbuf + (uint32_t)((key0 >> 6) * (UQ * 128)) + sw128(r, (key0 >> 3) & 7), pk[4 * q], pk[4 * q + 1],
               pk[4 * q + 2], pk[4 * q + 3]);
      }
    };
    tc_ld_32x32b_x32(t_row + (uint32_t)(kh * 96), sa);
    prob_chunk(0, sa, sb);
    prob_chunk(1, sb, sa);
    prob_chunk(2, sa, sb);
    red_sum[kh * UQ + r] = sum;
    fence_proxy_async_smem();
  }
    tc_fence_before();
    __syncthreads();
    // ---- O = P . V
    if (tid == 0) {
      bulk_wait_group_read_all();  // the previous tile's context store has read the staging
      if (mbar_wait(bar_v, ph, abort_flag, p.status, PK_STATUS_TIMEOUT_TMA)) {
        tc_fence_after();
        const uint32_t pbuf = smem_addr(sm + U_P), vbase = smem_addr(sm + U_KV);
#pragma unroll
        for (int ks = 0; ks < UKEYS / 16; ++ks) {
          const uint32_t ao = (uint32_t)((ks >> 2) * (UQ * 128) + (ks & 3) * 32);
          tc_mma_f16(tmem_base, umma_smem_desc(pbuf + ao, 16, 1024, 2),
                     umma_smem_desc(vbase + (uint32_t)(ks * 2048), UKEYS * 128, 1024, 2), IDESC_PV,
                     ks > 0 ? 1u : 0u);
        }
        tc_commit(bar_o);
        ++arms[5];
      }
    }
    ok = mbar_wait(bar_o, ph, abort_flag, p.status, PK_STATUS_TIMEOUT_EPILOGUE);
    ok = __syncthreads_and(ok) != 0;
    if (!ok) break;
    tc_fence_after();
    if (tid == 0 && has_next) {  // the probabilities and V are consumed
      load_q(tn);
      load_kv(tn, bar_k, 1024, 1);
    }
    {
      // ---- epilogue: warp w stages dims [64 (w / 4), +64) of its 32 rows
      // (f16, swizzled) in the context buffer; one TMA store per dim block
      // (rows past the window are clipped by the tensor bounds).
      const int dh = warp >> 2;
      uint32_t o0[32], o1[32];
      tc_ld_32x32b_x32(t_row + (uint32_t)(dh * 64), o0);
      tc_ld_32x32b_x32(t_row + (uint32_t)(dh * 64 + 32), o1);
      tc_wait_ld();
      const bool live = q0 + r < valid;
      const float inv = live ? 1.0f / (red_sum[r] + red_sum[UQ + r]) : 0.0f;  // rows past valid: zero
      const uint32_t obuf = smem_addr(sm + U_CTX + dh * (UQ * 128));
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const uint32_t(&o)[32] = q < 4 ? o0 : o1;
        const int e = (q & 3) * 8;
        sts128(obuf + sw128(r, q), pack_h2f(__uint_as_float(o[e]) * inv, __uint_as_float(o[e + 1]) * inv),
               pack_h2f(__uint_as_float(o[e + 2]) * inv, __uint_as_float(o[e + 3]) * inv),
               pack_h2f(__uint_as_float(o[e + 4]) * inv, __uint_as_float(o[e + 5]) * inv),
               pack_h2f(__uint_as_float(o[e + 6]) * inv, __uint_as_float(o[e + 7]) * inv));
      }
      fence_proxy_async_smem();
    }
    tc_fence_before();
    __syncthreads();  // O read out of TMEM (the next tile's MMAs may overwrite it) and staged
    if (tid == 0) {
      for (int kb = 0; kb < 2; ++kb)
        tma_store_3d(&p.tmap_ctx, sm + U_CTX + kb * (UQ * 128), h * 128 + kb * 64, q0, b);
      bulk_commit_group();
    }
  }
  // Unwind: every load and MMA commit this CTA armed has completed, and its
  // stores are done, before shared memory and TMEM are released (immediate on
  // the normal path).
  if (tid == 0) {
    for (int i = 0; i < 6; ++i)
      if (arms[i] > 0) mbar_wait_drain(&bars[i], (arms[i] - 1) & 1, p.status);
    bulk_wait_group_all();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

bool encode_tmap(const DeviceCtx& dev, CUtensorMap* map, int rank, const void* base, const cuuint64_t* dims,
                 const cuuint64_t* strides_bytes, const cuuint32_t* box) {
  auto fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(dev.encode_tiled);
  if (!fn) return false;
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, (cuuint32_t)rank, const_cast<void*>(base), dims,
                        strides_bytes, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace

bool rel_attention_umma_supported(const DeviceCtx& dev, int frames, const void* qkv, const void* positions_rowmajor,
                                  const void* context) {
  return dev.encode_tiled != nullptr && frames >= 1 && frames <= UKEYS && positions_rowmajor != nullptr &&
         (reinterpret_cast<uintptr_t>(qkv) & 15) == 0 && (reinterpret_cast<uintptr_t>(positions_rowmajor) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(context) & 15) == 0;
}

int launch_rel_attention_umma(const DeviceCtx& dev, int batch, int frames, const void* qkv,
                              const void* positions_rowmajor, const float* bias_u, const float* bias_v,
                              const uint32_t* valid_lengths, void* context, cudaStream_t stream) {
  if (!rel_attention_umma_supported(dev, frames, qkv, positions_rowmajor, context))
    return set_error(PK_E_SHAPE, "tensor-core attention needs frames <= 192, row-major positions and 16-byte "
                                 "aligned buffers");
  UmmaAttnParams p;
  const int P = 2 * frames - 1;
  const cuuint64_t T = (cuuint64_t)frames, B = (cuuint64_t)batch;
  {
    const cuuint64_t dims[3] = {3072, T, B};
    const cuuint64_t strides[2] = {3072 * 2, T * 3072 * 2};
    const cuuint32_t box_q[3] = {64, UQ, 1}, box_kv[3] = {64, UKEYS, 1};
    if (!encode_tmap(dev, &p.tmap_q, 3, qkv, dims, strides, box_q) ||
        !encode_tmap(dev, &p.tmap_kv, 3, qkv, dims, strides, box_kv))
      return set_error(PK_E_CUDA, "cuTensorMapEncodeTiled failed (attention qkv)");
  }
  {
    const cuuint64_t dims[3] = {128, (cuuint64_t)P, 8};
    const cuuint64_t strides[2] = {128 * 2, (cuuint64_t)P * 128 * 2};
    const cuuint32_t box[3] = {64, UBAND / 2, 1};
    if (!encode_tmap(dev, &p.tmap_pos, 3, positions_rowmajor, dims, strides, box))
      return set_error(PK_E_CUDA, "cuTensorMapEncodeTiled failed (attention positions)");
  }
  {
    const cuuint64_t dims[3] = {1024, T, B};
    const cuuint64_t strides[2] = {1024 * 2, T * 1024 * 2};
    const cuuint32_t box[3] = {64, UQ, 1};
    if (!encode_tmap(dev, &p.tmap_ctx, 3, context, dims, strides, box))
      return set_error(PK_E_CUDA, "cuTensorMapEncodeTiled failed (attention context)");
  }
  p.bias_u = bias_u;
  p.bias_v = bias_v;
  p.valid_lengths = valid_lengths;
  p.context = static_cast<__half*>(context);
  p.status = dev.status;
  p.batch = batch;
  p.frames = frames;
  const int st = set_max_dynamic_smem(reinterpret_cast<const void*>(rel_attention_umma_kernel), U_SMEM);
  if (st != PK_OK) return st;
  const int num_tiles = (frames + UQ - 1) / UQ * 8 * batch;
  const dim3 grid((unsigned)std::min(num_tiles, dev.sm_count));  // persistent: one CTA per SM
  return cuda_error(launch_kernel(rel_attention_umma_kernel, grid, dim3(UTHREADS), U_SMEM, stream, p),
                    "rel_attention_umma launch");
}

}  // namespace pk
