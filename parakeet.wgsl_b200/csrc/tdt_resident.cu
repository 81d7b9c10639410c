// tdt_resident.cu -- the greedy TDT decoder with its FP16 weights resident on
// chip, all windows in lockstep (up to 40 windows per launch, the reference's
// batch capacity, src/webgpu/encoder.ts:68).
//
// The cluster-per-window decoder (tdt_decoder.cu) re-streams every LSTM
// weight for every emitted token of every window, which bounds it by L2->SM
// bandwidth.  Here 128 co-resident CTAs (a cooperative launch, one per SM)
// each hold a fixed 1/128 of every decoder weight in shared memory for the
// whole launch: LSTM channels [5 c, 5 c + 5) of both layers (all four gates
// of each, so the cell update is local), the projector outputs of those
// channels and head columns [8 c, 8 c + 8) (CTA 0 also the blank's column,
// CTAs 1..5 one duration column each).  Each step every CTA computes its slice for every
// window that needs it, writes the slice to an exchange area in global memory
// and meets the others at a grid barrier (thread 0 arrives on a counter and
// waits with an acquire load, bounded by %globaltimer); readers fetch the
// exchanged vectors through L2 (ld.global.cg).  A step is: the LSTM update of
// the windows that emitted a token (layer 0, layer 1, projector: 3 barriers),
// then the joint of the active windows (1 barrier); argmax partials of all
// CTAs are reduced by every CTA, so all take the same decisions and run the
// same number of barriers.
//
// Shared memory holds the weight slices (~131 KB) and one half of a phase's
// inputs at a time: the 1280 LSTM inputs, the 640 projector inputs and the
// 640 joint inputs are staged in two halves, and the chains -- whose order is
// fixed -- carry their accumulators in registers across the halves.  Chain
// threads prefetch the next chunk of operands while they compute the current
// one.
//
// Two windows share each HFMA2 (one per half2 lane), so every lane computes
// exactly the per-window chain the shader does: two f16 FMA chains per gate
// (even inputs from f16(bias), odd from zero) in increasing input order,
// summed in f16; one f16 chain per head column with the +0-skip rule applied
// per lane; an f32 projection chain; the same nonlinearities and tie rules as
// tdt_decoder.cu -- the two kernels return identical tokens.
#include <cuda_fp16.h>

#include <cstdint>

#include "pk_common.cuh"
#include "pk_internal.h"

namespace pk {
namespace {

constexpr int RH = 640;
constexpr int RKIN = 1280;
constexpr int ROUT = 1032;
constexpr int RBLANK = 1024;
constexpr int RMAXSYM = 10;
constexpr int RG = 128;               // CTAs, all resident at once
constexpr int RCH = RH / RG;          // 5 LSTM channels per CTA
constexpr int RGATES = 4 * RCH;       // 20 gate outputs per CTA
constexpr int RTOK = 1024 / RG;       // 8 token columns per CTA
constexpr int RHEADCOLS = 9;          // head columns per CTA: 8 tokens, + one tail column in CTAs 0..5
constexpr int RTAIL_CTAS = 6;         // CTA 0: the blank (head column 1024); CTA c in 1..5: duration c - 1
constexpr int RHG = 3;                // head columns per chain thread
constexpr int RMAXB = 40;             // windows per launch
constexpr int RPAIRS = RMAXB / 2;     // window pairs (half2 lanes)
constexpr int RHALF = RH / 2;         // joint / projector inputs per staged half
constexpr int RLSTM_R = 4;            // gate outputs per LSTM chain thread
constexpr int RLSTM_RQ = RGATES / RLSTM_R;  // their groups: 5
constexpr int RLSTM_PP = RPAIRS / 2;  // window-pair pairs (a chain thread also owns two window pairs)
constexpr int RLSTM_PER_PAR = RLSTM_RQ * RLSTM_PP;       // chain threads per parity: 50
constexpr int RLSTM_THREADS = 2 * RLSTM_PER_PAR;         // 100
constexpr int RPW = RH / 2;           // same-parity inputs of a staged half
constexpr int RW1P = RH + 8;          // layer-1 weight row of one parity (640 inputs), padded
constexpr int RW0P = RPW + 8;         // layer-0 recurrent weight row of one parity (320 inputs), padded
constexpr int RHW_STRIDE = RH + 8;    // padded head / layer-0 row: consecutive rows' loads hit different banks
constexpr int RHEAD_THREADS = RHEADCOLS / RHG * RPAIRS;  // column group x window pair: 60
constexpr int RPROJ_THREADS = RCH * RMAXB;               // output x window: 200
constexpr int RCHUNK = 8;             // chain steps per operand load
constexpr int RTHREADS = 640;
constexpr int RROW16 = RMAXB * 2 / 16;  // 16-byte chunks per exchanged f16 row (one value per window)
constexpr float RNEG = -3.402823466e+38f;
static_assert(RG * RCH == RH && RG * RTOK == 1024, "slices tile the matrices");
static_assert(RTHREADS == RH, "one thread per joint input");
static_assert(RLSTM_THREADS <= RTHREADS && RHEAD_THREADS <= RTHREADS && RHEADCOLS % RHG == 0, "thread roles fit");
static_assert((RMAXB * 2) % 16 == 0, "exchanged f16 rows are whole 16-byte chunks");
static_assert(RH % (2 * RCHUNK) == 0 && RHALF % RCHUNK == 0, "chunks never straddle a staged half");

// Exchange area (bytes from DeviceCtx::tdt_exchange).  Hidden vectors are
// input-major with the windows fastest ([640][40]), so a CTA stages a phase's
// inputs for all windows as plain row copies.  Each LSTM layer writes its new
// hidden slice to the *N array (read by the next layer / the projector) and
// commits it to the current array one barrier later, when every CTA has
// finished reading the old values.
constexpr size_t XH0 = 0;                                 // __half [640][40]: layer-0 hidden (current)
constexpr size_t XH0N = XH0 + 1ull * RH * RMAXB * 2;      // __half [640][40]: layer-0 hidden (this update)
constexpr size_t XH1 = XH0N + 1ull * RH * RMAXB * 2;      // __half [640][40]: layer-1 hidden (current)
constexpr size_t XH1N = XH1 + 1ull * RH * RMAXB * 2;      // __half [640][40]: layer-1 hidden (this update)
constexpr size_t XH1F = XH1N + 1ull * RH * RMAXB * 2;     // float [40][640]: layer-1 hidden for the projector
constexpr size_t XPROJ = XH1F + 1ull * RH * RMAXB * 4;    // float [40][640]: predictor projection
// Argmax partials of every CTA, double-buffered by step parity: the token
// part {value, id} of all 128 CTAs ([2][40][128] x 8 bytes), the duration
// part of CTAs 1..5 ([2][40][5] x 8 bytes).
constexpr size_t XPART = XPROJ + 1ull * RMAXB * RH * 4;
constexpr size_t XDPART = XPART + 2ull * RMAXB * RG * 8;
constexpr size_t XSYNC = XDPART + 2ull * RMAXB * 8 * 8;  // barrier counter, abort flag
// __half [128 CTAs][1024 tokens][20 gates][2 parities]: the state of each of a
// CTA's layer-0 gate chains after the 640 embedding inputs of a token (even
// chain from f16(bias), odd chain from zero), written by tdt_token_table_kernel
// before the decode; a token's 80 bytes per CTA are contiguous.
constexpr size_t XTT = XSYNC + 256;
constexpr int RTOKENS = 1024;         // tokens that feed the LSTM (the blank never does)
constexpr size_t XTT_BYTES = 1ull * RG * RTOKENS * RGATES * 2 * 2;
// float [640][40]: the joint inputs max(enc + proj, 0) of the step, row k
// written by the CTA that owns projector output k (steps with an LSTM update).
constexpr size_t XJIN = XTT + XTT_BYTES;
// uint32 [20][640]: the same inputs rounded to f16, as the half2 of windows
// 2 p, 2 p + 1 (the head chains' operand layout, staged by plain copies).
constexpr size_t XJ2 = XJIN + 1ull * RH * RMAXB * 4;
static_assert(XJ2 + 1ull * RPAIRS * RH * 4 <= kTdtExchangeBytes, "exchange area fits");
static_assert(XSYNC % 16 == 0, "exchange arrays stay 16-byte aligned");

struct __align__(16) RPartial {
  float tv;
  uint32_t ti;
  float dv;
  uint32_t di;
};

// Decoder control of one window; every CTA keeps an identical copy.
struct RWin {
  int t, enc_len, len_c, start, flushreq;
  int sym, count, flags, mode, fsym, blanks, ft;
  int joint, joint_t;  // a joint at encoder frame joint_t comes next
  int pending;         // 0: none, 1: start-of-sequence update, 2: update with `token`
  int token;
};

struct RSmem {
  __half w0[2][RGATES][RW0P];        // layer 0, recurrent input 640 + 2 m + parity: [parity][gate output][m]
  __half w1[2][RGATES][RW1P];        // layer 1, input 2 m + parity: [parity][gate output][m]
  __half hw[RHEADCOLS][RHW_STRIDE];  // [head column][input]
  float pwf[RCH][RH];                // projector weights as f32, [output][input]
  union {
    __half2 x2[RH][RPAIRS];          // one half of an LSTM layer's inputs, [input][window pair]
    float hf[RMAXB][RHALF + 4];      // one half of the projector inputs, [window][input] (rows padded)
    struct {
      uint32_t j2[RPAIRS][RHALF + 4];    // one half of the joint inputs, [window pair][input] (half2 bits)
      uint32_t keep[RPAIRS][RHALF + 4];  // per pair and input: the lanes whose head chain skips it
    } jt;                                // (rows padded: the pairs of a warp read different banks)
  } in;
  // The second half of a phase's inputs, staged by the threads that run no
  // chains while the chain threads work through the first half in `in`.
  union {
    __half2 x2[RH][RPAIRS];
    float hf[RMAXB][RHALF + 4];
    uint32_t j2[RPAIRS][RHALF + 4];
    RPartial red[RMAXB][20];  // argmax reduction
  } in2;
  float gates[RMAXB][RGATES];
  float projv[RMAXB][RCH];           // this CTA's projector outputs of every window (last update)
  float c0[RMAXB][RCH];
  float c1[RMAXB][RCH];
  __half hnew[RMAXB][RCH];           // this CTA's new hidden slice, committed one barrier later
  uint32_t psum[2][RPAIRS][RGATES];  // the parity chains' sums (half2 bits), [parity][window pair][gate]
  uint32_t l0init[2][RPAIRS][RGATES];  // layer-0 chains after the token's embedding inputs (half2 bits)
  float b0[RGATES], b1[RGATES], pb[8], hb[RHEADCOLS];
  int first_exc[RMAXB];
  RPartial hred[RMAXB][RHEADCOLS / RHG];  // per window: the column groups' partials
  RWin win[RMAXB];
  int any_pending, any_token, any_joint;
  int head_finite;                   // every head weight of this CTA is finite (the head chains skip no input)
  int h0_staged;                     // in.x2 already holds the committed h0 (prefetched by the joint phase)
  unsigned int gen;
};
static_assert(sizeof(RSmem) + 128 <= 232448, "resident decoder shared memory");

struct RParams {
  const __half* enc;  // [batch, frames, 640]
  const __half* emb;  // [1025, 640]
  const __half* w0;   // [1280, 2560]
  const __half* w1;
  const __half* pw;   // [640, 640]
  const __half* hw;   // [640, 1032]
  const float* b0;
  const float* b1;
  const float* pb;
  const float* hb;
  const uint32_t* lengths;
  const uint32_t* starts;
  const uint32_t* ends;
  const uint32_t* flush;
  uint32_t* tokens;
  uint32_t* token_frames;
  uint32_t* token_durations;
  uint32_t* metadata;
  unsigned int* status;
  unsigned char* xchg;
  int batch, frames, max_tokens;
};

// Grid barrier of the cooperative launch; bounded (a wait that expires sets
// the abort flag and a status bit, after which barriers no longer wait).
__device__ void grid_sync(RSmem& s, const RParams& p) {
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned int* ctr = reinterpret_cast<unsigned int*>(p.xchg + XSYNC);
    s.gen += 1;
    grid_arrive_wait(ctr, ctr + 1, s.gen * gridDim.x, p.status, PK_STATUS_TIMEOUT_GRID, PK_WAIT_NS);
  }
  __syncthreads();
}

__device__ __forceinline__ uint32_t h2_bits(__half2 v) { return *reinterpret_cast<uint32_t*>(&v); }
// The 100 LSTM chain threads are lanes 0..24 of warps 0..3, one warp per SM
// sub-partition (not three full warps on three sub-partitions and one lane
// group on the fourth).
constexpr int RSPREAD_LANES = 25;
constexpr int RSPREAD_WARPS = RLSTM_THREADS / RSPREAD_LANES;
static_assert(RSPREAD_WARPS * RSPREAD_LANES == RLSTM_THREADS && RSPREAD_WARPS == 4, "spread roles");
__device__ __forceinline__ int spread_index(int tid, bool& on) {
  const int lane = tid & 31, wid = tid >> 5;
  on = wid < RSPREAD_WARPS && lane < RSPREAD_LANES;
  return wid * RSPREAD_LANES + lane;
}
__device__ __forceinline__ __half2 bits_h2(uint32_t v) { return *reinterpret_cast<__half2*>(&v); }
// Lane masks: keep `old` in the lanes of `m` (a skipped input leaves the
// accumulator exactly as it was), take `fresh` elsewhere -- one LOP3.
__device__ __forceinline__ __half2 keep_mask(__half2 old, __half2 fresh, uint32_t m) {
  return bits_h2((h2_bits(old) & m) | (h2_bits(fresh) & ~m));
}
__device__ __forceinline__ uint32_t lane_mask(bool lo, bool hi) {
  return (lo ? 0x0000ffffu : 0u) | (hi ? 0xffff0000u : 0u);
}
__device__ __forceinline__ void set_lane(__half2* pair, int lane, __half v) {
  reinterpret_cast<__half*>(pair)[lane] = v;
}
__device__ __forceinline__ bool better(float lv, uint32_t li, float rv, uint32_t ri) {
  return rv > lv || (rv == lv && ri < li);
}
__device__ __forceinline__ float sanitize(float v) { return v != v ? RNEG : v; }

__device__ __forceinline__ __half* xh(const RParams& p, size_t off) { return reinterpret_cast<__half*>(p.xchg + off); }
__device__ __forceinline__ float* h1f_at(const RParams& p) { return reinterpret_cast<float*>(p.xchg + XH1F); }
__device__ __forceinline__ float* jin_at(const RParams& p) { return reinterpret_cast<float*>(p.xchg + XJIN); }
__device__ __forceinline__ __half* j2_at(const RParams& p) { return reinterpret_cast<__half*>(p.xchg + XJ2); }
__device__ __forceinline__ float* proj_at(const RParams& p, int w) {
  return reinterpret_cast<float*>(p.xchg + XPROJ) + (size_t)w * RH;
}
__device__ __forceinline__ uint2* part_at(const RParams& p, int slot, int w, int cta) {
  return reinterpret_cast<uint2*>(p.xchg + XPART) + ((size_t)slot * RMAXB + w) * RG + cta;
}
__device__ __forceinline__ uint2* dpart_at(const RParams& p, int slot, int w, int d) {
  return reinterpret_cast<uint2*>(p.xchg + XDPART) + ((size_t)slot * RMAXB + w) * 8 + d;
}

// Copies the 640 exchanged f16 rows at `src` (one value per window) into x2:
// every thread issues all of its 16-byte loads before any store.
__device__ void stage_rows(RSmem& s, const __half* src) {
  constexpr int CHUNKS = RH * RROW16;
  constexpr int PER = CHUNKS / RTHREADS;
  static_assert(CHUNKS % RTHREADS == 0, "whole chunks per thread");
  uint4 v[PER];
#pragma unroll
  for (int j = 0; j < PER; ++j) v[j] = __ldcg(reinterpret_cast<const uint4*>(src) + threadIdx.x + j * RTHREADS);
#pragma unroll
  for (int j = 0; j < PER; ++j) reinterpret_cast<uint4*>(&s.in.x2[0][0])[threadIdx.x + j * RTHREADS] = v[j];
}

// Background staging by the threads of warps `first_warp` .. 19 (the others
// run chains meanwhile): `chunks` 16-byte chunks, chunk i read from
// src_chunk(i) and written to dst_chunk(i).
constexpr int RWARPS = RTHREADS / 32;
template <typename Src, typename Dst>
__device__ __forceinline__ void stage_background(int first_warp, int chunks, Src src_chunk, Dst dst_chunk) {
  const int idx = (int)threadIdx.x - first_warp * 32, n = (RWARPS - first_warp) * 32;
  if (idx < 0) return;
  for (int i = idx; i < chunks; i += 2 * n) {
    const uint4 a = __ldcg(src_chunk(i));
    uint4 b = make_uint4(0u, 0u, 0u, 0u);
    if (i + n < chunks) b = __ldcg(src_chunk(i + n));
    *dst_chunk(i) = a;
    if (i + n < chunks) *dst_chunk(i + n) = b;
  }
}

// The layer-0 chain states after the embedding inputs of each updating
// window's token (the token table), into l0init: thread (window, q) loads
// gates 4 q .. 4 q + 3 of both parities (16 bytes).
__device__ void stage_token_init(RSmem& s, const RParams& p) {
  const int tid = threadIdx.x;
  if (tid >= RMAXB * 5) return;
  const int w = tid / 5, q = tid % 5;
  uint4 v = make_uint4(0u, 0u, 0u, 0u);
  if (w < p.batch && s.win[w].pending == 2) {
    const size_t at = ((size_t)blockIdx.x * RTOKENS + s.win[w].token) * RGATES * 2 + 8 * q;
    v = __ldcg(reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(p.xchg + XTT) + at));
  }
  const __half* h = reinterpret_cast<const __half*>(&v);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    set_lane(reinterpret_cast<__half2*>(&s.l0init[0][w >> 1][4 * q + e]), w & 1, h[2 * e]);
    set_lane(reinterpret_cast<__half2*>(&s.l0init[1][w >> 1][4 * q + e]), w & 1, h[2 * e + 1]);
  }
}

// Operands of 8 same-parity chain steps from m: 8 weights of each of the
// thread's RLSTM_R gate outputs and the two window pairs' inputs of each step.
struct LstmOps {
  uint4 w[RLSTM_R];
  uint2 x[8];
};

__device__ __forceinline__ void lstm_load(const __half2 (*x2)[RPAIRS], const __half* w0, int wstride, int m, int pp,
                                          int par, LstmOps& c) {
#pragma unroll
  for (int r = 0; r < RLSTM_R; ++r) c.w[r] = *reinterpret_cast<const uint4*>(w0 + r * wstride + m);
#pragma unroll
  for (int j = 0; j < 8; ++j) c.x[j] = *reinterpret_cast<const uint2*>(&x2[2 * (m + j) + par][2 * pp]);
}

__device__ __forceinline__ void lstm_math(const LstmOps& c, __half2 (&acc)[RLSTM_R][2]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) {
#pragma unroll
    for (int r = 0; r < RLSTM_R; ++r) {
      // Broadcast of one half of a weight pair (an operand selector of the
      // f16x2 FMA, not a separate instruction).
      const uint32_t wp = (&c.w[r].x)[j >> 1];
      const __half2 wv = (j & 1) ? __high2half2(bits_h2(wp)) : __low2half2(bits_h2(wp));
      acc[r][0] = __hfma2(bits_h2(c.x[j].x), wv, acc[r][0]);
      acc[r][1] = __hfma2(bits_h2(c.x[j].y), wv, acc[r][1]);
    }
  }
}

// One staged half (640 inputs, in `x2`) of this thread's gate chains: RLSTM_R gate
// outputs whose same-parity weights of this half start at `w0` (rows
// `wstride` apart), parity `par`, window pairs 2 pp and 2 pp + 1 (2 RLSTM_R
// chains per thread, each in increasing input order).  Each 16-byte weight
// load serves 8 steps of two window pairs, each 8-byte input load 2 steps of
// RLSTM_R gate outputs.
__device__ __forceinline__ void lstm_chain_half(const __half2 (*x2)[RPAIRS], const __half* w0, int wstride, int pp,
                                                int par, __half2 (&acc)[RLSTM_R][2]) {
#pragma unroll 4
  for (int m = 0; m < RPW; m += 8) {
    LstmOps a;
    lstm_load(x2, w0, wstride, m, pp, par, a);
    lstm_math(a, acc);
  }
}

// Gate chains of one LSTM layer for the windows that need them; gates land in
// s.gates[window][gate * 5 + channel].  Chain thread t (spread_index) < 100:
// parity t / 50, gate outputs 4 q .. 4 q + 3 with q = (t % 50) / 10, window
// pairs 2 v and 2 v + 1 with v = t % 10.  Inputs: layer 0 [embedding(token) | h0] (the
// chains' states after the embedding half come from the token table), layer 1
// [new h0 | h1], staged one half at a time.  Layer 1's start-of-sequence
// windows stop at input 640 (their recurrent input is zero and the shader
// does not run those steps): their lanes take back the accumulator they had
// before the recurrent half.  Lanes of windows that do not update compute
// values nobody reads.
__device__ void lstm_layer(RSmem& s, const RParams& p, bool layer1) {
  const int tid = threadIdx.x;
  bool chain;
  const int ci = spread_index(tid, chain);
  const int par = (ci / RLSTM_PER_PAR) & 1, r = ci % RLSTM_PER_PAR;
  const int oa = RLSTM_R * (r / RLSTM_PP), pp = r % RLSTM_PP;
  const __half* w0 = layer1 ? &s.w1[par][oa][0] : &s.w0[par][oa][0];
  const int wstride = layer1 ? RW1P : RW0P;
  bool any = false, any_full = false;
  uint32_t keep_rec[2];
  __half2 acc[RLSTM_R][2];
  if (chain) {
#pragma unroll
    for (int rr = 0; rr < RLSTM_R; ++rr) {
      const __half2 init = par == 0 ? __float2half2_rn((layer1 ? s.b1 : s.b0)[oa + rr]) : __float2half2_rn(0.0f);
      acc[rr][0] = init;
      acc[rr][1] = init;
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int w0i = (2 * pp + i) * 2;
      const int p0 = s.win[w0i].pending, p1 = s.win[w0i + 1].pending;
      keep_rec[i] = lane_mask(p0 == 1, p1 == 1);
      any |= layer1 ? (p0 | p1) != 0 : (p0 == 2 || p1 == 2);
      any_full |= p0 == 2 || p1 == 2;
    }
  }
  const bool tokens = s.any_token != 0;
  if (layer1) {
    stage_rows(s, xh(p, XH0N));
    __syncthreads();
    if (chain && any) lstm_chain_half(s.in.x2, w0, wstride, pp, par, acc);
    if (tokens) {
      // The recurrent half (h1) is staged into in2 by warps 4.. while the
      // chain warps run the first half.
      const uint4* src = reinterpret_cast<const uint4*>(xh(p, XH1));
      uint4* dst = reinterpret_cast<uint4*>(&s.in2.x2[0][0]);
      stage_background(RSPREAD_WARPS, RH * RROW16, [&](int i) { return src + i; }, [&](int i) { return dst + i; });
      __syncthreads();
      if (chain && any_full) {
        __half2 before[RLSTM_R][2];
#pragma unroll
        for (int rr = 0; rr < RLSTM_R; ++rr) before[rr][0] = acc[rr][0], before[rr][1] = acc[rr][1];
        lstm_chain_half(s.in2.x2, w0 + RPW, wstride, pp, par, acc);
#pragma unroll
        for (int rr = 0; rr < RLSTM_R; ++rr)
#pragma unroll
          for (int i = 0; i < 2; ++i) acc[rr][i] = keep_mask(before[rr][i], acc[rr][i], keep_rec[i]);
      }
    }
  } else if (tokens) {
    // Layer 0: the chains over the token's embedding inputs are read from the
    // token table; the recurrent inputs (h0) continue them here.
    stage_token_init(s, p);
    if (!s.h0_staged) stage_rows(s, xh(p, XH0));
    __syncthreads();
    if (chain && any) {
#pragma unroll
      for (int rr = 0; rr < RLSTM_R; ++rr)
#pragma unroll
        for (int i = 0; i < 2; ++i) acc[rr][i] = bits_h2(s.l0init[par][2 * pp + i][oa + rr]);
      lstm_chain_half(s.in.x2, w0, wstride, pp, par, acc);
    }
  }
  // The two parity chains of a gate sum in f16.
  if (chain && any) {
#pragma unroll
    for (int rr = 0; rr < RLSTM_R; ++rr)
#pragma unroll
      for (int i = 0; i < 2; ++i) s.psum[par][2 * pp + i][oa + rr] = h2_bits(acc[rr][i]);
  }
  __syncthreads();
  for (int i = tid; i < RPAIRS * RGATES; i += RTHREADS) {
    const int pr = i / RGATES, g = i % RGATES;
    const bool upd = (s.win[2 * pr].pending | s.win[2 * pr + 1].pending) != 0;
    if (upd) {
      const float2 v = __half22float2(__hadd2(bits_h2(s.psum[0][pr][g]), bits_h2(s.psum[1][pr][g])));
      // Layer 0's start-of-sequence windows take the bias as their gates.
      const float bias = layer1 ? 0.0f : __half2float(__float2half_rn(s.b0[g]));
      s.gates[2 * pr][g] = !layer1 && s.win[2 * pr].pending == 1 ? bias : v.x;
      s.gates[2 * pr + 1][g] = !layer1 && s.win[2 * pr + 1].pending == 1 ? bias : v.y;
    }
  }
}

// Cell update of this CTA's 5 channels for the updating windows: the new
// hidden slice goes to the layer's *N array now and to s.hnew for the commit.
__device__ void cell_update(RSmem& s, const RParams& p, float (*cst)[RCH], bool layer1) {
  for (int i = threadIdx.x; i < p.batch * RCH; i += RTHREADS) {
    const int w = i / RCH, c = i % RCH;
    if (!s.win[w].pending) continue;
    const float gi = tdt_sigmoid(s.gates[w][c]);
    const float gf = tdt_sigmoid(s.gates[w][RCH + c]);
    const float gg = tdt_tanh(s.gates[w][2 * RCH + c]);
    const float go = tdt_sigmoid(s.gates[w][3 * RCH + c]);
    const float cell = __fmaf_rn(gf, cst[w][c], __fmul_rn(gi, gg));
    cst[w][c] = cell;
    const float h = __fmul_rn(go, tdt_tanh(cell));
    const size_t at = (size_t)(blockIdx.x * RCH + c) * RMAXB + w;
    const __half hh = __float2half_rn(h);
    s.hnew[w][c] = hh;
    xh(p, layer1 ? XH1N : XH0N)[at] = hh;
    if (layer1) h1f_at(p)[(size_t)w * RH + blockIdx.x * RCH + c] = h;
  }
}

// Commits this CTA's slice of a layer's new hidden state (called once every
// CTA has finished reading the old one).
__device__ void commit_hidden(RSmem& s, const RParams& p, bool layer1) {
  for (int i = threadIdx.x; i < p.batch * RCH; i += RTHREADS) {
    const int w = i / RCH, c = i % RCH;
    if (s.win[w].pending) xh(p, layer1 ? XH1 : XH0)[(size_t)(blockIdx.x * RCH + c) * RMAXB + w] = s.hnew[w][c];
  }
}

// The f32 projection chains of this CTA's 5 projector outputs, in two staged
// halves of the new layer-1 hidden state (exchanged as [window][input], so
// the staging is a plain copy and a thread's inputs and weights are 16-byte
// loads along k);
// thread: (output, window).  The same threads then build this CTA's rows of
// the step's joint inputs.
__device__ void projector(RSmem& s, const RParams& p) {
  const int tid = threadIdx.x;
  const int o = tid / RMAXB, w = tid % RMAXB;
  const bool live = tid < RPROJ_THREADS && w < p.batch && s.win[w].pending;
  const bool joint = tid < RPROJ_THREADS && w < p.batch && s.win[w].joint;
  // The encoder value of this thread's joint input (read now, used at the end).
  const __half ev = joint ? p.enc[((size_t)w * p.frames + s.win[w].joint_t) * RH + blockIdx.x * RCH + o]
                          : __float2half_rn(0.0f);
  float acc = live ? s.pb[o] : 0.0f;
  // Row w of the exchanged state holds window w's 640 values: a half is 80
  // chunks of 16 bytes per window, copied as they lie.  All threads stage the
  // first half; the second is staged into in2 by warps 7.. (no chain thread
  // among them) while the chains run through the first.
  constexpr int Q = RHALF / 4;
  constexpr int PER = RMAXB * Q / RTHREADS;
  static_assert(RMAXB * Q % RTHREADS == 0 && RPROJ_THREADS <= 7 * 32, "whole chunks per thread; chain warps 0..6");
  {
    uint4 v[PER];
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int i = tid + j * RTHREADS, r = i / Q, c4 = 4 * (i % Q);
      v[j] = __ldcg(reinterpret_cast<const uint4*>(h1f_at(p) + (size_t)r * RH + c4));
    }
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int i = tid + j * RTHREADS, r = i / Q, c4 = 4 * (i % Q);
      *reinterpret_cast<uint4*>(&s.in.hf[r][c4]) = v[j];
    }
  }
  __syncthreads();
  auto chain_half = [&](const float (*hf)[RHALF + 4], int h) {
    const float* hrow = &hf[w][0];
    const float* wrow = &s.pwf[o][h * RHALF];
    float4 ha = *reinterpret_cast<const float4*>(hrow), wa = *reinterpret_cast<const float4*>(wrow);
#pragma unroll 1
    for (int k = 0; k < RHALF; k += 8) {
      const float4 hb = *reinterpret_cast<const float4*>(hrow + k + 4);
      const float4 wb = *reinterpret_cast<const float4*>(wrow + k + 4);
      acc = __fmaf_rn(ha.x, wa.x, acc);
      acc = __fmaf_rn(ha.y, wa.y, acc);
      acc = __fmaf_rn(ha.z, wa.z, acc);
      acc = __fmaf_rn(ha.w, wa.w, acc);
      if (k + 8 < RHALF) {
        ha = *reinterpret_cast<const float4*>(hrow + k + 8);
        wa = *reinterpret_cast<const float4*>(wrow + k + 8);
      }
      acc = __fmaf_rn(hb.x, wb.x, acc);
      acc = __fmaf_rn(hb.y, wb.y, acc);
      acc = __fmaf_rn(hb.z, wb.z, acc);
      acc = __fmaf_rn(hb.w, wb.w, acc);
    }
  };
  if (live) chain_half(s.in.hf, 0);
  stage_background(
      7, RMAXB * Q,
      [&](int i) { return reinterpret_cast<const uint4*>(h1f_at(p) + (size_t)(i / Q) * RH + RHALF + 4 * (i % Q)); },
      [&](int i) { return reinterpret_cast<uint4*>(&s.in2.hf[i / Q][4 * (i % Q)]); });
  __syncthreads();
  if (live) chain_half(s.in2.hf, 1);
  if (live) {
    proj_at(p, w)[blockIdx.x * RCH + o] = acc;
    s.projv[w][o] = acc;
  }
  // Joint input k = 5 cta + o of every window that takes a joint next (the
  // windows that did not update keep their last projector output).
  if (joint) {
    const float x = __fadd_rn(__half2float(ev), s.projv[w][o]);
    const float jv = x < 0.0f ? 0.0f : x;  // as in joint_partials
    jin_at(p)[(size_t)(blockIdx.x * RCH + o) * RMAXB + w] = jv;
    j2_at(p)[((size_t)(w >> 1) * RH + blockIdx.x * RCH + o) * 2 + (w & 1)] = __float2half_rn(jv);
  }
}

__device__ void lstm_update(RSmem& s, const RParams& p) {
  const int tid = threadIdx.x;
  // Layer 0: inputs [embedding(token) | h0]; start-of-sequence windows take the bias.
  lstm_layer(s, p, false);
  __syncthreads();
  cell_update(s, p, s.c0, false);
  grid_sync(s, p);
  // Every CTA has read the old h0: commit the new slice.  Layer 1: inputs
  // [new h0 | h1] (the h1 lanes of start-of-sequence windows are not used).
  commit_hidden(s, p, false);
  lstm_layer(s, p, true);
  __syncthreads();
  cell_update(s, p, s.c1, true);
  grid_sync(s, p);
  // Projector over the new f32 h1; h1 itself is committed now (every CTA has
  // read the old one).
  commit_hidden(s, p, true);
  projector(s, p);
  grid_sync(s, p);
  if (tid < p.batch) s.win[tid].pending = 0;
  __syncthreads();
}

// Operands of 8 head-chain steps from input k0: 8 weights of each of the
// thread's columns, the pair's 8 inputs and (MASKED) their skip masks.
template <bool MASKED>
struct HeadOps {
  uint4 w[RHG];
  uint4 xa, xb;
  uint4 ma, mb;
};

template <bool MASKED>
__device__ __forceinline__ void head_load(const __half* wrow, const uint32_t* xrow, const uint32_t* mrow, int k0,
                                          HeadOps<MASKED>& c) {
#pragma unroll
  for (int j = 0; j < RHG; ++j) c.w[j] = *reinterpret_cast<const uint4*>(wrow + j * RHW_STRIDE + k0);
  c.xa = *reinterpret_cast<const uint4*>(xrow + k0);
  c.xb = *reinterpret_cast<const uint4*>(xrow + k0 + 4);
  if constexpr (MASKED) {
    c.ma = *reinterpret_cast<const uint4*>(mrow + k0);
    c.mb = *reinterpret_cast<const uint4*>(mrow + k0 + 4);
  }
}

template <bool MASKED>
__device__ __forceinline__ void head_math(const HeadOps<MASKED>& c, __half2 (&acc)[RHG]) {
  const uint32_t xs[RCHUNK] = {c.xa.x, c.xa.y, c.xa.z, c.xa.w, c.xb.x, c.xb.y, c.xb.z, c.xb.w};
  uint32_t ms[RCHUNK] = {};
  bool masked = false;
  if constexpr (MASKED) {
    const uint32_t m8[RCHUNK] = {c.ma.x, c.ma.y, c.ma.z, c.ma.w, c.mb.x, c.mb.y, c.mb.z, c.mb.w};
#pragma unroll
    for (int j = 0; j < RCHUNK; ++j) ms[j] = m8[j];
    masked = (c.ma.x | c.ma.y | c.ma.z | c.ma.w | c.mb.x | c.mb.y | c.mb.z | c.mb.w) != 0u;
  }
#pragma unroll
  for (int j = 0; j < RCHUNK; ++j) {
#pragma unroll
    for (int q = 0; q < RHG; ++q) {
      const uint32_t wp = (&c.w[q].x)[j >> 1];
      const __half2 wv = (j & 1) ? __high2half2(bits_h2(wp)) : __low2half2(bits_h2(wp));
      const __half2 v = __hfma2(bits_h2(xs[j]), wv, acc[q]);
      acc[q] = MASKED && masked ? keep_mask(acc[q], v, ms[j]) : v;
    }
  }
}

// One staged half (320 inputs) of this thread's head chains: columns
// 3 g .. 3 g + 2, window pair `pair`, starting at input `kb`.  Per 8 inputs
// the three columns share the pair's input (and mask) loads; unmasked, the
// next 8 inputs' operands are loaded while the current 8 steps run.  MASKED: lanes
// set in the staged masks skip the input (the shader's +0 rule); unmasked,
// every input is applied -- used when the CTA's head weights are all finite,
// where applying a skipped input (+0 x w) changes an accumulator at most in
// the sign of a zero, which no argmax comparison sees.
template <bool MASKED>
__device__ __forceinline__ void head_chain_half(const RSmem& s, const uint32_t (*j2)[RHALF + 4], int g, int pair, int kb,
                                                __half2 (&acc)[RHG]) {
  const __half* wrow = &s.hw[RHG * g][kb];
  const uint32_t* xrow = &j2[pair][0];
  const uint32_t* mrow = &s.in.jt.keep[pair][0];
  if constexpr (MASKED) {
    // The masked form (head weights that are not all finite) loads as it goes.
#pragma unroll 1
    for (int k0 = 0; k0 < RHALF; k0 += RCHUNK) {
      HeadOps<MASKED> a;
      head_load<MASKED>(wrow, xrow, mrow, k0, a);
      head_math<MASKED>(a, acc);
    }
  } else {
    HeadOps<MASKED> a, b;
    head_load<MASKED>(wrow, xrow, mrow, 0, a);
#pragma unroll 1
    for (int k0 = 0; k0 < RHALF; k0 += 2 * RCHUNK) {
      head_load<MASKED>(wrow, xrow, mrow, k0 + RCHUNK, b);
      head_math<MASKED>(a, acc);
      if (k0 + 2 * RCHUNK < RHALF) head_load<MASKED>(wrow, xrow, mrow, k0 + 2 * RCHUNK, a);
      head_math<MASKED>(b, acc);
    }
  }
}

// The general path of the joint inputs (a step without an LSTM update, or a
// CTA whose head weights are not all finite): thread k builds input k of
// every window, applies the shader's skip rule when `fast` is false, and
// stages the inputs (and skip masks) for the head chains in two halves.
__device__ void joint_inputs_staged(RSmem& s, const RParams& p, bool built, bool fast, int g, int pair, bool run,
                                    __half2 (&acc)[RHG]) {
  const int tid = threadIdx.x;
  if (tid < RMAXB) s.first_exc[tid] = RH;
  __syncthreads();
  const int k = tid;
  uint32_t packed[RPAIRS];  // half2 bits of input k, per window pair
  uint64_t zero_bits = 0ull;
  constexpr int WG = 20;  // windows whose loads are in flight together
#pragma unroll
  for (int w0 = 0; w0 < RMAXB; w0 += WG) {
    float jvs[WG];
    if (built) {
      // Row k of the inputs the projector phase built (windows w0 .. w0 + 19).
      const uint4* src = reinterpret_cast<const uint4*>(jin_at(p) + (size_t)k * RMAXB + w0);
#pragma unroll
      for (int q = 0; q < WG / 4; ++q) {
        const uint4 v = __ldcg(src + q);
        jvs[4 * q] = __uint_as_float(v.x);
        jvs[4 * q + 1] = __uint_as_float(v.y);
        jvs[4 * q + 2] = __uint_as_float(v.z);
        jvs[4 * q + 3] = __uint_as_float(v.w);
      }
    } else {
      __half ev[WG];
      float pv[WG];
#pragma unroll
      for (int i = 0; i < WG; ++i) {
        const int w = w0 + i;
        ev[i] = __float2half_rn(0.0f);
        pv[i] = 0.0f;
        if (w < p.batch && s.win[w].joint) {
          ev[i] = p.enc[((size_t)w * p.frames + s.win[w].joint_t) * RH + k];
          pv[i] = __ldcg(proj_at(p, w) + k);
        }
      }
#pragma unroll
      for (int i = 0; i < WG; ++i) {
        const float x = __fadd_rn(__half2float(ev[i]), pv[i]);
        jvs[i] = x < 0.0f ? 0.0f : x;  // max(x, 0) keeping -0 and NaN, as the oracle's std::max
      }
    }
#pragma unroll
    for (int i = 0; i < WG; i += 2) {
      __half hv[2];
#pragma unroll
      for (int l = 0; l < 2; ++l) {
        const int w = w0 + i + l;
        hv[l] = __float2half_rn(0.0f);
        if (w < p.batch && s.win[w].joint) {
          const float jv = jvs[i + l];
          const uint32_t bits = __float_as_uint(jv);
          hv[l] = __float2half_rn(jv);
          if (bits == 0u) zero_bits |= 1ull << w;
          if (bits == 0x80000000u || (bits & 0x7fffffffu) > 0x7f800000u) atomicMin(&s.first_exc[w], k);
        }
      }
      packed[(w0 + i) / 2] = h2_bits(__halves2half2(hv[0], hv[1]));
    }
  }
  __syncthreads();  // first_exc is final
  for (int h = 0; h < 2; ++h) {
    if (h) __syncthreads();  // the first half is consumed
    if (k / RHALF == h) {
      // The shader skips input k while no -0 / NaN input has been seen and k is +0.
#pragma unroll
      for (int pr = 0; pr < RPAIRS; ++pr) {
        const bool lo = ((zero_bits >> (2 * pr)) & 1ull) && k < s.first_exc[2 * pr];
        const bool hi = ((zero_bits >> (2 * pr + 1)) & 1ull) && k < s.first_exc[2 * pr + 1];
        s.in.jt.j2[pr][k - h * RHALF] = packed[pr];
        s.in.jt.keep[pr][k - h * RHALF] = lane_mask(lo, hi);
      }
    }
    __syncthreads();
    if (run) {
      if (fast)
        head_chain_half<false>(s, s.in.jt.j2, g, pair, h * RHALF, acc);
      else
        head_chain_half<true>(s, s.in.jt.j2, g, pair, h * RHALF, acc);
    }
  }
}

// Each thread's best token and duration of its two windows over its three
// columns, then per window over the column groups: this CTA's partials.
__device__ void joint_reduce(RSmem& s, const RParams& p, int slot, int g, int pair, bool head,
                             const __half2 (&acc)[RHG]) {
  const int tid = threadIdx.x;
  // This thread's best token and duration of each of its two windows; column
  // 8 is the tail column of CTAs 0..5 (the blank, or duration cta - 1).
  if (head) {
    const int ncols = blockIdx.x < RTAIL_CTAS ? RHEADCOLS : RTOK;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      RPartial b{RNEG, 0xffffffffu, RNEG, 0xffffffffu};
#pragma unroll
      for (int c = 0; c < RHG; ++c) {
        const int col = RHG * g + c;
        if (col >= ncols) continue;
        const float v = sanitize(i ? __high2float(acc[c]) : __low2float(acc[c]));
        if (col < RTOK) {
          if (better(b.tv, b.ti, v, blockIdx.x * RTOK + col)) b.tv = v, b.ti = blockIdx.x * RTOK + col;
        } else if (blockIdx.x == 0) {
          if (better(b.tv, b.ti, v, RBLANK)) b.tv = v, b.ti = RBLANK;
        } else {
          b.dv = v;
          b.di = blockIdx.x - 1;
        }
      }
      s.hred[2 * pair + i][g] = b;
    }
  }
  __syncthreads();
  if (tid < p.batch && s.win[tid].joint) {
    RPartial b = s.hred[tid][0];
#pragma unroll
    for (int q = 1; q < RHEADCOLS / RHG; ++q) {
      const RPartial v = s.hred[tid][q];
      if (better(b.tv, b.ti, v.tv, v.ti)) b.tv = v.tv, b.ti = v.ti;
      if (better(b.dv, b.di, v.dv, v.di)) b.dv = v.dv, b.di = v.di;
    }
    *part_at(p, slot, tid, blockIdx.x) = make_uint2(__float_as_uint(b.tv), b.ti);
    if (blockIdx.x >= 1 && blockIdx.x < RTAIL_CTAS)
      *dpart_at(p, slot, tid, blockIdx.x - 1) = make_uint2(__float_as_uint(b.dv), b.di);
  }
}

// Joint of the active windows: inputs, head columns, this CTA's partials.
// In a step that updated the LSTM (`built`) the projector phase has left the
// inputs in the exchange area: a CTA whose head weights are all finite copies
// their f16 form straight into the chains' layout; otherwise the general path
// below builds them (and the shader's skip masks) input by input.
__device__ void joint_partials(RSmem& s, const RParams& p, int slot, bool built) {
  const int tid = threadIdx.x;
  if (tid == 0) s.h0_staged = 0;  // the joint inputs reuse in
  const bool fast = s.head_finite != 0;  // no skip rule to apply (head_chain_half)
  const int g = tid % (RHEADCOLS / RHG), pair = tid / (RHEADCOLS / RHG);  // windows 2 pair, 2 pair + 1
  const bool head = tid < RHEAD_THREADS;
  __half2 acc[RHG];
#pragma unroll
  for (int c = 0; c < RHG; ++c) acc[c] = __float2half2_rn(head ? s.hb[RHG * g + c] : 0.0f);
  const bool run = head && (s.win[2 * pair].joint || s.win[2 * pair + 1].joint);
  if (built && fast) {
    // The projector phase left the f16 inputs in the chains' layout: each
    // half is a plain copy of 20 rows of 320 words.  The second half goes to
    // in2 (warps 2..) while the head chains (warps 0..1) run the first.
    constexpr int CH = RPAIRS * RHALF / 4;  // 16-byte chunks per half
    constexpr int QH = RHALF / 4;
    static_assert(RHEAD_THREADS <= 64, "head chain warps 0..1");
    auto src = [&](int i, int h) {
      return reinterpret_cast<const uint4*>(j2_at(p) + ((size_t)(i / QH) * RH + h * RHALF + 4 * (i % QH)) * 2);
    };
    for (int i = tid; i < CH; i += RTHREADS)
      *reinterpret_cast<uint4*>(&s.in.jt.j2[i / QH][4 * (i % QH)]) = __ldcg(src(i, 0));
    __syncthreads();
    if (run) head_chain_half<false>(s, s.in.jt.j2, g, pair, 0, acc);
    stage_background(
        2, CH, [&](int i) { return src(i, 1); },
        [&](int i) { return reinterpret_cast<uint4*>(&s.in2.j2[i / QH][4 * (i % QH)]); });
    __syncthreads();
    if (run) head_chain_half<false>(s, s.in2.j2, g, pair, RHALF, acc);
    // Meanwhile warps 2.. stage the committed h0 -- the recurrent inputs of
    // the next step's layer 0, unchanged until that step commits -- into
    // in.x2, which the head chains no longer read.
    {
      const uint4* h0 = reinterpret_cast<const uint4*>(xh(p, XH0));
      uint4* dst = reinterpret_cast<uint4*>(&s.in.x2[0][0]);
      stage_background(2, RH * RROW16, [&](int i) { return h0 + i; }, [&](int i) { return dst + i; });
    }
    if (tid == 0) s.h0_staged = 1;
  } else {
    joint_inputs_staged(s, p, built, fast, g, pair, run, acc);
  }
  joint_reduce(s, p, slot, g, pair, head, acc);
}

__device__ void emit(RSmem& s, const RParams& p, int w, uint32_t tok, uint32_t frame, uint32_t dur) {
  RWin& c = s.win[w];
  if (c.count < p.max_tokens) {
    if (blockIdx.x == 0) {
      const size_t o = (size_t)w * p.max_tokens + c.count;
      p.tokens[o] = tok;
      p.token_frames[o] = frame;
      p.token_durations[o] = dur;
    }
    ++c.count;
  } else {
    c.flags |= 1;
  }
}

// Reduce every CTA's partials (each CTA does it, so all agree) and advance the
// control of every active window (the shader's main loop and flush, :1702-1990).
__device__ void joint_decide(RSmem& s, const RParams& p, int slot) {
  const int tid = threadIdx.x;
  // Thread (window, q): the token partials of CTAs 8 q .. 8 q + 7 (four
  // 16-byte loads).
  constexpr int QN = RG / 8;
  static_assert(RMAXB * QN == RTHREADS && QN <= 20, "one thread per (window, group of 8 CTAs)");
  {
    const int w = tid / QN, q = tid % QN;
    RPartial b{RNEG, 0xffffffffu, RNEG, 0xffffffffu};
    if (w < p.batch && s.win[w].joint) {
      uint4 raw[4];
      const uint4* src = reinterpret_cast<const uint4*>(part_at(p, slot, w, 8 * q));
#pragma unroll
      for (int j = 0; j < 4; ++j) raw[j] = __ldcg(src + j);
      // Thread q < 5 also takes duration q's partial (from CTA q + 1).
      const uint2 dr = q < RTAIL_CTAS - 1 ? __ldcg(dpart_at(p, slot, w, q)) : make_uint2(__float_as_uint(RNEG), ~0u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float v0 = __uint_as_float(raw[j].x), v1 = __uint_as_float(raw[j].z);
        if (better(b.tv, b.ti, v0, raw[j].y)) b.tv = v0, b.ti = raw[j].y;
        if (better(b.tv, b.ti, v1, raw[j].w)) b.tv = v1, b.ti = raw[j].w;
      }
      b.dv = __uint_as_float(dr.x);
      b.di = dr.y;
    }
    s.in2.red[w][q] = b;
  }
  __syncthreads();
  if (tid < p.batch && s.win[tid].joint) {
    const int w = tid;
    RPartial b = s.in2.red[w][0];
    for (int q = 1; q < RG / 8; ++q) {
      const RPartial v = s.in2.red[w][q];
      if (better(b.tv, b.ti, v.tv, v.ti)) b.tv = v.tv, b.ti = v.ti;
      if (better(b.dv, b.di, v.dv, v.di)) b.dv = v.dv, b.di = v.di;
    }
    RWin& c = s.win[w];
    // Ids are in range unless a bounded wait expired (results then garbage and flagged).
    const uint32_t tok = b.ti, dur = min(b.di, 4u);
    const bool nonblank = tok < (uint32_t)RBLANK;
    int next = 0;
    if (c.mode == 0) {
      if (nonblank) emit(s, p, w, tok, (uint32_t)c.t, dur);
      c.sym += 1;
      if (dur != 0) {
        c.t += (int)dur;
        c.sym = 0;
      } else if (!nonblank || c.sym >= RMAXSYM) {
        c.t += 1;
        c.sym = 0;
      }
      if (c.t < c.enc_len) {
        next = 1;
      } else if (c.flushreq && c.start < c.enc_len) {
        c.mode = 1;
        c.fsym = 0;
        c.blanks = 0;
        c.ft = c.t;
        next = 1;
      }
    } else {
      if (!nonblank) {
        c.blanks += 1;
      } else {
        c.blanks = 0;
        emit(s, p, w, tok, (uint32_t)min(c.ft, c.enc_len - 1), dur);
      }
      c.ft = min(c.ft + max(1, (int)dur), c.enc_len);
      c.fsym += 1;
      next = (c.fsym < RMAXSYM && c.blanks < 5) ? 1 : 0;
    }
    if (next) {
      if (c.mode == 0) {
        c.joint_t = c.t;
      } else {
        const int v = c.fsym % 3;
        if (v == 0) c.t = min(c.ft, c.len_c - 1);
        else if (v == 1) c.t = min(c.enc_len - 1, p.frames - 1);
        else c.t = min(max(c.enc_len, 2) - 2, p.frames - 1);
        c.joint_t = c.t;
      }
    }
    c.joint = next;
    c.pending = (nonblank && next) ? 2 : 0;  // the shader's update after the last joint feeds nothing
    c.token = (int)tok;
  }
  __syncthreads();
}

// The token table: for every token that feeds the LSTM and every layer-0 gate
// column, the two parity chains' states after the 640 embedding inputs --
// exactly the first half of the chains the shader runs for that token (even
// chain from f16(bias), odd chain from zero, inputs in increasing order).
// Block (CTA slice c of the resident kernel, 64 tokens); thread (gate o,
// parity, 4 token pairs, one per half2 lane pair).
constexpr int TT_TOKENS = 64;
constexpr int TT_THREADS = RGATES * 2 * 8;
struct TtSmem {
  __half w[RGATES][RHW_STRIDE];   // the slice's embedding-input weights, [gate][input]
  __half2 x[RH][TT_TOKENS / 2];   // embedding rows, [input][token pair]
};
static_assert(RTOKENS % TT_TOKENS == 0 && TT_TOKENS / 2 == 4 * 8, "token blocks tile the table");

__global__ void __launch_bounds__(TT_THREADS) tdt_token_table_kernel(const __half* __restrict__ emb,
                                                                     const __half* __restrict__ w0,
                                                                     const float* __restrict__ b0,
                                                                     unsigned char* xchg) {
  extern __shared__ __align__(16) unsigned char tt_raw[];
  TtSmem& s = *reinterpret_cast<TtSmem*>(tt_raw);
  const int c = blockIdx.x, t0 = blockIdx.y * TT_TOKENS, tid = threadIdx.x;
  pdl_entry();
  for (int i = tid; i < RH * RGATES; i += TT_THREADS) {
    const int k = i / RGATES, o = i % RGATES;
    s.w[o][k] = w0[(size_t)k * 4 * RH + (o / RCH) * RH + c * RCH + o % RCH];
  }
  for (int i = tid; i < TT_TOKENS * (RH / 8); i += TT_THREADS) {
    const int tok = i / (RH / 8), k8 = 8 * (i % (RH / 8));
    const uint4 v = *reinterpret_cast<const uint4*>(emb + (size_t)(t0 + tok) * RH + k8);
    const __half* h = reinterpret_cast<const __half*>(&v);
#pragma unroll
    for (int e = 0; e < 8; ++e) set_lane(&s.x[k8 + e][tok >> 1], tok & 1, h[e]);
  }
  __syncthreads();
  const int o = tid % RGATES, par = (tid / RGATES) & 1, tg = tid / (2 * RGATES);
  const __half2 init = par == 0 ? __float2half2_rn(b0[(o / RCH) * RH + c * RCH + o % RCH]) : __float2half2_rn(0.0f);
  __half2 acc[4] = {init, init, init, init};
#pragma unroll 4
  for (int k = par; k < RH; k += 2) {
    const __half2 wv = __half2half2(s.w[o][k]);
    const uint4 xv = *reinterpret_cast<const uint4*>(&s.x[k][4 * tg]);
    acc[0] = __hfma2(bits_h2(xv.x), wv, acc[0]);
    acc[1] = __hfma2(bits_h2(xv.y), wv, acc[1]);
    acc[2] = __hfma2(bits_h2(xv.z), wv, acc[2]);
    acc[3] = __hfma2(bits_h2(xv.w), wv, acc[3]);
  }
  __half* out = reinterpret_cast<__half*>(xchg + XTT) + (size_t)c * RTOKENS * RGATES * 2;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int tok = t0 + 2 * (4 * tg + i);
    out[((size_t)tok * RGATES + o) * 2 + par] = __low2half(acc[i]);
    out[((size_t)(tok + 1) * RGATES + o) * 2 + par] = __high2half(acc[i]);
  }
}

__global__ void __launch_bounds__(RTHREADS, 1) tdt_resident_kernel(const RParams p) {
  extern __shared__ __align__(128) unsigned char rsmem_raw[];
  RSmem& s = *reinterpret_cast<RSmem*>((reinterpret_cast<uintptr_t>(rsmem_raw) + 127) & ~static_cast<uintptr_t>(127));
  const int tid = threadIdx.x, cta = blockIdx.x;
  // This CTA's weight slices (one-time; columns gate * 640 + 5 cta + channel).
  for (int i = tid; i < RKIN * RGATES; i += RTHREADS) {
    const int k = i / RGATES, o = i % RGATES;
    const size_t col = (size_t)(o / RCH) * RH + cta * RCH + o % RCH;
    if (k >= RH) s.w0[k & 1][o][(k - RH) >> 1] = p.w0[(size_t)k * 4 * RH + col];
    s.w1[k & 1][o][k >> 1] = p.w1[(size_t)k * 4 * RH + col];
  }
  for (int i = tid; i < RH * RCH; i += RTHREADS) {
    const int k = i / RCH, o = i % RCH;
    s.pwf[o][k] = __half2float(p.pw[(size_t)k * RH + cta * RCH + o]);
  }
  bool finite = true;
  for (int i = tid; i < RH * RHEADCOLS; i += RTHREADS) {
    const int k = i / RHEADCOLS, c = i % RHEADCOLS;
    const int col = c < RTOK ? cta * RTOK + c : (cta < RTAIL_CTAS ? RBLANK + cta : -1);
    const __half v = col >= 0 ? p.hw[(size_t)k * ROUT + col] : __float2half_rn(0.0f);
    s.hw[c][k] = v;
    finite = finite && !__hisinf(v) && !__hisnan(v);
  }
  finite = __syncthreads_and(finite) != 0;
  if (tid == 0) s.head_finite = finite;
  if (tid < RGATES) {
    const size_t col = (size_t)(tid / RCH) * RH + cta * RCH + tid % RCH;
    s.b0[tid] = p.b0[col];
    s.b1[tid] = p.b1[col];
  }
  if (tid < 8) s.pb[tid] = tid < RCH ? p.pb[cta * RCH + tid] : 0.0f;
  if (tid < RHEADCOLS) {
    const int col = tid < RTOK ? cta * RTOK + tid : (cta < RTAIL_CTAS ? RBLANK + cta : -1);
    s.hb[tid] = col >= 0 ? p.hb[col] : 0.0f;
  }
  for (int i = tid; i < RMAXB * RCH; i += RTHREADS) {
    (&s.c0[0][0])[i] = 0.0f;
    (&s.c1[0][0])[i] = 0.0f;
  }
  if (tid < RMAXB) {
    RWin c{};
    if (tid < p.batch) {
      c.len_c = (int)min(p.lengths[tid], (uint32_t)p.frames);
      c.enc_len = (int)min((uint32_t)c.len_c, p.ends[tid]);
      c.start = (int)min(p.starts[tid], (uint32_t)INT32_MAX);
      c.t = min(c.start, c.enc_len);
      c.flushreq = p.flush[tid] != 0;
      if (c.t < c.enc_len) {
        c.pending = 1;
        c.joint = 1;
        c.joint_t = c.t;
      }
    }
    s.win[tid] = c;
  }
  if (tid == 0) {
    s.gen = 0;
    s.h0_staged = 0;
  }
  __syncthreads();
  int slot = 0;
  while (true) {
    if (tid == 0) {
      int ap = 0, at = 0, aj = 0;
      for (int w = 0; w < p.batch; ++w) {
        ap |= s.win[w].pending != 0;
        at |= s.win[w].pending == 2;
        aj |= s.win[w].joint != 0;
      }
      s.any_pending = ap;
      s.any_token = at;
      s.any_joint = aj;
    }
    __syncthreads();
    const bool ap = s.any_pending != 0, aj = s.any_joint != 0;
    if (!ap && !aj) break;
    if (ap) lstm_update(s, p);
    if (aj) {
      joint_partials(s, p, slot, ap);
      grid_sync(s, p);
      joint_decide(s, p, slot);
      slot ^= 1;
    }
  }
  if (cta == 0 && tid < p.batch) {
    p.metadata[tid] = (uint32_t)s.win[tid].count;
    p.metadata[p.batch + tid] = (uint32_t)s.win[tid].flags;
  }
}

}  // namespace

int launch_tdt_resident(const DeviceCtx& dev, const pk_tdt_desc& d, cudaStream_t stream) {
  if (d.precision != PK_FP16 || d.batch > RMAXB || !dev.tdt_exchange || dev.sm_count < RG)
    return set_error(PK_E_SHAPE, "the resident decoder takes FP16 batches of at most %d windows on >= %d SMs", RMAXB,
                     RG);
  const int smem = (int)sizeof(RSmem) + 128;
  int st = set_max_dynamic_smem(reinterpret_cast<const void*>(tdt_resident_kernel), smem);
  if (st != PK_OK) return st;
  int per_sm = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, tdt_resident_kernel, RTHREADS, smem);
  if (e != cudaSuccess) return cuda_error(e, "occupancy query (resident decoder)");
  if (per_sm < 1) return set_error(PK_E_SHAPE, "the resident decoder does not fit one CTA per SM");
  RParams p;
  p.enc = static_cast<const __half*>(d.encoder_projected);
  p.emb = static_cast<const __half*>(d.embedding);
  p.w0 = static_cast<const __half*>(d.lstm_weight0);
  p.w1 = static_cast<const __half*>(d.lstm_weight1);
  p.pw = static_cast<const __half*>(d.projector_weight);
  p.hw = static_cast<const __half*>(d.head_weight);
  p.b0 = d.lstm_bias0;
  p.b1 = d.lstm_bias1;
  p.pb = d.projector_bias;
  p.hb = d.head_bias;
  p.lengths = d.encoded_lengths;
  p.starts = d.decode_starts;
  p.ends = d.decode_ends;
  p.flush = d.flush_finals;
  p.tokens = d.tokens;
  p.token_frames = d.token_frames;
  p.token_durations = d.token_durations;
  p.metadata = d.metadata;
  p.status = dev.status;
  p.xchg = static_cast<unsigned char*>(dev.tdt_exchange);
  p.batch = d.batch;
  p.frames = d.frames;
  p.max_tokens = d.max_tokens;
  // The token table for these weights (read by every decode step's layer 0).
  st = set_max_dynamic_smem(reinterpret_cast<const void*>(tdt_token_table_kernel), (int)sizeof(TtSmem));
  if (st != PK_OK) return st;
  if ((e = launch_kernel(tdt_token_table_kernel, dim3(RG, RTOKENS / TT_TOKENS), dim3(TT_THREADS), sizeof(TtSmem),
                         stream, p.emb, p.w0, p.b0, p.xchg)) != cudaSuccess)
    return cuda_error(e, "tdt_token_table launch");
  // The barrier counter and abort flag start at zero every launch.
  if ((e = cudaMemsetAsync(p.xchg + XSYNC, 0, 256, stream)) != cudaSuccess)
    return cuda_error(e, "clearing the decoder barrier");
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.gridDim = dim3(RG);
  cfg.blockDim = dim3(RTHREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_error(cudaLaunchKernelEx(&cfg, tdt_resident_kernel, p), "tdt_resident launch");
}

}  // namespace pk
