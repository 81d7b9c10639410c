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
// channels and head columns [8 c, 8 c + 8) (the last CTA also the 8-column
// blank/duration tail).  Each step every CTA computes its slice for every
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
constexpr int RHEADCOLS = 16;         // token columns + the tail slot
constexpr int RMAXB = 40;             // windows per launch
constexpr int RPAIRS = RMAXB / 2;     // window pairs (half2 lanes)
constexpr int RHALF = RH / 2;         // joint / projector inputs per staged half
constexpr int RLSTM_PAIRS = 4;        // window pairs per LSTM chain thread
constexpr int RLSTM_GROUPS = RPAIRS / RLSTM_PAIRS;       // 5
constexpr int RLSTM_PER_PAR = RGATES * RLSTM_GROUPS;     // chain threads per parity: (output, group), 100
constexpr int RLSTM_THREADS = 2 * RLSTM_PER_PAR;         // 200
constexpr int RW_STRIDE = RKIN + 8;   // padded weight row (halfs): rows start 16 bytes apart in the banks
constexpr int RHW_STRIDE = RH + 8;    // padded head row: the 16 columns' loads spread over the banks
constexpr int RHEAD_THREADS = RHEADCOLS * RPAIRS;        // column x window pair: 320
constexpr int RPROJ_THREADS = RCH * RMAXB;               // output x window: 200
constexpr int RCHUNK = 8;             // chain steps per operand load
constexpr int RTHREADS = 640;
constexpr int RROW16 = RMAXB * 2 / 16;  // 16-byte chunks per exchanged f16 row (one value per window)
constexpr float RNEG = -3.402823466e+38f;
static_assert(RG * RCH == RH && RG * RTOK == 1024, "slices tile the matrices");
static_assert(RTHREADS == RH, "one thread per joint input");
static_assert(RLSTM_THREADS <= RTHREADS && RHEAD_THREADS % 32 == 0 && RHEAD_THREADS <= RTHREADS, "thread roles fit");
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
constexpr size_t XH1F = XH1N + 1ull * RH * RMAXB * 2;     // float [640][40]: layer-1 hidden for the projector
constexpr size_t XPROJ = XH1F + 1ull * RH * RMAXB * 4;    // float [40][640]: predictor projection
constexpr size_t XPART = XPROJ + 1ull * RMAXB * RH * 4;   // RPartial [2][40][128]: argmax partials
constexpr size_t XSYNC = XPART + 2ull * RMAXB * RG * 16;  // barrier counter, abort flag
static_assert(XSYNC + 256 <= kTdtExchangeBytes, "exchange area fits");
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
  __half w0[RGATES][RW_STRIDE];      // [gate output][input] (inputs fastest)
  __half w1[RGATES][RW_STRIDE];
  __half hw[RHEADCOLS][RHW_STRIDE];  // [head column][input]
  float pwf[RCH][RH];                // projector weights as f32, [output][input]
  union {
    __half2 x2[RH][RPAIRS];          // one half of an LSTM layer's inputs, [input][window pair]
    float hf[RMAXB][RHALF + 4];      // one half of the projector inputs, [window][input] (rows padded)
    struct {
      uint32_t j2[RPAIRS][RHALF];    // one half of the joint inputs, [window pair][input] (half2 bits)
      uint32_t keep[RPAIRS][RHALF];  // per pair and input: the lanes whose head chain skips it
    } jt;
    RPartial red[RMAXB][20];         // argmax reduction
  } in;
  float gates[RMAXB][RGATES];
  float c0[RMAXB][RCH];
  float c1[RMAXB][RCH];
  __half hnew[RMAXB][RCH];           // this CTA's new hidden slice, committed one barrier later
  uint32_t psum[2][RPAIRS][RGATES];  // the parity chains' sums (half2 bits), [parity][window pair][gate]
  float b0[RGATES], b1[RGATES], pb[8], hb[RHEADCOLS];
  int first_exc[RMAXB];
  RWin win[RMAXB];
  int any_pending, any_token, any_joint;
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
__device__ __forceinline__ float* proj_at(const RParams& p, int w) {
  return reinterpret_cast<float*>(p.xchg + XPROJ) + (size_t)w * RH;
}
__device__ __forceinline__ RPartial* part_at(const RParams& p, int slot, int w, int cta) {
  return reinterpret_cast<RPartial*>(p.xchg + XPART) + ((size_t)slot * RMAXB + w) * RG + cta;
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

// The embedding rows of the windows updating with a token, into x2; lane =
// window (8 halfs per 16-byte load), so a warp's half-word stores land in
// adjacent words.
__device__ void stage_embeddings(RSmem& s, const RParams& p) {
  constexpr int PER = RMAXB * RH / 8 / RTHREADS;
  static_assert(RMAXB * RH / 8 % RTHREADS == 0, "whole chunks per thread");
  uint4 v[PER];
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int i = threadIdx.x + j * RTHREADS, w = i % RMAXB, k = 8 * (i / RMAXB);
    v[j] = make_uint4(0u, 0u, 0u, 0u);
    if (w < p.batch && s.win[w].pending == 2)
      v[j] = *reinterpret_cast<const uint4*>(p.emb + (size_t)s.win[w].token * RH + k);
  }
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int i = threadIdx.x + j * RTHREADS, w = i % RMAXB, k = 8 * (i / RMAXB);
    const __half* h = reinterpret_cast<const __half*>(&v[j]);
#pragma unroll
    for (int e = 0; e < 8; ++e) set_lane(&s.in.x2[k + e][w >> 1], w & 1, h[e]);
  }
}

// One staged half (640 inputs) of this thread's gate chains: gate output of
// `wrow` (its 640 weights of this half, both parities interleaved), parity
// `par`, window pairs 4 g .. 4 g + 3.  REC: lanes in `keep` leave their
// accumulator as it was (start-of-sequence windows skip the recurrent half).
// The chain threads of one warp share their parity, so every x2 load of a
// warp reads one 80-byte row (one wavefront) and its weight loads a few rows.
// Operands of 4 chain steps (8 inputs from k): this parity's 4 weights and
// the 4 window pairs' inputs.
struct LstmChunk {
  uint4 w;     // 8 weights, inputs k .. k + 7
  uint4 x[4];  // inputs k + par, k + 2 + par, ... for the thread's 4 pairs
};

__device__ __forceinline__ void lstm_load(const RSmem& s, const __half* wrow, int k, int g, int par, LstmChunk& c) {
  c.w = *reinterpret_cast<const uint4*>(wrow + k);
#pragma unroll
  for (int j = 0; j < 4; ++j) c.x[j] = *reinterpret_cast<const uint4*>(&s.in.x2[k + 2 * j + par][4 * g]);
}

template <bool REC>
__device__ __forceinline__ void lstm_math(const LstmChunk& c, int par, const uint32_t (&keep)[RLSTM_PAIRS],
                                          __half2 (&acc)[RLSTM_PAIRS]) {
  const uint32_t ww[4] = {c.w.x, c.w.y, c.w.z, c.w.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const __half2 wv = __half2half2(__ushort_as_half((unsigned short)(par ? ww[j] >> 16 : ww[j] & 0xffffu)));
    const uint32_t xs[RLSTM_PAIRS] = {c.x[j].x, c.x[j].y, c.x[j].z, c.x[j].w};
#pragma unroll
    for (int i = 0; i < RLSTM_PAIRS; ++i) {
      if constexpr (REC)
        acc[i] = keep_mask(acc[i], __hfma2(bits_h2(xs[i]), wv, acc[i]), keep[i]);
      else
        acc[i] = __hfma2(bits_h2(xs[i]), wv, acc[i]);
    }
  }
}

// One staged half (640 inputs) of this thread's gate chains: gate output of
// `wrow` (its 640 weights of this half, both parities interleaved), parity
// `par`, window pairs 4 g .. 4 g + 3.  REC: lanes in `keep` leave their
// accumulator as it was (start-of-sequence windows skip the recurrent half).
// The chain threads of one warp share their parity, so every x2 load of a
// warp reads one 80-byte row (one wavefront) and its weight loads a few rows.
// Two operand buffers alternate: the loads of the next 8 inputs are issued
// before the chain steps of the current 8.
template <bool REC>
__device__ __forceinline__ void lstm_chain_half(const RSmem& s, const __half* wrow, int g, int par,
                                                const uint32_t (&keep)[RLSTM_PAIRS], __half2 (&acc)[RLSTM_PAIRS]) {
  LstmChunk a, b;
  lstm_load(s, wrow, 0, g, par, a);
#pragma unroll 1
  for (int k = 0; k < RH; k += 16) {
    lstm_load(s, wrow, k + 8, g, par, b);
    lstm_math<REC>(a, par, keep, acc);
    if (k + 16 < RH) lstm_load(s, wrow, k + 16, g, par, a);
    lstm_math<REC>(b, par, keep, acc);
  }
}

// Gate chains of one LSTM layer for the windows that need them; gates land in
// s.gates[window][gate * 5 + channel].  Chain thread t < 200: parity t / 100,
// output (t % 100) / 5, group of 4 window pairs t % 5.  Inputs: layer 0
// [embedding(token) | h0], layer 1 [new h0 | h1], staged one half at a time.
// Layer 1's start-of-sequence windows stop at input 640 (their recurrent
// input is zero and the shader does not run those steps); lanes of windows
// that do not update compute values nobody reads.
__device__ void lstm_layer(RSmem& s, const RParams& p, bool layer1) {
  const int tid = threadIdx.x;
  const bool chain = tid < RLSTM_THREADS;
  const int par = tid / RLSTM_PER_PAR, idx = tid % RLSTM_PER_PAR;
  const int o = idx / RLSTM_GROUPS, grp = idx % RLSTM_GROUPS;
  const __half* wrow = layer1 ? &s.w1[o][0] : &s.w0[o][0];
  bool any = false, any_full = false;
  uint32_t keep_rec[RLSTM_PAIRS];
  __half2 acc[RLSTM_PAIRS];
  if (chain) {
    const __half2 init = par == 0 ? __float2half2_rn((layer1 ? s.b1 : s.b0)[o]) : __float2half2_rn(0.0f);
#pragma unroll
    for (int i = 0; i < RLSTM_PAIRS; ++i) {
      const int w0 = (grp * RLSTM_PAIRS + i) * 2;
      const int p0 = s.win[w0].pending, p1 = s.win[w0 + 1].pending;
      keep_rec[i] = lane_mask(p0 == 1, p1 == 1);
      any |= layer1 ? (p0 | p1) != 0 : (p0 == 2 || p1 == 2);
      any_full |= p0 == 2 || p1 == 2;
      acc[i] = init;
    }
  }
  const bool tokens = s.any_token != 0;
  if (layer1 || tokens) {
    if (layer1)
      stage_rows(s, xh(p, XH0N));
    else
      stage_embeddings(s, p);
    __syncthreads();
    if (chain && any) lstm_chain_half<false>(s, wrow, grp, par, keep_rec, acc);
  }
  if (tokens) {
    __syncthreads();  // the first half is consumed
    stage_rows(s, xh(p, layer1 ? XH1 : XH0));
    __syncthreads();
    if (chain && (layer1 ? any_full : any)) {
      if (layer1)
        lstm_chain_half<true>(s, wrow + RH, grp, par, keep_rec, acc);
      else
        lstm_chain_half<false>(s, wrow + RH, grp, par, keep_rec, acc);
    }
  }
  // The two parity chains of a gate sum in f16.
  if (chain && any) {
#pragma unroll
    for (int i = 0; i < RLSTM_PAIRS; ++i) s.psum[par][grp * RLSTM_PAIRS + i][o] = h2_bits(acc[i]);
  }
  __syncthreads();
  for (int i = tid; i < RPAIRS * RGATES; i += RTHREADS) {
    const int pr = i / RGATES, g = i % RGATES;
    const bool upd = layer1 ? (s.win[2 * pr].pending | s.win[2 * pr + 1].pending) != 0
                            : (s.win[2 * pr].pending == 2 || s.win[2 * pr + 1].pending == 2);
    if (upd) {
      const float2 v = __half22float2(__hadd2(bits_h2(s.psum[0][pr][g]), bits_h2(s.psum[1][pr][g])));
      s.gates[2 * pr][g] = v.x;
      s.gates[2 * pr + 1][g] = v.y;
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
    if (layer1) h1f_at(p)[at] = h;
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
// halves of the new layer-1 hidden state (transposed to [window][input] while
// staging, so a thread's inputs and weights are 16-byte loads along k);
// thread: (output, window).
__device__ void projector(RSmem& s, const RParams& p) {
  const int tid = threadIdx.x;
  const int o = tid / RMAXB, w = tid % RMAXB;
  const bool live = tid < RPROJ_THREADS && w < p.batch && s.win[w].pending;
  float acc = live ? s.pb[o] : 0.0f;
  for (int h = 0; h < 2; ++h) {
    if (h) __syncthreads();  // the first half is consumed
    {
      constexpr int Q = RMAXB / 4;  // 16-byte chunks per exchanged row
      constexpr int PER = RHALF * Q / RTHREADS;
      static_assert(RHALF * Q % RTHREADS == 0, "whole chunks per thread");
      const uint4* src = reinterpret_cast<const uint4*>(h1f_at(p) + (size_t)h * RHALF * RMAXB);
      uint4 v[PER];
#pragma unroll
      for (int j = 0; j < PER; ++j) v[j] = __ldcg(src + tid + j * RTHREADS);
#pragma unroll
      for (int j = 0; j < PER; ++j) {
        const int i = tid + j * RTHREADS, k = i / Q, w4 = 4 * (i % Q);
        s.in.hf[w4][k] = __uint_as_float(v[j].x);
        s.in.hf[w4 + 1][k] = __uint_as_float(v[j].y);
        s.in.hf[w4 + 2][k] = __uint_as_float(v[j].z);
        s.in.hf[w4 + 3][k] = __uint_as_float(v[j].w);
      }
    }
    __syncthreads();
    if (live) {
      const float* hrow = &s.in.hf[w][0];
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
    }
  }
  if (live) proj_at(p, w)[blockIdx.x * RCH + o] = acc;
}

__device__ void lstm_update(RSmem& s, const RParams& p) {
  const int tid = threadIdx.x;
  // Layer 0: inputs [embedding(token) | h0]; start-of-sequence windows take the bias.
  lstm_layer(s, p, false);
  __syncthreads();
  for (int i = tid; i < p.batch * RGATES; i += RTHREADS) {
    const int w = i / RGATES, o = i % RGATES;
    if (s.win[w].pending == 1) s.gates[w][o] = __half2float(__float2half_rn(s.b0[o]));
  }
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

// One staged half (320 inputs) of this thread's head chain: column `col`,
// window pair `pair`, starting at input `kb`.
__device__ __forceinline__ void head_chain_half(const RSmem& s, int col, int pair, int kb, __half2& acc) {
  const __half* wrow = &s.hw[col][kb];
  const uint32_t* xrow = &s.in.jt.j2[pair][0];
  const uint32_t* mrow = &s.in.jt.keep[pair][0];
#pragma unroll 2
  for (int k0 = 0; k0 < RHALF; k0 += RCHUNK) {
    // 8 steps per 16-byte load of each operand.
    const uint4 wq = *reinterpret_cast<const uint4*>(wrow + k0);
    const uint4 xa = *reinterpret_cast<const uint4*>(xrow + k0), xb = *reinterpret_cast<const uint4*>(xrow + k0 + 4);
    const uint4 ma = *reinterpret_cast<const uint4*>(mrow + k0), mb = *reinterpret_cast<const uint4*>(mrow + k0 + 4);
    const uint32_t wpair[4] = {wq.x, wq.y, wq.z, wq.w};
    const uint32_t xs[RCHUNK] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
    const uint32_t ms[RCHUNK] = {ma.x, ma.y, ma.z, ma.w, mb.x, mb.y, mb.z, mb.w};
    if ((ma.x | ma.y | ma.z | ma.w | mb.x | mb.y | mb.z | mb.w) == 0u) {  // no skipped input here
#pragma unroll
      for (int j = 0; j < RCHUNK; ++j) {
        const uint32_t wb = (j & 1) ? (wpair[j >> 1] >> 16) : (wpair[j >> 1] & 0xffffu);
        acc = __hfma2(bits_h2(xs[j]), __half2half2(__ushort_as_half((unsigned short)wb)), acc);
      }
    } else {
#pragma unroll
      for (int j = 0; j < RCHUNK; ++j) {
        const uint32_t wb = (j & 1) ? (wpair[j >> 1] >> 16) : (wpair[j >> 1] & 0xffffu);
        acc = keep_mask(acc, __hfma2(bits_h2(xs[j]), __half2half2(__ushort_as_half((unsigned short)wb)), acc), ms[j]);
      }
    }
  }
}

// Joint of the active windows: inputs, head columns, this CTA's partials.
// Thread k builds input k for every window (coalesced loads along k) and
// keeps them in registers; the inputs are staged for the head chains in two
// halves.
__device__ void joint_partials(RSmem& s, const RParams& p, int slot) {
  const int tid = threadIdx.x;
  if (tid < RMAXB) s.first_exc[tid] = RH;
  __syncthreads();
  const int k = tid;
  uint32_t packed[RPAIRS];  // half2 bits of input k, per window pair
  uint64_t zero_bits = 0ull;
  constexpr int WG = 20;  // windows whose loads are in flight together
#pragma unroll
  for (int w0 = 0; w0 < RMAXB; w0 += WG) {
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
    for (int i = 0; i < WG; i += 2) {
      __half hv[2];
#pragma unroll
      for (int l = 0; l < 2; ++l) {
        const int w = w0 + i + l;
        hv[l] = __float2half_rn(0.0f);
        if (w < p.batch && s.win[w].joint) {
          const float x = __fadd_rn(__half2float(ev[i + l]), pv[i + l]);
          const float jv = x < 0.0f ? 0.0f : x;  // max(x, 0) keeping -0 and NaN, as the oracle's std::max
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
  const int col = tid % RHEADCOLS, pair = tid / RHEADCOLS;  // windows 2 pair, 2 pair + 1
  const bool head = tid < RHEAD_THREADS;
  const bool tail = col >= RTOK;
  const bool live = head && (!tail || blockIdx.x == RG - 1);
  __half2 acc = __float2half2_rn(head ? s.hb[col] : 0.0f);
  const bool run = live && (s.win[2 * pair].joint || s.win[2 * pair + 1].joint);
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
    if (run) head_chain_half(s, col, pair, h * RHALF, acc);
  }
  if (head) {
    const float2 v01 = __half22float2(acc);
    const float vals[2] = {sanitize(v01.x), sanitize(v01.y)};
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      float tv = RNEG, dv = RNEG;
      uint32_t ti = 0xffffffffu, di = 0xffffffffu;
      if (live) {
        if (!tail) {
          tv = vals[i];
          ti = blockIdx.x * RTOK + col;
        } else if (col == RTOK) {
          tv = vals[i];
          ti = RBLANK;
        } else if (col <= RTOK + 5) {
          dv = vals[i];
          di = col - RTOK - 1;
        }
      }
#pragma unroll
      for (int off = RHEADCOLS / 2; off > 0; off >>= 1) {
        const float otv = __shfl_xor_sync(0xffffffffu, tv, off);
        const uint32_t oti = __shfl_xor_sync(0xffffffffu, ti, off);
        const float odv = __shfl_xor_sync(0xffffffffu, dv, off);
        const uint32_t odi = __shfl_xor_sync(0xffffffffu, di, off);
        if (better(tv, ti, otv, oti)) tv = otv, ti = oti;
        if (better(dv, di, odv, odi)) dv = odv, di = odi;
      }
      const int w = pair * 2 + i;
      if (col == 0 && w < p.batch && s.win[w].joint) *part_at(p, slot, w, blockIdx.x) = RPartial{tv, ti, dv, di};
    }
  }
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
// Thread (window, q) loads its 6 or 7 partials at once, then reduces them.
__device__ void joint_decide(RSmem& s, const RParams& p, int slot) {
  const int tid = threadIdx.x;
  constexpr int PER = (RG + 19) / 20;
  for (int i = tid; i < RMAXB * 20; i += RTHREADS) {
    const int w = i / 20, q = i % 20;
    RPartial b{RNEG, 0xffffffffu, RNEG, 0xffffffffu};
    if (w < p.batch && s.win[w].joint) {
      uint4 raw[PER];
#pragma unroll
      for (int j = 0; j < PER; ++j)
        if (q + 20 * j < RG) raw[j] = __ldcg(reinterpret_cast<const uint4*>(part_at(p, slot, w, q + 20 * j)));
#pragma unroll
      for (int j = 0; j < PER; ++j) {
        if (q + 20 * j >= RG) continue;
        const RPartial v{__uint_as_float(raw[j].x), raw[j].y, __uint_as_float(raw[j].z), raw[j].w};
        if (better(b.tv, b.ti, v.tv, v.ti)) b.tv = v.tv, b.ti = v.ti;
        if (better(b.dv, b.di, v.dv, v.di)) b.dv = v.dv, b.di = v.di;
      }
    }
    s.in.red[w][q] = b;
  }
  __syncthreads();
  if (tid < p.batch && s.win[tid].joint) {
    const int w = tid;
    RPartial b = s.in.red[w][0];
    for (int q = 1; q < 20; ++q) {
      const RPartial v = s.in.red[w][q];
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

__global__ void __launch_bounds__(RTHREADS, 1) tdt_resident_kernel(const RParams p) {
  extern __shared__ __align__(128) unsigned char rsmem_raw[];
  RSmem& s = *reinterpret_cast<RSmem*>((reinterpret_cast<uintptr_t>(rsmem_raw) + 127) & ~static_cast<uintptr_t>(127));
  const int tid = threadIdx.x, cta = blockIdx.x;
  // This CTA's weight slices (one-time; columns gate * 640 + 5 cta + channel).
  for (int i = tid; i < RKIN * RGATES; i += RTHREADS) {
    const int k = i / RGATES, o = i % RGATES;
    const size_t col = (size_t)(o / RCH) * RH + cta * RCH + o % RCH;
    s.w0[o][k] = p.w0[(size_t)k * 4 * RH + col];
    s.w1[o][k] = p.w1[(size_t)k * 4 * RH + col];
  }
  for (int i = tid; i < RH * RCH; i += RTHREADS) {
    const int k = i / RCH, o = i % RCH;
    s.pwf[o][k] = __half2float(p.pw[(size_t)k * RH + cta * RCH + o]);
  }
  for (int i = tid; i < RH * RHEADCOLS; i += RTHREADS) {
    const int k = i / RHEADCOLS, c = i % RHEADCOLS;
    const int col = c < RTOK ? cta * RTOK + c : (cta == RG - 1 ? RBLANK + (c - RTOK) : -1);
    s.hw[c][k] = col >= 0 ? p.hw[(size_t)k * ROUT + col] : __float2half_rn(0.0f);
  }
  if (tid < RGATES) {
    const size_t col = (size_t)(tid / RCH) * RH + cta * RCH + tid % RCH;
    s.b0[tid] = p.b0[col];
    s.b1[tid] = p.b1[col];
  }
  if (tid < 8) s.pb[tid] = tid < RCH ? p.pb[cta * RCH + tid] : 0.0f;
  if (tid < RHEADCOLS) {
    const int col = tid < RTOK ? cta * RTOK + tid : (cta == RG - 1 ? RBLANK + (tid - RTOK) : -1);
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
  if (tid == 0) s.gen = 0;
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
      joint_partials(s, p, slot);
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
