// tdt_decoder.cu -- persistent greedy TDT decoder (prediction net + joint)
// for sm_100a, the B200 counterpart of PersistentTdtDecoderKernel
// (src/webgpu/kernels/tdt-decoder.ts:155-330, shader :1076-2000).
//
// Work split: one thread-block cluster of TCL = 4 CTAs decodes one window.
// CTA r of the cluster owns LSTM channels [160 r, 160 r + 160) -- the four
// gates (i, f, g, o) of those channels, so the cell update is local -- the
// projector outputs of the same channels and head outputs [256 r, 256 r + 256)
// (the last CTA also the blank/duration tail 1024..1031).  Each CTA pushes
// the hidden / projection slices it produces into every peer's shared memory
// (distributed shared memory stores) and the cluster synchronises with an
// mbarrier that each CTA arrives on remotely (every wait bounded); the
// argmax partials are read back from the peers the same way, so all CTAs
// take the same decision and follow the same control flow.
//
// Weights (14.6 MB FP16, L2-resident after the first windows) stream through
// a 10-stage (FP32: 9) shared-memory ring filled by TMA from four producer warps that
// take the stages in turn (one 20 KB box each; a single thread's boxes are
// serviced one after another, so four issuing warps stream four boxes at
// once), running ahead across the LSTM layers, the projector and the next
// head pass (everything but the choice after each joint is known in
// advance).
//
// Arithmetic is the reference shader's, step for step: each LSTM gate is two
// FMA chains in increasing input index (even indices from the bias, odd
// indices from zero) summed at the end; FP16 chains are f16 FMAs (HFMA2,
// single rounding) on f16 inputs; the head is one chain per output that
// skips +0 inputs until a -0 or NaN input is seen; the projection is an f32
// FMA chain; sigmoid / tanh clamp as the shader does (their exp / tanh
// correctly rounded to f32).  Token choice: largest
// score, lowest id on ties, NaN as -FLT_MAX.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "pk_common.cuh"
#include "pk_internal.h"

namespace pk {
namespace {

constexpr int TH = 640;                 // prediction-net hidden size
constexpr int TKIN = 1280;              // LSTM input [x | h]
constexpr int TOUT = 1032;              // head storage outputs (1025 tokens + 5 durations + 2 pad)
constexpr int TBLANK = 1024;
constexpr int TMAXSYM = 10;             // symbols per frame before a forced advance
constexpr int TCL = 4;                  // CTAs per cluster (one window per cluster)
constexpr int TCH = TH / TCL;           // 160 channels per CTA
constexpr int TPAIRS = 2 * TCH;         // 320 (gate, channel pair) outputs per CTA
constexpr int TCOMPUTE = 2 * TPAIRS;    // 640 compute threads: output pair x even/odd chain
constexpr int TCWARPS = TCOMPUTE / 32;  // 20
constexpr int TPROD = 4;                // TMA producer warps: each issues one quarter of every stage
constexpr int TTHREADS = TCOMPUTE + 32 * TPROD;
constexpr int THEAD = 1024 / TCL;       // 256 token outputs per CTA
// Ring depth: as many 20 KB stages as shared memory holds beside the rest.
template <typename T>
constexpr int tdt_stages() { return sizeof(T) == 2 ? 10 : 9; }
constexpr int TSTAGE_BYTES = 20480;
constexpr int TTAIL_OFFSET = 16384;     // the tail columns follow the 256-column head tile
constexpr int TCHUNK = 8;               // rows whose operands a consumer loads before chaining them
constexpr float TNEG = -3.402823466e+38f;

static_assert(TCOMPUTE == TH, "one compute thread per joint input");

template <typename T>
struct TdtType;
template <>
struct TdtType<__half> {
  using T2 = __half2;
  static __device__ __forceinline__ T2 bias2(float a, float b) { return __floats2half2_rn(a, b); }
  static __device__ __forceinline__ T2 zero2() { return __float2half2_rn(0.0f); }
  static __device__ __forceinline__ T2 fma2(__half x, T2 w, T2 acc) { return __hfma2(__half2half2(x), w, acc); }
  static __device__ __forceinline__ float2 sum2(T2 a, T2 b) { return __half22float2(__hadd2(a, b)); }
  static __device__ __forceinline__ float2 to_f2(T2 a) { return __half22float2(a); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
  static __device__ __forceinline__ float round_bias(float v) { return __half2float(__float2half_rn(v)); }
};
template <>
struct TdtType<float> {
  using T2 = float2;
  static __device__ __forceinline__ T2 bias2(float a, float b) { return make_float2(a, b); }
  static __device__ __forceinline__ T2 zero2() { return make_float2(0.0f, 0.0f); }
  static __device__ __forceinline__ T2 fma2(float x, T2 w, T2 acc) {
    return make_float2(__fmaf_rn(x, w.x, acc.x), __fmaf_rn(x, w.y, acc.y));
  }
  static __device__ __forceinline__ float2 sum2(T2 a, T2 b) { return make_float2(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y)); }
  static __device__ __forceinline__ float2 to_f2(T2 a) { return a; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
  static __device__ __forceinline__ float round_bias(float v) { return v; }
};

// Rows (input indices) per ring stage: every tile is 20 KB (the head 16 KB).
template <typename T>
constexpr int rows_lstm() { return 32 / (int)sizeof(T); }   // [rows][4 gates][160 channels]
template <typename T>
constexpr int rows_proj() { return 128 / (int)sizeof(T); }  // [rows][160 outputs]
template <typename T>
constexpr int rows_head() { return 64 / (int)sizeof(T); }   // [rows][256 outputs] (+ [rows][8] tail)

struct __align__(16) TdtPartial {
  float tv;
  uint32_t ti;
  float dv;
  uint32_t di;
};

// What follows a decision, published to the whole CTA.
struct TdtPlan {
  int lstm;     // run an LSTM update with `token` before the next joint
  int initial;  // the update is the start-of-sequence one (zero input and state)
  int token;
  int joint;    // another joint follows
  int joint_t;  // its encoder frame
};

template <typename T>
struct TdtSmem {
  alignas(128) unsigned char ring[tdt_stages<T>()][TSTAGE_BYTES];
  alignas(16) T emb[TH];
  alignas(16) T h0[2][TH];
  alignas(16) T h1[2][TH];
  alignas(16) T jin[TH];
  alignas(16) float h1f[TH];
  alignas(16) float proj[TH];
  alignas(16) float gates[4 * TCH];
  alignas(16) float c0[TCH];
  alignas(16) float c1[TCH];
  alignas(16) typename TdtType<T>::T2 odd[TPAIRS];
  alignas(16) TdtPartial wpart[TCWARPS];
  alignas(16) TdtPartial part[2];
  unsigned char jzero[TH];
  uint32_t jskip[TH / 32];  // bit r of word w: the head skips input 32 w + r
  alignas(8) uint64_t full[tdt_stages<T>()];
  alignas(8) uint64_t empty[tdt_stages<T>()];
  alignas(8) uint64_t emb_bar;
  alignas(8) uint64_t cbar;
  TdtPlan plan;
  int first_exc;
  volatile int abort;
};

// Dynamic shared memory (plus 1 KB of alignment slack) stays within the
// 227 KB a CTA may opt into.
static_assert(sizeof(TdtSmem<__half>) + 1024 <= 232448, "FP16 decoder shared memory");
static_assert(sizeof(TdtSmem<float>) + 1024 <= 232448, "FP32 decoder shared memory");

struct TdtParams {
  CUtensorMap map_l0;    // [1280 k][4 gates][640 ch], box {160, 4, rows_lstm}
  CUtensorMap map_l1;
  CUtensorMap map_proj;  // [640 k][640 out], box {160, rows_proj}
  CUtensorMap map_head;  // [640 k][1032 out], box {256, rows_head}
  CUtensorMap map_tail;  // same tensor, box {8, rows_head}
  const void* enc;       // [batch, frames, 640]
  const void* emb;       // [1025, 640]
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
  int batch;
  int frames;
  int max_tokens;
};

// ------------------------------------------------------------ primitives
// bar.sync is warp-aligned: reconverge the warp first (callers reach it from
// code where one lane did extra work).
__device__ __forceinline__ void named_sync(uint32_t id, uint32_t count) {
  __syncwarp();
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
__device__ __forceinline__ void block_sync() {
  __syncwarp();
  __syncthreads();
}
__device__ __forceinline__ void remote_arrive(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ bool try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity), "r"(20000u)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ void st_cluster_b16(uint32_t addr, unsigned short v) {
  asm volatile("st.shared::cluster.b16 [%0], %1;" ::"r"(addr), "h"(v) : "memory");
}
__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ TdtPartial ld_cluster_partial(uint32_t addr) {
  TdtPartial r;
  asm volatile("ld.shared::cluster.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=f"(r.tv), "=r"(r.ti), "=f"(r.dv), "=r"(r.di)
               : "r"(addr)
               : "memory");
  return r;
}
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_addr(dst)),
               "l"(src), "r"(bytes), "r"(smem_addr(bar))
               : "memory");
}
template <typename T>
__device__ __forceinline__ void push_scalar(uint32_t addr, T v);
template <>
__device__ __forceinline__ void push_scalar<__half>(uint32_t addr, __half v) {
  st_cluster_b16(addr, __half_as_ushort(v));
}
template <>
__device__ __forceinline__ void push_scalar<float>(uint32_t addr, float v) {
  st_cluster_f32(addr, v);
}

__device__ __forceinline__ bool better(float lv, uint32_t li, float rv, uint32_t ri) {
  return rv > lv || (rv == lv && ri < li);
}
__device__ __forceinline__ float sanitize(float v) { return v != v ? TNEG : v; }
__device__ __forceinline__ float sig_ref(float v) { return tdt_sigmoid(v); }
__device__ __forceinline__ float tanh_ref(float v) { return tdt_tanh(v); }

// Ring position shared by the producer and every consumer warp (each keeps
// its own copy; all walk the same stage sequence).
template <int NS>
struct Ring {
  uint32_t slot = 0, phase = 0, issued = 0;
  __device__ __forceinline__ void advance() {
    if (++slot == NS) {
      slot = 0;
      phase ^= 1u;
    }
    ++issued;
  }
};

template <typename T>
struct Ctx {
  TdtSmem<T>& s;
  const TdtParams& p;
  int rank, ct, lane;
  int pw = 0;             // producer warp index (producer threads)
  Ring<tdt_stages<T>()> ring;
  uint32_t cph = 0;       // cluster-barrier phase
  uint32_t emb_phase = 0; // embedding-row barrier phase
  int cur = 0;            // which h0 / h1 buffer holds the current state
};

// ------------------------------------------------------------ producer side
template <typename T>
__device__ __forceinline__ void produce_acquire(Ctx<T>& c) {
  mbar_wait(&c.s.empty[c.ring.slot], c.ring.phase ^ 1u, &c.s.abort, c.p.status, PK_STATUS_TIMEOUT_TMA);
}
// The producer warps take the ring's stages in turn: warp pw issues every
// stage whose index is pw modulo TPROD (all warps walk the same sequence).
template <typename T>
__device__ __forceinline__ bool my_stage(const Ctx<T>& c) {
  return c.ring.issued % TPROD == (uint32_t)c.pw;
}
template <typename T>
__device__ void produce_lstm(Ctx<T>& c, const CUtensorMap* map, int krows) {
  constexpr int R = rows_lstm<T>();
  for (int k0 = 0; k0 < krows; k0 += R) {
    if (my_stage(c)) {
      produce_acquire(c);
      mbar_arrive_expect_tx(&c.s.full[c.ring.slot], TSTAGE_BYTES);
      tma_load_3d(c.s.ring[c.ring.slot], map, &c.s.full[c.ring.slot], c.rank * TCH, 0, k0);
    }
    c.ring.advance();
  }
}
template <typename T>
__device__ void produce_proj(Ctx<T>& c) {
  constexpr int R = rows_proj<T>();
  for (int k0 = 0; k0 < TH; k0 += R) {
    if (my_stage(c)) {
      produce_acquire(c);
      mbar_arrive_expect_tx(&c.s.full[c.ring.slot], TSTAGE_BYTES);
      tma_load_2d(c.s.ring[c.ring.slot], &c.p.map_proj, &c.s.full[c.ring.slot], c.rank * TCH, k0);
    }
    c.ring.advance();
  }
}
template <typename T>
__device__ void produce_head(Ctx<T>& c) {
  constexpr int R = rows_head<T>();
  const bool tail = c.rank == TCL - 1;
  const uint32_t bytes = THEAD * R * sizeof(T) + (tail ? 8 * R * sizeof(T) : 0);
  for (int k0 = 0; k0 < TH; k0 += R) {
    if (my_stage(c)) {
      produce_acquire(c);
      mbar_arrive_expect_tx(&c.s.full[c.ring.slot], bytes);
      tma_load_2d(c.s.ring[c.ring.slot], &c.p.map_head, &c.s.full[c.ring.slot], c.rank * THEAD, k0);
      if (tail) tma_load_2d(c.s.ring[c.ring.slot] + TTAIL_OFFSET, &c.p.map_tail, &c.s.full[c.ring.slot], TBLANK, k0);
    }
    c.ring.advance();
  }
}
template <typename T>
__device__ void produce_update(Ctx<T>& c, const TdtPlan& pl) {
  if (!pl.initial) {
    if (c.pw == 0) {
      mbar_arrive_expect_tx(&c.s.emb_bar, TH * sizeof(T));
      bulk_load(c.s.emb, static_cast<const char*>(c.p.emb) + (size_t)pl.token * TH * sizeof(T), TH * sizeof(T),
                &c.s.emb_bar);
    }
    produce_lstm(c, &c.p.map_l0, TKIN);
  }
  produce_lstm(c, &c.p.map_l1, pl.initial ? TH : TKIN);
  produce_proj(c);
}

// ------------------------------------------------------------ consumer side
template <typename T>
__device__ __forceinline__ const T* consume_begin(Ctx<T>& c) {
  mbar_wait(&c.s.full[c.ring.slot], c.ring.phase, &c.s.abort, c.p.status, PK_STATUS_TIMEOUT_TMA);
  return reinterpret_cast<const T*>(c.s.ring[c.ring.slot]);
}
template <typename T>
__device__ __forceinline__ void consume_end(Ctx<T>& c) {
  __syncwarp();
  if (c.lane == 0) mbar_arrive(&c.s.empty[c.ring.slot]);
  c.ring.advance();
}

// Compute threads only: every CTA of the cluster reaches this point; the
// data each CTA pushed before it is visible to all after it.
template <typename T>
__device__ void cluster_barrier(Ctx<T>& c) {
  named_sync(1, TCOMPUTE);
  if (c.ct == 0) {
    asm volatile("fence.acq_rel.cluster;" ::: "memory");
    const uint32_t local = smem_addr(&c.s.cbar);
#pragma unroll
    for (int r = 0; r < TCL; ++r) remote_arrive(mapa_shared(local, (uint32_t)r));
    if (!try_wait_cluster(&c.s.cbar, c.cph)) {
      const uint64_t start = global_timer_ns();
      while (!try_wait_cluster(&c.s.cbar, c.cph)) {
        if (c.s.abort) break;
        if (global_timer_ns() - start > PK_WAIT_NS) {
          c.s.abort = 1;
          atomicOr(c.p.status, PK_STATUS_TIMEOUT_EPILOGUE);
          break;
        }
      }
    }
  }
  c.cph ^= 1u;
  named_sync(1, TCOMPUTE);
}

// One LSTM layer's gate chains over `krows` inputs: x[k] = k < 640 ? lo[k] :
// hi[k - 640].  Leaves f32 gates of this CTA's channels in s.gates
// ([gate][160]).  `bias` is the layer's [2560] gate bias.
template <typename T>
__device__ void lstm_gates(Ctx<T>& c, int krows, const T* lo, const T* hi, const float* bias) {
  using Ty = TdtType<T>;
  using T2 = typename Ty::T2;
  constexpr int R = rows_lstm<T>();
  const int par = c.ct / TPAIRS, j = c.ct % TPAIRS;
  const int g = j / (TCH / 2), q = j % (TCH / 2);
  const int ch = c.rank * TCH + 2 * q;
  T2 acc = par == 0 ? Ty::bias2(bias[g * TH + ch], bias[g * TH + ch + 1]) : Ty::zero2();
  for (int k0 = 0; k0 < krows; k0 += R) {
    const T* tile = consume_begin(c);
    const T* x = (k0 < TH ? lo + k0 : hi + (k0 - TH)) + par;
    const T* w = tile + (par * 4 + g) * TCH + 2 * q;
    // This parity's R/2 rows: all operands loaded first, then the chain.
    T xs[R / 2];
    T2 ws[R / 2];
#pragma unroll
    for (int i = 0; i < R / 2; ++i) {
      xs[i] = x[2 * i];
      ws[i] = *reinterpret_cast<const T2*>(w + 2 * i * 4 * TCH);
    }
#pragma unroll
    for (int i = 0; i < R / 2; ++i) acc = Ty::fma2(xs[i], ws[i], acc);
    consume_end(c);
  }
  if (par == 1) c.s.odd[j] = acc;
  named_sync(1, TCOMPUTE);
  if (par == 0) {
    const float2 v = Ty::sum2(acc, c.s.odd[j]);
    c.s.gates[g * TCH + 2 * q] = v.x;
    c.s.gates[g * TCH + 2 * q + 1] = v.y;
  }
  named_sync(1, TCOMPUTE);
}

// Cell update of this CTA's channels; pushes h (and, for layer 1, f32 h) to
// every CTA of the cluster.
template <typename T>
__device__ void cell_update(Ctx<T>& c, float* cstate, T* hdst, float* hf32dst) {
  if (c.ct < TCH) {
    const int ch = c.ct;
    const float i = sig_ref(c.s.gates[ch]);
    const float f = sig_ref(c.s.gates[TCH + ch]);
    const float g = tanh_ref(c.s.gates[2 * TCH + ch]);
    const float o = sig_ref(c.s.gates[3 * TCH + ch]);
    const float cell = __fmaf_rn(f, cstate[ch], __fmul_rn(i, g));
    cstate[ch] = cell;
    const float h = __fmul_rn(o, tanh_ref(cell));
    const int gch = c.rank * TCH + ch;
    const T hv = TdtType<T>::from_f(h);
    const uint32_t a_h = smem_addr(hdst + gch);
#pragma unroll
    for (int r = 0; r < TCL; ++r) push_scalar<T>(mapa_shared(a_h, (uint32_t)r), hv);
    if (hf32dst) {
      const uint32_t a_f = smem_addr(hf32dst + gch);
#pragma unroll
      for (int r = 0; r < TCL; ++r) st_cluster_f32(mapa_shared(a_f, (uint32_t)r), h);
    }
  }
}

template <typename T>
__device__ void consume_update(Ctx<T>& c, const TdtPlan& pl) {
  const int nxt = c.cur ^ 1;
  // Layer 0.
  if (pl.initial) {
    if (c.ct < 4 * TCH) {
      const int g = c.ct / TCH, ch = c.ct % TCH;
      c.s.gates[c.ct] = TdtType<T>::round_bias(c.p.b0[g * TH + c.rank * TCH + ch]);
    }
    named_sync(1, TCOMPUTE);
  } else {
    mbar_wait(&c.s.emb_bar, c.emb_phase, &c.s.abort, c.p.status, PK_STATUS_TIMEOUT_TMA);
    c.emb_phase ^= 1u;
    lstm_gates(c, TKIN, c.s.emb, c.s.h0[c.cur], c.p.b0);
  }
  cell_update(c, c.s.c0, c.s.h0[nxt], static_cast<float*>(nullptr));
  cluster_barrier(c);
  // Layer 1.
  lstm_gates(c, pl.initial ? TH : TKIN, c.s.h0[nxt], c.s.h1[c.cur], c.p.b1);
  cell_update(c, c.s.c1, c.s.h1[nxt], c.s.h1f);
  cluster_barrier(c);
  // Projector: 80 threads x 2 outputs, f32 chains.
  {
    constexpr int R = rows_proj<T>();
    const bool act = c.ct < TCH / 2;
    const int o = c.rank * TCH + 2 * c.ct;
    float2 acc = act ? make_float2(c.p.pb[o], c.p.pb[o + 1]) : make_float2(0.f, 0.f);
    for (int k0 = 0; k0 < TH; k0 += R) {
      const T* tile = consume_begin(c);
      if (act) {
        for (int r0 = 0; r0 < R; r0 += TCHUNK) {
          float hs[TCHUNK];
          float2 ws[TCHUNK];
#pragma unroll
          for (int i = 0; i < TCHUNK; ++i) {
            hs[i] = c.s.h1f[k0 + r0 + i];
            ws[i] = TdtType<T>::to_f2(
                *reinterpret_cast<const typename TdtType<T>::T2*>(tile + (r0 + i) * TCH + 2 * c.ct));
          }
#pragma unroll
          for (int i = 0; i < TCHUNK; ++i) {
            acc.x = __fmaf_rn(hs[i], ws[i].x, acc.x);
            acc.y = __fmaf_rn(hs[i], ws[i].y, acc.y);
          }
        }
      }
      consume_end(c);
    }
    if (act) {
      const uint32_t a = smem_addr(c.s.proj + o);
#pragma unroll
      for (int r = 0; r < TCL; ++r) {
        const uint32_t ra = mapa_shared(a, (uint32_t)r);
        st_cluster_f32(ra, acc.x);
        st_cluster_f32(ra + 4, acc.y);
      }
    }
  }
  cluster_barrier(c);
  c.cur = nxt;
}

// Joint at encoder frame t: head chains, this CTA's argmax partial, the
// cluster barrier, then (thread 0) the combined token / duration.
template <typename T>
__device__ void consume_joint(Ctx<T>& c, int window, int t, uint32_t jslot, uint32_t* token, uint32_t* duration) {
  using Ty = TdtType<T>;
  using T2 = typename Ty::T2;
  constexpr int R = rows_head<T>();
  {
    const int k = c.ct;
    const T* erow = static_cast<const T*>(c.p.enc) + ((size_t)window * c.p.frames + t) * TH;
    float e;
    if constexpr (sizeof(T) == 2) e = __half2float(erow[k]);
    else e = erow[k];
    const float x = __fadd_rn(e, c.s.proj[k]);
    const float jv = x < 0.0f ? 0.0f : x;  // max(x, 0) keeping x for -0 and NaN, as the oracle's std::max
    const uint32_t bits = __float_as_uint(jv);
    c.s.jin[k] = Ty::from_f(jv);
    c.s.jzero[k] = bits == 0u;
    if (bits == 0x80000000u || (bits & 0x7fffffffu) > 0x7f800000u) atomicMin(&c.s.first_exc, k);
  }
  named_sync(1, TCOMPUTE);
  {
    // The shader skips input k while no -0 / NaN input has been seen and k is
    // +0: one bit per input, 32 inputs per word (one word per warp).
    const int k = c.ct;
    const bool skip = k < c.s.first_exc && c.s.jzero[k];
    const uint32_t m = __ballot_sync(0xffffffffu, skip);
    if (c.lane == 0) c.s.jskip[k / 32] = m;
  }
  named_sync(1, TCOMPUTE);
  const bool tok_thread = c.ct < THEAD / 2;
  const bool tail_thread = c.rank == TCL - 1 && c.ct >= THEAD / 2 && c.ct < THEAD / 2 + 4;
  int o0;  // first of this thread's two outputs
  float b0v = 0.f, b1v = 0.f;
  if (tok_thread) o0 = c.rank * THEAD + 2 * c.ct;
  else if (tail_thread) o0 = TBLANK + 2 * (c.ct - THEAD / 2);
  else o0 = 0;
  if (tok_thread || tail_thread) {
    b0v = c.p.hb[o0];
    b1v = c.p.hb[o0 + 1];
  }
  T2 acc = Ty::bias2(b0v, b1v);
  for (int k0 = 0; k0 < TH; k0 += R) {
    const T* tile = consume_begin(c);
    if (tok_thread || tail_thread) {
      const T* wbase = tok_thread ? tile + 2 * c.ct : tile + TTAIL_OFFSET / sizeof(T) + 2 * (c.ct - THEAD / 2);
      const int wstride = tok_thread ? THEAD : 8;
      for (int r0 = 0; r0 < R; r0 += TCHUNK) {
        const int kk = k0 + r0;
        const uint32_t skips = c.s.jskip[kk / 32] >> (kk % 32);
        T xs[TCHUNK];
        T2 ws[TCHUNK];
#pragma unroll
        for (int i = 0; i < TCHUNK; ++i) {
          xs[i] = c.s.jin[kk + i];
          ws[i] = *reinterpret_cast<const T2*>(wbase + (r0 + i) * wstride);
        }
        // A skipped input leaves the accumulator exactly as it was.
#pragma unroll
        for (int i = 0; i < TCHUNK; ++i) {
          const T2 f = Ty::fma2(xs[i], ws[i], acc);
          acc = (skips >> i) & 1u ? acc : f;
        }
      }
    }
    consume_end(c);
  }
  // Local argmax.
  float tv = TNEG, dv = TNEG;
  uint32_t ti = 0xffffffffu, di = 0xffffffffu;
  if (tok_thread || tail_thread) {
    const float2 v = Ty::to_f2(acc);
    const float s0 = sanitize(v.x), s1 = sanitize(v.y);
    if (tok_thread) {
      if (better(tv, ti, s0, (uint32_t)o0)) tv = s0, ti = (uint32_t)o0;
      if (better(tv, ti, s1, (uint32_t)o0 + 1)) tv = s1, ti = (uint32_t)o0 + 1;
    } else {
      const int tp = c.ct - THEAD / 2;  // tail pair: outputs 1024 + 2 tp, +1
      if (tp == 0) {
        tv = s0, ti = TBLANK;           // blank token
        dv = s1, di = 0;                // duration 0
      } else if (tp <= 2) {
        dv = s0, di = (uint32_t)(2 * tp - 1);
        if (better(dv, di, s1, (uint32_t)(2 * tp))) dv = s1, di = (uint32_t)(2 * tp);
      }
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float otv = __shfl_xor_sync(0xffffffffu, tv, off);
    const uint32_t oti = __shfl_xor_sync(0xffffffffu, ti, off);
    const float odv = __shfl_xor_sync(0xffffffffu, dv, off);
    const uint32_t odi = __shfl_xor_sync(0xffffffffu, di, off);
    if (better(tv, ti, otv, oti)) tv = otv, ti = oti;
    if (better(dv, di, odv, odi)) dv = odv, di = odi;
  }
  if (c.lane == 0) c.s.wpart[c.ct / 32] = TdtPartial{tv, ti, dv, di};
  named_sync(1, TCOMPUTE);
  if (c.ct == 0) {
    TdtPartial best{TNEG, 0xffffffffu, TNEG, 0xffffffffu};
    for (int w = 0; w < TCWARPS; ++w) {
      const TdtPartial q = c.s.wpart[w];
      if (better(best.tv, best.ti, q.tv, q.ti)) best.tv = q.tv, best.ti = q.ti;
      if (better(best.dv, best.di, q.dv, q.di)) best.dv = q.dv, best.di = q.di;
    }
    c.s.part[jslot] = best;
  }
  cluster_barrier(c);
  if (c.ct == 0) {
    TdtPartial best{TNEG, 0xffffffffu, TNEG, 0xffffffffu};
    const uint32_t a = smem_addr(&c.s.part[jslot]);
    for (int r = 0; r < TCL; ++r) {
      const TdtPartial q = ld_cluster_partial(mapa_shared(a, (uint32_t)r));
      if (better(best.tv, best.ti, q.tv, q.ti)) best.tv = q.tv, best.ti = q.ti;
      if (better(best.dv, best.di, q.dv, q.di)) best.dv = q.dv, best.di = q.di;
    }
    *token = best.ti;
    *duration = best.di;
  }
}

template <typename T>
__global__ void __launch_bounds__(TTHREADS, 1) tdt_decoder_kernel(const __grid_constant__ TdtParams p) {
  extern __shared__ __align__(1024) unsigned char tdt_smem_raw[];
  TdtSmem<T>& s = *reinterpret_cast<TdtSmem<T>*>(
      (reinterpret_cast<uintptr_t>(tdt_smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  pdl_entry();
  const int tid = threadIdx.x;
  const int window = blockIdx.x / TCL;
  Ctx<T> c{s, p, (int)cluster_ctarank(), tid, tid & 31};
  const bool producer = tid >= TCOMPUTE;
  if (producer) c.pw = (tid - TCOMPUTE) / 32;

  if (tid == 0) {
    for (int i = 0; i < tdt_stages<T>(); ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], TCWARPS);
    }
    mbar_init(&s.emb_bar, 1);
    mbar_init(&s.cbar, TCL);
    s.abort = 0;
    s.first_exc = TH;
    fence_mbar_init();
  }
  for (int i = tid; i < 2 * TH; i += TTHREADS) {
    (&s.h0[0][0])[i] = TdtType<T>::from_f(0.0f);
    (&s.h1[0][0])[i] = TdtType<T>::from_f(0.0f);
  }
  for (int i = tid; i < TCH; i += TTHREADS) {
    s.c0[i] = 0.0f;
    s.c1[i] = 0.0f;
  }
  if (producer && c.lane == 0) {
    tma_prefetch_desc(&p.map_l0);
    tma_prefetch_desc(&p.map_l1);
    tma_prefetch_desc(&p.map_proj);
    tma_prefetch_desc(&p.map_head);
    tma_prefetch_desc(&p.map_tail);
  }
  block_sync();
  cluster_sync();  // every CTA's barriers exist before any remote arrive

  // Decoder control (thread 0 of every CTA keeps an identical copy).
  uint32_t enc_len = 0, t = 0, sym = 0, count = 0, flags = 0, fsym = 0, blanks = 0, ft = 0, jslot = 0;
  int mode = 0;  // 0 = main loop, 1 = end-of-stream flush
  const uint32_t len_c = min(p.lengths[window], (uint32_t)p.frames);
  if (tid == 0) {
    enc_len = min(len_c, p.ends[window]);
    t = min(p.starts[window], enc_len);
    TdtPlan pl{0, 0, 0, 0, 0};
    if (t < enc_len) pl = TdtPlan{1, 1, 0, 1, (int)t};
    s.plan = pl;
  }
  block_sync();
  TdtPlan pl = s.plan;

  while (true) {
    if (pl.lstm) {
      if (producer) {
        if (c.lane == 0) produce_update(c, pl);
        __syncwarp();
      } else {
        consume_update(c, pl);
      }
    }
    if (!pl.joint) break;
    if (producer) {
      if (c.lane == 0) produce_head(c);
      __syncwarp();
    } else {
      uint32_t tok = 0, dur = 0;
      consume_joint(c, window, pl.joint_t, jslot, &tok, &dur);
      if (tid == 0) {
        // Ids are always in range unless a bounded wait expired (the results
        // are then garbage and flagged); keep even that path in bounds.
        const bool nonblank = tok < (uint32_t)TBLANK;
        dur = min(dur, 4u);
        auto emit = [&](uint32_t frame) {
          if (count < (uint32_t)p.max_tokens) {
            if (c.rank == 0) {
              const size_t o = (size_t)window * p.max_tokens + count;
              p.tokens[o] = tok;
              p.token_frames[o] = frame;
              p.token_durations[o] = dur;
            }
            ++count;
          } else {
            flags |= 1u;
          }
        };
        TdtPlan next{nonblank ? 1 : 0, 0, (int)tok, 0, 0};
        if (mode == 0) {
          if (nonblank) emit(t);
          sym += 1;
          if (dur != 0) {
            t += dur;
            sym = 0;
          } else if (!nonblank || sym >= (uint32_t)TMAXSYM) {
            t += 1;
            sym = 0;
          }
          if (t < enc_len) {
            next.joint = 1;
          } else if (p.flush[window] != 0 && p.starts[window] < enc_len) {
            mode = 1;
            fsym = 0;
            blanks = 0;
            ft = t;
            next.joint = 1;
          }
        } else {
          if (!nonblank) {
            blanks += 1;
          } else {
            blanks = 0;
            emit(min(ft, enc_len - 1));
          }
          ft = min(ft + max(1u, dur), enc_len);
          fsym += 1;
          next.joint = (fsym < (uint32_t)TMAXSYM && blanks < 5u) ? 1 : 0;
        }
        if (next.joint) {
          if (mode == 0) {
            next.joint_t = (int)t;
          } else {
            const uint32_t v = fsym % 3u;
            if (v == 0) t = min(ft, len_c - 1);
            else if (v == 1) t = min(enc_len - 1, (uint32_t)p.frames - 1);
            else t = min(max(enc_len, 2u) - 2, (uint32_t)p.frames - 1);
            next.joint_t = (int)t;
          }
        }
        if (!next.joint) next.lstm = 0;  // the shader's last update feeds nothing
        s.plan = next;
        s.first_exc = TH;
      }
    }
    jslot ^= 1u;
    block_sync();
    pl = s.plan;
  }

  if (tid == 0 && c.rank == 0) {
    p.metadata[window] = count;
    p.metadata[p.batch + window] = flags;
  }
  // Drain: every load issued has landed before the CTA exits.
  if (producer && c.lane == 0) {
    auto r = c.ring;
    const uint32_t n = min(r.issued, (uint32_t)tdt_stages<T>());
    for (uint32_t i = 0; i < n; ++i) {
      // step back one stage
      if (r.slot == 0) {
        r.slot = tdt_stages<T>() - 1;
        r.phase ^= 1u;
      } else {
        --r.slot;
      }
      mbar_wait_drain(&s.full[r.slot], r.phase, p.status);
    }
  }
  block_sync();
  cluster_sync();  // no CTA leaves while a peer may still read or write its shared memory
}

bool encode_map(const DeviceCtx& dev, CUtensorMap* map, CUtensorMapDataType type, int rank, const void* base,
                const cuuint64_t* dims, const cuuint64_t* strides, const cuuint32_t* box) {
  auto fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(dev.encode_tiled);
  if (!fn) return false;
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, type, (cuuint32_t)rank, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename T>
int launch_tdt_typed(const DeviceCtx& dev, const pk_tdt_desc& d, cudaStream_t stream) {
  const CUtensorMapDataType type = sizeof(T) == 2 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  const cuuint64_t es = sizeof(T);
  TdtParams p;
  {
    const cuuint64_t dims[3] = {TH, 4, TKIN};
    const cuuint64_t strides[2] = {TH * es, 4 * TH * es};
    const cuuint32_t box[3] = {TCH, 4, (cuuint32_t)rows_lstm<T>()};
    if (!encode_map(dev, &p.map_l0, type, 3, d.lstm_weight0, dims, strides, box) ||
        !encode_map(dev, &p.map_l1, type, 3, d.lstm_weight1, dims, strides, box))
      return set_error(PK_E_CUDA, "cuTensorMapEncodeTiled failed (decoder LSTM weights)");
  }
  {
    const cuuint64_t dims[2] = {TH, TH};
    const cuuint64_t strides[1] = {TH * es};
    const cuuint32_t box[2] = {TCH, (cuuint32_t)rows_proj<T>()};
    if (!encode_map(dev, &p.map_proj, type, 2, d.projector_weight, dims, strides, box))
      return set_error(PK_E_CUDA, "cuTensorMapEncodeTiled failed (decoder projector)");
  }
  {
    const cuuint64_t dims[2] = {TOUT, TH};
    const cuuint64_t strides[1] = {TOUT * es};
    const cuuint32_t box[2] = {THEAD, (cuuint32_t)rows_head<T>()};
    const cuuint32_t tbox[2] = {8, (cuuint32_t)rows_head<T>()};
    if (!encode_map(dev, &p.map_head, type, 2, d.head_weight, dims, strides, box) ||
        !encode_map(dev, &p.map_tail, type, 2, d.head_weight, dims, strides, tbox))
      return set_error(PK_E_CUDA, "cuTensorMapEncodeTiled failed (joint head)");
  }
  p.enc = d.encoder_projected;
  p.emb = d.embedding;
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
  p.batch = d.batch;
  p.frames = d.frames;
  p.max_tokens = d.max_tokens;
  const int smem = (int)sizeof(TdtSmem<T>) + 1024;
  int st = set_max_dynamic_smem(reinterpret_cast<const void*>(tdt_decoder_kernel<T>), smem);
  if (st != PK_OK) return st;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = TCL;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3((unsigned)(d.batch * TCL));
  cfg.blockDim = dim3(TTHREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cuda_error(cudaLaunchKernelEx(&cfg, tdt_decoder_kernel<T>, p), "tdt_decoder launch");
}

}  // namespace

int launch_tdt_decode(const DeviceCtx& dev, const pk_tdt_desc& d, cudaStream_t stream) {
  return d.precision == PK_FP16 ? launch_tdt_typed<__half>(dev, d, stream) : launch_tdt_typed<float>(dev, d, stream);
}

}  // namespace pk
