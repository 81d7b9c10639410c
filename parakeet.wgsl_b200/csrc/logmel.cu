// logmel.cu -- log-mel front end on the GPU, replaying the reference's
// native front end (src/cpp/fbank/parakeet_fbank.cpp) operation for operation:
// 16 kHz f32 PCM, hop 160, centered 512-point frames holding a 400-sample
// Hann window (periodic = false), preemphasis 0.97 in double inside each
// frame, a radix-2 decimation-in-time FFT in f32 on bit-reversed input (the
// first butterfly of every block without a twiddle), power in double, 128
// Slaney mel filters summed in double in bin order, log(energy + 2^-24) in
// double, then per-window, per-bin normalization over the valid frames
// (unbiased standard deviation + 1e-5) with zeros beyond them.
//
// Every f32 / f64 operation is an explicit round-to-nearest intrinsic so the
// compiler cannot contract a multiply and an add into one FMA (the reference
// runs as WebAssembly, which has no contraction).  The tables (window,
// twiddles, mel weights) are computed on the host with the reference's
// double-precision formulas and live in a device-global table, uploaded once per
// device by the first call on it (make that call before any stream capture).
//
// Kernel 1 (raw): each warp takes 16 consecutive frames, one at a time:
// window + preemphasis into shared memory, nine butterfly stages (8
// butterflies per lane per stage, twiddles from a per-CTA shared copy), power,
// four mel bins per lane, log; raw values go straight into the output buffer.
// Kernel 2 (normalize): one warp per (window, mel bin) row: the row is staged
// in shared memory, lane 0 forms the mean and deviation sums in frame order
// (the reference's order), all lanes write the normalized row and the zero
// tail.
#include <cuda_runtime.h>

#include <cmath>
#include <cstring>
#include <mutex>

#include "pk_common.cuh"
#include "pk_internal.h"

namespace pk {
namespace {

constexpr int LFFT = 512;
constexpr int LBINS = LFFT / 2 + 1;
constexpr int LWIN = 400;
constexpr int LHOP = 160;
constexpr int LMELS = 128;
constexpr int LSR = 16000;
constexpr int LMAX_SAMPLES = 240000;
constexpr int LMAX_FRAMES = LMAX_SAMPLES / LHOP + 1;  // 1501
constexpr int LWEIGHTS = 640;                         // packed nonzero mel weights (504 used)
constexpr int RAW_WARPS = 4;
constexpr int RAW_FRAMES_PER_WARP = 16;  // the CTA's staged tables serve 64 frames
constexpr int NORM_WARPS = 4;
constexpr double LPI = 3.14159265358979323846264338327950288;

struct LogmelTables {
  float hann[LFFT];
  float tw_re[LFFT / 2];
  float tw_im[LFFT / 2];
  unsigned short rev[LFFT];
  unsigned short first[LMELS];
  unsigned short count[LMELS];
  unsigned short offset[LMELS];
  float weights[LWEIGHTS];
};

// Global (not constant) memory: lanes index the tables at different
// positions, which the constant cache would serialise.
__device__ LogmelTables g_lm;

// Host tables from the reference's formulas (parakeet_fbank.cpp:85-186).
bool build_tables(LogmelTables* t) {
  std::memset(t, 0, sizeof(*t));
  for (int i = 0; i < LWIN; ++i)
    t->hann[(LFFT - LWIN) / 2 + i] =
        static_cast<float>(0.5 * (1.0 - std::cos((2.0 * LPI * static_cast<double>(i)) / static_cast<double>(LWIN - 1))));
  for (int i = 0; i < LFFT / 2; ++i) {
    const double ph = (-2.0 * LPI * static_cast<double>(i)) / static_cast<double>(LFFT);
    t->tw_re[i] = static_cast<float>(std::cos(ph));
    t->tw_im[i] = static_cast<float>(std::sin(ph));
  }
  for (int i = 0; i < LFFT; ++i) {
    int r = 0;
    for (int b = 0; b < 9; ++b) r |= ((i >> b) & 1) << (8 - b);
    t->rev[i] = static_cast<unsigned short>(r);
  }
  const double lin = 200.0 / 3.0, f_t = 1000.0, m_t = f_t / lin, step = 0.06875177742094912;
  auto to_mel = [&](double f) { return f >= f_t ? m_t + std::log(f / f_t) / step : f / lin; };
  auto to_hz = [&](double m) { return m >= m_t ? f_t * std::exp(step * (m - m_t)) : m * lin; };
  double freq[LBINS], pts[LMELS + 2];
  for (int b = 0; b < LBINS; ++b) freq[b] = (static_cast<double>(LSR) * 0.5 * b) / static_cast<double>(LBINS - 1);
  const double m0 = to_mel(0.0), m1 = to_mel(LSR * 0.5);
  for (int i = 0; i < LMELS + 2; ++i) pts[i] = to_hz(m0 + (m1 - m0) * i / (LMELS + 1));
  int n = 0;
  for (int m = 0; m < LMELS; ++m) {
    const double norm = 2.0 / (pts[m + 2] - pts[m]);
    float w[LBINS];
    int first = -1, last = -1;
    for (int b = 0; b < LBINS; ++b) {
      const double down = (freq[b] - pts[m]) / (pts[m + 1] - pts[m]);
      const double up = (pts[m + 2] - freq[b]) / (pts[m + 2] - pts[m + 1]);
      double tri = down < up ? down : up;
      if (tri < 0.0) tri = 0.0;
      w[b] = static_cast<float>(tri * norm);
      if (w[b] > 0.0f) {
        if (first < 0) first = b;
        last = b;
      }
    }
    const int cnt = first < 0 ? 0 : last - first + 1;
    if (n + cnt > LWEIGHTS) return false;
    t->first[m] = static_cast<unsigned short>(first < 0 ? 0 : first);
    t->count[m] = static_cast<unsigned short>(cnt);
    t->offset[m] = static_cast<unsigned short>(n);
    for (int b = 0; b < cnt; ++b) t->weights[n++] = w[first + b];
  }
  return true;
}

int ensure_tables() {
  static std::mutex mu;
  static bool ready[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_error(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return set_error(PK_E_INVALID, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (ready[dev]) return PK_OK;
  static LogmelTables host;
  static bool built = false;
  if (!built) {
    if (!build_tables(&host)) return set_error(PK_E_INVALID, "mel filterbank has more weights than its table");
    built = true;
  }
  if ((e = cudaMemcpyToSymbol(g_lm, &host, sizeof(host))) != cudaSuccess)
    return cuda_error(e, "uploading the log-mel tables");
  ready[dev] = true;
  return PK_OK;
}

__global__ void __launch_bounds__(RAW_WARPS * 32) logmel_raw_kernel(const float* __restrict__ samples,
                                                                     const uint32_t* __restrict__ valid,
                                                                     float* __restrict__ features, int sample_count,
                                                                     int frames) {
  pdl_entry();
  __shared__ float s_re[RAW_WARPS][LFFT];
  __shared__ float s_im[RAW_WARPS][LFFT];
  __shared__ double s_pw[RAW_WARPS][LBINS + 1];
  __shared__ float s_hann[LFFT];
  __shared__ float s_twr[LFFT / 2];
  __shared__ float s_twi[LFFT / 2];
  __shared__ unsigned short s_rev[LFFT];
  for (int i = threadIdx.x; i < LFFT; i += blockDim.x) {
    s_hann[i] = g_lm.hann[i];
    s_rev[i] = g_lm.rev[i];
    if (i < LFFT / 2) {
      s_twr[i] = g_lm.tw_re[i];
      s_twi[i] = g_lm.tw_im[i];
    }
  }
  __syncthreads();
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int b = blockIdx.y;
  const int n = (int)min(valid[b], (uint32_t)sample_count);
  const int nf = n / LHOP;  // frames beyond the valid count are written by the normalization
  float* re = s_re[warp];
  float* im = s_im[warp];
  double* pw = s_pw[warp];
  const float* x = samples + (size_t)b * sample_count;
  const double pre = static_cast<double>(0.97f);
  const int t0 = (blockIdx.x * RAW_WARPS + warp) * RAW_FRAMES_PER_WARP;
  const int t1 = min(t0 + RAW_FRAMES_PER_WARP, nf);
  for (int t = t0; t < t1; ++t) {
    for (int i = lane; i < LFFT; i += 32) {
      re[i] = 0.0f;
      im[i] = 0.0f;
    }
    __syncwarp();
    const int center = t * LHOP;
    const int lo = max(0, center - LWIN / 2), hi = min(n, center + LWIN / 2);
    for (int src = lo + lane; src < hi; src += 32) {
      const double e = src == 0 ? static_cast<double>(x[0])
                                : __dsub_rn(static_cast<double>(x[src]), __dmul_rn(pre, static_cast<double>(x[src - 1])));
      const int fi = src - center + LFFT / 2;
      re[s_rev[fi]] = __double2float_rn(__dmul_rn(e, static_cast<double>(s_hann[fi])));
    }
    __syncwarp();
#pragma unroll 1
    for (int len = 2; len <= LFFT; len <<= 1) {
      const int half = len >> 1, step = LFFT / len;
#pragma unroll
      for (int k = 0; k < LFFT / 2 / 32; ++k) {
        const int i = lane + 32 * k;                 // butterfly index in [0, 256)
        const int j = i & (half - 1);
        const int l = (i - j) * 2 + j, r = l + half;  // block (i / half) * len, lane j
        const float rr = re[r], ri = im[r], lr = re[l], li = im[l];
        float xr, xi;
        if (j == 0) {
          xr = rr;
          xi = ri;
        } else {
          const float wr = s_twr[j * step], wi = s_twi[j * step];
          xr = __fsub_rn(__fmul_rn(wr, rr), __fmul_rn(wi, ri));
          xi = __fadd_rn(__fmul_rn(wr, ri), __fmul_rn(wi, rr));
        }
        re[l] = __fadd_rn(lr, xr);
        im[l] = __fadd_rn(li, xi);
        re[r] = __fsub_rn(lr, xr);
        im[r] = __fsub_rn(li, xi);
      }
      __syncwarp();
    }
    for (int k = lane; k < LBINS; k += 32) {
      const double a = static_cast<double>(re[k]), c = static_cast<double>(im[k]);
      pw[k] = __dadd_rn(__dmul_rn(a, a), __dmul_rn(c, c));
    }
    __syncwarp();
#pragma unroll
    for (int q = 0; q < LMELS / 32; ++q) {
      const int m = lane + 32 * q;
      const int f0 = g_lm.first[m], cnt = g_lm.count[m], off = g_lm.offset[m];
      double en = 0.0;
      for (int k = 0; k < cnt; ++k)
        en = __dadd_rn(en, __dmul_rn(static_cast<double>(__ldg(&g_lm.weights[off + k])), pw[f0 + k]));
      features[((size_t)b * LMELS + m) * frames + t] = __double2float_rn(log(__dadd_rn(en, 1.0 / 16777216.0)));
    }
    __syncwarp();  // the next frame reuses this warp's buffers
  }
}

__global__ void __launch_bounds__(NORM_WARPS * 32) logmel_normalize_kernel(const uint32_t* __restrict__ valid,
                                                                           float* __restrict__ features,
                                                                           int sample_count, int frames) {
  pdl_entry();
  __shared__ float s_row[NORM_WARPS][LMAX_FRAMES + 3];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int m = blockIdx.x * NORM_WARPS + warp;
  const int b = blockIdx.y;
  const int nf = (int)min(valid[b], (uint32_t)sample_count) / LHOP;
  float* row = features + ((size_t)b * LMELS + m) * frames;
  float* sr = s_row[warp];
  for (int t = lane; t < nf; t += 32) sr[t] = row[t];
  __syncwarp();
  double mean = 0.0, inv = 0.0;
  if (lane == 0) {
    double sum = 0.0;
    for (int t = 0; t < nf; ++t) sum = __dadd_rn(sum, static_cast<double>(sr[t]));
    mean = nf > 0 ? __ddiv_rn(sum, static_cast<double>(nf)) : 0.0;
    double sq = 0.0;
    for (int t = 0; t < nf; ++t) {
      const double d = __dsub_rn(static_cast<double>(sr[t]), mean);
      sq = __dadd_rn(sq, __dmul_rn(d, d));
    }
    const double sd = nf > 1 ? __dsqrt_rn(__ddiv_rn(sq, static_cast<double>(nf - 1))) : 0.0;
    inv = __ddiv_rn(1.0, __dadd_rn(sd, 1.0e-5));
  }
  mean = __shfl_sync(0xffffffffu, mean, 0);
  inv = __shfl_sync(0xffffffffu, inv, 0);
  for (int t = lane; t < frames; t += 32)
    row[t] = t < nf ? __double2float_rn(__dmul_rn(__dsub_rn(static_cast<double>(sr[t]), mean), inv)) : 0.0f;
}

}  // namespace

int launch_logmel(int batch, int sample_count, const float* samples, const uint32_t* valid_samples, float* features,
                  cudaStream_t stream) {
  int st = ensure_tables();
  if (st != PK_OK) return st;
  const int frames = sample_count / LHOP + 1;
  const int raw_blocks = (frames + RAW_WARPS * RAW_FRAMES_PER_WARP - 1) / (RAW_WARPS * RAW_FRAMES_PER_WARP);
  cudaError_t e = launch_kernel(logmel_raw_kernel, dim3(raw_blocks, batch), dim3(RAW_WARPS * 32), 0, stream, samples,
                                valid_samples, features, sample_count, frames);
  if (e != cudaSuccess) return cuda_error(e, "logmel_raw launch");
  e = launch_kernel(logmel_normalize_kernel, dim3(LMELS / NORM_WARPS, batch), dim3(NORM_WARPS * 32), 0, stream,
                    valid_samples, features, sample_count, frames);
  return cuda_error(e, "logmel_normalize launch");
}

}  // namespace pk
