// fault_probe.cu -- pk_debug_wait_probe: makes one of the library's bounded
// device waits run out, on purpose and safely, so a test can check that the
// wait gives up after its limit, reports PK_E_TIMEOUT through the device status
// word and leaves the CUDA context usable.
//
// The waits are the production helpers of pk_common.cuh (mbar_wait_for, the
// loop behind every mbarrier wait of the GEMM, attention and decoder kernels;
// grid_arrive_wait, the resident decoder's grid barrier), called with a short
// limit instead of PK_WAIT_NS.  What never arrives is plain: an mbarrier that
// no thread arrives on, or a CTA of a cooperative launch that returns before
// the barrier.  Nothing traps, faults or spins without a bound; no copy is in
// flight and no TMEM is held when a probe gives up, so it simply returns.
#include "pk_common.cuh"
#include "pk_internal.h"

namespace pk {
namespace {

// kinds of pk_debug_wait_probe
constexpr int kMbarComplete = 0;  // a producer warp arrives: the wait completes
constexpr int kMbarNever = 1;     // nothing arrives: the wait runs out
constexpr int kGridComplete = 2;  // both CTAs reach the grid barrier
constexpr int kGridNever = 3;     // CTA 1 returns before it: CTA 0's wait runs out

// One CTA, two warps: warp 1 waits on a one-arrival mbarrier, warp 0 is the
// producer that arrives (kMbarComplete) or never does (kMbarNever).
__global__ void __launch_bounds__(64) mbar_probe_kernel(int kind, uint64_t limit_ns, unsigned int* status) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0 && kind == kMbarComplete) mbar_arrive(&bar);
  if (threadIdx.x == 32) mbar_wait_for(&bar, 0, &abort_flag, status, PK_STATUS_TIMEOUT_TMA, limit_ns);
  __syncthreads();
}

// Cooperative launch of two CTAs; thread 0 of each takes the grid barrier,
// except CTA 1 under kGridNever, which returns first.
__global__ void __launch_bounds__(32) grid_probe_kernel(int kind, uint64_t limit_ns, unsigned int* sync,
                                                        unsigned int* status) {
  if (kind == kGridNever && blockIdx.x == 1) return;
  if (threadIdx.x == 0) grid_arrive_wait(sync, sync + 1, gridDim.x, status, PK_STATUS_TIMEOUT_GRID, limit_ns);
  __syncwarp();
}

}  // namespace
}  // namespace pk

using namespace pk;

extern "C" int pk_debug_wait_probe(pk_device* device, int kind, uint32_t limit_ms, pk_stream stream) {
  if (!device) return set_error(PK_E_INVALID, "null device");
  if (device->closed) return set_error(PK_E_DESTROYED, "device handle is closed");
  if (kind < kMbarComplete || kind > kGridNever) return set_error(PK_E_INVALID, "unknown probe kind %d", kind);
  if (limit_ms < 1 || limit_ms > 2000) return set_error(PK_E_INVALID, "probe limit must be 1..2000 ms");
  cudaSetDevice(device->ctx.ordinal);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint64_t limit_ns = uint64_t(limit_ms) * 1000000ull;
  cudaError_t e;
  if (kind <= kMbarNever) {
    mbar_probe_kernel<<<1, 64, 0, s>>>(kind, limit_ns, device->ctx.status);
    if ((e = cudaGetLastError()) != cudaSuccess) return cuda_error(e, "wait probe launch");
    return cuda_error(cudaStreamSynchronize(s), "wait probe");
  }
  int coop = 0;
  cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, device->ctx.ordinal);
  if (!coop) return set_error(PK_E_SHAPE, "device has no cooperative launch");
  unsigned int* sync = nullptr;  // barrier counter, abort flag
  if ((e = cudaMalloc(&sync, 2 * sizeof(unsigned int))) != cudaSuccess) return cuda_error(e, "probe counter");
  if ((e = cudaMemsetAsync(sync, 0, 2 * sizeof(unsigned int), s)) != cudaSuccess) {
    cudaFree(sync);
    return cuda_error(e, "probe counter reset");
  }
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.gridDim = dim3(2);
  cfg.blockDim = dim3(32);
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, grid_probe_kernel, kind, limit_ns, sync, device->ctx.status);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  cudaFree(sync);
  return cuda_error(e, "grid wait probe");
}
