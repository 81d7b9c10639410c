// attention_noalloc.cu -- pk_rel_attention_noalloc: the FP16 relative-position
// attention for callers that cannot allocate device memory.
//
// Who needs it: hosts that hand this library buffers they manage themselves
// and forbid it from calling cudaMalloc -- an embedding runtime that owns a
// fixed device pool, a process that runs under a memory cap set by its
// scheduler, or a capture/replay harness that must see every allocation
// happen up front.  Such a caller cannot even open a pk_device (opening one
// allocates the device status word), so this entry point takes no handle and
// runs on the calling thread's current CUDA device.
//
// What it does: re-lays the package's head-vector-position-vec4 positions out
// row-major ([8][2T-1][128] f16) into a scratch array, then runs the tcgen05
// attention kernel (the one the encoder uses) on them.  The scratch is the
// file-scope device array below, not a runtime allocation: 256 bytes of
// status word followed by room for the positions of the longest window this
// path accepts (192 frames, 383 position rows): 784,640 bytes in all, held by
// every GPU that loads the library until the process exits.
//
// Rules a caller must know: every call shares the one array, so calls whose
// work overlaps on the GPU (two streams, two host threads) race on it --
// serialise them.  The first call on a device resolves the array's device
// address and the driver entry point it needs; make that first call before
// any stream capture.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "pk_internal.h"

namespace pk {
namespace {

constexpr int kNoAllocMaxFrames = 192;
constexpr size_t kNoAllocStatusBytes = 256;
constexpr size_t kNoAllocPositionBytes = (size_t)8 * (2 * kNoAllocMaxFrames - 1) * 128 * sizeof(__half);
constexpr size_t kNoAllocScratchBytes = kNoAllocStatusBytes + kNoAllocPositionBytes;
constexpr int kNoAllocMaxDevices = 64;

// Host code must not take this array's address directly (that is a host-side
// stand-in): it uses the address cudaGetSymbolAddress returns per device.
static __device__ __align__(256) unsigned char g_attention_scratch[kNoAllocScratchBytes];

struct NoAllocDevice {
  bool ready = false;
  DeviceCtx ctx;                       // sm count, shared-memory limit, tensor-map encoder, status word
  unsigned char* scratch = nullptr;    // device address of g_attention_scratch on this device
};

std::mutex g_noalloc_mu;
NoAllocDevice g_noalloc_devices[kNoAllocMaxDevices];

// Resolves, once per device and with that device current, everything the
// launch needs without allocating.
int noalloc_setup(NoAllocDevice** out) {
  int ordinal = 0;
  cudaError_t e = cudaGetDevice(&ordinal);
  if (e != cudaSuccess) return cuda_error(e, "cudaGetDevice");
  if (ordinal < 0 || ordinal >= kNoAllocMaxDevices)
    return set_error(PK_E_INVALID, "device ordinal %d is beyond the %d devices this entry point tracks", ordinal,
                     kNoAllocMaxDevices);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  NoAllocDevice& d = g_noalloc_devices[ordinal];
  if (!d.ready) {
    cudaDeviceProp prop;
    if ((e = cudaGetDeviceProperties(&prop, ordinal)) != cudaSuccess)
      return cuda_error(e, "cudaGetDeviceProperties");
    if (prop.major != 10)
      return set_error(PK_E_INVALID, "device %d is sm_%d%d; libpk_b200 targets sm_100a", ordinal, prop.major,
                       prop.minor);
    cudaDriverEntryPointQueryResult q;
    void* fn = nullptr;
    e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
      return set_error(PK_E_CUDA, "cuTensorMapEncodeTiled is unavailable");
    void* ptr = nullptr;
    if ((e = cudaGetSymbolAddress(&ptr, g_attention_scratch)) != cudaSuccess)
      return cuda_error(e, "cudaGetSymbolAddress(attention scratch)");
    d.ctx.ordinal = ordinal;
    d.ctx.sm_count = prop.multiProcessorCount;
    d.ctx.max_smem_optin = (int)prop.sharedMemPerBlockOptin;
    d.ctx.encode_tiled = fn;
    d.ctx.status = reinterpret_cast<unsigned int*>(ptr);
    d.scratch = static_cast<unsigned char*>(ptr);
    d.ready = true;
  }
  *out = &d;
  return PK_OK;
}

}  // namespace
}  // namespace pk

using namespace pk;

extern "C" int pk_rel_attention_noalloc(int batch, int frames, const void* qkv, const void* positions,
                                        const float* bias_u, const float* bias_v, const uint32_t* valid_lengths,
                                        void* context, uint32_t* wait_status, pk_stream stream) {
  if (!qkv || !positions || !bias_u || !bias_v || !valid_lengths || !context)
    return set_error(PK_E_INVALID, "null argument");
  if (batch <= 0 || batch > 65535 || frames <= 0 || frames > kNoAllocMaxFrames)
    return set_error(PK_E_SHAPE,
                     "Unsupported attention shape (batch=%d, frames=%d): the allocation-free attention holds "
                     "positions for at most %d frames",
                     batch, frames, kNoAllocMaxFrames);
  if (((reinterpret_cast<uintptr_t>(qkv) | reinterpret_cast<uintptr_t>(positions) |
        reinterpret_cast<uintptr_t>(context)) & 15) != 0)
    return set_error(PK_E_INVALID, "qkv, positions and context must be 16-byte aligned");
  NoAllocDevice* d = nullptr;
  int st = noalloc_setup(&d);
  if (st != PK_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The status word starts every call at zero; the positions region is fully
  // rewritten for this call's 2T-1 rows (the kernel never reads beyond them).
  cudaError_t e = cudaMemsetAsync(d->ctx.status, 0, sizeof(unsigned int), s);
  if (e != cudaSuccess) return cuda_error(e, "clearing the attention status word");
  void* positions_rm = d->scratch + kNoAllocStatusBytes;
  if ((st = launch_positions_rowmajor(positions, positions_rm, frames, s)) != PK_OK) return st;
  if ((st = launch_rel_attention_umma(d->ctx, batch, frames, qkv, positions_rm, bias_u, bias_v, valid_lengths,
                                      context, s)) != PK_OK)
    return st;
  if (wait_status) {
    unsigned int v = 0;
    if ((e = cudaMemcpyAsync(&v, d->ctx.status, sizeof(v), cudaMemcpyDeviceToHost, s)) != cudaSuccess)
      return cuda_error(e, "reading the attention status word");
    if ((e = cudaStreamSynchronize(s)) != cudaSuccess) return cuda_error(e, "cudaStreamSynchronize");
    *wait_status = v;
    if (v) return set_error(PK_E_TIMEOUT, "a bounded device wait expired (status bits 0x%x)", v);
  }
  return PK_OK;
}
