// palette_expand.cu -- bit-exact palette expansion (diagnostic / parity path).
//
// Restates paletteDequantWgslForScalar (src/model/palette-expander.ts:478-587):
// one thread per packed code group (32 five-bit or 16 six-bit codes), LSB-first
// unpacking across u32 words, palette group = min(col / group_cols, G - 1)
// taken at the group's first scalar, and either a k-by-output row-major target
// or the n256/n128-k32 tile-major target of runtimeGemmTileMajorScalarIndex
// (src/model/runtime-plan.ts:454-490).  The GEMMs never call this: they decode
// on chip.  It exists so expansion can be checked bit-exactly and so callers
// of the reference's PaletteWeightExpander keep an equivalent.
#include "pk_common.cuh"
#include "pk_internal.h"

namespace pk {

template <typename T, int BITS, bool TILE>
__global__ void palette_expand_kernel(const uint32_t* __restrict__ codes, const T* __restrict__ palette,
                                      T* __restrict__ target, int64_t inner, int64_t columns, int groups,
                                      int64_t group_cols) {
  pdl_entry();
  constexpr int CPG = BITS == 5 ? 32 : 16, WPG = BITS == 5 ? 5 : 3, E = 1 << BITS;
  constexpr int64_t TILE_COLS = sizeof(T) == 2 ? 256 : 128;
  const int64_t group = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t base = group * CPG;
  if (base >= inner * columns) return;
  uint32_t w[WPG];
#pragma unroll
  for (int j = 0; j < WPG; ++j) w[j] = codes[group * WPG + j];
  const int64_t pg = min(base % columns / group_cols, (int64_t)groups - 1);
  const T* lut = palette + pg * E;
  const int64_t k = base / columns, n = base % columns;
#pragma unroll
  for (int c = 0; c < CPG; ++c) {
    const int bit = c * BITS, word = bit >> 5, sh = bit & 31;
    uint32_t v = w[word] >> sh;
    if (sh + BITS > 32) v |= w[word + 1] << (32 - sh);
    int64_t dst;
    if (TILE) {
      const int64_t nn = n + c;
      dst = (((nn / TILE_COLS) * (inner / 32) + k / 32) * 32 + k % 32) * TILE_COLS + nn % TILE_COLS;
    } else {
      dst = base + c;
    }
    target[dst] = lut[v & (E - 1)];
  }
}

template <typename T>
static void dispatch_expand(const pk_palette_desc& d, cudaStream_t s) {
  const int cpg = d.bits == 5 ? 32 : 16;
  const int64_t groups_total = d.inner * d.columns / cpg;
  const int threads = 256;
  const unsigned blocks = (unsigned)((groups_total + threads - 1) / threads);
  auto* codes = d.codes;
  auto* pal = static_cast<const T*>(d.palette);
  auto* tgt = static_cast<T*>(d.target);
  const bool tile = d.layout == PK_LAYOUT_TILE_MAJOR;
  if (d.bits == 5) {
    if (tile)
      launch_kernel(palette_expand_kernel<T, 5, true>, blocks, threads, 0, s, codes, pal, tgt, d.inner, d.columns,
                                                                 d.palette_groups, d.palette_group_columns);
    else
      launch_kernel(palette_expand_kernel<T, 5, false>, blocks, threads, 0, s, codes, pal, tgt, d.inner, d.columns,
                                                                  d.palette_groups, d.palette_group_columns);
  } else {
    if (tile)
      launch_kernel(palette_expand_kernel<T, 6, true>, blocks, threads, 0, s, codes, pal, tgt, d.inner, d.columns,
                                                                 d.palette_groups, d.palette_group_columns);
    else
      launch_kernel(palette_expand_kernel<T, 6, false>, blocks, threads, 0, s, codes, pal, tgt, d.inner, d.columns,
                                                                  d.palette_groups, d.palette_group_columns);
  }
}

int launch_palette_expand(const pk_palette_desc& d, cudaStream_t stream) {
  if (d.precision == PK_FP16) dispatch_expand<uint16_t>(d, stream);
  else dispatch_expand<float>(d, stream);
  return cuda_error(cudaGetLastError(), "palette_expand launch");
}

}  // namespace pk
