/* Host build of the reference's Emscripten sources (test infrastructure): the
 * few WebAssembly SIMD operations parakeet_fbank.cpp uses, as four IEEE f32
 * lanes.  wasm f32x4 add / sub / mul round each lane like the scalar
 * operations, and the recipe compiles with -ffp-contract=off, so each lane
 * computes what the wasm instruction computes. */
#pragma once
#include <cstring>

typedef struct {
  float lane[4];
} v128_t;

static inline v128_t wasm_v128_load(const void* p) {
  v128_t v;
  std::memcpy(v.lane, p, sizeof(v.lane));
  return v;
}
static inline void wasm_v128_store(void* p, v128_t v) { std::memcpy(p, v.lane, sizeof(v.lane)); }
static inline v128_t wasm_f32x4_splat(float x) { return v128_t{{x, x, x, x}}; }
static inline v128_t wasm_f32x4_add(v128_t a, v128_t b) {
  return v128_t{{a.lane[0] + b.lane[0], a.lane[1] + b.lane[1], a.lane[2] + b.lane[2], a.lane[3] + b.lane[3]}};
}
static inline v128_t wasm_f32x4_sub(v128_t a, v128_t b) {
  return v128_t{{a.lane[0] - b.lane[0], a.lane[1] - b.lane[1], a.lane[2] - b.lane[2], a.lane[3] - b.lane[3]}};
}
static inline v128_t wasm_f32x4_mul(v128_t a, v128_t b) {
  return v128_t{{a.lane[0] * b.lane[0], a.lane[1] * b.lane[1], a.lane[2] * b.lane[2], a.lane[3] * b.lane[3]}};
}
