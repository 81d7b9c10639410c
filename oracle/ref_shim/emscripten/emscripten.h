/* Host build of the reference's Emscripten sources (test infrastructure):
 * EMSCRIPTEN_KEEPALIVE only has to export the symbol from a shared object. */
#pragma once
#define EMSCRIPTEN_KEEPALIVE __attribute__((visibility("default"), used))
