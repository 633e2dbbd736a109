// Host-only check of the TMA descriptor cache's key (csrc/tmap_cache.h):
// buffers that differ in any field of the descriptor tuple get distinct keys,
// including pairs whose fields a bit-mixing key (pointer XOR shifted sizes)
// would fold onto the same 64-bit value.  Built and run by
// tests/test_native_cpu.py with g++; needs the CUDA headers, not a GPU.
#include <cstdio>
#include <cstdint>

#include "tmap_cache.h"

static uint64_t folded(uint64_t ptr, uint64_t nb, uint64_t kvh, uint64_t bs, uint64_t hd) {
  return ptr ^ (nb << 40) ^ (bs << 32) ^ (hd << 24) ^ (kvh << 48);
}

int main() {
  using pse::TmapKey;
  int fails = 0;
  // pool A: 1000 blocks; pool B: 1001 blocks at an address chosen so the
  // folded keys agree.
  const uint64_t pa = 0x7f0000000000ull, nba = 1000, nbb = 1001, kvh = 8, bs = 16, hd = 64;
  const uint64_t pb = pa ^ ((nba ^ nbb) << 40);
  if (folded(pa, nba, kvh, bs, hd) != folded(pb, nbb, kvh, bs, hd)) {
    std::printf("setup: folded keys differ\n");
    return 2;
  }
  const TmapKey ka{pa, hd, nba * kvh * bs, hd * 2, 64, (uint32_t)bs, 128};
  const TmapKey kb{pb, hd, nbb * kvh * bs, hd * 2, 64, (uint32_t)bs, 128};
  if (ka == kb) { std::printf("colliding pools share a key\n"); ++fails; }
  // one field at a time
  TmapKey k = ka;
  uint64_t* f64[4] = {&k.ptr, &k.inner, &k.outer, &k.stride};
  for (auto* f : f64) { const uint64_t o = *f; *f ^= 16; if (k == ka) { std::printf("64-bit field ignored\n"); ++fails; } *f = o; }
  uint32_t* f32[3] = {&k.box_inner, &k.box_outer, &k.swizzle};
  for (auto* f : f32) { const uint32_t o = *f; *f ^= 1; if (k == ka) { std::printf("32-bit field ignored\n"); ++fails; } *f = o; }
  if (!(k == ka) || pse::TmapKeyHash()(k) != pse::TmapKeyHash()(ka)) { std::printf("equal keys differ\n"); ++fails; }
  std::printf(fails ? "FAIL\n" : "OK\n");
  return fails ? 1 : 0;
}
