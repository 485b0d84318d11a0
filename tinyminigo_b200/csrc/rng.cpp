// The uniform draws of the reference's sampler: rand 0.10.2's StdRng is a
// ChaCha12 generator (chacha20 0.10.2 crate) keyed by
// SeedableRng::seed_from_u64 (rand_core 0.10.1: eight PCG32 outputs,
// little-endian, form the 256-bit key; block counter and stream start at 0),
// and StandardUniform for f32 maps one u32 to (u >> 8) * 2^-24 in [0, 1).
// One draw per sampled step (src/tensor.rs:1204, src/model.rs:629).
#include <cstring>

#include "loader.h"

namespace tmg {

namespace {

inline uint32_t rotl32(uint32_t v, int c) { return (v << c) | (v >> (32 - c)); }

inline void quarter(uint32_t* s, int a, int b, int c, int d) {
  s[a] += s[b]; s[d] = rotl32(s[d] ^ s[a], 16);
  s[c] += s[d]; s[b] = rotl32(s[b] ^ s[c], 12);
  s[a] += s[b]; s[d] = rotl32(s[d] ^ s[a], 8);
  s[c] += s[d]; s[b] = rotl32(s[b] ^ s[c], 7);
}

struct ChaCha12 {
  uint32_t key[8];
  uint64_t block = 0;
  uint32_t out[16];
  int used = 16;

  explicit ChaCha12(uint64_t seed) {
    // PCG32 key expansion
    for (int i = 0; i < 8; ++i) {
      seed = seed * 6364136223846793005ull + 11634580027462260723ull;
      const uint32_t xorshifted = uint32_t(((seed >> 18) ^ seed) >> 27);
      const uint32_t rot = uint32_t(seed >> 59);
      key[i] = (xorshifted >> rot) | (xorshifted << ((32u - rot) & 31u));
    }
  }
  void next_block() {
    const uint32_t init[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u,
                               key[0], key[1], key[2], key[3], key[4], key[5], key[6], key[7],
                               uint32_t(block), uint32_t(block >> 32), 0u, 0u};
    uint32_t s[16];
    std::memcpy(s, init, sizeof(s));
    for (int dr = 0; dr < 6; ++dr) {  // 12 rounds
      quarter(s, 0, 4, 8, 12);
      quarter(s, 1, 5, 9, 13);
      quarter(s, 2, 6, 10, 14);
      quarter(s, 3, 7, 11, 15);
      quarter(s, 0, 5, 10, 15);
      quarter(s, 1, 6, 11, 12);
      quarter(s, 2, 7, 8, 13);
      quarter(s, 3, 4, 9, 14);
    }
    for (int i = 0; i < 16; ++i) out[i] = s[i] + init[i];
    ++block;
    used = 0;
  }
  uint32_t next_u32() {
    if (used == 16) next_block();
    return out[used++];
  }
};

}  // namespace

void stdrng_uniforms(uint64_t seed, int64_t n, float* out) {
  ChaCha12 g(seed);
  for (int64_t i = 0; i < n; ++i) out[i] = float(g.next_u32() >> 8) * (1.0f / 16777216.0f);
}

}  // namespace tmg
