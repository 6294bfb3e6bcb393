// Restatement of rng.rs (SplitMix64-seeded xoshiro256++, 24-bit uniform, f32
// Box-Muller), used on the host to draw the reference's parameter
// initialisation bit for bit; the integer part (seeding, next_u64, uniform)
// also runs on the device, where the DropPath masks are drawn.
#pragma once

#include <math.h>
#include <stdint.h>

#ifdef __CUDACC__
#define RNN_HD __host__ __device__
#else
#define RNN_HD
#endif

namespace rnn {

struct Rng {
  uint64_t s[4];

  RNN_HD explicit Rng(uint64_t seed) {
    // rng.rs:8-20
    uint64_t z = seed + 0x9E3779B97F4A7C15ULL;
    for (int i = 0; i < 4; i++) {
      z += 0x9E3779B97F4A7C15ULL;
      uint64_t x = z;
      x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ULL;
      x = (x ^ (x >> 27)) * 0x94D049BB133111EBULL;
      s[i] = x ^ (x >> 31);
    }
  }

  static RNN_HD uint64_t rotl(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }

  RNN_HD uint64_t next_u64() {
    // rng.rs:23-36
    const uint64_t r = rotl(s[0] + s[3], 23) + s[0];
    const uint64_t t = s[1] << 17;
    s[2] ^= s[0];
    s[3] ^= s[1];
    s[1] ^= s[2];
    s[0] ^= s[3];
    s[2] ^= t;
    s[3] = rotl(s[3], 45);
    return r;
  }

  RNN_HD float uniform() { return (float)(next_u64() >> 40) * (1.0f / (float)(1ULL << 24)); }  // rng.rs:50-52

  float normal() {
    // rng.rs:55-59
    float u1 = uniform();
    if (u1 < 1e-7f) u1 = 1e-7f;
    const float u2 = uniform();
    return sqrtf(-2.0f * logf(u1)) * cosf(6.28318530717958647692f * u2);
  }
};

}  // namespace rnn
