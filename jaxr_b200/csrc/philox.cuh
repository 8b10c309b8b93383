// XLA's RngBitGenerator as the rbg and unsafe_rbg key implementations use it
// (R/prng.R:264-426 lowers lax_rng_bit_generator to stablehlo.rng_bit_generator with the
// default algorithm, which XLA's CPU backend runs as Philox4x32-10).
//
// Philox4x32-10 is J. K. Salmon, M. A. Moraes, R. O. Dror and D. E. Shaw, "Parallel random
// numbers: as easy as 1, 2, 3" (SC'11): ten rounds of two 32x32 -> 64-bit multiplies
// (0xD2511F53, 0xCD9E8D57) mixed by xors with the key, the key bumped by the Weyl constants
// (0x9E3779B9, 0xBB67AE85) after each round.  How XLA feeds it, pinned by the reference's
// recorded rbg / unsafe_rbg values (tests/testthat/test-prng.R:48-54): the u32[4] key
// (k0, k1, k2, k3) gives the Philox key (k0, k1) and the 128-bit counter
// k0 | k1 << 32 | k2 << 64 | k3 << 96; block b (counter + b) yields outputs 4b .. 4b+3 of
// a 32-bit request.  8- and 16-bit requests take the low bits of one 32-bit output per
// element; 64-bit requests take two outputs per element (low word first), an arrangement
// the recorded values do not cover.
#pragma once

#include <cstdint>

namespace jxr {

struct PhiloxOut {
  uint32_t w[4];
};

__device__ __forceinline__ PhiloxOut philox4x32_10(uint32_t c0, uint32_t c1, uint32_t c2,
                                                   uint32_t c3, uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t lo0 = 0xD2511F53u * c0, hi0 = __umulhi(0xD2511F53u, c0);
    const uint32_t lo1 = 0xCD9E8D57u * c2, hi1 = __umulhi(0xCD9E8D57u, c2);
    const uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
    c0 = n0;
    c1 = lo1;
    c2 = n2;
    c3 = lo0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  PhiloxOut o;
  o.w[0] = c0;
  o.w[1] = c1;
  o.w[2] = c2;
  o.w[3] = c3;
  return o;
}

// block b of the stream of key (q0, q1, q2, q3): counter (q as 128 bits) + b
__device__ __forceinline__ PhiloxOut rbg_block(const uint32_t q[4], uint64_t b) {
  const uint64_t lo = ((uint64_t)q[1] << 32 | q[0]);
  const uint64_t hi = ((uint64_t)q[3] << 32 | q[2]);
  const uint64_t l2 = lo + b;
  const uint64_t h2 = hi + (l2 < lo ? 1u : 0u);
  return philox4x32_10((uint32_t)l2, (uint32_t)(l2 >> 32), (uint32_t)h2, (uint32_t)(h2 >> 32),
                       q[0], q[1]);
}

}  // namespace jxr
