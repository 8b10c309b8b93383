// Threefry-2x32 with 20 rounds, the block cipher of jaxR's default PRNG
// (R/prng.R:51-86, the rolled-loop lowering of threefry2x32.py).
//
// One 64-bit block (c0, c1) -> (x0, x1) under key (k0, k1):
//   ks = (k0, k1, k0 ^ k1 ^ 0x1BD11BDA); x0 = c0 + ks0; x1 = c1 + ks1
//   5 steps of 4 rounds  x0 += x1; x1 = rotl(x1, r); x1 ^= x0
//   rotations (13, 15, 26, 6) and (17, 29, 16, 24) alternating, and after step i
//   x0 += ks[(i+1) % 3], x1 += ks[(i+2) % 3] + (i+1).
//
// Everything stays in registers.  The key schedule (including the step counters
// folded into the x1 injections) is hoisted once per key; N independent blocks
// are advanced round by round so that a thread has N dependency chains in
// flight; rotations are single funnel shifts.
#pragma once

#include <cstdint>

namespace jxr {

struct KeySchedule {
  uint32_t k0, k1;  // initial injection
  uint32_t a[5];    // added to x0 after step i: k1, k2, k0, k1, k2
  uint32_t b[5];    // added to x1 after step i: k2+1, k0+2, k1+3, k2+4, k0+5
};

__host__ __device__ __forceinline__ KeySchedule make_schedule(uint32_t k0, uint32_t k1) {
  const uint32_t k2 = k0 ^ k1 ^ 0x1BD11BDAu;
  KeySchedule s;
  s.k0 = k0;
  s.k1 = k1;
  s.a[0] = k1; s.a[1] = k2; s.a[2] = k0; s.a[3] = k1; s.a[4] = k2;
  s.b[0] = k2 + 1u; s.b[1] = k0 + 2u; s.b[2] = k1 + 3u; s.b[3] = k2 + 4u; s.b[4] = k0 + 5u;
  return s;
}

__device__ __forceinline__ uint32_t rotl(uint32_t x, int r) { return __funnelshift_l(x, x, r); }

// Four rounds of one step over N blocks, round-major so the N chains interleave.
template <int N, int R0, int R1, int R2, int R3>
__device__ __forceinline__ void four_rounds(uint32_t (&x0)[N], uint32_t (&x1)[N]) {
#pragma unroll
  for (int j = 0; j < N; ++j) { x0[j] += x1[j]; x1[j] = rotl(x1[j], R0) ^ x0[j]; }
#pragma unroll
  for (int j = 0; j < N; ++j) { x0[j] += x1[j]; x1[j] = rotl(x1[j], R1) ^ x0[j]; }
#pragma unroll
  for (int j = 0; j < N; ++j) { x0[j] += x1[j]; x1[j] = rotl(x1[j], R2) ^ x0[j]; }
#pragma unroll
  for (int j = 0; j < N; ++j) { x0[j] += x1[j]; x1[j] = rotl(x1[j], R3) ^ x0[j]; }
}

template <int N>
__device__ __forceinline__ void inject(uint32_t (&x0)[N], uint32_t (&x1)[N], uint32_t a,
                                       uint32_t b) {
#pragma unroll
  for (int j = 0; j < N; ++j) { x0[j] += a; x1[j] += b; }
}

// N blocks in place: on entry x0/x1 hold the counters (c0, c1), on exit the cipher words.
template <int N>
__device__ __forceinline__ void threefry20(const KeySchedule& s, uint32_t (&x0)[N],
                                           uint32_t (&x1)[N]) {
  inject<N>(x0, x1, s.k0, s.k1);
  four_rounds<N, 13, 15, 26, 6>(x0, x1);
  inject<N>(x0, x1, s.a[0], s.b[0]);
  four_rounds<N, 17, 29, 16, 24>(x0, x1);
  inject<N>(x0, x1, s.a[1], s.b[1]);
  four_rounds<N, 13, 15, 26, 6>(x0, x1);
  inject<N>(x0, x1, s.a[2], s.b[2]);
  four_rounds<N, 17, 29, 16, 24>(x0, x1);
  inject<N>(x0, x1, s.a[3], s.b[3]);
  four_rounds<N, 13, 15, 26, 6>(x0, x1);
  inject<N>(x0, x1, s.a[4], s.b[4]);
}

}  // namespace jxr
