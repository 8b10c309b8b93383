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
// are advanced round by round so that a thread has N dependency chains in flight.
//
// Pipe balance.  The cipher is integer work only: per block 20 rotations, 20 xors and
// 32 adds.  Bitwise ops and funnel shifts issue to the ALU pipe; integer multiply-adds
// issue to the FMA pipe, which is otherwise idle here.  An add can be written as a
// multiply-add by a 1 the compiler cannot see (a kernel parameter), and a rotation as a
// 32x32->64-bit multiply by 2^r whose two halves, or-ed, are the rotated word; the xor
// that follows the rotation then takes the or for free in one three-input logic op.
// MixPolicy selects, per round, which rotations and adds take the FMA pipe.
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

// Constants passed as kernel parameters so that the compiler emits multiply-adds:
// one == 1 and pow2[r] == 2^r.  make_pipe_consts() fills them on the host.
struct PipeConsts {
  uint32_t one;
  uint32_t pow2[32];
};

inline PipeConsts make_pipe_consts() {
  PipeConsts c;
  c.one = 1u;
  for (int r = 0; r < 32; ++r) c.pow2[r] = 1u << r;
  return c;
}

// Per-round choices, bit q (q = 4 * step + round, 0..19) of each mask:
//   kWide  rotation as one 32x32->64 multiply (both halves from one instruction)
//   kPair  rotation as a low and a high 32-bit multiply (two instructions)
//   kMadd  the x0 += x1 of the round as a multiply-add
// kMaddInject: the key injections are multiply-adds.
template <unsigned kWide, unsigned kMadd, bool kMaddInject, unsigned kPair = 0u>
struct MixPolicy {
  static constexpr unsigned wide = kWide;
  static constexpr unsigned madd = kMadd;
  static constexpr unsigned pair = kPair;
  static constexpr bool madd_inject = kMaddInject;
};

// Funnel shifts and plain adds, left to the compiler's scheduling (the small kernels).
using DefaultMix = MixPolicy<0u, 0u, false>;

template <bool kMad>
__device__ __forceinline__ uint32_t add32(uint32_t a, uint32_t b, const PipeConsts& pc) {
  if constexpr (kMad) return a * pc.one + b;
  else return a + b;
}

// rotl(x1, R) ^ x0; kHow 0: funnel shift, 1: one wide multiply, 2: low and high multiplies
template <int R, int kHow>
__device__ __forceinline__ uint32_t rotxor(uint32_t x1, uint32_t x0, const PipeConsts& pc) {
  if constexpr (kHow == 1) {
    const uint64_t t = (uint64_t)x1 * pc.pow2[R];
    return ((uint32_t)t | (uint32_t)(t >> 32)) ^ x0;
  } else if constexpr (kHow == 2) {
    return ((x1 * pc.pow2[R]) | __umulhi(x1, pc.pow2[R])) ^ x0;
  } else {
    return __funnelshift_l(x1, x1, R) ^ x0;
  }
}

template <class Mix, int Q, int R, int N>
__device__ __forceinline__ void round_n(uint32_t (&x0)[N], uint32_t (&x1)[N], const PipeConsts& pc) {
  constexpr int how = ((Mix::wide >> Q) & 1u) ? 1 : (((Mix::pair >> Q) & 1u) ? 2 : 0);
#pragma unroll
  for (int j = 0; j < N; ++j) {
    x0[j] = add32<((Mix::madd >> Q) & 1u) != 0>(x0[j], x1[j], pc);
    x1[j] = rotxor<R, how>(x1[j], x0[j], pc);
  }
}

// Four rounds of step S over N blocks, round-major so the N chains interleave.
template <class Mix, int N, int S, int R0, int R1, int R2, int R3>
__device__ __forceinline__ void four_rounds(uint32_t (&x0)[N], uint32_t (&x1)[N],
                                            const PipeConsts& pc) {
  round_n<Mix, 4 * S + 0, R0>(x0, x1, pc);
  round_n<Mix, 4 * S + 1, R1>(x0, x1, pc);
  round_n<Mix, 4 * S + 2, R2>(x0, x1, pc);
  round_n<Mix, 4 * S + 3, R3>(x0, x1, pc);
}

template <class Mix, int N>
__device__ __forceinline__ void inject(uint32_t (&x0)[N], uint32_t (&x1)[N], uint32_t a,
                                       uint32_t b, const PipeConsts& pc) {
#pragma unroll
  for (int j = 0; j < N; ++j) {
    x0[j] = add32<Mix::madd_inject>(x0[j], a, pc);
    x1[j] = add32<Mix::madd_inject>(x1[j], b, pc);
  }
}

// N blocks in place: on entry x0/x1 hold the counters (c0, c1), on exit the cipher words.
template <int N, class Mix = DefaultMix>
__device__ __forceinline__ void threefry20(const KeySchedule& s, uint32_t (&x0)[N],
                                           uint32_t (&x1)[N], const PipeConsts& pc) {
  inject<Mix, N>(x0, x1, s.k0, s.k1, pc);
  four_rounds<Mix, N, 0, 13, 15, 26, 6>(x0, x1, pc);
  inject<Mix, N>(x0, x1, s.a[0], s.b[0], pc);
  four_rounds<Mix, N, 1, 17, 29, 16, 24>(x0, x1, pc);
  inject<Mix, N>(x0, x1, s.a[1], s.b[1], pc);
  four_rounds<Mix, N, 2, 13, 15, 26, 6>(x0, x1, pc);
  inject<Mix, N>(x0, x1, s.a[2], s.b[2], pc);
  four_rounds<Mix, N, 3, 17, 29, 16, 24>(x0, x1, pc);
  inject<Mix, N>(x0, x1, s.a[3], s.b[3], pc);
  four_rounds<Mix, N, 4, 13, 15, 26, 6>(x0, x1, pc);
  inject<Mix, N>(x0, x1, s.a[4], s.b[4], pc);
}

// Plain form for code with no PipeConsts at hand (small kernels): DefaultMix only uses
// funnel shifts and adds, so the constants are never read.
template <int N>
__device__ __forceinline__ void threefry20(const KeySchedule& s, uint32_t (&x0)[N],
                                           uint32_t (&x1)[N]) {
  PipeConsts unused;
  threefry20<N, DefaultMix>(s, x0, x1, unused);
}

}  // namespace jxr
