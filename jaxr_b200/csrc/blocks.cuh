// k_blocks: one threefry block per output element, the bulk kernel of the
// partitionable layout (R/prng.R:212-227) and of the original layout's 64-bit draws
// (R/prng.R:246-251).
//
// Element i of a request hashes the counters
//   kCtrIndex  (i >> 32, i & 0xFFFFFFFF)   the C-order index split into two words
//   kCtrPair   (i, size + i)              original layout, 64 bits, size < 2^31
// and the op turns the cipher words into the stored value (bits, uniform, normal, ...).
//
// Work decomposition.  A CTA of 256 threads owns tiles of TILE = 256 * G * V elements,
// V = 16 / sizeof(Out) so that one thread-group of V elements is one 16-byte store;
// group g of thread t covers elements [tile + (g * 256 + t) * V, ... + V), so each warp
// store instruction writes 512 contiguous bytes.  The grid is one resident wave and
// strides over the tiles.  For a single key the tile's counter words are derived from
// per-tile uniform values: inside a tile that does not cross a multiple of 2^32 the
// high word is constant and the low word is base + immediate, so the cipher's integer
// pipe work is almost all the per-element cost.
#pragma once

#include <cstdint>
#include <type_traits>

#include "samplers.cuh"
#include "threefry.cuh"

namespace jxr {

constexpr int kThreads = 256;

// The pipe mix the bulk kernels use: round adds as multiply-adds on the FMA pipe,
// rotations and xors on the ALU pipe (the fastest mix measured on B200).
using ProductMix = MixPolicy<0u, 0xFFFFFu, false>;

enum { kCtrIndex = 0, kCtrPair = 1 };

// kBits == -1 stores the key pair (x0, x1) itself (split); otherwise W-bit draws:
// 64 bits are x0 << 32 | x1 (R/prng.R:220-224), narrower ones x0 ^ x1 truncated
// (R/prng.R:225-226).
template <int kBits>
struct Draw;
template <> struct Draw<64> {
  __device__ static uint64_t get(uint32_t x0, uint32_t x1) { return ((uint64_t)x0 << 32) | x1; }
};
template <> struct Draw<32> {
  __device__ static uint32_t get(uint32_t x0, uint32_t x1) { return x0 ^ x1; }
};
template <> struct Draw<16> {
  __device__ static uint16_t get(uint32_t x0, uint32_t x1) { return (uint16_t)(x0 ^ x1); }
};
template <> struct Draw<8> {
  __device__ static uint8_t get(uint32_t x0, uint32_t x1) { return (uint8_t)(x0 ^ x1); }
};

struct OpKeyPair {
  static constexpr int kBits = -1;
  using Out = uint64_t;  // little-endian: (x0, x1) in memory
};

template <class Op>
__device__ __forceinline__ typename Op::Out apply(const Op& op, uint32_t x0, uint32_t x1) {
  if constexpr (Op::kBits == -1) return ((uint64_t)x1 << 32) | x0;
  else return op(Draw<Op::kBits>::get(x0, x1));
}

// 16 bytes of outputs, stored as one vector
template <class T>
union Vec16 {
  static constexpr int N = 16 / sizeof(T);
  T v[N];
  uint4 u;
};

template <class Out>
__host__ __device__ constexpr int groups_for() {
  // blocks in flight per thread: G groups of 16 / sizeof(Out) outputs (16 blocks for 4-byte
  // outputs: 40 registers, 6 CTAs per SM, measured fastest on B200)
  return sizeof(Out) >= 4 ? 4 : (sizeof(Out) == 2 ? 2 : 1);
}

// An op may set kGroups (e.g. transform-heavy samplers, which need registers for the
// transform more than blocks in flight); otherwise groups_for<Out>.
template <class Op, class = void>
struct GroupsOf {
  static constexpr int value = groups_for<typename Op::Out>();
};
template <class Op>
struct GroupsOf<Op, std::void_t<decltype(Op::kGroups)>> {
  static constexpr int value = Op::kGroups;
};

__host__ __device__ __forceinline__ uint64_t umin(uint64_t a, uint64_t b) { return a < b ? a : b; }

// Ops with kDirect > 0 (OpTableHybridF32) evaluate the last kDirect of a thread's outputs
// per tile with op.direct and gather the rest from their table; others evaluate every
// output alike.
template <class Op, class = void>
struct DirectOutputsOf {
  static constexpr int value = 0;
};
template <class Op>
struct DirectOutputsOf<Op, std::void_t<decltype(Op::kDirect)>> {
  static constexpr int value = Op::kDirect;
};

// Ops with kBatch (the float64 normal) transform a thread's N draws at once (op.batch<N>)
// in the bulk kernels' full tiles; others one draw at a time.
template <class Op, class = void>
struct BatchOf {
  static constexpr bool value = false;
};
template <class Op>
struct BatchOf<Op, std::void_t<decltype(Op::kBatch)>> {
  static constexpr bool value = Op::kBatch;
};

// out[k] = the op's value of draw k, k < N, through op.batch where the op has it
template <int N, class Op>
__device__ __forceinline__ void apply_all(const Op& op, const uint32_t* x0, const uint32_t* x1,
                                          typename Op::Out* out) {
  if constexpr (BatchOf<Op>::value) {
    typename Op::Bits b[N];
#pragma unroll
    for (int k = 0; k < N; ++k) b[k] = Draw<Op::kBits>::get(x0[k], x1[k]);
    op.template batch<N>(b, out);
  } else {
#pragma unroll
    for (int k = 0; k < N; ++k) out[k] = apply(op, x0[k], x1[k]);
  }
}

template <class Op>
__device__ __forceinline__ typename Op::Out apply_direct(const Op& op, uint32_t x0, uint32_t x1) {
  if constexpr (DirectOutputsOf<Op>::value > 0) return op.direct(Draw<Op::kBits>::get(x0, x1));
  else return apply(op, x0, x1);
}

// ---- single key ---------------------------------------------------------------------------

template <class Op, int kCtr, class Mix = ProductMix, int G = GroupsOf<Op>::value>
__global__ void __launch_bounds__(kThreads)
    k_blocks_1key(const uint32_t* __restrict__ keys, uint64_t size, uint64_t begin,
                  uint64_t count, int vec_ok, Op op, PipeConsts pc,
                  typename Op::Out* __restrict__ out) {
  using Out = typename Op::Out;
  constexpr int V = 16 / sizeof(Out);
  constexpr int N = G * V;
  constexpr uint32_t TILE = (uint32_t)kThreads * G * V;
  const KeySchedule s = make_schedule(__ldg(keys), __ldg(keys + 1));
  const uint64_t ntiles = (count + TILE - 1) / TILE;
  const uint32_t toff = threadIdx.x * V;
  for (uint64_t t = blockIdx.x; t < ntiles; t += gridDim.x) {
    const uint64_t p0 = t * TILE;   // first output of the tile
    const uint64_t e0 = begin + p0; // its element index in the request
    uint32_t x0[N], x1[N];
    if (kCtr == kCtrIndex) {
      const uint32_t lo = (uint32_t)e0;
      if (lo <= 0xFFFFFFFFu - TILE) {  // the whole tile shares the high word
        const uint32_t hi = (uint32_t)(e0 >> 32), base = lo + toff;
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
          for (int v = 0; v < V; ++v) {
            x0[g * V + v] = hi;
            x1[g * V + v] = base + (uint32_t)(g * kThreads * V + v);
          }
      } else {
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
          for (int v = 0; v < V; ++v) {
            const uint64_t i = e0 + toff + (uint32_t)(g * kThreads * V + v);
            x0[g * V + v] = (uint32_t)(i >> 32);
            x1[g * V + v] = (uint32_t)i;
          }
      }
    } else {  // (i, size + i), all below 2^32
      const uint32_t a = (uint32_t)e0 + toff, b = (uint32_t)(size + e0) + toff;
#pragma unroll
      for (int g = 0; g < G; ++g)
#pragma unroll
        for (int v = 0; v < V; ++v) {
          x0[g * V + v] = a + (uint32_t)(g * kThreads * V + v);
          x1[g * V + v] = b + (uint32_t)(g * kThreads * V + v);
        }
    }
    threefry20<N, Mix>(s, x0, x1, pc);
    Out* dst = out + p0 + toff;
    constexpr int D = DirectOutputsOf<Op>::value;
    static_assert(D <= N, "direct outputs per thread");
    if (D > 0 && vec_ok && p0 + TILE <= count) {
      // the table gathers of outputs 0 .. N - D are issued first, the last D outputs are
      // computed while they are in flight, then all groups are stored
      Vec16<Out> r[G];
#pragma unroll
      for (int k = 0; k < N - D; ++k) r[k / V].v[k % V] = apply(op, x0[k], x1[k]);
#pragma unroll
      for (int k = N - D; k < N; ++k) r[k / V].v[k % V] = apply_direct(op, x0[k], x1[k]);
#pragma unroll
      for (int g = 0; g < G; ++g) *reinterpret_cast<uint4*>(dst + g * kThreads * V) = r[g].u;
    } else if (vec_ok && p0 + TILE <= count) {
      Out o[N];
      apply_all<N>(op, x0, x1, o);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        Vec16<Out> r;
#pragma unroll
        for (int v = 0; v < V; ++v) r.v[v] = o[g * V + v];
        *reinterpret_cast<uint4*>(dst + g * kThreads * V) = r.u;
      }
    } else {
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const uint64_t p = p0 + toff + (uint64_t)g * kThreads * V;
#pragma unroll
        for (int v = 0; v < V; ++v)
          if (p + v < count) out[p + v] = apply(op, x0[g * V + v], x1[g * V + v]);
      }
    }
  }
}

// ---- key batches (vmap): rows of `count` outputs, one key per row ---------------------------

// A warp owns tiles of WT = 32 * G * V consecutive outputs of one row, so the key schedule
// and the counters are per-warp values (as the single-key kernel's are per-CTA values);
// row and column advance by a fixed stride per iteration, with one division per thread at
// the start instead of one per tile.
template <class Op, int kCtr, class Mix = ProductMix, int G = GroupsOf<Op>::value>
__global__ void __launch_bounds__(kThreads)
    k_blocks_nkey(const uint32_t* __restrict__ keys, uint64_t size, uint64_t begin,
                  uint64_t count, uint64_t tiles_per_row, uint64_t ntiles, int vec_ok, Op op,
                  PipeConsts pc, typename Op::Out* __restrict__ out) {
  using Out = typename Op::Out;
  constexpr int V = 16 / sizeof(Out);
  constexpr int N = G * V;
  constexpr uint32_t WT = 32u * G * V;
  const uint32_t lane = threadIdx.x & 31u, loff = lane * V;
  const uint64_t w0 = ((uint64_t)blockIdx.x * kThreads + threadIdx.x) >> 5;
  const uint64_t nw = ((uint64_t)gridDim.x * kThreads) >> 5;
  if (w0 >= ntiles) return;
  uint64_t row = w0 / tiles_per_row, col = w0 - row * tiles_per_row;
  const uint64_t drow = nw / tiles_per_row, dcol = nw - drow * tiles_per_row;
  for (uint64_t w = w0; w < ntiles; w += nw) {
    const KeySchedule s = make_schedule(__ldg(keys + 2 * row), __ldg(keys + 2 * row + 1));
    const uint64_t p0 = col * WT;     // first output of the tile within its row
    const uint64_t e0 = begin + p0;   // its element index in the request
    uint32_t x0[N], x1[N];
    if (kCtr == kCtrIndex) {
      const uint32_t lo = (uint32_t)e0;
      if (lo <= 0xFFFFFFFFu - WT) {
        const uint32_t hi = (uint32_t)(e0 >> 32), base = lo + loff;
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
          for (int v = 0; v < V; ++v) {
            x0[g * V + v] = hi;
            x1[g * V + v] = base + (uint32_t)(g * 32 * V + v);
          }
      } else {
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
          for (int v = 0; v < V; ++v) {
            const uint64_t i = e0 + loff + (uint32_t)(g * 32 * V + v);
            x0[g * V + v] = (uint32_t)(i >> 32);
            x1[g * V + v] = (uint32_t)i;
          }
      }
    } else {
      const uint32_t a = (uint32_t)e0 + loff, b = (uint32_t)(size + e0) + loff;
#pragma unroll
      for (int g = 0; g < G; ++g)
#pragma unroll
        for (int v = 0; v < V; ++v) {
          x0[g * V + v] = a + (uint32_t)(g * 32 * V + v);
          x1[g * V + v] = b + (uint32_t)(g * 32 * V + v);
        }
    }
    threefry20<N, Mix>(s, x0, x1, pc);
    Out* orow = out + row * count;
    constexpr int D = DirectOutputsOf<Op>::value;
    static_assert(D <= N, "direct outputs per thread");
    if (D > 0 && vec_ok && p0 + WT <= count) {
      // as in k_blocks_1key: gathers first, the last D outputs computed meanwhile
      Vec16<Out> r[G];
#pragma unroll
      for (int k = 0; k < N - D; ++k) r[k / V].v[k % V] = apply(op, x0[k], x1[k]);
#pragma unroll
      for (int k = N - D; k < N; ++k) r[k / V].v[k % V] = apply_direct(op, x0[k], x1[k]);
#pragma unroll
      for (int g = 0; g < G; ++g)
        *reinterpret_cast<uint4*>(orow + p0 + loff + g * 32 * V) = r[g].u;
    } else if (vec_ok && p0 + WT <= count) {
      Out o[N];
      apply_all<N>(op, x0, x1, o);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        Vec16<Out> r;
#pragma unroll
        for (int v = 0; v < V; ++v) r.v[v] = o[g * V + v];
        *reinterpret_cast<uint4*>(orow + p0 + loff + g * 32 * V) = r.u;
      }
    } else {
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const uint64_t p = p0 + loff + (uint64_t)g * 32 * V;
#pragma unroll
        for (int v = 0; v < V; ++v)
          if (p + v < count) orow[p + v] = apply(op, x0[g * V + v], x1[g * V + v]);
      }
    }
    col += dcol;
    row += drow;
    if (col >= tiles_per_row) {
      col -= tiles_per_row;
      ++row;
    }
  }
}

}  // namespace jxr
