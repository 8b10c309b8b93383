// jxrng: sm_100a kernels and the C ABI (include/jxrng.h) for jaxR's threefry2x32
// random-bits path.
//
// Two cipher kernels cover every request:
//   k_blocks  one cipher block per output element.  Counters are either the (hi, lo)
//             words of the element's C-order index (the partitionable layout,
//             R/prng.R:212-227, any bit width) or (i, size + i) (the original layout's
//             64-bit draws, R/prng.R:246-251).
//   k_words   the original layout's hash of iota(n) (R/prng.R:101-120, :229-262):
//             block j hashes (j, half + j) and yields words j and half + j, each
//             unpacked into 32 / W elements of W bits.
// Both fuse the sampler transform (samplers.cuh) into the same pass, keep each
// thread's blocks in registers, and write 16-byte vector stores that a warp
// issues as one contiguous 512-byte segment.  Grids are persistent: one wave of
// resident CTAs (a multiple of the SM count) strides over the work.
#include "jxrng.h"

#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <limits>
#include <mutex>
#include <type_traits>
#include <type_traits>
#include <string>
#include <vector>

#include "blocks.cuh"
#include "philox.cuh"
#include "samplers.cuh"
#include "sort.cuh"
#include "threefry.cuh"

namespace jxr {
namespace {

const PipeConsts kPipe = make_pipe_consts();


thread_local std::string g_error;

// jax_accurate_erf_inv for this host thread (jxr_set_accurate_erf_inv): which erf_inv the
// normal and truncated-normal samplers and jxr_erf_inv evaluate.
thread_local int g_accurate_erf_inv = 0;

// f(std::true_type{}) under the accurate erf_inv, else f(std::false_type{}): the variant
// becomes a compile-time constant of the kernel that f launches.
template <class F>
int with_erfinv(F&& f) {
  if (g_accurate_erf_inv) return f(std::true_type{});
  return f(std::false_type{});
}

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_error = buf;
  return code;
}

#define JXR_CUDA(expr)                                                                   \
  do {                                                                                   \
    cudaError_t e_ = (expr);                                                             \
    if (e_ != cudaSuccess) return fail(JXR_ERR_CUDA, "%s: %s", #expr, cudaGetErrorString(e_)); \
  } while (0)

struct DeviceInfo {
  int sms = 0;
  int major = 0;
};

int device_info(DeviceInfo* info) {
  static DeviceInfo cache[64];
  int dev = 0;
  JXR_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(JXR_ERR_NO_DEVICE, "device index %d out of range", dev);
  if (cache[dev].sms == 0) {
    int sms = 0, major = 0;
    JXR_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    JXR_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
    cache[dev].major = major;
    cache[dev].sms = sms;
  }
  *info = cache[dev];
  if (info->major != 10)
    return fail(JXR_ERR_NO_DEVICE, "device %d has compute capability %d.x; this library is built for sm_100a",
                dev, info->major);
  return JXR_OK;
}

// jxr_random_bits_host keeps, per device, two staging buffers of kStageBytes, a device
// copy of the keys, two non-blocking streams (generate, copy) and their events, created on
// the first call and reused by later calls (calls on one device are serialised).
constexpr size_t kStageBytes = 64ull << 20;

struct HostCopyCtx {
  std::mutex mu;
  bool ready = false;
  cudaStream_t gen = nullptr, cpy = nullptr;
  cudaEvent_t done[2] = {nullptr, nullptr}, freed[2] = {nullptr, nullptr};
  void* stage[2] = {nullptr, nullptr};
  uint32_t* dkeys = nullptr;
  size_t key_cap = 0;

  // Creates what is missing (a failed call leaves what it made for the next one to reuse).
  int ensure(size_t nkeys) {
    if (!ready) {
      if (!gen) JXR_CUDA(cudaStreamCreateWithFlags(&gen, cudaStreamNonBlocking));
      if (!cpy) JXR_CUDA(cudaStreamCreateWithFlags(&cpy, cudaStreamNonBlocking));
      for (int b = 0; b < 2; ++b) {
        if (!done[b]) JXR_CUDA(cudaEventCreateWithFlags(&done[b], cudaEventDisableTiming));
        if (!freed[b]) JXR_CUDA(cudaEventCreateWithFlags(&freed[b], cudaEventDisableTiming));
        if (!stage[b]) JXR_CUDA(cudaMalloc(&stage[b], kStageBytes));
      }
      ready = true;
    }
    if (key_cap < nkeys) {
      if (nkeys > (SIZE_MAX >> 3)) return fail(JXR_ERR_INVALID_ARGUMENT, "too many keys");
      if (dkeys) JXR_CUDA(cudaFree(dkeys));
      dkeys = nullptr;
      key_cap = 0;
      JXR_CUDA(cudaMalloc(&dkeys, 8 * nkeys));
      key_cap = nkeys;
    }
    return JXR_OK;
  }

  // Releases everything (the caller holds mu and the current device is this context's).
  void release() {
    for (int b = 0; b < 2; ++b) {
      if (stage[b]) cudaFree(stage[b]);
      if (done[b]) cudaEventDestroy(done[b]);
      if (freed[b]) cudaEventDestroy(freed[b]);
      stage[b] = nullptr;
      done[b] = freed[b] = nullptr;
    }
    if (dkeys) cudaFree(dkeys);
    if (gen) cudaStreamDestroy(gen);
    if (cpy) cudaStreamDestroy(cpy);
    dkeys = nullptr;
    gen = cpy = nullptr;
    key_cap = 0;
    ready = false;
  }
};

HostCopyCtx g_host_ctx[64];

// Resident CTAs per SM of each kernel, queried once per kernel (all devices this library
// runs on are sm_100, so the answer does not depend on the device).
std::mutex g_occ_mu;
std::vector<std::pair<const void*, int>> g_occ;

template <class K>
int resident_grid(K kernel, uint64_t work_ctas, int* grid) {
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  int per_sm = 0;
  {
    std::lock_guard<std::mutex> lock(g_occ_mu);
    for (const auto& e : g_occ)
      if (e.first == (const void*)kernel) per_sm = e.second;
    if (per_sm == 0) {
      JXR_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, 0));
      if (per_sm < 1) per_sm = 1;
      g_occ.emplace_back((const void*)kernel, per_sm);
    }
  }
  const uint64_t wave = (uint64_t)di.sms * (uint64_t)per_sm;
  *grid = (int)std::min<uint64_t>(std::max<uint64_t>(work_ctas, 1), wave);
  return JXR_OK;
}

template <class Op, int kCtr>
int launch_blocks(const uint32_t* keys, int64_t nkeys, uint64_t size, uint64_t begin,
                  uint64_t count, const Op& op, void* out, cudaStream_t st) {
  using Out = typename Op::Out;
  constexpr int V = 16 / sizeof(Out);
  constexpr int G = GroupsOf<Op>::value;
  if (count == 0 || nkeys == 0) return JXR_OK;
  int grid = 0, rc;
  if (nkeys == 1) {
    const int vec_ok = ((uintptr_t)out % 16 == 0);
    const uint64_t ntiles = (count + (uint64_t)kThreads * G * V - 1) / ((uint64_t)kThreads * G * V);
    auto k = k_blocks_1key<Op, kCtr>;
    if ((rc = resident_grid(k, ntiles, &grid))) return rc;
    k<<<grid, kThreads, 0, st>>>(keys, size, begin, count, vec_ok, op, kPipe, (Out*)out);
  } else {
    constexpr uint64_t WT = 32ull * G * V;
    const uint64_t tpr = (count + WT - 1) / WT;
    if (tpr > ~0ull / (uint64_t)nkeys) return fail(JXR_ERR_INVALID_ARGUMENT, "request too large");
    const uint64_t ntiles = tpr * (uint64_t)nkeys;
    const int vec_ok = ((uintptr_t)out % 16 == 0) && (count * sizeof(Out)) % 16 == 0;
    const uint64_t ctas = (ntiles + kThreads / 32 - 1) / (kThreads / 32);
    auto k = k_blocks_nkey<Op, kCtr>;
    if ((rc = resident_grid(k, ctas, &grid))) return rc;
    k<<<grid, kThreads, 0, st>>>(keys, size, begin, count, tpr, ntiles, vec_ok, op, kPipe,
                                 (Out*)out);
  }
  JXR_CUDA(cudaGetLastError());
  return JXR_OK;
}

// ---- k_words: the original layout's hash of iota(nwords) --------------------------------

template <class Op>
__host__ __device__ constexpr int words_per_thread() {
  // enough blocks that one slab chunk is a whole number of 16-byte vectors (>= 4 blocks)
  constexpr int per = Op::kBits > 0 ? 32 / Op::kBits : 1;
  constexpr int b = 16 / (per * (int)sizeof(typename Op::Out));
  return b > 4 ? b : 4;
}

// Word w (0 <= w < nwords) holds elements [w * per, w * per + per) of the request, in
// little-endian W-bit pieces (R/prng.R:252-260).  Block j hashes counts (j, half + j),
// the second count being the zero pad when half + j == nwords (R/prng.R:112-116).
template <class Op>
__global__ void __launch_bounds__(kThreads)
    k_words(const uint32_t* __restrict__ keys, uint64_t nwords, uint64_t half, uint64_t jlo,
            uint64_t jhi, uint64_t units_per_row, uint64_t nunits, uint64_t begin, uint64_t count,
            Op op, PipeConsts pc, typename Op::Out* __restrict__ out) {
  using Out = typename Op::Out;
  constexpr int B = words_per_thread<Op>();
  constexpr int W = Op::kBits;
  constexpr int per = 32 / W;
  const uint64_t end = begin + count;
  const uint64_t stride = (uint64_t)gridDim.x * kThreads;
  for (uint64_t u = (uint64_t)blockIdx.x * kThreads + threadIdx.x; u < nunits; u += stride) {
    const uint64_t row = u / units_per_row;
    const uint64_t j0 = jlo + (u - row * units_per_row) * B;
    const KeySchedule s = make_schedule(__ldg(keys + 2 * row), __ldg(keys + 2 * row + 1));
    uint32_t x0[B], x1[B];
#pragma unroll
    for (int b = 0; b < B; ++b) {
      const uint64_t j = j0 + b;
      x0[b] = (uint32_t)j;
      x1[b] = half + j < nwords ? (uint32_t)(half + j) : 0u;
    }
    threefry20<B, ProductMix>(s, x0, x1, pc);
    Out* orow = out + row * count;
    // table-backed samplers (32-bit words, one output each): both slabs' values first,
    // the table gathers before the directly evaluated share (the op's kDirect per 16
    // outputs, rounded down), then the stores
    constexpr int kDirectWords = DirectOutputsOf<Op>::value * 2 * B / 16;
    if constexpr (kDirectWords > 0 && W == 32) {
      Vec16<Out> r[2][(B + Vec16<Out>::N - 1) / Vec16<Out>::N];
#pragma unroll
      for (int k = 0; k < 2 * B; ++k) {
        const uint32_t word = k < B ? x0[k] : x1[k - B];
        Out* rv = &r[k / B][0].v[0];
        if (k < 2 * B - kDirectWords) rv[k % B] = op(word);
        else rv[k % B] = op.direct(word);
      }
#pragma unroll
      for (int slab = 0; slab < 2; ++slab) {
        const uint64_t w0 = slab == 0 ? j0 : half + j0;
        const uint64_t wlim = slab == 0 ? umin(half, jhi) : umin(nwords, half + jhi);
        const bool all_in = w0 + B <= wlim && w0 >= begin && w0 + B <= end;
        Out* dst = orow + (w0 - begin);
        const Out* rv = &r[slab][0].v[0];
        if (all_in && ((uintptr_t)dst % 16) == 0) {
#pragma unroll
          for (int k = 0; k < (B * (int)sizeof(Out)) / 16; ++k)
            reinterpret_cast<uint4*>(dst)[k] = r[slab][k].u;
        } else {
#pragma unroll
          for (int k = 0; k < B; ++k) {
            const uint64_t e = w0 + k;
            if (e < wlim && e >= begin && e < end) orow[e - begin] = rv[k];
          }
        }
      }
    } else {
#pragma unroll
      for (int slab = 0; slab < 2; ++slab) {
        const uint64_t w0 = slab == 0 ? j0 : half + j0;  // first word of this slab chunk
        // words of this slab that exist: slab 0 needs j < half, slab 1 half + j < nwords
        const uint64_t wlim = slab == 0 ? umin(half, jhi) : umin(nwords, half + jhi);
        const uint64_t e0 = w0 * per;  // first element
        Vec16<Out> r[(B * per + Vec16<Out>::N - 1) / Vec16<Out>::N];
        Out* rv = &r[0].v[0];
#pragma unroll
        for (int b = 0; b < B; ++b) {
          const uint32_t word = slab == 0 ? x0[b] : x1[b];
#pragma unroll
          for (int q = 0; q < per; ++q) {
            if constexpr (W == 32) rv[b * per + q] = op(word);
            else rv[b * per + q] = op((typename Op::Bits)(word >> (W * q)));
          }
        }
        constexpr int NE = B * per;
        const bool all_in = w0 + B <= wlim && e0 >= begin && e0 + NE <= end;
        Out* dst = orow + (e0 - begin);
        if (all_in && ((uintptr_t)dst % 16) == 0) {
#pragma unroll
          for (int k = 0; k < (NE * (int)sizeof(Out)) / 16; ++k)
            reinterpret_cast<uint4*>(dst)[k] = r[k].u;
        } else {
#pragma unroll
          for (int k = 0; k < NE; ++k) {
            const uint64_t e = e0 + k;
            if (w0 + k / per < wlim && e >= begin && e < end) orow[e - begin] = rv[k];
          }
        }
      }
    }
  }
}

template <class Op>
int launch_words(const uint32_t* keys, int64_t nkeys, uint64_t size, uint64_t begin,
                 uint64_t count, const Op& op, void* out, cudaStream_t st) {
  using Out = typename Op::Out;
  constexpr int B = words_per_thread<Op>();
  constexpr int per = 32 / Op::kBits;
  if (count == 0 || nkeys == 0) return JXR_OK;
  const uint64_t nwords = (size + per - 1) / per;
  if (nwords >= 0xFFFFFFFFull)
    return fail(JXR_ERR_NOT_IMPLEMENTED,
                "original-layout requests of 2^32-1 or more 32-bit words (key splitting, "
                "R/prng.R:236-245) are not supported");
  const uint64_t half = (nwords + 1) / 2;
  const uint64_t wb = begin / per, we = (begin + count + per - 1) / per;
  // blocks whose first word (j) or second word (half + j) falls in [wb, we)
  uint64_t r1lo = wb, r1hi = std::min(we, half);
  uint64_t r2lo = (std::max(wb, half)) - half, r2hi = we > half ? we - half : 0;
  struct Range { uint64_t lo, hi; } ranges[2];
  int nr = 0;
  if (r1lo < r1hi) ranges[nr++] = {r1lo, r1hi};
  if (r2lo < r2hi) {
    if (nr && r2lo <= ranges[0].hi && r2hi >= ranges[0].lo) {
      ranges[0].lo = std::min(ranges[0].lo, r2lo);
      ranges[0].hi = std::max(ranges[0].hi, r2hi);
    } else {
      ranges[nr++] = {r2lo, r2hi};
    }
  }
  for (int k = 0; k < nr; ++k) {
    const uint64_t upr = (ranges[k].hi - ranges[k].lo + B - 1) / B;
    const uint64_t nunits = upr * (uint64_t)nkeys;
    int grid = 0, rc;
    auto kern = k_words<Op>;
    if ((rc = resident_grid(kern, (nunits + kThreads - 1) / kThreads, &grid))) return rc;
    kern<<<grid, kThreads, 0, st>>>(keys, nwords, half, ranges[k].lo, ranges[k].hi, upr, nunits,
                                    begin, count, op, kPipe, (Out*)out);
    JXR_CUDA(cudaGetLastError());
  }
  return JXR_OK;
}

// ---- original layout, requests of 2^32 - 1 words or more ----------------------------------

// Above 2^32 - 1 words the original layout splits the key (R/prng.R:233-245): with
// U = 2^32 - 1, nseg = nwords / U + 1 keys come from split_original(key, nseg), key s
// hashes iota(U) (the last one iota(nwords mod U)), and the word streams are
// concatenated.  Each thread derives the key of the segment it is in (two cipher blocks,
// cached while the segment stays the same) and computes every word it needs directly:
// one block per 32-bit word, so this path runs at half the rate of k_words, which serves
// all smaller requests.
struct SegState {
  uint64_t seg = ~0ull;
  uint64_t len = 0;
  KeySchedule ks;
};

__device__ __forceinline__ uint32_t word_of_hash(const KeySchedule& ks, uint64_t n, uint64_t j) {
  // word j of threefry_2x32(key, iota(n)) (R/prng.R:102-120)
  const uint64_t half = (n + 1) / 2;
  uint32_t a[1], b[1];
  const bool first = j < half;
  a[0] = (uint32_t)(first ? j : j - half);
  b[0] = first ? (half + j < n ? (uint32_t)(half + j) : 0u) : (uint32_t)j;
  threefry20<1>(ks, a, b);
  return first ? a[0] : b[0];
}

__device__ __forceinline__ uint32_t segmented_word(const KeySchedule& parent, uint64_t nwords,
                                                   uint64_t g, SegState& st) {
  constexpr uint64_t U = 0xFFFFFFFFull;
  const uint64_t nseg = nwords / U + 1;
  const uint64_t seg = g / U;
  if (seg != st.seg) {
    st.ks = make_schedule(word_of_hash(parent, 2 * nseg, 2 * seg),
                          word_of_hash(parent, 2 * nseg, 2 * seg + 1));
    st.len = seg + 1 < nseg ? U : nwords - seg * U;
    st.seg = seg;
  }
  return word_of_hash(st.ks, st.len, g - seg * U);
}

template <class Op>
__global__ void __launch_bounds__(kThreads)
    k_original_segmented(const uint32_t* __restrict__ key, uint64_t size, uint64_t begin,
                         uint64_t count, Op op, typename Op::Out* __restrict__ out) {
  constexpr int W = Op::kBits;
  const KeySchedule parent = make_schedule(__ldg(key), __ldg(key + 1));
  SegState hi_st, lo_st;
  const uint64_t stride = (uint64_t)gridDim.x * kThreads;
  for (uint64_t p = (uint64_t)blockIdx.x * kThreads + threadIdx.x; p < count; p += stride) {
    const uint64_t e = begin + p;
    if constexpr (W == 64) {  // (bits[e] << 32) | bits[size + e] over 2 size words
      const uint64_t hi = segmented_word(parent, 2 * size, e, hi_st);
      const uint64_t lo = segmented_word(parent, 2 * size, size + e, lo_st);
      out[p] = op((hi << 32) | lo);
    } else if constexpr (W == 32) {
      out[p] = op(segmented_word(parent, size, e, hi_st));
    } else {  // little-endian W-bit pieces of ceil(W size / 32) words
      constexpr int per = 32 / W;
      const uint64_t nwords = (size + per - 1) / per;
      const uint32_t w = segmented_word(parent, nwords, e / per, hi_st);
      out[p] = op((typename Op::Bits)(w >> (W * (int)(e % per))));
    }
  }
}

template <class Op>
int launch_original_segmented(const uint32_t* keys, int64_t nkeys, uint64_t size, uint64_t begin,
                              uint64_t count, const Op& op, void* out, cudaStream_t st) {
  using Out = typename Op::Out;
  if (count == 0 || nkeys == 0) return JXR_OK;
  int grid = 0, rc;
  auto k = k_original_segmented<Op>;
  if ((rc = resident_grid(k, (count + kThreads - 1) / kThreads, &grid))) return rc;
  for (int64_t r = 0; r < nkeys; ++r)
    k<<<grid, kThreads, 0, st>>>(keys + 2 * r, size, begin, count, op, (Out*)out + (uint64_t)r * count);
  JXR_CUDA(cudaGetLastError());
  return JXR_OK;
}

// ---- dispatch by layout -------------------------------------------------------------------

// Ops drawing W <= 32 bits: partitionable -> k_blocks, original -> k_words.
// Ops drawing 64 bits: k_blocks with index counters or (i, size + i) pairs.
template <class Op>
int launch_op(const uint32_t* keys, int64_t nkeys, uint64_t size, uint64_t begin, uint64_t count,
              int layout, const Op& op, void* out, cudaStream_t st) {
  if (layout == JXR_LAYOUT_PARTITIONABLE)
    return launch_blocks<Op, kCtrIndex>(keys, nkeys, size, begin, count, op, out, st);
  if constexpr (Op::kBits == 64) {
    if (size >= 0x7FFFFFFFull)  // 2 size >= 2^32 - 1 words: the key is split
      return launch_original_segmented<Op>(keys, nkeys, size, begin, count, op, out, st);
    return launch_blocks<Op, kCtrPair>(keys, nkeys, size, begin, count, op, out, st);
  } else {
    constexpr uint64_t per = 32 / Op::kBits;
    if ((size + per - 1) / per >= 0xFFFFFFFFull)
      return launch_original_segmented<Op>(keys, nkeys, size, begin, count, op, out, st);
    return launch_words<Op>(keys, nkeys, size, begin, count, op, out, st);
  }
}

// ---- float32 sampler tables ----------------------------------------------------------

template <class Op>
__global__ void k_build_table(Op op, float* __restrict__ table) {
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < (1u << 23);
       i += gridDim.x * blockDim.x)
    table[i] = op(i << 9);
}

// Requests of at least this many float32 samples use (and, the first time, build) the
// sampler's table.
constexpr uint64_t kTableMin = 1ull << 22;
// A truncated normal builds its table in the call (it depends on the bounds): worth it from
// 2^25 samples, where the 2^23 evaluations of the build are under a quarter of the request.
constexpr uint64_t kTruncTableMin = 1ull << 25;
constexpr int kTables = 8;  // 0: normal, 1 + kind: the log-transform samplers, 5: normal
                            // with the accurate erf_inv
constexpr int kTableNormalAccurate = 5;
std::mutex g_tab_mu;
float* g_tables[64][kTables];

// The current device's table in slot `id` once jxr_prepare_device has built it, else
// nullptr: the caller then evaluates the op.  Sampling entry points only look tables up;
// they never allocate, build or wait for one.
const float* f32_table(int id) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_tab_mu);
  return g_tables[dev][id];
}

// Builds the table of `op` in slot `id` of device `dev` (current), on stream st, and waits
// for it (jxr_prepare_device; the caller holds g_tab_mu).
template <class Op>
int build_f32_table(int dev, int id, const Op& op, cudaStream_t st) {
  if (g_tables[dev][id]) return JXR_OK;
  float* t = nullptr;
  JXR_CUDA(cudaMalloc(&t, sizeof(float) << 23));
  k_build_table<Op><<<1024, 256, 0, st>>>(op, t);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) {
    cudaFree(t);
    return fail(JXR_ERR_CUDA, "building a float32 sampler table: %s", cudaGetErrorString(e));
  }
  g_tables[dev][id] = t;
  return JXR_OK;
}

// Outputs per thread (of 16) that a table-backed sampler evaluates directly: where the
// integer pipe's time for the cipher plus those evaluations meets the L1TEX time of the
// remaining gathers.  Measured on B200 (2^26 outputs, one key): 4 for the normal (0.283
// -> 0.245 ms), 6 for the exponential, whose one table-driven logarithm is cheapest
// (0.283 -> 0.229 ms; 4: 0.239 ms), 3 for gumbel and logistic, which take two logarithms
// (0.283 -> 0.256 / 0.258 ms).
template <class Op>
struct DirectShare {
  static constexpr int value = 4;
};
template <>
struct DirectShare<OpLogSampler<kExponential, 0>> {
  static constexpr int value = 6;
};
template <>
struct DirectShare<OpLogSampler<kGumbel, 0>> {
  static constexpr int value = 3;
};
template <>
struct DirectShare<OpLogSampler<kLogistic, 0>> {
  static constexpr int value = 3;
};

// A float32 sampler through its table: part of every thread's outputs are evaluated
// directly while the rest are gathered (OpTableHybridF32), in the bulk kernels of both
// layouts and of key batches.
template <class Op>
int launch_table(const uint32_t* keys, int64_t nkeys, uint64_t size, uint64_t begin,
                 uint64_t count, int layout, const float* table, const Op& op, void* out,
                 cudaStream_t st) {
  using H = OpTableHybridF32<Op, DirectShare<Op>::value>;
  return launch_op(keys, nkeys, size, begin, count, layout, H{table, op}, out, st);
}

// The 16-bit samplers' tables (OpTableH): slot 2 * sampler + (bfloat16), sampler 0..3 the
// log-transform kinds, 4 the normal, 5 the normal with the accurate erf_inv.  Requests of
// at least kTable16Min samples use them.
constexpr uint64_t kTable16Min = 1ull << 16;
constexpr int kTables16 = 12;
uint16_t* g_tables16[64][kTables16];

template <class Op, class T>
__global__ void k_build_table16(Op op, uint16_t* __restrict__ table) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < (uint32_t)T::kEntries) table[i] = op((typename Op::Bits)(i << T::kShift));
}

// The current device's 16-bit table in `slot` once jxr_prepare_device has built it, else
// nullptr (the caller evaluates), as f32_table.
const uint16_t* h16_table(int slot) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_tab_mu);
  return g_tables16[dev][slot];
}

// Builds the 16-bit op's table in `slot` of device `dev` (current) and waits for it
// (jxr_prepare_device; the caller holds g_tab_mu).
template <class Op>
int build_h16_table(int dev, int slot, const Op& op, cudaStream_t st) {
  using T = OpTableH<Op::kBits>;
  if (g_tables16[dev][slot]) return JXR_OK;
  uint16_t* t = nullptr;
  JXR_CUDA(cudaMalloc(&t, sizeof(uint16_t) * T::kEntries));
  k_build_table16<Op, T><<<(T::kEntries + 255) / 256, 256, 0, st>>>(op, t);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) {
    cudaFree(t);
    return fail(JXR_ERR_CUDA, "building a 16-bit sampler table: %s", cudaGetErrorString(e));
  }
  g_tables16[dev][slot] = t;
  return JXR_OK;
}

// A 16-bit sampler: through its table (OpTableH) for requests of kTable16Min or more
// samples once the table is prepared, else evaluated.
template <class Op>
int launch_h(const uint32_t* keys, int64_t nkeys, uint64_t size, uint64_t begin, uint64_t count,
             int layout, int slot, const Op& op, void* out, cudaStream_t st) {
  if (count * (uint64_t)nkeys >= kTable16Min)
    if (const uint16_t* t = h16_table(slot))
      return launch_op(keys, nkeys, size, begin, count, layout, OpTableH<Op::kBits>{t}, out, st);
  return launch_op(keys, nkeys, size, begin, count, layout, op, out, st);
}

int check_request(const void* keys, int64_t nkeys, uint64_t size, uint64_t begin, uint64_t count,
                  int layout, const void* out) {
  if (nkeys < 0) return fail(JXR_ERR_INVALID_ARGUMENT, "nkeys must be >= 0, got %lld", (long long)nkeys);
  if (layout != JXR_LAYOUT_ORIGINAL && layout != JXR_LAYOUT_PARTITIONABLE)
    return fail(JXR_ERR_INVALID_ARGUMENT, "layout must be 0 (original) or 1 (partitionable), got %d", layout);
  if (begin > size || count > size - begin)
    return fail(JXR_ERR_INVALID_ARGUMENT,
                "range [%llu, %llu + %llu) is outside a request of %llu elements",
                (unsigned long long)begin, (unsigned long long)begin, (unsigned long long)count,
                (unsigned long long)size);
  if (count && nkeys && (!keys || !out)) return fail(JXR_ERR_INVALID_ARGUMENT, "null pointer");
  return JXR_OK;
}

int check_dtype(int dtype) {
  if (dtype < JXR_F32 || dtype > JXR_BF16)
    return fail(JXR_ERR_INVALID_ARGUMENT, "dtype must be 0 (f32), 1 (f64), 2 (f16) or 3 (bf16), got %d", dtype);
  return JXR_OK;
}

// host-side conversion of a double bound to a 16-bit float value (round to nearest even)
float to_half_value(double x, bool bf) {
  // round to odd into float, then to nearest even at 16 bits: one correct rounding
  float f = (float)x;
  if (std::isfinite(x) && (double)f != x) {
    if (std::fabs((double)f) > std::fabs(x)) f = std::nextafter(f, 0.0f);
    uint32_t b;
    std::memcpy(&b, &f, 4);
    b |= 1u;
    std::memcpy(&f, &b, 4);
  }
  uint32_t b;
  std::memcpy(&b, &f, 4);
  uint32_t hb;
  if (bf) {
    if ((b & 0x7F800000u) == 0x7F800000u && (b & 0x7FFFFFu)) hb = (b >> 16) | 0x40u;
    else hb = (b + 0x7FFFu + ((b >> 16) & 1u)) >> 16;
    uint32_t r = hb << 16;
    float out;
    std::memcpy(&out, &r, 4);
    return out;
  }
  const __half h = __float2half_rn(f);
  return __half2float(h);
}

// ---- small kernels --------------------------------------------------------------------------

__global__ void k_threefry2x32_elem(const uint32_t* __restrict__ k0, const uint32_t* __restrict__ k1,
                                    const uint32_t* __restrict__ c0, const uint32_t* __restrict__ c1,
                                    uint32_t* __restrict__ x0, uint32_t* __restrict__ x1, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const KeySchedule s = make_schedule(k0[i], k1[i]);
    uint32_t a[1] = {c0[i]}, b[1] = {c1[i]};
    threefry20<1>(s, a, b);
    x0[i] = a[0];
    x1[i] = b[0];
  }
}

__global__ void k_hash_counts(const uint32_t* __restrict__ keys, int64_t nkeys,
                              const uint32_t* __restrict__ cnt, int64_t n, uint32_t* __restrict__ out) {
  const int64_t half = (n + 1) / 2;
  const int64_t total = half * nkeys;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = t / half, j = t - row * half;
    const KeySchedule s = make_schedule(keys[2 * row], keys[2 * row + 1]);
    uint32_t a[1] = {cnt[j]}, b[1] = {half + j < n ? cnt[half + j] : 0u};
    threefry20<1>(s, a, b);
    out[row * n + j] = a[0];
    if (half + j < n) out[row * n + half + j] = b[0];
  }
}

__global__ void k_fold_in(const uint32_t* __restrict__ keys, int64_t nkeys,
                          const uint32_t* __restrict__ data, int64_t ndata, uint32_t* __restrict__ out,
                          int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t kk = nkeys == 1 ? 0 : i, dd = ndata == 1 ? 0 : i;
    const KeySchedule s = make_schedule(keys[2 * kk], keys[2 * kk + 1]);
    uint32_t a[1] = {0u}, b[1] = {data[dd]};
    threefry20<1>(s, a, b);
    out[2 * i] = a[0];
    out[2 * i + 1] = b[0];
  }
}

template <class Op>
__global__ void k_from_bits(const typename Op::Bits* __restrict__ bits, int64_t n, Op op,
                            typename Op::Out* __restrict__ out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = op(bits[i]);
}

template <class Op>
int launch_from_bits(const void* bits, int64_t n, const Op& op, void* out, cudaStream_t st,
                     int grid) {
  k_from_bits<Op><<<grid, 256, 0, st>>>((const typename Op::Bits*)bits, n, op,
                                        (typename Op::Out*)out);
  JXR_CUDA(cudaGetLastError());
  return JXR_OK;
}

// A sampler's transform of given draws through its table (float32: 2^22 or more draws,
// 16-bit: 2^16 or more) once prepared, else evaluated; slot32 / slot16 are the op's slots.
template <class Op>
int launch_from_bits_table(const void* bits, int64_t n, int slot32, int slot16, const Op& op,
                           void* out, cudaStream_t st, int grid) {
  using Out = typename Op::Out;
  if constexpr (std::is_same_v<Out, float> && Op::kBits == 32) {
    if ((uint64_t)n >= kTableMin)
      if (const float* t = f32_table(slot32))
        return launch_from_bits(bits, n, OpTableF32{t}, out, st, grid);
  } else if constexpr (std::is_same_v<Out, uint16_t>) {
    if ((uint64_t)n >= kTable16Min)
      if (const uint16_t* t = h16_table(slot16))
        return launch_from_bits(bits, n, OpTableH<Op::kBits>{t}, out, st, grid);
  }
  return launch_from_bits(bits, n, op, out, st, grid);
}

template <bool kAcc>
__global__ void k_erfinv_f32(const float* __restrict__ x, int64_t n, float* __restrict__ out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = erfinv32<kAcc>(x[i]);
}
template <bool kAcc>
__global__ void k_erfinv_f64(const double* __restrict__ x, int64_t n, double* __restrict__ out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = erfinv64<kAcc>(x[i]);
}

// ---- element-wise helpers for array-valued parameters ------------------------------------

// uniform with per-element bounds from the unit draw u = uniform(0, 1) (which is the unit
// float itself): max(minval, u * (maxval - minval) + minval), R/random.R:297-303.
template <class T, bool kFused>
__global__ void k_affine(const T* __restrict__ u, const T* __restrict__ mn, const T* __restrict__ mx,
                         int64_t nrows, int64_t n, T* __restrict__ out) {
  for (int64_t r = blockIdx.y; r < nrows; r += gridDim.y) {
    const T* ur = u + r * n;
    T* outr = out + r * n;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
      const T lo = mn[i];
      T res;
      if constexpr (sizeof(T) == 4) {
        const T d = __fsub_rn(mx[i], lo);
        res = kFused ? __fmaf_rn(ur[i], d, lo) : __fadd_rn(__fmul_rn(ur[i], d), lo);
      } else {
        const T d = __dsub_rn(mx[i], lo);
        res = kFused ? __fma_rn(ur[i], d, lo) : __dadd_rn(__dmul_rn(ur[i], d), lo);
      }
      outr[i] = xla_max(lo, res);
    }
  }
}

template <bool BF, bool kFused>
__global__ void k_affine_h(const uint16_t* __restrict__ u, const uint16_t* __restrict__ mn,
                           const uint16_t* __restrict__ mx, int64_t nrows, int64_t n,
                           uint16_t* __restrict__ out) {
  for (int64_t r = blockIdx.y; r < nrows; r += gridDim.y) {
    const uint16_t* ur = u + r * n;
    uint16_t* outr = out + r * n;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
      const float f = h2f<BF>(ur[i]), lo = h2f<BF>(mn[i]);
      const float d = rh<BF>(__fsub_rn(h2f<BF>(mx[i]), lo));
      float res;
      if (kFused) res = h2f<BF>(d2h<BF>(__fma_rn((double)f, (double)d, (double)lo)));
      else res = rh<BF>(__fadd_rn(rh<BF>(__fmul_rn(f, d)), lo));
      outr[i] = f2h<BF>(xla_max(lo, res));
    }
  }
}

// bernoulli from unit draws (R/random.R:656-666): mode "low" u < p; mode "high"
// u_hi * 2^-nmant < p - u_lo, all in the dtype of p.
template <class T>
__global__ void k_bern_unit(const T* __restrict__ ulo, const T* __restrict__ uhi,
                            const T* __restrict__ p, int64_t n, T scale, uint8_t* __restrict__ out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    if (uhi == nullptr) {
      out[i] = ulo[i] < p[i];
    } else if constexpr (sizeof(T) == 4) {
      out[i] = __fmul_rn(uhi[i], scale) < __fsub_rn(p[i], ulo[i]);
    } else {
      out[i] = __dmul_rn(uhi[i], scale) < __dsub_rn(p[i], ulo[i]);
    }
  }
}

template <bool BF>
__global__ void k_bern_unit_h(const uint16_t* __restrict__ ulo, const uint16_t* __restrict__ uhi,
                              const uint16_t* __restrict__ p, int64_t n, float scale,
                              uint8_t* __restrict__ out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float pv = h2f<BF>(p[i]), lo = h2f<BF>(ulo[i]);
    if (uhi == nullptr) out[i] = lo < pv;
    else out[i] = rh<BF>(__fmul_rn(h2f<BF>(uhi[i]), scale)) < rh<BF>(__fsub_rn(pv, lo));
  }
}

// the 16-bit float next to the 16-bit value x toward +inf (up) or -inf, as raw bits
__device__ __forceinline__ uint16_t half_next(float x, bool up, bool bf) {
  const uint16_t b = bf ? __bfloat16_as_ushort(__float2bfloat16_rn(x))
                        : __half_as_ushort(__float2half_rn(x));
  const uint16_t inf = bf ? 0x7F80u : 0x7C00u;
  if (x != x || b == (up ? inf : (uint16_t)(0x8000u | inf))) return b;
  if ((b & 0x7FFFu) == 0) return up ? 0x0001u : 0x8001u;  // +-0 -> smallest subnormal
  const bool neg = b & 0x8000u;
  return (uint16_t)((up != neg) ? b + 1 : b - 1);
}

// complex normals (R/random.R:489-499): (re + i im) / sqrt(2) from the two real normals,
// each part divided in the real dtype, interleaved as complex64 / complex128
template <class T>
__global__ void k_complex_div(const T* __restrict__ re, const T* __restrict__ im, int64_t n,
                              T divisor, T* __restrict__ out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    if constexpr (sizeof(T) == 4) {
      out[2 * i] = __fdiv_rn(re[i], divisor);
      out[2 * i + 1] = __fdiv_rn(im[i], divisor);
    } else {
      out[2 * i] = __ddiv_rn(re[i], divisor);
      out[2 * i + 1] = __ddiv_rn(im[i], divisor);
    }
  }
}

// cumulative sum, left to right in the dtype (one thread: the order of the additions
// defines the rounding)
template <class T>
__global__ void k_cumsum_seq(const T* __restrict__ x, int64_t m, T* __restrict__ out) {
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    T acc = 0;
    for (int64_t i = 0; i < m; ++i) {
      if constexpr (sizeof(T) == 4) acc = __fadd_rn(acc, x[i]);
      else acc = __dadd_rn(acc, x[i]);
      out[i] = acc;
    }
  }
}

// random_choice with p and replace (R/random.R:446-450): r = total * (1 - u) in the dtype,
// index = number of cumulative sums strictly below r (searchsorted, side left)
template <class T>
__global__ void k_choice_p(const T* __restrict__ unit, int64_t n, const T* __restrict__ cuml,
                           int64_t m, int out_bits, void* __restrict__ out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    T r;
    if constexpr (sizeof(T) == 4) r = __fmul_rn(cuml[m - 1], __fsub_rn(1.0f, unit[i]));
    else r = __dmul_rn(cuml[m - 1], __dsub_rn(1.0, unit[i]));
    int64_t lo = 0, hi = m;  // first index with cuml[idx] >= r
    while (lo < hi) {
      const int64_t mid = (lo + hi) >> 1;
      if (cuml[mid] < r) lo = mid + 1;
      else hi = mid;
    }
    if (out_bits == 64) ((int64_t*)out)[i] = lo;
    else ((int32_t*)out)[i] = (int32_t)lo;
  }
}

// x[i] += log(p[i]) in the dtype (the log evaluated in double and rounded once)
template <class T>
__global__ void k_add_log(T* __restrict__ x, const T* __restrict__ p, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    if constexpr (sizeof(T) == 4) x[i] = __fadd_rn(x[i], __double2float_rn(log_pos((double)p[i])));
    else x[i] = __dadd_rn(x[i], log_pos(p[i]));
  }
}

// truncated normal with per-element bounds (R/random.R:586-603) from the unit draw
// f = uniform(0, 1): a = erf(lower / sqrt2), b = erf(upper / sqrt2) (CUDA's erf in double,
// rounded to the dtype), u = max(a, f (b - a) + a), sqrt2 erf_inv(u), clipped to
// [nextafter(lower, inf), nextafter(upper, -inf)].  Bounds have stride 0 or 1.
template <int D, bool kAcc>
__global__ void k_trunc_unit(const void* __restrict__ unit, const void* __restrict__ lower,
                             int64_t ls, const void* __restrict__ upper, int64_t us, int64_t n,
                             void* __restrict__ out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    if constexpr (D == JXR_F32) {
      const float s2 = 1.41421354f;
      const float lo = ((const float*)lower)[i * ls], hi = ((const float*)upper)[i * us];
      const float a = __double2float_rn(erf((double)__fdiv_rn(lo, s2)));
      const float b = __double2float_rn(erf((double)__fdiv_rn(hi, s2)));
      const float u = xla_max(a, __fmaf_rn(((const float*)unit)[i], __fsub_rn(b, a), a));
      const float x = __fmul_rn(s2, erfinv32<kAcc>(u));
      const float cl = nextafterf(lo, __int_as_float(0x7F800000)),
                  ch = nextafterf(hi, __int_as_float(0xFF800000));
      ((float*)out)[i] = xla_min(ch, xla_max(cl, x));
    } else if constexpr (D == JXR_F64) {
      const double s2 = 1.4142135623730951;
      const double lo = ((const double*)lower)[i * ls], hi = ((const double*)upper)[i * us];
      const double a = erf(__ddiv_rn(lo, s2)), b = erf(__ddiv_rn(hi, s2));
      const double u = xla_max(a, __fma_rn(((const double*)unit)[i], __dsub_rn(b, a), a));
      const double x = __dmul_rn(s2, erfinv64<kAcc>(u));
      const double inf = __longlong_as_double(0x7FF0000000000000ll);
      ((double*)out)[i] = xla_min(nextafter(hi, -inf), xla_max(nextafter(lo, inf), x));
    } else {
      constexpr bool BF = D == JXR_BF16;
      const float s2 = rh<BF>(1.41421354f);
      const uint16_t lb = ((const uint16_t*)lower)[i * ls], ub = ((const uint16_t*)upper)[i * us];
      const float lo = h2f<BF>(lb), hi = h2f<BF>(ub);
      const float a = rh<BF>(__double2float_rn(erf((double)rh<BF>(__fdiv_rn(lo, s2)))));
      const float b = rh<BF>(__double2float_rn(erf((double)rh<BF>(__fdiv_rn(hi, s2)))));
      const float d = rh<BF>(__fsub_rn(b, a));
      const float f = h2f<BF>(((const uint16_t*)unit)[i]);
      const float u = xla_max(a, h2f<BF>(d2h<BF>(__fma_rn((double)f, (double)d, (double)a))));
      const float x = rh<BF>(__fmul_rn(s2, rh<BF>(erfinv32<kAcc>(u))));
      ((uint16_t*)out)[i] = f2h<BF>(xla_min(h2f<BF>(half_next(hi, false, BF)),
                                            xla_max(h2f<BF>(half_next(lo, true, BF)), x)));
    }
  }
}

// gumbel modes "high"/"highest" from the two rows of a (2, n) draw
template <int D, int kMode>
__global__ void k_gumbel_rows(const void* __restrict__ row0, const void* __restrict__ row1,
                              int64_t n, void* __restrict__ out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    if constexpr (kMode == 1) {  // highest, float32 bits
      ((float*)out)[i] = gumbel_highest_f32(((const uint32_t*)row0)[i], ((const uint32_t*)row1)[i]);
    } else if constexpr (D == JXR_F32) {
      ((float*)out)[i] = gumbel_high_f32(((const float*)row0)[i], ((const float*)row1)[i]);
    } else if constexpr (D == JXR_F64) {
      ((double*)out)[i] = gumbel_high_f64(((const double*)row0)[i], ((const double*)row1)[i]);
    } else {
      constexpr bool BF = D == JXR_BF16;
      const float r = gumbel_high_h<BF>(h2f<BF>(((const uint16_t*)row0)[i]),
                                        h2f<BF>(((const uint16_t*)row1)[i]));
      ((uint16_t*)out)[i] = f2h<BF>(r);
    }
  }
}

// rbg bits: elements [begin, begin + count) of a request of bit_width-bit values from the
// Philox stream of key q.  Each thread takes G consecutive blocks (one 16-byte store's
// worth when the output allows it); per block: 4 elements (8/16/32-bit) or 2 (64-bit).
template <int kBits>
__global__ void __launch_bounds__(256)
k_rbg_bits(const uint32_t* __restrict__ key, uint64_t begin, uint64_t count, void* __restrict__ out) {
  constexpr int kPer = kBits == 64 ? 2 : 4;           // elements per block
  constexpr int kG = kBits == 8 ? 4 : kBits == 16 ? 2 : 1;  // blocks per 16-byte store
  constexpr int kEsz = kBits / 8;
  uint32_t q[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) q[i] = key[i];
  const uint64_t end = begin + count;
  const uint64_t b_first = begin / kPer, b_last = (end + kPer - 1) / kPer;  // [b_first, b_last)
  const uint64_t groups = (b_last - b_first + kG - 1) / kG;
  for (uint64_t g = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; g < groups;
       g += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t b0 = b_first + g * kG;
    uint32_t w[4 * kG];
#pragma unroll
    for (int j = 0; j < kG; ++j) {
      const PhiloxOut o = rbg_block(q, b0 + j);
#pragma unroll
      for (int t = 0; t < 4; ++t) w[4 * j + t] = o.w[t];
    }
    const uint64_t e0 = b0 * kPer;  // first element of the group
    char* dst = (char*)out + (int64_t)(e0 - begin) * kEsz;
    const bool full = e0 >= begin && e0 + kPer * kG <= end && ((uintptr_t)dst & 15u) == 0;
    if (full) {
      uint4 v;
      if constexpr (kBits == 8) {
        uint32_t p[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
          p[j] = (w[4 * j] & 0xFFu) | (w[4 * j + 1] & 0xFFu) << 8 | (w[4 * j + 2] & 0xFFu) << 16 |
                 (w[4 * j + 3] & 0xFFu) << 24;
        v = make_uint4(p[0], p[1], p[2], p[3]);
      } else if constexpr (kBits == 16) {
        v = make_uint4((w[0] & 0xFFFFu) | w[1] << 16, (w[2] & 0xFFFFu) | w[3] << 16,
                       (w[4] & 0xFFFFu) | w[5] << 16, (w[6] & 0xFFFFu) | w[7] << 16);
      } else {
        v = make_uint4(w[0], w[1], w[2], w[3]);  // 32-bit: 4 outputs; 64-bit: (w0|w1<<32, w2|w3<<32)
      }
      *(uint4*)dst = v;
    } else {
#pragma unroll
      for (int t = 0; t < kPer * kG; ++t) {
        const uint64_t e = e0 + t;
        if (e < begin || e >= end) continue;
        const int64_t i = (int64_t)(e - begin);
        if constexpr (kBits == 8) ((uint8_t*)out)[i] = (uint8_t)w[t];
        else if constexpr (kBits == 16) ((uint16_t*)out)[i] = (uint16_t)w[t];
        else if constexpr (kBits == 32) ((uint32_t*)out)[i] = w[t];
        else ((uint64_t*)out)[i] = (uint64_t)w[2 * t] | (uint64_t)w[2 * t + 1] << 32;
      }
    }
  }
}

// blocks first + i * stride (i < n) of the stream of key q, 4 words each (unsafe_rbg split:
// rows 0, 10, 20, ... of a (10 num, 4) request)
__global__ void k_rbg_blocks(const uint32_t* __restrict__ key, uint64_t first, uint64_t stride,
                             int64_t n, uint32_t* __restrict__ out) {
  uint32_t q[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) q[i] = key[i];
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const PhiloxOut o = rbg_block(q, first + (uint64_t)i * stride);
    *(uint4*)(out + 4 * i) = make_uint4(o.w[0], o.w[1], o.w[2], o.w[3]);
  }
}

// unsafe_rbg fold_in (R/prng.R:423-426): key ^ row 9 of a (10, 4) request from the key
// rbg_seed(data) = (0, d, 0, d); the keys and data broadcast against each other.  With
// lane_blocks > 0 every output i instead draws row 9 + 10 i of data[0]'s stream (the
// batching rule of rng_bit_generator: all lanes from the first key).
__global__ void k_rbg_unsafe_fold_in(const uint32_t* __restrict__ keys, int64_t nkeys,
                                     const uint32_t* __restrict__ data, int64_t ndata,
                                     int64_t n, int lanes_from_first, uint32_t* __restrict__ out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t* k = keys + 4 * (nkeys == 1 ? 0 : i);
    const uint32_t d = data[lanes_from_first || ndata == 1 ? 0 : i];
    const uint32_t q[4] = {0u, d, 0u, d};
    const PhiloxOut o = rbg_block(q, lanes_from_first ? 9u + 10u * (uint64_t)i : 9u);
    *(uint4*)(out + 4 * i) =
        make_uint4(k[0] ^ o.w[0], k[1] ^ o.w[1], k[2] ^ o.w[2], k[3] ^ o.w[3]);
  }
}

// new state of rng_bit_generator: the 128-bit counter advanced by the blocks used
__global__ void k_rbg_advance(const uint32_t* __restrict__ key, uint64_t nblocks,
                              uint32_t* __restrict__ out) {
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    const uint64_t lo = ((uint64_t)key[1] << 32 | key[0]);
    const uint64_t hi = ((uint64_t)key[3] << 32 | key[2]);
    const uint64_t l2 = lo + nblocks;
    const uint64_t h2 = hi + (l2 < lo ? 1u : 0u);
    out[0] = (uint32_t)l2;
    out[1] = (uint32_t)(l2 >> 32);
    out[2] = (uint32_t)h2;
    out[3] = (uint32_t)(h2 >> 32);
  }
}

// randint with scalar bounds in one pass (partitionable layout): element c of key row r
// draws hi and lo from the two halves (kh, kl) of split(key) at counter c and writes the
// low out_bits of a + offset (randint_offset with the span's multiplier precomputed).
// Each thread takes kRandintV consecutive elements of one row; rows and columns advance
// by a fixed stride (one division per thread, not one per unit).
constexpr int kRandintV = 8;
template <class U, class OutT>
__global__ void __launch_bounds__(256)
k_randint_fused(const uint32_t* __restrict__ kh, const uint32_t* __restrict__ kl, int64_t nkeys,
                uint64_t begin, uint64_t count, U a, U span, U mult, PipeConsts pc,
                OutT* __restrict__ out) {
  constexpr int V = kRandintV;
  const uint64_t per_row = (count + V - 1) / V;
  const uint64_t units = per_row * (uint64_t)nkeys;
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  uint64_t u = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (u >= units) return;
  uint64_t r = u / per_row, col = u - r * per_row;
  const uint64_t dr = stride / per_row, dc = stride - dr * per_row;
  for (; u < units; u += stride) {
    const uint64_t j0 = col * V;
    const KeySchedule sh = make_schedule(kh[2 * r], kh[2 * r + 1]);
    const KeySchedule sl = make_schedule(kl[2 * r], kl[2 * r + 1]);
    uint32_t h0[V], h1[V], l0[V], l1[V];
#pragma unroll
    for (int t = 0; t < V; ++t) {
      const uint64_t c = begin + j0 + t;
      h0[t] = l0[t] = (uint32_t)(c >> 32);
      h1[t] = l1[t] = (uint32_t)c;
    }
    threefry20<V, ProductMix>(sh, h0, h1, pc);
    threefry20<V, ProductMix>(sl, l0, l1, pc);
    OutT* dst = out + r * count + j0;
    union {
      OutT v[V];
      uint4 q[(V * sizeof(OutT) + 15) / 16];
    } res;
#pragma unroll
    for (int t = 0; t < V; ++t) {
      U hi, lo;
      if constexpr (sizeof(U) == 4) {
        hi = h0[t] ^ h1[t];
        lo = l0[t] ^ l1[t];
      } else {
        hi = (uint64_t)h0[t] << 32 | h1[t];
        lo = (uint64_t)l0[t] << 32 | l1[t];
      }
      const U off = span == 0 ? lo : (U)((U)((hi % span) * mult) + lo % span) % span;
      res.v[t] = (OutT)(U)(a + off);
    }
    constexpr bool kVec = (V * sizeof(OutT)) % 16 == 0;
    if (kVec && j0 + V <= count && ((uintptr_t)dst % 16) == 0) {
#pragma unroll
      for (int k = 0; k < (int)(V * sizeof(OutT)) / 16; ++k)
        reinterpret_cast<uint4*>(dst)[k] = res.q[k];
    } else {
#pragma unroll
      for (int t = 0; t < V; ++t)
        if (j0 + t < count) dst[t] = res.v[t];
    }
    col += dc;
    r += dr;
    if (col >= per_row) {
      col -= per_row;
      ++r;
    }
  }
}

// randint: out = low out_bits of (minval + offset(hi, lo, span)) in the sampling dtype
template <class U, bool kSigned>
__global__ void k_randint_combine(const U* __restrict__ hi, const U* __restrict__ lo, int64_t n,
                                  const int64_t* __restrict__ mn, int64_t mn_stride,
                                  const int64_t* __restrict__ mx, int64_t mx_stride,
                                  const uint8_t* __restrict__ oor, int64_t oor_stride,
                                  int out_bits, void* __restrict__ out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t a = mn[i * mn_stride], b = mx[i * mx_stride];
    const bool empty = kSigned ? (b <= a) : ((uint64_t)b <= (uint64_t)a);
    U span = (U)((U)b - (U)a);
    if (empty) span = 1;
    if (oor[i * oor_stride] && !empty) span = (U)(span + 1);
    U off;
    if (span == 0) {  // full range: x % 0 is x (XLA), the multiplier is 0
      off = lo[i];
    } else {
      off = randint_offset<U>(hi[i], lo[i], span);
    }
    const uint64_t r = (uint64_t)(U)((U)a + off);
    switch (out_bits) {
      case 8: ((uint8_t*)out)[i] = (uint8_t)r; break;
      case 16: ((uint16_t*)out)[i] = (uint16_t)r; break;
      case 32: ((uint32_t*)out)[i] = (uint32_t)r; break;
      default: ((uint64_t*)out)[i] = r; break;
    }
  }
}

int small_grid(int64_t n, int* grid) {
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  const int64_t want = (n + 255) / 256;
  *grid = (int)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)di.sms * 8));
  return JXR_OK;
}

// ---- fused normal + bernoulli (same key and shape: one cipher pass, two outputs) ---------

constexpr int kNBBytes = 32;  // normal bytes per thread and iteration of k_normal_bernoulli

template <class OpN, class OpB, int kCtr, bool kOneKey>
__global__ void __launch_bounds__(kThreads)
    k_normal_bernoulli(const uint32_t* __restrict__ keys, uint64_t size, uint64_t begin,
                       uint64_t count, uint64_t chunks_per_row, uint64_t nchunks, int vec_ok, OpN opn,
                       OpB opb, PipeConsts pc, typename OpN::Out* __restrict__ nout,
                       uint8_t* __restrict__ bout) {
  using Out = typename OpN::Out;
  constexpr int V = kNBBytes / sizeof(Out);  // outputs per iteration: two 16-byte stores
  const uint64_t stride = (uint64_t)gridDim.x * kThreads;
  for (uint64_t c = (uint64_t)blockIdx.x * kThreads + threadIdx.x; c < nchunks; c += stride) {
    const uint64_t row = kOneKey ? 0 : c / chunks_per_row;
    const uint64_t pos = (c - row * chunks_per_row) * V;
    const KeySchedule s = make_schedule(__ldg(keys + 2 * row), __ldg(keys + 2 * row + 1));
    uint32_t x0[V], x1[V];
#pragma unroll
    for (int v = 0; v < V; ++v) {
      const uint64_t i = begin + pos + v;
      x0[v] = kCtr == kCtrIndex ? (uint32_t)(i >> 32) : (uint32_t)i;
      x1[v] = kCtr == kCtrIndex ? (uint32_t)i : (uint32_t)(size + i);
    }
    threefry20<V, ProductMix>(s, x0, x1, pc);
    Vec16<Out> r[2];
    uint8_t bb[V];
    Out o[V];
    apply_all<V>(opn, x0, x1, o);  // every draw's normal (OpN::batch where it has one)
#pragma unroll
    for (int v = 0; v < V; ++v) {
      r[v / (V / 2)].v[v % (V / 2)] = o[v];
      bb[v] = opb(Draw<OpB::kBits>::get(x0[v], x1[v]));
    }
    Out* dst = nout + row * count + pos;
    uint8_t* bdst = bout + row * count + pos;
    if (vec_ok && pos + V <= count) {
      reinterpret_cast<uint4*>(dst)[0] = r[0].u;
      reinterpret_cast<uint4*>(dst)[1] = r[1].u;
      if (vec_ok & 2) {  // the V flags as one V-byte store
        uint32_t w[V / 4];
#pragma unroll
        for (int q = 0; q < V / 4; ++q)
          w[q] = bb[4 * q] | (bb[4 * q + 1] << 8) | (bb[4 * q + 2] << 16) |
                 ((uint32_t)bb[4 * q + 3] << 24);
        if constexpr (V == 4) *reinterpret_cast<uint32_t*>(bdst) = w[0];
        else *reinterpret_cast<uint2*>(bdst) = make_uint2(w[0], w[1]);
      } else {
#pragma unroll
        for (int v = 0; v < V; ++v) bdst[v] = bb[v];
      }
    } else {
#pragma unroll
      for (int v = 0; v < V; ++v)
        if (pos + v < count) { dst[v] = r[v / (V / 2)].v[v % (V / 2)]; bdst[v] = bb[v]; }
    }
  }
}

template <class OpN, class OpB>
int launch_normal_bernoulli(const uint32_t* keys, int64_t nkeys, uint64_t size, uint64_t begin,
                            uint64_t count, int layout, const OpN& opn, const OpB& opb, void* nout,
                            uint8_t* bout, cudaStream_t st) {
  using Out = typename OpN::Out;
  constexpr int V = kNBBytes / sizeof(Out);
  if (count == 0 || nkeys == 0) return JXR_OK;
  const uint64_t cpr = (count + V - 1) / V;
  const uint64_t nchunks = cpr * (uint64_t)nkeys;
  // a chunk is two 16-byte stores of normals (the kernel writes r[0] and r[1])
  static_assert(kNBBytes == 32 && (V == 4 || V == 8), "32-byte chunks of 4 or 8 outputs");
  // bit 0: 16-byte normal stores; bit 1: also the V flag bytes as one store
  int vec_ok = ((uintptr_t)nout % 16 == 0) && (nkeys == 1 || (count * sizeof(Out)) % 16 == 0);
  if (vec_ok && (uintptr_t)bout % V == 0 && (nkeys == 1 || count % V == 0)) vec_ok |= 2;
  const uint64_t ctas = (nchunks + kThreads - 1) / kThreads;
  int grid = 0, rc;
#define JXR_NB_LAUNCH(CTR, ONE)                                                              \
  {                                                                                          \
    auto k = k_normal_bernoulli<OpN, OpB, CTR, ONE>;                                         \
    if ((rc = resident_grid(k, ctas, &grid))) return rc;                                     \
    k<<<grid, kThreads, 0, st>>>(keys, size, begin, count, cpr, nchunks, vec_ok, opn, opb,   \
                                 kPipe, (Out*)nout, bout);                                   \
  }
  if (layout == JXR_LAYOUT_PARTITIONABLE) {
    if (nkeys == 1) JXR_NB_LAUNCH(kCtrIndex, true) else JXR_NB_LAUNCH(kCtrIndex, false)
  } else {
    if (nkeys == 1) JXR_NB_LAUNCH(kCtrPair, true) else JXR_NB_LAUNCH(kCtrPair, false)
  }
#undef JXR_NB_LAUNCH
  JXR_CUDA(cudaGetLastError());
  return JXR_OK;
}


// ---- throughput probe: the cipher alone, in registers ----------------------------------------

// Each thread advances 8 independent blocks through `iters` full threefry20 passes, with
// no counters, loads or stores: the integer-pipe ceiling of the cipher on this GPU, used
// as the roofline denominator.  The xor of the final words is stored so the work stays.
__global__ void __launch_bounds__(kThreads) k_probe_cipher(uint64_t iters, uint32_t* sink,
                                                           PipeConsts pc) {
  const uint32_t t = blockIdx.x * kThreads + threadIdx.x;
  const KeySchedule s = make_schedule(t * 0x9E3779B9u, t ^ 0x85EBCA6Bu);
  uint32_t x0[8], x1[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) { x0[j] = t + j; x1[j] = ~t * (j + 1); }
  for (uint64_t i = 0; i < iters; ++i) threefry20<8, ProductMix>(s, x0, x1, pc);
  uint32_t acc = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) acc ^= x0[j] ^ x1[j];
  sink[t] = acc;
}
}  // namespace
}  // namespace jxr

// ==== C ABI ==================================================================================

using namespace jxr;

// ---- fixed device scratch for jxr_random_bits_host_static -----------------------------------

// Some callers cannot allocate device memory while they run, so jxr_random_bits_host_static
// works entirely in this statically sized array: the first kStaticKeyBytes hold the keys,
// the rest is the staging buffer that each chunk is generated into before it is copied to
// the host.  Every GPU that loads the library holds the array until the process exits.
constexpr int64_t kStaticMaxKeys = 4096;
constexpr size_t kStaticKeyBytes = 8 * (size_t)kStaticMaxKeys;  // 32 KiB
constexpr size_t kStaticStageBytes = 16ull << 20;                // 16 MiB
static __device__ __align__(256) unsigned char g_static_scratch[kStaticKeyBytes + kStaticStageBytes];

// Device address of g_static_scratch per device, looked up once with that device current
// (the name is only a host-side stand-in for the array; host code must not pass it), and
// cleared by jxr_free_caches (after a device reset the module, and the array, may move).
static void* g_static_scratch_addr[64] = {};
static std::mutex g_static_scratch_mu;
// Held for the whole of a jxr_random_bits_host_static call on that device: calls from
// several host threads take turns, so they cannot overlap on the GPU through the array.
static std::mutex g_static_call_mu[64];

// Loads, on the current device, every kernel that jxr_random_bits_host_static can launch
// for bit width W: CUDA loads a module's functions lazily, on first use, which allocates
// their code on the device; querying a function's attributes loads it now.
template <int W>
static int preload_bits_kernels() {
  using Op = OpBits<W>;
  cudaFuncAttributes a;
  JXR_CUDA(cudaFuncGetAttributes(&a, (const void*)k_blocks_1key<Op, kCtrIndex>));
  JXR_CUDA(cudaFuncGetAttributes(&a, (const void*)k_original_segmented<Op>));
  if constexpr (W == 64) JXR_CUDA(cudaFuncGetAttributes(&a, (const void*)k_blocks_1key<Op, kCtrPair>));
  else JXR_CUDA(cudaFuncGetAttributes(&a, (const void*)k_words<Op>));
  return JXR_OK;
}

static int static_scratch(int dev, unsigned char** out) {
  std::lock_guard<std::mutex> lock(g_static_scratch_mu);
  if (!g_static_scratch_addr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess || !p)
      return fail(JXR_ERR_CUDA, "cudaGetSymbolAddress(g_static_scratch): %s", cudaGetErrorString(e));
    g_static_scratch_addr[dev] = p;
  }
  *out = (unsigned char*)g_static_scratch_addr[dev];
  return JXR_OK;
}


extern "C" {

int jxr_abi_version(void) { return JXR_ABI_VERSION; }

const char* jxr_last_error(void) { return g_error.c_str(); }

int jxr_seed(const int64_t* seeds, int64_t n, int x64, uint32_t* keys_out) {
  if (n < 0 || (n && (!seeds || !keys_out))) return fail(JXR_ERR_INVALID_ARGUMENT, "bad seed arrays");
  for (int64_t i = 0; i < n; ++i) {
    const uint64_t s = (uint64_t)seeds[i];
    keys_out[2 * i] = x64 ? (uint32_t)(s >> 32) : 0u;
    keys_out[2 * i + 1] = (uint32_t)s;
  }
  return JXR_OK;
}

int jxr_threefry2x32(const uint32_t* k0, const uint32_t* k1, const uint32_t* c0, const uint32_t* c1,
                     uint32_t* x0, uint32_t* x1, int64_t n, void* stream) {
  if (n < 0) return fail(JXR_ERR_INVALID_ARGUMENT, "n must be >= 0");
  if (n == 0) return JXR_OK;
  if (!k0 || !k1 || !c0 || !c1 || !x0 || !x1) return fail(JXR_ERR_INVALID_ARGUMENT, "null pointer");
  int grid, rc;
  if ((rc = small_grid(n, &grid))) return rc;
  k_threefry2x32_elem<<<grid, 256, 0, (cudaStream_t)stream>>>(k0, k1, c0, c1, x0, x1, n);
  JXR_CUDA(cudaGetLastError());
  return JXR_OK;
}

int jxr_threefry_2x32(const uint32_t* keys, int64_t nkeys, const uint32_t* count, int64_t n,
                      uint32_t* out, void* stream) {
  if (nkeys < 0 || n < 0) return fail(JXR_ERR_INVALID_ARGUMENT, "sizes must be >= 0");
  if (n > 0xFFFFFFFFll) return fail(JXR_ERR_INVALID_ARGUMENT, "count vector longer than 2^32");
  if (!nkeys || !n) return JXR_OK;
  if (!keys || !count || !out) return fail(JXR_ERR_INVALID_ARGUMENT, "null pointer");
  int grid, rc;
  if ((rc = small_grid(((n + 1) / 2) * nkeys, &grid))) return rc;
  k_hash_counts<<<grid, 256, 0, (cudaStream_t)stream>>>(keys, nkeys, count, n, out);
  JXR_CUDA(cudaGetLastError());
  return JXR_OK;
}

int jxr_split(const uint32_t* keys, int64_t nkeys, int64_t num, int layout, uint32_t* out,
              void* stream) {
  if (num < 0) return fail(JXR_ERR_INVALID_ARGUMENT, "num must be >= 0");
  int rc = check_request(keys, nkeys, (uint64_t)num, 0, (uint64_t)num, layout, out);
  if (rc) return rc;
  if (layout == JXR_LAYOUT_PARTITIONABLE)  // key j = threefry(key, (hi(j), lo(j)))
    return launch_blocks<OpKeyPair, kCtrIndex>(keys, nkeys, (uint64_t)num, 0, (uint64_t)num,
                                               OpKeyPair{}, out, (cudaStream_t)stream);
  // original: threefry_2x32(key, iota(2 num)) reshaped to (num, 2)
  return launch_words<OpBits<32>>(keys, nkeys, 2 * (uint64_t)num, 0, 2 * (uint64_t)num,
                                  OpBits<32>{}, out, (cudaStream_t)stream);
}

int jxr_fold_in(const uint32_t* keys, int64_t nkeys, const uint32_t* data, int64_t ndata,
                uint32_t* out, void* stream) {
  if (nkeys < 0 || ndata < 0) return fail(JXR_ERR_INVALID_ARGUMENT, "sizes must be >= 0");
  if (nkeys != ndata && nkeys != 1 && ndata != 1)
    return fail(JXR_ERR_INVALID_ARGUMENT, "nkeys (%lld) and ndata (%lld) do not broadcast",
                (long long)nkeys, (long long)ndata);
  const int64_t n = (nkeys == 0 || ndata == 0) ? 0 : std::max(nkeys, ndata);
  if (!n) return JXR_OK;
  if (!keys || !data || !out) return fail(JXR_ERR_INVALID_ARGUMENT, "null pointer");
  int grid, rc;
  if ((rc = small_grid(n, &grid))) return rc;
  k_fold_in<<<grid, 256, 0, (cudaStream_t)stream>>>(keys, nkeys, data, ndata, out, n);
  JXR_CUDA(cudaGetLastError());
  return JXR_OK;
}

int jxr_random_bits(const uint32_t* keys, int64_t nkeys, uint64_t size, uint64_t begin,
                    uint64_t count, int layout, int bit_width, void* out, void* stream) {
  int rc = check_request(keys, nkeys, size, begin, count, layout, out);
  if (rc) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  switch (bit_width) {
    case 8: return launch_op(keys, nkeys, size, begin, count, layout, OpBits<8>{}, out, st);
    case 16: return launch_op(keys, nkeys, size, begin, count, layout, OpBits<16>{}, out, st);
    case 32: return launch_op(keys, nkeys, size, begin, count, layout, OpBits<32>{}, out, st);
    case 64: return launch_op(keys, nkeys, size, begin, count, layout, OpBits<64>{}, out, st);
  }
  return fail(JXR_ERR_INVALID_ARGUMENT, "requires 8-, 16-, 32- or 64-bit field width, got %d", bit_width);
}

int jxr_uniform(const uint32_t* keys, int64_t nkeys, uint64_t size, uint64_t begin, uint64_t count,
                int layout, int dtype, double minval, double maxval, uint32_t flags, void* out,
                void* stream) {
  int rc = check_dtype(dtype);
  if (rc || (rc = check_request(keys, nkeys, size, begin, count, layout, out))) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  const bool unfused = flags & JXR_FLAG_UNFUSED_MUL_ADD;
  switch (dtype) {
    case JXR_F32: {
      const float mn = (float)minval, mx = (float)maxval, d = mx - mn;
      if (unfused) return launch_op(keys, nkeys, size, begin, count, layout, OpUniformF32<false>{mn, d}, out, st);
      return launch_op(keys, nkeys, size, begin, count, layout, OpUniformF32<true>{mn, d}, out, st);
    }
    case JXR_F64: {
      const double d = maxval - minval;
      if (unfused) return launch_op(keys, nkeys, size, begin, count, layout, OpUniformF64<false>{minval, d}, out, st);
      return launch_op(keys, nkeys, size, begin, count, layout, OpUniformF64<true>{minval, d}, out, st);
    }
    case JXR_F16: {
      const float mn = to_half_value(minval, false), mx = to_half_value(maxval, false);
      const float d = to_half_value((double)mx - (double)mn, false);
      if (unfused) return launch_op(keys, nkeys, size, begin, count, layout, OpUniformH<false, false>{mn, d}, out, st);
      return launch_op(keys, nkeys, size, begin, count, layout, OpUniformH<false, true>{mn, d}, out, st);
    }
    default: {
      const float mn = to_half_value(minval, true), mx = to_half_value(maxval, true);
      const float d = to_half_value((double)mx - (double)mn, true);
      if (unfused) return launch_op(keys, nkeys, size, begin, count, layout, OpUniformH<true, false>{mn, d}, out, st);
      return launch_op(keys, nkeys, size, begin, count, layout, OpUniformH<true, true>{mn, d}, out, st);
    }
  }
}

int jxr_normal(const uint32_t* keys, int64_t nkeys, uint64_t size, uint64_t begin, uint64_t count,
               int layout, int dtype, void* out, void* stream) {
  int rc = check_dtype(dtype);
  if (rc || (rc = check_request(keys, nkeys, size, begin, count, layout, out))) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  return with_erfinv([&](auto acc) -> int {
    constexpr bool A = decltype(acc)::value;
    switch (dtype) {
      case JXR_F32: {
        if (count * (uint64_t)nkeys >= kTableMin)
          if (const float* t = f32_table(A ? kTableNormalAccurate : 0))
            return launch_table(keys, nkeys, size, begin, count, layout, t, OpNormalF32T<A>{},
                                out, st);
        return launch_op(keys, nkeys, size, begin, count, layout, OpNormalF32T<A>{}, out, st);
      }
      case JXR_F64: return launch_op(keys, nkeys, size, begin, count, layout, OpNormalF64T<A>{}, out, st);
      case JXR_F16: return launch_h(keys, nkeys, size, begin, count, layout, 2 * (A ? 5 : 4),
                                    OpNormalH<false, A>{}, out, st);
      default: return launch_h(keys, nkeys, size, begin, count, layout, 2 * (A ? 5 : 4) + 1,
                               OpNormalH<true, A>{}, out, st);
    }
  });
}

int jxr_bernoulli(const uint32_t* keys, int64_t nkeys, uint64_t size, uint64_t begin,
                  uint64_t count, int layout, int p_dtype, double p, uint8_t* out, void* stream) {
  int rc = check_dtype(p_dtype);
  if (rc || (rc = check_request(keys, nkeys, size, begin, count, layout, out))) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  switch (p_dtype) {
    case JXR_F32: return launch_op(keys, nkeys, size, begin, count, layout, OpBernoulliF32{(float)p}, out, st);
    case JXR_F64: return launch_op(keys, nkeys, size, begin, count, layout, OpBernoulliF64{p}, out, st);
    case JXR_F16: return launch_op(keys, nkeys, size, begin, count, layout, OpBernoulliH<false>{to_half_value(p, false)}, out, st);
    default: return launch_op(keys, nkeys, size, begin, count, layout, OpBernoulliH<true>{to_half_value(p, true)}, out, st);
  }
}

int jxr_normal_bernoulli(const uint32_t* keys, int64_t nkeys, uint64_t size, uint64_t begin,
                         uint64_t count, int layout, int dtype, double p, void* normal_out,
                         uint8_t* bern_out, void* stream) {
  int rc = check_dtype(dtype);
  if (rc || (rc = check_request(keys, nkeys, size, begin, count, layout, normal_out))) return rc;
  if (count && nkeys && !bern_out) return fail(JXR_ERR_INVALID_ARGUMENT, "null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == JXR_F64 && !(layout == JXR_LAYOUT_ORIGINAL && size >= 0x7FFFFFFFull)) {
    return with_erfinv([&](auto acc) -> int {
      return launch_normal_bernoulli(keys, nkeys, size, begin, count, layout,
                                     OpNormalF64T<decltype(acc)::value>{}, OpBernoulliF64{p},
                                     normal_out, bern_out, st);
    });
  }
  if (dtype == JXR_F32 && layout == JXR_LAYOUT_PARTITIONABLE)
    return with_erfinv([&](auto acc) -> int {
      return launch_normal_bernoulli(keys, nkeys, size, begin, count, layout,
                                     OpNormalF32T<decltype(acc)::value>{},
                                     OpBernoulliF32{(float)p}, normal_out, bern_out, st);
    });
  // other dtypes and layouts: the two samplers one after the other (same results)
  if ((rc = jxr_normal(keys, nkeys, size, begin, count, layout, dtype, normal_out, stream))) return rc;
  return jxr_bernoulli(keys, nkeys, size, begin, count, layout, dtype, p, bern_out, stream);
}

int jxr_uniform_from_bits(const void* bits, int64_t n, int dtype, double minval, double maxval,
                          uint32_t flags, void* out, void* stream) {
  int rc;
  if ((rc = check_dtype(dtype))) return rc;
  if (n < 0) return fail(JXR_ERR_INVALID_ARGUMENT, "n must be >= 0");
  if (!n) return JXR_OK;
  if (!bits || !out) return fail(JXR_ERR_INVALID_ARGUMENT, "null pointer");
  int grid;
  if ((rc = small_grid(n, &grid))) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  const bool unfused = flags & JXR_FLAG_UNFUSED_MUL_ADD;
if (dtype == JXR_F32) {
    const float mn = (float)minval, d = (float)maxval - mn;
    if (unfused) return launch_from_bits(bits, n, OpUniformF32<false>{mn, d}, out, st, grid);
    return launch_from_bits(bits, n, OpUniformF32<true>{mn, d}, out, st, grid);
  }
  if (dtype == JXR_F64) {
    const double d = maxval - minval;
    if (unfused) return launch_from_bits(bits, n, OpUniformF64<false>{minval, d}, out, st, grid);
    return launch_from_bits(bits, n, OpUniformF64<true>{minval, d}, out, st, grid);
  }
  const bool bf = dtype == JXR_BF16;
  const float mn = to_half_value(minval, bf), mx = to_half_value(maxval, bf);
  const float d = to_half_value((double)mx - (double)mn, bf);
  if (bf) {
    if (unfused) return launch_from_bits(bits, n, OpUniformH<true, false>{mn, d}, out, st, grid);
    return launch_from_bits(bits, n, OpUniformH<true, true>{mn, d}, out, st, grid);
  }
  if (unfused) return launch_from_bits(bits, n, OpUniformH<false, false>{mn, d}, out, st, grid);
  return launch_from_bits(bits, n, OpUniformH<false, true>{mn, d}, out, st, grid);
}

int jxr_normal_from_bits(const void* bits, int64_t n, int dtype, void* out, void* stream) {
  int rc;
  if ((rc = check_dtype(dtype))) return rc;
  if (n < 0) return fail(JXR_ERR_INVALID_ARGUMENT, "n must be >= 0");
  if (!n) return JXR_OK;
  if (!bits || !out) return fail(JXR_ERR_INVALID_ARGUMENT, "null pointer");
  int grid;
  if ((rc = small_grid(n, &grid))) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  return with_erfinv([&](auto acc) -> int {
    constexpr bool A = decltype(acc)::value;
    switch (dtype) {
      case JXR_F32:
        return launch_from_bits_table(bits, n, A ? kTableNormalAccurate : 0, 0,
                                      OpNormalF32T<A>{}, out, st, grid);
      case JXR_F64: return launch_from_bits(bits, n, OpNormalF64T<A>{}, out, st, grid);
      case JXR_F16:
        return launch_from_bits_table(bits, n, 0, 2 * (A ? 5 : 4), OpNormalH<false, A>{}, out,
                                      st, grid);
      default:
        return launch_from_bits_table(bits, n, 0, 2 * (A ? 5 : 4) + 1, OpNormalH<true, A>{},
                                      out, st, grid);
    }
  });
}

int jxr_uniform_affine(const void* unit, const void* minval, const void* maxval, int64_t n,
                       int dtype, uint32_t flags, void* out, void* stream) {
  return jxr_uniform_affine_rows(unit, minval, maxval, 1, n, dtype, flags, out, stream);
}

int jxr_uniform_affine_rows(const void* unit, const void* minval, const void* maxval,
                            int64_t nrows, int64_t n, int dtype, uint32_t flags, void* out,
                            void* stream) {
  int rc;
  if ((rc = check_dtype(dtype))) return rc;
  if (n < 0 || nrows < 0) return fail(JXR_ERR_INVALID_ARGUMENT, "n and nrows must be >= 0");
  if (!n || !nrows) return JXR_OK;
  if (!unit || !minval || !maxval || !out) return fail(JXR_ERR_INVALID_ARGUMENT, "null pointer");
  if (nrows > INT64_MAX / n) return fail(JXR_ERR_INVALID_ARGUMENT, "nrows * n overflows");
  // columns of 256-thread CTAs over a row, rows over grid.y: one wave of 8 CTAs per SM
  DeviceInfo di;
  if ((rc = device_info(&di))) return rc;
  const int64_t wave = (int64_t)di.sms * 8;
  const int64_t gx = std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, wave));
  const int64_t gy = std::max<int64_t>(1, std::min<int64_t>({nrows, std::max<int64_t>(1, wave / gx), 65535}));
  const dim3 grid((unsigned)gx, (unsigned)gy);
  cudaStream_t st = (cudaStream_t)stream;
  const bool f = !(flags & JXR_FLAG_UNFUSED_MUL_ADD);
  using U16 = const uint16_t*;
  switch (dtype) {
    case JXR_F32:
      if (f) k_affine<float, true><<<grid, 256, 0, st>>>((const float*)unit, (const float*)minval, (const float*)maxval, nrows, n, (float*)out);
      else k_affine<float, false><<<grid, 256, 0, st>>>((const float*)unit, (const float*)minval, (const float*)maxval, nrows, n, (float*)out);
      break;
    case JXR_F64:
      if (f) k_affine<double, true><<<grid, 256, 0, st>>>((const double*)unit, (const double*)minval, (const double*)maxval, nrows, n, (double*)out);
      else k_affine<double, false><<<grid, 256, 0, st>>>((const double*)unit, (const double*)minval, (const double*)maxval, nrows, n, (double*)out);
      break;
    case JXR_F16:
      if (f) k_affine_h<false, true><<<grid, 256, 0, st>>>((U16)unit, (U16)minval, (U16)maxval, nrows, n, (uint16_t*)out);
      else k_affine_h<false, false><<<grid, 256, 0, st>>>((U16)unit, (U16)minval, (U16)maxval, nrows, n, (uint16_t*)out);
      break;
    default:
      if (f) k_affine_h<true, true><<<grid, 256, 0, st>>>((U16)unit, (U16)minval, (U16)maxval, nrows, n, (uint16_t*)out);
      else k_affine_h<true, false><<<grid, 256, 0, st>>>((U16)unit, (U16)minval, (U16)maxval, nrows, n, (uint16_t*)out);
  }
  JXR_CUDA(cudaGetLastError());
  return JXR_OK;
}

int jxr_bernoulli_from_uniform(const void* u_lo, const void* u_hi, const void* p, int64_t n,
                               int dtype, uint8_t* out, void* stream) {
  int rc;
  if ((rc = check_dtype(dtype))) return rc;
  if (n < 0) return fail(JXR_ERR_INVALID_ARGUMENT, "n must be >= 0");
  if (!n) return JXR_OK;
  if (!u_lo || !p || !out) return fail(JXR_ERR_INVALID_ARGUMENT, "null pointer");
  int grid;
  if ((rc = small_grid(n, &grid))) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  using U16 = const uint16_t*;
  switch (dtype) {
    case JXR_F32:
      k_bern_unit<float><<<grid, 256, 0, st>>>((const float*)u_lo, (const float*)u_hi, (const float*)p, n, 0x1p-23f, out);
      break;
    case JXR_F64:
      k_bern_unit<double><<<grid, 256, 0, st>>>((const double*)u_lo, (const double*)u_hi, (const double*)p, n, 0x1p-52, out);
      break;
    case JXR_F16:
      k_bern_unit_h<false><<<grid, 256, 0, st>>>((U16)u_lo, (U16)u_hi, (U16)p, n, 0x1p-10f, out);
      break;
    default:
      k_bern_unit_h<true><<<grid, 256, 0, st>>>((U16)u_lo, (U16)u_hi, (U16)p, n, 0x1p-7f, out);
  }
  JXR_CUDA(cudaGetLastError());
  return JXR_OK;
}

}  // extern "C"

namespace {
// Calls f(op) with the fused op of a log-transform sampler of `kind` and `dtype`: the
// kind's uniform draw is (0, 1), (tiny, 1) or (-1 + 2^-(nmant+1), 1).
template <int K, class F>
int visit_sample_kind(int dtype, F&& f) {
  auto lo_of = [](double tiny, double epsneg) {
    return K == kExponential ? 0.0 : (K == kLaplace ? -1.0 + epsneg : tiny);
  };
  switch (dtype) {
    case JXR_F32: {
      const float mn = (float)lo_of(0x1p-126, 0x1p-24), d = 1.0f - mn;
      return f(OpLogSampler<K, 0>{{mn, d}});
    }
    case JXR_F64: {
      const double mn = lo_of(0x1p-1022, 0x1p-53), d = 1.0 - mn;
      return f(OpLogSampler<K, 1>{{mn, d}});
    }
    case JXR_F16: {
      const float mn = to_half_value(lo_of(0x1p-14, 0x1p-11), false);
      const float d = to_half_value(1.0 - (double)mn, false);
      return f(OpLogSampler<K, 2>{{{mn, d}}});
    }
    default: {
      const float mn = to_half_value(lo_of(0x1p-126, 0x1p-8), true);
      const float d = to_half_value(1.0 - (double)mn, true);
      return f(OpLogSampler<K, 3>{{{mn, d}}});
    }
  }
}

template <class F>
int visit_sample_op(int kind, int dtype, F&& f) {
  switch (kind) {
    case kExponential: return visit_sample_kind<kExponential>(dtype, f);
    case kGumbel: return visit_sample_kind<kGumbel>(dtype, f);
    case kLogistic: return visit_sample_kind<kLogistic>(dtype, f);
    case kLaplace: return visit_sample_kind<kLaplace>(dtype, f);
  }
  return fail(JXR_ERR_INVALID_ARGUMENT,
              "kind must be 0..3 (exponential, gumbel, logistic, laplace), got %d", kind);
}
}  // namespace

extern "C" {

int jxr_sample(const uint32_t* keys, int64_t nkeys, uint64_t size, uint64_t begin,
               uint64_t count, int layout, int kind, int dtype, void* out, void* stream) {
  int rc = check_dtype(dtype);
  if (rc || (rc = check_request(keys, nkeys, size, begin, count, layout, out))) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  const bool big = count * (uint64_t)nkeys >= kTableMin;
  return visit_sample_op(kind, dtype, [&](const auto& op) {
    using O = std::decay_t<decltype(op)>;
    if constexpr (std::is_same_v<typename O::Out, float>) {
      if (big)
        if (const float* t = f32_table(1 + kind))
          return launch_table(keys, nkeys, size, begin, count, layout, t, op, out, st);
    } else if constexpr (std::is_same_v<typename O::Out, uint16_t>) {
      return launch_h(keys, nkeys, size, begin, count, layout,
                      2 * kind + (dtype == JXR_BF16 ? 1 : 0), op, out, st);
    }
    return launch_op(keys, nkeys, size, begin, count, layout, op, out, st);
  });
}

int jxr_sample_from_bits(const void* bits, int64_t n, int kind, int dtype, void* out,
                         void* stream) {
  int rc = check_dtype(dtype);
  if (rc) return rc;
  if (n < 0) return fail(JXR_ERR_INVALID_ARGUMENT, "n must be >= 0");
  if (!n) return visit_sample_op(kind, dtype, [](const auto&) { return (int)JXR_OK; });
  if (!bits || !out) return fail(JXR_ERR_INVALID_ARGUMENT, "null pointer");
  int grid;
  if ((rc = small_grid(n, &grid))) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  return visit_sample_op(kind, dtype, [&](const auto& op) {
    return launch_from_bits_table(bits, n, 1 + kind, 2 * kind + (dtype == JXR_BF16 ? 1 : 0), op,
                                  out, st, grid);
  });
}

int jxr_randint(const uint32_t* keys_hi, const uint32_t* keys_lo, int64_t nkeys, uint64_t size,
                uint64_t begin, uint64_t count, int nbits, int is_signed, int64_t minval,
                int64_t maxval, int out_of_range, int out_bits, void* out, void* stream) {
  if (nbits != 32 && nbits != 64)
    return fail(JXR_ERR_INVALID_ARGUMENT, "randint samples in 32 or 64 bits, got %d", nbits);
  if (out_bits != 8 && out_bits != 16 && out_bits != 32 && out_bits != 64)
    return fail(JXR_ERR_INVALID_ARGUMENT, "out_bits must be 8, 16, 32 or 64, got %d", out_bits);
  if (out_bits > nbits)
    return fail(JXR_ERR_INVALID_ARGUMENT, "out_bits (%d) wider than the sampling width (%d)",
                out_bits, nbits);
  int rc = check_request(keys_hi, nkeys, size, begin, count, JXR_LAYOUT_PARTITIONABLE, out);
  if (rc) return rc;
  if (!count || !nkeys) return JXR_OK;
  if (!keys_lo) return fail(JXR_ERR_INVALID_ARGUMENT, "null pointer");
  // the span rules of R/random.R:343-350, in the sampling width
  const bool empty = is_signed ? (maxval <= minval) : ((uint64_t)maxval <= (uint64_t)minval);
  uint64_t span = (uint64_t)maxval - (uint64_t)minval;
  if (nbits == 32) span &= 0xFFFFFFFFull;
  if (empty) span = 1;
  else if (out_of_range) span = nbits == 32 ? ((span + 1) & 0xFFFFFFFFull) : span + 1;
  // multiplier = ((2^(nbits/2) % span)^2 mod 2^nbits) % span, as the reference's unsigned
  // lax_mul wraps
  uint64_t mult = 0;
  if (span) {
    if (nbits == 32) {
      const uint32_t m = (uint32_t)((1ull << 16) % span);
      mult = (uint32_t)(m * m) % span;
    } else {
      const uint64_t m = (1ull << 32) % span;
      mult = (m * m) % span;
    }
  }
  const uint64_t units = (count + kRandintV - 1) / kRandintV * (uint64_t)nkeys;
  int grid;
  if ((rc = resident_grid(k_randint_fused<uint32_t, uint32_t>, (units + 255) / 256, &grid)))
    return rc;
  cudaStream_t st = (cudaStream_t)stream;
#define JXR_RI(U, O)                                                                          \
  k_randint_fused<U, O><<<grid, 256, 0, st>>>(keys_hi, keys_lo, nkeys, begin, count,          \
                                              (U)(uint64_t)minval, (U)span, (U)mult, kPipe,  \
                                              (O*)out)
  if (nbits == 32) {
    switch (out_bits) {
      case 8: JXR_RI(uint32_t, uint8_t); break;
      case 16: JXR_RI(uint32_t, uint16_t); break;
      default: JXR_RI(uint32_t, uint32_t);
    }
  } else {
    JXR_RI(uint64_t, uint64_t);
  }
#undef JXR_RI
  JXR_CUDA(cudaGetLastError());
  return JXR_OK;
}

int jxr_randint_combine(const void* hi, const void* lo, int64_t n, int nbits, int is_signed,
                        const int64_t* minval, int64_t minval_stride, const int64_t* maxval,
                        int64_t maxval_stride, const uint8_t* out_of_range, int64_t oor_stride,
                        int out_bits, void* out, void* stream) {
  if (nbits != 32 && nbits != 64)
    return fail(JXR_ERR_INVALID_ARGUMENT, "randint samples in 32 or 64 bits, got %d", nbits);
  if (out_bits != 8 && out_bits != 16 && out_bits != 32 && out_bits != 64)
    return fail(JXR_ERR_INVALID_ARGUMENT, "out_bits must be 8, 16, 32 or 64, got %d", out_bits);
  if (n < 0) return fail(JXR_ERR_INVALID_ARGUMENT, "n must be >= 0");
  if (!n) return JXR_OK;
  if (!hi || !lo || !minval || !maxval || !out_of_range || !out)
    return fail(JXR_ERR_INVALID_ARGUMENT, "null pointer");
  if ((minval_stride | maxval_stride | oor_stride) & ~1ll)
    return fail(JXR_ERR_INVALID_ARGUMENT, "parameter strides must be 0 (broadcast) or 1");
  int grid, rc;
  if ((rc = small_grid(n, &grid))) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  if (nbits == 32) {
    if (is_signed)
      k_randint_combine<uint32_t, true><<<grid, 256, 0, st>>>((const uint32_t*)hi, (const uint32_t*)lo, n, minval, minval_stride, maxval, maxval_stride, out_of_range, oor_stride, out_bits, out);
    else
      k_randint_combine<uint32_t, false><<<grid, 256, 0, st>>>((const uint32_t*)hi, (const uint32_t*)lo, n, minval, minval_stride, maxval, maxval_stride, out_of_range, oor_stride, out_bits, out);
  } else {
    if (is_signed)
      k_randint_combine<uint64_t, true><<<grid, 256, 0, st>>>((const uint64_t*)hi, (const uint64_t*)lo, n, minval, minval_stride, maxval, maxval_stride, out_of_range, oor_stride, out_bits, out);
    else
      k_randint_combine<uint64_t, false><<<grid, 256, 0, st>>>((const uint64_t*)hi, (const uint64_t*)lo, n, minval, minval_stride, maxval, maxval_stride, out_of_range, oor_stride, out_bits, out);
  }
  JXR_CUDA(cudaGetLastError());
  return JXR_OK;
}

int jxr_gumbel_rows(const void* row0, const void* row1, int64_t n, int mode, int dtype,
                    void* out, void* stream) {
  int rc = check_dtype(dtype);
  if (rc) return rc;
  if (mode != 0 && mode != 1)
    return fail(JXR_ERR_INVALID_ARGUMENT, "mode must be 0 (high) or 1 (highest), got %d", mode);
  if (mode == 1 && dtype != JXR_F32)
    return fail(JXR_ERR_INVALID_ARGUMENT, "mode highest is float32 only");
  if (n < 0) return fail(JXR_ERR_INVALID_ARGUMENT, "n must be >= 0");
  if (!n) return JXR_OK;
  if (!row0 || !row1 || !out) return fail(JXR_ERR_INVALID_ARGUMENT, "null pointer");
  int grid;
  if ((rc = small_grid(n, &grid))) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  if (mode == 1) k_gumbel_rows<JXR_F32, 1><<<grid, 256, 0, st>>>(row0, row1, n, out);
  else if (dtype == JXR_F32) k_gumbel_rows<JXR_F32, 0><<<grid, 256, 0, st>>>(row0, row1, n, out);
  else if (dtype == JXR_F64) k_gumbel_rows<JXR_F64, 0><<<grid, 256, 0, st>>>(row0, row1, n, out);
  else if (dtype == JXR_F16) k_gumbel_rows<JXR_F16, 0><<<grid, 256, 0, st>>>(row0, row1, n, out);
  else k_gumbel_rows<JXR_BF16, 0><<<grid, 256, 0, st>>>(row0, row1, n, out);
  JXR_CUDA(cudaGetLastError());
  return JXR_OK;
}

namespace {
// The 16-bit float next to the 16-bit value x toward +inf (up) or -inf, on the host.
float half_step(float x, bool up, bool bf) {
  uint16_t b;
  if (bf) {
    uint32_t w;
    std::memcpy(&w, &x, 4);
    b = (uint16_t)(w >> 16);
  } else {
    b = __half_as_ushort(__float2half_rn(x));
  }
  const uint16_t inf = bf ? 0x7F80u : 0x7C00u;
  if (x != x || b == (up ? inf : (uint16_t)(0x8000u | inf))) return x;
  if ((b & 0x7FFFu) == 0) b = up ? 0x0001u : 0x8001u;
  else b = (uint16_t)((up != (bool)(b & 0x8000u)) ? b + 1 : b - 1);
  if (bf) {
    const uint32_t w = (uint32_t)b << 16;
    float f;
    std::memcpy(&f, &w, 4);
    return f;
  }
  return __half2float(__ushort_as_half(b));
}
}  // namespace

}  // extern "C"

namespace {
// Calls f(op) with the fused truncated-normal op of dtype for scalar bounds: a, b =
// erf(lower / sqrt2), erf(upper / sqrt2) and the clip bounds, computed here once.
template <bool A, class F>
int visit_trunc_op_as(int dtype, double lower, double upper, F&& f) {
  const double inf = std::numeric_limits<double>::infinity();
  switch (dtype) {
    case JXR_F32: {
      const float s2 = 1.41421354f, lo = (float)lower, hi = (float)upper;
      const float a = (float)std::erf((double)(lo / s2)), b = (float)std::erf((double)(hi / s2));
      const float cl = std::nextafter(lo, (float)inf), ch = std::nextafter(hi, (float)-inf);
      return f(OpTruncNormal<0, A>{{a, b - a}, cl, ch});
    }
    case JXR_F64: {
      const double s2 = 1.4142135623730951;
      const double a = std::erf(lower / s2), b = std::erf(upper / s2);
      return f(OpTruncNormal<1, A>{{a, b - a}, std::nextafter(lower, inf), std::nextafter(upper, -inf)});
    }
    default: {
      const bool bf = dtype == JXR_BF16;
      const float s2 = to_half_value(1.4142135623730951, bf);
      const float lo = to_half_value(lower, bf), hi = to_half_value(upper, bf);
      // the division and erf are evaluated in float32 and rounded to 16 bits
      const float ql = to_half_value((double)(lo / s2), bf), qh = to_half_value((double)(hi / s2), bf);
      const float a = to_half_value((double)(float)std::erf((double)ql), bf);
      const float b = to_half_value((double)(float)std::erf((double)qh), bf);
      const float d = to_half_value((double)b - (double)a, bf);
      const float cl = half_step(lo, true, bf), ch = half_step(hi, false, bf);
      if (bf) return f(OpTruncNormal<3, A>{{{a, d}, cl, ch}});
      return f(OpTruncNormal<2, A>{{{a, d}, cl, ch}});
    }
  }
}

template <class F>
int visit_trunc_op(int dtype, double lower, double upper, F&& f) {
  return with_erfinv([&](auto acc) -> int {
    return visit_trunc_op_as<decltype(acc)::value>(dtype, lower, upper, f);
  });
}
}  // namespace

extern "C" {

int jxr_truncated_normal(const uint32_t* keys, int64_t nkeys, uint64_t size, uint64_t begin,
                         uint64_t count, int layout, int dtype, double lower, double upper,
                         void* out, void* stream) {
  int rc = check_dtype(dtype);
  if (rc || (rc = check_request(keys, nkeys, size, begin, count, layout, out))) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  return visit_trunc_op(dtype, lower, upper, [&](const auto& op) {
    return launch_op(keys, nkeys, size, begin, count, layout, op, out, st);
  });
}

int jxr_truncated_normal_scratch(const uint32_t* keys, int64_t nkeys, uint64_t size,
                                 uint64_t begin, uint64_t count, int layout, int dtype,
                                 double lower, double upper, void* scratch, size_t scratch_bytes,
                                 void* out, void* stream) {
  int rc = check_dtype(dtype);
  if (rc || (rc = check_request(keys, nkeys, size, begin, count, layout, out))) return rc;
  const bool table = dtype == JXR_F32 && count * (uint64_t)nkeys >= kTruncTableMin && scratch &&
                     scratch_bytes >= (sizeof(float) << 23) && (uintptr_t)scratch % 16 == 0;
  const bool table16 = (dtype == JXR_F16 || dtype == JXR_BF16) &&
                       count * (uint64_t)nkeys >= kTable16Min && scratch &&
                       scratch_bytes >= 2048 && (uintptr_t)scratch % 16 == 0;
  if (table16) {
    cudaStream_t st = (cudaStream_t)stream;
    return visit_trunc_op(dtype, lower, upper, [&](const auto& op) -> int {
      using O = std::decay_t<decltype(op)>;
      if constexpr (std::is_same_v<typename O::Out, uint16_t>) {
        // this call's table: the op at all 1024 (float16) / 128 (bfloat16) draws it tells apart
        using T = OpTableH<O::kBits>;
        k_build_table16<O, T><<<(T::kEntries + 255) / 256, 256, 0, st>>>(op, (uint16_t*)scratch);
        JXR_CUDA(cudaGetLastError());
        return launch_op(keys, nkeys, size, begin, count, layout, T{(const uint16_t*)scratch}, out,
                         st);
      } else {
        return launch_op(keys, nkeys, size, begin, count, layout, op, out, st);
      }
    });
  }
  if (!table)
    return jxr_truncated_normal(keys, nkeys, size, begin, count, layout, dtype, lower, upper,
                                out, stream);
  cudaStream_t st = (cudaStream_t)stream;
  return visit_trunc_op(dtype, lower, upper, [&](const auto& op) -> int {
    using O = std::decay_t<decltype(op)>;
    if constexpr (std::is_same_v<typename O::Out, float>) {
      // this call's table: the op at all 2^23 values of bits >> 9
      k_build_table<O><<<1024, 256, 0, st>>>(op, (float*)scratch);
      JXR_CUDA(cudaGetLastError());
      return launch_table(keys, nkeys, size, begin, count, layout, (const float*)scratch, op,
                          out, st);
    } else {
      return launch_op(keys, nkeys, size, begin, count, layout, op, out, st);
    }
  });
}

int jxr_truncated_normal_from_bits(const void* bits, int64_t n, int dtype, double lower,
                                   double upper, void* out, void* stream) {
  int rc = check_dtype(dtype);
  if (rc) return rc;
  if (n < 0) return fail(JXR_ERR_INVALID_ARGUMENT, "n must be >= 0");
  if (!n) return JXR_OK;
  if (!bits || !out) return fail(JXR_ERR_INVALID_ARGUMENT, "null pointer");
  int grid;
  if ((rc = small_grid(n, &grid))) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  return visit_trunc_op(dtype, lower, upper, [&](const auto& op) {
    return launch_from_bits(bits, n, op, out, st, grid);
  });
}

int jxr_truncated_normal_from_unit(const void* unit, const void* lower, int64_t lower_stride,
                                   const void* upper, int64_t upper_stride, int64_t n, int dtype,
                                   void* out, void* stream) {
  int rc = check_dtype(dtype);
  if (rc) return rc;
  if (n < 0) return fail(JXR_ERR_INVALID_ARGUMENT, "n must be >= 0");
  if (!n) return JXR_OK;
  if (!unit || !lower || !upper || !out) return fail(JXR_ERR_INVALID_ARGUMENT, "null pointer");
  if ((lower_stride | upper_stride) & ~1ll)
    return fail(JXR_ERR_INVALID_ARGUMENT, "bound strides must be 0 (broadcast) or 1");
  int grid;
  if ((rc = small_grid(n, &grid))) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  return with_erfinv([&](auto acc) -> int {
    constexpr bool A = decltype(acc)::value;
    switch (dtype) {
      case JXR_F32: k_trunc_unit<JXR_F32, A><<<grid, 256, 0, st>>>(unit, lower, lower_stride, upper, upper_stride, n, out); break;
      case JXR_F64: k_trunc_unit<JXR_F64, A><<<grid, 256, 0, st>>>(unit, lower, lower_stride, upper, upper_stride, n, out); break;
      case JXR_F16: k_trunc_unit<JXR_F16, A><<<grid, 256, 0, st>>>(unit, lower, lower_stride, upper, upper_stride, n, out); break;
      default: k_trunc_unit<JXR_BF16, A><<<grid, 256, 0, st>>>(unit, lower, lower_stride, upper, upper_stride, n, out);
    }
    JXR_CUDA(cudaGetLastError());
    return JXR_OK;
  });
}

// ---- permutation: stable radix sort of (random key, position) pairs ----------------------

namespace jxr {
// A shuffle round's sort keys as random_bits(key, 32, n) draws them in the partitionable
// layout (element e < 2^31 hashes the counters (0, e); the key is x0 ^ x1, R/prng.R:212-226),
// and each sort tile's digit counts at `shift` for the first radix pass, in one pass: one CTA
// per tile of kSortTile keys, 16 cipher blocks in flight per thread, 16-byte stores.
__global__ void __launch_bounds__(kSortThreads)
k_sort_keys_hist(const uint32_t* __restrict__ key, int64_t n, int shift, int64_t ntiles,
                 PipeConsts pc, uint32_t* __restrict__ keys_out, uint32_t* __restrict__ counts) {
  constexpr int G = 4, V = 4, N = G * V;
  constexpr int kRound = kSortThreads * N;  // keys per round of the CTA
  static_assert(kSortThreads == 256 && kSortTile % kRound == 0, "one digit per thread");
  __shared__ uint32_t h[256];
  h[threadIdx.x] = 0;
  const KeySchedule ks = make_schedule(__ldg(key), __ldg(key + 1));
  const int64_t base = (int64_t)blockIdx.x * kSortTile;
  __syncthreads();
  for (int r = 0; r < kSortTile / kRound; ++r) {
    const int64_t p0 = base + (int64_t)r * kRound + threadIdx.x * V;
    // n < 2^31: the high counter word is 0
    uint32_t x0[N], x1[N];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int v = 0; v < V; ++v) {
        x0[g * V + v] = 0u;
        x1[g * V + v] = (uint32_t)p0 + (uint32_t)(g * kSortThreads * V + v);
      }
    threefry20<N, ProductMix>(ks, x0, x1, pc);
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const int64_t q = p0 + g * kSortThreads * V;
      uint32_t w[V];
#pragma unroll
      for (int v = 0; v < V; ++v) w[v] = x0[g * V + v] ^ x1[g * V + v];
      if (q + V <= n) {
        *reinterpret_cast<uint4*>(keys_out + q) = make_uint4(w[0], w[1], w[2], w[3]);
#pragma unroll
        for (int v = 0; v < V; ++v) atomicAdd(&h[(w[v] >> shift) & 255u], 1u);
      } else {
#pragma unroll
        for (int v = 0; v < V; ++v)
          if (q + v < n) {
            keys_out[q + v] = w[v];
            atomicAdd(&h[(w[v] >> shift) & 255u], 1u);
          }
      }
    }
  }
  __syncthreads();
  counts[(int64_t)threadIdx.x * ntiles + blockIdx.x] = h[threadIdx.x];
}

}  // namespace jxr


namespace {
int64_t sort_tiles(int64_t n) { return (n + kSortTile - 1) / kSortTile; }

struct SortScratch {
  uint32_t *ka, *kb, *va, *vb, *counts, *totals, *keys12;  // keys12: 20 words of key scratch
  int* err;
};

// Bytes of scratch for a shuffle of `total` elements; with base != nullptr also the
// pointers into it.
size_t shuffle_scratch(int64_t total, char* base, SortScratch* s) {
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += (bytes + 255) & ~(size_t)255;
    return o;
  };
  const size_t nb = (size_t)total * 4;
  const size_t o_ka = take(nb), o_kb = take(nb), o_va = take(nb), o_vb = take(nb);
  const size_t o_counts = take((size_t)256 * (size_t)sort_tiles(total) * 4);
  const size_t o_tot = take(256 * 4), o_keys = take(20 * 4), o_err = take(16);
  if (base) {
    s->ka = (uint32_t*)(base + o_ka);
    s->kb = (uint32_t*)(base + o_kb);
    s->va = (uint32_t*)(base + o_va);
    s->vb = (uint32_t*)(base + o_vb);
    s->counts = (uint32_t*)(base + o_counts);
    s->totals = (uint32_t*)(base + o_tot);
    s->keys12 = (uint32_t*)(base + o_keys);
    s->err = (int*)(base + o_err);
  }
  return off;
}

// One stable 8-bit radix pass of (k, v) by the digit at `shift` into (k2, v2); the pointers
// are swapped, so k / v hold the result.  counted: the tile counts are in s.counts already;
// iota: the values are the positions (v is not read).
int radix_pass(uint32_t*& k, uint32_t*& v, uint32_t*& k2, uint32_t*& v2, int64_t n, int shift,
               const SortScratch& s, cudaStream_t st, bool counted = false, bool iota = false) {
  const int64_t nt = sort_tiles(n);
  JXR_CUDA(cudaFuncSetAttribute(k_sort_scatter, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                kSortScatterSmem));
  // the scatter's CTAs are persistent: as many as are resident at once, or one per tile
  static int per_sm = 0;
  if (!per_sm) {
    JXR_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_sort_scatter,
                                                           kScatterThreads, kSortScatterSmem));
    per_sm = std::max(per_sm, 1);
  }
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  const int64_t grid = std::min<int64_t>(nt, (int64_t)di.sms * per_sm);
  if (!counted) k_sort_hist<<<(unsigned)nt, kSortThreads, 0, st>>>(k, n, shift, nt, s.counts);
  k_sort_scan_rows<<<256, 1024, 0, st>>>(s.counts, nt, s.totals);
  k_sort_scatter<<<(unsigned)grid, kScatterThreads, kSortScatterSmem, st>>>(
      k, iota ? nullptr : v, n, shift, nt, s.counts, s.totals, k2, v2, s.err);
  JXR_CUDA(cudaGetLastError());
  std::swap(k, k2);
  std::swap(v, v2);
  return JXR_OK;
}

// Sorts (k, v) by the low `bits` bits of k (a multiple of 8), stably; k2 / v2 are scratch
// of the same size.  On return k / v point at the sorted pairs, k2 / v2 at free buffers.
int sort_pairs(uint32_t*& k, uint32_t*& v, uint32_t*& k2, uint32_t*& v2, int64_t n, int bits,
               const SortScratch& s, cudaStream_t st, bool iota = false) {
  int rc;
  for (int shift = 0; shift < bits; shift += 8)
    if ((rc = radix_pass(k, v, k2, v2, n, shift, s, st, false, iota && shift == 0))) return rc;
  return JXR_OK;
}

// Mean bucket size (elements of equal top bits) that the span sort is given at most: a
// span is kSpanOwn positions plus the rest of the bucket running past them, so buckets well
// below kSpanCap - kSpanOwn keep every span within kSpanCap.
constexpr int64_t kSpanBucketMean = 1536;

// Radix passes over the top 8 g bits of the keys, the fewest that leave buckets of at most
// kSpanBucketMean elements on average (none when the whole array fits one span).
int span_sort_passes(int64_t n, int cap) {
  if (n <= cap) return 0;
  int g = 1;
  while (g < 3 && (n >> (8 * g)) > kSpanBucketMean) ++g;
  return g;
}

// The stable sort of a shuffle round, whose keys are uniformly random 32-bit words: radix
// passes over the top 8 g bits, then k_sort_spans sorts every bucket in shared memory.
// On return v holds the values in sorted order (k is not sorted).  A span longer than
// `cap` sets s.err[1]; the caller then repeats the shuffle with the radix passes alone.
int sort_random_keys(uint32_t*& k, uint32_t*& v, uint32_t*& k2, uint32_t*& v2, int64_t n,
                     int cap, const SortScratch& s, cudaStream_t st, bool first_counted = false,
                     bool iota = false) {
  const int g = span_sort_passes(n, cap);
  int rc;
  if (iota && !g) {  // the span sort reads the values: write the positions
    int grid;
    if ((rc = small_grid(n, &grid))) return rc;
    k_iota_u32<<<grid, 256, 0, st>>>(v, n);
  }
  for (int p = g; p >= 1; --p)
    if ((rc = radix_pass(k, v, k2, v2, n, 32 - 8 * p, s, st, first_counted && p == g,
                         iota && p == g)))
      return rc;
  JXR_CUDA(cudaFuncSetAttribute(k_sort_spans, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                kSpanSmem));
  const int64_t ctas = (n + kSpanOwn - 1) / kSpanOwn;
  k_sort_spans<<<(unsigned)ctas, kSpanThreads, kSpanSmem, st>>>(k, v, n, 32 - 8 * g, cap, v2,
                                                                s.err + 1, s.err);
  JXR_CUDA(cudaGetLastError());
  std::swap(v, v2);
  return JXR_OK;
}
}  // namespace

// Longest span k_sort_spans sorts for this host thread's shuffles (0: radix passes only).
thread_local int g_shuffle_span_cap = kSpanCap;

size_t jxr_shuffle_scratch_bytes(int64_t total) {
  if (total < 0) return 0;
  return shuffle_scratch(total, nullptr, nullptr);
}

int jxr_shuffle(const uint32_t* key, int impl, int64_t outer, int64_t n, int64_t inner,
                int layout, uint32_t* perm, void* scratch, size_t scratch_bytes, void* stream) {
  if (impl < JXR_IMPL_THREEFRY || impl > JXR_IMPL_UNSAFE_RBG)
    return fail(JXR_ERR_INVALID_ARGUMENT, "impl must be 0 (threefry2x32), 1 (rbg) or 2 "
                "(unsafe_rbg), got %d", impl);
  if (outer < 0 || n < 0 || inner < 0)
    return fail(JXR_ERR_INVALID_ARGUMENT, "outer, n and inner must be >= 0");
  if (layout != JXR_LAYOUT_ORIGINAL && layout != JXR_LAYOUT_PARTITIONABLE)
    return fail(JXR_ERR_INVALID_ARGUMENT, "layout must be 0 or 1, got %d", layout);
  if ((n && outer > INT64_MAX / n) || (n && outer && inner > INT64_MAX / (outer * n)))
    return fail(JXR_ERR_INVALID_ARGUMENT, "outer * n * inner overflows");
  const int64_t total = outer * n * inner;
  if (total > (int64_t)0x7FFFFFFF)
    return fail(JXR_ERR_INVALID_ARGUMENT,
                "shuffle of %lld elements: at most 2^31 - 1 (32-bit positions)", (long long)total);
  if (!total) return JXR_OK;
  if (!key || !perm || !scratch) return fail(JXR_ERR_INVALID_ARGUMENT, "null pointer");
  if ((uintptr_t)scratch % 256)
    return fail(JXR_ERR_INVALID_ARGUMENT, "scratch must be 256-byte aligned");
  const size_t need = shuffle_scratch(total, nullptr, nullptr);
  if (scratch_bytes < need)
    return fail(JXR_ERR_INVALID_ARGUMENT, "scratch of %zu bytes, need %zu", scratch_bytes, need);
  SortScratch s;
  shuffle_scratch(total, (char*)scratch, &s);
  cudaStream_t st = (cudaStream_t)stream;
  int grid, rc;
  if ((rc = small_grid(total, &grid))) return rc;
  // rounds = ceil(3 log(max(1, size)) / log(2^32 - 1)) (R/random.R:404-406)
  const int rounds =
      (int)std::ceil(3.0 * std::log(std::max(1.0, (double)total)) / std::log(4294967295.0));
  int segbits = 0;
  for (int64_t nseg = outer * inner; nseg > 1 && ((int64_t)1 << segbits) < nseg;) ++segbits;
  // every round: the 32-bit sort by span sort (cap > 0) or by radix passes alone (cap == 0)
  auto run = [&](int cap) -> int {
    JXR_CUDA(cudaMemsetAsync(s.err, 0, 2 * sizeof(int), st));
    // keys12: the running key (words 0..3), ks[0] (4..7), ks[1] (8..11); threefry keys use
    // the first two words of each
    const size_t kw = impl == JXR_IMPL_THREEFRY ? 8 : 16;
    JXR_CUDA(cudaMemcpyAsync(s.keys12, key, kw, cudaMemcpyDeviceToDevice, st));
    // values are original flat indices: v[f] = index of the element now at position f;
    // until the first sort writes them they are the positions themselves (iota)
    uint32_t *k = s.ka, *v = s.va, *k2 = s.kb, *v2 = s.vb;
    bool iota = true;
    for (int r = 0; r < rounds; ++r) {
      // ks = split(key); key = ks[0]; sort keys = random_bits(ks[1], 32, shape)
      uint32_t* ks0 = s.keys12 + 4;
      uint32_t* ks1 = s.keys12 + 8;
      if (impl == JXR_IMPL_THREEFRY) {
        if ((rc = jxr_split(s.keys12, 1, 2, layout, ks0, stream))) return rc;  // ks0, then ks1
        ks1 = ks0 + 2;
      } else if (impl == JXR_IMPL_RBG) {
        // each half split as a threefry key: (h0 ks0, h0 ks1, h1 ks0, h1 ks1) in tmp
        uint32_t* tmp = s.keys12 + 12;
        if ((rc = jxr_split(s.keys12, 2, 2, layout, tmp, stream))) return rc;
        JXR_CUDA(cudaMemcpyAsync(ks0, tmp, 8, cudaMemcpyDeviceToDevice, st));
        JXR_CUDA(cudaMemcpyAsync(ks0 + 2, tmp + 4, 8, cudaMemcpyDeviceToDevice, st));
        JXR_CUDA(cudaMemcpyAsync(ks1, tmp + 2, 8, cudaMemcpyDeviceToDevice, st));
        JXR_CUDA(cudaMemcpyAsync(ks1 + 2, tmp + 6, 8, cudaMemcpyDeviceToDevice, st));
      } else {  // unsafe_rbg: rows 0 and 10 of the key's (20, 4) request
        if ((rc = jxr_rbg_blocks(s.keys12, 0, 10, 2, ks0, stream))) return rc;
      }
      JXR_CUDA(cudaMemcpyAsync(s.keys12, ks0, kw, cudaMemcpyDeviceToDevice, st));
      // the default keys (threefry, partitionable) are drawn together with the counts of
      // the first radix pass
      const int g = span_sort_passes(total, cap);
      const bool fused = cap && g && impl == JXR_IMPL_THREEFRY && layout == JXR_LAYOUT_PARTITIONABLE;
      if (fused)
        k_sort_keys_hist<<<(unsigned)sort_tiles(total), kSortThreads, 0, st>>>(
            ks1, total, 32 - 8 * g, sort_tiles(total), kPipe, k, s.counts);
      else if (impl == JXR_IMPL_THREEFRY)
        rc = jxr_random_bits(ks1, 1, (uint64_t)total, 0, (uint64_t)total, layout, 32, k, stream);
      else
        rc = jxr_rbg_bits(ks1, (uint64_t)total, 0, (uint64_t)total, 32, k, nullptr, stream);
      if (rc) return rc;
      if (cap) rc = sort_random_keys(k, v, k2, v2, total, cap, s, st, fused, iota);
      else rc = sort_pairs(k, v, k2, v2, total, 32, s, st, iota);
      if (rc) return rc;
      iota = false;
      if (segbits) {  // then by segment (the slice along the middle axis), stably
        k_segment_keys<<<grid, 256, 0, st>>>(v, total, n, inner, k);
        if ((rc = sort_pairs(k, v, k2, v2, total, (segbits + 7) / 8 * 8, s, st))) return rc;
        k_shuffle_place<<<grid, 256, 0, st>>>(v, total, n, inner, v2, s.err);
        std::swap(v, v2);
      }
    }
    if (iota) k_iota_u32<<<grid, 256, 0, st>>>(v, total);  // no rounds (a single element)
    JXR_CUDA(cudaMemcpyAsync(perm, v, (size_t)total * 4, cudaMemcpyDeviceToDevice, st));
    JXR_CUDA(cudaGetLastError());
    return JXR_OK;
  };
  int flags[2] = {0, 0};
  const int cap = std::min(g_shuffle_span_cap, kSpanCap);
  if ((rc = run(cap))) return rc;
  JXR_CUDA(cudaMemcpyAsync(flags, s.err, sizeof flags, cudaMemcpyDeviceToHost, st));
  JXR_CUDA(cudaStreamSynchronize(st));
  if (flags[1] && !flags[0]) {  // a span over the cap: the whole shuffle by radix passes
    if ((rc = run(0))) return rc;
    JXR_CUDA(cudaMemcpyAsync(flags, s.err, sizeof flags, cudaMemcpyDeviceToHost, st));
    JXR_CUDA(cudaStreamSynchronize(st));
  }
  const int err = flags[0];
  if (err) return fail(JXR_ERR_CUDA, "shuffle: a bounds check in the sort failed (code %d)", err);
  return JXR_OK;
}

// ---- the shuffle of random_permutation under vmap with rbg / unsafe_rbg keys --------------

size_t jxr_shuffle_lanes_scratch_bytes(int64_t nlanes, int64_t total) {
  if (nlanes < 0 || total < 0 || (total && nlanes > INT64_MAX / 4 / total)) return 0;
  const size_t bits = ((size_t)nlanes * (size_t)total * 4 + 255) & ~(size_t)255;
  return shuffle_scratch(total, nullptr, nullptr) + bits;
}

int jxr_shuffle_lanes(const uint32_t* key, int impl, int64_t nlanes, int64_t outer, int64_t n,
                      int64_t inner, int layout, uint32_t* perm, void* scratch,
                      size_t scratch_bytes, void* stream) {
  if (impl != JXR_IMPL_RBG && impl != JXR_IMPL_UNSAFE_RBG)
    return fail(JXR_ERR_INVALID_ARGUMENT, "impl must be 1 (rbg) or 2 (unsafe_rbg), got %d "
                "(threefry lanes shuffle with their own keys: jxr_shuffle per lane)", impl);
  if (nlanes < 0 || outer < 0 || n < 0 || inner < 0)
    return fail(JXR_ERR_INVALID_ARGUMENT, "nlanes, outer, n and inner must be >= 0");
  if (layout != JXR_LAYOUT_ORIGINAL && layout != JXR_LAYOUT_PARTITIONABLE)
    return fail(JXR_ERR_INVALID_ARGUMENT, "layout must be 0 or 1, got %d", layout);
  if ((n && outer > INT64_MAX / n) || (n && outer && inner > INT64_MAX / (outer * n)))
    return fail(JXR_ERR_INVALID_ARGUMENT, "outer * n * inner overflows");
  const int64_t total = outer * n * inner;
  if (total > (int64_t)0x7FFFFFFF)
    return fail(JXR_ERR_INVALID_ARGUMENT,
                "shuffle of %lld elements: at most 2^31 - 1 (32-bit positions)", (long long)total);
  if (!total || !nlanes) return JXR_OK;
  if (nlanes > INT64_MAX / 4 / total)
    return fail(JXR_ERR_INVALID_ARGUMENT, "nlanes * total overflows");
  if (!key || !perm || !scratch) return fail(JXR_ERR_INVALID_ARGUMENT, "null pointer");
  if ((uintptr_t)scratch % 256)
    return fail(JXR_ERR_INVALID_ARGUMENT, "scratch must be 256-byte aligned");
  const size_t need = jxr_shuffle_lanes_scratch_bytes(nlanes, total);
  if (scratch_bytes < need)
    return fail(JXR_ERR_INVALID_ARGUMENT, "scratch of %zu bytes, need %zu", scratch_bytes, need);
  SortScratch s;
  const size_t sort_bytes = shuffle_scratch(total, (char*)scratch, &s);
  uint32_t* bits = (uint32_t*)((char*)scratch + sort_bytes);  // [nlanes][total]
  cudaStream_t st = (cudaStream_t)stream;
  int grid, rc;
  if ((rc = small_grid(total, &grid))) return rc;
  const int rounds =
      (int)std::ceil(3.0 * std::log(std::max(1.0, (double)total)) / std::log(4294967295.0));
  int segbits = 0;
  for (int64_t nseg = outer * inner; nseg > 1 && ((int64_t)1 << segbits) < nseg;) ++segbits;
  const size_t bytes = (size_t)total * 4;
  auto run = [&](int cap) -> int {
    JXR_CUDA(cudaMemsetAsync(s.err, 0, 2 * sizeof(int), st));
    JXR_CUDA(cudaMemcpyAsync(s.keys12, key, 16, cudaMemcpyDeviceToDevice, st));
    for (int64_t i = 0; i < nlanes; ++i) k_iota_u32<<<grid, 256, 0, st>>>(perm + i * total, total);
    for (int r = 0; r < rounds; ++r) {
      // the first lane's key is split as without vmap (an rbg key splits its halves per
      // lane, and lane 0's rows of a batched unsafe_rbg split are rows 0 and 10 of its own
      // request); every lane's sort keys are its row of one (nlanes, shape) request from the
      // first lane's ks[1]
      uint32_t* ks0 = s.keys12 + 4;
      uint32_t* ks1 = s.keys12 + 8;
      if (impl == JXR_IMPL_RBG) {
        uint32_t* tmp = s.keys12 + 12;
        if ((rc = jxr_split(s.keys12, 2, 2, layout, tmp, stream))) return rc;
        JXR_CUDA(cudaMemcpyAsync(ks0, tmp, 8, cudaMemcpyDeviceToDevice, st));
        JXR_CUDA(cudaMemcpyAsync(ks0 + 2, tmp + 4, 8, cudaMemcpyDeviceToDevice, st));
        JXR_CUDA(cudaMemcpyAsync(ks1, tmp + 2, 8, cudaMemcpyDeviceToDevice, st));
        JXR_CUDA(cudaMemcpyAsync(ks1 + 2, tmp + 6, 8, cudaMemcpyDeviceToDevice, st));
      } else {
        if ((rc = jxr_rbg_blocks(s.keys12, 0, 10, 2, ks0, stream))) return rc;
      }
      JXR_CUDA(cudaMemcpyAsync(s.keys12, ks0, 16, cudaMemcpyDeviceToDevice, st));
      const uint64_t req = (uint64_t)nlanes * (uint64_t)total;
      if ((rc = jxr_rbg_bits(ks1, req, 0, req, 32, bits, nullptr, stream))) return rc;
      for (int64_t i = 0; i < nlanes; ++i) {
        uint32_t *k = s.ka, *v = s.va, *k2 = s.kb, *v2 = s.vb;
        JXR_CUDA(cudaMemcpyAsync(k, bits + i * total, bytes, cudaMemcpyDeviceToDevice, st));
        JXR_CUDA(cudaMemcpyAsync(v, perm + i * total, bytes, cudaMemcpyDeviceToDevice, st));
        if (cap) rc = sort_random_keys(k, v, k2, v2, total, cap, s, st);
        else rc = sort_pairs(k, v, k2, v2, total, 32, s, st);
        if (rc) return rc;
        if (segbits) {  // then by segment (the slice along the middle axis), stably
          k_segment_keys<<<grid, 256, 0, st>>>(v, total, n, inner, k);
          if ((rc = sort_pairs(k, v, k2, v2, total, (segbits + 7) / 8 * 8, s, st))) return rc;
          k_shuffle_place<<<grid, 256, 0, st>>>(v, total, n, inner, v2, s.err);
          std::swap(v, v2);
        }
        JXR_CUDA(cudaMemcpyAsync(perm + i * total, v, bytes, cudaMemcpyDeviceToDevice, st));
      }
    }
    JXR_CUDA(cudaGetLastError());
    return JXR_OK;
  };
  int flags[2] = {0, 0};
  if ((rc = run(std::min(g_shuffle_span_cap, kSpanCap)))) return rc;
  JXR_CUDA(cudaMemcpyAsync(flags, s.err, sizeof flags, cudaMemcpyDeviceToHost, st));
  JXR_CUDA(cudaStreamSynchronize(st));
  if (flags[1] && !flags[0]) {  // a span over the cap: the whole shuffle by radix passes
    if ((rc = run(0))) return rc;
    JXR_CUDA(cudaMemcpyAsync(flags, s.err, sizeof flags, cudaMemcpyDeviceToHost, st));
    JXR_CUDA(cudaStreamSynchronize(st));
  }
  if (flags[0])
    return fail(JXR_ERR_CUDA, "shuffle: a bounds check in the sort failed (code %d)", flags[0]);
  return JXR_OK;
}

int jxr_take(const void* src, int64_t outer, int64_t n_src, const uint32_t* idx, int64_t n_idx,
             int64_t row_bytes, void* out, int* err, void* stream) {
  if (outer < 0 || n_src < 0 || n_idx < 0 || row_bytes < 0)
    return fail(JXR_ERR_INVALID_ARGUMENT, "sizes must be >= 0");
  if ((n_idx && outer > INT64_MAX / n_idx) ||
      (n_idx && outer && row_bytes > INT64_MAX / (outer * n_idx)) ||
      (n_src && outer > INT64_MAX / n_src) ||
      (n_src && outer && row_bytes > INT64_MAX / (outer * n_src)))
    return fail(JXR_ERR_INVALID_ARGUMENT, "outer * n * row_bytes overflows");
  const int64_t total_bytes = outer * n_idx * row_bytes;
  if (!total_bytes) return JXR_OK;
  if (!src || !idx || !out) return fail(JXR_ERR_INVALID_ARGUMENT, "null pointer");
  const uintptr_t al = (uintptr_t)src | (uintptr_t)out | (uintptr_t)row_bytes;
  cudaStream_t st = (cudaStream_t)stream;
  int grid, rc;
#define JXR_TAKE(T)                                                                           \
  {                                                                                           \
    const int64_t row = row_bytes / (int64_t)sizeof(T);                                       \
    if ((rc = small_grid(outer * n_idx * row, &grid))) return rc;                             \
    k_take_rows<T><<<grid, 256, 0, st>>>((const T*)src, outer, n_src, idx, n_idx, row,         \
                                         (T*)out, err);                                       \
  }
  if (al % 16 == 0) JXR_TAKE(uint4)
  else if (al % 8 == 0) JXR_TAKE(uint2)
  else if (al % 4 == 0) JXR_TAKE(uint32_t)
  else if (al % 2 == 0) JXR_TAKE(uint16_t)
  else JXR_TAKE(uint8_t)
#undef JXR_TAKE
  JXR_CUDA(cudaGetLastError());
  return JXR_OK;
}

int jxr_choice_p_from_unit(const void* unit, int64_t n, int dtype, const void* cuml, int64_t m,
                           int out_bits, void* out, void* stream) {
  if (dtype != JXR_F32 && dtype != JXR_F64)
    return fail(JXR_ERR_INVALID_ARGUMENT, "dtype must be float32 or float64, got %d", dtype);
  if (out_bits != 32 && out_bits != 64)
    return fail(JXR_ERR_INVALID_ARGUMENT, "out_bits must be 32 or 64, got %d", out_bits);
  if (n < 0 || m < 1) return fail(JXR_ERR_INVALID_ARGUMENT, "n must be >= 0 and m >= 1");
  if (!n) return JXR_OK;
  if (!unit || !cuml || !out) return fail(JXR_ERR_INVALID_ARGUMENT, "null pointer");
  int grid, rc;
  if ((rc = small_grid(n, &grid))) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == JXR_F32)
    k_choice_p<float><<<grid, 256, 0, st>>>((const float*)unit, n, (const float*)cuml, m, out_bits, out);
  else
    k_choice_p<double><<<grid, 256, 0, st>>>((const double*)unit, n, (const double*)cuml, m, out_bits, out);
  JXR_CUDA(cudaGetLastError());
  return JXR_OK;
}

int jxr_add_log(void* x, const void* p, int64_t n, int dtype, void* stream) {
  if (dtype != JXR_F32 && dtype != JXR_F64)
    return fail(JXR_ERR_INVALID_ARGUMENT, "dtype must be float32 or float64, got %d", dtype);
  if (n < 0) return fail(JXR_ERR_INVALID_ARGUMENT, "n must be >= 0");
  if (!n) return JXR_OK;
  if (!x || !p) return fail(JXR_ERR_INVALID_ARGUMENT, "null pointer");
  int grid, rc;
  if ((rc = small_grid(n, &grid))) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == JXR_F32) k_add_log<float><<<grid, 256, 0, st>>>((float*)x, (const float*)p, n);
  else k_add_log<double><<<grid, 256, 0, st>>>((double*)x, (const double*)p, n);
  JXR_CUDA(cudaGetLastError());
  return JXR_OK;
}

size_t jxr_argsort_scratch_bytes(int64_t n) { return jxr_shuffle_scratch_bytes(n); }

int jxr_argsort_float(const void* x, int64_t n, int dtype, int descending, uint32_t* idx,
                      void* scratch, size_t scratch_bytes, void* stream) {
  if (dtype != JXR_F32 && dtype != JXR_F64)
    return fail(JXR_ERR_INVALID_ARGUMENT, "dtype must be float32 or float64, got %d", dtype);
  if (n < 0 || n > (int64_t)0x7FFFFFFF)
    return fail(JXR_ERR_INVALID_ARGUMENT, "n must be in [0, 2^31 - 1]");
  if (!n) return JXR_OK;
  if (!x || !idx || !scratch) return fail(JXR_ERR_INVALID_ARGUMENT, "null pointer");
  if ((uintptr_t)scratch % 256)
    return fail(JXR_ERR_INVALID_ARGUMENT, "scratch must be 256-byte aligned");
  const size_t need = shuffle_scratch(n, nullptr, nullptr);
  if (scratch_bytes < need)
    return fail(JXR_ERR_INVALID_ARGUMENT, "scratch of %zu bytes, need %zu", scratch_bytes, need);
  SortScratch s;
  shuffle_scratch(n, (char*)scratch, &s);
  cudaStream_t st = (cudaStream_t)stream;
  int grid, rc;
  if ((rc = small_grid(n, &grid))) return rc;
  JXR_CUDA(cudaMemsetAsync(s.err, 0, sizeof(int), st));
  // keys: ka = high (or only) word, kb = low word of float64
  if (dtype == JXR_F32) k_float_sort_keys<false><<<grid, 256, 0, st>>>(x, n, descending != 0, s.ka, s.kb);
  else k_float_sort_keys<true><<<grid, 256, 0, st>>>(x, n, descending != 0, s.ka, s.kb);
  uint32_t *k, *v = s.va, *k2, *v2 = s.vb;
  k_iota_u32<<<grid, 256, 0, st>>>(v, n);
  if (dtype == JXR_F64) {
    // LSD: by the low word, then the high words (gathered into the new order) stably
    k = s.kb;
    k2 = idx;  // free until the end: holds one ping-pong buffer of keys
    if ((rc = sort_pairs(k, v, k2, v2, n, 32, s, st))) return rc;
    uint32_t* hi_sorted = (k == s.kb) ? idx : s.kb;
    k_gather_u32<<<grid, 256, 0, st>>>(s.ka, v, n, hi_sorted);
    k = hi_sorted;
    k2 = s.ka;
  } else {
    k = s.ka;
    k2 = s.kb;
  }
  if ((rc = sort_pairs(k, v, k2, v2, n, 32, s, st))) return rc;
  JXR_CUDA(cudaMemcpyAsync(idx, v, (size_t)n * 4, cudaMemcpyDeviceToDevice, st));
  JXR_CUDA(cudaGetLastError());
  int err = 0;
  JXR_CUDA(cudaMemcpyAsync(&err, s.err, sizeof(int), cudaMemcpyDeviceToHost, st));
  JXR_CUDA(cudaStreamSynchronize(st));
  if (err) return fail(JXR_ERR_CUDA, "argsort: a bounds check in the sort failed (code %d)", err);
  return JXR_OK;
}

int jxr_rbg_bits(const uint32_t* key, uint64_t size, uint64_t begin, uint64_t count, int bit_width,
                 void* out, uint32_t* new_key, void* stream) {
  if (bit_width != 8 && bit_width != 16 && bit_width != 32 && bit_width != 64)
    return fail(JXR_ERR_INVALID_ARGUMENT, "bit_width must be 8, 16, 32 or 64, got %d", bit_width);
  if (begin > size || count > size - begin)
    return fail(JXR_ERR_INVALID_ARGUMENT, "range [%llu, +%llu) outside a request of %llu",
                (unsigned long long)begin, (unsigned long long)count, (unsigned long long)size);
  if (!key) return fail(JXR_ERR_INVALID_ARGUMENT, "null key");
  if (count && !out) return fail(JXR_ERR_INVALID_ARGUMENT, "null output");
  cudaStream_t st = (cudaStream_t)stream;
  if (new_key) {  // the state after the request: counter + ceil(size / outputs per block)
    const uint64_t per = bit_width == 64 ? 2 : 4;
    k_rbg_advance<<<1, 32, 0, st>>>(key, (size + per - 1) / per, new_key);
  }
  if (count) {
    const uint64_t per = bit_width == 64 ? 2 : 4, g = bit_width == 8 ? 4 : bit_width == 16 ? 2 : 1;
    const uint64_t blocks = (begin + count + per - 1) / per - begin / per;
    const uint64_t ctas = ((blocks + g - 1) / g + 255) / 256;  // one group of blocks per thread
    int grid, rc;
    if ((rc = resident_grid(k_rbg_bits<32>, ctas, &grid))) return rc;
    switch (bit_width) {
      case 8: k_rbg_bits<8><<<grid, 256, 0, st>>>(key, begin, count, out); break;
      case 16: k_rbg_bits<16><<<grid, 256, 0, st>>>(key, begin, count, out); break;
      case 32: k_rbg_bits<32><<<grid, 256, 0, st>>>(key, begin, count, out); break;
      default: k_rbg_bits<64><<<grid, 256, 0, st>>>(key, begin, count, out);
    }
  }
  JXR_CUDA(cudaGetLastError());
  return JXR_OK;
}

int jxr_rbg_blocks(const uint32_t* key, uint64_t first, uint64_t stride, int64_t n, uint32_t* out,
                   void* stream) {
  if (n < 0) return fail(JXR_ERR_INVALID_ARGUMENT, "n must be >= 0");
  if (!n) return JXR_OK;
  if (!key || !out) return fail(JXR_ERR_INVALID_ARGUMENT, "null pointer");
  if ((uintptr_t)out % 16) return fail(JXR_ERR_INVALID_ARGUMENT, "out must be 16-byte aligned");
  int grid, rc;
  if ((rc = small_grid(n, &grid))) return rc;
  k_rbg_blocks<<<grid, 256, 0, (cudaStream_t)stream>>>(key, first, stride, n, out);
  JXR_CUDA(cudaGetLastError());
  return JXR_OK;
}

int jxr_rbg_unsafe_fold_in(const uint32_t* keys, int64_t nkeys, const uint32_t* data, int64_t ndata,
                           int lanes_from_first, uint32_t* out, void* stream) {
  if (nkeys < 1 || ndata < 1 || (nkeys != ndata && nkeys != 1 && ndata != 1))
    return fail(JXR_ERR_INVALID_ARGUMENT, "nkeys (%lld) and ndata (%lld) do not broadcast",
                (long long)nkeys, (long long)ndata);
  if (!keys || !data || !out) return fail(JXR_ERR_INVALID_ARGUMENT, "null pointer");
  if ((uintptr_t)out % 16) return fail(JXR_ERR_INVALID_ARGUMENT, "out must be 16-byte aligned");
  const int64_t n = std::max(nkeys, ndata);
  int grid, rc;
  if ((rc = small_grid(n, &grid))) return rc;
  k_rbg_unsafe_fold_in<<<grid, 256, 0, (cudaStream_t)stream>>>(keys, nkeys, data, ndata, n,
                                                               lanes_from_first, out);
  JXR_CUDA(cudaGetLastError());
  return JXR_OK;
}

int jxr_random_bits_multi(const int* devices, int ndev, const uint32_t* const* keys, uint64_t size,
                          int layout, int bit_width, void* const* outs, int gather_to,
                          void* gather_out, void* const* streams) {
  if (ndev < 1 || !devices || !keys)
    return fail(JXR_ERR_INVALID_ARGUMENT, "need ndev >= 1 devices and their keys");
  if (gather_to >= ndev) return fail(JXR_ERR_INVALID_ARGUMENT, "gather_to must be < ndev");
  if (gather_to >= 0 ? !gather_out && size : !outs)
    return fail(JXR_ERR_INVALID_ARGUMENT, "null output");
  if (bit_width != 8 && bit_width != 16 && bit_width != 32 && bit_width != 64)
    return fail(JXR_ERR_INVALID_ARGUMENT, "bit_width must be 8, 16, 32 or 64, got %d", bit_width);
  int prev = 0;
  JXR_CUDA(cudaGetDevice(&prev));
  int rc = JXR_OK;
  for (int i = 0; i < ndev && rc == JXR_OK; ++i) {
    // slab bounds in 128 bits: size * i overflows 64 bits for requests above 2^61
    const uint64_t lo = (uint64_t)((unsigned __int128)size * (unsigned)i / (unsigned)ndev);
    const uint64_t hi = (uint64_t)((unsigned __int128)size * (unsigned)(i + 1) / (unsigned)ndev);
    if (cudaSetDevice(devices[i]) != cudaSuccess) {
      rc = fail(JXR_ERR_CUDA, "cannot select device %d", devices[i]);
      break;
    }
    void* dst;
    if (gather_to >= 0) {
      const int root = devices[gather_to];
      if (root != devices[i]) {  // this device stores straight into the root's buffer
        int can = 0;
        cudaDeviceCanAccessPeer(&can, devices[i], root);
        if (!can) {
          rc = fail(JXR_ERR_CUDA, "device %d cannot access device %d's memory", devices[i], root);
          break;
        }
        const cudaError_t e = cudaDeviceEnablePeerAccess(root, 0);
        if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled) {
          rc = fail(JXR_ERR_CUDA, "peer access %d -> %d: %s", devices[i], root, cudaGetErrorString(e));
          break;
        }
        cudaGetLastError();  // clear "already enabled"
      }
      dst = (char*)gather_out + lo * (uint64_t)(bit_width / 8);
    } else {
      dst = outs[i];
    }
    rc = jxr_random_bits(keys[i], 1, size, lo, hi - lo, layout, bit_width, dst,
                         streams ? streams[i] : nullptr);
  }
  cudaSetDevice(prev);
  return rc;
}

int jxr_complex_from_parts(const void* re, const void* im, int64_t n, int dtype, double divisor,
                           void* out, void* stream) {
  if (dtype != JXR_F32 && dtype != JXR_F64)
    return fail(JXR_ERR_INVALID_ARGUMENT, "dtype must be float32 or float64, got %d", dtype);
  if (n < 0) return fail(JXR_ERR_INVALID_ARGUMENT, "n must be >= 0");
  if (!n) return JXR_OK;
  if (!re || !im || !out) return fail(JXR_ERR_INVALID_ARGUMENT, "null pointer");
  int grid, rc;
  if ((rc = small_grid(n, &grid))) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == JXR_F32)
    k_complex_div<float><<<grid, 256, 0, st>>>((const float*)re, (const float*)im, n, (float)divisor, (float*)out);
  else
    k_complex_div<double><<<grid, 256, 0, st>>>((const double*)re, (const double*)im, n, divisor, (double*)out);
  JXR_CUDA(cudaGetLastError());
  return JXR_OK;
}

int jxr_cumsum(const void* x, int64_t m, int dtype, void* out, void* stream) {
  if (dtype != JXR_F32 && dtype != JXR_F64)
    return fail(JXR_ERR_INVALID_ARGUMENT, "dtype must be float32 or float64, got %d", dtype);
  if (m < 0) return fail(JXR_ERR_INVALID_ARGUMENT, "m must be >= 0");
  if (!m) return JXR_OK;
  if (!x || !out) return fail(JXR_ERR_INVALID_ARGUMENT, "null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == JXR_F32) k_cumsum_seq<float><<<1, 32, 0, st>>>((const float*)x, m, (float*)out);
  else k_cumsum_seq<double><<<1, 32, 0, st>>>((const double*)x, m, (double*)out);
  JXR_CUDA(cudaGetLastError());
  return JXR_OK;
}

int jxr_erf_inv(const void* x, int64_t n, int dtype, void* out, void* stream) {
  if (dtype != JXR_F32 && dtype != JXR_F64)
    return fail(JXR_ERR_INVALID_ARGUMENT, "erf_inv supports dtype 0 (f32) or 1 (f64), got %d", dtype);
  if (n < 0) return fail(JXR_ERR_INVALID_ARGUMENT, "n must be >= 0");
  if (!n) return JXR_OK;
  if (!x || !out) return fail(JXR_ERR_INVALID_ARGUMENT, "null pointer");
  int grid, rc;
  if ((rc = small_grid(n, &grid))) return rc;
  return with_erfinv([&](auto acc) -> int {
    constexpr bool A = decltype(acc)::value;
    if (dtype == JXR_F32)
      k_erfinv_f32<A><<<grid, 256, 0, (cudaStream_t)stream>>>((const float*)x, n, (float*)out);
    else
      k_erfinv_f64<A><<<grid, 256, 0, (cudaStream_t)stream>>>((const double*)x, n, (double*)out);
    JXR_CUDA(cudaGetLastError());
    return JXR_OK;
  });
}

int jxr_free_caches(void) {
  int dev = 0;
  JXR_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(JXR_ERR_NO_DEVICE, "device index %d out of range", dev);
  // tables may still be read by kernels in flight on any stream of this device
  JXR_CUDA(cudaDeviceSynchronize());
  {
    std::lock_guard<std::mutex> lock(g_tab_mu);
    for (int id = 0; id < kTables; ++id) {
      if (g_tables[dev][id]) cudaFree(g_tables[dev][id]);
      g_tables[dev][id] = nullptr;
    }
    for (int id = 0; id < kTables16; ++id) {
      if (g_tables16[dev][id]) cudaFree(g_tables16[dev][id]);
      g_tables16[dev][id] = nullptr;
    }
  }
  {
    std::lock_guard<std::mutex> lock(g_static_scratch_mu);
    g_static_scratch_addr[dev] = nullptr;
  }
  HostCopyCtx& cx = g_host_ctx[dev];
  std::lock_guard<std::mutex> lock(cx.mu);
  cx.release();
  JXR_CUDA(cudaGetLastError());
  return JXR_OK;
}

int jxr_prepare_device(uint32_t what, void* stream) {
  if (what & ~(uint32_t)JXR_PREPARE_ALL)
    return fail(JXR_ERR_INVALID_ARGUMENT, "unknown bits 0x%x in what (JXR_PREPARE_ALL is 0x%x)",
                what & ~(uint32_t)JXR_PREPARE_ALL, (unsigned)JXR_PREPARE_ALL);
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  int dev = 0;
  JXR_CUDA(cudaGetDevice(&dev));
  cudaStream_t st = (cudaStream_t)stream;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  JXR_CUDA(cudaStreamIsCapturing(st, &cap));
  if (cap != cudaStreamCaptureStatusNone)
    return fail(JXR_ERR_INVALID_ARGUMENT,
                "jxr_prepare_device allocates and waits for its stream: call it outside stream "
                "capture");
  // Looking the array up makes the runtime load this library's module on the device now
  // (CUDA loads modules lazily), which is when the module's fixed arrays are created, and
  // the kernels of jxr_random_bits_host_static are loaded too; every call does this,
  // whatever `what` asks for.
  unsigned char* scratch = nullptr;
  if ((rc = static_scratch(dev, &scratch)) || (rc = preload_bits_kernels<8>()) ||
      (rc = preload_bits_kernels<16>()) || (rc = preload_bits_kernels<32>()) ||
      (rc = preload_bits_kernels<64>()))
    return rc;
  std::lock_guard<std::mutex> lock(g_tab_mu);
  if (what & JXR_PREPARE_TABLE_NORMAL) {
    if ((rc = build_f32_table(dev, 0, OpNormalF32T<false>{}, st)) ||
        (rc = build_h16_table(dev, 2 * 4, OpNormalH<false, false>{}, st)) ||
        (rc = build_h16_table(dev, 2 * 4 + 1, OpNormalH<true, false>{}, st)))
      return rc;
  }
  if (what & JXR_PREPARE_TABLE_NORMAL_ACCURATE) {
    if ((rc = build_f32_table(dev, kTableNormalAccurate, OpNormalF32T<true>{}, st)) ||
        (rc = build_h16_table(dev, 2 * 5, OpNormalH<false, true>{}, st)) ||
        (rc = build_h16_table(dev, 2 * 5 + 1, OpNormalH<true, true>{}, st)))
      return rc;
  }
  for (int kind = 0; kind < 4; ++kind) {
    if (!(what & ((uint32_t)JXR_PREPARE_TABLE_EXPONENTIAL << kind))) continue;
    for (int dtype : {JXR_F32, JXR_F16, JXR_BF16}) {
      rc = visit_sample_op(kind, dtype, [&](const auto& op) -> int {
        using O = std::decay_t<decltype(op)>;
        if constexpr (std::is_same_v<typename O::Out, float>)
          return build_f32_table(dev, 1 + kind, op, st);
        else if constexpr (std::is_same_v<typename O::Out, uint16_t>)
          return build_h16_table(dev, 2 * kind + (dtype == JXR_BF16 ? 1 : 0), op, st);
        else
          return JXR_OK;
      });
      if (rc) return rc;
    }
  }
  return JXR_OK;
}

int jxr_set_accurate_erf_inv(int enable) {
  const int prev = g_accurate_erf_inv;
  g_accurate_erf_inv = enable ? 1 : 0;
  return prev;
}

int jxr_get_accurate_erf_inv(void) { return g_accurate_erf_inv; }

int jxr_set_shuffle_span_cap(int cap) {
  if (cap < 0 || cap > kSpanCap) {
    fail(JXR_ERR_INVALID_ARGUMENT, "span cap must be in [0, %d], got %d", kSpanCap, cap);
    return -1;
  }
  const int prev = g_shuffle_span_cap;
  g_shuffle_span_cap = cap;
  return prev;
}

int jxr_random_bits_host(const uint32_t* keys_host, int64_t nkeys, uint64_t size, uint64_t begin,
                         uint64_t count, int layout, int bit_width, void* host_out) {
  int rc = check_request(keys_host, nkeys, size, begin, count, layout, host_out);
  if (rc) return rc;
  if (bit_width != 8 && bit_width != 16 && bit_width != 32 && bit_width != 64)
    return fail(JXR_ERR_INVALID_ARGUMENT, "requires 8-, 16-, 32- or 64-bit field width, got %d", bit_width);
  if (!count || !nkeys) return JXR_OK;
  int dev = 0;
  JXR_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(JXR_ERR_NO_DEVICE, "device index %d out of range", dev);
  HostCopyCtx& cx = g_host_ctx[dev];
  std::lock_guard<std::mutex> lock(cx.mu);
  if ((rc = cx.ensure((size_t)nkeys))) return rc;
  const size_t esz = (size_t)bit_width / 8;
  const uint64_t chunk = kStageBytes / esz;
  JXR_CUDA(cudaMemcpyAsync(cx.dkeys, keys_host, 8 * (size_t)nkeys, cudaMemcpyHostToDevice, cx.gen));
  int status = JXR_OK;
  int buf = 0;
  uint64_t issued = 0;
  for (int64_t r = 0; r < nkeys && status == JXR_OK; ++r) {
    for (uint64_t off = 0; off < count && status == JXR_OK; off += chunk, ++issued) {
      const uint64_t n = std::min(chunk, count - off);
      // the staging buffer is free once the copy issued two chunks ago has finished
      if (issued >= 2 && cudaStreamWaitEvent(cx.gen, cx.freed[buf], 0) != cudaSuccess) {
        status = fail(JXR_ERR_CUDA, "cudaStreamWaitEvent failed");
        break;
      }
      if ((status = jxr_random_bits(cx.dkeys + 2 * r, 1, size, begin + off, n, layout, bit_width,
                                    cx.stage[buf], cx.gen)))
        break;
      char* dst = (char*)host_out + ((uint64_t)r * count + off) * esz;
      cudaError_t e = cudaEventRecord(cx.done[buf], cx.gen);
      if (e == cudaSuccess) e = cudaStreamWaitEvent(cx.cpy, cx.done[buf], 0);
      if (e == cudaSuccess) e = cudaMemcpyAsync(dst, cx.stage[buf], n * esz, cudaMemcpyDeviceToHost, cx.cpy);
      if (e == cudaSuccess) e = cudaEventRecord(cx.freed[buf], cx.cpy);
      if (e != cudaSuccess) status = fail(JXR_ERR_CUDA, "staged copy: %s", cudaGetErrorString(e));
      buf ^= 1;
    }
  }
  cudaError_t e1 = cudaStreamSynchronize(cx.cpy), e2 = cudaStreamSynchronize(cx.gen);
  if (status == JXR_OK && (e1 != cudaSuccess || e2 != cudaSuccess))
    status = fail(JXR_ERR_CUDA, "cudaStreamSynchronize: %s",
                  cudaGetErrorString(e1 != cudaSuccess ? e1 : e2));
  return status;
}

int jxr_probe_cipher(uint64_t iters, int ctas_per_sm, uint32_t* sink, uint64_t* blocks_out,
                     void* stream) {
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  if (ctas_per_sm < 1 || ctas_per_sm > 8)
    return fail(JXR_ERR_INVALID_ARGUMENT, "ctas_per_sm must be in [1, 8], got %d", ctas_per_sm);
  if (!sink || !blocks_out) return fail(JXR_ERR_INVALID_ARGUMENT, "null pointer");
  const int grid = di.sms * ctas_per_sm;
  k_probe_cipher<<<grid, kThreads, 0, (cudaStream_t)stream>>>(iters, sink, kPipe);
  JXR_CUDA(cudaGetLastError());
  *blocks_out = (uint64_t)grid * kThreads * 8ull * iters;
  return JXR_OK;
}

int jxr_random_bits_host_static(const uint32_t* keys_host, int64_t nkeys, uint64_t size,
                                uint64_t begin, uint64_t count, int layout, int bit_width,
                                void* host_out, void* stream) {
  int rc = check_request(keys_host, nkeys, size, begin, count, layout, host_out);
  if (rc) return rc;
  if (bit_width != 8 && bit_width != 16 && bit_width != 32 && bit_width != 64)
    return fail(JXR_ERR_INVALID_ARGUMENT, "requires 8-, 16-, 32- or 64-bit field width, got %d", bit_width);
  if (nkeys > kStaticMaxKeys)
    return fail(JXR_ERR_INVALID_ARGUMENT,
                "jxr_random_bits_host_static takes at most %lld keys per call (its fixed device "
                "scratch holds %lld), got %lld; split the batch or use jxr_random_bits_host",
                (long long)kStaticMaxKeys, (long long)kStaticMaxKeys, (long long)nkeys);
  if (!count || !nkeys) return JXR_OK;
  int dev = 0;
  JXR_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(JXR_ERR_NO_DEVICE, "device index %d out of range", dev);
  std::lock_guard<std::mutex> call_lock(g_static_call_mu[dev]);
  unsigned char* scratch = nullptr;
  if ((rc = static_scratch(dev, &scratch))) return rc;
  uint32_t* dkeys = (uint32_t*)scratch;
  void* stage = scratch + kStaticKeyBytes;
  cudaStream_t st = (cudaStream_t)stream;
  const size_t esz = (size_t)bit_width / 8;
  const uint64_t chunk = kStaticStageBytes / esz;
  // Everything is ordered on the caller's stream: the staging buffer is regenerated only
  // after the copy of the previous chunk out of it has run.
  JXR_CUDA(cudaMemcpyAsync(dkeys, keys_host, 8 * (size_t)nkeys, cudaMemcpyHostToDevice, st));
  for (int64_t r = 0; r < nkeys && rc == JXR_OK; ++r) {
    for (uint64_t off = 0; off < count; off += chunk) {
      const uint64_t n = std::min(chunk, count - off);
      if ((rc = jxr_random_bits(dkeys + 2 * r, 1, size, begin + off, n, layout, bit_width, stage,
                                stream)))
        break;
      char* dst = (char*)host_out + ((uint64_t)r * count + off) * esz;
      cudaError_t e = cudaMemcpyAsync(dst, stage, n * esz, cudaMemcpyDeviceToHost, st);
      if (e != cudaSuccess) {
        rc = fail(JXR_ERR_CUDA, "cudaMemcpyAsync: %s", cudaGetErrorString(e));
        break;
      }
    }
  }
  // also on failure: copies already queued into host_out finish before the call returns
  cudaError_t e = cudaStreamSynchronize(st);
  if (rc == JXR_OK && e != cudaSuccess)
    rc = fail(JXR_ERR_CUDA, "cudaStreamSynchronize: %s", cudaGetErrorString(e));
  return rc;
}

// ---- device memory shared between the processes of one node (CUDA IPC) -------------------

int jxr_ipc_export(const void* dev_ptr, void* handle, uint64_t* offset) {
  if (!dev_ptr || !handle || !offset) return fail(JXR_ERR_INVALID_ARGUMENT, "null pointer");
  using AddrRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
  static AddrRangeFn addr_range = nullptr;
  if (!addr_range) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    JXR_CUDA(cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q));
    if (!fn || q != cudaDriverEntryPointSuccess)
      return fail(JXR_ERR_CUDA, "cuMemGetAddressRange is not available from the driver");
    addr_range = (AddrRangeFn)fn;
  }
  CUdeviceptr base = 0;
  size_t bytes = 0;
  if (addr_range(&base, &bytes, (CUdeviceptr)dev_ptr) != CUDA_SUCCESS)
    return fail(JXR_ERR_INVALID_ARGUMENT, "pointer %p is not device memory", dev_ptr);
  cudaIpcMemHandle_t h;
  JXR_CUDA(cudaIpcGetMemHandle(&h, (void*)base));
  std::memcpy(handle, &h, sizeof h);
  *offset = (uint64_t)((CUdeviceptr)dev_ptr - base);
  return JXR_OK;
}

int jxr_ipc_open(const void* handle, void** base_out) {
  if (!handle || !base_out) return fail(JXR_ERR_INVALID_ARGUMENT, "null pointer");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof h);
  JXR_CUDA(cudaIpcOpenMemHandle(base_out, h, cudaIpcMemLazyEnablePeerAccess));
  return JXR_OK;
}

int jxr_ipc_close(void* base) {
  if (!base) return fail(JXR_ERR_INVALID_ARGUMENT, "null pointer");
  JXR_CUDA(cudaIpcCloseMemHandle(base));
  return JXR_OK;
}

}  // extern "C"

