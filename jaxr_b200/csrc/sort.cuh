// Stable LSD radix sort of (uint32 key, uint32 value) pairs and the shuffle built on it
// (random_permutation, R/random.R:378-413).
//
// rnd_shuffle sorts the array by fresh 32-bit random keys, num_rounds times, with a
// stable key-value sort (lax_sort_key_val).  Here every round sorts (key, position)
// pairs: 8 bits per pass, each pass a histogram kernel, a scan of the per-tile counts and
// a scatter.  The scatter ranks a tile's elements stably (per warp and chunk of 32, the
// lanes of equal digit from bits ORed into shared memory, running counts per warp),
// places them by digit in shared memory and writes each digit's run to its global
// offset, so the global stores are contiguous runs.
#pragma once

#include <cstdint>

namespace jxr {

constexpr int kSortThreads = 256;  // histogram CTAs
constexpr int kSortItems = 32;
constexpr int kSortTile = kSortThreads * kSortItems;  // 8192 elements per tile
constexpr int kScatterThreads = 512;                  // scatter CTAs: 16 warps per tile
constexpr int kScatterWarps = kScatterThreads / 32;
// dynamic shared memory of the scatter: keys and values of a tile, per warp the running
// digit counts and the lane masks of one chunk, three 256-entry tables
constexpr int kSortScatterSmem = 2 * kSortTile * 4 + 2 * kScatterWarps * 256 * 4 + 3 * 256 * 4;

// counts[d * ntiles + t] = number of keys of tile t whose digit at `shift` is d
__global__ void __launch_bounds__(kSortThreads)
k_sort_hist(const uint32_t* __restrict__ keys, int64_t n, int shift, int64_t ntiles,
            uint32_t* __restrict__ counts) {
  __shared__ uint32_t h[256];
  h[threadIdx.x] = 0;
  const int64_t base = (int64_t)blockIdx.x * kSortTile;
  const int64_t rem = n - base;
  const int cnt = rem < kSortTile ? (int)rem : kSortTile;
  // 16-byte loads when the buffer allows (tiles start 32 KiB apart, so the tile has the
  // buffer's alignment); scalar loads for the rest
  const int nvec = ((uintptr_t)keys & 15u) == 0 ? cnt / 4 : 0;
  const uint4* k4 = reinterpret_cast<const uint4*>(keys + base);
  uint4 q[kSortItems / 4];
#pragma unroll
  for (int j = 0; j < kSortItems / 4; ++j) {
    const int v = j * kSortThreads + threadIdx.x;
    q[j] = v < nvec ? k4[v] : make_uint4(0u, 0u, 0u, 0u);
  }
  __syncthreads();
#pragma unroll
  for (int j = 0; j < kSortItems / 4; ++j) {
    if (j * kSortThreads + (int)threadIdx.x < nvec) {
      atomicAdd(&h[(q[j].x >> shift) & 255u], 1u);
      atomicAdd(&h[(q[j].y >> shift) & 255u], 1u);
      atomicAdd(&h[(q[j].z >> shift) & 255u], 1u);
      atomicAdd(&h[(q[j].w >> shift) & 255u], 1u);
    }
  }
  for (int i = nvec * 4 + threadIdx.x; i < cnt; i += kSortThreads)
    atomicAdd(&h[(keys[base + i] >> shift) & 255u], 1u);
  __syncthreads();
  counts[(int64_t)threadIdx.x * ntiles + blockIdx.x] = h[threadIdx.x];
}

// Exclusive scan of each digit's row of tile counts, in place; totals[d] = the row's sum.
// One block of 1024 threads per digit.
__global__ void __launch_bounds__(1024)
k_sort_scan_rows(uint32_t* __restrict__ counts, int64_t ntiles, uint32_t* __restrict__ totals) {
  __shared__ uint32_t sh[1024];
  uint32_t* row = counts + (int64_t)blockIdx.x * ntiles;
  const int64_t per = (ntiles + 1023) / 1024;
  const int64_t b0 = (int64_t)threadIdx.x * per;
  const int64_t b1 = b0 + per < ntiles ? b0 + per : ntiles;
  uint32_t s = 0;
  for (int64_t i = b0; i < b1; ++i) s += row[i];
  sh[threadIdx.x] = s;
  __syncthreads();
  for (int off = 1; off < 1024; off <<= 1) {
    const uint32_t v = threadIdx.x >= (unsigned)off ? sh[threadIdx.x - off] : 0u;
    __syncthreads();
    sh[threadIdx.x] += v;
    __syncthreads();
  }
  uint32_t run = sh[threadIdx.x] - s;
  for (int64_t i = b0; i < b1; ++i) {
    const uint32_t c = row[i];
    row[i] = run;
    run += c;
  }
  if (threadIdx.x == 1023) totals[blockIdx.x] = sh[1023];
}

// exclusive scan over the 256 values v of threads 0..255 (every thread of the block calls
// it; threads 256 and up pass 0 and get 0)
__device__ __forceinline__ uint32_t block256_exclusive(uint32_t v, uint32_t* tmp) {
  const bool on = threadIdx.x < 256u;
  if (on) tmp[threadIdx.x] = v;
  __syncthreads();
  for (int off = 1; off < 256; off <<= 1) {
    const uint32_t a = on && threadIdx.x >= (unsigned)off ? tmp[threadIdx.x - off] : 0u;
    __syncthreads();
    if (on) tmp[threadIdx.x] += a;
    __syncthreads();
  }
  const uint32_t r = on ? tmp[threadIdx.x] - v : 0u;
  __syncthreads();
  return r;
}

// One pass: pairs of tile t go, stably by digit, to their global positions.  Warp w of 16
// ranks the tile's elements [w * 512, (w + 1) * 512) in chunks of 32: the lanes of equal
// digit are found by ORing each lane's bit into the warp's slot for its digit in shared
// memory, and the group's leader adds the group's size to the warp's running count of that
// digit with an atomic that returns the count before it (the group's start).  One scan over
// (digit, warp) then gives every element its place in the tile; the tile is staged in
// shared memory by digit and each digit's run written to its global offset, so the global
// stores are contiguous runs.  Positions outside [0, n) or a local rank outside the tile
// (which correct scans never give) are skipped and set *err.
__global__ void __launch_bounds__(kScatterThreads, 2)
k_sort_scatter(const uint32_t* __restrict__ keys, const uint32_t* __restrict__ vals, int64_t n,
               int shift, int64_t ntiles, const uint32_t* __restrict__ counts,
               const uint32_t* __restrict__ totals, uint32_t* __restrict__ keys_out,
               uint32_t* __restrict__ vals_out, int* __restrict__ err) {
  constexpr int kPerWarp = kSortTile / kScatterWarps, kChunks = kPerWarp / 32;  // 512, 16
  extern __shared__ uint32_t smem[];
  uint32_t* s_keys = smem;                          // [kSortTile]
  uint32_t* s_vals = s_keys + kSortTile;            // [kSortTile]
  uint32_t* s_wc = s_vals + kSortTile;              // [warps][256] counts, then starts
  uint32_t* s_mask = s_wc + kScatterWarps * 256;    // [warps][256] lanes of a digit
  uint32_t* s_lbase = s_mask + kScatterWarps * 256; // [256] tile-local start of each digit
  uint32_t* s_gbase = s_lbase + 256;                // [256] global start of this tile's run
  uint32_t* s_tmp = s_gbase + 256;                  // [256]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t base = (int64_t)blockIdx.x * kSortTile;
  const int64_t rem = n - base;
  const int cnt = rem < kSortTile ? (int)rem : kSortTile;
  uint32_t* wc = s_wc + warp * 256;
  uint32_t* wm = s_mask + warp * 256;
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    wc[lane * 8 + q] = 0;
    wm[lane * 8 + q] = 0;
  }
  __syncwarp();

  const unsigned lt = (1u << lane) - 1u, me = 1u << lane;
  const int i0 = warp * kPerWarp + lane;  // element of chunk c: i0 + c * 32
  uint32_t kreg[kChunks], vreg[kChunks], pk[kChunks];
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    const int i = i0 + c * 32;
    kreg[c] = i < cnt ? keys[base + i] : 0u;
    vreg[c] = i < cnt ? vals[base + i] : 0u;
  }
  // per chunk: lanes of equal digit from the OR of their bits in the warp's mask slot; the
  // group's leader takes the group's start from the running count and clears the slot
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    const bool valid = i0 + c * 32 < cnt;
    const uint32_t d = (kreg[c] >> shift) & 255u;
    if (valid) atomicOr(&wm[d], me);
    __syncwarp();
    const unsigned peers = valid ? wm[d] : 0u;
    __syncwarp();
    const int leader = valid ? __ffs(peers) - 1 : lane;
    uint32_t start = 0;
    if (valid && lane == leader) {
      start = atomicAdd(&wc[d], (uint32_t)__popc(peers));
      wm[d] = 0;
    }
    start = __shfl_sync(0xFFFFFFFFu, start, leader);
    __syncwarp();
    pk[c] = valid ? (d << 16) | (start + (uint32_t)__popc(peers & lt)) : 0xFFFFFFFFu;
  }
  __syncthreads();

  // thread d < 256: starts of digit d for each warp within the tile, the tile's digit
  // starts, and the global start of the tile's run of digit d
  uint32_t run = 0;
  if (tid < 256) {
#pragma unroll
    for (int w = 0; w < kScatterWarps; ++w) {
      const uint32_t c = s_wc[w * 256 + tid];
      s_wc[w * 256 + tid] = run;
      run += c;
    }
  }
  const uint32_t lbase = block256_exclusive(run, s_tmp);
  const uint32_t gb = block256_exclusive(tid < 256 ? totals[tid] : 0u, s_tmp);
  if (tid < 256) {
#pragma unroll
    for (int w = 0; w < kScatterWarps; ++w) s_wc[w * 256 + tid] += lbase;
    s_lbase[tid] = lbase;
    s_gbase[tid] = gb + counts[(int64_t)tid * ntiles + blockIdx.x];
  }
  __syncthreads();

#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    if (pk[c] != 0xFFFFFFFFu) {
      const uint32_t lp = wc[pk[c] >> 16] + (pk[c] & 0xFFFFu);
      if (lp < (uint32_t)kSortTile) {
        s_keys[lp] = kreg[c];
        s_vals[lp] = vreg[c];
      } else {
        atomicExch(err, 1);
      }
    }
  }
  __syncthreads();

  // write each digit's run to its global position
  for (int i = tid; i < cnt; i += kScatterThreads) {
    const uint32_t key = s_keys[i];
    const uint32_t d = (key >> shift) & 255u;
    const int64_t g = (int64_t)s_gbase[d] + (int64_t)i - (int64_t)s_lbase[d];
    if (g >= 0 && g < n) {
      keys_out[g] = key;
      vals_out[g] = s_vals[i];
    } else {
      atomicExch(err, 2);
    }
  }
}

__global__ void k_iota_u32(uint32_t* __restrict__ out, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = (uint32_t)i;
}

// segment id of an element of an (outer, n, inner) array from its flat index f, the
// segment being the 1-D slice along the middle axis: seg = o * inner + r.  An element
// never leaves its slice, so its original index gives the segment of its current position.
__global__ void k_segment_keys(const uint32_t* __restrict__ idx, int64_t total, int64_t n,
                               int64_t inner, uint32_t* __restrict__ seg) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t f = idx[i];
    const int64_t o = f / (n * inner), r = f % inner;
    seg[i] = (uint32_t)(o * inner + r);
  }
}

// After a segmented round's sort (segment-major, by key within a segment) the element at
// sorted position p = seg * n + j moves to (o, j, r): perm_out[(o n + j) inner + r] =
// sorted[p], sorted holding original indices.
__global__ void k_shuffle_place(const uint32_t* __restrict__ sorted, int64_t total, int64_t n,
                                int64_t inner, uint32_t* __restrict__ perm_out,
                                int* __restrict__ err) {
  for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < total;
       p += (int64_t)gridDim.x * blockDim.x) {
    const int64_t seg = p / n, j = p % n;
    const int64_t o = seg / inner, r = seg % inner;
    const int64_t dst = (o * n + j) * inner + r;
    if (dst < total) perm_out[dst] = sorted[p];
    else atomicExch(err, 3);
  }
}

// out[o][i][:] = src[o][idx[i]][:] for rows of `row` units of W bytes; idx values must be
// < n_src (rows of src along the middle axis); others are skipped and set *err
template <class W>
__global__ void k_take_rows(const W* __restrict__ src, int64_t outer, int64_t n_src,
                            const uint32_t* __restrict__ idx, int64_t n_idx, int64_t row,
                            W* __restrict__ out, int* __restrict__ err) {
  const int64_t total = outer * n_idx * row;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t u = t % row, oi = t / row;
    const int64_t i = oi % n_idx, o = oi / n_idx;
    const uint32_t s = idx[i];
    if ((int64_t)s < n_src) out[t] = src[(o * n_src + s) * row + u];
    else if (err) atomicExch(err, 4);
  }
}

// Sortable unsigned keys of floats (ascending order of value; -0 ordered as +0);
// descending flips them.  float64 keys are split into high and low words.
__device__ __forceinline__ uint32_t float_order_key(uint32_t b) {
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
template <bool kF64>
__global__ void k_float_sort_keys(const void* __restrict__ x, int64_t n, bool descending,
                                  uint32_t* __restrict__ hi, uint32_t* __restrict__ lo) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    if constexpr (kF64) {
      const double v = ((const double*)x)[i];
      unsigned long long b = (unsigned long long)__double_as_longlong(v == 0.0 ? 0.0 : v);
      b = (b & 0x8000000000000000ull) ? ~b : (b | 0x8000000000000000ull);
      if (descending) b = ~b;
      hi[i] = (uint32_t)(b >> 32);
      lo[i] = (uint32_t)b;
    } else {
      const float v = ((const float*)x)[i];
      uint32_t k = float_order_key(__float_as_uint(v == 0.0f ? 0.0f : v));
      hi[i] = descending ? ~k : k;
    }
  }
}

// out[i] = src[idx[i]] for 32-bit words
__global__ void k_gather_u32(const uint32_t* __restrict__ src, const uint32_t* __restrict__ idx,
                             int64_t n, uint32_t* __restrict__ out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = src[idx[i]];
}

}  // namespace jxr
