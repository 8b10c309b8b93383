// Stable LSD radix sort of (uint32 key, uint32 value) pairs and the shuffle built on it
// (random_permutation, R/random.R:378-413).
//
// rnd_shuffle sorts the array by fresh 32-bit random keys, num_rounds times, with a
// stable key-value sort (lax_sort_key_val).  Here every round sorts (key, position)
// pairs: radix passes of 8 bits over the keys' top bits (each pass a histogram kernel, a
// scan of the per-tile counts and a scatter), then the span sort (k_sort_spans) orders
// each run of equal top bits in shared memory.  Sorts of other keys (argsort of floats,
// segment ids) take radix passes over every digit.  The scatter ranks a tile's elements
// stably (per warp and chunk of 32, the lanes of equal digit from bits ORed into shared
// memory, running counts per warp), places them by digit in shared memory and writes each
// digit's run to its global offset, so the global stores are contiguous runs.
#pragma once

#include <cstdint>

namespace jxr {

constexpr int kSortThreads = 256;  // histogram CTAs
constexpr int kSortItems = 32;
constexpr int kSortTile = kSortThreads * kSortItems;  // 8192 elements per tile
constexpr int kScatterThreads = 512;                  // scatter CTAs: 16 warps per tile
constexpr int kScatterWarps = kScatterThreads / 32;
// dynamic shared memory of the scatter: keys and values of a tile, per warp the running
// digit counts and the lane masks of one chunk, two 256-entry tables
constexpr int kSortScatterSmem = 2 * kSortTile * 4 + 2 * kScatterWarps * 256 * 4 + 2 * 256 * 4;

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

// Exclusive scans of two values a, b held by threads 0..255 (every thread of the block
// calls it; threads 256 and up get 0): warp shuffles, then the 8 warp totals through
// shared memory (tmp: 16 words).
__device__ __forceinline__ void block256_exclusive2(uint32_t a, uint32_t b, uint32_t* ra,
                                                    uint32_t* rb, uint32_t* tmp) {
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  uint32_t ia = a, ib = b;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const uint32_t ya = __shfl_up_sync(0xFFFFFFFFu, ia, off);
    const uint32_t yb = __shfl_up_sync(0xFFFFFFFFu, ib, off);
    if (lane >= off) {
      ia += ya;
      ib += yb;
    }
  }
  if (tid < 256 && lane == 31) {
    tmp[w] = ia;
    tmp[8 + w] = ib;
  }
  __syncthreads();
  uint32_t pa = 0, pb = 0;
  if (tid < 256) {
    for (int q = 0; q < w; ++q) {
      pa += tmp[q];
      pb += tmp[8 + q];
    }
  }
  *ra = tid < 256 ? pa + ia - a : 0u;
  *rb = tid < 256 ? pb + ib - b : 0u;
  __syncthreads();
}

// One pass: pairs of tile t go, stably by digit, to their global positions.  Warp w of 16
// ranks the tile's elements [w * 512, (w + 1) * 512) in chunks of 32: the lanes of equal
// digit are found by ORing each lane's bit into the warp's slot for its digit in shared
// memory, and the group's leader adds the group's size to the warp's running count of that
// digit with an atomic that returns the count before it (the group's start).  One scan over
// (digit, warp) then gives every element its place in the tile; the tile is staged in
// shared memory by digit and each digit's run written to its global offset, so the global
// stores are contiguous runs.  The CTAs are persistent (tiles blockIdx.x, + gridDim.x, ...):
// once a tile is staged, the next tile's keys and values are loaded into the same
// registers, so those loads are in flight while the staged tile is written out.  With vals
// == nullptr the values are the elements' positions.  Positions outside [0, n) or a local
// rank outside the tile (which correct scans never give) are skipped and set *err.
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
  // [256] global start of the tile's run of each digit minus its start within the tile
  // (a 32-bit wrap-around difference: the sum with a tile position is the global position)
  uint32_t* s_shift = s_mask + kScatterWarps * 256;
  uint32_t* s_tmp = s_shift + 256;                  // [256]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint32_t* wc = s_wc + warp * 256;
  uint32_t* wm = s_mask + warp * 256;
  const unsigned lt = (1u << lane) - 1u, me = 1u << lane;
  const int i0 = warp * kPerWarp + lane;  // element of chunk c: i0 + c * 32
  uint32_t kreg[kChunks], vreg[kChunks], pk[kChunks];

  int64_t t = blockIdx.x;
  auto tile_count = [&](int64_t tt) {
    const int64_t rem = n - tt * kSortTile;
    return rem < kSortTile ? (int)rem : kSortTile;
  };
  auto load = [&](int64_t tt) {
    const int64_t base = tt * kSortTile;
    const int cnt = tile_count(tt);
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
      const int i = i0 + c * 32;
      kreg[c] = i < cnt ? keys[base + i] : 0u;
      vreg[c] = i < cnt ? (vals ? vals[base + i] : (uint32_t)(base + i)) : 0u;
    }
  };
  if (t < ntiles) load(t);
  for (; t < ntiles; t += gridDim.x) {
    const int cnt = tile_count(t);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      wc[lane * 8 + q] = 0;
      wm[lane * 8 + q] = 0;
    }
    __syncwarp();
    // per chunk: lanes of equal digit from the OR of their bits in the warp's mask slot;
    // the group's leader takes the group's start from the running count and clears the slot
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
    uint32_t lbase, gb;
    block256_exclusive2(run, tid < 256 ? totals[tid] : 0u, &lbase, &gb, s_tmp);
    if (tid < 256) {
#pragma unroll
      for (int w = 0; w < kScatterWarps; ++w) s_wc[w * 256 + tid] += lbase;
      s_shift[tid] = gb + counts[(int64_t)tid * ntiles + t] - lbase;
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
    // the next tile's loads go out before this tile is written
    if (t + gridDim.x < ntiles) load(t + gridDim.x);

    // write each digit's run to its global position
    for (int i = tid; i < cnt; i += kScatterThreads) {
      const uint32_t key = s_keys[i];
      const uint32_t d = (key >> shift) & 255u;
      const uint32_t g = s_shift[d] + (uint32_t)i;  // n < 2^32
      if (g < n) {
        keys_out[g] = key;
        vals_out[g] = s_vals[i];
      } else {
        atomicExch(err, 2);
      }
    }
    __syncthreads();
  }
}

// ---- span sort: the low digits of a shuffle round's sort in shared memory ---------------
//
// After the radix passes over the top `8 g` bits, the pairs are grouped in buckets of equal
// top bits, in key order, each bucket in original order.  Sorting every bucket stably by
// the whole key finishes the sort.  Each CTA owns kSpanOwn positions and sorts the span of
// the buckets that start inside them (ending where the first bucket after them starts), at
// most `cap` elements: it loads a window of keys and values around its positions into
// shared memory (16-byte loads), finds the span there, maps each key to one of M slots by a
// monotone map of its offset from the span's first bucket, counts the slots, scans the
// counts (listing the slots that hold more than one element), places each element at its
// slot's start plus its order of arrival, and sorts each listed slot by (key, position in
// the span) with an insertion sort, the list shared out over the threads; that is the
// stable order.  Only the values are written.  A span longer than `cap`, or running past
// the window, sets *overflow and is skipped (the caller then sorts with the radix passes
// alone); for uniformly random keys and the bucket sizes the caller picks this does not
// happen.  The key and value buffers must be readable up to the 16-byte boundary after
// element n - 1.
constexpr int kSpanThreads = 512;
constexpr int kSpanOwn = 2048;                 // positions owned by one CTA
constexpr int kSpanCap = 4096;                 // longest span sorted in shared memory
constexpr int kSpanSlots = kSpanCap;           // most slots
// the window: keys [lo - 4, lo + 2 kSpanOwn) and values [lo, lo + 2 kSpanOwn) of the CTA
constexpr int kSpanWinK = 2 * kSpanOwn + 4, kSpanWinV = 2 * kSpanOwn;
// dynamic shared memory: the window's keys and values, slot starts, the span's positions
// in slot order (u16), each element's order of arrival in its slot (u16), the slots of more
// than one element (u16, at most kSpanCap / 2)
constexpr int kSpanSmem = kSpanWinK * 4 + kSpanWinV * 4 + kSpanSlots * 4 + kSpanCap * 2 * 2 +
                          kSpanCap;
static_assert(kSpanWinV >= kSpanCap && kSpanOwn % 4 == 0, "a span fits the window");

__device__ __forceinline__ uint32_t span_top(uint32_t k, int top_shift) {
  return top_shift >= 32 ? 0u : k >> top_shift;
}

__global__ void __launch_bounds__(kSpanThreads, 3)
k_sort_spans(const uint32_t* __restrict__ keys, const uint32_t* __restrict__ vals, int64_t n,
             int top_shift, int cap, uint32_t* __restrict__ vals_out, int* __restrict__ overflow,
             int* __restrict__ err) {
  constexpr int kWarps = kSpanThreads / 32;
  extern __shared__ uint32_t smem[];
  uint32_t* s_wk = smem;                                   // [kSpanWinK]
  uint32_t* s_wv = s_wk + kSpanWinK;                       // [kSpanWinV]
  uint32_t* s_start = s_wv + kSpanWinV;                    // [kSpanSlots], 16-byte aligned
  uint16_t* s_member = (uint16_t*)(s_start + kSpanSlots);  // [kSpanCap]
  uint16_t* s_arr = s_member + kSpanCap;                   // [kSpanCap]
  uint16_t* s_work = s_arr + kSpanCap;                     // [kSpanCap / 2]
  __shared__ int s_first, s_end;
  __shared__ uint32_t s_pre[kWarps + 1], s_nwork;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t lo = (int64_t)blockIdx.x * kSpanOwn;
  const int64_t hi = lo + kSpanOwn < n ? lo + kSpanOwn : n;
  const int64_t w0 = lo > 0 ? lo - 4 : 0;  // 16-byte aligned
  const int64_t w1 = lo + 2 * kSpanOwn < n ? lo + 2 * kSpanOwn : n;
  const int wn = (int)(w1 - w0);           // keys in the window, <= kSpanWinK
  const int lo_w = (int)(lo - w0), hi_w = (int)(hi - w0);

  {  // the window, in 16-byte pieces (the last may run past n, inside the buffers)
    const uint4* k4 = reinterpret_cast<const uint4*>(keys + w0);
    const uint4* v4 = reinterpret_cast<const uint4*>(vals + lo);
    uint4* sk4 = reinterpret_cast<uint4*>(s_wk);
    uint4* sv4 = reinterpret_cast<uint4*>(s_wv);
    const int nk = (wn + 3) / 4, nv = ((int)(w1 - lo) + 3) / 4;
    constexpr int RK = (kSpanWinK / 4 + kSpanThreads - 1) / kSpanThreads;
    constexpr int RV = (kSpanWinV / 4 + kSpanThreads - 1) / kSpanThreads;
    uint4 kq[RK], vq[RV];  // every load in flight before the first store
#pragma unroll
    for (int r = 0; r < RK; ++r)
      if (tid + r * kSpanThreads < nk) kq[r] = k4[tid + r * kSpanThreads];
#pragma unroll
    for (int r = 0; r < RV; ++r)
      if (tid + r * kSpanThreads < nv) vq[r] = v4[tid + r * kSpanThreads];
#pragma unroll
    for (int r = 0; r < RK; ++r)
      if (tid + r * kSpanThreads < nk) sk4[tid + r * kSpanThreads] = kq[r];
#pragma unroll
    for (int r = 0; r < RV; ++r)
      if (tid + r * kSpanThreads < nv) sv4[tid + r * kSpanThreads] = vq[r];
  }
  if (tid == 0) {
    s_first = hi_w;
    s_end = wn;
    s_nwork = 0;
  }
  __syncthreads();
  // window position i starts a bucket (i >= 1, or the array's first element)
  auto is_start = [&](int i) {
    return (w0 == 0 && i == 0) || span_top(s_wk[i], top_shift) != span_top(s_wk[i - 1], top_shift);
  };
  // the first bucket start in [lo, hi) (the span's start) and in [hi, w1) (its end), both
  // searched in rounds of kSpanThreads positions until each is found
  for (int b = 0; lo_w + b < hi_w || hi_w + b < wn; b += kSpanThreads) {
    const int i = lo_w + b + tid, j = hi_w + b + tid;
    if (i < hi_w && is_start(i)) atomicMin(&s_first, i);
    if (j < wn && is_start(j)) atomicMin(&s_end, j);
    __syncthreads();
    const bool done = (s_first < hi_w || lo_w + b + kSpanThreads >= hi_w) &&
                      (s_end < wn || hi_w + b + kSpanThreads >= wn);
    __syncthreads();
    if (done) break;
  }
  const int a = s_first;
  if (a >= hi_w) return;  // every bucket here started before lo
  const int e = s_end;
  const int S = e - a;
  if (S > cap || (e == wn && w1 < n)) {  // too long, or no end inside the window
    if (tid == 0) atomicExch(overflow, 1);
    return;
  }
  const uint32_t* s_key = s_wk + a;                 // the span's keys
  const uint32_t* s_val = s_wv + (a - lo_w);        // and values

  // slots: M = the power of two >= 2 S, at most kSpanSlots (>= S always; fewer slots with
  // several elements to sort than with M >= S); slot of key k = the monotone map
  // floor((k - base) M / R) of its offset in the span's range of buckets R
  int M = 128;
  while (M < 2 * S && M < kSpanSlots) M <<= 1;
  const uint32_t t_first = span_top(s_key[0], top_shift), t_last = span_top(s_key[S - 1], top_shift);
  const uint32_t base = top_shift >= 32 ? 0u : t_first << top_shift;
  const float range = top_shift >= 32 ? 4294967296.0f
                                        : (float)((uint64_t)(t_last - t_first + 1u) << top_shift);
  const float scale = __fdiv_rn((float)M, range);
  auto slot_of = [&](int i) {
    const uint32_t slot = __float2uint_rz(__fmul_rn(__uint2float_rz(s_key[i] - base), scale));
    return slot < (uint32_t)M ? slot : (uint32_t)M - 1u;
  };
  uint4* s_start4 = reinterpret_cast<uint4*>(s_start);
  for (int q = tid; q < M / 4; q += kSpanThreads) s_start4[q] = make_uint4(0u, 0u, 0u, 0u);
  __syncthreads();
  for (int i = tid; i < S; i += kSpanThreads)
    s_arr[i] = (uint16_t)atomicAdd(&s_start[slot_of(i)], 1u);  // order of arrival in the slot
  __syncthreads();
  // exclusive scan of the slot counts within chunks of C slots (warp w: chunk w; each lane
  // four consecutive slots per step of 128), the chunks' offsets in s_pre: the start of slot
  // s is s_start[s] + s_pre[s >> logC].  Slots of two or more elements go to s_work.
  const int C = M / kWarps > 128 ? M / kWarps : 128;
  const int logC = 31 - __clz(C);
  const int nchunks = M >> logC;
  if (warp < nchunks) {
    uint32_t total = 0;
    for (int q = 0; q < C; q += 128) {
      const int s4 = (warp * C + q) / 4 + lane;  // this lane's slots 4 s4 .. 4 s4 + 3
      const uint4 v = s_start4[s4];
      const uint32_t t1 = v.x + v.y, t2 = t1 + v.z, t3 = t2 + v.w;
      uint32_t incl = t3;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, incl, off);
        if (lane >= off) incl += y;
      }
      const uint32_t ex = total + incl - t3;
      s_start4[s4] = make_uint4(ex, ex + v.x, ex + t1, ex + t2);
      total += __shfl_sync(0xFFFFFFFFu, incl, 31);
      const uint32_t multi = (v.x > 1u) | (v.y > 1u) << 1 | (v.z > 1u) << 2 | (v.w > 1u) << 3;
      if (multi) {
        uint32_t w = atomicAdd(&s_nwork, (uint32_t)__popc(multi));
#pragma unroll
        for (int c = 0; c < 4; ++c)
          if (((multi >> c) & 1u) && w < (uint32_t)(kSpanCap / 2)) s_work[w++] = (uint16_t)(4 * s4 + c);
      }
    }
    if (lane == 0) s_pre[warp] = total;
  }
  __syncthreads();
  if (warp == 0) {  // exclusive scan of the chunk totals
    const uint32_t t = lane < nchunks ? s_pre[lane] : 0u;
    uint32_t incl = t;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, incl, off);
      if (lane >= off) incl += y;
    }
    if (lane <= nchunks) s_pre[lane] = incl - t;  // s_pre[nchunks] = S
  }
  __syncthreads();
  auto slot_start = [&](uint32_t slot) {
    return slot < (uint32_t)M ? s_start[slot] + s_pre[slot >> logC] : (uint32_t)S;
  };
  // every element at its slot's start + its order of arrival
  for (int i = tid; i < S; i += kSpanThreads) {
    const uint32_t p = slot_start(slot_of(i)) + s_arr[i];
    if (p < (uint32_t)S) s_member[p] = (uint16_t)i;
    else atomicExch(err, 5);
  }
  __syncthreads();
  // the listed slots: insertion sort by (key, position in the span)
  const int nwork = s_nwork < (uint32_t)(kSpanCap / 2) ? (int)s_nwork : kSpanCap / 2;
  for (int w = tid; w < nwork; w += kSpanThreads) {
    const uint32_t slot = s_work[w];
    const uint32_t st = slot_start(slot), en = slot_start(slot + 1u);
    if (en > (uint32_t)S || en < st) {
      atomicExch(err, 6);
      continue;
    }
    for (uint32_t q = st + 1u; q < en; ++q) {
      const uint32_t x = s_member[q], kx = s_key[x < (uint32_t)S ? x : 0u];
      uint32_t r = q;
      while (r > st) {
        const uint32_t y = s_member[r - 1u], ky = s_key[y < (uint32_t)S ? y : 0u];
        if (ky < kx || (ky == kx && y < x)) break;
        s_member[r] = (uint16_t)y;
        --r;
      }
      s_member[r] = (uint16_t)x;
    }
  }
  __syncthreads();
  const int64_t s0 = w0 + a;
  for (int i = tid; i < S; i += kSpanThreads) {
    const uint32_t m = s_member[i];
    vals_out[s0 + i] = s_val[m < (uint32_t)S ? m : 0u];
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
