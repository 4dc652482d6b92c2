// Per-segment run analysis shared by the cached-step and tiled-layout
// builders.  One CTA of kThreads threads handles one query segment whose key
// list is a concatenation of candidate runs (contiguous rows of one key/value
// stream).  The caller fills, per candidate c in the reference's order,
//   w[c]    width if the segment attends to the run (0 otherwise),
//   key[c]  (stream << kStreamShift) | first row within the stream,
//   pool[c] first index in the reference's concatenated pool,
// and analyse_runs() derives the key offsets, the merged runs (a run that
// continues the previous attended run's rows in the same stream merges with
// it) and the 64-row key boxes that cover them; emit_plan() writes the boxes
// as 128-key tiles with per-key masks for the attention kernel.
#pragma once

#include <limits.h>

#include "common.cuh"

namespace hier {
namespace segplan {

constexpr int kThreads = 256;
constexpr int kBoxRows = 64;
constexpr int kStreamShift = 24;
constexpr int kMiscInts = 32 + kThreads;

// Block-wide inclusive scan (sum or max) of one value per thread; every
// thread of the block must call it.
template <bool kMax>
__device__ __forceinline__ int block_scan(int v, int* warp_tmp) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v = kMax ? max(v, t) : v + t;
  }
  if (lane == 31) warp_tmp[w] = v;
  __syncthreads();
  if (w == 0) {
    int x = lane < kThreads / 32 ? warp_tmp[lane] : (kMax ? INT_MIN : 0);
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x = kMax ? max(x, t) : x + t;
    }
    if (lane < kThreads / 32) warp_tmp[lane] = x;
  }
  __syncthreads();
  if (w > 0) v = kMax ? max(v, warp_tmp[w - 1]) : v + warp_tmp[w - 1];
  __syncthreads();
  return v;
}

struct SegSmem {
  int* w;     // [C] attended width
  int* key;   // [C] stream-packed first row
  int* pool;  // [C] first pool index
  int* off;   // [C] exclusive key offset (attended runs)
  int* rf;    // [C+1] key offset of each merged run (rf[n_runs] = total)
  int* rk;    // [C] stream-packed first row of each merged run
  int* rb;    // [C+1] exclusive box offset of each merged run
  int* dw;    // [C] dense width (tiled layouts: every candidate's slots)
  int* doff;  // [C+1] exclusive dense offset
  int* misc;  // [0] keys, [1] runs, [2] boxes, [3] status, [8..] scratch
};

__device__ __forceinline__ SegSmem seg_smem(int* base, int C) {
  SegSmem m;
  m.w = base;
  m.key = m.w + C;
  m.pool = m.key + C;
  m.off = m.pool + C;
  m.rf = m.off + C;
  m.rk = m.rf + C + 1;
  m.rb = m.rk + C;
  m.dw = m.rb + C + 1;
  m.doff = m.dw + C;
  m.misc = m.doff + C + 1;
  return m;
}

__host__ __device__ inline size_t seg_smem_ints(int C) { return (size_t)9 * C + 3 + kMiscInts; }

// Key offsets, merged runs and box offsets from w / key (all threads).
__device__ inline void analyse_runs(const SegSmem& m, int C) {
  int* wtmp = m.misc + 8;       // block_scan scratch
  int* carry = m.misc + 16;     // values carried from one chunk to the next
  int* incl_max = m.misc + 32;  // [kThreads] inclusive max-scan of one chunk
  int carry_sum = 0, carry_prev = -1, carry_runs = 0;
  for (int base = 0; base < C; base += kThreads) {
    const int c = base + threadIdx.x;
    const int wc = c < C ? m.w[c] : 0;
    const int incl = block_scan<false>(wc, wtmp) + carry_sum;
    const int pm = max(block_scan<true>(wc > 0 ? c : -1, wtmp), carry_prev);
    incl_max[threadIdx.x] = pm;
    __syncthreads();
    const int prev = threadIdx.x == 0 ? carry_prev : incl_max[threadIdx.x - 1];
    const bool start = wc > 0 && (prev < 0 || m.key[prev] + m.w[prev] != m.key[c]);
    if (wc > 0) m.off[c] = incl - wc;
    const int rid = block_scan<false>(start ? 1 : 0, wtmp) + carry_runs - 1;
    if (start) {
      m.rf[rid] = incl - wc;
      m.rk[rid] = m.key[c];
    }
    if (threadIdx.x == kThreads - 1) {
      carry[0] = incl;
      carry[1] = pm;
      carry[2] = rid + 1;
    }
    __syncthreads();
    carry_sum = carry[0];
    carry_prev = carry[1];
    carry_runs = carry[2];
    __syncthreads();
  }
  const int total = carry_sum, n_runs = carry_runs;
  if (threadIdx.x == 0) m.rf[n_runs] = total;
  __syncthreads();
  int carry_box = 0;
  for (int base = 0; base < n_runs; base += kThreads) {
    const int r = base + threadIdx.x;
    const int nbx = r < n_runs ? (m.rf[r + 1] - m.rf[r] + kBoxRows - 1) / kBoxRows : 0;
    const int incl = block_scan<false>(nbx, wtmp) + carry_box;
    if (r < n_runs) m.rb[r] = incl - nbx;
    if (threadIdx.x == kThreads - 1) carry[0] = incl;
    __syncthreads();
    carry_box = carry[0];
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    m.rb[n_runs] = carry_box;
    m.misc[0] = total;
    m.misc[1] = n_runs;
    m.misc[2] = carry_box;
  }
  __syncthreads();
}

// Exclusive scan of n_boxes over the segments before s (tiles = ceil(boxes/2)).
__device__ inline int tile_base_of(const int32_t* n_boxes, int s, int* wtmp) {
  int tb = 0;
  for (int i = threadIdx.x; i < s; i += kThreads) tb += (n_boxes[i] + 1) >> 1;
  tb = block_scan<false>(tb, wtmp);  // inclusive: the last thread holds the sum
  __shared__ int tile_base_s;
  if (threadIdx.x == kThreads - 1) tile_base_s = tb;
  __syncthreads();
  return tile_base_s;
}

__device__ __forceinline__ uint32_t low_bits(int n) {  // n in [0, 32]
  return n >= 32 ? 0xffffffffu : ((1u << n) - 1u);
}

__device__ __forceinline__ int run_of_box(const SegSmem& m, int n_runs, int b) {
  int lo = 0, hi = n_runs - 1;  // last run with rb[r] <= b
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (m.rb[mid] <= b) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

// Boxes of the segment as tiles [tile_base, tile_base + ceil(n_box/2)):
// kv_tiles (row0, row1, sel, sel) with sel = -1 for a full tile, else the
// tile index into tile_masks (4 words: keys 0-31, 32-63 of box 0, then box 1).
__device__ inline void emit_plan(const SegSmem& m, int tile_base, int32_t* kv_tiles,
                                 uint32_t* tile_masks) {
  const int n_runs = m.misc[1], n_box = m.misc[2];
  const int n_tiles = (n_box + 1) >> 1;
  for (int b = threadIdx.x; b < 2 * n_tiles; b += kThreads) {
    const int t = tile_base + (b >> 1), slot = b & 1;
    const int bb = b < n_box ? b : b - 1;  // odd count: the last tile repeats its first box
    const int r = run_of_box(m, n_runs, bb);
    const int k = bb - m.rb[r];
    const int key = m.rk[r] + kBoxRows * k;
    const int valid = b < n_box ? min(kBoxRows, m.rf[r + 1] - m.rf[r] - kBoxRows * k) : 0;
    kv_tiles[(int64_t)t * 4 + slot] = key;
    tile_masks[(int64_t)t * 4 + 2 * slot] = low_bits(valid);
    tile_masks[(int64_t)t * 4 + 2 * slot + 1] = low_bits(max(valid - 32, 0));
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n_tiles; i += kThreads) {
    const int t = tile_base + i;
    const uint32_t* mk = tile_masks + (int64_t)t * 4;
    const bool full = (mk[0] & mk[1] & mk[2] & mk[3]) == 0xffffffffu;
    kv_tiles[(int64_t)t * 4 + 2] = full ? -1 : t;
    kv_tiles[(int64_t)t * 4 + 3] = full ? -1 : t;
  }
}

// Query pairs of a segment of ql rows from q0: pair i = rows [q0+256i, +128)
// and [q0+256i+128, +128), both over the segment's tiles.
__device__ inline void emit_pairs(int q0, int ql, int pair_base, int tile_base, int n_tiles,
                                  int32_t* q_pairs) {
  const int per = (((ql + 127) / 128) + 1) / 2;
  for (int i = threadIdx.x; i < per; i += kThreads) {
    int32_t* r = q_pairs + (int64_t)(pair_base + i) * 8;
    const int r0 = 256 * i;
    r[0] = q0 + r0;
    r[1] = min(128, ql - r0);
    r[2] = q0 + r0 + 128;
    r[3] = max(0, min(128, ql - r0 - 128));
    r[4] = tile_base;
    r[5] = tile_base + n_tiles;
    r[6] = 0;
    r[7] = 0;
  }
}

inline int ceil_div(int a, int b) { return (a + b - 1) / b; }
inline int pairs_for_rows(int ql) { return ceil_div(ceil_div(ql, 128), 2); }

}  // namespace segplan
}  // namespace hier
