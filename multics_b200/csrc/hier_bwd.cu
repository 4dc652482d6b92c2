// Attention backward for sm_100a (tcgen05 + TMEM + TMA) over the forward's
// block plans.
//
// The reference trains the hierarchical self-attention through FlexAttention's
// backward over its BlockMask (multics/models/attention.py:322-353, and the
// Flex Jacobian of forward_hier_tiled_ste, attention.py:367-434).  Here the
// same gradients come from three kernels over the 128x128 block plan the
// forward ran (hier_block_plan_build / hier_dense_block_plan_build), with
// P recomputed from the forward's log2-sum-exp:
//
//   s = q.k * scale * log2(e),  P = 2^(s - lse),  dP = dO . v,
//   Delta_r = dO_r . O_r,  dS = P (dP - Delta),
//   dQ = scale * dS K,  dK = scale * dS^T Q,  dV = P^T dO.
//
// * bwd_prep_kernel: Delta per (row, head) and the log2-sum-exp transposed
//   to head-major rows (+inf for rows without keys and for padding rows, so
//   that their P is 0).
// * bwd_dq_kernel: one CTA per (query tile, head), the forward's query-major
//   plan; per key tile S = Q K^T and dP = dO V^T (SS MMAs), dS by the row
//   threads into TMEM, dQ += dS K (TS MMA, dQ accumulated in TMEM).
// * bwd_dkv_kernel: one CTA per (key block, head) over the transposed plan
//   (hier_bwd_plan_transpose: per key block its query blocks and per-key-row
//   masks); per query tile S^T = K Q^T and dP^T = V dO^T, P^T and dS^T by
//   the key-row threads, dV += P^T dO and dK += dS^T Q (TS MMAs, both
//   accumulated in TMEM, written once).
//
// TMEM holds one score tile and one dP tile (128 columns each) besides the
// accumulators, so the tile is split in two 64-wide sub-tiles, one per row
// warpgroup (warps 4-7 and 8-11, the same 128 lanes), and one thread issues
// the MMAs in the order S0(0) S1(0) | PV0(0) S0(1) PV1(0) S1(1) | ...: while
// one warpgroup turns its sub-tile into P / dS, the tensor core works on the
// other's.
//
// No atomics in the gradients: every dQ, dK and dV row is written by one CTA.
// Every mbarrier wait is bounded (device error word).

#include <math.h>
#include <stdio.h>
#include <string.h>

#include "common.cuh"
#include "tile_mma.cuh"
#include "tmap.h"

namespace hier {
namespace {

constexpr int kStages = 2;
constexpr uint32_t kBwdTmemCols = 512;

// 32 lanes x 16 columns of 32-bit words.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}

// Two row warpgroups share the 128 TMEM lanes: group g reads the fp32 columns
// [64g, 64g + 64) of a score tile and writes their bf16 pairs to columns
// [64g, 64g + 32), its own columns, so neither group overwrites columns the
// other still has to read.  Element k of a packed row therefore sits at
// column k/2 (k < 64) or 32 + k/2 (k >= 64), and the TS MMA that reads it
// takes its K steps 4-7 from 32 columns further on.
__device__ __forceinline__ uint32_t packed_col(int chunk) { return 16 * chunk + (chunk >= 2 ? 32 : 0); }

template <int k>
__device__ __forceinline__ void issue_pv_split_step(uint32_t o_tmem, uint32_t a_tmem, uint32_t blo,
                                                    bool accumulate) {
  constexpr uint32_t idesc = idesc_bf16(kBM, kHD, true);
  constexpr uint32_t offb = (k * 2048) >> 4;
  umma_ts_lo<k * 8 + (k >= 4 ? 32 : 0), offb>(o_tmem, a_tmem, blo, idesc,
                                              (accumulate || k > 0) ? 1u : 0u);
}

// D (128 x 128) (+)= A (bf16 pairs in TMEM, split layout) * B (MN-major) over
// K steps 4g .. 4g+3: the half of the reduction that sub-tile g (elements
// 64g .. 64g+63 of A's rows) contributes.
template <int g>
__device__ __forceinline__ void issue_pv_sub(uint32_t o_tmem, uint32_t a_tmem, uint32_t blo,
                                             bool accumulate) {
  issue_pv_split_step<4 * g + 0>(o_tmem, a_tmem, blo, accumulate);
  issue_pv_split_step<4 * g + 1>(o_tmem, a_tmem, blo, accumulate);
  issue_pv_split_step<4 * g + 2>(o_tmem, a_tmem, blo, accumulate);
  issue_pv_split_step<4 * g + 3>(o_tmem, a_tmem, blo, accumulate);
}

// D (128 x 64, columns 64g.. of a score tile) = A (128 x 128) * B^T with B the
// rows 64g .. 64g+63 of a tile (both K-major): one sub-tile of S.
template <int k, int g>
__device__ __forceinline__ void issue_s64_step(uint32_t d_tmem, uint32_t alo, uint32_t blo) {
  constexpr uint32_t idesc = idesc_bf16(kBM, 64, false);
  constexpr uint32_t off = ((k >> 2) * kHalf + (k & 3) * 32) >> 4;
  constexpr uint32_t offb = off + ((g * 64 * 128) >> 4);
  umma_ss_lo<off, offb>(d_tmem + 64 * g, alo, blo, idesc, k > 0 ? 1u : 0u);
}
template <int g>
__device__ __forceinline__ void issue_s64(uint32_t d_tmem, uint32_t alo, uint32_t blo) {
  issue_s64_step<0, g>(d_tmem, alo, blo);
  issue_s64_step<1, g>(d_tmem, alo, blo);
  issue_s64_step<2, g>(d_tmem, alo, blo);
  issue_s64_step<3, g>(d_tmem, alo, blo);
  issue_s64_step<4, g>(d_tmem, alo, blo);
  issue_s64_step<5, g>(d_tmem, alo, blo);
  issue_s64_step<6, g>(d_tmem, alo, blo);
  issue_s64_step<7, g>(d_tmem, alo, blo);
}

__device__ __forceinline__ uint32_t word_of(const uint4& m, int q) {
  return q == 0 ? m.x : (q == 1 ? m.y : (q == 2 ? m.z : m.w));
}

// Columns [32 q0, 32 q0 + 64) of a 128-wide fp32 row of TMEM (this thread's
// lane) times `scale`, as bf16 to global memory (16-byte stores).
__device__ __forceinline__ void store_row_bf16(uint32_t t_row, float scale, __nv_bfloat16* dst,
                                               bool store, int q0) {
#pragma unroll 1
  for (int q = q0; q < q0 + 2; ++q) {
    uint32_t r[32];
    tmem_ld32(t_row + 32 * q, r);
    tmem_wait_ld();
    if (store) {
      uint32_t w[16];
#pragma unroll
      for (int i = 0; i < 16; ++i)
        w[i] = pack_bf16x2(__uint_as_float(r[2 * i]) * scale, __uint_as_float(r[2 * i + 1]) * scale);
      uint4* d = reinterpret_cast<uint4*>(dst + 32 * q);
#pragma unroll
      for (int k = 0; k < 4; ++k) d[k] = make_uint4(w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
    }
  }
}

// Columns [32 q0, 32 q0 + 64) of a row set to 0.
__device__ __forceinline__ void zero_row(__nv_bfloat16* dst, int q0) {
  uint4* d = reinterpret_cast<uint4*>(dst + 32 * q0);
#pragma unroll
  for (int k = 0; k < 8; ++k) d[k] = make_uint4(0u, 0u, 0u, 0u);
}

// ---------------------------------------------------------------------------
// Delta and head-major log2-sum-exp
// ---------------------------------------------------------------------------
__global__ void bwd_prep_kernel(const __nv_bfloat16* __restrict__ o, int64_t o_stride,
                                const __nv_bfloat16* __restrict__ dout, int64_t do_stride,
                                const float* __restrict__ lse, int64_t rows, int64_t rows_pad,
                                int H, float* __restrict__ delta, float* __restrict__ lse_t) {
  const int lane = threadIdx.x & 31;
  const int64_t w0 = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t r = w0; r < rows_pad; r += nw) {
    for (int h = 0; h < H; ++h) {
      float acc = 0.f;
      if (r < rows) {
        const uint2 a = *reinterpret_cast<const uint2*>(o + r * o_stride + h * kHD + 4 * lane);
        const uint2 b = *reinterpret_cast<const uint2*>(dout + r * do_stride + h * kHD + 4 * lane);
        const float2 a0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&a.x));
        const float2 a1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&a.y));
        const float2 b0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&b.x));
        const float2 b1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&b.y));
        acc = a0.x * b0.x + a0.y * b0.y + a1.x * b1.x + a1.y * b1.y;
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
      if (lane == 0) {
        float l = r < rows ? lse[r * H + h] : INFINITY;
        if (l == -INFINITY) l = INFINITY;  // a row without keys: P = 0
        delta[h * rows_pad + r] = acc;
        lse_t[h * rows_pad + r] = l;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Transposed (key-major) plan of a block plan
// ---------------------------------------------------------------------------
// A reference to key block kb by query block qb is one (entry, half) of the
// query-major plan whose selector is not "skip".  Entries: (q_start, q_rows,
// selector, q_start / 128), per key block ascending in q_start.

__device__ __forceinline__ bool tplan_ref(const int4& pq, const int4& t, int h, int n_kb,
                                          int* kb, int* qs, int* rows, int* sel, int* status) {
  *rows = h ? pq.w : pq.y;
  *sel = h ? t.w : t.z;
  *qs = h ? pq.z : pq.x;
  if (*rows <= 0 || *sel == -2) return false;
  const int kr = t.x;
  if (kr < 0 || (kr & 127) != 0 || t.y != kr + 64 || (*qs & 127) != 0 || kr / 128 >= n_kb) {
    atomicOr(status, 1);  // not an aligned single-stream block plan
    return false;
  }
  *kb = kr / 128;
  return true;
}

__global__ void tplan_count_kernel(const int4* __restrict__ pairs, int np,
                                   const int4* __restrict__ kv_tiles, int n_kb, int* cnt,
                                   int* status) {
  for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < np; p += gridDim.x * blockDim.x) {
    const int4 pq = pairs[2 * p], pk = pairs[2 * p + 1];
    for (int e = pk.x; e < pk.y; ++e) {
      const int4 t = kv_tiles[e];
      for (int h = 0; h < 2; ++h) {
        int kb, qs, rows, sel;
        if (tplan_ref(pq, t, h, n_kb, &kb, &qs, &rows, &sel, status)) atomicAdd(&cnt[kb], 1);
      }
    }
  }
}

// Exclusive scan of n counts by one block: off[0..n], the total in off[n].
__global__ void tplan_scan_kernel(const int* cnt, int n, int* off) {
  __shared__ int part[1024];
  const int t = threadIdx.x, T = blockDim.x;
  const int per = (n + T - 1) / T;
  const int b = t * per, e = min(n, b + per);
  int s = 0;
  for (int i = b; i < e; ++i) s += cnt[i];
  part[t] = s;
  __syncthreads();
  if (t == 0) {
    int run = 0;
    for (int i = 0; i < T; ++i) {
      const int v = part[i];
      part[i] = run;
      run += v;
    }
    off[n] = run;
  }
  __syncthreads();
  int run = part[t];
  for (int i = b; i < e; ++i) {
    off[i] = run;
    run += cnt[i];
  }
}

__global__ void tplan_fill_kernel(const int4* __restrict__ pairs, int np,
                                  const int4* __restrict__ kv_tiles, int n_kb, const int* off,
                                  int* fill, int4* ent, int capacity, int* status) {
  for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < np; p += gridDim.x * blockDim.x) {
    const int4 pq = pairs[2 * p], pk = pairs[2 * p + 1];
    for (int e = pk.x; e < pk.y; ++e) {
      const int4 t = kv_tiles[e];
      for (int h = 0; h < 2; ++h) {
        int kb, qs, rows, sel;
        if (!tplan_ref(pq, t, h, n_kb, &kb, &qs, &rows, &sel, status)) continue;
        const int slot = off[kb] + atomicAdd(&fill[kb], 1);
        if (slot >= capacity) {
          atomicOr(status, 2);
          continue;
        }
        ent[slot] = make_int4(qs, rows, sel, qs >> 7);
      }
    }
  }
}

// Each key block's list in ascending query order (deterministic gradients).
__global__ void tplan_sort_kernel(const int* off, int n_kb, int4* ent, int capacity) {
  for (int kb = blockIdx.x * blockDim.x + threadIdx.x; kb < n_kb; kb += gridDim.x * blockDim.x) {
    const int b = off[kb], e = min(off[kb + 1], capacity);
    for (int i = b + 1; i < e; ++i) {
      const int4 x = ent[i];
      int j = i - 1;
      while (j >= b && ent[j].w > x.w) {
        ent[j + 1] = ent[j];
        --j;
      }
      ent[j + 1] = x;
    }
  }
}

// One warp per 128x128 bit matrix: out row j (a key) bit r = in row r bit j.
__global__ void mask_transpose_kernel(const uint4* __restrict__ in, int n, uint4* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t w0 = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t mi = w0; mi < n; mi += nw) {
    uint4 m[4];
#pragma unroll
    for (int g = 0; g < 4; ++g) m[g] = in[mi * 128 + 32 * g + lane];
#pragma unroll 1
    for (int wq = 0; wq < 4; ++wq) {
      uint32_t col[4];
#pragma unroll
      for (int g = 0; g < 4; ++g) col[g] = word_of(m[g], wq);
#pragma unroll 4
      for (int b = 0; b < 32; ++b) {
        const uint32_t x0 = __ballot_sync(0xffffffffu, (col[0] >> b) & 1u);
        const uint32_t x1 = __ballot_sync(0xffffffffu, (col[1] >> b) & 1u);
        const uint32_t x2 = __ballot_sync(0xffffffffu, (col[2] >> b) & 1u);
        const uint32_t x3 = __ballot_sync(0xffffffffu, (col[3] >> b) & 1u);
        if (lane == b) out[mi * 128 + 32 * wq + b] = make_uint4(x0, x1, x2, x3);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// dQ: one CTA per (query tile, head)
// ---------------------------------------------------------------------------
struct DqMaps {
  CUtensorMap q, dout, k, v;
};

struct DqArgs {
  const int4* pairs;
  const int4* kv_tiles;
  const uint4* masks;
  int mask_stride, mask_row_and;
  const float* lse_t;
  const float* delta;
  int64_t rows_pad;
  __nv_bfloat16* dq;
  int64_t dq_stride;
  float scale_log2, scale;
  int n_pairs, n_heads;
  int* err;
};

constexpr int kDqSmemQ = 0;
constexpr int kDqSmemDo = kTile;
constexpr int kDqSmemK = 2 * kTile;
constexpr int kDqSmemV = kDqSmemK + kStages * kTile;
constexpr int kDqSmemBar = kDqSmemV + kStages * kTile;
constexpr int kDqNumBars = 1 + 3 * kStages + 5;
constexpr int kDqSmemBytes = kDqSmemBar + kDqNumBars * 8 + 16 + 1024;

__global__ void __launch_bounds__(384, 1)
    bwd_dq_kernel(const __grid_constant__ DqMaps m, DqArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kDqSmemBar);
  uint64_t* q_full = bars;
  uint64_t* k_full = q_full + 1;
  uint64_t* v_full = k_full + kStages;
  uint64_t* kv_empty = v_full + kStages;
  uint64_t* s_full = kv_empty + kStages;  // [sub-tile]
  uint64_t* ds_full = s_full + 2;         // [sub-tile], its warpgroup
  uint64_t* o_final = ds_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kDqNumBars);

  const int warp = warp_id(), lane = lane_id();
  const int head = blockIdx.x / (2 * a.n_pairs);
  const int item = blockIdx.x % (2 * a.n_pairs);
  const int pr = item >> 1, h = item & 1;
  const int4 pq = a.pairs[2 * pr], pk = a.pairs[2 * pr + 1];
  const int q_start = h ? pq.z : pq.x, q_rows = h ? pq.w : pq.y;
  if (q_rows <= 0) return;  // uniform: before any barrier or TMEM allocation
  const int kv_begin = pk.x, kv_end = pk.y;
  const int mask_stride = pk.z == 1 ? kBM : a.mask_stride;
  const int mask_row_and = pk.z == 1 ? kBM - 1 : a.mask_row_and;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(k_full + s, 1);
      mbar_init(v_full + s, 1);
      mbar_init(kv_empty + s, 1);
    }
    for (int g = 0; g < 2; ++g) {
      mbar_init(s_full + g, 1);
      mbar_init(ds_full + g, 128);
    }
    mbar_init(o_final, 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kBwdTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  const int col = head * kHD;
  constexpr uint32_t kColS = 0, kColDp = 128, kColDq = 256;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------- Q, dO, then K and V tiles
    prefetch_tmap(&m.q);
    prefetch_tmap(&m.k);
    mbar_arrive_expect_tx(q_full, 2 * kTile);
    tma_load_2d(smem + kDqSmemQ, &m.q, q_full, col, q_start);
    tma_load_2d(smem + kDqSmemQ + kHalf, &m.q, q_full, col + 64, q_start);
    tma_load_2d(smem + kDqSmemDo, &m.dout, q_full, col, q_start);
    tma_load_2d(smem + kDqSmemDo + kHalf, &m.dout, q_full, col + 64, q_start);
    int c = 0;
    for (int e = kv_begin; e < kv_end; ++e) {
      const int4 t = a.kv_tiles[e];
      if ((h ? t.w : t.z) == -2) continue;
      const int st = c % kStages;
      if (c >= kStages && !mbar_wait(kv_empty + st, ((c / kStages) - 1) & 1, a.err, 31)) break;
      load_kv_tile<1>(smem + kDqSmemK + st * kTile, &m.k, k_full + st, col, t.x, t.y);
      load_kv_tile<1>(smem + kDqSmemV + st * kTile, &m.v, v_full + st, col, t.x, t.y);
      ++c;
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    const uint32_t q_lo = sdesc_lo_kmajor(smem_u32(smem + kDqSmemQ));
    const uint32_t do_lo = sdesc_lo_kmajor(smem_u32(smem + kDqSmemDo));
    const uint32_t k_lo0 = sdesc_lo_kmajor(smem_u32(smem + kDqSmemK));
    const uint32_t k_mn0 = sdesc_lo_mnmajor(smem_u32(smem + kDqSmemK));
    const uint32_t v_lo0 = sdesc_lo_kmajor(smem_u32(smem + kDqSmemV));
    // Sub-tiles g = 0, 1 (keys 64g.. of a tile) alternate as in the forward:
    //   S0(0) S1(0) | dQ0(0) S0(1) dQ1(0) S1(1) | dQ0(1) S0(2) dQ1(1) S1(2) | ...
    // S_g(j+1) overwrites the dS_g(j) that dQ_g(j), issued just before it, reads.
    auto used = [&](int e) {
      while (e < kv_end && (h ? a.kv_tiles[e].w : a.kv_tiles[e].z) == -2) ++e;
      return e;
    };
    bool ok = mbar_wait(q_full, 0, a.err, 32);
    int e = used(kv_begin);
    if (ok && e < kv_end) {
      ok = mbar_wait(k_full, 0, a.err, 33) && mbar_wait(v_full, 0, a.err, 34);
      if (ok) {
        tc_fence_after();
        issue_s64<0>(tbase + kColS, q_lo, k_lo0);   // S = Q K^T
        issue_s64<0>(tbase + kColDp, do_lo, v_lo0);  // dP = dO V^T
        umma_commit(s_full);
        issue_s64<1>(tbase + kColS, q_lo, k_lo0);
        issue_s64<1>(tbase + kColDp, do_lo, v_lo0);
        umma_commit(s_full + 1);
      }
    }
    for (int c = 0; ok && e < kv_end; ++c) {
      const int st = c % kStages, stn = (c + 1) % kStages;
      const uint32_t off = (st * kTile) >> 4, offn = (stn * kTile) >> 4;
      const int en = used(e + 1);
      const bool more = en < kv_end;
      if (!mbar_wait(ds_full, c & 1, a.err, 35)) break;
      tc_fence_after();
      issue_pv_sub<0>(tbase + kColDq, tbase + kColS, k_mn0 + off, c > 0);  // dQ += dS K
      if (more) {
        const uint32_t phn = ((c + 1) / kStages) & 1;
        if (!mbar_wait(k_full + stn, phn, a.err, 33) || !mbar_wait(v_full + stn, phn, a.err, 34))
          break;
        tc_fence_after();
        issue_s64<0>(tbase + kColS, q_lo, k_lo0 + offn);
        issue_s64<0>(tbase + kColDp, do_lo, v_lo0 + offn);
        umma_commit(s_full);
      }
      if (!mbar_wait(ds_full + 1, c & 1, a.err, 38)) break;
      tc_fence_after();
      issue_pv_sub<1>(tbase + kColDq, tbase + kColS, k_mn0 + off, true);
      umma_commit(kv_empty + st);
      if (more) {
        issue_s64<1>(tbase + kColS, q_lo, k_lo0 + offn);
        issue_s64<1>(tbase + kColDp, do_lo, v_lo0 + offn);
        umma_commit(s_full + 1);
      }
      e = en;
    }
    umma_commit(o_final);
  } else if (warp >= 4) {
    // --------------------------------- dS of one query row, half its keys
    const int grp = warp >= 8 ? 1 : 0;
    const int r = threadIdx.x - 128 - 128 * grp;
    const uint32_t lane_base = static_cast<uint32_t>(32 * (warp & 3)) << 16;
    const uint32_t t_s = tbase + lane_base + kColS, t_dp = tbase + lane_base + kColDp;
    const bool valid = r < q_rows;
    const int64_t grow = (int64_t)q_start + r;
    const float lse2 = valid ? a.lse_t[head * a.rows_pad + grow] : INFINITY;
    const float dlt = valid ? a.delta[head * a.rows_pad + grow] : 0.f;
    const float sl2 = a.scale_log2;
    int c = 0;
    bool ok = true;
    for (int e = kv_begin; e < kv_end; ++e) {
      const int4 t = a.kv_tiles[e];
      const int sel = h ? t.w : t.z;
      if (sel == -2) continue;
      uint4 mk = make_uint4(~0u, ~0u, ~0u, ~0u);
      if (sel >= 0) mk = a.masks[(int64_t)sel * mask_stride + (r & mask_row_and)];
      if (!mbar_wait(s_full + grp, c & 1, a.err, 36)) {
        ok = false;
        break;
      }
      tc_fence_after();
#pragma unroll 1
      for (int q = 2 * grp; q < 2 * grp + 2; ++q) {
        uint32_t sv[32], dv[32];
        tmem_ld32(t_s + 32 * q, sv);
        tmem_ld32(t_dp + 32 * q, dv);
        tmem_wait_ld();
        const uint32_t w = valid ? word_of(mk, q) : 0u;
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float ds[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int kk = 2 * i + u;
            const float p = ((w >> kk) & 1u)
                                ? ex2_approx(fmaf(__uint_as_float(sv[kk]), sl2, -lse2))
                                : 0.f;
            ds[u] = p * (__uint_as_float(dv[kk]) - dlt);
          }
          pk[i] = pack_bf16x2(ds[0], ds[1]);
        }
        // dS of keys 32q.. over this group's S columns (already read)
        tmem_st16(t_s + packed_col(q), pk);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(ds_full + grp);
      ++c;
    }
    __nv_bfloat16* dst = a.dq + grow * a.dq_stride + col;
    if (ok && c > 0) {
      if (mbar_wait(o_final, 0, a.err, 37)) {
        tc_fence_after();
        store_row_bf16(tbase + lane_base + kColDq, a.scale, dst, valid, 2 * grp);
      }
    } else if (ok && valid) {
      zero_row(dst, 2 * grp);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, kBwdTmemCols);
  }
}

// ---------------------------------------------------------------------------
// dK, dV: one CTA per (key block, head)
// ---------------------------------------------------------------------------
struct DkvArgs {
  const int* k_off;
  const int4* k_ent;
  const uint4* t_masks;
  const float* lse_t;
  const float* delta;
  int64_t rows_pad;
  __nv_bfloat16* dk;
  __nv_bfloat16* dv;
  int64_t dk_stride, dv_stride, kv_rows;
  float scale_log2, scale;
  int n_kb, n_heads;
  int* err;
};

constexpr int kKvSmemK = 0;
constexpr int kKvSmemV = kTile;
constexpr int kKvSmemStage = 2 * kTile;  // per stage: Q, dO
constexpr int kKvSmemVec = kKvSmemStage + kStages * 2 * kTile;  // per stage: lse[128], delta[128]
constexpr int kKvSmemBar = kKvSmemVec + kStages * 1024;
constexpr int kKvNumBars = 2 + 2 * kStages + 5;
constexpr int kKvSmemBytes = kKvSmemBar + kKvNumBars * 8 + 16 + 1024;

__global__ void __launch_bounds__(384, 1)
    bwd_dkv_kernel(const __grid_constant__ DqMaps m, DkvArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kKvSmemBar);
  uint64_t* k_full = bars;
  uint64_t* v_full = bars + 1;
  uint64_t* qd_full = bars + 2;
  uint64_t* qd_empty = qd_full + kStages;
  uint64_t* s_full = qd_empty + kStages;  // [sub-tile]
  uint64_t* p_full = s_full + 2;          // [sub-tile], its warpgroup
  uint64_t* o_final = p_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kKvNumBars);

  const int warp = warp_id(), lane = lane_id();
  const int head = blockIdx.x / a.n_kb;
  const int kb = blockIdx.x % a.n_kb;
  const int ent0 = a.k_off[kb], n_ent = a.k_off[kb + 1] - ent0;
  const int col = head * kHD;
  const int key0 = kb * kBN;

  if (threadIdx.x == 0) {
    mbar_init(k_full, 1);
    mbar_init(v_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(qd_full + s, 1);
      mbar_init(qd_empty + s, 1);
    }
    for (int g = 0; g < 2; ++g) {
      mbar_init(s_full + g, 1);
      mbar_init(p_full + g, 128);
    }
    mbar_init(o_final, 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kBwdTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  constexpr uint32_t kColS = 0, kColDp = 128, kColDk = 256, kColDv = 384;

  if (warp == 0 && lane == 0 && n_ent > 0) {
    // -------------------------- K, V of the block, then Q, dO, lse, Delta tiles
    prefetch_tmap(&m.q);
    prefetch_tmap(&m.dout);
    load_kv_tile<1>(smem + kKvSmemK, &m.k, k_full, col, key0, key0 + 64);
    load_kv_tile<1>(smem + kKvSmemV, &m.v, v_full, col, key0, key0 + 64);
    for (int i = 0; i < n_ent; ++i) {
      const int st = i % kStages;
      if (i >= kStages && !mbar_wait(qd_empty + st, ((i / kStages) - 1) & 1, a.err, 41)) break;
      const int4 e = a.k_ent[ent0 + i];
      uint8_t* sq = smem + kKvSmemStage + st * 2 * kTile;
      float* vec = reinterpret_cast<float*>(smem + kKvSmemVec + st * 1024);
      mbar_arrive_expect_tx(qd_full + st, 2 * kTile + 1024);
      tma_load_2d(sq, &m.q, qd_full + st, col, e.x);
      tma_load_2d(sq + kHalf, &m.q, qd_full + st, col + 64, e.x);
      tma_load_2d(sq + kTile, &m.dout, qd_full + st, col, e.x);
      tma_load_2d(sq + kTile + kHalf, &m.dout, qd_full + st, col + 64, e.x);
      bulk_load(vec, a.lse_t + head * a.rows_pad + e.x, 512, qd_full + st);
      bulk_load(vec + 128, a.delta + head * a.rows_pad + e.x, 512, qd_full + st);
    }
  } else if (warp == 1 && lane == 0 && n_ent > 0) {
    // ------------------------------------------------------------ MMA issuer
    const uint32_t k_lo = sdesc_lo_kmajor(smem_u32(smem + kKvSmemK));
    const uint32_t v_lo = sdesc_lo_kmajor(smem_u32(smem + kKvSmemV));
    const uint32_t sq_lo = sdesc_lo_kmajor(smem_u32(smem + kKvSmemStage));
    const uint32_t sq_mn = sdesc_lo_mnmajor(smem_u32(smem + kKvSmemStage));
    // Sub-tiles g = 0, 1 (query rows 64g.. of a tile) alternate:
    //   S0(0) S1(0) | PV0(0) S0(1) PV1(0) S1(1) | ...   (PV_g: dV and dK)
    bool ok = mbar_wait(k_full, 0, a.err, 42) && mbar_wait(v_full, 0, a.err, 43) &&
              mbar_wait(qd_full, 0, a.err, 44);
    if (ok) {
      tc_fence_after();
      issue_s64<0>(tbase + kColS, k_lo, sq_lo);            // S^T = K Q^T
      issue_s64<0>(tbase + kColDp, v_lo, sq_lo + (kTile >> 4));  // dP^T = V dO^T
      umma_commit(s_full);
      issue_s64<1>(tbase + kColS, k_lo, sq_lo);
      issue_s64<1>(tbase + kColDp, v_lo, sq_lo + (kTile >> 4));
      umma_commit(s_full + 1);
    }
    for (int i = 0; ok && i < n_ent; ++i) {
      const int st = i % kStages, stn = (i + 1) % kStages;
      const bool more = i + 1 < n_ent;
      const uint32_t oq = (st * 2 * kTile) >> 4, od = (st * 2 * kTile + kTile) >> 4;
      const uint32_t oqn = (stn * 2 * kTile) >> 4, odn = (stn * 2 * kTile + kTile) >> 4;
      if (!mbar_wait(p_full, i & 1, a.err, 45)) break;
      tc_fence_after();
      issue_pv_sub<0>(tbase + kColDv, tbase + kColS, sq_mn + od, i > 0);   // dV += P^T dO
      issue_pv_sub<0>(tbase + kColDk, tbase + kColDp, sq_mn + oq, i > 0);  // dK += dS^T Q
      if (more) {
        if (!mbar_wait(qd_full + stn, ((i + 1) / kStages) & 1, a.err, 44)) break;
        tc_fence_after();
        issue_s64<0>(tbase + kColS, k_lo, sq_lo + oqn);
        issue_s64<0>(tbase + kColDp, v_lo, sq_lo + odn);
        umma_commit(s_full);
      }
      if (!mbar_wait(p_full + 1, i & 1, a.err, 49)) break;
      tc_fence_after();
      issue_pv_sub<1>(tbase + kColDv, tbase + kColS, sq_mn + od, true);
      issue_pv_sub<1>(tbase + kColDk, tbase + kColDp, sq_mn + oq, true);
      umma_commit(qd_empty + st);
      if (more) {
        issue_s64<1>(tbase + kColS, k_lo, sq_lo + oqn);
        issue_s64<1>(tbase + kColDp, v_lo, sq_lo + odn);
        umma_commit(s_full + 1);
      }
    }
    umma_commit(o_final);
  } else if (warp >= 4) {
    // ------------------------- P^T, dS^T of one key row, half its queries
    const int grp = warp >= 8 ? 1 : 0;
    const int j = threadIdx.x - 128 - 128 * grp;
    const uint32_t lane_base = static_cast<uint32_t>(32 * (warp & 3)) << 16;
    const uint32_t t_s = tbase + lane_base + kColS, t_dp = tbase + lane_base + kColDp;
    const float sl2 = a.scale_log2;
    bool ok = true;
    for (int i = 0; i < n_ent; ++i) {
      const int st = i % kStages;
      const int4 e = a.k_ent[ent0 + i];
      uint4 mk = make_uint4(~0u, ~0u, ~0u, ~0u);
      if (e.z >= 0) mk = a.t_masks[(int64_t)e.z * 128 + j];
      // the stage's lse / Delta vectors are visible after its load barrier
      if (!mbar_wait(qd_full + st, (i / kStages) & 1, a.err, 46) ||
          !mbar_wait(s_full + grp, i & 1, a.err, 47)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const float* vec = reinterpret_cast<const float*>(smem + kKvSmemVec + st * 1024);
#pragma unroll 1
      for (int q = 2 * grp; q < 2 * grp + 2; ++q) {
        uint32_t sv[32], dv[32];
        tmem_ld32(t_s + 32 * q, sv);
        tmem_ld32(t_dp + 32 * q, dv);
        tmem_wait_ld();
        uint32_t w = word_of(mk, q);
        const int lim = e.y - 32 * q;  // query rows of the tile in this word
        if (lim < 32) w &= lim <= 0 ? 0u : ((1u << lim) - 1u);
        uint32_t pp[16], pd[16];
#pragma unroll
        for (int i2 = 0; i2 < 16; ++i2) {
          float p2[2], d2[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int rr = 2 * i2 + u;
            const float l = vec[32 * q + rr], dl = vec[128 + 32 * q + rr];
            const float p = ((w >> rr) & 1u)
                                ? ex2_approx(fmaf(__uint_as_float(sv[rr]), sl2, -l))
                                : 0.f;
            p2[u] = p;
            d2[u] = p * (__uint_as_float(dv[rr]) - dl);
          }
          pp[i2] = pack_bf16x2(p2[0], p2[1]);
          pd[i2] = pack_bf16x2(d2[0], d2[1]);
        }
        tmem_st16(t_s + packed_col(q), pp);
        tmem_st16(t_dp + packed_col(q), pd);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(p_full + grp);
    }
    const int64_t krow = (int64_t)key0 + j;
    const bool store = krow < a.kv_rows;
    __nv_bfloat16* dkr = a.dk + krow * a.dk_stride + col;
    __nv_bfloat16* dvr = a.dv + krow * a.dv_stride + col;
    if (ok && n_ent > 0) {
      if (mbar_wait(o_final, 0, a.err, 48)) {
        tc_fence_after();
        store_row_bf16(tbase + lane_base + kColDk, a.scale, dkr, store, 2 * grp);
        store_row_bf16(tbase + lane_base + kColDv, 1.f, dvr, store, 2 * grp);
      }
    } else if (ok && store) {
      zero_row(dkr, 2 * grp);
      zero_row(dvr, 2 * grp);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, kBwdTmemCols);
  }
}

int check_rows(const void* p, int64_t stride, const char* what) {
  if ((reinterpret_cast<uintptr_t>(p) & 15) || stride % 8) {
    set_error(HIER_EVALUE, "%s must be 16-byte aligned with a row stride that is a multiple of 8 "
              "elements", what);
    return HIER_EVALUE;
  }
  return HIER_OK;
}

int grid_blocks(int64_t work, int per_block) {
  const int64_t b = (work + per_block - 1) / per_block;
  return (int)(b < 148 * 8 ? (b > 0 ? b : 1) : 148 * 8);
}

}  // namespace
}  // namespace hier

using namespace hier;

extern "C" int hier_attn_bwd_prep(const void* o, int64_t o_stride, const void* dout,
                                  int64_t do_stride, const float* lse, int64_t rows, int32_t H,
                                  int32_t D, float* delta, float* lse_t, int64_t rows_pad,
                                  void* stream) {
  clear_error();
  if (D != kHD || H <= 0 || rows < 0 || rows_pad < rows || rows_pad % 128) {
    set_error(HIER_EVALUE, "hier_attn_bwd_prep: head_dim must be 128 (got %d), heads > 0, "
              "rows_pad a multiple of 128 >= rows", D);
    return HIER_EVALUE;
  }
  int rc = check_rows(o, o_stride, "O");
  if (!rc) rc = check_rows(dout, do_stride, "dO");
  if (rc) return rc;
  if (rows_pad == 0) return HIER_OK;
  bwd_prep_kernel<<<grid_blocks(rows_pad, 8), 256, 0, (cudaStream_t)stream>>>(
      (const __nv_bfloat16*)o, o_stride, (const __nv_bfloat16*)dout, do_stride, lse, rows,
      rows_pad, H, delta, lse_t);
  HIER_CHECK_CUDA(cudaGetLastError(), "bwd_prep_kernel launch");
  return HIER_OK;
}

extern "C" int hier_bwd_plan_transpose(const int32_t* q_pairs, int32_t n_pairs,
                                       const int32_t* kv_tiles, const uint32_t* row_masks,
                                       int32_t n_masks, int32_t n_kb, int32_t* workspace,
                                       int32_t* k_off, int32_t* k_ent, int32_t capacity,
                                       uint32_t* t_masks, int32_t* status, void* stream) {
  clear_error();
  if (n_pairs < 0 || n_masks < 0 || n_kb <= 0 || capacity < 0) {
    set_error(HIER_EVALUE, "hier_bwd_plan_transpose: invalid sizes (pairs %d, masks %d, key "
              "blocks %d, capacity %d)", n_pairs, n_masks, n_kb, capacity);
    return HIER_EVALUE;
  }
  cudaStream_t s = (cudaStream_t)stream;
  int32_t* cnt = workspace;
  int32_t* fill = workspace + n_kb;
  HIER_CHECK_CUDA(cudaMemsetAsync(workspace, 0, sizeof(int32_t) * 2 * (size_t)n_kb, s),
                  "transpose workspace clear");
  HIER_CHECK_CUDA(cudaMemsetAsync(status, 0, sizeof(int32_t), s), "transpose status clear");
  const int pb = grid_blocks(n_pairs, 128);
  if (n_pairs > 0)
    tplan_count_kernel<<<pb, 128, 0, s>>>((const int4*)q_pairs, n_pairs, (const int4*)kv_tiles,
                                           n_kb, cnt, status);
  tplan_scan_kernel<<<1, 1024, 0, s>>>(cnt, n_kb, k_off);
  if (n_pairs > 0)
    tplan_fill_kernel<<<pb, 128, 0, s>>>((const int4*)q_pairs, n_pairs, (const int4*)kv_tiles,
                                          n_kb, k_off, fill, (int4*)k_ent, capacity, status);
  tplan_sort_kernel<<<grid_blocks(n_kb, 128), 128, 0, s>>>(k_off, n_kb, (int4*)k_ent, capacity);
  if (n_masks > 0)
    mask_transpose_kernel<<<grid_blocks((int64_t)n_masks * 32, 256), 256, 0, s>>>(
        (const uint4*)row_masks, n_masks, (uint4*)t_masks);
  HIER_CHECK_CUDA(cudaGetLastError(), "transposed plan kernels launch");
  return HIER_OK;
}

namespace {

int bwd_maps(DqMaps* m, const void* q, int64_t q_rows, int64_t q_stride, const void* k,
             const void* v, int64_t kv_rows, int64_t kv_stride, const void* dout,
             int64_t do_stride, int32_t H) {
  if (kv_rows > kRowMask) {
    set_error(HIER_EVALUE, "key/value rows %lld exceed %d", (long long)kv_rows, kRowMask);
    return HIER_EVALUE;
  }
  const uint64_t dim = (uint64_t)H * kHD;
  int rc = make_tmap_bf16_2d(&m->q, q, dim, (uint64_t)q_rows, q_stride, 64, 128);
  if (!rc) rc = make_tmap_bf16_2d(&m->dout, dout, dim, (uint64_t)q_rows, do_stride, 64, 128);
  if (!rc) rc = make_tmap_bf16_2d(&m->k, k, dim, (uint64_t)kv_rows, kv_stride, 64, 64);
  if (!rc) rc = make_tmap_bf16_2d(&m->v, v, dim, (uint64_t)kv_rows, kv_stride, 64, 64);
  return rc;
}

}  // namespace

extern "C" int hier_attn_bwd_dq(const void* q, int64_t q_rows, int64_t q_stride, const void* k,
                                const void* v, int64_t kv_rows, int64_t kv_stride,
                                const void* dout, int64_t do_stride, const float* lse_t,
                                const float* delta, int64_t rows_pad, int32_t H, int32_t D,
                                const int32_t* q_pairs, int32_t n_pairs, const int32_t* kv_tiles,
                                const uint32_t* row_masks, int32_t mask_rows,
                                float softmax_scale, void* dq, int64_t dq_stride,
                                int32_t* dev_err, void* stream) {
  clear_error();
  if (D != kHD || H <= 0 || n_pairs < 0 || (mask_rows != 1 && mask_rows != kBM) ||
      rows_pad < q_rows || (int64_t)n_pairs * 2 * H > INT32_MAX) {
    set_error(HIER_EVALUE, "hier_attn_bwd_dq: head_dim must be 128 (got %d), heads > 0, "
              "mask_rows 1 or 128, rows_pad >= query rows", D);
    return HIER_EVALUE;
  }
  if (n_pairs == 0) return HIER_OK;
  int rc = check_rows(dq, dq_stride, "dQ");
  if (rc) return rc;
  DqMaps m;
  rc = bwd_maps(&m, q, q_rows, q_stride, k, v, kv_rows, kv_stride, dout, do_stride, H);
  if (rc) return rc;
  HIER_CHECK_CUDA(cudaFuncSetAttribute(bwd_dq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       kDqSmemBytes),
                  "cudaFuncSetAttribute(bwd_dq_kernel)");
  DqArgs a;
  a.pairs = (const int4*)q_pairs;
  a.kv_tiles = (const int4*)kv_tiles;
  a.masks = (const uint4*)row_masks;
  a.mask_stride = mask_rows;
  a.mask_row_and = mask_rows - 1;
  a.lse_t = lse_t;
  a.delta = delta;
  a.rows_pad = rows_pad;
  a.dq = (__nv_bfloat16*)dq;
  a.dq_stride = dq_stride;
  a.scale_log2 = softmax_scale * 1.4426950408889634f;
  a.scale = softmax_scale;
  a.n_pairs = n_pairs;
  a.n_heads = H;
  a.err = dev_err;
  bwd_dq_kernel<<<n_pairs * 2 * H, 384, kDqSmemBytes, (cudaStream_t)stream>>>(m, a);
  HIER_CHECK_CUDA(cudaGetLastError(), "bwd_dq_kernel launch");
  return HIER_OK;
}

extern "C" int hier_attn_bwd_dkv(const void* q, int64_t q_rows, int64_t q_stride, const void* k,
                                 const void* v, int64_t kv_rows, int64_t kv_stride,
                                 const void* dout, int64_t do_stride, const float* lse_t,
                                 const float* delta, int64_t rows_pad, int32_t H, int32_t D,
                                 const int32_t* k_off, const int32_t* k_ent,
                                 const uint32_t* t_masks, int32_t n_kb, float softmax_scale,
                                 void* dk, int64_t dk_stride, void* dv, int64_t dv_stride,
                                 int32_t* dev_err, void* stream) {
  clear_error();
  if (D != kHD || H <= 0 || n_kb < 0 || rows_pad < q_rows || rows_pad % 128 ||
      (int64_t)n_kb * kBN < kv_rows || (int64_t)n_kb * H > INT32_MAX) {
    set_error(HIER_EVALUE, "hier_attn_bwd_dkv: head_dim must be 128 (got %d), heads > 0, "
              "rows_pad a multiple of 128 >= query rows, n_kb * 128 >= key rows", D);
    return HIER_EVALUE;
  }
  if (n_kb == 0) return HIER_OK;
  int rc = check_rows(dk, dk_stride, "dK");
  if (!rc) rc = check_rows(dv, dv_stride, "dV");
  if (rc) return rc;
  DqMaps m;
  rc = bwd_maps(&m, q, q_rows, q_stride, k, v, kv_rows, kv_stride, dout, do_stride, H);
  if (rc) return rc;
  HIER_CHECK_CUDA(cudaFuncSetAttribute(bwd_dkv_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, kKvSmemBytes),
                  "cudaFuncSetAttribute(bwd_dkv_kernel)");
  DkvArgs a;
  a.k_off = k_off;
  a.k_ent = (const int4*)k_ent;
  a.t_masks = (const uint4*)t_masks;
  a.lse_t = lse_t;
  a.delta = delta;
  a.rows_pad = rows_pad;
  a.dk = (__nv_bfloat16*)dk;
  a.dv = (__nv_bfloat16*)dv;
  a.dk_stride = dk_stride;
  a.dv_stride = dv_stride;
  a.kv_rows = kv_rows;
  a.scale_log2 = softmax_scale * 1.4426950408889634f;
  a.scale = softmax_scale;
  a.n_kb = n_kb;
  a.n_heads = H;
  a.err = dev_err;
  bwd_dkv_kernel<<<n_kb * H, 384, kKvSmemBytes, (cudaStream_t)stream>>>(m, a);
  HIER_CHECK_CUDA(cudaGetLastError(), "bwd_dkv_kernel launch");
  return HIER_OK;
}
