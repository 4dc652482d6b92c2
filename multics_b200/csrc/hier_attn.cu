// Block-sparse flash attention forward for sm_100a (tcgen05 + TMEM + TMA).
//
// One CTA per (query pair, head): a query pair is two 128-row query tiles
// ("halves") that share one list of 128-key tiles; each key tile carries one
// mask selector per half (full / skip / index of a per-row key bitmask).
//
// Per half h and key tile j the tensor pipe runs S_h(j) = Q_h K(j)^T
// (128 x 128, fp32 in TMEM) and O_h += P_h(j) V(j); the softmax warpgroup of
// the half turns S_h(j) into P_h(j) in between.  The two halves ping-pong:
// while one half's softmax runs, the other half's MMAs keep the tensor core
// busy.  One thread issues all MMAs in the order
//
//   S0(0) S1(0) | PV0(0) S0(1) PV1(0) S1(1) | PV0(1) S0(2) PV1(1) S1(2) | ...
//
// which keeps the two halves out of phase (with one issuer per half they
// drift into phase and their softmaxes contend for the exp unit).
//
// Warp roles (384 threads, three warpgroups):
//   warp 0      TMA producer of Q0, Q1 and the K tiles (3-stage ring)
//   warp 1      MMA issuer (one lane), TMEM allocator
//   warp 2      TMA producer of the V tiles (2-stage ring)
//   warp 3      idle
//   warps 4-7   softmax of half 0 (one query row per thread)
//   warps 8-11  softmax of half 1
// setmaxnreg moves registers from the control warpgroup to the softmax ones.
//
// Tensor memory (512 columns): S0 | S1 | O0 | O1, 128 fp32 columns each.
// P (bf16, two per 32-bit column) is written over the first 64 columns of the
// S buffer it came from and read by the TS-form MMA; S_h(j+1) is issued after
// PV_h(j) by the same thread, and tcgen05 MMAs of one thread execute in issue
// order, so it never overwrites P_h(j) before PV_h(j) has read it.  The
// softmax signals P's first 64 keys before it computes the other 64, and
// PV_h(j) is issued in those two halves: the tensor core multiplies the first
// half while the exponentials of the second are still being computed.
//
// Shared memory: Q0, Q1 (32 KiB each), K ring 3 x 32 KiB, V ring 2 x 32 KiB;
// each tile is two 64-column halves in the 128-byte swizzled layout, loaded
// as two 64-row TMA boxes whose pool rows come from the plan (contiguous,
// paged or gathered pools use the same code).  Shared-memory descriptors are
// built once per operand and advanced by adding constant offsets.
//
// Online softmax: fp32 running max/sum per row; O is rescaled in TMEM only
// when the running max grows by more than 2^8 (the final O/l is exact for any
// reference max).  Rows without keys are written as 0.  Every mbarrier wait
// is bounded and records a timeout in dev_err instead of hanging.

#include <math.h>
#include <stdio.h>
#include <string.h>

#include "common.cuh"
#include "tile_mma.cuh"
#include "tmap.h"

namespace hier {

constexpr int kKStages = 3;
constexpr int kVStages = 2;
constexpr int kSmemQ = 0;               // Q0, Q1
constexpr int kSmemK = 2 * kTile;
constexpr int kSmemV = kSmemK + kKStages * kTile;
constexpr int kSmemBar = kSmemV + kVStages * kTile;
constexpr int kNumBars = 1 + 2 * kKStages + 2 * kVStages + 2 + 2 + 2 + 2;
constexpr int kSmemBytes = kSmemBar + 256 + 1024;  // + slack for 1024-byte alignment
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 256;
constexpr int kSkip = -2;  // mask selector: this half does not use the key tile

constexpr float kRescaleThreshold = 8.0f;  // log2 units
constexpr uint32_t kRegsControl = 40;
constexpr uint32_t kRegsSoftmax = 224;
static_assert(4 * 32 * kRegsControl + 8 * 32 * kRegsSoftmax <= 384 * 168,
              "register split exceeds the launch allocation");

struct AttnArgs {
  const int4* pairs;     // per pair: (q_start0, q_rows0, q_start1, q_rows1), (kv_begin, kv_end, -, -)
  const int4* kv_tiles;  // (pool row of keys 0-63, pool row of keys 64-127, mask0, mask1)
  const uint4* row_masks;
  const int* order;
  __nv_bfloat16* out;
  int64_t out_stride;
  const int32_t* out_rows;  // output (and lse) row of each query row; NULL: the same row
  // pairs flagged in q_pairs[7] write partial rows: row r to part_out row
  // r - part_row0 and its log-sum-exp to part_lse
  __nv_bfloat16* part_out;
  int64_t part_stride;
  float* part_lse;
  int part_row0;
  int64_t part_slot_rows;  // q_pairs[7] >> 8 = partial slot: rows of one slot
  int q2_row0;  // query rows from q2_row0 on are read from the second query map
  int n_pairs;
  int mask_stride;    // entries per partial-tile mask: 128 (per row) or 1 (per key only)
  int mask_row_and;   // 127 or 0
  float scale_log2;
  float* lse;  // optional [q_rows_total][H]: log2-sum-exp of the scaled scores per row
  int n_heads;
  int* err;
};

// Query tensor maps: rows below q2_row0 from q[0], the others from q[1].
struct QMaps {
  CUtensorMap q[2];
};

// Key and value tensor maps, one per KV stream (a contiguous pool uses one).
template <int kMaps>
struct KVMaps {
  CUtensorMap k[kMaps];
  CUtensorMap v[kMaps];
};

// Mask selector of half h for a key tile; a half without query rows skips
// every tile.
__device__ __forceinline__ int half_sel(const int4& e, int h, int use) {
  return ((use >> h) & 1) ? (h ? e.w : e.z) : kSkip;
}

struct Bars {
  uint64_t* q_full;
  uint64_t* k_full;
  uint64_t* k_empty;
  uint64_t* v_full;
  uint64_t* v_empty;
  uint64_t* s_full;   // [half]
  uint64_t* p_full;   // [half], 128 softmax threads
  uint64_t* p_lo;     // [half], 128 softmax threads: P of keys 0-63 written
  uint64_t* o_final;  // [half], one phase after the last PV
};

template <int kMaps>
__device__ __forceinline__ void control_role(const AttnArgs& a, int4 pq, int kv_begin, int n_kv,
                                             uint32_t tbase, int warp, int lane, uint8_t* smem,
                                             const QMaps& qm, const KVMaps<kMaps>& kv,
                                             const Bars& B, int col, int use) {
  if (n_kv > 0 && warp == 0 && lane == 0) {
    // -------------------------------------------------------- Q + K producer
    const bool q2a = pq.x >= a.q2_row0, q2b = pq.z >= a.q2_row0;
    const CUtensorMap* qa = &qm.q[q2a ? 1 : 0];
    const CUtensorMap* qb = &qm.q[q2b ? 1 : 0];
    const int ra = pq.x - (q2a ? a.q2_row0 : 0), rb = pq.z - (q2b ? a.q2_row0 : 0);
    prefetch_tmap(qa);
    if (kMaps == 1) prefetch_tmap(&kv.k[0]);
    mbar_arrive_expect_tx(B.q_full, 2 * kTile);
    tma_load_2d(smem + kSmemQ, qa, B.q_full, col, ra);
    tma_load_2d(smem + kSmemQ + kHalf, qa, B.q_full, col + 64, ra);
    tma_load_2d(smem + kSmemQ + kTile, qb, B.q_full, col, rb);
    tma_load_2d(smem + kSmemQ + kTile + kHalf, qb, B.q_full, col + 64, rb);
    for (int j = 0; j < n_kv; ++j) {
      const int st = j % kKStages;
      if (j >= kKStages && !mbar_wait(B.k_empty + st, ((j / kKStages) - 1) & 1, a.err, 1)) break;
      const int4 e = a.kv_tiles[kv_begin + j];
      load_kv_tile<kMaps>(smem + kSmemK + st * kTile, kv.k, B.k_full + st, col, e.x, e.y);
    }
  } else if (n_kv > 0 && warp == 2 && lane == 0) {
    // ------------------------------------------------------------ V producer
    if (kMaps == 1) prefetch_tmap(&kv.v[0]);
    for (int j = 0; j < n_kv; ++j) {
      const int st = j % kVStages;
      if (j >= kVStages && !mbar_wait(B.v_empty + st, ((j / kVStages) - 1) & 1, a.err, 2)) break;
      const int4 e = a.kv_tiles[kv_begin + j];
      load_kv_tile<kMaps>(smem + kSmemV + st * kTile, kv.v, B.v_full + st, col, e.x, e.y);
    }
  } else if (n_kv > 0 && warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    const uint32_t q_lo[2] = {sdesc_lo_kmajor(smem_u32(smem + kSmemQ)),
                              sdesc_lo_kmajor(smem_u32(smem + kSmemQ + kTile))};
    const uint32_t k_lo0 = sdesc_lo_kmajor(smem_u32(smem + kSmemK));
    const uint32_t v_lo0 = sdesc_lo_mnmajor(smem_u32(smem + kSmemV));
    int cp[2] = {0, 0};  // PVs issued per half
    if (!mbar_wait(B.q_full, 0, a.err, 3)) return;
    // Every phase of the stage barriers is waited for, used or not, so a
    // parity wait never matches an older phase.
    int4 e_cur = a.kv_tiles[kv_begin];
    if (!mbar_wait(B.k_full, 0, a.err, 4)) return;
    tc_fence_after();
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if (half_sel(e_cur, h, use) == kSkip) continue;
      issue_s(tbase + h * kBN, q_lo[h], k_lo0);
      umma_commit(B.s_full + h);
    }
    umma_commit(B.k_empty);
    for (int j = 0; j < n_kv; ++j) {
      const bool more = j + 1 < n_kv;
      const int4 e_next = more ? a.kv_tiles[kv_begin + j + 1] : e_cur;
      const int stv = j % kVStages, stk = (j + 1) % kKStages;
      if (!mbar_wait(B.v_full + stv, (j / kVStages) & 1, a.err, 5)) return;
      // PV0(j) S0(j+1) PV1(j) S1(j+1): S_h(j+1) overwrites P_h(j), which the
      // PV_h(j) issued just before it reads first (in-order execution).
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (half_sel(e_cur, h, use) != kSkip) {
          const uint32_t o_t = tbase + kColO + h * kBN, p_t = tbase + h * kBN;
          const uint32_t v_lo = v_lo0 + ((stv * kTile) >> 4);
          if (!mbar_wait(B.p_lo + h, cp[h] & 1, a.err, 6 + h)) return;
          tc_fence_after();
          issue_pv_half<0>(o_t, p_t, v_lo, cp[h] > 0);
          if (!mbar_wait(B.p_full + h, cp[h] & 1, a.err, 6 + h)) return;
          tc_fence_after();
          issue_pv_half<1>(o_t, p_t, v_lo, true);
          ++cp[h];
        }
        if (!more) continue;
        if (h == 0 && !mbar_wait(B.k_full + stk, ((j + 1) / kKStages) & 1, a.err, 4)) return;
        if (half_sel(e_next, h, use) != kSkip) {
          tc_fence_after();
          issue_s(tbase + h * kBN, q_lo[h], k_lo0 + ((stk * kTile) >> 4));
          umma_commit(B.s_full + h);
        }
      }
      umma_commit(B.v_empty + stv);
      if (more) umma_commit(B.k_empty + stk);
      e_cur = e_next;
    }
#pragma unroll
    for (int h = 0; h < 2; ++h)
      if (cp[h] > 0) umma_commit(B.o_final + h);
  }
}

// 32 bytes (8 words) to a 32-byte aligned global address.
__device__ __forceinline__ void st_global_v8(void* p, const uint32_t* w) {
  asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(w[0]),
               "r"(w[1]), "r"(w[2]), "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7])
               : "memory");
}

// O (128 x 128 fp32 in TMEM) rescaled by alpha, 8 columns at a time (few
// registers: it runs while the scores of the tile are held in registers).
__device__ __forceinline__ void rescale_o(uint32_t o_col, float alpha) {
#pragma unroll 1
  for (int q = 0; q < 16; ++q) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                   "=r"(r[6]), "=r"(r[7])
                 : "r"(o_col + q * 8));
    tmem_wait_ld();
#pragma unroll
    for (int i = 0; i < 8; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};"
                 ::"r"(o_col + q * 8), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]),
                   "r"(r[5]), "r"(r[6]), "r"(r[7])
                 : "memory");
  }
}

__device__ __forceinline__ void softmax_role(const AttnArgs& a, int4 pq, int kv_begin, int n_kv,
                                             uint32_t tbase, int warp, const Bars& B, int col,
                                             int use, bool row_masks128, int pflags) {
  const bool partial_rows = (pflags & 1) != 0;
  const int h = (warp >> 2) - 1;  // 0 for warps 4-7, 1 for warps 8-11
  const int row = threadIdx.x - 128 * (h + 1);
  const uint32_t lane_base = static_cast<uint32_t>(32 * (warp & 3)) << 16;
  const uint32_t s_col = tbase + lane_base + h * kBN;
  const uint32_t o_col = tbase + lane_base + kColO + h * kBN;
  const int q_start = h ? pq.z : pq.x;
  const int q_rows = h ? pq.w : pq.y;
  const bool store_row = row < q_rows;
  int64_t dst_row;
  __nv_bfloat16* orow;
  float* lse_out;
  if (partial_rows) {
    dst_row = (int64_t)(q_start + row) - a.part_row0 + (int64_t)(pflags >> 8) * a.part_slot_rows;
    orow = a.part_out + dst_row * a.part_stride + col;
    lse_out = a.part_lse;
  } else {
    dst_row = (a.out_rows && store_row) ? (int64_t)a.out_rows[q_start + row]
                                        : (int64_t)(q_start + row);
    orow = a.out + dst_row * a.out_stride + col;
    lse_out = a.lse;
  }
  // a pair flagged in q_pairs[6] carries one mask per query row whatever the
  // launch's mask format
  const int mask_stride = row_masks128 ? kBM : a.mask_stride;
  const int mask_row_and = row_masks128 ? kBM - 1 : a.mask_row_and;
  float m_run = -INFINITY, l_run = 0.f;  // running max in scaled log2 units
  int c = 0;                             // key tiles processed by this half
  const float sc = a.scale_log2;
  // Entries are loaded one tile ahead and a partial tile's row mask is
  // requested before the S wait, keeping both global loads off the S -> P path.
  int4 e_next = n_kv > 0 ? a.kv_tiles[kv_begin] : make_int4(0, 0, kSkip, kSkip);
  for (int j = 0; j < n_kv; ++j) {
    const int4 e = e_next;
    if (j + 1 < n_kv) e_next = a.kv_tiles[kv_begin + j + 1];
    const int mi = half_sel(e, h, use);
    if (mi == kSkip) continue;
    const bool partial = mi >= 0;  // uniform across the CTA
    uint4 mk = make_uint4(~0u, ~0u, ~0u, ~0u);
    if (partial) mk = a.row_masks[(int64_t)mi * mask_stride + (row & mask_row_and)];
    // S_h(c) is committed after PV_h(c-1), so once it is visible O holds
    // every earlier P V product and can be rescaled without another wait.
    if (!mbar_wait(B.s_full + h, c & 1, a.err, 11)) return;
    tc_fence_after();
    float sv[kBN];
    {
      uint32_t* r = reinterpret_cast<uint32_t*>(sv);
#pragma unroll
      for (int q = 0; q < 4; ++q)
        tmem_ld32(s_col + q * 32, *reinterpret_cast<uint32_t(*)[32]>(r + 32 * q));
      tmem_wait_ld();
    }
    if (partial) {
      const uint32_t w[4] = {mk.x, mk.y, mk.z, mk.w};
#pragma unroll
      for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int i = 0; i < 32; ++i)
          sv[32 * q + i] = ((w[q] >> i) & 1u) ? sv[32 * q + i] : -INFINITY;
    }
    float m8[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) m8[i] = sv[i];
#pragma unroll
    for (int i = 8; i < kBN; ++i) m8[i & 7] = fmaxf(m8[i & 7], sv[i]);
    const float mx = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])),
                           fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7]))) * sc;
    const bool grow = mx > m_run + kRescaleThreshold;
    const bool need_rescale = grow && m_run != -INFINITY;
    if (__any_sync(0xffffffffu, need_rescale)) {
      const float alpha = need_rescale ? ex2_approx(m_run - mx) : 1.f;
      rescale_o(o_col, alpha);
      l_run *= alpha;
    }
    if (grow) m_run = mx;
    const float nref = m_run == -INFINITY ? 0.f : -m_run;
    // exponent arguments and row sums two lanes at a time (fp32x2 FMA / add)
    const uint64_t sc2 = f2_pack(sc, sc), nref2 = f2_pack(nref, nref);
    uint64_t acc[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      uint32_t pk[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const uint64_t arg =
            f2_fma(f2_pack(sv[64 * half + 2 * i], sv[64 * half + 2 * i + 1]), sc2, nref2);
        float a0, a1;
        f2_unpack(arg, a0, a1);
        const float p0 = ex2_approx(a0), p1 = ex2_approx(a1);
        acc[i & 3] = f2_add(acc[i & 3], f2_pack(p0, p1));
        pk[i] = pack_bf16x2(p0, p1);
      }
      tmem_st32(s_col + 32 * half, pk);
      if (half == 0) {  // keys 0-63 of P: the first half of PV can start
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(B.p_lo + h);
      }
    }
    {
      const uint64_t s2 = f2_add(f2_add(acc[0], acc[1]), f2_add(acc[2], acc[3]));
      float s0, s1;
      f2_unpack(s2, s0, s1);
      l_run += s0 + s1;
    }
    tmem_wait_st();
    tc_fence_before();
    mbar_arrive(B.p_full + h);
    ++c;
  }
  if (c == 0) {
    if (store_row) {
      const uint4 z = make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int q = 0; q < kHD / 8; ++q) reinterpret_cast<uint4*>(orow)[q] = z;
      if (lse_out) lse_out[dst_row * a.n_heads + col / kHD] = -INFINITY;
    }
    return;
  }
  if (!mbar_wait(B.o_final + h, 0, a.err, 13)) return;
  tc_fence_after();
  const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
  if (lse_out && store_row)  // O = sum_j 2^(s_j - lse) v_j
    lse_out[dst_row * a.n_heads + col / kHD] =
        l_run > 0.f ? m_run + __log2f(l_run) : -INFINITY;
  // each thread writes its own 256-byte row; 32-byte stores fill whole
  // sectors (half as many transactions as 16-byte ones)
  const bool v8 = (reinterpret_cast<uintptr_t>(orow) & 31) == 0;
  uint32_t r[32];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    tmem_ld32(o_col + q * 32, r);
    tmem_wait_ld();
    if (store_row) {
      uint32_t w[16];
#pragma unroll
      for (int i = 0; i < 16; ++i)
        w[i] = pack_bf16x2(__uint_as_float(r[2 * i]) * inv, __uint_as_float(r[2 * i + 1]) * inv);
      if (v8) {
        st_global_v8(orow + q * 32, w);
        st_global_v8(orow + q * 32 + 16, w + 8);
      } else {
        uint4* dst = reinterpret_cast<uint4*>(orow + q * 32);
#pragma unroll
        for (int k = 0; k < 4; ++k) dst[k] = make_uint4(w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
      }
    }
  }
}

template <int kMaps>
__global__ void __launch_bounds__(384, 1)
    hier_attn_kernel(const __grid_constant__ QMaps qm,
                     const __grid_constant__ KVMaps<kMaps> kv, AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kSmemBar);
  Bars B;
  B.q_full = bars;
  B.k_full = B.q_full + 1;
  B.k_empty = B.k_full + kKStages;
  B.v_full = B.k_empty + kKStages;
  B.v_empty = B.v_full + kVStages;
  B.s_full = B.v_empty + kVStages;
  B.p_full = B.s_full + 2;
  B.p_lo = B.p_full + 2;
  B.o_final = B.p_lo + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);

  const int warp = warp_id();
  const int lane = lane_id();
  const int head = blockIdx.x / a.n_pairs;
  const int rank = blockIdx.x % a.n_pairs;
  const int pr = a.order ? a.order[rank] : rank;
  const int4 pq = a.pairs[2 * pr];
  const int4 pk = a.pairs[2 * pr + 1];
  const int kv_begin = pk.x;
  const int n_kv = pk.y - pk.x;
  const int use = (pq.y > 0 ? 1 : 0) | (pq.w > 0 ? 2 : 0);  // halves with query rows

  if (threadIdx.x == 0) {
    mbar_init(B.q_full, 1);
    for (int s = 0; s < kKStages; ++s) {
      mbar_init(B.k_full + s, 1);
      mbar_init(B.k_empty + s, 1);
    }
    for (int s = 0; s < kVStages; ++s) {
      mbar_init(B.v_full + s, 1);
      mbar_init(B.v_empty + s, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(B.s_full + i, 1);
      mbar_init(B.p_full + i, 128);
      mbar_init(B.p_lo + i, 128);
      mbar_init(B.o_final + i, 1);
    }
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  const int col = head * kHD;
  if (warp >= 4) {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsSoftmax));
    softmax_role(a, pq, kv_begin, n_kv, tbase, warp, B, col, use, pk.z == 1, pk.w);
  } else {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsControl));
    control_role<kMaps>(a, pq, kv_begin, n_kv, tbase, warp, lane, smem, qm, kv, B, col, use);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, kTmemCols);
  }
}

}  // namespace hier

using namespace hier;

namespace {

int attn_setup(const void* q, int64_t q_rows_total, int64_t q_stride, int32_t H, int32_t D,
               int32_t n_pairs, CUtensorMap* tmq) {
  if (D != kHD) {
    set_error(HIER_ENOTIMPL, "hier_attn_fwd supports head_dim=128 only; got head_dim=%d", D);
    return HIER_ENOTIMPL;
  }
  if (H <= 0 || n_pairs < 0) {
    set_error(HIER_EVALUE, "invalid heads=%d or query pairs=%d", H, n_pairs);
    return HIER_EVALUE;
  }
  if ((int64_t)n_pairs * H > INT32_MAX) {
    set_error(HIER_EVALUE, "too many work items");
    return HIER_EVALUE;
  }
  if (n_pairs == 0) return HIER_OK;
  return make_tmap_bf16_2d(tmq, q, (uint64_t)H * D, (uint64_t)q_rows_total, q_stride, 64, 128);
}

template <int kMaps>
int attn_launch(const QMaps& qm, int q2_row0, const KVMaps<kMaps>& kv, void* out,
                int64_t out_stride, const int32_t* out_rows, int32_t H, const int32_t* q_pairs,
                int32_t n_pairs, const int32_t* kv_tiles, const uint32_t* row_masks,
                int mask_rows, const int32_t* order, float softmax_scale, float* lse,
                const hier_partial_out* part, int32_t* dev_err, void* stream) {
  // The shared-memory limit is a per-device attribute of the function: set
  // it on every launch (a host call of about a microsecond), as the other
  // launchers do, so that a process driving several devices or host threads
  // needs no shared flag.
  HIER_CHECK_CUDA(cudaFuncSetAttribute(hier_attn_kernel<kMaps>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes),
                  "cudaFuncSetAttribute(hier_attn_kernel)");
  AttnArgs args;
  args.pairs = reinterpret_cast<const int4*>(q_pairs);
  args.kv_tiles = reinterpret_cast<const int4*>(kv_tiles);
  args.row_masks = reinterpret_cast<const uint4*>(row_masks);
  args.order = order;
  args.out = reinterpret_cast<__nv_bfloat16*>(out);
  args.out_stride = out_stride;
  args.out_rows = out_rows;
  args.part_out = part ? reinterpret_cast<__nv_bfloat16*>(part->o) : nullptr;
  args.part_stride = part ? part->o_stride : 0;
  args.part_lse = part ? part->lse : nullptr;
  args.part_row0 = part ? (int)part->row0 : 0;
  args.part_slot_rows = part ? part->slot_rows : 0;
  args.q2_row0 = q2_row0;
  args.n_pairs = n_pairs;
  args.mask_stride = mask_rows;
  args.mask_row_and = mask_rows - 1;
  args.scale_log2 = softmax_scale * 1.4426950408889634f;
  args.lse = lse;
  args.n_heads = H;
  args.err = dev_err;
  hier_attn_kernel<kMaps><<<n_pairs * H, 384, kSmemBytes, (cudaStream_t)stream>>>(qm, kv, args);
  HIER_CHECK_CUDA(cudaGetLastError(), "hier_attn_kernel launch");
  return HIER_OK;
}

}  // namespace

extern "C" int hier_attn_fwd(const void* q, int64_t q_rows_total, int64_t q_stride, const void* k,
                             const void* v, int64_t kv_rows_total, int64_t kv_stride, void* out,
                             int64_t out_stride, int32_t H, int32_t D, const int32_t* q_pairs,
                             int32_t n_pairs, const int32_t* kv_tiles, const uint32_t* row_masks,
                             const int32_t* order, float softmax_scale, int32_t* dev_err,
                             void* stream) {
  clear_error();
  QMaps qm;
  int rc = attn_setup(q, q_rows_total, q_stride, H, D, n_pairs, &qm.q[0]);
  if (rc || n_pairs == 0) return rc;
  qm.q[1] = qm.q[0];
  if (kv_rows_total > kRowMask) {
    set_error(HIER_EVALUE, "key/value pool of %lld rows exceeds %d", (long long)kv_rows_total,
              kRowMask);
    return HIER_EVALUE;
  }
  KVMaps<1> kv;
  rc = make_tmap_bf16_2d(&kv.k[0], k, (uint64_t)H * D, (uint64_t)kv_rows_total, kv_stride, 64, 64);
  if (!rc) rc = make_tmap_bf16_2d(&kv.v[0], v, (uint64_t)H * D, (uint64_t)kv_rows_total, kv_stride, 64, 64);
  if (rc) return rc;
  return attn_launch<1>(qm, INT_MAX, kv, out, out_stride, nullptr, H, q_pairs, n_pairs, kv_tiles,
                        row_masks, kBM, order, softmax_scale, nullptr, nullptr, dev_err, stream);
}

extern "C" int hier_attn_fwd_streams(const void* q, int64_t q_rows_total, int64_t q_stride,
                                     int32_t n_streams, const void* const* k, const void* const* v,
                                     const int64_t* stream_rows, const int64_t* kv_stride,
                                     void* out, int64_t out_stride, const int32_t* out_rows,
                                     int32_t H, int32_t D, const int32_t* q_pairs, int32_t n_pairs,
                                     const int32_t* kv_tiles, const uint32_t* tile_masks,
                                     int32_t mask_rows, const int32_t* order,
                                     float softmax_scale, float* lse,
                                     const hier_partial_out* part, int32_t* dev_err,
                                     void* stream) {
  clear_error();
  if (mask_rows != 1 && mask_rows != kBM) {
    set_error(HIER_EVALUE, "mask_rows must be 1 or %d; got %d", kBM, mask_rows);
    return HIER_EVALUE;
  }
  if (n_streams <= 0 || n_streams > HIER_MAX_KV_STREAMS || !k || !v || !stream_rows || !kv_stride) {
    set_error(HIER_EVALUE, "need 1..%d key/value streams; got %d", HIER_MAX_KV_STREAMS, n_streams);
    return HIER_EVALUE;
  }
  QMaps qm;
  int rc = attn_setup(q, q_rows_total, q_stride, H, D, n_pairs, &qm.q[0]);
  if (rc || n_pairs == 0) return rc;
  int q2_row0 = INT_MAX;
  qm.q[1] = qm.q[0];
  if (part && part->q2) {
    if (part->q2_row0 < 0 || part->q2_row0 > INT_MAX / 2 || part->q2_rows <= 0) {
      set_error(HIER_EVALUE, "invalid second query block (row0 %lld, %lld rows)",
                (long long)part->q2_row0, (long long)part->q2_rows);
      return HIER_EVALUE;
    }
    rc = make_tmap_bf16_2d(&qm.q[1], part->q2, (uint64_t)H * D, (uint64_t)part->q2_rows,
                           part->q2_stride, 64, 128);
    if (rc) return rc;
    q2_row0 = (int)part->q2_row0;
  }
  if (part && part->o && (part->row0 < 0 || part->row0 > INT_MAX / 2)) {
    set_error(HIER_EVALUE, "invalid partial-row offset %lld", (long long)part->row0);
    return HIER_EVALUE;
  }
  // Streams without rows are never addressed by a plan; their slots (and the
  // unused ones) repeat the first non-empty stream's maps.
  int first = -1;
  for (int s = 0; s < n_streams; ++s) {
    if (stream_rows[s] < 0 || stream_rows[s] > kRowMask) {
      set_error(HIER_EVALUE, "key/value stream %d has %lld rows; allowed 0..%d", s,
                (long long)stream_rows[s], kRowMask);
      return HIER_EVALUE;
    }
    if (first < 0 && stream_rows[s] > 0) first = s;
  }
  KVMaps<HIER_MAX_KV_STREAMS> kv;
  memset(&kv, 0, sizeof(kv));
  if (first >= 0) {
    for (int s = 0; s < n_streams; ++s) {
      if (stream_rows[s] == 0) continue;
      rc = make_tmap_bf16_2d(&kv.k[s], k[s], (uint64_t)H * D, (uint64_t)stream_rows[s],
                             kv_stride[s], 64, 64);
      if (!rc)
        rc = make_tmap_bf16_2d(&kv.v[s], v[s], (uint64_t)H * D, (uint64_t)stream_rows[s],
                               kv_stride[s], 64, 64);
      if (rc) return rc;
    }
    for (int s = 0; s < HIER_MAX_KV_STREAMS; ++s) {
      if (s < n_streams && stream_rows[s] > 0) continue;
      kv.k[s] = kv.k[first];
      kv.v[s] = kv.v[first];
    }
  }
  return attn_launch<HIER_MAX_KV_STREAMS>(qm, q2_row0, kv, out, out_stride, out_rows, H, q_pairs, n_pairs, kv_tiles,
                                          tile_masks, mask_rows, order, softmax_scale, lse,
                                          part, dev_err, stream);
}

// ---------------------------------------------------------------------------
// Merge of partial attention rows computed over disjoint key sets
// ---------------------------------------------------------------------------
//
// Target row t has partial rows rows[off[t] .. off[t+1]) (bf16 outputs o,
// each normalised over its own keys, and their log2-sum-exp lse); the merged
// row is sum_i 2^(lse_i - M) o_i / sum_i 2^(lse_i - M) with M the largest
// lse_i (0 without any key).  Across ranks the partial rows are either
// gathered to every rank first, or read in place from the owning rank's
// memory (symmetric buffers mapped over NVLink).

namespace hier {
namespace {

__device__ __forceinline__ void bf16x8_load(const __nv_bfloat16* p, float (&f)[8]) {
  const uint4 raw = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* p2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 v = __bfloat1622float2(p2[i]);
    f[2 * i] = v.x;
    f[2 * i + 1] = v.y;
  }
}

__device__ __forceinline__ void bf16x8_store(__nv_bfloat16* p, const float (&f)[8], float s) {
  uint4 v;
  v.x = pack_bf16x2(f[0] * s, f[1] * s);
  v.y = pack_bf16x2(f[2] * s, f[3] * s);
  v.z = pack_bf16x2(f[4] * s, f[5] * s);
  v.w = pack_bf16x2(f[6] * s, f[7] * s);
  *reinterpret_cast<uint4*>(p) = v;
}

// Where partial row pr lives: in one buffer, or (kPeers) in the buffer of
// its owner: rows below local_rows in this rank's, then one slot of
// slot_rows rows per rank, read in place from that rank's memory.
struct PartialSrc {
  const __nv_bfloat16* o;
  const float* lse;
  const __nv_bfloat16* const* o_bases;  // per rank (kPeers)
  const float* const* lse_bases;
  const int32_t* local_owner;  // rank of each partial row below local_rows (NULL: self)
  int self;
  int64_t local_rows, slot_rows;
};

template <bool kPeers>
__device__ __forceinline__ void partial_at(const PartialSrc& p, int64_t pr,
                                           const __nv_bfloat16** o, const float** lse) {
  if (!kPeers) {
    *o = p.o;
    *lse = p.lse;
    return;
  }
  const int owner = pr < p.local_rows ? (p.local_owner ? p.local_owner[pr] : p.self)
                                      : (int)((pr - p.local_rows) / p.slot_rows);
  *o = p.o_bases[owner];
  *lse = p.lse_bases[owner];
}

// Per (target, head, 8 channels): the normalised weighted sum of the partials.
template <bool kPeers>
__global__ void lse_gather_kernel(PartialSrc src, int64_t o_stride, int H, int D,
                                  const int32_t* off, const int32_t* rows, int64_t n_targets,
                                  __nv_bfloat16* out, int64_t out_stride,
                                  const int32_t* out_rows) {
  const int per = D / 8;
  const int64_t n = n_targets * H * per;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < n;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t rh = t / per;
    const int part = (int)(t % per);
    const int64_t r = rh / H;
    const int h = (int)(rh % H);
    const int b = off[r], e = off[r + 1];
    float m = -INFINITY;
    for (int i = b; i < e; ++i) {
      const __nv_bfloat16* o;
      const float* lse;
      partial_at<kPeers>(src, rows[i], &o, &lse);
      m = fmaxf(m, lse[(int64_t)rows[i] * H + h]);
    }
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    float ws = 0.f;
    for (int i = b; i < e; ++i) {
      const int64_t pr = rows[i];
      const __nv_bfloat16* o;
      const float* lse;
      partial_at<kPeers>(src, pr, &o, &lse);
      const float l = lse[pr * H + h];
      if (l == -INFINITY || m == -INFINITY) continue;
      const float wt = exp2f(l - m);
      float f[8];
      bf16x8_load(o + pr * o_stride + h * D + part * 8, f);
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] = fmaf(wt, f[q], acc[q]);
      ws += wt;
    }
    const int64_t dr = out_rows ? (int64_t)out_rows[r] : r;
    bf16x8_store(out + dr * out_stride + h * D + part * 8, acc, ws > 0.f ? 1.f / ws : 0.f);
  }
}

int merge_grid(int64_t n) {
  int64_t b = (n + 255) / 256;
  return (int)(b < 1 ? 1 : (b > 148 * 32 ? 148 * 32 : b));
}

int merge_check(int64_t rows, int H, int D, int64_t stride) {
  if (rows < 0 || H <= 0 || D <= 0 || D % 8 || stride % 8) {
    set_error(HIER_EVALUE, "invalid merge shape rows=%lld H=%d D=%d", (long long)rows, H, D);
    return HIER_EVALUE;
  }
  return HIER_OK;
}

}  // namespace
}  // namespace hier

extern "C" int hier_lse_gather_merge(const void* o, int64_t o_stride, const float* lse, int32_t H,
                                     int32_t D, const int32_t* off, const int32_t* rows,
                                     int64_t n_targets, void* out, int64_t out_stride,
                                     const int32_t* out_rows, void* stream) {
  clear_error();
  int rc = merge_check(n_targets, H, D, o_stride);
  if (!rc) rc = merge_check(n_targets, H, D, out_stride);
  if (rc || n_targets == 0) return rc;
  PartialSrc src{};
  src.o = reinterpret_cast<const __nv_bfloat16*>(o);
  src.lse = lse;
  lse_gather_kernel<false><<<merge_grid(n_targets * H * (D / 8)), 256, 0, (cudaStream_t)stream>>>(
      src, o_stride, H, D, off, rows, n_targets, reinterpret_cast<__nv_bfloat16*>(out),
      out_stride, out_rows);
  HIER_CHECK_CUDA(cudaGetLastError(), "lse_gather_kernel launch");
  return HIER_OK;
}

extern "C" int hier_lse_gather_merge_peers(const void* const* o_bases, const float* const* lse_bases,
                                           int32_t n_ranks, int32_t self, int64_t local_rows,
                                           int64_t slot_rows, int64_t o_stride, int32_t H,
                                           int32_t D, const int32_t* off, const int32_t* rows,
                                           int64_t n_targets, void* out, int64_t out_stride,
                                           const int32_t* out_rows, const int32_t* local_owner,
                                           void* stream) {
  clear_error();
  int rc = merge_check(n_targets, H, D, o_stride);
  if (!rc) rc = merge_check(n_targets, H, D, out_stride);
  if (rc || n_targets == 0) return rc;
  if (!o_bases || !lse_bases || n_ranks <= 0 || self < 0 || self >= n_ranks || local_rows < 0 ||
      slot_rows <= 0) {
    set_error(HIER_EVALUE, "invalid peer partial buffers (%d ranks, self %d, slot %lld)", n_ranks,
              self, (long long)slot_rows);
    return HIER_EVALUE;
  }
  PartialSrc src{};
  src.o_bases = reinterpret_cast<const __nv_bfloat16* const*>(o_bases);
  src.lse_bases = lse_bases;
  src.self = self;
  src.local_owner = local_owner;
  src.local_rows = local_rows;
  src.slot_rows = slot_rows;
  lse_gather_kernel<true><<<merge_grid(n_targets * H * (D / 8)), 256, 0, (cudaStream_t)stream>>>(
      src, o_stride, H, D, off, rows, n_targets, reinterpret_cast<__nv_bfloat16*>(out),
      out_stride, out_rows);
  HIER_CHECK_CUDA(cudaGetLastError(), "lse_gather_kernel launch");
  return HIER_OK;
}
