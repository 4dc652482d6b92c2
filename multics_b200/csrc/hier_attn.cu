// Block-sparse flash attention forward for sm_100a (tcgen05 + TMEM + TMA),
// the fused camera/RMSNorm/RoPE Q-K prologue, and a self-test of the
// tensor-core operand encodings.
//
// Attention kernel structure (one CTA per (query tile, head), 256 threads):
//   warp 0      TMA producer: Q tile once, then K and V tiles of the plan's
//               key-tile list into a 3-stage shared-memory ring.
//   warp 1      MMA issuer: S = Q K^T (SS form, both K-major, 128B swizzle)
//               into a double-buffered TMEM S tile, then O += P V with P read
//               from TMEM (TS form) and V as an MMN-major operand.
//   warps 4-7   softmax: one query row per thread; masks partial tiles with
//               the plan's per-row key bitmasks, online softmax with lazy
//               rescaling of O in TMEM, writes P (bf16) over its S tile,
//               epilogue O / l -> bf16 global.
// Every mbarrier wait is bounded (common.cuh: mbar_wait) and reports a
// timeout through dev_err instead of hanging.

#include <math.h>
#include <stdio.h>

#include "common.cuh"
#include "tmap.h"

namespace hier {

constexpr int kBM = 128;             // query rows per tile
constexpr int kBN = 128;             // keys per tile
constexpr int kHD = 128;             // head dim
constexpr int kStages = 3;           // K/V ring depth
constexpr int kTile = kBM * kHD * 2;  // 32 KiB
constexpr int kHalf = kTile / 2;      // one 64-column (128-byte) half
constexpr int kSmemQ = 0;
constexpr int kSmemK = kSmemQ + kTile;
constexpr int kSmemV = kSmemK + kStages * kTile;
constexpr int kSmemBar = kSmemV + kStages * kTile;
constexpr int kNumBars = 1 + 3 * kStages + 2 + 2 + 1;
constexpr int kSmemBytes = kSmemBar + 256 + 1024;  // + slack for 1024-byte alignment
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 256;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale O when the max grows by 2^8

struct AttnArgs {
  const int4* q_tiles;
  const int4* kv_tiles;
  const uint4* row_masks;
  const int* order;
  __nv_bfloat16* out;
  int64_t out_stride;
  int n_qt;
  int H;
  float scale_log2;
  int* err;
};

__global__ void __launch_bounds__(256, 1)
    hier_attn_kernel(const __grid_constant__ CUtensorMap tmq,
                     const __grid_constant__ CUtensorMap tmk,
                     const __grid_constant__ CUtensorMap tmv, AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kSmemBar);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* v_full = k_full + kStages;
  uint64_t* kv_empty = v_full + kStages;
  uint64_t* s_full = kv_empty + kStages;
  uint64_t* p_full = s_full + 2;
  uint64_t* o_done = p_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);

  const int warp = warp_id();
  const int lane = lane_id();
  const int head = blockIdx.x / a.n_qt;
  const int rank = blockIdx.x % a.n_qt;
  const int qt = a.order ? a.order[rank] : rank;
  const int4 qi = a.q_tiles[qt];  // (q_start, q_rows, kv_begin, kv_end)
  const int n_kv = qi.w - qi.z;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(k_full + s, 1);
      mbar_init(v_full + s, 1);
      mbar_init(kv_empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(s_full + b, 1);
      mbar_init(p_full + b, 128);
    }
    mbar_init(o_done, 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  if (n_kv > 0 && warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    prefetch_tmap(&tmq);
    prefetch_tmap(&tmk);
    prefetch_tmap(&tmv);
    const int col = head * kHD;
    mbar_arrive_expect_tx(q_full, kTile);
    tma_load_2d(smem + kSmemQ, &tmq, q_full, col, qi.x);
    tma_load_2d(smem + kSmemQ + kHalf, &tmq, q_full, col + 64, qi.x);
    for (int j = 0; j < n_kv; ++j) {
      const int st = j % kStages;
      if (j >= kStages && !mbar_wait(kv_empty + st, ((j / kStages) - 1) & 1, a.err, 1)) break;
      const int4 e = a.kv_tiles[qi.z + j];
      uint8_t* kd = smem + kSmemK + st * kTile;
      uint8_t* vd = smem + kSmemV + st * kTile;
      mbar_arrive_expect_tx(k_full + st, kTile);
      tma_load_2d(kd, &tmk, k_full + st, col, e.x);
      tma_load_2d(kd + kHalf / 2, &tmk, k_full + st, col, e.y);
      tma_load_2d(kd + kHalf, &tmk, k_full + st, col + 64, e.x);
      tma_load_2d(kd + kHalf + kHalf / 2, &tmk, k_full + st, col + 64, e.y);
      mbar_arrive_expect_tx(v_full + st, kTile);
      tma_load_2d(vd, &tmv, v_full + st, col, e.x);
      tma_load_2d(vd + kHalf / 2, &tmv, v_full + st, col, e.y);
      tma_load_2d(vd + kHalf, &tmv, v_full + st, col + 64, e.x);
      tma_load_2d(vd + kHalf + kHalf / 2, &tmv, v_full + st, col + 64, e.y);
    }
  } else if (n_kv > 0 && warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc_qk = idesc_bf16(kBM, kBN, false);
    constexpr uint32_t idesc_pv = idesc_bf16(kBM, kHD, true);
    const uint32_t qaddr = smem_u32(smem + kSmemQ);
    bool ok = mbar_wait(q_full, 0, a.err, 2);
    for (int j = 0; ok && j <= n_kv; ++j) {
      if (j < n_kv) {
        const int st = j % kStages, b = j & 1;
        if (!mbar_wait(k_full + st, (j / kStages) & 1, a.err, 3)) break;
        if (j >= 2 && !mbar_wait(o_done, (j - 2) & 1, a.err, 4)) break;
        tc_fence_after();
        const uint32_t kaddr = smem_u32(smem + kSmemK + st * kTile);
#pragma unroll
        for (int k = 0; k < kHD / 16; ++k) {
          const uint32_t off = (k >> 2) * kHalf + (k & 3) * 32;
          umma_ss(tbase + b * kBN, sdesc_sw128(qaddr + off, 16, 1024),
                  sdesc_sw128(kaddr + off, 16, 1024), idesc_qk, k > 0 ? 1u : 0u);
        }
        umma_commit(s_full + b);
      }
      if (j >= 1) {
        const int jj = j - 1, st = jj % kStages, b = jj & 1;
        if (!mbar_wait(p_full + b, (jj >> 1) & 1, a.err, 5)) break;
        if (!mbar_wait(v_full + st, (jj / kStages) & 1, a.err, 6)) break;
        tc_fence_after();
        const uint32_t vaddr = smem_u32(smem + kSmemV + st * kTile);
#pragma unroll
        for (int k = 0; k < kBN / 16; ++k) {
          umma_ts(tbase + kColO, tbase + b * kBN + k * 8,
                  sdesc_sw128(vaddr + k * 2048, kHalf, 1024), idesc_pv,
                  (jj > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(kv_empty + st);
        umma_commit(o_done);
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ softmax
    const int row = threadIdx.x - 128;
    const uint32_t lane_base = static_cast<uint32_t>(32 * (warp & 3)) << 16;
    const bool store_row = row < qi.y;
    __nv_bfloat16* orow = a.out + (int64_t)(qi.x + row) * a.out_stride + head * kHD;
    if (n_kv == 0) {
      if (store_row) {
        uint4 z = make_uint4(0, 0, 0, 0);
        for (int c = 0; c < kHD / 8; ++c) reinterpret_cast<uint4*>(orow)[c] = z;
      }
    } else {
      float m_run = -INFINITY, l_run = 0.f;
      bool ok = true;
      for (int j = 0; j < n_kv; ++j) {
        const int b = j & 1;
        const int4 e = a.kv_tiles[qi.z + j];
        uint4 mk = make_uint4(~0u, ~0u, ~0u, ~0u);
        if (e.z >= 0) mk = a.row_masks[(int64_t)e.z * kBM + row];
        if (e.w < kBN) {
          const int nc = e.w;
          mk.x &= nc >= 32 ? ~0u : ((1u << nc) - 1u);
          mk.y &= nc >= 64 ? ~0u : (nc <= 32 ? 0u : ((1u << (nc - 32)) - 1u));
          mk.z &= nc >= 96 ? ~0u : (nc <= 64 ? 0u : ((1u << (nc - 64)) - 1u));
          mk.w &= nc <= 96 ? 0u : ((1u << (nc - 96)) - 1u);
        }
        if (!mbar_wait(s_full + b, (j >> 1) & 1, a.err, 7)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float s[kBN];
        {
          uint32_t r[32];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            tmem_ld32(tbase + lane_base + b * kBN + c * 32, r);
            tmem_wait_ld();
            const uint32_t w = c == 0 ? mk.x : c == 1 ? mk.y : c == 2 ? mk.z : mk.w;
#pragma unroll
            for (int i = 0; i < 32; ++i)
              s[c * 32 + i] = ((w >> i) & 1u) ? __uint_as_float(r[i]) * a.scale_log2 : -INFINITY;
          }
        }
        float mx = -INFINITY;
#pragma unroll
        for (int c = 0; c < kBN; ++c) mx = fmaxf(mx, s[c]);
        const bool grow = mx > m_run + kRescaleThreshold;
        const bool rescale_o = grow && m_run != -INFINITY;
        if (__any_sync(0xffffffffu, rescale_o)) {
          // O holds P(<j) V: wait for PV(j-1), then scale this warp's rows.
          if (!mbar_wait(o_done, (j - 1) & 1, a.err, 8)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const float alpha = rescale_o ? ex2_approx(m_run - mx) : 1.f;
          uint32_t r[32];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            tmem_ld32(tbase + lane_base + kColO + c * 32, r);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
            tmem_st32(tbase + lane_base + kColO + c * 32, r);
          }
          tmem_wait_st();
          l_run *= alpha;
        }
        if (grow) m_run = mx;
        const float mref = m_run == -INFINITY ? 0.f : m_run;
        float rs = 0.f;
        uint32_t pk[kBN / 2];
#pragma unroll
        for (int c = 0; c < kBN / 2; ++c) {
          const float p0 = ex2_approx(s[2 * c] - mref);
          const float p1 = ex2_approx(s[2 * c + 1] - mref);
          rs += p0 + p1;
          pk[c] = pack_bf16x2(p0, p1);
        }
        l_run += rs;
        {
          uint32_t r[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = pk[i];
          tmem_st32(tbase + lane_base + b * kBN, r);
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = pk[32 + i];
          tmem_st32(tbase + lane_base + b * kBN + 32, r);
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(p_full + b);
      }
      if (ok && mbar_wait(o_done, (n_kv - 1) & 1, a.err, 9)) {
        tc_fence_after();
        const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
        uint32_t r[32];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          tmem_ld32(tbase + lane_base + kColO + c * 32, r);
          tmem_wait_ld();
          if (store_row) {
            uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              uint4 v;
              v.x = pack_bf16x2(__uint_as_float(r[8 * q + 0]) * inv, __uint_as_float(r[8 * q + 1]) * inv);
              v.y = pack_bf16x2(__uint_as_float(r[8 * q + 2]) * inv, __uint_as_float(r[8 * q + 3]) * inv);
              v.z = pack_bf16x2(__uint_as_float(r[8 * q + 4]) * inv, __uint_as_float(r[8 * q + 5]) * inv);
              v.w = pack_bf16x2(__uint_as_float(r[8 * q + 6]) * inv, __uint_as_float(r[8 * q + 7]) * inv);
              dst[q] = v;
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// fused camera + RMSNorm + RoPE prologue for Q and K
// ---------------------------------------------------------------------------

struct PrepArgs {
  const __nv_bfloat16* qx;
  const __nv_bfloat16* kx;
  int64_t x_stride;
  const __nv_bfloat16* cam;
  int cam_dim;
  const __nv_bfloat16* wcq;
  const __nv_bfloat16* wck;
  const __nv_bfloat16* nqw;
  const __nv_bfloat16* nkw;
  const float2* freqs;
  int64_t S;
  int dim;
  int D;
  float eps;
  __nv_bfloat16* q_out;
  __nv_bfloat16* k_out;
  int64_t out_stride;
};

constexpr int kMaxCam = 16;

__device__ __forceinline__ void bf16x8_to_f32(uint4 v, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

// One thread owns 8 consecutive channels of a token row (blockDim = dim/8);
// blockIdx.y selects Q (0) or K (1); blocks stride over tokens.  The camera
// weights of the thread's channels stay in registers for the whole kernel.
template <int CAM>
__global__ void __launch_bounds__(512) prep_qk_kernel(PrepArgs a) {
  __shared__ float red[32];
  __shared__ float camv[CAM > 0 ? CAM : 1];
  const bool is_k = blockIdx.y == 1;
  const __nv_bfloat16* x = is_k ? a.kx : a.qx;
  const __nv_bfloat16* wc = is_k ? a.wck : a.wcq;
  const __nv_bfloat16* nw = is_k ? a.nkw : a.nqw;
  __nv_bfloat16* out = is_k ? a.k_out : a.q_out;
  const int t = threadIdx.x;
  const int d0 = t * 8;
  const int nwarps = blockDim.x / 32;
  float wr[8][CAM > 0 ? CAM : 1];
  if (CAM > 0) {
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int c = 0; c < CAM; ++c) wr[i][c] = __bfloat162float(wc[(int64_t)(d0 + i) * CAM + c]);
  }
  float nv[8];
  bf16x8_to_f32(*reinterpret_cast<const uint4*>(nw + d0), nv);
  const int pair0 = (d0 % a.D) / 2;
  const int half = a.D / 2;
  for (int64_t row = blockIdx.x; row < a.S; row += gridDim.x) {
    float xv[8];
    bf16x8_to_f32(*reinterpret_cast<const uint4*>(x + row * a.x_stride + d0), xv);
    if (CAM > 0) {
      if (t < CAM) camv[t] = __bfloat162float(a.cam[row * CAM + t]);
      __syncthreads();
#pragma unroll
      for (int c = 0; c < CAM; ++c) {
        const float cv = camv[c];
#pragma unroll
        for (int i = 0; i < 8; ++i) xv[i] = fmaf(cv, wr[i][c], xv[i]);
      }
    }
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) ss = fmaf(xv[i], xv[i], ss);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((t & 31) == 0) red[t >> 5] = ss;
    __syncthreads();
    ss = 0.f;
    for (int w = 0; w < nwarps; ++w) ss += red[w];
    const float r = rsqrtf(ss / a.dim + a.eps);
    const float4* fr = reinterpret_cast<const float4*>(a.freqs + row * half + pair0);
    uint4 o;
    uint32_t* po = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 f2 = fr[i / 2];
      const float c = (i & 1) ? f2.z : f2.x;
      const float s = (i & 1) ? f2.w : f2.y;
      const float a0 = xv[2 * i] * r * nv[2 * i], a1 = xv[2 * i + 1] * r * nv[2 * i + 1];
      po[i] = pack_bf16x2(a0 * c - a1 * s, a0 * s + a1 * c);
    }
    *reinterpret_cast<uint4*>(out + row * a.out_stride + d0) = o;
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// tensor-core operand self-test
// ---------------------------------------------------------------------------

__global__ void __launch_bounds__(256, 1)
    selftest_umma_kernel(const __grid_constant__ CUtensorMap tma_a,
                         const __grid_constant__ CUtensorMap tma_bk,
                         const __grid_constant__ CUtensorMap tma_bm, const __nv_bfloat16* a,
                         float* c_ss, float* c_mn, float* c_ts, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sa = smem;
  uint8_t* sbk = smem + kTile;
  uint8_t* sbm = smem + 2 * kTile;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 3 * kTile);
  uint32_t* slot = reinterpret_cast<uint32_t*>(bars + 4);
  const int warp = warp_id(), lane = lane_id();
  if (threadIdx.x == 0) {
    mbar_init(bars + 0, 1);    // loads
    mbar_init(bars + 1, 1);    // mma done
    mbar_init(bars + 2, 128);  // A staged in TMEM
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tb = *slot;
  if (warp == 0 && lane == 0) {
    mbar_arrive_expect_tx(bars, 3 * kTile);
    tma_load_2d(sa, &tma_a, bars, 0, 0);
    tma_load_2d(sa + kHalf, &tma_a, bars, 64, 0);
    tma_load_2d(sbk, &tma_bk, bars, 0, 0);
    tma_load_2d(sbk + kHalf, &tma_bk, bars, 64, 0);
    // B as [K rows][N cols]: two 64-column halves of 128 rows each
    tma_load_2d(sbm, &tma_bm, bars, 0, 0);
    tma_load_2d(sbm + kHalf, &tma_bm, bars, 64, 0);
  } else if (warp == 1 && lane == 0) {
    if (mbar_wait(bars, 0, err, 20) && mbar_wait(bars + 2, 0, err, 21)) {
      tc_fence_after();
      const uint32_t aa = smem_u32(sa), bk = smem_u32(sbk), bm = smem_u32(sbm);
      for (int k = 0; k < 8; ++k) {
        const uint32_t off = (k >> 2) * kHalf + (k & 3) * 32;
        umma_ss(tb + 0, sdesc_sw128(aa + off, 16, 1024), sdesc_sw128(bk + off, 16, 1024),
                idesc_bf16(128, 128, false), k > 0);
      }
      for (int k = 0; k < 8; ++k) {
        const uint32_t off = (k >> 2) * kHalf + (k & 3) * 32;
        umma_ss(tb + 128, sdesc_sw128(aa + off, 16, 1024), sdesc_sw128(bm + k * 2048, kHalf, 1024),
                idesc_bf16(128, 128, true), k > 0);
      }
      for (int k = 0; k < 8; ++k) {
        umma_ts(tb + 384, tb + 256 + k * 8, sdesc_sw128(bm + k * 2048, kHalf, 1024),
                idesc_bf16(128, 128, true), k > 0);
      }
      umma_commit(bars + 1);
    }
  } else if (warp >= 4) {
    const int row = threadIdx.x - 128;
    const uint32_t lb = static_cast<uint32_t>(32 * (warp & 3)) << 16;
    // stage A row (bf16 pairs) into TMEM columns [256, 320)
    uint32_t r[32];
    const uint32_t* arow = reinterpret_cast<const uint32_t*>(a + row * 128);
    for (int c = 0; c < 2; ++c) {
      for (int i = 0; i < 32; ++i) r[i] = arow[c * 32 + i];
      tmem_st32(tb + lb + 256 + c * 32, r);
    }
    tmem_wait_st();
    tc_fence_before();
    mbar_arrive(bars + 2);
    if (mbar_wait(bars + 1, 0, err, 22)) {
      tc_fence_after();
      float* outs[3] = {c_ss, c_mn, c_ts};
      const uint32_t cols[3] = {0, 128, 384};
      for (int m = 0; m < 3; ++m)
        for (int c = 0; c < 4; ++c) {
          tmem_ld32(tb + lb + cols[m] + c * 32, r);
          tmem_wait_ld();
          for (int i = 0; i < 32; ++i) outs[m][row * 128 + c * 32 + i] = __uint_as_float(r[i]);
        }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tb, 512);
  }
}

}  // namespace hier

using namespace hier;

extern "C" int hier_attn_fwd(const void* q, int64_t q_rows_total, int64_t q_stride, const void* k,
                             const void* v, int64_t kv_rows_total, int64_t kv_stride, void* out,
                             int64_t out_stride, int32_t H, int32_t D, const int32_t* q_tiles,
                             int32_t n_q_tiles, const int32_t* kv_tiles,
                             const uint32_t* row_masks, const int32_t* order,
                             float softmax_scale, int32_t* dev_err, void* stream) {
  clear_error();
  if (D != kHD) {
    set_error(HIER_ENOTIMPL, "hier_attn_fwd supports head_dim=128 only; got head_dim=%d", D);
    return HIER_ENOTIMPL;
  }
  if (H <= 0 || n_q_tiles < 0) {
    set_error(HIER_EVALUE, "invalid heads=%d or query tiles=%d", H, n_q_tiles);
    return HIER_EVALUE;
  }
  if (n_q_tiles == 0) return HIER_OK;
  if ((int64_t)n_q_tiles * H > INT32_MAX) {
    set_error(HIER_EVALUE, "too many work items");
    return HIER_EVALUE;
  }
  CUtensorMap tmq, tmk, tmv;
  int rc = make_tmap_bf16_2d(&tmq, q, (uint64_t)H * D, (uint64_t)q_rows_total, q_stride, 64, 128);
  if (!rc) rc = make_tmap_bf16_2d(&tmk, k, (uint64_t)H * D, (uint64_t)kv_rows_total, kv_stride, 64, 64);
  if (!rc) rc = make_tmap_bf16_2d(&tmv, v, (uint64_t)H * D, (uint64_t)kv_rows_total, kv_stride, 64, 64);
  if (rc) return rc;
  static bool attr_set = false;
  if (!attr_set) {
    HIER_CHECK_CUDA(cudaFuncSetAttribute(hier_attn_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes),
                    "cudaFuncSetAttribute(hier_attn_kernel)");
    attr_set = true;
  }
  AttnArgs args;
  args.q_tiles = reinterpret_cast<const int4*>(q_tiles);
  args.kv_tiles = reinterpret_cast<const int4*>(kv_tiles);
  args.row_masks = reinterpret_cast<const uint4*>(row_masks);
  args.order = order;
  args.out = reinterpret_cast<__nv_bfloat16*>(out);
  args.out_stride = out_stride;
  args.n_qt = n_q_tiles;
  args.H = H;
  args.scale_log2 = softmax_scale * 1.4426950408889634f;
  args.err = dev_err;
  hier_attn_kernel<<<n_q_tiles * H, 256, kSmemBytes, (cudaStream_t)stream>>>(tmq, tmk, tmv, args);
  HIER_CHECK_CUDA(cudaGetLastError(), "hier_attn_kernel launch");
  return HIER_OK;
}

extern "C" int hier_prep_qk(const void* qx, const void* kx, int64_t x_stride, const void* cam,
                            int32_t cam_dim, const void* wcq, const void* wck, const void* nqw,
                            const void* nkw, const float* freqs, int64_t S, int32_t H, int32_t D,
                            float eps, void* q_out, void* k_out, int64_t out_stride,
                            void* stream) {
  clear_error();
  const int dim = H * D;
  if (dim % 8 != 0 || dim / 8 > 512 || dim / 8 < 32 || (dim / 8) % 32 != 0 || D % 8 != 0) {
    set_error(HIER_ENOTIMPL, "hier_prep_qk needs dim = H*D with dim/8 a multiple of 32 and <= 512; got dim=%d", dim);
    return HIER_ENOTIMPL;
  }
  if (cam && (cam_dim <= 0 || cam_dim > kMaxCam || !wcq || !wck)) {
    set_error(HIER_EVALUE, "camera tokens need 1..%d channels and both cam_q/cam_k weights", kMaxCam);
    return HIER_EVALUE;
  }
  if (S == 0) return HIER_OK;
  PrepArgs p;
  p.qx = (const __nv_bfloat16*)qx;
  p.kx = (const __nv_bfloat16*)kx;
  p.x_stride = x_stride;
  p.cam = (const __nv_bfloat16*)cam;
  p.cam_dim = cam_dim;
  p.wcq = (const __nv_bfloat16*)wcq;
  p.wck = (const __nv_bfloat16*)wck;
  p.nqw = (const __nv_bfloat16*)nqw;
  p.nkw = (const __nv_bfloat16*)nkw;
  p.freqs = (const float2*)freqs;
  p.S = S;
  p.dim = dim;
  p.D = D;
  p.eps = eps;
  p.q_out = (__nv_bfloat16*)q_out;
  p.k_out = (__nv_bfloat16*)k_out;
  p.out_stride = out_stride;
  const int threads = dim / 8;
  const int64_t blocks = S < 148 * 6 ? S : 148 * 6;
  const dim3 grid((unsigned)blocks, 2);
  cudaStream_t st = (cudaStream_t)stream;
  if (!cam)
    prep_qk_kernel<0><<<grid, threads, 0, st>>>(p);
  else if (cam_dim == 12)
    prep_qk_kernel<12><<<grid, threads, 0, st>>>(p);
  else if (cam_dim == 16)
    prep_qk_kernel<16><<<grid, threads, 0, st>>>(p);
  else {
    set_error(HIER_ENOTIMPL, "hier_prep_qk supports cam_dim 12 or 16; got %d", cam_dim);
    return HIER_ENOTIMPL;
  }
  HIER_CHECK_CUDA(cudaGetLastError(), "prep_qk_kernel launch");
  return HIER_OK;
}

extern "C" int hier_selftest_umma(const void* a, const void* b, float* c_ss, float* c_mn,
                                  float* c_ts, int32_t* dev_err, void* stream) {
  clear_error();
  CUtensorMap ta, tbk, tbm;
  int rc = make_tmap_bf16_2d(&ta, a, 128, 128, 128, 64, 128);
  if (!rc) rc = make_tmap_bf16_2d(&tbk, b, 128, 128, 128, 64, 128);
  if (!rc) rc = make_tmap_bf16_2d(&tbm, b, 128, 128, 128, 64, 128);
  if (rc) return rc;
  const int smem = 3 * kTile + 256 + 1024;
  HIER_CHECK_CUDA(cudaFuncSetAttribute(selftest_umma_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                  "cudaFuncSetAttribute(selftest)");
  selftest_umma_kernel<<<1, 256, smem, (cudaStream_t)stream>>>(
      ta, tbk, tbm, (const __nv_bfloat16*)a, c_ss, c_mn, c_ts, dev_err);
  HIER_CHECK_CUDA(cudaGetLastError(), "selftest_umma_kernel launch");
  return HIER_OK;
}
