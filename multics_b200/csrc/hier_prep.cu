// Fused camera + RMSNorm + RoPE prologue for Q and K (sm_100a).
//
// q = RoPE(RMSNorm(qx + cam @ Wq^T) * wq) and the same for k, in fp32 with one
// bf16 rounding at the end; the post-projection part of the reference's
// SelfAttention._project_self_attn_qkv (multics/models/attention.py:355-365,
// camera add :307-320, RMSNorm :231-242, rope_apply multics/models/rope.py:248-254).
// Memory-bound: each token row of q and k is read and written once.

#include <math.h>
#include <stdio.h>

#include "common.cuh"

namespace hier {

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
  int64_t freqs_rows;  // token r uses table row r % freqs_rows
  int64_t S;
  int dim;
  int D;
  float eps;
  __nv_bfloat16* q_out;
  __nv_bfloat16* k_out;
  int64_t out_stride;
  const int32_t* out_rows;    // output row of each input row (NULL: the same row)
  const int32_t* k_out_rows;  // the same for k (NULL: out_rows)
};

constexpr int kMaxCam = 16;

// Camera weights W [dim][CAM] (bf16, row-major) into shared memory
// transposed, wt[c * dim + d]: one thread per channel d reads its CAM
// contiguous weights (8-byte loads when aligned) and writes them to CAM rows,
// consecutive threads to consecutive channels (no bank conflicts); the loop is
// unrolled so that a thread's loads are in flight together.
template <int CAM>
__device__ __forceinline__ void load_cam_weights_t(__nv_bfloat16* wt, const __nv_bfloat16* wc,
                                                   int dim) {
  if (CAM == 0) return;
  const bool vec = CAM % 4 == 0 && (reinterpret_cast<uintptr_t>(wc) & 7) == 0;
#pragma unroll 2
  for (int d = threadIdx.x; d < dim; d += blockDim.x) {
    __nv_bfloat16 w[CAM > 0 ? CAM : 1];
    if (vec) {
      const uint2* src = reinterpret_cast<const uint2*>(wc + (int64_t)d * CAM);
#pragma unroll
      for (int j = 0; j < CAM / 4; ++j) {
        const uint2 v = src[j];
        memcpy(&w[4 * j], &v, sizeof(v));
      }
    } else {
#pragma unroll
      for (int c = 0; c < CAM; ++c) w[c] = wc[(int64_t)d * CAM + c];
    }
#pragma unroll
    for (int c = 0; c < CAM; ++c) wt[c * dim + d] = w[c];
  }
}

// x rounded to the nearest bf16 (the value the forward keeps for y = x + proj)
__device__ __forceinline__ float round_bf16(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

// two bf16 channels (low half first) as an fp32x2 pair
__device__ __forceinline__ uint64_t bf16x2_to_f2(uint32_t v) {
  return f2_pack(__uint_as_float(v << 16), __uint_as_float(v & 0xffff0000u));
}

// eight bf16 channels added pairwise, each sum rounded to bf16 once
__device__ __forceinline__ uint4 bf16x8_add(uint4 a, uint4 b) {
  uint4 r;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(r.x) : "r"(a.x), "r"(b.x));
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(r.y) : "r"(a.y), "r"(b.y));
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(r.z) : "r"(a.z), "r"(b.z));
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(r.w) : "r"(a.w), "r"(b.w));
  return r;
}

__device__ __forceinline__ void bf16x8_to_f32(uint4 v, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

// One warp per token row.  Lane l owns the 8-channel chunks starting at
// channels 8l + 256i (i = 0..dim/256-1): every load and store of a row is
// one coalesced 512-byte access per chunk, the row's sum of squares is a
// warp reduction (no block barrier), and the RoPE pairs of a lane are the
// same for all its chunks (channel offsets 256i are whole heads apart), so
// a lane reads 4 (cos, sin) pairs per row.  A warp walks a contiguous run of
// rows with the next row's channels loaded while it computes the current one
// (8 warps per CTA leave the registers for both rows); the camera projection
// W cam_r of its channels (camera weights transposed into shared memory, fp32
// sums, kept as bf16 in the warp's slice of shared memory) is recomputed only
// when the camera row changes: the rows of a player frame share one camera
// row and hub rows have none.  Per channel pair: one bf16x2 add of the
// projection (y, rounded to bf16 as the reference's add), one fp32x2 FMA for
// the sum of squares, one fp32x2 multiply by the norm weight, and the rotation
// with rstd folded into the row's (cos, sin) pairs.
constexpr int kPrepWarps = 8;
constexpr int kPrepMaxChunks = 12;  // dim <= 256 * 12 = 3072

// chunk i of a lane exists (a row of dim = 256k + 128 leaves the upper half of
// the lanes without a last chunk)
__device__ __forceinline__ bool chunk_ok(int dim, int lane, int i) { return 8 * lane + 256 * i < dim; }

template <int CAM, int NCH>
__global__ void __launch_bounds__(kPrepWarps * 32, 1) prep_qk_kernel(PrepArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  // [CAM][dim] bf16 transposed camera weights, [dim] bf16 norm weights, then
  // per warp its projection [NCH][32 lanes][8 channels] bf16
  __nv_bfloat16* wt = reinterpret_cast<__nv_bfloat16*>(smem);
  __nv_bfloat16* nws = wt + CAM * a.dim;
  uint4* proj = reinterpret_cast<uint4*>(nws + a.dim) + (threadIdx.x >> 5) * (NCH * 32);
  const bool is_k = blockIdx.y == 1;
  const __nv_bfloat16* x = is_k ? a.kx : a.qx;
  const __nv_bfloat16* wc = is_k ? a.wck : a.wcq;
  const __nv_bfloat16* nw = is_k ? a.nkw : a.nqw;
  __nv_bfloat16* out = is_k ? a.k_out : a.q_out;
  load_cam_weights_t<CAM>(wt, wc, a.dim);
  for (int e = threadIdx.x; e < a.dim / 8; e += blockDim.x)
    reinterpret_cast<uint4*>(nws)[e] = reinterpret_cast<const uint4*>(nw)[e];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * kPrepWarps + (threadIdx.x >> 5);
  const int64_t nw_total = (int64_t)gridDim.x * kPrepWarps;
  const int64_t per = (a.S + nw_total - 1) / nw_total;
  const int64_t r_begin = gw * per, r_end = min(a.S, r_begin + per);
  const int half = a.D / 2;
  const int pair0 = (8 * lane % a.D) / 2;  // first RoPE pair of every chunk of this lane
  float cam_prev = 0.f;  // lane c < CAM: camera value c of the projected row
  bool have_proj = false;
  const float inv_dim = 1.f / (float)a.dim;
  // the camera value and the output row of a token are loaded one row ahead:
  // the camera value decides whether the projection is recomputed and the
  // output row addresses the stores, so neither load waits on its own row
  const int32_t* rows_map = (is_k && a.k_out_rows) ? a.k_out_rows : a.out_rows;
  float cv_next = 0.f;
  int64_t dst_next = r_begin;
  if (r_begin < r_end) {
    if (CAM > 0 && lane < CAM) cv_next = __bfloat162float(a.cam[r_begin * CAM + lane]);
    if (rows_map) dst_next = rows_map[r_begin];
  }
  uint4 xn[NCH];
  if (r_begin < r_end) {
    const __nv_bfloat16* xr = x + r_begin * a.x_stride;
#pragma unroll
    for (int i = 0; i < NCH; ++i)
      xn[i] = chunk_ok(a.dim, lane, i) ? *reinterpret_cast<const uint4*>(xr + 8 * lane + 256 * i)
                                       : make_uint4(0u, 0u, 0u, 0u);
  }
  for (int64_t r = r_begin; r < r_end; ++r) {
    uint4 xv[NCH];
#pragma unroll
    for (int i = 0; i < NCH; ++i) xv[i] = xn[i];
    if (r + 1 < r_end) {
      const __nv_bfloat16* xr = x + (r + 1) * a.x_stride;
#pragma unroll
      for (int i = 0; i < NCH; ++i)
        xn[i] = chunk_ok(a.dim, lane, i) ? *reinterpret_cast<const uint4*>(xr + 8 * lane + 256 * i)
                                         : make_uint4(0u, 0u, 0u, 0u);
    }
    const int64_t rf = a.freqs_rows == a.S ? r : r % a.freqs_rows;
    const float4* fr = reinterpret_cast<const float4*>(a.freqs + rf * half + pair0);
    const float4 f0 = fr[0], f1 = fr[1];
    const float cv = cv_next;
    const int64_t dst = dst_next;
    if (r + 1 < r_end) {
      if (CAM > 0 && lane < CAM) cv_next = __bfloat162float(a.cam[(r + 1) * CAM + lane]);
      dst_next = rows_map ? (int64_t)rows_map[r + 1] : r + 1;
    }
    if (CAM > 0) {
      const bool same = __all_sync(0xffffffffu, cv == cam_prev);
      if (!(same && have_proj)) {
        const bool zero = __all_sync(0xffffffffu, cv == 0.f);
        const bool ok_last = chunk_ok(a.dim, lane, NCH - 1);
#pragma unroll
        for (int i = 0; i < NCH; ++i) {
          float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
          if (!zero) {
#pragma unroll
            for (int c = 0; c < CAM; ++c) {
              // every lane takes part in the shuffle, lanes without a last chunk too
              const float cc = __shfl_sync(0xffffffffu, cv, c);
              if (i + 1 < NCH || ok_last) {
                float w[8];
                bf16x8_to_f32(*reinterpret_cast<const uint4*>(wt + c * a.dim + 8 * lane + 256 * i), w);
#pragma unroll
                for (int q = 0; q < 8; ++q) acc[q] = fmaf(cc, w[q], acc[q]);
              }
            }
          }
          proj[i * 32 + lane] = make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]),
                                           pack_bf16x2(acc[4], acc[5]), pack_bf16x2(acc[6], acc[7]));
        }
        cam_prev = cv;
        have_proj = true;
      }
    }
    // pass 1: y = x + proj rounded to bf16 (the reference adds the camera
    // projection in bf16, attention.py:320) kept in place of x, and the row's
    // sum of squares of y, two channels per fp32x2 FMA
    uint64_t ss2 = f2_pack(0.f, 0.f);
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
      if (CAM > 0) xv[i] = bf16x8_add(xv[i], proj[i * 32 + lane]);
      const uint32_t* yw = reinterpret_cast<const uint32_t*>(&xv[i]);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint64_t v = bf16x2_to_f2(yw[q]);
        ss2 = f2_fma(v, v, ss2);
      }
    }
    float ss_lo, ss_hi;
    f2_unpack(ss2, ss_lo, ss_hi);
    float ss = ss_lo + ss_hi;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float rs = rsqrtf(ss * inv_dim + a.eps);
    // pass 2: (y * w) rotated, with rstd folded into the row's (cos, sin)
    // pairs (RoPE is linear), one bf16 rounding
    float rc[4], rsn[4];
    rc[0] = f0.x * rs, rsn[0] = f0.y * rs, rc[1] = f0.z * rs, rsn[1] = f0.w * rs;
    rc[2] = f1.x * rs, rsn[2] = f1.y * rs, rc[3] = f1.z * rs, rsn[3] = f1.w * rs;
    __nv_bfloat16* orow = out + dst * a.out_stride;
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
      const uint4 wv = chunk_ok(a.dim, lane, i)
                           ? *reinterpret_cast<const uint4*>(nws + 8 * lane + 256 * i)
                           : make_uint4(0u, 0u, 0u, 0u);
      const uint32_t* yw = reinterpret_cast<const uint32_t*>(&xv[i]);
      const uint32_t* ww = reinterpret_cast<const uint32_t*>(&wv);
      uint4 o;
      uint32_t* po = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float a0, a1;
        f2_unpack(f2_mul(bf16x2_to_f2(yw[q]), bf16x2_to_f2(ww[q])), a0, a1);
        po[q] = pack_bf16x2(fmaf(a0, rc[q], -a1 * rsn[q]), fmaf(a0, rsn[q], a1 * rc[q]));
      }
      if (chunk_ok(a.dim, lane, i)) *reinterpret_cast<uint4*>(orow + 8 * lane + 256 * i) = o;
    }
  }
}

template <int CAM>
int prep_launch(const PrepArgs& p, int sms, cudaStream_t st) {
  const int nch = (p.dim + 255) / 256;
  // weights and norm, then per warp NCH chunks x 32 lanes x 16 bytes of projection
  const size_t smem = (size_t)(CAM + 1) * p.dim * 2 + (CAM > 0 ? (size_t)kPrepWarps * nch * 512 : 0);
  const int64_t warps = (p.S + 3) / 4;  // at least 4 rows per warp
  int64_t blocks = (warps + kPrepWarps - 1) / kPrepWarps;
  if (blocks > (sms + 1) / 2) blocks = (sms + 1) / 2;  // with Q and K: one CTA per SM
  const dim3 grid((unsigned)blocks, 2);
  switch (nch) {
#define HIER_PREP_CASE(n)                                                                     \
  case n:                                                                                     \
    HIER_CHECK_CUDA(cudaFuncSetAttribute(prep_qk_kernel<CAM, n>,                              \
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,         \
                                         (int)smem),                                          \
                    "cudaFuncSetAttribute(prep_qk_kernel)");                                  \
    prep_qk_kernel<CAM, n><<<grid, kPrepWarps * 32, smem, st>>>(p);                           \
    break;
    HIER_PREP_CASE(1)
    HIER_PREP_CASE(2)
    HIER_PREP_CASE(3)
    HIER_PREP_CASE(4)
    HIER_PREP_CASE(5)
    HIER_PREP_CASE(6)
    HIER_PREP_CASE(7)
    HIER_PREP_CASE(8)
    HIER_PREP_CASE(9)
    HIER_PREP_CASE(10)
    HIER_PREP_CASE(11)
    HIER_PREP_CASE(12)
#undef HIER_PREP_CASE
    default:
      set_error(HIER_ENOTIMPL, "hier_prep_qk supports dim = 128..3072 in steps of 128; got %d",
                p.dim);
      return HIER_ENOTIMPL;
  }
  HIER_CHECK_CUDA(cudaGetLastError(), "prep_qk_kernel launch");
  return HIER_OK;
}

// ---------------------------------------------------------------------------
// Backward of the prologue (training)
// ---------------------------------------------------------------------------
//
// For q = RoPE(RMSNorm(y) * w) with y = x + cam @ Wc^T, given the gradient g
// of q: the rotation is undone (g_n = R^T g), and with yh = y * rstd,
//   dx = rstd * (g_n * w - yh * mean(g_n * w * yh)),   dw = sum_rows g_n * yh.
// One warp per row as in the forward (a lane holds 8-element chunks of the
// row); dw is accumulated per warp in registers and written as one partial
// row per warp (summed by the caller: deterministic).  The camera adapter's
// gradient dx^T @ cam is a plain GEMM left to the caller.

struct PrepBwdArgs {
  PrepArgs f;  // the forward's inputs (x, camera, weights, table, sizes)
  const __nv_bfloat16* gq;
  const __nv_bfloat16* gk;
  int64_t g_stride;
  __nv_bfloat16* dqx;
  __nv_bfloat16* dkx;
  int64_t dx_stride;
  float* dw_part;  // [2][warps][dim]
};

constexpr int kPrepBwdWarps = 8;

template <int CAM, int NCH>
__global__ void __launch_bounds__(kPrepBwdWarps * 32, 1) prep_qk_bwd_kernel(PrepBwdArgs b) {
  const PrepArgs& a = b.f;
  extern __shared__ __align__(16) uint8_t smem[];
  __nv_bfloat16* wt = reinterpret_cast<__nv_bfloat16*>(smem);
  __nv_bfloat16* nws = wt + CAM * a.dim;
  uint4* proj = reinterpret_cast<uint4*>(nws + a.dim) + (threadIdx.x >> 5) * (NCH * 32);
  const bool is_k = blockIdx.y == 1;
  const __nv_bfloat16* x = is_k ? a.kx : a.qx;
  const __nv_bfloat16* wc = is_k ? a.wck : a.wcq;
  const __nv_bfloat16* nw = is_k ? a.nkw : a.nqw;
  const __nv_bfloat16* g = is_k ? b.gk : b.gq;
  __nv_bfloat16* dx = is_k ? b.dkx : b.dqx;
  load_cam_weights_t<CAM>(wt, wc, a.dim);
  for (int e = threadIdx.x; e < a.dim / 8; e += blockDim.x)
    reinterpret_cast<uint4*>(nws)[e] = reinterpret_cast<const uint4*>(nw)[e];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * kPrepBwdWarps + (threadIdx.x >> 5);
  const int64_t nw_total = (int64_t)gridDim.x * kPrepBwdWarps;
  const int64_t per = (a.S + nw_total - 1) / nw_total;
  const int64_t r_begin = gw * per, r_end = min(a.S, r_begin + per);
  const int half = a.D / 2;
  const int pair0 = (8 * lane % a.D) / 2;
  float cam_prev = 0.f;
  bool have_proj = false;
  const float inv_dim = 1.f / (float)a.dim;
  float accw[NCH][8];
#pragma unroll
  for (int i = 0; i < NCH; ++i)
#pragma unroll
    for (int q = 0; q < 8; ++q) accw[i][q] = 0.f;
  for (int64_t r = r_begin; r < r_end; ++r) {
    const __nv_bfloat16* xr = x + r * a.x_stride;
    const __nv_bfloat16* gr = g + r * b.g_stride;
    // chunk i of the row (x, the gradient, the norm weight): read from global
    // memory / shared memory in each pass (the row stays in L1 between them)
    auto ld = [&](const __nv_bfloat16* base, int i, float (&f)[8]) {
      bf16x8_to_f32(chunk_ok(a.dim, lane, i)
                        ? *reinterpret_cast<const uint4*>(base + 8 * lane + 256 * i)
                        : make_uint4(0u, 0u, 0u, 0u), f);
    };
    const int64_t rf = a.freqs_rows == a.S ? r : r % a.freqs_rows;
    const float4* fr = reinterpret_cast<const float4*>(a.freqs + rf * half + pair0);
    const float4 f0 = fr[0], f1 = fr[1];
    if (CAM > 0) {
      const float cv = lane < CAM ? __bfloat162float(a.cam[r * CAM + lane]) : 0.f;
      const bool same = __all_sync(0xffffffffu, cv == cam_prev);
      if (!(same && have_proj)) {
        const bool zero = __all_sync(0xffffffffu, cv == 0.f);
        const bool ok_last = chunk_ok(a.dim, lane, NCH - 1);
#pragma unroll
        for (int i = 0; i < NCH; ++i) {
          float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
          if (!zero) {
#pragma unroll
            for (int c = 0; c < CAM; ++c) {
              const float cc = __shfl_sync(0xffffffffu, cv, c);
              if (i + 1 < NCH || ok_last) {
                float w[8];
                bf16x8_to_f32(*reinterpret_cast<const uint4*>(wt + c * a.dim + 8 * lane + 256 * i), w);
#pragma unroll
                for (int q = 0; q < 8; ++q) acc[q] = fmaf(cc, w[q], acc[q]);
              }
            }
          }
          proj[i * 32 + lane] = make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]),
                                           pack_bf16x2(acc[4], acc[5]), pack_bf16x2(acc[6], acc[7]));
        }
        cam_prev = cv;
        have_proj = true;
      }
    }
    // y = x + projection, rounded to bf16 as in the forward; its sum of squares
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
      float xf[8], pf[8];
      ld(xr, i, xf);
      if (CAM > 0) {
        bf16x8_to_f32(proj[i * 32 + lane], pf);
#pragma unroll
        for (int q = 0; q < 8; ++q) xf[q] = round_bf16(xf[q] + pf[q]);
      }
#pragma unroll
      for (int q = 0; q < 8; ++q) ss = fmaf(xf[q], xf[q], ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float rs = rsqrtf(ss * inv_dim + a.eps);
    // g_n = R^T g; mean(g_n * w * yh); dw partial
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
      float xf[8], pf[8], wf[8], gf[8];
      ld(xr, i, xf);
      if (CAM > 0) {
        bf16x8_to_f32(proj[i * 32 + lane], pf);
#pragma unroll
        for (int q = 0; q < 8; ++q) xf[q] = round_bf16(xf[q] + pf[q]);
      }
      ld(gr, i, gf);
      ld(nws, i, wf);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 f = q < 2 ? f0 : f1;
        const float c = (q & 1) ? f.z : f.x;
        const float s = (q & 1) ? f.w : f.y;
        const float g0 = gf[2 * q], g1 = gf[2 * q + 1];
        const float n0 = g0 * c + g1 * s, n1 = g1 * c - g0 * s;
        const float y0 = xf[2 * q] * rs, y1 = xf[2 * q + 1] * rs;
        accw[i][2 * q] = fmaf(n0, y0, accw[i][2 * q]);
        accw[i][2 * q + 1] = fmaf(n1, y1, accw[i][2 * q + 1]);
        dot = fmaf(n0 * wf[2 * q], y0, dot);
        dot = fmaf(n1 * wf[2 * q + 1], y1, dot);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    dot *= inv_dim;
    __nv_bfloat16* dr = dx + r * b.dx_stride;
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
      float xf[8], pf[8], wf[8], gf[8];
      ld(xr, i, xf);
      if (CAM > 0) {
        bf16x8_to_f32(proj[i * 32 + lane], pf);
#pragma unroll
        for (int q = 0; q < 8; ++q) xf[q] = round_bf16(xf[q] + pf[q]);
      }
      ld(gr, i, gf);
      ld(nws, i, wf);
      uint4 o;
      uint32_t* po = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 f = q < 2 ? f0 : f1;
        const float c = (q & 1) ? f.z : f.x;
        const float s = (q & 1) ? f.w : f.y;
        const float g0 = gf[2 * q], g1 = gf[2 * q + 1];
        const float n0 = g0 * c + g1 * s, n1 = g1 * c - g0 * s;
        const float y0 = xf[2 * q] * rs, y1 = xf[2 * q + 1] * rs;
        po[q] = pack_bf16x2(rs * (n0 * wf[2 * q] - y0 * dot), rs * (n1 * wf[2 * q + 1] - y1 * dot));
      }
      if (chunk_ok(a.dim, lane, i)) *reinterpret_cast<uint4*>(dr + 8 * lane + 256 * i) = o;
    }
  }
  float* part = b.dw_part + ((int64_t)(is_k ? nw_total : 0) + gw) * a.dim;
#pragma unroll
  for (int i = 0; i < NCH; ++i) {
    if (!chunk_ok(a.dim, lane, i)) continue;
    float4* d = reinterpret_cast<float4*>(part + 8 * lane + 256 * i);
    d[0] = make_float4(accw[i][0], accw[i][1], accw[i][2], accw[i][3]);
    d[1] = make_float4(accw[i][4], accw[i][5], accw[i][6], accw[i][7]);
  }
}

// CTAs of the backward launch (the partial rows of dw are 8 per CTA).
int prep_bwd_blocks(int64_t S, int sms) {
  const int64_t warps = (S + 3) / 4;
  int64_t blocks = (warps + kPrepBwdWarps - 1) / kPrepBwdWarps;
  if (blocks > (sms + 1) / 2) blocks = (sms + 1) / 2;
  return (int)(blocks > 0 ? blocks : 1);
}

template <int CAM>
int prep_bwd_launch(const PrepBwdArgs& p, int blocks, cudaStream_t st) {
  const int nch = (p.f.dim + 255) / 256;
  const size_t smem =
      (size_t)(CAM + 1) * p.f.dim * 2 + (CAM > 0 ? (size_t)kPrepBwdWarps * nch * 512 : 0);
  const dim3 grid((unsigned)blocks, 2);
  switch (nch) {
#define HIER_PREP_BWD_CASE(n)                                                                 \
  case n:                                                                                     \
    HIER_CHECK_CUDA(cudaFuncSetAttribute(prep_qk_bwd_kernel<CAM, n>,                          \
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,         \
                                         (int)smem),                                          \
                    "cudaFuncSetAttribute(prep_qk_bwd_kernel)");                              \
    prep_qk_bwd_kernel<CAM, n><<<grid, kPrepBwdWarps * 32, smem, st>>>(p);                    \
    break;
    HIER_PREP_BWD_CASE(1)
    HIER_PREP_BWD_CASE(2)
    HIER_PREP_BWD_CASE(3)
    HIER_PREP_BWD_CASE(4)
    HIER_PREP_BWD_CASE(5)
    HIER_PREP_BWD_CASE(6)
    HIER_PREP_BWD_CASE(7)
    HIER_PREP_BWD_CASE(8)
    HIER_PREP_BWD_CASE(9)
    HIER_PREP_BWD_CASE(10)
    HIER_PREP_BWD_CASE(11)
    HIER_PREP_BWD_CASE(12)
#undef HIER_PREP_BWD_CASE
    default:
      set_error(HIER_ENOTIMPL, "hier_prep_qk_bwd supports dim = 128..3072 in steps of 128; got %d",
                p.f.dim);
      return HIER_ENOTIMPL;
  }
  HIER_CHECK_CUDA(cudaGetLastError(), "prep_qk_bwd_kernel launch");
  return HIER_OK;
}

}  // namespace hier

using namespace hier;

extern "C" int hier_prep_qk(const void* qx, const void* kx, int64_t x_stride, const void* cam,
                            int32_t cam_dim, const void* wcq, const void* wck, const void* nqw,
                            const void* nkw, const float* freqs, int64_t freqs_rows, int64_t S,
                            int32_t H, int32_t D,
                            float eps, void* q_out, void* k_out, int64_t out_stride,
                            const int32_t* out_rows, const int32_t* k_out_rows, void* stream) {
  clear_error();
  const int dim = H * D;
  if (dim % 128 != 0 || dim > 256 * kPrepMaxChunks || D <= 0 || D % 8 != 0 || 256 % D != 0) {
    set_error(HIER_ENOTIMPL,
              "hier_prep_qk needs dim = H*D a multiple of 128 up to %d and head_dim dividing 256; "
              "got dim=%d head_dim=%d", 256 * kPrepMaxChunks, dim, D);
    return HIER_ENOTIMPL;
  }
  if (cam && (cam_dim <= 0 || cam_dim > kMaxCam || !wcq || !wck)) {
    set_error(HIER_EVALUE, "camera tokens need 1..%d channels and both cam_q/cam_k weights", kMaxCam);
    return HIER_EVALUE;
  }
  if (S == 0) return HIER_OK;
  if (freqs_rows <= 0 || freqs_rows > S) {
    set_error(HIER_EVALUE, "hier_prep_qk: freqs_rows=%lld must be in [1, S=%lld]",
              (long long)freqs_rows, (long long)S);
    return HIER_EVALUE;
  }
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
  p.freqs_rows = freqs_rows;
  p.S = S;
  p.dim = dim;
  p.D = D;
  p.eps = eps;
  p.q_out = (__nv_bfloat16*)q_out;
  p.k_out = (__nv_bfloat16*)k_out;
  p.out_stride = out_stride;
  p.out_rows = out_rows;
  p.k_out_rows = k_out_rows;
  if (x_stride % 8 || out_stride % 8 || (reinterpret_cast<uintptr_t>(qx) & 15) ||
      (reinterpret_cast<uintptr_t>(kx) & 15) || (reinterpret_cast<uintptr_t>(freqs) & 15) ||
      (reinterpret_cast<uintptr_t>(q_out) & 15) || (reinterpret_cast<uintptr_t>(k_out) & 15) ||
      (reinterpret_cast<uintptr_t>(nqw) & 15) || (reinterpret_cast<uintptr_t>(nkw) & 15)) {
    set_error(HIER_EVALUE, "hier_prep_qk needs 16-byte aligned rows (strides %lld, %lld)",
              (long long)x_stride, (long long)out_stride);
    return HIER_EVALUE;
  }
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaStream_t st = (cudaStream_t)stream;
  if (!cam) return prep_launch<0>(p, sms, st);
  if (cam_dim == 12) return prep_launch<12>(p, sms, st);
  if (cam_dim == 16) return prep_launch<16>(p, sms, st);
  set_error(HIER_ENOTIMPL, "hier_prep_qk supports cam_dim 12 or 16; got %d", cam_dim);
  return HIER_ENOTIMPL;
}

extern "C" int hier_prep_qk_bwd_partials(int64_t S, int32_t* n_warps) {
  clear_error();
  if (S <= 0 || !n_warps) {
    set_error(HIER_EVALUE, "hier_prep_qk_bwd_partials: S=%lld must be positive", (long long)S);
    return HIER_EVALUE;
  }
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  *n_warps = prep_bwd_blocks(S, sms) * kPrepBwdWarps;
  return HIER_OK;
}

extern "C" int hier_prep_qk_bwd(const void* qx, const void* kx, int64_t x_stride, const void* cam,
                                int32_t cam_dim, const void* wcq, const void* wck,
                                const void* nqw, const void* nkw, const float* freqs,
                                int64_t freqs_rows, int64_t S, int32_t H, int32_t D, float eps,
                                const void* gq, const void* gk, int64_t g_stride, void* dqx,
                                void* dkx, int64_t dx_stride, float* dw_part, void* stream) {
  clear_error();
  const int dim = H * D;
  if (dim % 128 != 0 || dim > 256 * kPrepMaxChunks || D <= 0 || D % 8 != 0 || 256 % D != 0) {
    set_error(HIER_ENOTIMPL,
              "hier_prep_qk_bwd needs dim = H*D a multiple of 128 up to %d and head_dim dividing "
              "256; got dim=%d head_dim=%d", 256 * kPrepMaxChunks, dim, D);
    return HIER_ENOTIMPL;
  }
  if (cam && (cam_dim <= 0 || cam_dim > kMaxCam || !wcq || !wck)) {
    set_error(HIER_EVALUE, "camera tokens need 1..%d channels and both cam_q/cam_k weights", kMaxCam);
    return HIER_EVALUE;
  }
  if (S <= 0 || freqs_rows <= 0 || freqs_rows > S) {
    set_error(HIER_EVALUE, "hier_prep_qk_bwd: S=%lld, freqs_rows=%lld", (long long)S,
              (long long)freqs_rows);
    return HIER_EVALUE;
  }
  if (x_stride % 8 || g_stride % 8 || dx_stride % 8 || (reinterpret_cast<uintptr_t>(qx) & 15) ||
      (reinterpret_cast<uintptr_t>(kx) & 15) || (reinterpret_cast<uintptr_t>(gq) & 15) ||
      (reinterpret_cast<uintptr_t>(gk) & 15) || (reinterpret_cast<uintptr_t>(dqx) & 15) ||
      (reinterpret_cast<uintptr_t>(dkx) & 15) || (reinterpret_cast<uintptr_t>(freqs) & 15) ||
      (reinterpret_cast<uintptr_t>(dw_part) & 15) || (reinterpret_cast<uintptr_t>(nqw) & 15) ||
      (reinterpret_cast<uintptr_t>(nkw) & 15)) {
    set_error(HIER_EVALUE, "hier_prep_qk_bwd needs 16-byte aligned rows (strides %lld, %lld, %lld)",
              (long long)x_stride, (long long)g_stride, (long long)dx_stride);
    return HIER_EVALUE;
  }
  PrepBwdArgs b;
  memset(&b, 0, sizeof(b));
  PrepArgs& p = b.f;
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
  p.freqs_rows = freqs_rows;
  p.S = S;
  p.dim = dim;
  p.D = D;
  p.eps = eps;
  b.gq = (const __nv_bfloat16*)gq;
  b.gk = (const __nv_bfloat16*)gk;
  b.g_stride = g_stride;
  b.dqx = (__nv_bfloat16*)dqx;
  b.dkx = (__nv_bfloat16*)dkx;
  b.dx_stride = dx_stride;
  b.dw_part = dw_part;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int blocks = prep_bwd_blocks(S, sms);
  cudaStream_t st = (cudaStream_t)stream;
  if (!cam) return prep_bwd_launch<0>(b, blocks, st);
  if (cam_dim == 12) return prep_bwd_launch<12>(b, blocks, st);
  if (cam_dim == 16) return prep_bwd_launch<16>(b, blocks, st);
  set_error(HIER_ENOTIMPL, "hier_prep_qk_bwd supports cam_dim 12 or 16; got %d", cam_dim);
  return HIER_ENOTIMPL;
}
