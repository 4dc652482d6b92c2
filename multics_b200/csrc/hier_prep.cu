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
  int64_t S;
  int dim;
  int D;
  float eps;
  __nv_bfloat16* q_out;
  __nv_bfloat16* k_out;
  int64_t out_stride;
  const int32_t* out_rows;  // output row of each input row (NULL: the same row)
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
// blockIdx.y selects Q (0) or K (1).  The CTA walks chunks of kPrepRows
// consecutive tokens; thread 0 streams each chunk's rows and RoPE rows into a
// kPrepStages-deep shared-memory ring with bulk async copies, so several
// chunks of loads are in flight per SM while the block computes one.  The
// camera weights of a thread's 8 channels sit in registers.
constexpr int kPrepRows = 8;
constexpr int kPrepStages = 3;

__device__ int g_prep_err;  // pipeline wait timeouts of the prologue kernel

__host__ __device__ constexpr int align16i(int x) { return (x + 15) & ~15; }

template <int CAM>
__global__ void __launch_bounds__(384, 1) prep_qk_kernel(PrepArgs a) {
  constexpr int R = kPrepRows;
  extern __shared__ __align__(128) uint8_t ring[];
  __shared__ uint64_t full[kPrepStages];
  __shared__ float red[R][12];
  __shared__ float rsq[R];
  __shared__ float camv[R][CAM > 0 ? CAM : 1];
  const bool is_k = blockIdx.y == 1;
  const __nv_bfloat16* x = is_k ? a.kx : a.qx;
  const __nv_bfloat16* wc = is_k ? a.wck : a.wcq;
  const __nv_bfloat16* nw = is_k ? a.nkw : a.nqw;
  __nv_bfloat16* out = is_k ? a.k_out : a.q_out;
  const int t = threadIdx.x;
  const int d0 = t * 8;
  const int nt = blockDim.x;
  const int nwarps = nt / 32;
  const int half = a.D / 2;
  const int row_bytes = a.dim * 2;
  const int fr_bytes = half * 8;  // (cos, sin) float pairs of one token
  const int stage_bytes = align16i(R * (row_bytes + fr_bytes));
  // camera weights W[d0 + i][c] of this thread's channels, bf16 pairs
  constexpr int kc = CAM > 0 ? CAM : 1;
  uint32_t wr[kc][4];
  if (CAM > 0) {
    const uint16_t* w16 = reinterpret_cast<const uint16_t*>(wc);
#pragma unroll
    for (int c = 0; c < CAM; ++c)
#pragma unroll
      for (int i = 0; i < 4; ++i)
        wr[c][i] = (uint32_t)w16[(int64_t)(d0 + 2 * i) * CAM + c] |
                   ((uint32_t)w16[(int64_t)(d0 + 2 * i + 1) * CAM + c] << 16);
  }
  float nv[8];
  bf16x8_to_f32(*reinterpret_cast<const uint4*>(nw + d0), nv);
  const int pair0 = (d0 % a.D) / 2;
  const int64_t n_chunks = (a.S + R - 1) / R;
  if (t == 0) {
    for (int s = 0; s < kPrepStages; ++s) mbar_init(full + s, 1);
    fence_mbar_init();
  }
  __syncthreads();
  // chunk i of this CTA is chunk blockIdx.x + i * gridDim.x of the sequence
  auto issue = [&](int64_t i) {
    const int64_t c = blockIdx.x + i * (int64_t)gridDim.x;
    if (c >= n_chunks) return;
    const int64_t r0 = c * R;
    const int nr = (int)min((int64_t)R, a.S - r0);
    uint8_t* st = ring + (i % kPrepStages) * stage_bytes;
    uint64_t* bar = full + (i % kPrepStages);
    mbar_arrive_expect_tx(bar, nr * (row_bytes + fr_bytes));
    for (int r = 0; r < nr; ++r)
      bulk_load(st + r * row_bytes, x + (r0 + r) * a.x_stride, row_bytes, bar);
    bulk_load(st + R * row_bytes, a.freqs + r0 * half, nr * fr_bytes, bar);
  };
  if (t == 0)
    for (int i = 0; i < kPrepStages - 1; ++i) issue(i);
  // camera rows are tiny: plain loads, one chunk ahead, through registers
  const int n_cam = CAM > 0 ? R * CAM : 0;
  // R*CAM <= 128 camera values per chunk, >= 32 threads per block
  constexpr int kCamPer = (R * kMaxCam + 31) / 32;
  float cam_r[kCamPer];
  auto fetch_cam = [&](int64_t i) {
    const int64_t r0 = (blockIdx.x + i * (int64_t)gridDim.x) * R;
#pragma unroll
    for (int k = 0; k < kCamPer; ++k) {
      const int j = t + k * nt;
      cam_r[k] = 0.f;
      if (j < n_cam && r0 + j / kc < a.S) cam_r[k] = __bfloat162float(a.cam[(r0 + j / kc) * CAM + j % kc]);
    }
  };
  if (CAM > 0) fetch_cam(0);
  for (int64_t i = 0;; ++i) {
    const int64_t row0 = (blockIdx.x + i * (int64_t)gridDim.x) * R;
    if (row0 >= a.S) break;
    if (t == 0) issue(i + kPrepStages - 1);  // into the stage freed by iteration i-1
    if (CAM > 0) {
#pragma unroll
      for (int k = 0; k < kCamPer; ++k) {
        const int j = t + k * nt;
        if (j < n_cam) camv[j / kc][j % kc] = cam_r[k];
      }
      fetch_cam(i + 1);
    }
    const uint8_t* st = ring + (i % kPrepStages) * stage_bytes;
    mbar_wait(full + (i % kPrepStages), (uint32_t)((i / kPrepStages) & 1), &g_prep_err, 1);
    __syncthreads();  // camv visible
    const int nr = (int)min((int64_t)R, a.S - row0);
    // rows of one player frame share their camera row: project it once
    bool shared_cam = true;
    float proj[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) proj[q] = 0.f;
    auto project = [&](int r) {  // proj = W cam_r for this thread's 8 channels
#pragma unroll
      for (int q = 0; q < 8; ++q) proj[q] = 0.f;
#pragma unroll
      for (int c = 0; c < CAM; ++c) {
        float w[8];
        bf16x8_to_f32(make_uint4(wr[c][0], wr[c][1], wr[c][2], wr[c][3]), w);
        const float cv = camv[r][c];
#pragma unroll
        for (int q = 0; q < 8; ++q) proj[q] = fmaf(cv, w[q], proj[q]);
      }
    };
    if (CAM > 0) {
#pragma unroll
      for (int r = 1; r < R; ++r)
#pragma unroll
        for (int c = 0; c < CAM; ++c) shared_cam &= camv[r][c] == camv[0][c];
      if (shared_cam) project(0);
    }
    // pass 1: sums of squares of all rows, reduced together
    float ss[R];
    if (CAM == 0 || shared_cam) {
#pragma unroll
      for (int r = 0; r < R; ++r) {
        float xv[8];
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(st + r * row_bytes + d0 * 2), xv);
        float sq = 0.f;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float v = CAM > 0 ? xv[q] + proj[q] : xv[q];
          sq = fmaf(v, v, sq);
        }
        ss[r] = r < nr ? sq : 0.f;
      }
    } else {  // a chunk across a frame boundary: one projection per row
#pragma unroll 1
      for (int r = 0; r < R; ++r) {
        project(r);
        float xv[8];
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(st + r * row_bytes + d0 * 2), xv);
        float sq = 0.f;
#pragma unroll
        for (int q = 0; q < 8; ++q) sq = fmaf(xv[q] + proj[q], xv[q] + proj[q], sq);
        ss[r] = r < nr ? sq : 0.f;
      }
    }
    // warp sums of the R = 8 rows by a halving exchange: after the offsets
    // 16, 8, 4 each lane holds one row's partial (row = lane bits 4, 3, 2),
    // then offsets 2 and 1 finish it (9 shuffles instead of 40)
    static_assert(R == 8, "the row-sum exchange below assumes 8 rows per chunk");
    {
      const int lane = t & 31;
#pragma unroll
      for (int k = 0; k < 3; ++k) {
        const int o = 16 >> k, keep = (lane & o) ? 1 : 0;
        const int n = 4 >> k;  // values kept after this step
#pragma unroll
        for (int i = 0; i < n; ++i) {
          const float send = keep ? ss[i] : ss[i + n];
          const float recv = __shfl_xor_sync(0xffffffffu, send, o);
          ss[i] = (keep ? ss[i + n] : ss[i]) + recv;
        }
      }
      ss[0] += __shfl_xor_sync(0xffffffffu, ss[0], 2);
      ss[0] += __shfl_xor_sync(0xffffffffu, ss[0], 1);
      if ((lane & 3) == 0) {
        const int row = ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1);
        red[row][t >> 5] = ss[0];
      }
    }
    __syncthreads();
    if (t < R) {  // row scales once per chunk
      float tot = 0.f;
      for (int w = 0; w < nwarps; ++w) tot += red[t][w];
      rsq[t] = rsqrtf(tot / a.dim + a.eps);
    }
    __syncthreads();
    // pass 2: normalise, rotate, store
    const float4* fr = reinterpret_cast<const float4*>(st + R * row_bytes);
    auto finish = [&](int r) {
      const float rs = rsq[r];
      float xv[8];
      bf16x8_to_f32(*reinterpret_cast<const uint4*>(st + r * row_bytes + d0 * 2), xv);
      if (CAM > 0) {
#pragma unroll
        for (int q = 0; q < 8; ++q) xv[q] += proj[q];
      }
      const float4 f0 = fr[r * (half / 2) + pair0 / 2], f1 = fr[r * (half / 2) + pair0 / 2 + 1];
      uint4 o;
      uint32_t* po = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 f2 = q < 2 ? f0 : f1;
        const float c = (q & 1) ? f2.z : f2.x;
        const float s = (q & 1) ? f2.w : f2.y;
        const float a0 = xv[2 * q] * rs * nv[2 * q], a1 = xv[2 * q + 1] * rs * nv[2 * q + 1];
        po[q] = pack_bf16x2(a0 * c - a1 * s, a0 * s + a1 * c);
      }
      const int64_t dst = a.out_rows ? (int64_t)a.out_rows[row0 + r] : row0 + r;
      *reinterpret_cast<uint4*>(out + dst * a.out_stride + d0) = o;
    };
    if (CAM == 0 || shared_cam) {  // proj still holds the chunk's shared projection
#pragma unroll
      for (int r = 0; r < R; ++r)
        if (r < nr) finish(r);
    } else {
#pragma unroll 1
      for (int r = 0; r < nr; ++r) {
        project(r);
        finish(r);
      }
    }
    __syncthreads();  // stage and red free for the next chunks
  }
}

}  // namespace hier

using namespace hier;

extern "C" int hier_prep_qk(const void* qx, const void* kx, int64_t x_stride, const void* cam,
                            int32_t cam_dim, const void* wcq, const void* wck, const void* nqw,
                            const void* nkw, const float* freqs, int64_t S, int32_t H, int32_t D,
                            float eps, void* q_out, void* k_out, int64_t out_stride,
                            const int32_t* out_rows, void* stream) {
  clear_error();
  const int dim = H * D;
  if (dim % 8 != 0 || dim / 8 > 384 || dim / 8 < 32 || (dim / 8) % 32 != 0 || D % 8 != 0) {
    set_error(HIER_ENOTIMPL, "hier_prep_qk needs dim = H*D with dim/8 a multiple of 32 and <= 384; got dim=%d", dim);
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
  p.out_rows = out_rows;
  const int threads = dim / 8;
  if (x_stride % 8 || out_stride % 8 || (reinterpret_cast<uintptr_t>(qx) & 15) ||
      (reinterpret_cast<uintptr_t>(kx) & 15) || (reinterpret_cast<uintptr_t>(freqs) & 15)) {
    set_error(HIER_EVALUE, "hier_prep_qk needs 16-byte aligned rows (strides %lld, %lld)",
              (long long)x_stride, (long long)out_stride);
    return HIER_EVALUE;
  }
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // one resident block per SM for each of Q and K
  const int64_t chunks = (S + kPrepRows - 1) / kPrepRows;
  const int64_t blocks = chunks < (sms + 1) / 2 ? chunks : (sms + 1) / 2;
  const dim3 grid((unsigned)blocks, 2);
  cudaStream_t st = (cudaStream_t)stream;
  const size_t ring = (size_t)kPrepStages * align16i(kPrepRows * (dim * 2 + (D / 2) * 8));
  if (!cam) {
    HIER_CHECK_CUDA(cudaFuncSetAttribute(prep_qk_kernel<0>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ring),
                    "cudaFuncSetAttribute(prep_qk_kernel)");
    prep_qk_kernel<0><<<grid, threads, ring, st>>>(p);
  } else if (cam_dim == 12) {
    HIER_CHECK_CUDA(cudaFuncSetAttribute(prep_qk_kernel<12>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ring),
                    "cudaFuncSetAttribute(prep_qk_kernel)");
    prep_qk_kernel<12><<<grid, threads, ring, st>>>(p);
  } else if (cam_dim == 16) {
    HIER_CHECK_CUDA(cudaFuncSetAttribute(prep_qk_kernel<16>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ring),
                    "cudaFuncSetAttribute(prep_qk_kernel)");
    prep_qk_kernel<16><<<grid, threads, ring, st>>>(p);
  } else {
    set_error(HIER_ENOTIMPL, "hier_prep_qk supports cam_dim 12 or 16; got %d", cam_dim);
    return HIER_ENOTIMPL;
  }
  HIER_CHECK_CUDA(cudaGetLastError(), "prep_qk_kernel launch");
  return HIER_OK;
}
