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
// blockIdx.y selects Q (0) or K (1).  Each block iteration handles kRows
// consecutive tokens, so every thread keeps kRows independent 16-byte loads
// in flight and the block does one reduction round per kRows tokens.  The
// camera weights are transposed once into shared memory, channel-contiguous,
// so a thread reads its 8 channels of one camera input with one 16-byte load.
constexpr int kPrepRows = 4;

// proj[i] = sum_c cam[c] * W[d0+i][c] with W staged as wsm[c][thread] (8 bf16)
template <int CAM>
__device__ __forceinline__ void cam_project(const uint4* wsm, int nthreads, int t,
                                            const float* cam, float (&proj)[8]) {
#pragma unroll
  for (int i = 0; i < 8; ++i) proj[i] = 0.f;
#pragma unroll
  for (int c = 0; c < CAM; ++c) {
    float w[8];
    bf16x8_to_f32(wsm[c * nthreads + t], w);
    const float cv = cam[c];
#pragma unroll
    for (int i = 0; i < 8; ++i) proj[i] = fmaf(cv, w[i], proj[i]);
  }
}

template <int CAM>
__global__ void __launch_bounds__(384, 1) prep_qk_kernel(PrepArgs a) {
  constexpr int R = kPrepRows;
  extern __shared__ uint4 wsm[];  // [CAM][blockDim] x 8 bf16
  __shared__ float red[R][12];
  __shared__ float camv[R][CAM > 0 ? CAM : 1];
  __shared__ float4 frs[R][64];  // RoPE (cos, sin) pairs of the chunk's rows, D <= 256
  const bool is_k = blockIdx.y == 1;
  const __nv_bfloat16* x = is_k ? a.kx : a.qx;
  const __nv_bfloat16* wc = is_k ? a.wck : a.wcq;
  const __nv_bfloat16* nw = is_k ? a.nkw : a.nqw;
  __nv_bfloat16* out = is_k ? a.k_out : a.q_out;
  const int t = threadIdx.x;
  const int d0 = t * 8;
  const int nt = blockDim.x;
  const int nwarps = nt / 32;
  if (CAM > 0) {
    const uint16_t* w16 = reinterpret_cast<const uint16_t*>(wc);
    for (int c = 0; c < CAM; ++c) {
      uint32_t p[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        p[i] = (uint32_t)w16[(int64_t)(d0 + 2 * i) * CAM + c] |
               ((uint32_t)w16[(int64_t)(d0 + 2 * i + 1) * CAM + c] << 16);
      wsm[c * nt + t] = make_uint4(p[0], p[1], p[2], p[3]);
    }
  }
  float nv[8];
  bf16x8_to_f32(*reinterpret_cast<const uint4*>(nw + d0), nv);
  const int pair0 = (d0 % a.D) / 2;
  const int half = a.D / 2;
  const int64_t stride = (int64_t)gridDim.x * R;
  // Every global load of a chunk (its R rows, camera values and RoPE pairs)
  // is issued one chunk ahead into registers; camera values and RoPE pairs
  // are then staged in shared memory for the whole block.
  constexpr int kc = CAM > 0 ? CAM : 1;
  const int fq = half / 2;  // float4 (two pairs) per row of the RoPE table
  const int n_cam = CAM > 0 ? R * CAM : 0;
  const int n_fr = R * fq;
  uint4 raw[R];
  float cam_r[2];
  float4 fr_r[4];
  auto fetch = [&](int64_t r0, uint4 (&rows)[R], float (&cr)[2], float4 (&fr)[4]) {
#pragma unroll
    for (int r = 0; r < R; ++r)
      rows[r] = r0 + r < a.S ? *reinterpret_cast<const uint4*>(x + (r0 + r) * a.x_stride + d0)
                             : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int i = t + k * nt;
      cr[k] = 0.f;
      if (i < n_cam && r0 + i / kc < a.S) cr[k] = __bfloat162float(a.cam[(r0 + i / kc) * CAM + i % kc]);
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = t + k * nt;
      fr[k] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (i < n_fr && r0 + i / fq < a.S)
        fr[k] = reinterpret_cast<const float4*>(a.freqs + (r0 + i / fq) * half)[i % fq];
    }
  };
  fetch((int64_t)blockIdx.x * R, raw, cam_r, fr_r);
  for (int64_t row0 = (int64_t)blockIdx.x * R; row0 < a.S; row0 += stride) {
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int i = t + k * nt;
      if (i < n_cam) camv[i / kc][i % kc] = cam_r[k];
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = t + k * nt;
      if (i < n_fr) frs[i / fq][i % fq] = fr_r[k];
    }
    uint4 nxt[R];
    float cam_n[2];
    float4 fr_n[4];
    fetch(row0 + stride, nxt, cam_n, fr_n);
    __syncthreads();
    float xv[R][8];
    float ss[R];
    // Camera rows repeat over a player frame's patches, so the chunk usually
    // shares one row: project it once (exact: same inputs, same result).
    bool shared_cam = true;
    float proj[8];
    if (CAM > 0) {
#pragma unroll
      for (int r = 1; r < R; ++r)
#pragma unroll
        for (int c = 0; c < CAM; ++c) shared_cam &= camv[r][c] == camv[0][c];
      if (shared_cam) cam_project<CAM>(wsm, nt, t, camv[0], proj);
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
      bf16x8_to_f32(raw[r], xv[r]);
      if (CAM > 0) {
        if (!shared_cam) cam_project<CAM>(wsm, nt, t, camv[r], proj);
#pragma unroll
        for (int i = 0; i < 8; ++i) xv[r][i] += proj[i];
      }
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) s = fmaf(xv[r][i], xv[r][i], s);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      ss[r] = s;
    }
    if ((t & 31) == 0) {
#pragma unroll
      for (int r = 0; r < R; ++r) red[r][t >> 5] = ss[r];
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if (row0 + r >= a.S) break;
      float tot = 0.f;
      for (int w = 0; w < nwarps; ++w) tot += red[r][w];
      const float rs = rsqrtf(tot / a.dim + a.eps);
      const float4 f0 = frs[r][pair0 / 2], f1 = frs[r][pair0 / 2 + 1];
      uint4 o;
      uint32_t* po = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 f2 = i < 2 ? f0 : f1;
        const float c = (i & 1) ? f2.z : f2.x;
        const float s = (i & 1) ? f2.w : f2.y;
        const float a0 = xv[r][2 * i] * rs * nv[2 * i], a1 = xv[r][2 * i + 1] * rs * nv[2 * i + 1];
        po[i] = pack_bf16x2(a0 * c - a1 * s, a0 * s + a1 * c);
      }
      *reinterpret_cast<uint4*>(out + (row0 + r) * a.out_stride + d0) = o;
    }
#pragma unroll
    for (int r = 0; r < R; ++r) raw[r] = nxt[r];
#pragma unroll
    for (int k = 0; k < 2; ++k) cam_r[k] = cam_n[k];
#pragma unroll
    for (int k = 0; k < 4; ++k) fr_r[k] = fr_n[k];
    __syncthreads();
  }
}

}  // namespace hier

using namespace hier;

extern "C" int hier_prep_qk(const void* qx, const void* kx, int64_t x_stride, const void* cam,
                            int32_t cam_dim, const void* wcq, const void* wck, const void* nqw,
                            const void* nkw, const float* freqs, int64_t S, int32_t H, int32_t D,
                            float eps, void* q_out, void* k_out, int64_t out_stride,
                            void* stream) {
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
  const int threads = dim / 8;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // one resident block per SM for each of Q and K
  const int64_t chunks = (S + kPrepRows - 1) / kPrepRows;
  const int64_t blocks = chunks < (sms + 1) / 2 ? chunks : (sms + 1) / 2;
  const dim3 grid((unsigned)blocks, 2);
  cudaStream_t st = (cudaStream_t)stream;
  const size_t wbytes = (size_t)(cam ? cam_dim : 0) * threads * sizeof(uint4);
  if (!cam) {
    prep_qk_kernel<0><<<grid, threads, 0, st>>>(p);
  } else if (cam_dim == 12) {
    HIER_CHECK_CUDA(cudaFuncSetAttribute(prep_qk_kernel<12>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)wbytes),
                    "cudaFuncSetAttribute(prep_qk_kernel)");
    prep_qk_kernel<12><<<grid, threads, wbytes, st>>>(p);
  } else if (cam_dim == 16) {
    HIER_CHECK_CUDA(cudaFuncSetAttribute(prep_qk_kernel<16>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)wbytes),
                    "cudaFuncSetAttribute(prep_qk_kernel)");
    prep_qk_kernel<16><<<grid, threads, wbytes, st>>>(p);
  } else {
    set_error(HIER_ENOTIMPL, "hier_prep_qk supports cam_dim 12 or 16; got %d", cam_dim);
    return HIER_ENOTIMPL;
  }
  HIER_CHECK_CUDA(cudaGetLastError(), "prep_qk_kernel launch");
  return HIER_OK;
}
