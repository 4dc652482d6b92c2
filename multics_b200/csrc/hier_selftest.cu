// Self-tests: the tcgen05 operand encodings used by the attention kernel (SS
// form with K-major A and B, SS form with an MN-major B, and the TS form with
// A read from tensor memory, bf16 pairs packed per 32-bit column), and the
// bounded mbarrier wait that every pipeline wait uses (it must give up and
// report, never hang).

#include <stdio.h>

#include "common.cuh"
#include "tmap.h"

namespace hier {

constexpr int kTile = 128 * 128 * 2;
constexpr int kHalf = kTile / 2;

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

namespace hier {
// One thread waits, with the given limit, on a fresh mbarrier phase that
// nothing completes: the wait must give up, record DEV_WAIT_TIMEOUT with the
// site in *err and report the cycles it waited.
__global__ void selftest_wait_kernel(long long limit, int* err, long long* cycles) {
  __shared__ uint64_t bar;
  if (threadIdx.x != 0) return;
  mbar_init(&bar, 1);
  fence_mbar_init();
  const long long t0 = clock64();
  const bool done = mbar_wait_limit(&bar, 0, err, 30, limit);
  *cycles = done ? -1 : clock64() - t0;
}
}  // namespace hier

extern "C" int hier_selftest_wait_timeout(int64_t limit_cycles, int32_t* dev_err,
                                          int64_t* dev_cycles, void* stream) {
  clear_error();
  if (limit_cycles <= 0 || limit_cycles > kWaitLimitCycles || !dev_err || !dev_cycles) {
    set_error(HIER_EVALUE, "wait limit must be 1..%lld cycles with both outputs given",
              (long long)kWaitLimitCycles);
    return HIER_EVALUE;
  }
  selftest_wait_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(
      (long long)limit_cycles, dev_err, reinterpret_cast<long long*>(dev_cycles));
  HIER_CHECK_CUDA(cudaGetLastError(), "selftest_wait_kernel launch");
  return HIER_OK;
}
