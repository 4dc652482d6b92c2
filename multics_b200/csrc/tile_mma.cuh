// 128 x 128 bf16 tiles for tcgen05 kind::f16 MMAs: the shared-memory tile
// layout, descriptors and issue sequences used by the attention forward and
// backward kernels.
//
// A tile is 128 rows x 128 columns of bf16 in shared memory, stored as two
// 64-column halves, each 128 rows of 128 bytes in the 128-byte swizzled
// layout, and loaded as 64-column TMA boxes (128 rows, or two boxes of 64
// rows whose source rows the caller chooses).  The same bytes serve as a
// K-major operand (rows = M or N, the 128 columns = the reduction) and as an
// MN-major B operand (rows = the reduction, the 128 columns = N).
#pragma once

#include "common.cuh"

namespace hier {

constexpr int kBM = 128;                // query rows per tile
constexpr int kBN = 128;                // keys per tile
constexpr int kHD = 128;                // head dim
constexpr int kTile = kBM * kHD * 2;    // 32 KiB
constexpr int kHalf = kTile / 2;        // one 64-column half (128-byte rows)
constexpr int kBoxBytes = kHalf / 2;    // one 64-row TMA box inside a column half

// A key-box row carries the index of its key/value tensor map in the top bits.
constexpr int kMapShift = 24;
constexpr int kRowMask = (1 << kMapShift) - 1;

// Shared-memory descriptors are built once per operand base (low word) and
// advanced per 16-element k-step by adding a compile-time offset to the start
// address field (16-byte units).
constexpr uint32_t kDescHi = (1024u >> 4) | (1u << 14) | (2u << 29);  // SBO=1024, v1, SW128
__device__ __forceinline__ uint32_t sdesc_lo_kmajor(uint32_t saddr) {
  return ((saddr >> 4) & 0x3FFFu) | (1u << 16);  // LBO = 16 B (unused for SW128 K-major)
}
__device__ __forceinline__ uint32_t sdesc_lo_mnmajor(uint32_t saddr) {
  return ((saddr >> 4) & 0x3FFFu) | (static_cast<uint32_t>(kHalf >> 4) << 16);  // LBO = 16 KiB
}
__device__ __forceinline__ uint64_t sdesc(uint32_t lo) {
  return (static_cast<uint64_t>(kDescHi) << 32) | lo;
}

// tcgen05.mma with the shared-memory descriptors assembled inside the PTX
// from their low words (the high word is the constant kDescHi), so that the
// issuing thread keeps 32-bit operand addresses only.
// The constant offsets (16-byte units) are added inside the PTX as well.
template <uint32_t kOffA, uint32_t kOffB>
__device__ __forceinline__ void umma_ss_lo(uint32_t d_tmem, uint32_t alo, uint32_t blo,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b32 la, lb;\n\t.reg .b64 da, db;\n\t"
      "add.u32 la, %1, %6;\n\t"
      "add.u32 lb, %2, %7;\n\t"
      "mov.b64 da, {la, %5};\n\t"
      "mov.b64 db, {lb, %5};\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(alo), "r"(blo), "r"(idesc), "r"(accumulate), "n"(kDescHi), "n"(kOffA), "n"(kOffB)
      : "memory");
}
template <uint32_t kOffA, uint32_t kOffB>
__device__ __forceinline__ void umma_ts_lo(uint32_t d_tmem, uint32_t a_tmem, uint32_t blo,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b32 ta, lb;\n\t.reg .b64 db;\n\t"
      "add.u32 ta, %1, %6;\n\t"
      "add.u32 lb, %2, %7;\n\t"
      "mov.b64 db, {lb, %5};\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], db, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "r"(blo), "r"(idesc), "r"(accumulate), "n"(kDescHi), "n"(kOffA), "n"(kOffB)
      : "memory");
}

template <int k>
__device__ __forceinline__ void issue_s_step(uint32_t d_tmem, uint32_t qlo, uint32_t klo) {
  constexpr uint32_t idesc = idesc_bf16(kBM, kBN, false);
  constexpr uint32_t off = ((k >> 2) * kHalf + (k & 3) * 32) >> 4;
  umma_ss_lo<off, off>(d_tmem, qlo, klo, idesc, k > 0 ? 1u : 0u);
}
template <int k>
__device__ __forceinline__ void issue_pv_step(uint32_t o_tmem, uint32_t p_tmem, uint32_t vlo,
                                              bool accumulate) {
  constexpr uint32_t idesc = idesc_bf16(kBM, kHD, true);
  constexpr uint32_t offv = (k * 2048) >> 4;
  umma_ts_lo<k * 8, offv>(o_tmem, p_tmem, vlo, idesc, (accumulate || k > 0) ? 1u : 0u);
}

// S (128 x 128, fp32 in TMEM) = Q (128 x 128) * K (128 x 128)^T
__device__ __forceinline__ void issue_s(uint32_t d_tmem, uint32_t qlo, uint32_t klo) {
  static_assert(kHD / 16 == 8, "eight K steps");
  issue_s_step<0>(d_tmem, qlo, klo);
  issue_s_step<1>(d_tmem, qlo, klo);
  issue_s_step<2>(d_tmem, qlo, klo);
  issue_s_step<3>(d_tmem, qlo, klo);
  issue_s_step<4>(d_tmem, qlo, klo);
  issue_s_step<5>(d_tmem, qlo, klo);
  issue_s_step<6>(d_tmem, qlo, klo);
  issue_s_step<7>(d_tmem, qlo, klo);
}

// O (128 x 128) += P (128 x 128 keys, bf16 in TMEM) * V (128 keys x 128), the
// half over keys 64*H .. 64*H + 63 (K steps 4H .. 4H+3): the first half can
// run while the second half of P is computed.
template <int H>
__device__ __forceinline__ void issue_pv_half(uint32_t o_tmem, uint32_t p_tmem, uint32_t vlo,
                                              bool accumulate) {
  static_assert(kBN / 16 == 8 && (H == 0 || H == 1), "two halves of four K steps");
  issue_pv_step<4 * H + 0>(o_tmem, p_tmem, vlo, accumulate);
  issue_pv_step<4 * H + 1>(o_tmem, p_tmem, vlo, accumulate);
  issue_pv_step<4 * H + 2>(o_tmem, p_tmem, vlo, accumulate);
  issue_pv_step<4 * H + 3>(o_tmem, p_tmem, vlo, accumulate);
}

template <int kMaps>
__device__ __forceinline__ void load_kv_tile(uint8_t* dst, const CUtensorMap* maps, uint64_t* bar,
                                             int col, int r0, int r1) {
  const CUtensorMap* m0 = maps + (kMaps == 1 ? 0 : (r0 >> kMapShift));
  const CUtensorMap* m1 = maps + (kMaps == 1 ? 0 : (r1 >> kMapShift));
  r0 &= kRowMask;
  r1 &= kRowMask;
  mbar_arrive_expect_tx(bar, kTile);
  tma_load_2d(dst, m0, bar, col, r0);
  tma_load_2d(dst + kBoxBytes, m1, bar, col, r1);
  tma_load_2d(dst + kHalf, m0, bar, col + 64, r0);
  tma_load_2d(dst + kHalf + kBoxBytes, m1, bar, col + 64, r1);
}

}  // namespace hier
