// Host-side plumbing of the C ABI: thread-local error state and TMA tensor
// map encoding through the driver entry point (no -lcuda link needed).

#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <cudaTypedefs.h>

#include "common.cuh"
#include "tmap.h"

namespace hier {

static thread_local char g_msg[1024] = "";
static thread_local int g_code = HIER_OK;

void set_error(int code, const char* fmt, ...) {
  g_code = code;
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
}

void clear_error() {
  g_code = HIER_OK;
  g_msg[0] = '\0';
}

int cuda_status(cudaError_t e, const char* what) {
  set_error(HIER_ECUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
  return HIER_ECUDA;
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

int make_tmap_bf16_2d(CUtensorMap* m, const void* ptr, uint64_t cols, uint64_t rows,
                      uint64_t row_stride_elems, uint32_t box_cols, uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) {
    set_error(HIER_ECUDA, "cuTensorMapEncodeTiled entry point unavailable");
    return HIER_ECUDA;
  }
  if ((reinterpret_cast<uintptr_t>(ptr) & 15) != 0 || (row_stride_elems * 2) % 16 != 0) {
    set_error(HIER_EVALUE, "TMA operand must be 16-byte aligned with 16-byte row stride");
    return HIER_EVALUE;
  }
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_stride_elems * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides,
                  box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error(HIER_ECUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
    return HIER_ECUDA;
  }
  return HIER_OK;
}

}  // namespace hier

extern "C" const char* hier_last_error(void) { return hier::g_msg; }
extern "C" int hier_last_error_code(void) { return hier::g_code; }
extern "C" int hier_abi_version(void) { return 5; }
