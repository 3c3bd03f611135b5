// Host-side plumbing shared by every entry point: thread-local error text,
// status codes, the device error word, SM count and TMA descriptor encoding.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace fvb {

static thread_local char t_err[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_err, sizeof(t_err), fmt, ap);
  va_end(ap);
}

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_err, sizeof(t_err), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(FVB_ERR_CUDA, "%s launch: %s", what, cudaGetErrorString(e));
  return FVB_OK;
}

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes,
                 uint64_t inner, uint64_t outer, uint64_t row_bytes, uint32_t box_inner,
                 uint32_t box_outer, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(FVB_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if (!aligned16(base)) return fail(FVB_ERR_INVALID, "TMA base pointer not 16-byte aligned");
  if (row_bytes % 16 != 0) return fail(FVB_ERR_INVALID, "TMA row pitch %llu not a multiple of 16",
                                       (unsigned long long)row_bytes);
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  (void)elem_bytes;
  CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FVB_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return FVB_OK;
}

}  // namespace fvb

extern "C" {

int fvb_abi_version(void) { return 1; }

const char* fvb_last_error(void) { return fvb::t_err; }

int fvb_device_error(unsigned int* code_out) {
  unsigned int v = 0, zero = 0;
  FVB_CUDA_TRY(cudaMemcpyFromSymbol(&v, fvb::g_device_error, sizeof(v)), "read device error");
  FVB_CUDA_TRY(cudaMemcpyToSymbol(fvb::g_device_error, &zero, sizeof(zero)), "clear device error");
  if (code_out) *code_out = v;
  return FVB_OK;
}

}  // extern "C"
