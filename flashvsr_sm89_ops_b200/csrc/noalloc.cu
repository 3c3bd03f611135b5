// Per-tensor FP8 quantisation that allocates nothing: its scratch lives in a
// fixed device array compiled into the library.
//
// Who needs this: callers that hold device pointers but cannot allocate device
// memory themselves -- a host application reaching this library only through
// the C ABI (an FFI binding with no device allocator of its own), a process whose
// device memory is owned by another framework's pool, or a latency-critical loop
// that must not pay cudaMalloc's implicit device synchronisation.  The regular
// fvb_quant_fp8(FVB_SCALE_TENSOR) needs a caller-provided workspace for its
// reduction; this variant needs none.
//
// Scratch: g_noalloc_partials, FVB_NOALLOC_QUANT_MAX_PARTIALS floats (64 KB),
// resident on every GPU that loads the library until the process exits.  Pass 1
// writes one partial |x| maximum per 65,536-element chunk; pass 2 reduces them
// (order-independent, so the result is bit-identical to fvb_quant_fp8's) and
// quantises.  Every slot pass 2 reads was written by pass 1 of the same call, so
// nothing has to be cleared; the array keeps the last call's partials.  All calls
// share the one array: calls whose kernels overlap on the GPU (two streams, two
// threads) race and must be ordered by the caller.
#include <mutex>

#include "common.cuh"

namespace fvb {
namespace noalloc {

constexpr int64_t kChunk = 65536;  // elements per pass-1 CTA (multiple of 8)
constexpr int kMaxPartials = FVB_NOALLOC_QUANT_MAX_PARTIALS;

static __device__ __align__(256) float g_noalloc_partials[kMaxPartials];

__global__ void __launch_bounds__(256) chunk_absmax_kernel(const __nv_bfloat16* __restrict__ x,
                                                            int64_t n, float* __restrict__ partials) {
  const int64_t begin = (int64_t)blockIdx.x * kChunk;
  const int64_t end = begin + kChunk < n ? begin + kChunk : n;
  float m = 0.f;
  const int64_t vend = begin + ((end - begin) & ~(int64_t)7);
  const uint4* xv = reinterpret_cast<const uint4*>(x + begin);
  for (int64_t v = threadIdx.x; begin + v * 8 < vend; v += blockDim.x) {
    float f[8];
    bf16x8_to_f32(__ldg(xv + v), f);
#pragma unroll
    for (int i = 0; i < 8; ++i) m = fmaxf(m, fabsf(f[i]));
  }
  for (int64_t i = vend + threadIdx.x; i < end; i += blockDim.x)
    m = fmaxf(m, fabsf(__bfloat162float(x[i])));
  m = warp_max(m);
  __shared__ float red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_max(t);
    if (threadIdx.x == 0) partials[blockIdx.x] = t;
  }
}

__global__ void __launch_bounds__(256) quant_from_partials_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t n, const float* __restrict__ partials,
    int nparts, uint8_t* __restrict__ q, float* __restrict__ scale_out) {
  // every CTA reduces the same partials, so every CTA derives the same amax
  float m = 0.f;
  for (int i = threadIdx.x; i < nparts; i += blockDim.x) m = fmaxf(m, partials[i]);
  m = warp_max(m);
  __shared__ float red[8];
  __shared__ float amax_s;
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_max(t);
    if (threadIdx.x == 0) amax_s = t;
  }
  __syncthreads();
  const float amax = amax_s;
  // s = max(amax, 1e-12) / 448, q = e4m3(clamp(x / s)), IEEE divides (fp8_quant.py:25-35);
  // the saturating conversion is the clamp and, like clamp-then-cast, keeps a NaN a NaN
  const float s = __fdiv_rn(fmaxf(amax, 1e-12f), 448.0f);
  if (blockIdx.x == 0 && threadIdx.x == 0) scale_out[0] = returned_scale(amax);
  const int64_t nvec = n >> 3;
  const uint4* xv = reinterpret_cast<const uint4*>(x);
  uint2* qv = reinterpret_cast<uint2*>(q);
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < nvec;
       v += (int64_t)gridDim.x * blockDim.x) {
    float f[8];
    bf16x8_to_f32(__ldg(xv + v), f);
    uint32_t w[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float a[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = __fdiv_rn(f[4 * h + i], s);
      w[h] = (uint32_t)f32x2_to_e4m3x2(a[0], a[1]) | ((uint32_t)f32x2_to_e4m3x2(a[2], a[3]) << 16);
    }
    qv[v] = make_uint2(w[0], w[1]);
  }
  if (blockIdx.x == 0) {
    for (int64_t i = nvec * 8 + threadIdx.x; i < n; i += blockDim.x)
      q[i] = f32_to_e4m3(__fdiv_rn(__bfloat162float(x[i]), s));
  }
}

// Device address of the scratch array, looked up once per device with that
// device current (in host code the symbol name is only a host-side stand-in).
static float* scratch_ptr(int* rc) {
  static std::mutex mu;
  static float* ptrs[64] = {nullptr};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    *rc = fail(FVB_ERR_CUDA, "fvb_quant_fp8_tensor_noalloc: cudaGetDevice: %s",
               cudaGetErrorString(e));
    return nullptr;
  }
  if (dev < 0 || dev >= 64) {
    *rc = fail(FVB_ERR_UNSUPPORTED, "fvb_quant_fp8_tensor_noalloc: device %d out of range", dev);
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!ptrs[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_partials);
    if (e != cudaSuccess || p == nullptr) {
      *rc = fail(FVB_ERR_CUDA, "fvb_quant_fp8_tensor_noalloc: cudaGetSymbolAddress: %s",
                 cudaGetErrorString(e));
      return nullptr;
    }
    ptrs[dev] = static_cast<float*>(p);
  }
  *rc = FVB_OK;
  return ptrs[dev];
}

}  // namespace noalloc
}  // namespace fvb

extern "C" int fvb_quant_fp8_tensor_noalloc(const void* x, int64_t M, int64_t K, void* q,
                                            float* scale_out, fvb_stream_t stream) {
  using namespace fvb;
  cudaStream_t st = (cudaStream_t)stream;
  FVB_REQUIRE(M >= 0 && K >= 0, "fvb_quant_fp8_tensor_noalloc: negative size");
  const int64_t max_n = (int64_t)noalloc::kMaxPartials * noalloc::kChunk;
  // reject before forming M * K, which could overflow int64 for huge sizes
  FVB_REQUIRE(K == 0 || M <= max_n / K,
              "fvb_quant_fp8_tensor_noalloc: %lld x %lld elements exceed the fixed scratch "
              "limit of %lld; use fvb_quant_fp8 with a workspace",
              (long long)M, (long long)K, (long long)max_n);
  const int64_t n = M * K;
  FVB_REQUIRE(n <= max_n,
              "fvb_quant_fp8_tensor_noalloc: %lld elements exceed the fixed scratch limit of "
              "%lld (%d partials x %lld elements); use fvb_quant_fp8 with a workspace",
              (long long)n, (long long)max_n, noalloc::kMaxPartials, (long long)noalloc::kChunk);
  FVB_REQUIRE(scale_out != nullptr, "fvb_quant_fp8_tensor_noalloc: scale_out is NULL");
  if (n == 0) {
    FVB_CUDA_TRY(cudaMemsetAsync(scale_out, 0, sizeof(float), st), "fvb_quant_fp8_tensor_noalloc");
    return FVB_OK;
  }
  FVB_REQUIRE(x && q, "fvb_quant_fp8_tensor_noalloc: NULL pointer");
  FVB_REQUIRE(aligned16(x) && (reinterpret_cast<uintptr_t>(q) & 7u) == 0,
              "fvb_quant_fp8_tensor_noalloc: x must be 16-byte and q 8-byte aligned");
  int rc = FVB_OK;
  float* partials = noalloc::scratch_ptr(&rc);
  if (!partials) return rc;
  const int nparts = (int)((n + noalloc::kChunk - 1) / noalloc::kChunk);
  noalloc::chunk_absmax_kernel<<<nparts, 256, 0, st>>>((const __nv_bfloat16*)x, n, partials);
  rc = check_launch("fvb_quant_fp8_tensor_noalloc");
  if (rc) return rc;
  int64_t blocks = ((n >> 3) + 255) / 256;
  const int64_t cap = (int64_t)sm_count() * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  noalloc::quant_from_partials_kernel<<<(unsigned)blocks, 256, 0, st>>>(
      (const __nv_bfloat16*)x, n, partials, nparts, (uint8_t*)q, scale_out);
  return check_launch("fvb_quant_fp8_tensor_noalloc");
}
