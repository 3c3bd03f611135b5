// Shared device/host helpers for the FlashVSR B200 operator pack (sm_100a only).
//
// Everything here is hand-written for Blackwell: mbarrier waits with an
// iteration limit, TMA tile loads (no multicast load anywhere in this
// library, since it also runs one process per GPU on 2-8 GPUs), and the
// tcgen05 tensor-memory / MMA instructions used by the GEMM and attention
// kernels.  Host helpers map CUDA errors to the library's status codes.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <stdint.h>
#include <stddef.h>

#include "../../include/flashvsr_b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "flashvsr_b200 is built for sm_100a only"
#endif

namespace fvb {

// ---------------------------------------------------------------------------
// host-side status plumbing
// ---------------------------------------------------------------------------
void set_error(const char* fmt, ...);
int fail(int code, const char* fmt, ...);
int check_launch(const char* what);

#define FVB_REQUIRE(cond, ...)                                   \
  do {                                                           \
    if (!(cond)) return ::fvb::fail(FVB_ERR_INVALID, __VA_ARGS__); \
  } while (0)

#define FVB_CUDA_TRY(expr, what)                                               \
  do {                                                                         \
    cudaError_t _e = (expr);                                                   \
    if (_e != cudaSuccess)                                                     \
      return ::fvb::fail(FVB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(_e)); \
  } while (0)

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int sm_count();  // cached multiprocessor count of the current device

// TMA descriptor creation through the driver entry point (no -lcuda needed).
// 2-D tensor: inner dimension `inner` elements (contiguous), `outer` rows with
// a row pitch of `row_bytes`.  Box = box_inner x box_outer elements.
int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes,
                 uint64_t inner, uint64_t outer, uint64_t row_bytes, uint32_t box_inner,
                 uint32_t box_outer, CUtensorMapSwizzle swizzle);

// Device-side error word: kernels that give up on a bounded wait record a code
// here; the host reads it back with fvb_device_error().  (The library is one
// translation unit, fvb_lib.cu, so this is its only definition.)
__device__ unsigned int g_device_error = 0;

// ---------------------------------------------------------------------------
// numeric helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float bf16r(float x) {  // round-trip through bf16 (RNE)
  return __bfloat162float(__float2bfloat16_rn(x));
}

// packed fp32x2 arithmetic (sm_100): two lanes of work per instruction
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1,%2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t r, float& a, float& b) {
  asm("mov.b64 {%0,%1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// fp32 -> e4m3 (round to nearest even, saturating to +-448): the rounding the
// reference gets from Triton's `.to(tl.float8e4nv)` after an explicit clamp.
__device__ __forceinline__ uint8_t f32_to_e4m3(float v) {
  return (uint8_t)__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3);
}

// two fp32 -> packed e4m3x2 (lo = a, hi = b)
__device__ __forceinline__ uint16_t f32x2_to_e4m3x2(float a, float b) {
  return (uint16_t)__nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
}

// GELU(tanh) of x (a bf16 value held in fp32), rounded to bf16: aten's formula
// 0.5f * x * (1.0f + tanhf(kBeta * (x + kKappa * x^3))) in fp32, rounded once (the
// rounding fp8_ffn.py:24-30 replicates).
__device__ __forceinline__ float gelu_tanh_bf16(float x) {
  const float kBeta = 0.7978845608028654f;  // sqrt(2/pi)
  const float kKappa = 0.044715f;
  const float x3 = x * x * x;
  const float inner = kBeta * __fmaf_rn(kKappa, x3, x);
  return bf16r(0.5f * x * (1.0f + tanhf(inner)));
}

// GELU(tanh) of a bf16 input through a shared-memory table.  The input is 16 bits, so the
// exact function (gelu_tanh_bf16) is tabulated for |x| in [2^-9, 16) = bf16 bit patterns
// [0x3B00, 0x4180), 1664 entries per sign (6.5 KB).  Outside the table: 0.5 x for |x| < 2^-9
// (1 + tanh u rounds to 1 within half a bf16 ulp), x for x >= 16 (tanh u is 1) and x * 0
// for x <= -16 (tanh u is -1; -0, or NaN for -inf).  Tests push every bf16 value through.
constexpr uint32_t kGeluLo = 0x3B00u;
constexpr uint32_t kGeluRange = 0x4180u - kGeluLo;
constexpr int kGeluTableBytes = (int)(2 * kGeluRange * 2);

__device__ __forceinline__ uint32_t bf16_bits_rn(float x) {
  return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(x));
}
// fill the table: thread t of the nthreads sharing the work
__device__ __forceinline__ void gelu_table_fill(uint16_t* lut, uint32_t t, uint32_t nthreads) {
  for (uint32_t i = t; i < 2 * kGeluRange; i += nthreads) {
    const uint32_t neg = i >= kGeluRange;
    const uint32_t h = (neg << 15) | (kGeluLo + i - neg * kGeluRange);
    lut[i] = (uint16_t)bf16_bits_rn(gelu_tanh_bf16(__uint_as_float(h << 16)));
  }
}
// bf16 bits of GELU(x) for the bf16 bit pattern h (low 16 bits)
__device__ __forceinline__ uint32_t gelu_bf16_bits(uint32_t h, const uint16_t* lut) {
  const uint32_t a = h & 0x7FFFu;
  const uint32_t k = a - kGeluLo;
  if (k < kGeluRange) return lut[(h >> 15) * kGeluRange + k];
  const float x = __uint_as_float(h << 16);
  return bf16_bits_rn(a < kGeluLo ? 0.5f * x : ((h & 0x8000u) ? x * 0.0f : x));
}
// bf16 bits of GELU(bf16(o))
__device__ __forceinline__ uint32_t gelu_bits(float o, const uint16_t* lut) {
  return gelu_bf16_bits(bf16_bits_rn(o), lut);
}

// The scale returned beside the codes, the reference's `amax / FP8_MAX` (fp8_quant.py:54,
// fp8_ffn.py:72) as torch evaluates it on a CUDA tensor: a division by a host scalar runs as
// a multiply by the scalar's fp32 reciprocal, fl(amax * fl(1/448)).  (Measured on a B200:
// the reference's returned scale equals this and differs from the IEEE quotient by one ulp
// for some amax.)  The scale the codes are divided by, max(amax, 1e-12) / 448, is an IEEE
// divide inside the reference's kernel and stays one here.
__device__ __forceinline__ float returned_scale(float amax) {
  return __fmul_rn(amax, 1.0f / 448.0f);
}

__device__ __noinline__ uint2 e4m3x8_exact(float f0, float f1, float f2, float f3, float f4,
                                           float f5, float f6, float f7, float s) {
  const uint32_t c0 = f32x2_to_e4m3x2(__fdiv_rn(f0, s), __fdiv_rn(f1, s));
  const uint32_t c1 = f32x2_to_e4m3x2(__fdiv_rn(f2, s), __fdiv_rn(f3, s));
  const uint32_t c2 = f32x2_to_e4m3x2(__fdiv_rn(f4, s), __fdiv_rn(f5, s));
  const uint32_t c3 = f32x2_to_e4m3x2(__fdiv_rn(f6, s), __fdiv_rn(f7, s));
  return make_uint2(c0 | (c1 << 16), c2 | (c3 << 16));
}

// 8 fp32 values -> 8 e4m3 codes of clamp(x / s, +-448), rounded to nearest even, packed in
// a uint2 (the quantisation of fp8_quant.py:16-35), without an IEEE divide in the common
// case.  rs = __frcp_rn(s), hoisted by the caller.  The saturating conversion is the clamp
// (finite values beyond +-448 go to +-448, NaN stays NaN as clamp-then-cast leaves it).
// x * rs(1 - 2^-20) and x * rs(1 + 2^-20), each rounded, bracket the IEEE quotient
// fl(x / s) (their relative distance from x / s exceeds 2^-21 after all roundings, the
// quotient's is at most 2^-24; below the fp32 normal range every value involved converts
// to a signed zero).  The conversion is monotone, so when both ends give the same code the
// quotient does too.  If any of the 8 values fails that test (a rounding boundary inside
// its bracket), all 8 take the exact divide (out of line: rare).
__device__ __forceinline__ uint2 e4m3_codes8(const float* f, float s, float rs) {
  const uint64_t lo2 = f2_pack(rs * 0.99999904632568359375f, rs * 0.99999904632568359375f);
  const uint64_t hi2 = f2_pack(rs * 1.00000095367431640625f, rs * 1.00000095367431640625f);
  uint32_t c[4];
  uint32_t diff = 0;  // OR of (lo ^ hi) over the pairs: one 3-input logic op per pair
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint64_t x2 = f2_pack(f[2 * i], f[2 * i + 1]);
    float a0, a1, b0, b1;
    f2_unpack(f2_mul(x2, lo2), a0, a1);
    f2_unpack(f2_mul(x2, hi2), b0, b1);
    const uint32_t lo = f32x2_to_e4m3x2(a0, a1), hi = f32x2_to_e4m3x2(b0, b1);
    diff |= lo ^ hi;
    c[i] = lo;
  }
  if (diff != 0) return e4m3x8_exact(f[0], f[1], f[2], f[3], f[4], f[5], f[6], f[7], s);
  return make_uint2(c[0] | (c[1] << 16), c[2] | (c[3] << 16));
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// atomic max on non-negative floats through their bit pattern (monotone for >= 0)
__device__ __forceinline__ void atomic_max_nonneg(float* addr, float v) {
  atomicMax(reinterpret_cast<unsigned int*>(addr), __float_as_uint(v));
}

// 16-byte read-only load of streamed data (read once: no L1 allocation)
__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// unpack 8 bf16 held in a uint4 into fp32
__device__ __forceinline__ void bf16x8_to_f32(const uint4& u, float* f) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
__device__ __forceinline__ uint4 f32_to_bf16x8(const float* f) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return u;
}

// ---------------------------------------------------------------------------
// row kernels (one warp per row of a row-major matrix)
// ---------------------------------------------------------------------------
// Rows are dealt to warps round-robin over a grid of at most 2 blocks per SM; each warp
// loads its next row while it works on the current one, so two rows per warp are in flight
// (one row per warp, load -> reduce -> store in series, left HBM idle between phases).
// Measured at the step's shapes: 2 blocks per SM 20.9 us for the FP8-only LN-modulate,
// 3 blocks 22.3 us, 4 blocks 27.3 us (register cap 64); the other row kernels within 1-2%.
constexpr int kRowBlocksPerSM = 2;

template <int NV, typename Load, typename Body>
__device__ __forceinline__ void row_pipeline(int64_t rows, Load load, Body body) {
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  uint4 cur[NV], nxt[NV];
  load(row, cur);
  for (; row < rows; row += nwarps) {
    if (row + nwarps < rows) load(row + nwarps, nxt);
    body(row, cur);
#pragma unroll
    for (int j = 0; j < NV; ++j) cur[j] = nxt[j];
  }
}

// The same schedule for rows that are combined from NL raw vectors per lane (e.g. a row
// and the residual added to it): prep(row, raw, cur) turns the arrived raw vectors into the
// row's NV working vectors before the next row's raw loads are issued into the same
// registers, so a lane holds NL + NV vectors instead of 2 * NL.
template <int NV, int NL, typename Load, typename Prep, typename Body>
__device__ __forceinline__ void row_pipeline_prep(int64_t rows, Load load, Prep prep, Body body) {
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  uint4 raw[NL], cur[NV];
  load(row, raw);
  for (; row < rows; row += nwarps) {
    prep(row, raw, cur);
    if (row + nwarps < rows) load(row + nwarps, raw);
    body(row, cur);
  }
}

// The schedule of row_pipeline_prep with the row held as fp32: prep(row, raw, f) turns the
// arrived raw vectors into the lane's NV * 8 fp32 values (unpacked once per row) before the
// next row's raw loads are issued into the same registers, so a lane holds 4 * NL + 8 * NV
// registers of row data.
template <int NV, int NL, typename Load, typename Prep, typename Body>
__device__ __forceinline__ void row_pipeline_f(int64_t rows, Load load, Prep prep, Body body) {
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  uint4 raw[NL];
  float f[NV * 8];
  load(row, raw);
  for (; row < rows; row += nwarps) {
    prep(row, raw, f);
    if (row + nwarps < rows) load(row + nwarps, raw);
    body(row, f);
  }
}

// ---------------------------------------------------------------------------
// shared-memory / mbarrier PTX
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16-byte global -> shared copy that bypasses registers (many in flight per thread);
// cp_async_wait_all() waits for this thread's copies, a barrier then publishes them.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)),
               "l"(gmem_src)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
          smem_u32(bar)),
      "r"(bytes)
      : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait: every spin in this library gives up after kWaitLimitNs of
// wall time (checked every 256 polls), records `code` in g_device_error and
// reports failure so the caller can unwind instead of hanging the GPU.  The
// longest legitimate wait (one K-loop of a tile, one key block of attention)
// is microseconds, so the limit only fires on a real fault.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
#pragma unroll 1
    for (int i = 0; i < 256; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > kWaitLimitNs) break;
  }
  atomicCAS(&g_device_error, 0u, code);
  return false;
}

// ---------------------------------------------------------------------------
// TMA (bulk tensor) loads/stores, CTA-local only
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
      "%4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int32_t x,
                                             int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tma_store_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void tma_store_wait_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void tma_store_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void tma_store_wait0() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: tensor memory, MMA, commit, loads
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Arrive on `bar` once every tcgen05.mma issued so far by this thread completes.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------------------
// CTA pairs (2-CTA clusters, tcgen05 cta_group::2).  One elected thread of the
// even CTA issues each MMA for both; every tile load stays a plain per-CTA TMA
// load into the issuing CTA's own shared memory, only its completion is counted
// on the even CTA's barrier.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// every thread of both CTAs; release/acquire orders shared-memory writes (barrier
// inits included) before the partner's accesses
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
// shared::cluster address of the same shared-memory offset in CTA `rank`
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ uint32_t ld_shared_cluster_u32(uint32_t caddr) {
  uint32_t v;
  asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(caddr) : "memory");
  return v;
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t caddr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(caddr)
               : "memory");
}
// tile load into this CTA's shared memory whose byte count completes on the barrier at
// shared::cluster address `bar_caddr` (this CTA's or its pair's)
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map,
                                                 uint32_t bar_caddr, int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_caddr), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
// arrive on `bar` (this CTA's) once every pair MMA issued so far by this thread completes
__device__ __forceinline__ void tc_commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}
// the same arrive on the barrier at this offset in every CTA of `cta_mask`
__device__ __forceinline__ void tc_commit_pair_both(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 "
      "[%0], %1;" ::"r"(smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}
// D (+)= A * B over a CTA pair: M = 256 rows, A's rows 0-127 and B's first N/2 rows from
// the even CTA's shared memory, the rest from its pair's at the same offsets; D rows
// 0-127 land in the even CTA's TMEM, rows 128-255 in its pair's, at the same address
__device__ __forceinline__ void mma_f8f6f4_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                                uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc], FP8 E4M3 inputs, fp32 accumulate
__device__ __forceinline__ void mma_f8f6f4(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc], bf16/f16 inputs, fp32 accumulate
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 lanes x 32 columns of 32-bit TMEM -> 32 registers per thread (thread i = lane i)
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 32 registers per thread -> 32 lanes x 32 columns of 32-bit TMEM (thread i = lane i)
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
      "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]),
      "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]),
      "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc], bf16/f16 inputs (A: one row per TMEM lane, two
// 16-bit K elements per 32-bit column), fp32 accumulate
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 2^x on the special-function unit (flush-to-zero; inputs here are <= 8)
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {  // sm_100 3-input max
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}


// Shared-memory matrix descriptor for a tcgen05 operand tile in the 128-byte
// swizzled canonical layout (8-row x 128-byte atoms, 1024-byte aligned base).
//   lbo/sbo in bytes: K-major -> lbo unused (16), sbo = 1024 (next 8-row group)
//                     MN-major -> lbo = byte distance between 64-element column
//                                 groups, sbo = 1024 (next 8 K-rows)
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo_bytes,
                                                    uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for sm_100
  d |= (uint64_t)2 << 61;  // SWIZZLE_128B
  return d;
}

// Instruction descriptor: fp32 accumulator, A/B format codes, majors, M x N.
__host__ __device__ constexpr uint32_t make_idesc(uint32_t a_fmt, uint32_t b_fmt, uint32_t a_mn_major,
                                                  uint32_t b_mn_major, uint32_t M, uint32_t N) {
  return (1u << 4)             // D format: f32
         | (a_fmt << 7) | (b_fmt << 10) | (a_mn_major << 15) | (b_mn_major << 16) |
         ((N >> 3) << 17) | ((M >> 4) << 24);
}

__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b32 r;\n\t"
      "elect.sync r|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

__device__ __forceinline__ int warp_id_uniform() {
  return __shfl_sync(0xffffffffu, (int)(threadIdx.x >> 5), 0);
}

}  // namespace fvb
