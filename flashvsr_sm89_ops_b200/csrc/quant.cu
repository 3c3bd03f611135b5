// FP8 E4M3 activation quantisation (a1), GELU(tanh)->FP8 (a5) and the
// quantise-with-known-amax pass of the FFN mid-section.
//
// Numerics follow flashvsr_sm89_ops/fp8_quant.py:25-35 and fp8_ffn.py:24-54:
//   s = max(amax, 1e-12) / 448   (fp32, IEEE divide)
//   q = e4m3_rn_satfinite(clamp(x / s, -448, 448))   (IEEE divide, never x * (1/s))
//   returned scale = amax / 448
// amax is order-independent, so codes and scales are bit-exact against any
// correct implementation of the same formula.
//
// Layout: x [M, K] bf16 row-major.  Per-token mode gives each row its own
// scale; rows are handled one warp each with 16-byte vector loads, the row
// held in registers when K <= 2048 and re-read from L1/L2 otherwise.
#include <type_traits>

#include "common.cuh"

namespace fvb {

constexpr float kFp8Max = 448.0f;

__device__ __forceinline__ float quant_scale_from_amax(float amax) {
  return __fdiv_rn(fmaxf(amax, 1e-12f), kFp8Max);
}

__device__ __forceinline__ uint2 quant8(const float* f, float s, float rs) {
  return e4m3_codes8(f, s, rs);
}

template <bool GELU>
__device__ __forceinline__ void load8(const uint4* src, int64_t v, float* f) {
  uint4 u = __ldg(src + v);
  bf16x8_to_f32(u, f);
  if (GELU) {
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = gelu_tanh_bf16(f[i]);
  }
}

// ---------------------------------------------------------------------------
// per-tensor: pass 1 = global amax (atomic max on the bit pattern), pass 2 = quantise
// ---------------------------------------------------------------------------
template <bool GELU>
__global__ void __launch_bounds__(256) absmax_kernel(const uint4* __restrict__ x, int64_t nvec,
                                                      const __nv_bfloat16* __restrict__ xs,
                                                      int64_t n, float* __restrict__ amax) {
  float m = 0.f;
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < nvec;
       v += (int64_t)gridDim.x * blockDim.x) {
    float f[8];
    load8<GELU>(x, v, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) m = fmaxf(m, fabsf(f[i]));
  }
  // scalar tail (n % 8)
  if (blockIdx.x == 0) {
    for (int64_t i = nvec * 8 + threadIdx.x; i < n; i += blockDim.x) {
      float f = __bfloat162float(xs[i]);
      if (GELU) f = gelu_tanh_bf16(f);
      m = fmaxf(m, fabsf(f));
    }
  }
  m = warp_max(m);
  __shared__ float red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_max(t);
    if (threadIdx.x == 0) atomic_max_nonneg(amax, t);
  }
}

template <bool GELU>
__global__ void __launch_bounds__(256) quant_tensor_kernel(
    const uint4* __restrict__ x, int64_t nvec, const __nv_bfloat16* __restrict__ xs, int64_t n,
    const float* __restrict__ amax_p, uint2* __restrict__ q, uint8_t* __restrict__ qs,
    float* __restrict__ scale_out) {
  const float amax = *amax_p;
  const float s = quant_scale_from_amax(amax);
  const float rs = __frcp_rn(s);
  if (blockIdx.x == 0 && threadIdx.x == 0) scale_out[0] = returned_scale(amax);
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < nvec;
       v += (int64_t)gridDim.x * blockDim.x) {
    float f[8];
    load8<GELU>(x, v, f);
    q[v] = quant8(f, s, rs);
  }
  if (blockIdx.x == 0) {
    for (int64_t i = nvec * 8 + threadIdx.x; i < n; i += blockDim.x) {
      float f = __bfloat162float(xs[i]);
      if (GELU) f = gelu_tanh_bf16(f);
      qs[i] = f32_to_e4m3(__fdiv_rn(f, s));  // saturating == clamp
    }
  }
}

// ---------------------------------------------------------------------------
// per-tensor GELU -> e4m3 (fused_gelu_quant_fp8's default mode) in three launches:
//   1. the raw maximum of h (no GELU); block 0 also evaluates GELU on every bf16 input of the
//      table range to get neg_max (the largest |GELU| of a negative input) and to check that
//      GELU is non-decreasing on the positive ones;
//   2. amax = GELU(max h) when max h > 0, GELU(max h) >= neg_max and the check held (GELU is
//      non-decreasing for x >= 0 and every negative input's |GELU| is at most neg_max);
//      otherwise every block takes GELU of its elements and the exact amax is reduced;
//   3. quantise, GELU through the block's shared table.
// Workspace (floats): [0] amax, [1] max h as an order-preserving uint32 key, [2] neg_max,
// [3] nonzero when the check failed.  NaN inputs are dropped from the maxima like fmaxf.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float order_key_value(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

__global__ void __launch_bounds__(256) gelu_rawmax_kernel(const uint4* __restrict__ x, int64_t nvec,
                                                          const __nv_bfloat16* __restrict__ xs,
                                                          int64_t n, float* __restrict__ ws) {
  float m = -INFINITY;
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < nvec;
       v += (int64_t)gridDim.x * blockDim.x) {
    float f[8];
    bf16x8_to_f32(__ldg(x + v), f);
#pragma unroll
    for (int i = 0; i < 8; ++i) m = fmaxf(m, f[i]);
  }
  if (blockIdx.x == 0) {
    for (int64_t i = nvec * 8 + threadIdx.x; i < n; i += blockDim.x)
      m = fmaxf(m, __bfloat162float(xs[i]));
    // the table range, both signs: neg_max and the positive side's order
    float nm = 0.f;
    uint32_t bad = 0u;
    for (uint32_t i = threadIdx.x; i < kGeluRange; i += blockDim.x) {
      const float xn = __uint_as_float((0x8000u | (kGeluLo + i)) << 16);
      nm = fmaxf(nm, fabsf(gelu_tanh_bf16(xn)));
      const float xp = __uint_as_float((kGeluLo + i) << 16);
      const float xp1 = __uint_as_float((kGeluLo + i + 1u) << 16);  // i + 1 == range: x = 16
      const float gp1 = i + 1u < kGeluRange ? gelu_tanh_bf16(xp1) : xp1;
      if (gelu_tanh_bf16(xp) > gp1) bad = 1u;
    }
    nm = warp_max(nm);
    if ((threadIdx.x & 31) == 0) atomic_max_nonneg(ws + 2, nm);
    if (bad) atomicOr(reinterpret_cast<unsigned int*>(ws + 3), 1u);
  }
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0 && m == m)
    atomicMax(reinterpret_cast<unsigned int*>(ws + 1), order_key(m));
}

__global__ void __launch_bounds__(256) gelu_amax_kernel(const uint4* __restrict__ x, int64_t nvec,
                                                        const __nv_bfloat16* __restrict__ xs,
                                                        int64_t n, float* __restrict__ ws) {
  const uint32_t key = *reinterpret_cast<const volatile uint32_t*>(ws + 1);
  const float xmax = key ? order_key_value(key) : -INFINITY;
  const float g = gelu_tanh_bf16(xmax);
  const bool bad = *reinterpret_cast<const volatile uint32_t*>(ws + 3) != 0u;
  if (!bad && xmax > 0.f && g >= ws[2]) {  // the shortcut holds (g may be +inf)
    if (blockIdx.x == 0 && threadIdx.x == 0) ws[0] = g;
    return;
  }
  // exact: |GELU| of every element
  float m = 0.f;
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < nvec;
       v += (int64_t)gridDim.x * blockDim.x) {
    float f[8];
    load8<true>(x, v, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) m = fmaxf(m, fabsf(f[i]));
  }
  if (blockIdx.x == 0)
    for (int64_t i = nvec * 8 + threadIdx.x; i < n; i += blockDim.x)
      m = fmaxf(m, fabsf(gelu_tanh_bf16(__bfloat162float(xs[i]))));
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) atomic_max_nonneg(ws, m);
}

__global__ void __launch_bounds__(256) gelu_quant_tensor_kernel(
    const uint4* __restrict__ x, int64_t nvec, const __nv_bfloat16* __restrict__ xs, int64_t n,
    const float* __restrict__ amax_p, uint2* __restrict__ q, uint8_t* __restrict__ qs,
    float* __restrict__ scale_out) {
  __shared__ uint16_t lut[2 * kGeluRange];
  gelu_table_fill(lut, threadIdx.x, blockDim.x);
  __syncthreads();
  const float amax = *amax_p;
  const float s = quant_scale_from_amax(amax);
  const float rs = __frcp_rn(s);
  if (blockIdx.x == 0 && threadIdx.x == 0) scale_out[0] = returned_scale(amax);
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < nvec;
       v += (int64_t)gridDim.x * blockDim.x) {
    const uint4 u = __ldg(x + v);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
    float f[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(gelu_bf16_bits(w[i] & 0xFFFFu, lut) << 16);
      f[2 * i + 1] = __uint_as_float(gelu_bf16_bits(w[i] >> 16, lut) << 16);
    }
    q[v] = quant8(f, s, rs);
  }
  if (blockIdx.x == 0)
    for (int64_t i = nvec * 8 + threadIdx.x; i < n; i += blockDim.x)
      qs[i] = f32_to_e4m3(__fdiv_rn(gelu_tanh_bf16(__bfloat162float(xs[i])), s));
}

// ---------------------------------------------------------------------------
// per-token: one warp per row
// ---------------------------------------------------------------------------
// K <= 2048: the row lives in registers (NV 16-byte vectors per lane), two rows per warp in
// flight (row_pipeline).  GELU values are bf16-rounded, so they are stored back into the
// row's bf16 registers losslessly between the amax and the quantisation passes.
template <bool GELU, int NV>
__global__ void __launch_bounds__(256, kRowBlocksPerSM) quant_row_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t M, int64_t K, uint8_t* __restrict__ q,
    float* __restrict__ scale_out) {
  const int lane = threadIdx.x & 31;
  const int nvec = (int)(K >> 3);  // K % 8 == 0 enforced by the host
  auto load = [&](int64_t row, uint4* xr) {
    const uint4* xv = reinterpret_cast<const uint4*>(x + row * K);
#pragma unroll
    for (int j = 0; j < NV; ++j)
      if (j * 32 + lane < nvec) xr[j] = __ldg(xv + j * 32 + lane);
  };
  auto body = [&](int64_t row, uint4* xr) {
    float m = 0.f;
    // the plain row's amax on packed bf16 pairs (|x| and max are exact on bf16 values;
    // __hmax2 drops a NaN operand like fmaxf)
    __nv_bfloat162 m2 = __float2bfloat162_rn(0.0f);
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      if (j * 32 + lane < nvec) {
        if (GELU) {
          float f[8];
          bf16x8_to_f32(xr[j], f);
#pragma unroll
          for (int i = 0; i < 8; ++i) f[i] = gelu_tanh_bf16(f[i]);
          xr[j] = f32_to_bf16x8(f);
#pragma unroll
          for (int i = 0; i < 8; ++i) m = fmaxf(m, fabsf(f[i]));
        } else {
          const __nv_bfloat162* x2 = reinterpret_cast<const __nv_bfloat162*>(&xr[j]);
#pragma unroll
          for (int p = 0; p < 4; ++p) m2 = __hmax2(m2, __habs2(x2[p]));
        }
      }
    }
    if (!GELU) {
      const float2 mf = __bfloat1622float2(m2);
      m = fmaxf(mf.x, mf.y);
    }
    m = warp_max(m);
    const float s = quant_scale_from_amax(m);
    const float rs = __frcp_rn(s);
    uint2* qv = reinterpret_cast<uint2*>(q + row * K);
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      if (j * 32 + lane < nvec) {
        float f[8];
        bf16x8_to_f32(xr[j], f);
        qv[j * 32 + lane] = quant8(f, s, rs);
      }
    }
    if (lane == 0) scale_out[row] = returned_scale(m);
  };
  row_pipeline<NV>(M, load, body);
}

// K > 2048: the row is read twice (amax, then quantise), the second pass from L1/L2.
// One warp per row, rows strided over a persistent grid.  GELU (GELU(tanh) -> e4m3 of
// fp8_ffn.py:57-72) goes through the block's shared table of the exact function of the
// 16-bit input (gelu_bf16_bits), built once per block.
// GELU's row amax without GELU in the first pass: GELU rounded to bf16 is non-decreasing
// for x >= 0 (checked on the block's table; if it were not, every row takes the exact pass),
// and every negative input has |GELU(x)| <= neg_max, the largest negative-half entry of the
// table (~0.17, at x ~ -0.75; inputs outside the table give |GELU| < 2^-10).  So when
// GELU(row max) >= neg_max, the amax of |GELU| over the row is GELU(row max), and the first
// pass is a packed bf16 max of the raw row; otherwise the row takes the exact pass (GELU of
// every element).  NaN inputs are dropped from the amax either way, like fmaxf.
template <bool GELU>
__device__ __forceinline__ void load8_lut(const uint4* src, int64_t v, const uint16_t* lut,
                                          float* f) {
  uint4 u = __ldg(src + v);
  if (GELU) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(gelu_bf16_bits(w[i] & 0xFFFFu, lut) << 16);
      f[2 * i + 1] = __uint_as_float(gelu_bf16_bits(w[i] >> 16, lut) << 16);
    }
  } else {
    bf16x8_to_f32(u, f);
  }
}

template <bool GELU>
__global__ void __launch_bounds__(256) quant_row_long_kernel(const __nv_bfloat16* __restrict__ x,
                                                             int64_t M, int64_t K,
                                                             uint8_t* __restrict__ q,
                                                             float* __restrict__ scale_out) {
  __shared__ uint16_t lut[GELU ? 2 * kGeluRange : 1];
  __shared__ uint32_t neg_max, not_mono;
  if (GELU) {
    if (threadIdx.x == 0) neg_max = not_mono = 0u;
    gelu_table_fill(lut, threadIdx.x, blockDim.x);
    __syncthreads();
    uint32_t nm = 0u, bad = 0u;
    for (uint32_t i = threadIdx.x; i < kGeluRange; i += blockDim.x) {
      nm = max(nm, (uint32_t)lut[kGeluRange + i] & 0x7FFFu);
      if (i + 1 < kGeluRange && lut[i + 1] < lut[i]) bad = 1u;  // positive half, ascending x
    }
    // the table's ends meet the rules outside it: 0.5 x below, x above
    if (threadIdx.x == 0 && (lut[0] < bf16_bits_rn(0.5f * __uint_as_float((kGeluLo - 1u) << 16)) ||
                             lut[kGeluRange - 1] > kGeluLo + kGeluRange))
      bad = 1u;
    if (nm) atomicMax(&neg_max, nm);
    if (bad) atomicOr(&not_mono, 1u);
    __syncthreads();
  }
  const int lane = threadIdx.x & 31;
  const int64_t nvec = K >> 3;
  for (int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < M;
       row += (int64_t)gridDim.x * (blockDim.x >> 5)) {
    const uint4* xv = reinterpret_cast<const uint4*>(x + row * K);
    uint2* qv = reinterpret_cast<uint2*>(q + row * K);
    float m = 0.f;
    bool exact = true;
    if (GELU && not_mono == 0u) {
      // packed bf16 max of the raw row (__hmax2 drops a NaN operand)
      __nv_bfloat162 mx2 = __halves2bfloat162(__ushort_as_bfloat16((unsigned short)0xFF80u),
                                               __ushort_as_bfloat16((unsigned short)0xFF80u));
      for (int64_t v = lane; v < nvec; v += 32) {
        const uint4 u = __ldg(xv + v);
        const __nv_bfloat162* x2 = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int p = 0; p < 4; ++p) mx2 = __hmax2(mx2, x2[p]);
      }
      const float2 mf = __bfloat1622float2(mx2);
      const float xmax = warp_max(fmaxf(mf.x, mf.y));
      const uint32_t gb = gelu_bf16_bits(bf16_bits_rn(xmax), lut);
      if (xmax > 0.f && (gb & 0x7FFFu) >= neg_max && (gb & 0x7FFFu) <= 0x7F80u) {
        m = __uint_as_float(gb << 16);
        exact = false;
      }
    }
    if (exact) {
      for (int64_t v = lane; v < nvec; v += 32) {
        float f[8];
        load8_lut<GELU>(xv, v, lut, f);
#pragma unroll
        for (int i = 0; i < 8; ++i) m = fmaxf(m, fabsf(f[i]));
      }
      m = warp_max(m);
    }
    const float s = quant_scale_from_amax(m);
    const float rs = __frcp_rn(s);
    for (int64_t v = lane; v < nvec; v += 32) {
      float f[8];
      load8_lut<GELU>(xv, v, lut, f);
      qv[v] = quant8(f, s, rs);
    }
    if (lane == 0) scale_out[row] = returned_scale(m);
  }
}

// Quantisation with a precomputed amax (the second half of fused_gelu_quant_fp8,
// fp8_ffn.py:57-72, once the GEMM epilogue has reduced the row amax).  One warp per row:
// the scale and its reciprocal are computed once per row, and each lane keeps four
// 16-byte loads in flight; one resident wave of 4 blocks of 8 warps per SM (measured at
// the FFN hidden: 4 loads 54.3 us, 6 loads 56.1 us, 8 loads 58.0 us, 10-12 loads with
// fewer blocks 66-70 us).  (A flat grid-stride
// loop over the whole matrix spent more time in its 64-bit row = v / (K/8) divides than
// in memory; a block per row left most threads idle in the row's tail.)
constexpr int kQaUnroll = 4;
__global__ void __launch_bounds__(256, 4) quant_with_amax_kernel(
    const uint4* __restrict__ g, int64_t M, int64_t K, const float* __restrict__ amax, int per_row,
    uint2* __restrict__ q, float* __restrict__ scale_out) {
  const int kv = (int)(K >> 3);  // vectors per row (K / 8 < 2^31 enforced by the host)
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = (int64_t)gridDim.x * 8;
  for (int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5); row < M; row += nwarps) {
    const float a = __ldg(amax + (per_row ? row : 0));
    const float s = quant_scale_from_amax(a);
    const float rs = __frcp_rn(s);
    if (lane == 0 && (per_row || row == 0)) scale_out[per_row ? row : 0] = returned_scale(a);
    const uint4* gr = g + row * kv;
    uint2* qr = q + row * kv;
    int v = lane;
    for (; v + (kQaUnroll - 1) * 32 < kv; v += kQaUnroll * 32) {
      uint4 u[kQaUnroll];
#pragma unroll
      for (int t = 0; t < kQaUnroll; ++t) u[t] = ld_stream(gr + v + t * 32);
#pragma unroll
      for (int t = 0; t < kQaUnroll; ++t) {
        float f[8];
        bf16x8_to_f32(u[t], f);
        qr[v + t * 32] = quant8(f, s, rs);
      }
    }
    if (v < kv) {  // the row's tail: fewer than kQaUnroll vectors per lane
      uint4 u[kQaUnroll];
#pragma unroll
      for (int t = 0; t < kQaUnroll; ++t)
        if (v + t * 32 < kv) u[t] = ld_stream(gr + v + t * 32);
#pragma unroll
      for (int t = 0; t < kQaUnroll; ++t) {
        if (v + t * 32 < kv) {
          float f[8];
          bf16x8_to_f32(u[t], f);
          qr[v + t * 32] = quant8(f, s, rs);
        }
      }
    }
  }
}

static int grid_for(int64_t nvec, int threads) {
  int64_t blocks = (nvec + threads - 1) / threads;
  int64_t cap = (int64_t)sm_count() * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return (int)blocks;
}

template <bool GELU>
static int quant_impl(const void* x, int64_t M, int64_t K, void* q, float* scale_out, int mode,
                      void* workspace, cudaStream_t st, const char* name) {
  FVB_REQUIRE(M >= 0 && K >= 0, "%s: negative size", name);
  FVB_REQUIRE(mode == FVB_SCALE_TENSOR || mode == FVB_SCALE_ROW, "%s: bad mode %d", name, mode);
  FVB_REQUIRE(scale_out != nullptr, "%s: scale_out is NULL", name);
  const int64_t n = M * K;
  if (n == 0) {
    // reference: empty input -> empty codes and a zero scale (fp8_quant.py:45-47)
    int64_t ns = (mode == FVB_SCALE_ROW) ? M : 1;
    if (ns > 0) FVB_CUDA_TRY(cudaMemsetAsync(scale_out, 0, ns * sizeof(float), st), name);
    return FVB_OK;
  }
  FVB_REQUIRE(x && q, "%s: NULL pointer", name);
  FVB_REQUIRE(aligned16(x), "%s: x not 16-byte aligned", name);
  if (mode == FVB_SCALE_ROW) {
    FVB_REQUIRE(K % 8 == 0, "%s: per-token mode needs K %% 8 == 0 (K=%lld)", name, (long long)K);
    FVB_REQUIRE((reinterpret_cast<uintptr_t>(q) & 7u) == 0, "%s: q not 8-byte aligned", name);
    const int64_t need = (M + 7) / 8;
    if (K <= 2048) {
      const int64_t cap = (int64_t)sm_count() * kRowBlocksPerSM;
      const unsigned grid = (unsigned)(need < cap ? need : cap);
      auto launch = [&](auto nv) {
        quant_row_kernel<GELU, decltype(nv)::value><<<grid, 256, 0, st>>>(
            (const __nv_bfloat16*)x, M, K, (uint8_t*)q, scale_out);
      };
      if (K <= 512) launch(std::integral_constant<int, 2>{});
      else if (K <= 1024) launch(std::integral_constant<int, 4>{});
      else if (K <= 1536) launch(std::integral_constant<int, 6>{});
      else launch(std::integral_constant<int, 8>{});
    } else {
      const int64_t cap = (int64_t)sm_count() * 8;
      quant_row_long_kernel<GELU><<<(unsigned)(need < cap ? need : cap), 256, 0, st>>>(
          (const __nv_bfloat16*)x, M, K, (uint8_t*)q, scale_out);
    }
    return check_launch(name);
  }
  FVB_REQUIRE(workspace != nullptr, "%s: per-tensor mode needs a workspace", name);
  FVB_REQUIRE((reinterpret_cast<uintptr_t>(q) & 7u) == 0, "%s: q not 8-byte aligned", name);
  float* amax = static_cast<float*>(workspace);
  FVB_CUDA_TRY(cudaMemsetAsync(amax, 0, (GELU ? 4 : 1) * sizeof(float), st), name);
  const int64_t nvec = n >> 3;
  const int g = grid_for(nvec > 0 ? nvec : 1, 256);
  if constexpr (GELU) {
    gelu_rawmax_kernel<<<g, 256, 0, st>>>((const uint4*)x, nvec, (const __nv_bfloat16*)x, n, amax);
    int rc = check_launch(name);
    if (rc) return rc;
    gelu_amax_kernel<<<g, 256, 0, st>>>((const uint4*)x, nvec, (const __nv_bfloat16*)x, n, amax);
    rc = check_launch(name);
    if (rc) return rc;
    const int64_t cap = (int64_t)sm_count() * 4;
    gelu_quant_tensor_kernel<<<(unsigned)(g < cap ? g : cap), 256, 0, st>>>(
        (const uint4*)x, nvec, (const __nv_bfloat16*)x, n, amax, (uint2*)q, (uint8_t*)q,
        scale_out);
    return check_launch(name);
  } else {
    absmax_kernel<GELU><<<g, 256, 0, st>>>((const uint4*)x, nvec, (const __nv_bfloat16*)x, n,
                                           amax);
    int rc = check_launch(name);
    if (rc) return rc;
    quant_tensor_kernel<GELU><<<g, 256, 0, st>>>((const uint4*)x, nvec, (const __nv_bfloat16*)x, n,
                                                 amax, (uint2*)q, (uint8_t*)q, scale_out);
    return check_launch(name);
  }
}

}  // namespace fvb

extern "C" {

size_t fvb_quant_fp8_workspace_bytes(int64_t M, int64_t K, int mode) {
  (void)M;
  (void)K;
  return mode == FVB_SCALE_TENSOR ? 256 : 0;
}

int fvb_quant_fp8(const void* x, int64_t M, int64_t K, void* q, float* scale_out, int mode,
                  void* workspace, fvb_stream_t stream) {
  return fvb::quant_impl<false>(x, M, K, q, scale_out, mode, workspace, (cudaStream_t)stream,
                                "fvb_quant_fp8");
}

int fvb_gelu_quant_fp8(const void* h, int64_t M, int64_t K, void* q, float* scale_out, int mode,
                       void* workspace, fvb_stream_t stream) {
  return fvb::quant_impl<true>(h, M, K, q, scale_out, mode, workspace, (cudaStream_t)stream,
                               "fvb_gelu_quant_fp8");
}

int fvb_quant_fp8_with_amax(const void* g, int64_t M, int64_t K, const float* amax, int mode,
                            void* q, float* scale_out, fvb_stream_t stream) {
  using namespace fvb;
  FVB_REQUIRE(M >= 0 && K >= 0, "fvb_quant_fp8_with_amax: negative size");
  FVB_REQUIRE(mode == FVB_SCALE_TENSOR || mode == FVB_SCALE_ROW, "fvb_quant_fp8_with_amax: mode");
  if (M * K == 0) return FVB_OK;
  FVB_REQUIRE(g && amax && q && scale_out, "fvb_quant_fp8_with_amax: NULL pointer");
  FVB_REQUIRE(K % 8 == 0, "fvb_quant_fp8_with_amax: K %% 8 != 0");
  FVB_REQUIRE(aligned16(g) && (reinterpret_cast<uintptr_t>(q) & 7u) == 0,
              "fvb_quant_fp8_with_amax: misaligned pointer");
  FVB_REQUIRE(K / 8 <= 0x7fffffff, "fvb_quant_fp8_with_amax: row too long");
  const int64_t blocks = (M + 7) / 8, cap = (int64_t)sm_count() * 4;
  quant_with_amax_kernel<<<(unsigned)(blocks < cap ? blocks : cap), 256, 0, (cudaStream_t)stream>>>(
      (const uint4*)g, M, K, amax, mode == FVB_SCALE_ROW, (uint2*)q, scale_out);
  return check_launch("fvb_quant_fp8_with_amax");
}

}  // extern "C"
