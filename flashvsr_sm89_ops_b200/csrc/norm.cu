// Row-wise memory-bound kernels of the DiT block: LayerNorm + AdaLN modulate
// (a8, optionally emitting the per-token FP8 codes the next linear consumes),
// affine LayerNorm (the block's norm3), gated residual add (a9) and
// RMSNorm + interleaved 3-D RoPE (a7).
//
// One warp owns one row of D bf16 (D % 8 == 0, D <= 2048): lane l holds the
// 16-byte vectors l, l+32, ... in registers, so every row is read from HBM
// once and written once; reductions are warp shuffles.  For D = 1536 that is
// 6 vectors per lane and a fully coalesced 512-byte access per instruction.
//
// Rounding chains replicate the reference kernels exactly:
//   fused_adaln.py:29-41  xn = bf16((x-mean)/sqrt(var+eps));
//                          y = bf16(bf16(xn * bf16(1+scale)) + shift)
//   fused_adaln.py:53-57  out = bf16(x + bf16(g * r))
//   fused_rms_rope.py:34-53  y = bf16(x * rsqrt(mean(x^2)+eps)) * w (fp32),
//                          even: y_e c - y_o s, odd: y_o c + y_e s, one bf16 rounding
#include "common.cuh"

namespace fvb {

constexpr int kRowNV = 8;  // vectors per lane -> D <= 8 * 8 * 32 = 2048

__device__ __forceinline__ float quant_scale_from_amax_n(float amax) {
  return __fdiv_rn(fmaxf(amax, 1e-12f), 448.0f);
}

template <bool EMIT_FP8>
__global__ void __launch_bounds__(256) ln_modulate_kernel(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ scale,
    const __nv_bfloat16* __restrict__ shift, int64_t rows, int64_t L, int D, float eps,
    __nv_bfloat16* __restrict__ out, uint8_t* __restrict__ q8, float* __restrict__ q_scale) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int nvec = D >> 3;
  const uint4* xv = reinterpret_cast<const uint4*>(x + row * D);
  float f[kRowNV][8];
  float sum = 0.f;
#pragma unroll
  for (int j = 0; j < kRowNV; ++j) {
    int v = j * 32 + lane;
    if (v < nvec) {
      bf16x8_to_f32(__ldg(xv + v), f[j]);
#pragma unroll
      for (int i = 0; i < 8; ++i) sum += f[j][i];
    }
  }
  const float mean = __fdiv_rn(warp_sum(sum), (float)D);
  float sq = 0.f;
#pragma unroll
  for (int j = 0; j < kRowNV; ++j) {
    int v = j * 32 + lane;
    if (v < nvec) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float d = f[j][i] - mean;
        sq = __fmaf_rn(d, d, sq);
      }
    }
  }
  const float var = __fdiv_rn(warp_sum(sq), (float)D);
  // (x - mean) / sqrt(var + eps) as a product with the correctly rounded reciprocal square
  // root: at most one fp32 ulp from the quotient, well inside the bf16 rounding that follows
  const float rden = __frsqrt_rn(var + eps);
  const int64_t b = row / L;
  const uint4* sv = reinterpret_cast<const uint4*>(scale + b * D);
  const uint4* hv = reinterpret_cast<const uint4*>(shift + b * D);
  uint4* ov = reinterpret_cast<uint4*>(out + row * D);
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < kRowNV; ++j) {
    int v = j * 32 + lane;
    if (v < nvec) {
      float s[8], h[8];
      bf16x8_to_f32(__ldg(sv + v), s);
      bf16x8_to_f32(__ldg(hv + v), h);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float xn = bf16r((f[j][i] - mean) * rden);
        float y = bf16r(xn * bf16r(1.0f + s[i]));
        y = bf16r(y + h[i]);
        f[j][i] = y;
        amax = fmaxf(amax, fabsf(y));
      }
      ov[v] = f32_to_bf16x8(f[j]);
    }
  }
  if (EMIT_FP8) {
    amax = warp_max(amax);
    const float qs = quant_scale_from_amax_n(amax);
    const float rqs = __frcp_rn(qs);
    uint2* qv = reinterpret_cast<uint2*>(q8 + row * D);
#pragma unroll
    for (int j = 0; j < kRowNV; ++j) {
      int v = j * 32 + lane;
      if (v < nvec) {
        uint32_t w[2];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          float a0 = fminf(fmaxf(div_for_e4m3(f[j][4 * hh + 0], qs, rqs), -448.f), 448.f);
          float a1 = fminf(fmaxf(div_for_e4m3(f[j][4 * hh + 1], qs, rqs), -448.f), 448.f);
          float a2 = fminf(fmaxf(div_for_e4m3(f[j][4 * hh + 2], qs, rqs), -448.f), 448.f);
          float a3 = fminf(fmaxf(div_for_e4m3(f[j][4 * hh + 3], qs, rqs), -448.f), 448.f);
          w[hh] = (uint32_t)f32x2_to_e4m3x2(a0, a1) | ((uint32_t)f32x2_to_e4m3x2(a2, a3) << 16);
        }
        qv[v] = make_uint2(w[0], w[1]);
      }
    }
    if (lane == 0) q_scale[row] = __fdiv_rn(amax, 448.0f);
  }
}

// LayerNorm with optional affine weight / bias, fp32 math and one bf16 rounding
// (the semantics of torch.nn.LayerNorm on bf16 tensors).
__global__ void __launch_bounds__(256) layer_norm_kernel(const __nv_bfloat16* __restrict__ x,
                                                          const __nv_bfloat16* __restrict__ w,
                                                          const __nv_bfloat16* __restrict__ bias,
                                                          int64_t rows, int D, float eps,
                                                          __nv_bfloat16* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int nvec = D >> 3;
  const uint4* xv = reinterpret_cast<const uint4*>(x + row * D);
  float f[kRowNV][8];
  float sum = 0.f;
#pragma unroll
  for (int j = 0; j < kRowNV; ++j) {
    int v = j * 32 + lane;
    if (v < nvec) {
      bf16x8_to_f32(__ldg(xv + v), f[j]);
#pragma unroll
      for (int i = 0; i < 8; ++i) sum += f[j][i];
    }
  }
  const float mean = __fdiv_rn(warp_sum(sum), (float)D);
  float sq = 0.f;
#pragma unroll
  for (int j = 0; j < kRowNV; ++j) {
    int v = j * 32 + lane;
    if (v < nvec) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float d = f[j][i] - mean;
        sq = __fmaf_rn(d, d, sq);
      }
    }
  }
  const float rstd = __frsqrt_rn(__fdiv_rn(warp_sum(sq), (float)D) + eps);
  uint4* ov = reinterpret_cast<uint4*>(out + row * D);
#pragma unroll
  for (int j = 0; j < kRowNV; ++j) {
    int v = j * 32 + lane;
    if (v < nvec) {
      float ww[8], bb[8];
      if (w) bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(w) + v), ww);
      if (bias) bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(bias) + v), bb);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float y = (f[j][i] - mean) * rstd;
        if (w) y = y * ww[i];
        if (bias) y = y + bb[i];
        f[j][i] = y;
      }
      ov[v] = f32_to_bf16x8(f[j]);
    }
  }
}

__global__ void __launch_bounds__(256) gate_add_kernel(const uint4* __restrict__ x,
                                                        const __nv_bfloat16* __restrict__ gate,
                                                        const uint4* __restrict__ r, int64_t nvec,
                                                        int64_t LD, int D, uint4* __restrict__ out) {
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < nvec;
       v += (int64_t)gridDim.x * blockDim.x) {
    float xf[8], rf[8];
    bf16x8_to_f32(__ldg(x + v), xf);
    bf16x8_to_f32(__ldg(r + v), rf);
    if (gate) {
      const int64_t idx = v * 8;
      const int64_t p = (idx / LD) * D + (idx % D);  // gate is [B, 1, D]
      float gf[8];
      bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(gate + p)), gf);
#pragma unroll
      for (int i = 0; i < 8; ++i) xf[i] = xf[i] + bf16r(gf[i] * rf[i]);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) xf[i] = xf[i] + rf[i];
    }
    out[v] = f32_to_bf16x8(xf);
  }
}

template <bool ROPE>
__global__ void __launch_bounds__(256) rms_rope_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t x_ld, const __nv_bfloat16* __restrict__ w,
    const float* __restrict__ cosv, const float* __restrict__ sinv, int64_t rows, int64_t L,
    int D, int head_dim, float eps, const int32_t* __restrict__ row_map,
    __nv_bfloat16* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int nvec = D >> 3;
  const uint4* xv = reinterpret_cast<const uint4*>(x + row * x_ld);
  float f[kRowNV][8];
  float sq = 0.f;
#pragma unroll
  for (int j = 0; j < kRowNV; ++j) {
    int v = j * 32 + lane;
    if (v < nvec) {
      bf16x8_to_f32(__ldg(xv + v), f[j]);
#pragma unroll
      for (int i = 0; i < 8; ++i) sq = __fmaf_rn(f[j][i], f[j][i], sq);
    }
  }
  const float rrms = __frsqrt_rn(__fdiv_rn(warp_sum(sq), (float)D) + eps);
  const int64_t s = row % L;
  const int half = head_dim >> 1;
  const int64_t orow = row_map ? (int64_t)__ldg(row_map + row) : row;
  uint4* ov = reinterpret_cast<uint4*>(out + orow * D);
#pragma unroll
  for (int j = 0; j < kRowNV; ++j) {
    int v = j * 32 + lane;
    if (v < nvec) {
      float wf[8];
      bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(w) + v), wf);
      float y[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) y[i] = bf16r(f[j][i] * rrms) * wf[i];
      if (ROPE) {
        const int pair0 = ((v * 8) % head_dim) >> 1;  // 4 consecutive pairs
        const float4 c = __ldg(reinterpret_cast<const float4*>(cosv + s * half + pair0));
        const float4 sn = __ldg(reinterpret_cast<const float4*>(sinv + s * half + pair0));
        const float cc[4] = {c.x, c.y, c.z, c.w};
        const float ss[4] = {sn.x, sn.y, sn.z, sn.w};
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          const float ye = y[2 * p], yo = y[2 * p + 1];
          f[j][2 * p] = __fadd_rn(__fmul_rn(ye, cc[p]), __fmul_rn(yo, -ss[p]));
          f[j][2 * p + 1] = __fadd_rn(__fmul_rn(yo, cc[p]), __fmul_rn(ye, ss[p]));
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) f[j][i] = y[i];
      }
      ov[v] = f32_to_bf16x8(f[j]);
    }
  }
}

static inline unsigned row_grid(int64_t rows) { return (unsigned)((rows + 7) / 8); }

}  // namespace fvb

extern "C" {

int fvb_ln_modulate(const void* x, const void* scale, const void* shift, int64_t B, int64_t L,
                    int64_t D, float eps, void* out, void* q8, float* q_scale,
                    fvb_stream_t stream) {
  using namespace fvb;
  FVB_REQUIRE(B >= 0 && L >= 0 && D > 0, "fvb_ln_modulate: bad shape");
  FVB_REQUIRE(D % 8 == 0 && D <= 2048, "fvb_ln_modulate: D must be a multiple of 8, <= 2048");
  FVB_REQUIRE((q8 == nullptr) == (q_scale == nullptr), "fvb_ln_modulate: q8/q_scale go together");
  const int64_t rows = B * L;
  if (rows == 0) return FVB_OK;
  FVB_REQUIRE(x && scale && shift && out, "fvb_ln_modulate: NULL pointer");
  FVB_REQUIRE(aligned16(x) && aligned16(scale) && aligned16(shift) && aligned16(out),
              "fvb_ln_modulate: pointers must be 16-byte aligned");
  if (q8) {
    FVB_REQUIRE((reinterpret_cast<uintptr_t>(q8) & 7u) == 0, "fvb_ln_modulate: q8 alignment");
    ln_modulate_kernel<true><<<row_grid(rows), 256, 0, (cudaStream_t)stream>>>(
        (const __nv_bfloat16*)x, (const __nv_bfloat16*)scale, (const __nv_bfloat16*)shift, rows, L,
        (int)D, eps, (__nv_bfloat16*)out, (uint8_t*)q8, q_scale);
  } else {
    ln_modulate_kernel<false><<<row_grid(rows), 256, 0, (cudaStream_t)stream>>>(
        (const __nv_bfloat16*)x, (const __nv_bfloat16*)scale, (const __nv_bfloat16*)shift, rows, L,
        (int)D, eps, (__nv_bfloat16*)out, nullptr, nullptr);
  }
  return check_launch("fvb_ln_modulate");
}

int fvb_layer_norm(const void* x, const void* w, const void* b, int64_t rows, int64_t D,
                   float eps, void* out, fvb_stream_t stream) {
  using namespace fvb;
  FVB_REQUIRE(rows >= 0 && D > 0 && D % 8 == 0 && D <= 2048, "fvb_layer_norm: bad shape");
  if (rows == 0) return FVB_OK;
  FVB_REQUIRE(x && out, "fvb_layer_norm: NULL pointer");
  FVB_REQUIRE(aligned16(x) && aligned16(out) && (!w || aligned16(w)) && (!b || aligned16(b)),
              "fvb_layer_norm: pointers must be 16-byte aligned");
  layer_norm_kernel<<<row_grid(rows), 256, 0, (cudaStream_t)stream>>>(
      (const __nv_bfloat16*)x, (const __nv_bfloat16*)w, (const __nv_bfloat16*)b, rows, (int)D, eps,
      (__nv_bfloat16*)out);
  return check_launch("fvb_layer_norm");
}

int fvb_gate_add(const void* x, const void* gate, const void* r, int64_t B, int64_t L,
                 int64_t D, void* out, fvb_stream_t stream) {
  using namespace fvb;
  FVB_REQUIRE(B >= 0 && L >= 0 && D > 0 && D % 8 == 0, "fvb_gate_add: D must be a multiple of 8");
  const int64_t n = B * L * D;
  if (n == 0) return FVB_OK;
  FVB_REQUIRE(x && r && out, "fvb_gate_add: NULL pointer");
  FVB_REQUIRE(aligned16(x) && aligned16(r) && aligned16(out) && (!gate || aligned16(gate)),
              "fvb_gate_add: pointers must be 16-byte aligned");
  const int64_t nvec = n / 8;
  int64_t blocks = (nvec + 255) / 256;
  int64_t cap = (int64_t)sm_count() * 8;
  if (blocks > cap) blocks = cap;
  gate_add_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(
      (const uint4*)x, (const __nv_bfloat16*)gate, (const uint4*)r, nvec, L * D, (int)D,
      (uint4*)out);
  return check_launch("fvb_gate_add");
}

int fvb_rms_rope(const void* x, int64_t x_ld, const void* w, const float* cos, const float* sin,
                 int64_t rows, int64_t L, int64_t D, int64_t head_dim, float eps, int rope,
                 const int32_t* out_row_map, void* out, fvb_stream_t stream) {
  using namespace fvb;
  FVB_REQUIRE(rows >= 0 && D > 0 && D % 8 == 0 && D <= 2048, "fvb_rms_rope: bad D");
  if (x_ld == 0) x_ld = D;
  FVB_REQUIRE(x_ld >= D && x_ld % 8 == 0, "fvb_rms_rope: x_ld must be >= D and a multiple of 8");
  if (rows == 0) return FVB_OK;
  FVB_REQUIRE(L > 0 && rows % L == 0, "fvb_rms_rope: rows must be a multiple of L");
  FVB_REQUIRE(x && w && out, "fvb_rms_rope: NULL pointer");
  FVB_REQUIRE(aligned16(x) && aligned16(w) && aligned16(out), "fvb_rms_rope: alignment");
  if (rope) {
    FVB_REQUIRE(head_dim > 0 && head_dim % 8 == 0 && D % head_dim == 0,
                "fvb_rms_rope: head_dim must divide D and be a multiple of 8");
    FVB_REQUIRE(cos && sin && aligned16(cos) && aligned16(sin), "fvb_rms_rope: cos/sin");
    rms_rope_kernel<true><<<row_grid(rows), 256, 0, (cudaStream_t)stream>>>(
        (const __nv_bfloat16*)x, x_ld, (const __nv_bfloat16*)w, cos, sin, rows, L, (int)D,
        (int)head_dim, eps, out_row_map, (__nv_bfloat16*)out);
  } else {
    rms_rope_kernel<false><<<row_grid(rows), 256, 0, (cudaStream_t)stream>>>(
        (const __nv_bfloat16*)x, x_ld, (const __nv_bfloat16*)w, nullptr, nullptr, rows, L,
        (int)D, head_dim > 0 ? (int)head_dim : 128, eps, out_row_map, (__nv_bfloat16*)out);
  }
  return check_launch("fvb_rms_rope");
}

}  // extern "C"
