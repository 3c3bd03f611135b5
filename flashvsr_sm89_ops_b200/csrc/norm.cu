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
#include <type_traits>

#include "common.cuh"

namespace fvb {

__device__ __forceinline__ float quant_scale_from_amax_n(float amax) {
  return __fdiv_rn(fmaxf(amax, 1e-12f), 448.0f);
}

// Per-token e4m3 codes of 8 bf16 values held in a uint4 (the bf16 output of a row kernel):
// q = e4m3_rn(clamp(y / qs, +-448)).
__device__ __forceinline__ uint2 fp8_codes8(const uint4& y, float qs, float rqs) {
  float f[8];
  bf16x8_to_f32(y, f);
  return e4m3_codes8(f, qs, rqs);
}

// Gated residual add of one row held in registers (the gate_add_kernel arithmetic):
// x <- bf16(x + bf16(g * r)) (g == nullptr: bf16(x + r)), also stored to xo; raw holds
// the row's x vectors then its r vectors.  Packed bf16 _rn operations: the product of two
// bf16 values is exact in fp32, and an fp32 sum of two bf16 values rounds to the same bf16
// as their exact sum, so the eager fp32 chain and one rounding per operation agree bit for
// bit (as in the FFN-down epilogue's gated residual add).
template <int NV, bool FULL>
__device__ __forceinline__ void gate_add_row(const uint4* raw, uint4* xr, int lane, int nvec,
                                             const __nv_bfloat16* g, uint4* xo) {
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int v = j * 32 + lane;
    if (FULL || v < nvec) {
      uint4 o = raw[j];
      const uint4 ru = raw[NV + j];
      __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
      const __nv_bfloat162* r2 = reinterpret_cast<const __nv_bfloat162*>(&ru);
      if (g) {
        const uint4 gu = __ldg(reinterpret_cast<const uint4*>(g) + v);
        const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&gu);
#pragma unroll
        for (int p = 0; p < 4; ++p) o2[p] = __hadd2_rn(o2[p], __hmul2_rn(g2[p], r2[p]));
      } else {
#pragma unroll
        for (int p = 0; p < 4; ++p) o2[p] = __hadd2_rn(o2[p], r2[p]);
      }
      xr[j] = o;
      xo[v] = o;
    }
  }
}

// Row mean and (x - mean) * rden with rden = 1/sqrt(var + eps), two-pass in registers.
// x holds NV 16-byte vectors per lane (bf16); sums use packed fp32 pairs.  FULL: the row
// fills every lane's NV vectors (D == 256 * NV), so no per-vector bounds test is needed.
template <int NV, bool FULL>
__device__ __forceinline__ void row_stats(const uint4* xr, int lane, int nvec, int D, float eps,
                                          float& mean, float& rden) {
  uint64_t s2 = f2_pack(0.f, 0.f);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    if ((FULL || j * 32 + lane < nvec)) {
      float f[8];
      bf16x8_to_f32(xr[j], f);
#pragma unroll
      for (int i = 0; i < 8; i += 2) s2 = f2_add(s2, f2_pack(f[i], f[i + 1]));
    }
  }
  float sa, sb;
  f2_unpack(s2, sa, sb);
  mean = warp_sum(sa + sb) * (1.0f / (float)D);
  const uint64_t nm = f2_pack(-mean, -mean);
  uint64_t q2 = f2_pack(0.f, 0.f);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    if ((FULL || j * 32 + lane < nvec)) {
      float f[8];
      bf16x8_to_f32(xr[j], f);
#pragma unroll
      for (int i = 0; i < 8; i += 2) {
        const uint64_t d = f2_add(f2_pack(f[i], f[i + 1]), nm);
        q2 = f2_fma(d, d, q2);
      }
    }
  }
  float qa, qb;
  f2_unpack(q2, qa, qb);
  // mean = sum * (1/D), var = sumsq * (1/D) and the approximate reciprocal square root: each
  // within an fp32 ulp or two of the reference's sum / D and 1 / sqrt(.) (which its Triton
  // kernel also evaluates approximately), far inside the bf16 rounding that follows
  rden = rsqrtf(warp_sum(qa + qb) * (1.0f / (float)D) + eps);
}

// LayerNorm + AdaLN modulate.  The modulate chain is bf16 arithmetic on bf16 operands:
// xn * bf16(1 + scale) and (.) + shift are exact fp32 operations followed by one bf16
// rounding in the reference; the packed bf16x2 instructions (non-contracting _rn forms) round
// the exact result once, which is the same value (fp32 carries more than twice bf16's
// precision plus two bits, so the fp32 intermediate never changes a bf16 rounding).
// GATE: the row is first the gated residual sum x + g * r of gate_add_kernel (stored to
// x_out), so the add and the norm that follows it read the residual stream once.  out may
// be nullptr when only the FP8 codes are consumed.
// MOD: the block's AdaLN modulation sum is formed here instead of by a separate add:
// `scale` is the block's modulation [6, D] and `shift` the timestep modulation t_mod
// [B, 6, D]; chunk c of item b is bf16(modulation[c] + t_mod[b, c]) (one rounding of the exact
// sum, as torch's bf16 add), scale = chunk 1, shift = chunk 0, and block 0 also stores all
// six chunks of every item to mod_out [B, 6, D] for the block's later consumers.
template <bool EMIT_FP8, int NV, bool GATE, bool FULL, bool MOD = false>
__global__ void __launch_bounds__(256, GATE ? 2 : kRowBlocksPerSM) ln_modulate_kernel(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ gate,
    const __nv_bfloat16* __restrict__ r, __nv_bfloat16* __restrict__ x_out,
    const __nv_bfloat16* __restrict__ scale, const __nv_bfloat16* __restrict__ shift,
    int64_t rows, int64_t L, int D, float eps, __nv_bfloat16* __restrict__ out,
    uint8_t* __restrict__ q8, float* __restrict__ q_scale, __nv_bfloat16* __restrict__ mod_out) {
  const int lane = threadIdx.x & 31;
  const int nvec = D >> 3;
  if (MOD && blockIdx.x == 0) {
    const int64_t nb = rows / L, per = 6 * (int64_t)nvec;
    const uint4* mb = reinterpret_cast<const uint4*>(scale);
    const uint4* mt = reinterpret_cast<const uint4*>(shift);
    uint4* mo = reinterpret_cast<uint4*>(mod_out);
    for (int64_t i = threadIdx.x; i < nb * per; i += blockDim.x) {
      const uint4 u = __ldg(mb + i % per), t = __ldg(mt + i);
      uint4 o;
      const __nv_bfloat162* u2 = reinterpret_cast<const __nv_bfloat162*>(&u);
      const __nv_bfloat162* t2 = reinterpret_cast<const __nv_bfloat162*>(&t);
      __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
      for (int p = 0; p < 4; ++p) o2[p] = __hadd2_rn(u2[p], t2[p]);
      mo[i] = o;
    }
  }
  auto load = [&](int64_t row, uint4* xr) {
    const uint4* xv = reinterpret_cast<const uint4*>(x + row * D);
#pragma unroll
    for (int j = 0; j < NV; ++j)
      if ((FULL || j * 32 + lane < nvec)) xr[j] = __ldg(xv + j * 32 + lane);
    if (GATE) {
      const uint4* rv = reinterpret_cast<const uint4*>(r + row * D);
#pragma unroll
      for (int j = 0; j < NV; ++j)
        if ((FULL || j * 32 + lane < nvec)) xr[NV + j] = __ldg(rv + j * 32 + lane);
    }
  };
  auto body = [&](int64_t row, uint4* xr) {
    const int64_t b = row / L;
    // scale / shift rows are shared by all rows of a batch item: L1 hits after the first.
    // MOD: chunk 1 (scale) and chunk 0 (shift) of the modulation and of t_mod[b]
    const uint4* sv = reinterpret_cast<const uint4*>(MOD ? scale + D : scale + b * D);
    const uint4* hv = reinterpret_cast<const uint4*>(MOD ? scale : shift + b * D);
    const uint4* tsv = reinterpret_cast<const uint4*>(shift + b * 6 * (int64_t)D + D);
    const uint4* thv = reinterpret_cast<const uint4*>(shift + b * 6 * (int64_t)D);
    float mean, rden;
    row_stats<NV, FULL>(xr, lane, nvec, D, eps, mean, rden);
    const uint64_t nm = f2_pack(-mean, -mean), rd = f2_pack(rden, rden);
    const __nv_bfloat162 one2 = __float2bfloat162_rn(1.0f);
    __nv_bfloat162 m2 = __float2bfloat162_rn(0.0f);
    uint4* ov = reinterpret_cast<uint4*>(out + row * D);
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int v = j * 32 + lane;
      if (FULL || v < nvec) {
        float f[8];
        bf16x8_to_f32(xr[j], f);
        uint4 su = __ldg(sv + v), hu = __ldg(hv + v);
        if (MOD) {
          const uint4 ts = __ldg(tsv + v), th = __ldg(thv + v);
          __nv_bfloat162* s2m = reinterpret_cast<__nv_bfloat162*>(&su);
          __nv_bfloat162* h2m = reinterpret_cast<__nv_bfloat162*>(&hu);
          const __nv_bfloat162* ts2 = reinterpret_cast<const __nv_bfloat162*>(&ts);
          const __nv_bfloat162* th2 = reinterpret_cast<const __nv_bfloat162*>(&th);
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            s2m[p] = __hadd2_rn(s2m[p], ts2[p]);
            h2m[p] = __hadd2_rn(h2m[p], th2[p]);
          }
        }
        const __nv_bfloat162* s2 = reinterpret_cast<const __nv_bfloat162*>(&su);
        const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&hu);
        uint4 yo;
        __nv_bfloat162* y2 = reinterpret_cast<__nv_bfloat162*>(&yo);
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          float a, c;
          f2_unpack(f2_mul(f2_add(f2_pack(f[2 * p], f[2 * p + 1]), nm), rd), a, c);
          const __nv_bfloat162 xn = __floats2bfloat162_rn(a, c);
          // _rn forms: no contraction of the multiply and the add into one bf16 fma
          const __nv_bfloat162 y = __hadd2_rn(__hmul2_rn(xn, __hadd2_rn(one2, s2[p])), h2[p]);
          y2[p] = y;
          if (EMIT_FP8) m2 = __hmax2(m2, __habs2(y));
        }
        if (out) ov[v] = yo;
        xr[j] = yo;
      }
    }
    if (EMIT_FP8) {
      const float2 mf = __bfloat1622float2(m2);
      const float amax = warp_max(fmaxf(mf.x, mf.y));
      const float qs = quant_scale_from_amax_n(amax);
      const float rqs = __frcp_rn(qs);
      uint2* qv = reinterpret_cast<uint2*>(q8 + row * D);
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        const int v = j * 32 + lane;
        if (FULL || v < nvec) qv[v] = fp8_codes8(xr[j], qs, rqs);
      }
      if (lane == 0) q_scale[row] = returned_scale(amax);
    }
  };
  if (GATE) {
    auto prep = [&](int64_t row, const uint4* raw, uint4* xr) {
      gate_add_row<NV, FULL>(raw, xr, lane, nvec, gate ? gate + (row / L) * D : nullptr,
                       reinterpret_cast<uint4*>(x_out + row * D));
    };
    row_pipeline_prep<NV, 2 * NV>(rows, load, prep, body);
  } else {
    row_pipeline<NV>(rows, load, body);
  }
}

// LayerNorm with optional affine weight / bias, fp32 math and one bf16 rounding (the
// semantics of torch.nn.LayerNorm on bf16 tensors; the affine step is one fused
// multiply-add per element); optionally also the per-token e4m3 codes of that bf16 output
// (what the next FP8 linear would compute from it).
// GATE: as for ln_modulate_kernel, the row is first x + g * r (stored to x_out; the gate
// row of batch item row / L).
template <bool EMIT_FP8, int NV, bool GATE, bool FULL>
__global__ void __launch_bounds__(256, 2) layer_norm_kernel(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ gate,
    const __nv_bfloat16* __restrict__ r, __nv_bfloat16* __restrict__ x_out, int64_t L,
    const __nv_bfloat16* __restrict__ w, const __nv_bfloat16* __restrict__ bias, int64_t rows,
    int D, float eps, __nv_bfloat16* __restrict__ out, uint8_t* __restrict__ q8,
    float* __restrict__ q_scale) {
  const int lane = threadIdx.x & 31;
  const int nvec = D >> 3;
  auto load = [&](int64_t row, uint4* xr) {
    const uint4* xv = reinterpret_cast<const uint4*>(x + row * D);
#pragma unroll
    for (int j = 0; j < NV; ++j)
      if ((FULL || j * 32 + lane < nvec)) xr[j] = __ldg(xv + j * 32 + lane);
    if (GATE) {
      const uint4* rv = reinterpret_cast<const uint4*>(r + row * D);
#pragma unroll
      for (int j = 0; j < NV; ++j)
        if ((FULL || j * 32 + lane < nvec)) xr[NV + j] = __ldg(rv + j * 32 + lane);
    }
  };
  auto body = [&](int64_t row, uint4* xr) {
    float mean, rstd;
    row_stats<NV, FULL>(xr, lane, nvec, D, eps, mean, rstd);
    const uint64_t nm = f2_pack(-mean, -mean), rs2 = f2_pack(rstd, rstd);
    __nv_bfloat162 m2 = __float2bfloat162_rn(0.0f);
    uint4* ov = reinterpret_cast<uint4*>(out + row * D);
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int v = j * 32 + lane;
      if (FULL || v < nvec) {
        float f[8], ww[8], bb[8];
        bf16x8_to_f32(xr[j], f);
        if (w) bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(w) + v), ww);
        if (bias) bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(bias) + v), bb);
        uint4 yo;
        __nv_bfloat162* y2 = reinterpret_cast<__nv_bfloat162*>(&yo);
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          // (x - mean) * rstd, then * w + b (one fused multiply-add), in fp32 pairs
          uint64_t y = f2_mul(f2_add(f2_pack(f[2 * p], f[2 * p + 1]), nm), rs2);
          if (w && bias)
            y = f2_fma(y, f2_pack(ww[2 * p], ww[2 * p + 1]), f2_pack(bb[2 * p], bb[2 * p + 1]));
          else if (w)
            y = f2_mul(y, f2_pack(ww[2 * p], ww[2 * p + 1]));
          else if (bias)
            y = f2_add(y, f2_pack(bb[2 * p], bb[2 * p + 1]));
          float a, c;
          f2_unpack(y, a, c);
          y2[p] = __floats2bfloat162_rn(a, c);
          if (EMIT_FP8) m2 = __hmax2(m2, __habs2(y2[p]));
        }
        if (out) ov[v] = yo;
        if (EMIT_FP8) xr[j] = yo;
      }
    }
    if (EMIT_FP8) {
      const float2 mf = __bfloat1622float2(m2);
      const float amax = warp_max(fmaxf(mf.x, mf.y));
      const float qs = quant_scale_from_amax_n(amax);
      const float rqs = __frcp_rn(qs);
      uint2* qv = reinterpret_cast<uint2*>(q8 + row * D);
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        const int v = j * 32 + lane;
        if (FULL || v < nvec) qv[v] = fp8_codes8(xr[j], qs, rqs);
      }
      if (lane == 0) q_scale[row] = returned_scale(amax);
    }
  };
  if (GATE) {
    auto prep = [&](int64_t row, const uint4* raw, uint4* xr) {
      gate_add_row<NV, FULL>(raw, xr, lane, nvec, gate ? gate + (row / L) * D : nullptr,
                       reinterpret_cast<uint4*>(x_out + row * D));
    };
    row_pipeline_prep<NV, 2 * NV>(rows, load, prep, body);
  } else {
    row_pipeline<NV>(rows, load, body);
  }
}

__global__ void __launch_bounds__(256) gate_add_kernel(const uint4* __restrict__ x,
                                                        const __nv_bfloat16* __restrict__ gate,
                                                        const uint4* __restrict__ r, int64_t nvec,
                                                        int64_t LD, int D, uint4* __restrict__ out) {
  // gate is [B, 1, D]: vector v of the [B, L, D] stream takes gate vector
  // (v / (L*D/8)) * (D/8) + v % (D/8); 32-bit index math when the stream allows it
  const uint32_t nvd = (uint32_t)(D >> 3);
  const int64_t per_b = LD >> 3;
  const bool small = nvec <= 0xFFFFFFFFll && per_b <= 0xFFFFFFFFll;
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < nvec;
       v += (int64_t)gridDim.x * blockDim.x) {
    uint4 o = __ldg(x + v);
    const uint4 ru = __ldg(r + v);
    __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
    const __nv_bfloat162* r2 = reinterpret_cast<const __nv_bfloat162*>(&ru);
    if (gate) {
      int64_t gv;
      if (small) {
        const uint32_t v32 = (uint32_t)v, pb = (uint32_t)per_b;
        const uint32_t b = v32 / pb;
        gv = (int64_t)b * nvd + (v32 - b * pb) % nvd;
      } else {
        gv = (v / per_b) * nvd + (v % per_b) % nvd;
      }
      const uint4 gu = __ldg(reinterpret_cast<const uint4*>(gate) + gv);
      const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&gu);
      // bf16(x + bf16(g * r)) with one rounding per operation (see gate_add_row)
#pragma unroll
      for (int p = 0; p < 4; ++p) o2[p] = __hadd2_rn(o2[p], __hmul2_rn(g2[p], r2[p]));
    } else {
#pragma unroll
      for (int p = 0; p < 4; ++p) o2[p] = __hadd2_rn(o2[p], r2[p]);
    }
    out[v] = o;
  }
}

template <int NV>
__device__ __forceinline__ void unpack_row_f(const uint4* raw, float* f, int lane, int nvec) {
#pragma unroll
  for (int j = 0; j < NV; ++j)
    if (j * 32 + lane < nvec) bf16x8_to_f32(raw[j], f + 8 * j);
}

// RMSNorm (+ interleaved RoPE).  y = bf16(x * rrms) * w in fp32 (an exact product of two
// bf16 values); the rotation rounds each product and the sum once, all in packed fp32 pairs
// (mul.rn / add.rn per lane, no contraction), then one bf16 rounding.  rrms =
// rsqrt(sum(x^2) / D + eps) with the approximate reciprocal square root, as the reference's
// Triton kernel takes it (tl.rsqrt).
// One row of RMSNorm (+ RoPE) from the lane's fp32 copy f of the row: input row `row` of a
// sequence of L rows (cos / sin row row % L), written to output row row_map[row] (or row)
// of out.  The position and the output row are formed after the row's reduction.
template <bool ROPE, int NV>
__device__ __forceinline__ void rms_rope_row(const float* f, int lane, int nvec, int D,
                                             float invD, float eps, int head_dim, int64_t row,
                                             int64_t L, const int32_t* __restrict__ row_map,
                                             const __nv_bfloat16* __restrict__ w,
                                             const float* __restrict__ cosv,
                                             const float* __restrict__ sinv,
                                             __nv_bfloat16* __restrict__ out) {
  uint64_t q2 = f2_pack(0.f, 0.f);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    if (j * 32 + lane < nvec) {
#pragma unroll
      for (int i = 0; i < 8; i += 2) {
        const uint64_t t = f2_pack(f[8 * j + i], f[8 * j + i + 1]);
        q2 = f2_fma(t, t, q2);
      }
    }
  }
  float qa, qb;
  f2_unpack(q2, qa, qb);
  const float rrms = rsqrtf(warp_sum(qa + qb) * invD + eps);
  const uint64_t rr = f2_pack(rrms, rrms);
  const int64_t srow = row % L;
  const int half = head_dim >> 1;
  const int64_t orow = row_map ? (int64_t)__ldg(row_map + row) : row;
  uint4* ov = reinterpret_cast<uint4*>(out + orow * D);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int v = j * 32 + lane;
    if (v < nvec) {
      float wf[8];
      bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(w) + v), wf);
      float4 c4 = make_float4(0.f, 0.f, 0.f, 0.f), s4 = c4;
      if (ROPE) {
        const int pair0 = ((v * 8) % head_dim) >> 1;  // 4 consecutive pairs
        c4 = __ldg(reinterpret_cast<const float4*>(cosv + srow * half + pair0));
        s4 = __ldg(reinterpret_cast<const float4*>(sinv + srow * half + pair0));
      }
      const float cc[4] = {c4.x, c4.y, c4.z, c4.w};
      const float ss[4] = {s4.x, s4.y, s4.z, s4.w};
      uint4 yo;
      __nv_bfloat162* y2 = reinterpret_cast<__nv_bfloat162*>(&yo);
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        float a, b;
        f2_unpack(f2_mul(f2_pack(f[8 * j + 2 * p], f[8 * j + 2 * p + 1]), rr), a, b);
        const float2 yb = __bfloat1622float2(__floats2bfloat162_rn(a, b));
        const uint64_t yw = f2_mul(f2_pack(yb.x, yb.y), f2_pack(wf[2 * p], wf[2 * p + 1]));
        if (ROPE) {
          float ye, yo_;
          f2_unpack(yw, ye, yo_);
          float e, o;
          f2_unpack(f2_add(f2_mul(yw, f2_pack(cc[p], cc[p])),
                           f2_mul(f2_pack(yo_, ye), f2_pack(-ss[p], ss[p]))),
                    e, o);
          y2[p] = __floats2bfloat162_rn(e, o);
        } else {
          float ye, yo_;
          f2_unpack(yw, ye, yo_);
          y2[p] = __floats2bfloat162_rn(ye, yo_);
        }
      }
      ov[v] = yo;
    }
  }
}

template <bool ROPE, int NV>
__global__ void __launch_bounds__(256, 2) rms_rope_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t x_ld, const __nv_bfloat16* __restrict__ w,
    const float* __restrict__ cosv, const float* __restrict__ sinv, int64_t rows, int64_t L,
    int D, int head_dim, float eps, const int32_t* __restrict__ row_map,
    __nv_bfloat16* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int nvec = D >> 3;
  const float invD = 1.0f / (float)D;
  auto load = [&](int64_t row, uint4* raw) {
    const uint4* xv = reinterpret_cast<const uint4*>(x + row * x_ld);
#pragma unroll
    for (int j = 0; j < NV; ++j)
      if (j * 32 + lane < nvec) raw[j] = __ldg(xv + j * 32 + lane);
  };
  auto prep = [&](int64_t, const uint4* raw, float* f) { unpack_row_f<NV>(raw, f, lane, nvec); };
  auto body = [&](int64_t row, float* f) {
    rms_rope_row<ROPE, NV>(f, lane, nvec, D, invD, eps, head_dim, row, L, row_map, w, cosv,
                           sinv, out);
  };
  row_pipeline_f<NV, NV>(rows, load, prep, body);
}

// The self-attention's q, k and v from the fused projection output qkv [rows, 3D] in one
// launch: rows [0, R) are RMSNorm(w_q) + RoPE of the q third, [R, 2R) the same for k with
// w_k, [2R, 3R) the v third copied; every output row r goes to row row_map[r] of its output
// (the window order), exactly as three rms_rope / window_partition launches would write it.
struct QkvRows {
  const __nv_bfloat16* x;
  int64_t x_ld;
  const __nv_bfloat16* w[2];
  float eps[2];
  const int32_t* row_map;
  __nv_bfloat16* out[3];
};

template <int NV>
__global__ void __launch_bounds__(256, 2) qkv_rope_window_kernel(
    const QkvRows a, const float* __restrict__ cosv, const float* __restrict__ sinv, int64_t R,
    int64_t L, int D, int head_dim) {
  const int lane = threadIdx.x & 31;
  const int nvec = D >> 3;
  const float invD = 1.0f / (float)D;
  auto load = [&](int64_t row, uint4* raw) {
    const int p = (int)(row / R);
    const uint4* xv = reinterpret_cast<const uint4*>(a.x + (row - p * R) * a.x_ld + p * D);
#pragma unroll
    for (int j = 0; j < NV; ++j)
      if (j * 32 + lane < nvec) raw[j] = __ldg(xv + j * 32 + lane);
  };
  auto prep = [&](int64_t, const uint4* raw, float* f) { unpack_row_f<NV>(raw, f, lane, nvec); };
  auto body = [&](int64_t row, float* f) {
    const int p = (int)(row / R);
    const int64_t r = row - p * R;
    if (p < 2) {
      rms_rope_row<true, NV>(f, lane, nvec, D, invD, a.eps[p], head_dim, r, L, a.row_map,
                             a.w[p], cosv, sinv, a.out[p]);
    } else {
      const int64_t orow = a.row_map ? (int64_t)__ldg(a.row_map + r) : r;
      uint4* ov = reinterpret_cast<uint4*>(a.out[p] + orow * D);
#pragma unroll
      for (int j = 0; j < NV; ++j)
        if (j * 32 + lane < nvec) ov[j * 32 + lane] = f32_to_bf16x8(f + 8 * j);  // exact
    }
  };
  row_pipeline_f<NV, NV>(3 * R, load, prep, body);
}

static inline unsigned row_grid(int64_t rows, int blocks_per_sm = kRowBlocksPerSM) {
  const int64_t need = (rows + 7) / 8, cap = (int64_t)sm_count() * blocks_per_sm;
  return (unsigned)(need < cap ? need : cap);
}

// Row kernels keep ceil(D / 256) 16-byte vectors per lane in registers; instantiate the
// count for the row length (D <= 2048).
template <typename F>
static void dispatch_nv(int64_t D, F&& f) {
  if (D <= 512) f(std::integral_constant<int, 2>{});
  else if (D <= 1024) f(std::integral_constant<int, 4>{});
  else if (D <= 1536) f(std::integral_constant<int, 6>{});
  else f(std::integral_constant<int, 8>{});
}

// Shared host paths of the plain and the gated-residual entry points (r == nullptr: plain).
// out may be nullptr when q8 is given (only the FP8 codes are consumed).
static int ln_modulate_impl(const void* x, const void* gate, const void* r, void* x_out,
                            const void* scale, const void* shift, int64_t B, int64_t L, int64_t D,
                            float eps, void* out, void* q8, float* q_scale, fvb_stream_t stream,
                            const char* name, void* mod_out = nullptr) {
  const int64_t rows = B * L;
  FVB_REQUIRE(x && scale && shift && (out || q8), "%s: NULL pointer", name);
  FVB_REQUIRE(aligned16(x) && aligned16(scale) && aligned16(shift) && (!out || aligned16(out)),
              "%s: pointers must be 16-byte aligned", name);
  if (q8) FVB_REQUIRE((reinterpret_cast<uintptr_t>(q8) & 7u) == 0, "%s: q8 alignment", name);
  auto launch = [&](auto emit, auto nv, auto gated) {
    constexpr int NV = decltype(nv)::value;
    auto go = [&](auto full) {
      constexpr bool E = decltype(emit)::value, G = decltype(gated)::value,
                     FL = decltype(full)::value;
      const unsigned grid = row_grid(rows, G ? 2 : kRowBlocksPerSM);
      if constexpr (!G && E) {
        if (mod_out != nullptr) {
          ln_modulate_kernel<E, NV, false, FL, true><<<grid, 256, 0, (cudaStream_t)stream>>>(
              (const __nv_bfloat16*)x, nullptr, nullptr, nullptr, (const __nv_bfloat16*)scale,
              (const __nv_bfloat16*)shift, rows, L, (int)D, eps, (__nv_bfloat16*)out,
              (uint8_t*)q8, q_scale, (__nv_bfloat16*)mod_out);
          return;
        }
      }
      ln_modulate_kernel<E, NV, G, FL><<<grid, 256, 0, (cudaStream_t)stream>>>(
            (const __nv_bfloat16*)x, (const __nv_bfloat16*)gate, (const __nv_bfloat16*)r,
            (__nv_bfloat16*)x_out, (const __nv_bfloat16*)scale, (const __nv_bfloat16*)shift,
            rows, L, (int)D, eps, (__nv_bfloat16*)out, (uint8_t*)q8, q_scale, nullptr);
    };
    // (the plain bf16-output form spills in its FULL build at this register budget)
    if (D == NV * 256 && (decltype(emit)::value || decltype(gated)::value)) go(std::true_type{});
    else go(std::false_type{});
  };
  dispatch_nv(D, [&](auto nv) {
    if (r) {
      if (q8) launch(std::true_type{}, nv, std::true_type{});
      else launch(std::false_type{}, nv, std::true_type{});
    } else {
      if (q8) launch(std::true_type{}, nv, std::false_type{});
      else launch(std::false_type{}, nv, std::false_type{});
    }
  });
  return check_launch(name);
}

static int layer_norm_impl(const void* x, const void* gate, const void* r, void* x_out, int64_t L,
                           int64_t rows, const void* w, const void* b, int64_t D, float eps,
                           void* out, void* q8, float* q_scale, fvb_stream_t stream,
                           const char* name) {
  FVB_REQUIRE(x && (out || q8), "%s: NULL pointer", name);
  FVB_REQUIRE(aligned16(x) && (!out || aligned16(out)) && (!w || aligned16(w)) &&
                  (!b || aligned16(b)),
              "%s: pointers must be 16-byte aligned", name);
  if (q8) FVB_REQUIRE((reinterpret_cast<uintptr_t>(q8) & 7u) == 0, "%s: q8 alignment", name);
  auto launch = [&](auto emit, auto nv, auto gated) {
    constexpr int NV = decltype(nv)::value;
    auto go = [&](auto full) {
      layer_norm_kernel<decltype(emit)::value, NV, decltype(gated)::value, decltype(full)::value>
          <<<row_grid(rows, 2), 256, 0, (cudaStream_t)stream>>>(
              (const __nv_bfloat16*)x, (const __nv_bfloat16*)gate, (const __nv_bfloat16*)r,
              (__nv_bfloat16*)x_out, L, (const __nv_bfloat16*)w, (const __nv_bfloat16*)b, rows,
              (int)D, eps, (__nv_bfloat16*)out, (uint8_t*)q8, q_scale);
    };
    if (D == NV * 256) go(std::true_type{});
    else go(std::false_type{});
  };
  dispatch_nv(D, [&](auto nv) {
    if (r) {
      if (q8) launch(std::true_type{}, nv, std::true_type{});
      else launch(std::false_type{}, nv, std::true_type{});
    } else {
      if (q8) launch(std::true_type{}, nv, std::false_type{});
      else launch(std::false_type{}, nv, std::false_type{});
    }
  });
  return check_launch(name);
}

}  // namespace fvb

extern "C" {

int fvb_ln_modulate(const void* x, const void* scale, const void* shift, int64_t B, int64_t L,
                    int64_t D, float eps, void* out, void* q8, float* q_scale,
                    fvb_stream_t stream) {
  using namespace fvb;
  FVB_REQUIRE(B >= 0 && L >= 0 && D > 0, "fvb_ln_modulate: bad shape");
  FVB_REQUIRE(D % 8 == 0 && D <= 2048, "fvb_ln_modulate: D must be a multiple of 8, <= 2048");
  FVB_REQUIRE((q8 == nullptr) == (q_scale == nullptr), "fvb_ln_modulate: q8/q_scale go together");
  if (B * L == 0) return FVB_OK;
  return ln_modulate_impl(x, nullptr, nullptr, nullptr, scale, shift, B, L, D, eps, out, q8,
                          q_scale, stream, "fvb_ln_modulate");
}

int fvb_ln_modulate_adaln(const void* x, const void* modulation, const void* t_mod, int64_t B,
                          int64_t L, int64_t D, float eps, void* out, void* q8, float* q_scale,
                          void* mod_out, fvb_stream_t stream) {
  using namespace fvb;
  FVB_REQUIRE(B >= 0 && L >= 0 && D > 0, "fvb_ln_modulate_adaln: bad shape");
  FVB_REQUIRE(D % 8 == 0 && D <= 2048, "fvb_ln_modulate_adaln: D must be a multiple of 8, <= 2048");
  FVB_REQUIRE(q8 != nullptr && q_scale != nullptr,
              "fvb_ln_modulate_adaln: q8 and q_scale are required (the FP8-emitting norm)");
  if (B * L == 0) return FVB_OK;
  FVB_REQUIRE(mod_out != nullptr && aligned16(mod_out), "fvb_ln_modulate_adaln: mod_out NULL or "
              "not 16-byte aligned");
  return ln_modulate_impl(x, nullptr, nullptr, nullptr, modulation, t_mod, B, L, D, eps, out, q8,
                          q_scale, stream, "fvb_ln_modulate_adaln", mod_out);
}

int fvb_gate_add_ln_modulate(const void* x, const void* gate, const void* r, void* x_out,
                             const void* scale, const void* shift, int64_t B, int64_t L, int64_t D,
                             float eps, void* out, void* q8, float* q_scale, fvb_stream_t stream) {
  using namespace fvb;
  FVB_REQUIRE(B >= 0 && L >= 0 && D > 0, "fvb_gate_add_ln_modulate: bad shape");
  FVB_REQUIRE(D % 8 == 0 && D <= 2048,
              "fvb_gate_add_ln_modulate: D must be a multiple of 8, <= 2048");
  FVB_REQUIRE((q8 == nullptr) == (q_scale == nullptr),
              "fvb_gate_add_ln_modulate: q8/q_scale go together");
  if (B * L == 0) return FVB_OK;
  FVB_REQUIRE(r && x_out && aligned16(r) && aligned16(x_out) && (!gate || aligned16(gate)),
              "fvb_gate_add_ln_modulate: r / x_out / gate NULL or not 16-byte aligned");
  FVB_REQUIRE(x_out != x && x_out != r, "fvb_gate_add_ln_modulate: x_out must not alias x or r");
  return ln_modulate_impl(x, gate, r, x_out, scale, shift, B, L, D, eps, out, q8, q_scale, stream,
                          "fvb_gate_add_ln_modulate");
}

int fvb_layer_norm(const void* x, const void* w, const void* b, int64_t rows, int64_t D,
                   float eps, void* out, void* q8, float* q_scale, fvb_stream_t stream) {
  using namespace fvb;
  FVB_REQUIRE(rows >= 0 && D > 0 && D % 8 == 0 && D <= 2048, "fvb_layer_norm: bad shape");
  FVB_REQUIRE((q8 == nullptr) == (q_scale == nullptr), "fvb_layer_norm: q8/q_scale go together");
  if (rows == 0) return FVB_OK;
  return layer_norm_impl(x, nullptr, nullptr, nullptr, 1, rows, w, b, D, eps, out, q8, q_scale,
                         stream, "fvb_layer_norm");
}

int fvb_gate_add_layer_norm(const void* x, const void* gate, const void* r, void* x_out,
                            const void* w, const void* b, int64_t B, int64_t L, int64_t D,
                            float eps, void* out, void* q8, float* q_scale, fvb_stream_t stream) {
  using namespace fvb;
  FVB_REQUIRE(B >= 0 && L >= 0 && D > 0 && D % 8 == 0 && D <= 2048,
              "fvb_gate_add_layer_norm: bad shape");
  FVB_REQUIRE((q8 == nullptr) == (q_scale == nullptr),
              "fvb_gate_add_layer_norm: q8/q_scale go together");
  if (B * L == 0) return FVB_OK;
  FVB_REQUIRE(r && x_out && aligned16(r) && aligned16(x_out) && (!gate || aligned16(gate)),
              "fvb_gate_add_layer_norm: r / x_out / gate NULL or not 16-byte aligned");
  FVB_REQUIRE(x_out != x && x_out != r, "fvb_gate_add_layer_norm: x_out must not alias x or r");
  return layer_norm_impl(x, gate, r, x_out, L, B * L, w, b, D, eps, out, q8, q_scale, stream,
                         "fvb_gate_add_layer_norm");
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

int fvb_qkv_rope_window(const void* qkv, int64_t x_ld, const void* w_q, const void* w_k,
                        const float* cos, const float* sin, int64_t rows, int64_t L, int64_t D,
                        int64_t head_dim, float eps_q, float eps_k, const int32_t* row_map,
                        void* out_q, void* out_k, void* out_v, fvb_stream_t stream) {
  using namespace fvb;
  FVB_REQUIRE(rows >= 0 && D > 0 && D % 8 == 0 && D <= 2048, "fvb_qkv_rope_window: bad D");
  if (x_ld == 0) x_ld = 3 * D;
  FVB_REQUIRE(x_ld >= 3 * D && x_ld % 8 == 0,
              "fvb_qkv_rope_window: x_ld must be >= 3 D and a multiple of 8");
  if (rows == 0) return FVB_OK;
  FVB_REQUIRE(L > 0 && rows % L == 0 && rows < (1ll << 40), "fvb_qkv_rope_window: rows / L");
  FVB_REQUIRE(qkv && w_q && w_k && out_q && out_k && out_v && cos && sin,
              "fvb_qkv_rope_window: NULL pointer");
  FVB_REQUIRE(aligned16(qkv) && aligned16(w_q) && aligned16(w_k) && aligned16(out_q) &&
                  aligned16(out_k) && aligned16(out_v) && aligned16(cos) && aligned16(sin),
              "fvb_qkv_rope_window: alignment");
  FVB_REQUIRE(head_dim > 0 && head_dim % 8 == 0 && D % head_dim == 0,
              "fvb_qkv_rope_window: head_dim must divide D and be a multiple of 8");
  QkvRows a;
  a.x = (const __nv_bfloat16*)qkv;
  a.x_ld = x_ld;
  a.w[0] = (const __nv_bfloat16*)w_q;
  a.w[1] = (const __nv_bfloat16*)w_k;
  a.eps[0] = eps_q;
  a.eps[1] = eps_k;
  a.row_map = row_map;
  a.out[0] = (__nv_bfloat16*)out_q;
  a.out[1] = (__nv_bfloat16*)out_k;
  a.out[2] = (__nv_bfloat16*)out_v;
  dispatch_nv(D, [&](auto nv) {
    qkv_rope_window_kernel<decltype(nv)::value><<<row_grid(3 * rows, 2), 256, 0,
                                                  (cudaStream_t)stream>>>(
        a, cos, sin, rows, L, (int)D, (int)head_dim);
  });
  return check_launch("fvb_qkv_rope_window");
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
  }
  const int hd = rope ? (int)head_dim : (head_dim > 0 ? (int)head_dim : 128);
  auto launch = [&](auto r, auto nv) {
    rms_rope_kernel<decltype(r)::value, decltype(nv)::value>
        <<<row_grid(rows, 2), 256, 0, (cudaStream_t)stream>>>(
            (const __nv_bfloat16*)x, x_ld, (const __nv_bfloat16*)w, rope ? cos : nullptr,
            rope ? sin : nullptr, rows, L, (int)D, hd, eps, out_row_map, (__nv_bfloat16*)out);
  };
  dispatch_nv(D, [&](auto nv) {
    if (rope) launch(std::true_type{}, nv);
    else launch(std::false_type{}, nv);
  });
  return check_launch("fvb_rms_rope");
}

}  // extern "C"
