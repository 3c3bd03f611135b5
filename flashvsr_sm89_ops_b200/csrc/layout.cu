// Layout and block-mask kernels around the block-sparse attention:
//   a14  window partition / reverse (raster <-> (2,8,8)-window order)
//   a11  keep mask -> CSR, on the device and without the reference's host sync
//   a13  draft_block_mask (reference selection semantics), and the causal top-k
//        rule of the benchmark configuration
#include "common.cuh"

namespace fvb {

// ---------------------------------------------------------------------------
// a14: window partition.  Token rows of C bf16 are permuted, one warp per row.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) window_kernel(const uint4* __restrict__ x, int64_t xvec_ld,
                                                      int64_t rows,
                                                      int64_t F, int64_t Hh, int64_t Ww,
                                                      int64_t cvec, int wf, int wh, int ww,
                                                      int reverse, uint4* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t o = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (o >= rows) return;
  // decompose the window-order index o
  const int64_t wsize = (int64_t)wf * wh * ww;
  const int64_t nF = F / wf, nH = Hh / wh, nW = Ww / ww;
  int64_t t = o;
  const int64_t inwin = t % wsize;
  t /= wsize;
  const int64_t wi = t % nW;
  t /= nW;
  const int64_t hi = t % nH;
  t /= nH;
  const int64_t fi = t % nF;
  const int64_t b = t / nF;
  const int64_t a = inwin / ((int64_t)wh * ww);
  const int64_t c = (inwin / ww) % wh;
  const int64_t d = inwin % ww;
  const int64_t r = ((b * F + fi * wf + a) * Hh + hi * wh + c) * Ww + wi * ww + d;  // raster row
  const int64_t src = reverse ? o : r;
  const int64_t dst = reverse ? r : o;
  const uint4* s = x + src * xvec_ld;
  uint4* dd = out + dst * cvec;
  for (int64_t v = lane; v < cvec; v += 32) dd[v] = __ldg(s + v);
}

// ---------------------------------------------------------------------------
// a11: keep [H*NQ, NK] -> sel (kept ascending, then unkept ascending), cnt
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) mask_to_csr_kernel(const uint8_t* __restrict__ keep,
                                                           int64_t nrows, int64_t NK,
                                                           int32_t* __restrict__ sel,
                                                           int32_t* __restrict__ cnt) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= nrows) return;
  const uint8_t* kr = keep + row * NK;
  int32_t* sr = sel + row * NK;
  const unsigned lt = (1u << lane) - 1u;
  int base = 0;
  for (int64_t k0 = 0; k0 < NK; k0 += 32) {
    const int64_t k = k0 + lane;
    const bool on = (k < NK) && kr[k] != 0;
    const unsigned bal = __ballot_sync(0xffffffffu, on);
    if (on) sr[base + __popc(bal & lt)] = (int32_t)k;
    base += __popc(bal);
  }
  if (lane == 0) cnt[row] = base;
  for (int64_t k0 = 0; k0 < NK; k0 += 32) {
    const int64_t k = k0 + lane;
    const bool off = (k < NK) && kr[k] == 0;
    const unsigned bal = __ballot_sync(0xffffffffu, off);
    if (off) sr[base + __popc(bal & lt)] = (int32_t)k;
    base += __popc(bal);
  }
}

// ---------------------------------------------------------------------------
// block pooling: mean over the 128 tokens of each window, per channel.
// round_bf16 mirrors torch.mean on a bf16 tensor (fp32 accumulate, bf16 result).
// ---------------------------------------------------------------------------
// grid (windows, ceil(C / 512)), 256 threads: threadIdx.x % 64 picks one 8-channel vector of
// this CTA's 512-channel slice, threadIdx.x / 64 one of 4 token groups (32 tokens each, 8
// loads in flight per thread); the 4 partial sums meet in shared memory in a fixed order.
// The order is part of the keep rules' definition (the oracle restates it): partial g sums
// tokens g, g+4, ..., g+124 in that order; mean = ((p0 + p1) + (p2 + p3)) / 128.
// TWO: two sources in one launch (grid.x = nblk + nblk2): the first nblk windows come from
// x into avg, the rest from x2 into avg2.
template <bool TWO = false>
__global__ void __launch_bounds__(256) pool_kernel(const __nv_bfloat16* __restrict__ x_in,
                                                    int64_t nblk, int64_t C, int round_bf16,
                                                    float* __restrict__ avg_in,
                                                    const __nv_bfloat16* __restrict__ x2 = nullptr,
                                                    float* __restrict__ avg2 = nullptr) {
  __shared__ float part[4][64][8];
  const bool second = TWO && (int64_t)blockIdx.x >= nblk;
  const int64_t blk = second ? (int64_t)blockIdx.x - nblk : (int64_t)blockIdx.x;
  const __nv_bfloat16* __restrict__ x = second ? x2 : x_in;
  float* __restrict__ avg = second ? avg2 : avg_in;
  const int vx = threadIdx.x & 63, ty = threadIdx.x >> 6;
  const int64_t c8 = (int64_t)blockIdx.y * 64 + vx;
  const bool on = c8 * 8 < C;
  const uint4* xb = reinterpret_cast<const uint4*>(x + blk * 128 * C) + c8;
  const int64_t cv = C >> 3;
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if (on) {
#pragma unroll 8
    for (int t = ty; t < 128; t += 4) {
      float f[8];
      bf16x8_to_f32(__ldg(xb + t * cv), f);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += f[i];
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) part[ty][vx][i] = acc[i];
  __syncthreads();
  if (ty == 0 && on) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float s = (part[0][vx][i] + part[1][vx][i]) + (part[2][vx][i] + part[3][vx][i]);
      const float m = __fdiv_rn(s, 128.0f);
      avg[blk * C + c8 * 8 + i] = round_bf16 ? bf16r(m) : m;
    }
  }
}

// ---------------------------------------------------------------------------
// a13 step 2: per (head, query block) scores over all key blocks, local mask,
// softmax -> probabilities (bf16-rounded like the bf16 reference tensors).
// grid (NQ, H), block 256; dynamic smem NK floats.
// Every fp32 step has one fixed evaluation order, which the oracle restates
// operation for operation, so the keep mask is bit-identical to it:
//   score  = bf16(bf16(sum_e q[e] k[e]) / sqrt(d)), the sum sequential over e (the
//            products of bf16 means are exact in fp32);
//   e_j    = fp32(exp(double(score_j - max)))  (a double exp, so both sides round the
//            same value to fp32);
//   total  = sequential fp32 sum of e_j over j = 0..NK-1;
//   prob_j = bf16(e_j / total).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) draft_scores_kernel(
    const float* __restrict__ aq, const float* __restrict__ ak, int64_t NQ, int64_t NK, int H,
    int d, const uint8_t* __restrict__ local, int64_t sq, int64_t sk, float* __restrict__ prob) {
  extern __shared__ float sc[];
  __shared__ float red[32];
  __shared__ float qsh[256];
  const int64_t qi = blockIdx.x;
  const int h = blockIdx.y;
  const int64_t C = (int64_t)H * d;
  const float* qv = aq + qi * C + (int64_t)h * d;
  const float sqrt_d = sqrtf((float)d);  // python float math.sqrt(D), used in fp32
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int e = threadIdx.x; e < d; e += blockDim.x) qsh[e] = qv[e];
  __syncthreads();
  // one thread per key block: the dot product in ascending e
  for (int64_t kj = threadIdx.x; kj < NK; kj += blockDim.x) {
    const float* kv = ak + kj * C + (int64_t)h * d;
    float acc = 0.f;
    for (int e = 0; e < d; ++e) acc = __fadd_rn(acc, __fmul_rn(qsh[e], __ldg(kv + e)));
    const float s = bf16r(__fdiv_rn(bf16r(acc), sqrt_d));
    const bool on = local[(qi % sq) * sk + (kj % sk)] != 0;
    sc[kj] = on ? s : -INFINITY;
  }
  __syncthreads();
  float m = -INFINITY;
  for (int64_t kj = threadIdx.x; kj < NK; kj += blockDim.x) m = fmaxf(m, sc[kj]);
  m = warp_max(m);
  if (lane == 0) red[wid] = m;
  __syncthreads();
  if (wid == 0) {
    float t = lane < nw ? red[lane] : -INFINITY;
    t = warp_max(t);
    if (lane == 0) red[0] = t;
  }
  __syncthreads();
  m = red[0];
  __syncthreads();
  for (int64_t kj = threadIdx.x; kj < NK; kj += blockDim.x)
    sc[kj] = (sc[kj] == -INFINITY) ? 0.f : (float)exp((double)__fsub_rn(sc[kj], m));
  __syncthreads();
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (int64_t kj = 0; kj < NK; ++kj) tot = __fadd_rn(tot, sc[kj]);
    red[0] = tot;
  }
  __syncthreads();
  const float tot = red[0];
  float* pr = prob + ((int64_t)h * NQ + qi) * NK;
  for (int64_t kj = threadIdx.x; kj < NK; kj += blockDim.x) pr[kj] = bf16r(__fdiv_rn(sc[kj], tot));
}

// ---------------------------------------------------------------------------
// a13 step 3: joint top-k per (head, query time row): threshold = the (k+1)-th
// largest probability of the flattened [per_row, NK] slab, keep = prob > thr.
// Probabilities are non-negative bf16 values, so their 16-bit patterns order
// like unsigned integers: a two-pass (high byte, low byte) radix select finds
// the exact threshold.  grid (q_temporal, H), block 1024.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) draft_topk_kernel(const float* __restrict__ prob,
                                                           int64_t NQ, int64_t NK,
                                                           int64_t per_row, int64_t topk,
                                                           uint8_t* __restrict__ keep) {
  __shared__ unsigned hist[256];
  __shared__ unsigned sel_hi, sel_lo, rank_left;
  const int64_t t = blockIdx.x;
  const int h = blockIdx.y;
  const int64_t n = per_row * NK;
  const float* p = prob + ((int64_t)h * NQ + t * per_row) * NK;
  uint8_t* kp = keep + ((int64_t)h * NQ + t * per_row) * NK;
  int64_t apply = topk < n - 1 ? topk : n - 1;
  if (apply < 0) apply = 0;
  const unsigned k = (unsigned)(apply + 1);  // 1-indexed rank from the top
  // pass 1: high byte
  for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    unsigned b = __float_as_uint(p[i]) >> 16;  // bf16 bit pattern
    atomicAdd(&hist[(b >> 8) & 0xFF], 1u);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned acc = 0, bin = 0;
    for (int b = 255; b >= 0; --b) {
      if (acc + hist[b] >= k) {
        bin = (unsigned)b;
        break;
      }
      acc += hist[b];
    }
    sel_hi = bin;
    rank_left = k - acc;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    unsigned b = __float_as_uint(p[i]) >> 16;
    if (((b >> 8) & 0xFF) == sel_hi) atomicAdd(&hist[b & 0xFF], 1u);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned acc = 0, bin = 0;
    for (int b = 255; b >= 0; --b) {
      if (acc + hist[b] >= rank_left) {
        bin = (unsigned)b;
        break;
      }
      acc += hist[b];
    }
    sel_lo = bin;
  }
  __syncthreads();
  const unsigned thr_bits = (sel_hi << 8) | sel_lo;
  const float thr = __uint_as_float(thr_bits << 16);
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) kp[i] = p[i] > thr ? 1 : 0;
}

// ---------------------------------------------------------------------------
// causal top-k rule (benchmark measurement input) from pooled fp32 means.
// grid (H, ceil(NQ / kTopkQ)), block 256: one CTA per head and group of kTopkQ query
// blocks, so a head's pooled keys cross L2 once per group, not once per query block.
//   1. the group's query vectors go to shared memory;
//   2. key rows stream through shared memory 128 at a time (16-byte asynchronous
//      copies, all in flight at once; a row pitch of d + 4 floats keeps the
//      per-thread 16-byte reads conflict-free);
//      thread (r, half) scores key row r against half of the group's queries;
//   3. warp w selects for query w: scores become order-preserving integer keys (held in
//      registers up to 256 past blocks), the nsel-th largest key is found bit by bit (32
//      warp-wide counts), and keys equal to it are taken in index order, so ties go to
//      the lower key index;
//   4. the warp writes the query's keep row: own time row, selected past blocks, never
//      a future row.
// ---------------------------------------------------------------------------
constexpr int kTopkThreads = 256;
constexpr int kTopkQ = 4;    // query blocks per CTA (one selecting warp each)
constexpr int kTopkKC = 128;  // key rows per shared-memory chunk

__device__ __forceinline__ uint32_t ordered_key(float s) {
  const uint32_t u = __float_as_uint(s + 0.0f);  // -0 -> +0: equal scores, equal keys
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__global__ void __launch_bounds__(kTopkThreads) causal_topk_kernel(
    const float* __restrict__ aq, const float* __restrict__ ak, int NQ, int NK, int H, int d,
    int per_row, float ratio, uint8_t* __restrict__ keep, int32_t* __restrict__ sel,
    int32_t* __restrict__ cnt) {
  extern __shared__ float4 dyn4[];
  const int h = blockIdx.x;
  const int q0 = blockIdx.y * kTopkQ;
  const int nq = min(kTopkQ, NQ - q0);
  const int pitch4 = (d >> 2) + 1;  // key row pitch in float4
  const int d4 = d >> 2;
  float4* qs4 = dyn4;                             // [kTopkQ][d4]
  float4* ks4 = qs4 + kTopkQ * d4;                // [kTopkKC][pitch4]
  uint32_t* key = reinterpret_cast<uint32_t*>(ks4 + kTopkKC * pitch4);  // [kTopkQ][NK]
  const int64_t C = (int64_t)H * d;
  const int cache_rows = (NK - NQ) / per_row;
  // past key blocks of the group's last query (the most any of its queries needs)
  const int np_max = (cache_rows + (q0 + nq - 1) / per_row) * per_row;

  for (int i = threadIdx.x; i < nq * d4; i += kTopkThreads) {
    const int qq = i / d4, e = i - qq * d4;
    cp_async16(qs4 + i, reinterpret_cast<const float4*>(aq + (int64_t)(q0 + qq) * C + (int64_t)h * d) + e);
  }
  const int r = threadIdx.x & (kTopkKC - 1);
  const int half = threadIdx.x / kTopkKC;  // queries half, half + 2, ...
  for (int k0 = 0; k0 < np_max; k0 += kTopkKC) {
    const int kn = min(kTopkKC, np_max - k0);
    __syncthreads();  // previous chunk fully read
    for (int i = threadIdx.x; i < kn * d4; i += kTopkThreads) {
      const int rr = i / d4, e = i - rr * d4;
      cp_async16(ks4 + rr * pitch4 + e,
                 reinterpret_cast<const float4*>(ak + (int64_t)(k0 + rr) * C + (int64_t)h * d) + e);
    }
    cp_async_wait_all();  // this thread's copies (and, first time, the query vectors)
    __syncthreads();
    if (r < kn) {
      float acc[kTopkQ / 2];
#pragma unroll
      for (int j = 0; j < kTopkQ / 2; ++j) acc[j] = 0.f;
      const float4* kr = ks4 + r * pitch4;
      for (int e = 0; e < d4; ++e) {
        const float4 kk = kr[e];
#pragma unroll
        for (int j = 0; j < kTopkQ / 2; ++j) {
          // ascending e, each product and sum rounded on its own (no FMA contraction):
          // the rule's defined evaluation order, restated exactly by the oracle
          const float4 qv = qs4[(half + 2 * j) * d4 + e];  // same address across the warp
          acc[j] = __fadd_rn(acc[j], __fmul_rn(qv.x, kk.x));
          acc[j] = __fadd_rn(acc[j], __fmul_rn(qv.y, kk.y));
          acc[j] = __fadd_rn(acc[j], __fmul_rn(qv.z, kk.z));
          acc[j] = __fadd_rn(acc[j], __fmul_rn(qv.w, kk.w));
        }
      }
#pragma unroll
      for (int j = 0; j < kTopkQ / 2; ++j) {
        const int qq = half + 2 * j;
        if (qq < nq) key[qq * NK + k0 + r] = ordered_key(acc[j]);
      }
    }
  }
  cp_async_wait_all();  // np_max == 0: the query copies were never waited for
  __syncthreads();
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (w >= nq) return;
  const int qi = q0 + w;
  const int qrow = cache_rows + qi / per_row;
  const int npast = qrow * per_row;
  const int nsel = (int)floorf(ratio * (float)npast);
  const uint32_t* kq = key + w * NK;
  // largest T with #{key >= T} >= nsel, i.e. the nsel-th largest key; up to 256 past
  // blocks the keys stay in registers (8 per lane), beyond that they are re-read
  uint32_t T = 0;
  constexpr int kRegKeys = 8;
  uint32_t kr[kRegKeys];
#pragma unroll
  for (int t = 0; t < kRegKeys; ++t) {
    const int i = lane + 32 * t;
    kr[t] = i < npast ? kq[i] : 0u;  // 0 is below every key of a finite score
  }
  const bool in_regs = npast <= 32 * kRegKeys;
  if (nsel > 0) {
    for (int b = 31; b >= 0; --b) {
      const uint32_t cand = T | (1u << b);
      int c = 0;
      if (in_regs) {
#pragma unroll
        for (int t = 0; t < kRegKeys; ++t) c += kr[t] >= cand;
      } else {
        for (int i = lane; i < npast; i += 32) c += kq[i] >= cand;
      }
      if ((int)__reduce_add_sync(0xffffffffu, (unsigned)c) >= nsel) T = cand;
    }
  }
  int gt = 0;
  for (int i = lane; i < npast; i += 32) gt += kq[i] > T;
  const int need = nsel - (int)__reduce_add_sync(0xffffffffu, (unsigned)gt);  // ties to keep
  const int64_t orow = (int64_t)h * NQ + qi;
  const unsigned lt = (1u << lane) - 1u;
  // whether key block k0 + lane is kept (every lane calls it for the same k0, in order:
  // ties are kept in ascending index order up to `need`)
  auto kept_of = [&](int k0, int& eq_before) {
    const int kj = k0 + lane;
    const bool past = kj < npast;
    const uint32_t kv = past ? kq[kj] : 0u;
    const bool eq = past && nsel > 0 && kv == T;
    const unsigned bal = __ballot_sync(0xffffffffu, eq);
    const bool tie_kept = eq && (eq_before + __popc(bal & lt)) < need;
    eq_before += __popc(bal);
    return kj < NK && ((kj / per_row == qrow) || (past && nsel > 0 && (kv > T || tie_kept)));
  };
  int eq_before = 0, base = 0;
  int32_t* sr = sel ? sel + orow * NK : nullptr;
  for (int k0 = 0; k0 < NK; k0 += 32) {
    const int kj = k0 + lane;
    const bool kept = kept_of(k0, eq_before);
    if (keep && kj < NK) keep[orow * NK + kj] = kept ? 1 : 0;
    if (sr) {  // CSR of the row (fvb_mask_to_csr's order): kept ids ascending ...
      const unsigned bal = __ballot_sync(0xffffffffu, kept);
      if (kept) sr[base + __popc(bal & lt)] = kj;
      base += __popc(bal);
    }
  }
  if (sr) {
    if (lane == 0) cnt[orow] = base;
    eq_before = 0;  // ... then the unkept ids ascending (the same decisions, recomputed)
    for (int k0 = 0; k0 < NK; k0 += 32) {
      const int kj = k0 + lane;
      const bool off = !kept_of(k0, eq_before) && kj < NK;
      const unsigned bal = __ballot_sync(0xffffffffu, off);
      if (off) sr[base + __popc(bal & lt)] = kj;
      base += __popc(bal);
    }
  }
}

// query vectors + one key chunk (padded rows) + the group's integer score keys
static size_t causal_topk_smem(int64_t NK, int64_t d) {
  return ((size_t)kTopkQ * (d / 4) + (size_t)kTopkKC * (d / 4 + 1)) * 16 + (size_t)kTopkQ * NK * 4;
}

static int launch_causal_topk(const float* aq, const float* ak, int64_t H, int64_t NQ, int64_t NK,
                              int64_t d, int64_t per_row, float ratio, uint8_t* keep,
                              cudaStream_t st, int32_t* sel = nullptr, int32_t* cnt = nullptr) {
  const size_t smem = causal_topk_smem(NK, d);
  if (smem > 48 * 1024)
    FVB_CUDA_TRY(cudaFuncSetAttribute(causal_topk_kernel,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                 "causal_topk smem");
  causal_topk_kernel<<<dim3((unsigned)H, (unsigned)((NQ + kTopkQ - 1) / kTopkQ)), kTopkThreads,
                       smem, st>>>(aq, ak, (int)NQ, (int)NK, (int)H, (int)d, (int)per_row, ratio,
                                   keep, sel, cnt);
  return check_launch("fvb_causal_topk_mask");
}

static inline unsigned warp_rows_grid(int64_t rows) { return (unsigned)((rows + 7) / 8); }

}  // namespace fvb

extern "C" {

int fvb_window_partition(const void* x, int64_t x_ld, int64_t B, int64_t F, int64_t Hh,
                         int64_t Ww, int64_t C, int wf, int wh, int ww, int reverse, void* out,
                         fvb_stream_t stream) {
  using namespace fvb;
  if (x_ld == 0) x_ld = C;
  FVB_REQUIRE(B >= 0 && F >= 0 && Hh >= 0 && Ww >= 0 && C > 0, "fvb_window_partition: shape");
  FVB_REQUIRE(wf > 0 && wh > 0 && ww > 0 && F % wf == 0 && Hh % wh == 0 && Ww % ww == 0,
              "fvb_window_partition: (F,H,W)=(%lld,%lld,%lld) not divisible by window (%d,%d,%d)",
              (long long)F, (long long)Hh, (long long)Ww, wf, wh, ww);
  FVB_REQUIRE(C % 8 == 0 && x_ld >= C && x_ld % 8 == 0,
              "fvb_window_partition: C and x_ld must be multiples of 8, x_ld >= C");
  const int64_t rows = B * F * Hh * Ww;
  if (rows == 0) return FVB_OK;
  FVB_REQUIRE(x && out && aligned16(x) && aligned16(out), "fvb_window_partition: pointers");
  FVB_REQUIRE(x != out, "fvb_window_partition: in-place not supported");
  window_kernel<<<warp_rows_grid(rows), 256, 0, (cudaStream_t)stream>>>(
      (const uint4*)x, x_ld / 8, rows, F, Hh, Ww, C / 8, wf, wh, ww, reverse, (uint4*)out);
  return check_launch("fvb_window_partition");
}

int fvb_mask_to_csr(const uint8_t* keep, int64_t H, int64_t NQ, int64_t NK, int32_t* sel,
                    int32_t* cnt, fvb_stream_t stream) {
  using namespace fvb;
  FVB_REQUIRE(H >= 0 && NQ >= 0 && NK >= 0, "fvb_mask_to_csr: shape");
  const int64_t rows = H * NQ;
  if (rows == 0) return FVB_OK;
  FVB_REQUIRE(keep && sel && cnt, "fvb_mask_to_csr: NULL pointer");
  mask_to_csr_kernel<<<warp_rows_grid(rows), 256, 0, (cudaStream_t)stream>>>(keep, rows, NK, sel,
                                                                             cnt);
  return check_launch("fvb_mask_to_csr");
}

size_t fvb_draft_mask_workspace_bytes(int64_t H, int64_t NQ, int64_t NK, int64_t d) {
  // pooled q [NQ, H*d] + pooled k [NK, H*d] + probabilities [H, NQ, NK], fp32
  size_t b = (size_t)(NQ + NK) * H * d * 4 + (size_t)H * NQ * NK * 4;
  return (b + 255) & ~(size_t)255;
}

int fvb_draft_block_mask(const void* q_w, const void* k_w, int64_t H, int64_t NQ, int64_t NK,
                         int64_t d, const uint8_t* local, int64_t sq, int64_t sk,
                         int64_t q_temporal, int64_t topk, uint8_t* keep, void* workspace,
                         fvb_stream_t stream) {
  using namespace fvb;
  cudaStream_t st = (cudaStream_t)stream;
  FVB_REQUIRE(H > 0 && NQ > 0 && NK > 0 && d > 0 && (H * d) % 8 == 0, "fvb_draft_block_mask: shape");
  FVB_REQUIRE(sq > 0 && sk > 0 && NQ % sq == 0 && NK % sk == 0,
              "fvb_draft_block_mask: local mask [%lld,%lld] must tile [%lld,%lld]", (long long)sq,
              (long long)sk, (long long)NQ, (long long)NK);
  FVB_REQUIRE(q_temporal > 0 && NQ % q_temporal == 0, "fvb_draft_block_mask: q_temporal");
  FVB_REQUIRE(q_w && k_w && local && keep && workspace, "fvb_draft_block_mask: NULL pointer");
  FVB_REQUIRE(aligned16(q_w) && aligned16(k_w), "fvb_draft_block_mask: alignment");
  FVB_REQUIRE(NK * 4 <= 200 * 1024, "fvb_draft_block_mask: NK too large");
  FVB_REQUIRE(d <= 256, "fvb_draft_block_mask: head_dim %lld > 256", (long long)d);
  const int64_t C = H * d;
  float* aq = static_cast<float*>(workspace);
  float* ak = aq + NQ * C;
  float* prob = ak + NK * C;
  pool_kernel<false><<<dim3((unsigned)NQ, (unsigned)((C + 511) / 512)), 256, 0, st>>>((const __nv_bfloat16*)q_w, NQ, C, 1, aq);
  pool_kernel<false><<<dim3((unsigned)NK, (unsigned)((C + 511) / 512)), 256, 0, st>>>((const __nv_bfloat16*)k_w, NK, C, 1, ak);
  int rc = check_launch("fvb_draft_block_mask pool");
  if (rc) return rc;
  const size_t smem = (size_t)NK * 4;
  if (smem > 48 * 1024)
    FVB_CUDA_TRY(cudaFuncSetAttribute(draft_scores_kernel,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                 "draft_scores smem");
  draft_scores_kernel<<<dim3((unsigned)NQ, (unsigned)H), 256, smem, st>>>(
      aq, ak, NQ, NK, (int)H, (int)d, local, sq, sk, prob);
  rc = check_launch("fvb_draft_block_mask scores");
  if (rc) return rc;
  draft_topk_kernel<<<dim3((unsigned)q_temporal, (unsigned)H), 1024, 0, st>>>(
      prob, NQ, NK, NQ / q_temporal, topk, keep);
  return check_launch("fvb_draft_block_mask topk");
}

int fvb_causal_topk_mask(const void* q_w, const void* k_w, int64_t H, int64_t NQ, int64_t NK,
                         int64_t d, int64_t per_row, float ratio, uint8_t* keep, void* workspace,
                         fvb_stream_t stream) {
  using namespace fvb;
  cudaStream_t st = (cudaStream_t)stream;
  FVB_REQUIRE(H > 0 && NQ > 0 && NK >= NQ && d > 0 && d % 4 == 0 && (H * d) % 8 == 0,
              "fvb_causal_topk_mask: shape");
  FVB_REQUIRE(per_row > 0 && NQ % per_row == 0 && NK % per_row == 0,
              "fvb_causal_topk_mask: blocks per time row must divide NQ and NK");
  FVB_REQUIRE(q_w && k_w && keep && workspace, "fvb_causal_topk_mask: NULL pointer");
  FVB_REQUIRE(aligned16(q_w) && aligned16(k_w), "fvb_causal_topk_mask: alignment");
  FVB_REQUIRE(NK < (1ll << 31) / H && causal_topk_smem(NK, d) <= 200 * 1024,
              "fvb_causal_topk_mask: NK or d too large");
  const int64_t C = H * d;
  float* aq = static_cast<float*>(workspace);
  float* ak = aq + NQ * C;
  pool_kernel<false><<<dim3((unsigned)NQ, (unsigned)((C + 511) / 512)), 256, 0, st>>>((const __nv_bfloat16*)q_w, NQ, C, 0, aq);
  pool_kernel<false><<<dim3((unsigned)NK, (unsigned)((C + 511) / 512)), 256, 0, st>>>((const __nv_bfloat16*)k_w, NK, C, 0, ak);
  int rc = check_launch("fvb_causal_topk_mask pool");
  if (rc) return rc;
  return launch_causal_topk(aq, ak, H, NQ, NK, d, per_row, ratio, keep, st);
}

int fvb_block_mean_pool(const void* x, int64_t nblk, int64_t C, float* out, fvb_stream_t stream) {
  using namespace fvb;
  FVB_REQUIRE(nblk >= 0 && C > 0 && C % 8 == 0, "fvb_block_mean_pool: shape");
  if (nblk == 0) return FVB_OK;
  FVB_REQUIRE(x && out && aligned16(x), "fvb_block_mean_pool: pointers");
  pool_kernel<false><<<dim3((unsigned)nblk, (unsigned)((C + 511) / 512)), 256, 0, (cudaStream_t)stream>>>(
      (const __nv_bfloat16*)x, nblk, C, 0, out);
  return check_launch("fvb_block_mean_pool");
}

int fvb_causal_topk_pooled_csr(const float* aq, const float* ak, int64_t H, int64_t NQ,
                               int64_t NK, int64_t d, int64_t per_row, float ratio,
                               uint8_t* keep, int32_t* sel, int32_t* cnt, fvb_stream_t stream) {
  using namespace fvb;
  FVB_REQUIRE(H > 0 && NQ > 0 && NK >= NQ && d > 0 && d % 4 == 0,
              "fvb_causal_topk_pooled_csr: shape");
  FVB_REQUIRE(per_row > 0 && NQ % per_row == 0 && NK % per_row == 0,
              "fvb_causal_topk_pooled_csr: blocks per time row must divide NQ and NK");
  FVB_REQUIRE(aq && ak && sel && cnt && aligned16(aq) && aligned16(ak),
              "fvb_causal_topk_pooled_csr: pointers");
  FVB_REQUIRE(NK < (1ll << 31) / H && causal_topk_smem(NK, d) <= 200 * 1024,
              "fvb_causal_topk_pooled_csr: NK or d too large");
  return launch_causal_topk(aq, ak, H, NQ, NK, d, per_row, ratio, keep, (cudaStream_t)stream,
                            sel, cnt);
}

int fvb_block_mean_pool2(const void* x, int64_t nblk, const void* x2, int64_t nblk2, int64_t C,
                         float* out, float* out2, fvb_stream_t stream) {
  using namespace fvb;
  FVB_REQUIRE(nblk >= 0 && nblk2 >= 0 && C > 0 && C % 8 == 0, "fvb_block_mean_pool2: shape");
  FVB_REQUIRE(nblk + nblk2 < (1ll << 31), "fvb_block_mean_pool2: too many windows");
  if (nblk + nblk2 == 0) return FVB_OK;
  FVB_REQUIRE((nblk == 0 || (x && out && aligned16(x))) && (nblk2 == 0 || (x2 && out2 && aligned16(x2))),
              "fvb_block_mean_pool2: pointers");
  pool_kernel<true><<<dim3((unsigned)(nblk + nblk2), (unsigned)((C + 511) / 512)), 256, 0,
                      (cudaStream_t)stream>>>((const __nv_bfloat16*)x, nblk, C, 0, out,
                                              (const __nv_bfloat16*)x2, out2);
  return check_launch("fvb_block_mean_pool2");
}

int fvb_causal_topk_pooled(const float* aq, const float* ak, int64_t H, int64_t NQ, int64_t NK,
                           int64_t d, int64_t per_row, float ratio, uint8_t* keep,
                           fvb_stream_t stream) {
  using namespace fvb;
  FVB_REQUIRE(H > 0 && NQ > 0 && NK >= NQ && d > 0 && d % 4 == 0,
              "fvb_causal_topk_pooled: shape");
  FVB_REQUIRE(per_row > 0 && NQ % per_row == 0 && NK % per_row == 0,
              "fvb_causal_topk_pooled: blocks per time row must divide NQ and NK");
  FVB_REQUIRE(aq && ak && keep && aligned16(aq) && aligned16(ak), "fvb_causal_topk_pooled: pointers");
  FVB_REQUIRE(NK < (1ll << 31) / H && causal_topk_smem(NK, d) <= 200 * 1024,
              "fvb_causal_topk_pooled: NK or d too large");
  return launch_causal_topk(aq, ak, H, NQ, NK, d, per_row, ratio, keep, (cudaStream_t)stream);
}

}  // extern "C"
