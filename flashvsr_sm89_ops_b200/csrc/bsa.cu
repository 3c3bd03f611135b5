// Block-sparse flash attention over 128-token windows on the 5th-generation
// tensor cores (a12).  Semantics of lcsa/triton_lcsa.py:19-61: for head h and
// query block qb, online softmax over the key blocks sel[h,qb,0:cnt[h,qb]]
// (128 keys each), scores * scale, fp32 statistics, P rounded to bf16 for the
// P.V product, rows without any kept block output 0.
//
// One CTA per (query block, head), 320 threads:
//   warps 0-7   softmax / accumulate.  Warpgroup g (warps 4g..4g+3) owns key
//               columns [64g, 64g+64) of S and value columns [64g, 64g+64) of
//               O; thread (warp%4, lane) owns query row 32*(warp%4)+lane.  The
//               two halves of a row exchange their partial max through shared
//               memory each key block; partial row sums combine at the end.
//   warp 8      TMA producer: Q once, then K and V tiles of each kept block
//               into a 2-stage ring (128-byte swizzle, 64-column boxes).
//   warp 9      MMA issuer: S_j = Q K_j^T (kind::f16, M=N=K=128) into one of
//               two TMEM S buffers, O_j = P_j V_j into one of two TMEM O
//               buffers; allocates / frees 512 TMEM columns.
// Pipelining: S_{j+1} is issued before O_j so the tensor core computes the
// next scores while the softmax warps work on block j.  O_j is accumulated
// into registers (acc = acc * alpha_j + O_j), so no rescale of TMEM is ever
// needed and every TMEM buffer has exactly one producer and one consumer.
#include <cstdlib>

#include "common.cuh"

namespace fvb {
namespace bsa {

constexpr int kThreads = 320;
constexpr int kSoftmaxThreads = 256;
constexpr int kTile = 128;                   // rows per block, head_dim
constexpr int kAtom = 128 * 128;             // one 64-column swizzle atom: 128 rows x 128 B
constexpr int kTileBytes = 2 * kAtom;        // 128 x 128 bf16 = 32 KB (two 64-column atoms)

struct Args {
  const int32_t* sel;
  const int32_t* cnt;
  int64_t sel_stride;
  int H, NQ, Lq, kv_len;
  float scale_log2;
  const int32_t* row_map;
  __nv_bfloat16* out;
  int64_t ldo;  // H * 128
};

constexpr size_t kSmemBytes = (size_t)kTileBytes * (1 /*Q*/ + 2 /*K*/ + 2 /*V*/ + 1 /*P*/) +
                              1024 /*align*/ + 4096 /*barriers + exchange*/;

__global__ void __launch_bounds__(kThreads, 1)
    bsa_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const Args args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~(uintptr_t)1023);
  uint8_t* sQ = base;
  uint8_t* sK = sQ + kTileBytes;        // 2 stages
  uint8_t* sV = sK + 2 * kTileBytes;    // 2 stages
  uint8_t* sP = sV + 2 * kTileBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + kTileBytes);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;    // [2]
  uint64_t* v_full = bars + 3;    // [2]
  uint64_t* kv_empty = bars + 5;  // [2]
  uint64_t* s_full = bars + 7;    // [2]
  uint64_t* s_empty = bars + 9;   // [2]
  uint64_t* p_full = bars + 11;
  uint64_t* o_full = bars + 12;   // [2]
  uint64_t* o_empty = bars + 14;  // [2]
  uint64_t* x_bar = bars + 16;    // [2] max exchange
  uint64_t* l_bar = bars + 18;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 20);
  float* xmax = reinterpret_cast<float*>(bars + 24);  // [2 parity][2 halves][128]
  float* xl = xmax + 2 * 2 * 128;                     // [2 halves][128]

  const int warp = warp_id_uniform();
  const int lane = threadIdx.x & 31;
  const int qb = blockIdx.x;
  const int h = blockIdx.y;
  const int64_t rowid = (int64_t)h * args.NQ + qb;
  const int cnt = __ldg(args.cnt + rowid);
  const int32_t* sel = args.sel + rowid * args.sel_stride;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 8);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_empty[i], 8);
      mbar_init(&x_bar[i], kSoftmaxThreads);
    }
    mbar_init(p_full, 8);
    mbar_init(l_bar, kSoftmaxThreads);
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // TMEM columns: S buffers at 0 / 128, O buffers at 256 / 384
  const int col_q = h * kTile;

  if (warp == 8) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && cnt > 0) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      mbar_arrive_expect_tx(q_full, kTileBytes);
      tma_load_2d(sQ, &tmQ, q_full, col_q, qb * kTile);
      tma_load_2d(sQ + kAtom, &tmQ, q_full, col_q + 64, qb * kTile);
      for (int j = 0; j < cnt; ++j) {
        const int st = j & 1;
        const uint32_t ph = (uint32_t)(j >> 1) & 1u;
        if (!mbar_wait(&kv_empty[st], ph ^ 1u, 0x201u)) break;
        const int krow = __ldg(sel + j) * kTile;
        mbar_arrive_expect_tx(&k_full[st], kTileBytes);
        tma_load_2d(sK + st * kTileBytes, &tmK, &k_full[st], col_q, krow);
        tma_load_2d(sK + st * kTileBytes + kAtom, &tmK, &k_full[st], col_q + 64, krow);
        mbar_arrive_expect_tx(&v_full[st], kTileBytes);
        tma_load_2d(sV + st * kTileBytes, &tmV, &v_full[st], col_q, krow);
        tma_load_2d(sV + st * kTileBytes + kAtom, &tmV, &v_full[st], col_q + 64, krow);
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && cnt > 0) {
      constexpr uint32_t idesc_s = make_idesc(1 /*bf16*/, 1 /*bf16*/, 0, 0, 128, 128);
      constexpr uint32_t idesc_o = make_idesc(1, 1, 0 /*P K-major*/, 1 /*V MN-major*/, 128, 128);
      const uint32_t q0 = smem_u32(sQ);
      const uint32_t p0 = smem_u32(sP);
      bool ok = mbar_wait(q_full, 0, 0x202u);
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1;
        const uint32_t ph = (uint32_t)(j >> 1) & 1u;
        if (!mbar_wait(&k_full[st], ph, 0x203u)) return false;
        if (!mbar_wait(&s_empty[st], ph ^ 1u, 0x204u)) return false;
        tc_fence_after();
        const uint32_t k0 = smem_u32(sK + st * kTileBytes);
        const uint32_t d = tmem + (uint32_t)(st * 128);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (uint32_t)((kk >> 2) * kAtom + (kk & 3) * 32);
          mma_f16(d, smem_desc_sw128(q0 + off, 16, 1024), smem_desc_sw128(k0 + off, 16, 1024),
                  idesc_s, kk > 0 ? 1u : 0u);
        }
        tc_commit(&s_full[st]);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; j < cnt && ok; ++j) {
        if (j + 1 < cnt && !issue_s(j + 1)) break;
        const int st = j & 1;
        const uint32_t ph = (uint32_t)(j >> 1) & 1u;
        if (!mbar_wait(p_full, (uint32_t)j & 1u, 0x205u)) break;
        if (!mbar_wait(&v_full[st], ph, 0x206u)) break;
        if (!mbar_wait(&o_empty[st], ph ^ 1u, 0x207u)) break;
        tc_fence_after();
        const uint32_t v0 = smem_u32(sV + st * kTileBytes);
        const uint32_t d = tmem + 256u + (uint32_t)(st * 128);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t aoff = (uint32_t)((kk >> 2) * kAtom + (kk & 3) * 32);
          mma_f16(d, smem_desc_sw128(p0 + aoff, 16, 1024),
                  smem_desc_sw128(v0 + (uint32_t)(kk * 16 * 128), (uint32_t)kAtom, 1024), idesc_o,
                  kk > 0 ? 1u : 0u);
        }
        tc_commit(&o_full[st]);
        tc_commit(&kv_empty[st]);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax warps
    const int g = warp >> 2;        // column half
    const int qr = warp & 3;        // TMEM lane quarter
    const int row = qr * 32 + lane;  // query row within the block
    const uint32_t lane_addr = (uint32_t)(qr * 32) << 16;
    float acc[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) acc[i] = 0.f;
    float m = -INFINITY, l = 0.f, alpha_prev = 1.f;
    bool ok = true;
    uint8_t* prow = sP + g * kAtom + row * 128;
    for (int j = 0; j < cnt; ++j) {
      const int st = j & 1;
      const uint32_t ph = (uint32_t)(j >> 1) & 1u;
      if (!mbar_wait(&s_full[st], ph, 0x208u)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[64];
      {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem + lane_addr + (uint32_t)(st * 128 + g * 64), r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) s[i] = __uint_as_float(r[i]);
        tmem_ld_32x32b_x32(tmem + lane_addr + (uint32_t)(st * 128 + g * 64 + 32), r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) s[32 + i] = __uint_as_float(r[i]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[st]);
      // scale into the log2 domain, mask keys past kv_len
      const int key0 = __ldg(sel + j) * kTile + g * 64;
      float pm = -INFINITY;
      if (key0 + 64 <= args.kv_len) {
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          s[i] *= args.scale_log2;
          pm = fmaxf(pm, s[i]);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          s[i] = (key0 + i < args.kv_len) ? s[i] * args.scale_log2 : -INFINITY;
          pm = fmaxf(pm, s[i]);
        }
      }
      // exchange the partial max with the other half of the row
      float* xm = xmax + st * 256;
      xm[g * 128 + row] = pm;
      mbar_arrive(&x_bar[st]);
      if (!mbar_wait(&x_bar[st], ph, 0x209u)) {
        ok = false;
        break;
      }
      const float m_new = fmaxf(m, fmaxf(pm, xm[(g ^ 1) * 128 + row]));
      float alpha, msub;
      if (m_new == -INFINITY) {  // nothing visible yet in this row
        alpha = 1.f;
        msub = 0.f;
      } else {
        alpha = exp2f(m - m_new);
        msub = m_new;
      }
      uint32_t pk[32];
      float ls = 0.f;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float p0 = exp2f(s[2 * i] - msub);
        const float p1 = exp2f(s[2 * i + 1] - msub);
        ls += p0 + p1;
        __nv_bfloat162 b2 = __floats2bfloat162_rn(p0, p1);
        pk[i] = *reinterpret_cast<uint32_t*>(&b2);
      }
      l = l * alpha + ls;
      // fold in O_{j-1}; its completion also frees the P buffer
      if (j > 0) {
        const int ps = (j - 1) & 1;
        const uint32_t pph = (uint32_t)((j - 1) >> 1) & 1u;
        if (!mbar_wait(&o_full[ps], pph, 0x20Au)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem + lane_addr + (uint32_t)(256 + ps * 128 + g * 64), r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[i] = __fmaf_rn(acc[i], alpha_prev, __uint_as_float(r[i]));
        tmem_ld_32x32b_x32(tmem + lane_addr + (uint32_t)(256 + ps * 128 + g * 64 + 32), r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i)
          acc[32 + i] = __fmaf_rn(acc[32 + i], alpha_prev, __uint_as_float(r[i]));
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&o_empty[ps]);
      }
      alpha_prev = alpha;
      // P_j (bf16, 64 keys of this half) into the swizzled K-major A operand
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint4 v = make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
        *reinterpret_cast<uint4*>(prow + ((c ^ (row & 7)) << 4)) = v;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
      m = m_new;
    }
    if (ok && cnt > 0) {
      const int ps = (cnt - 1) & 1;
      const uint32_t pph = (uint32_t)((cnt - 1) >> 1) & 1u;
      if (mbar_wait(&o_full[ps], pph, 0x20Bu)) {
        tc_fence_after();
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem + lane_addr + (uint32_t)(256 + ps * 128 + g * 64), r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[i] = __fmaf_rn(acc[i], alpha_prev, __uint_as_float(r[i]));
        tmem_ld_32x32b_x32(tmem + lane_addr + (uint32_t)(256 + ps * 128 + g * 64 + 32), r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i)
          acc[32 + i] = __fmaf_rn(acc[32 + i], alpha_prev, __uint_as_float(r[i]));
      } else {
        ok = false;
      }
    }
    // combine the two partial row sums
    float lt = 0.f;
    if (ok) {
      xl[g * 128 + row] = l;
      mbar_arrive(l_bar);
      if (mbar_wait(l_bar, 0, 0x20Cu)) lt = l + xl[(g ^ 1) * 128 + row];
    }
    const float inv = lt > 0.f ? 1.0f / lt : 0.f;
    const int qrow = qb * kTile + row;
    if (qrow < args.Lq) {
      const int64_t orow = args.row_map ? (int64_t)__ldg(args.row_map + qrow) : (int64_t)qrow;
      uint4* dst = reinterpret_cast<uint4*>(args.out + orow * args.ldo + col_q + g * 64);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        float f[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) f[i] = acc[8 * c + i] * inv;
        dst[c] = f32_to_bf16x8(f);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace bsa

// ===========================================================================
// v2: two CTAs per SM, P and O kept in tensor memory.
//
// Per CTA (one query block of 128 rows, one head): Q, one K and one V tile in
// shared memory (96 KB), 256 TMEM columns: S/P at [0,128), O at [128,256).
//   * S_j = Q K_j^T lands in the S columns; the softmax warps read it, and write
//     P_j = exp2(S*c - m) as packed bf16 over the first 64 of those columns
//     (tcgen05.st); the P.V product then takes A straight from TMEM
//     (tcgen05.mma ... [d], [a_tmem], b_desc) and accumulates into O.
//   * O stays in TMEM for the whole key loop.  The running max used for the
//     exponentials is only raised when a block's max exceeds it by more than
//     2^8 (lazy rescale); then O and the row sum are rescaled in place.  At that
//     moment every earlier MMA has completed (the S_j commit tracks them), so no
//     extra synchronisation is needed.
//   * A CTA runs S_j -> softmax_j -> PV_j serially; the second resident CTA fills
//     the tensor core while this one is in softmax, and vice versa.
// ===========================================================================
namespace bsa2 {

constexpr int kThreads = 320;
constexpr int kSoftmaxThreads = 256;
constexpr int kTile = 128;
constexpr int kAtom = 128 * 128;
constexpr int kTileBytes = 2 * kAtom;
constexpr float kLazy = 8.0f;  // log2 units: rescale only when the max grows by > 2^8

constexpr size_t kSmemBytes = (size_t)kTileBytes * 3 + 1024 /*align*/ + 3072 /*bars + xchg*/;

__global__ void __launch_bounds__(kThreads, 2)
    bsa_fwd_v2_kernel(const __grid_constant__ CUtensorMap tmQ,
                      const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, const bsa::Args args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~(uintptr_t)1023);
  uint8_t* sQ = base;
  uint8_t* sK = sQ + kTileBytes;
  uint8_t* sV = sK + kTileBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + kTileBytes);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = bars + 2;
  uint64_t* v_full = bars + 3;
  uint64_t* v_empty = bars + 4;
  uint64_t* s_full = bars + 5;
  uint64_t* p_full = bars + 6;
  uint64_t* pv_done = bars + 7;
  uint64_t* x_bar = bars + 8;  // [2]
  uint64_t* l_bar = bars + 10;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);
  float* xmax = reinterpret_cast<float*>(bars + 16);  // [2 parity][2 halves][128]
  float* xl = xmax + 2 * 2 * 128;                     // [2 halves][128]

  const int warp = warp_id_uniform();
  const int lane = threadIdx.x & 31;
  const int qb = blockIdx.x;
  const int h = blockIdx.y;
  const int64_t rowid = (int64_t)h * args.NQ + qb;
  const int cnt = __ldg(args.cnt + rowid);
  const int32_t* sel = args.sel + rowid * args.sel_stride;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(k_full, 1);
    mbar_init(k_empty, 1);
    mbar_init(v_full, 1);
    mbar_init(v_empty, 1);
    mbar_init(s_full, 1);
    mbar_init(p_full, 8);
    mbar_init(pv_done, 1);
    mbar_init(&x_bar[0], kSoftmaxThreads);
    mbar_init(&x_bar[1], kSoftmaxThreads);
    mbar_init(l_bar, kSoftmaxThreads);
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem;         // S / P
  const uint32_t tO = tmem + 128;   // O
  const int col_q = h * kTile;

  if (warp == 8) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && cnt > 0) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      mbar_arrive_expect_tx(q_full, kTileBytes);
      tma_load_2d(sQ, &tmQ, q_full, col_q, qb * kTile);
      tma_load_2d(sQ + kAtom, &tmQ, q_full, col_q + 64, qb * kTile);
      for (int j = 0; j < cnt; ++j) {
        const uint32_t ph = (uint32_t)j & 1u;
        const int krow = __ldg(sel + j) * kTile;
        if (!mbar_wait(k_empty, ph ^ 1u, 0x301u)) break;
        mbar_arrive_expect_tx(k_full, kTileBytes);
        tma_load_2d(sK, &tmK, k_full, col_q, krow);
        tma_load_2d(sK + kAtom, &tmK, k_full, col_q + 64, krow);
        if (!mbar_wait(v_empty, ph ^ 1u, 0x302u)) break;
        mbar_arrive_expect_tx(v_full, kTileBytes);
        tma_load_2d(sV, &tmV, v_full, col_q, krow);
        tma_load_2d(sV + kAtom, &tmV, v_full, col_q + 64, krow);
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && cnt > 0) {
      constexpr uint32_t idesc_s = make_idesc(1 /*bf16*/, 1 /*bf16*/, 0, 0, 128, 128);
      constexpr uint32_t idesc_o = make_idesc(1, 1, 0 /*P K-major*/, 1 /*V MN-major*/, 128, 128);
      const uint32_t q0 = smem_u32(sQ);
      const uint32_t k0 = smem_u32(sK);
      const uint32_t v0 = smem_u32(sV);
      bool ok = mbar_wait(q_full, 0, 0x303u);
      for (int j = 0; j < cnt && ok; ++j) {
        const uint32_t ph = (uint32_t)j & 1u;
        if (!mbar_wait(k_full, ph, 0x304u)) break;
        // S/P columns are reused: P_{j-1} must have been consumed by PV_{j-1}
        if (j > 0 && !mbar_wait(pv_done, ph ^ 1u, 0x305u)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (uint32_t)((kk >> 2) * kAtom + (kk & 3) * 32);
          mma_f16(tS, smem_desc_sw128(q0 + off, 16, 1024), smem_desc_sw128(k0 + off, 16, 1024),
                  idesc_s, kk > 0 ? 1u : 0u);
        }
        tc_commit(s_full);
        tc_commit(k_empty);
        if (!mbar_wait(p_full, ph, 0x306u)) break;
        if (!mbar_wait(v_full, ph, 0x307u)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          // keys [16kk, 16kk+16): P of half g sits in columns [64g, 64g+32) of the S region
          const uint32_t pcol = (uint32_t)((kk >> 2) * 64 + (kk & 3) * 8);
          mma_f16_ts(tO, tS + pcol,
                     smem_desc_sw128(v0 + (uint32_t)(kk * 16 * 128), (uint32_t)kAtom, 1024),
                     idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
        }
        tc_commit(pv_done);
        tc_commit(v_empty);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax warps
    const int g = warp >> 2;         // key / value column half
    const int qr = warp & 3;         // TMEM lane quarter
    const int row = qr * 32 + lane;  // query row within the block
    const uint32_t lane_addr = (uint32_t)(qr * 32) << 16;
    const float c = args.scale_log2;
    float m_used = -INFINITY;  // max (log2 domain) the exponentials are taken against
    float l = 0.f;
    bool ok = true;
    for (int j = 0; j < cnt; ++j) {
      const uint32_t ph = (uint32_t)j & 1u;
      if (!mbar_wait(s_full, ph, 0x308u)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t s[64];
      tmem_ld_32x32b_x32(tS + lane_addr + (uint32_t)(g * 64), s);
      tmem_ld_32x32b_x32(tS + lane_addr + (uint32_t)(g * 64 + 32), s + 32);
      tmem_ld_wait();
      const int key0 = __ldg(sel + j) * kTile + g * 64;
      if (key0 + 64 > args.kv_len) {
#pragma unroll
        for (int i = 0; i < 64; ++i)
          if (key0 + i >= args.kv_len) s[i] = __float_as_uint(-INFINITY);
      }
      float pm = -INFINITY;
#pragma unroll
      for (int i = 0; i < 64; ++i) pm = fmaxf(pm, __uint_as_float(s[i]));
      float* xm = xmax + (j & 1) * 256;
      xm[g * 128 + row] = pm;
      mbar_arrive(&x_bar[j & 1]);
      if (!mbar_wait(&x_bar[j & 1], (uint32_t)(j >> 1) & 1u, 0x309u)) {
        ok = false;
        break;
      }
      const float mb = fmaxf(pm, xm[(g ^ 1) * 128 + row]) * c;  // block max, log2 domain
      float alpha = 1.f;
      const bool raise = mb > m_used + kLazy;  // also true for the first finite block
      if (raise) {
        alpha = (m_used == -INFINITY) ? 0.f : ex2_approx(m_used - mb);
        m_used = mb;
      }
      // P = exp2(S*c - m_used), packed bf16 pairs, plus the partial row sum
      const float msub = (m_used == -INFINITY) ? 0.f : m_used;
      const uint64_t cc = f2_pack(c, c);
      const uint64_t nm = f2_pack(-msub, -msub);
      uint32_t pk[32];
      uint64_t acc2 = f2_pack(0.f, 0.f);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const uint64_t x = f2_fma(f2_pack(__uint_as_float(s[2 * i]), __uint_as_float(s[2 * i + 1])),
                                  cc, nm);
        float x0, x1;
        f2_unpack(x, x0, x1);
        const float p0 = ex2_approx(x0), p1 = ex2_approx(x1);
        acc2 = f2_add(acc2, f2_pack(p0, p1));
        __nv_bfloat162 b2 = __floats2bfloat162_rn(p0, p1);
        pk[i] = *reinterpret_cast<uint32_t*>(&b2);
      }
      float la, lb;
      f2_unpack(acc2, la, lb);
      l = l * alpha + (la + lb);
      // P_j of this half into the first 32 columns of its own 64-column S range
      tmem_st_32x32b_x32(tS + lane_addr + (uint32_t)(g * 64), pk);
      if (raise && j > 0) {  // rescale O in place; every earlier MMA is complete (S_j commit)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          uint32_t o[32];
          const uint32_t oa = tO + lane_addr + (uint32_t)(g * 64 + hh * 32);
          tmem_ld_32x32b_x32(oa, o);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st_32x32b_x32(oa, o);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    float lt = 0.f;
    bool have_o = false;
    if (ok && cnt > 0 && mbar_wait(pv_done, (uint32_t)(cnt - 1) & 1u, 0x30Au)) {
      tc_fence_after();
      xl[g * 128 + row] = l;
      mbar_arrive(l_bar);
      if (mbar_wait(l_bar, 0, 0x30Bu)) {
        lt = l + xl[(g ^ 1) * 128 + row];
        have_o = true;
      }
    }
    const float inv = lt > 0.f ? 1.0f / lt : 0.f;
    const int qrow = qb * kTile + row;
    const int64_t orow =
        args.row_map ? (int64_t)__ldg(args.row_map + (qrow < args.Lq ? qrow : 0)) : (int64_t)qrow;
    uint4* dst = reinterpret_cast<uint4*>(args.out + orow * args.ldo + col_q + g * 64);
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      uint32_t o[32];
      if (have_o) {
        tmem_ld_32x32b_x32(tO + lane_addr + (uint32_t)(g * 64 + hh * 32), o);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = 0u;
      }
      if (qrow < args.Lq) {
#pragma unroll
        for (int cch = 0; cch < 4; ++cch) {
          float f[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) f[i] = __uint_as_float(o[8 * cch + i]) * inv;
          dst[hh * 4 + cch] = f32_to_bf16x8(f);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

}  // namespace bsa2

// ===========================================================================
// v3: one CTA per SM, S double-buffered in TMEM, deep K/V prefetch.
//
// v2 runs S_j -> softmax_j -> P.V_j serially inside a CTA and single-buffers K and
// V, so the TMA latency of the next key window sits on the critical path (ncu: tensor
// pipe 40% active, issue slots 31%, stalls dominated by long-scoreboard waits).  v3
// keeps one query tile per CTA but:
//   * two S buffers in TMEM, so S_{j+1} = Q K_{j+1}^T runs while the softmax warps
//     work on S_j; P_j overwrites (half of) S_j's buffer as packed bf16 and the
//     P.V MMA reads it from TMEM; O accumulates in TMEM with the lazy rescale;
//   * a 3-stage K ring and a 2-stage V ring (160 KB) + Q (32 KB), so TMA runs two
//     windows ahead of the tensor core;
//   * the MMA warp issues PV_j, then (once PV_j has released the buffer) S_{j+2}.
// TMEM: S0 [0,128), S1 [128,256), O [256,384) of a 512-column allocation.
// ===========================================================================
namespace bsa3 {

constexpr int kThreads = 320;
constexpr int kSoftmaxThreads = 256;
constexpr int kTile = 128;
constexpr int kAtom = 128 * 128;
constexpr int kTileBytes = 2 * kAtom;
constexpr int kKStages = 3;
constexpr int kVStages = 2;
constexpr float kLazy = 8.0f;

constexpr size_t kSmemBytes =
    (size_t)kTileBytes * (1 + kKStages + kVStages) + 1024 /*align*/ + 3072 /*bars + xchg*/;

__global__ void __launch_bounds__(kThreads, 1)
    bsa_fwd_v3_kernel(const __grid_constant__ CUtensorMap tmQ,
                      const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, const bsa::Args args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~(uintptr_t)1023);
  uint8_t* sQ = base;
  uint8_t* sK = sQ + kTileBytes;               // kKStages tiles
  uint8_t* sV = sK + kKStages * kTileBytes;    // kVStages tiles
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + kVStages * kTileBytes);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;     // [3]
  uint64_t* k_empty = bars + 4;    // [3]
  uint64_t* v_full = bars + 7;     // [2]
  uint64_t* v_empty = bars + 9;    // [2]
  uint64_t* s_full = bars + 11;    // [2]
  uint64_t* s_free = bars + 13;    // [2]  P of this buffer consumed by its P.V
  uint64_t* p_full = bars + 15;    // [2]
  uint64_t* pv_done = bars + 17;   // completes once per P.V, in order
  uint64_t* x_bar = bars + 18;     // [2]
  uint64_t* l_bar = bars + 20;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 22);
  float* xmax = reinterpret_cast<float*>(bars + 24);  // [2 parity][2 halves][128]
  float* xl = xmax + 2 * 2 * 128;                     // [2 halves][128]

  const int warp = warp_id_uniform();
  const int lane = threadIdx.x & 31;
  const int qb = blockIdx.x;
  const int h = blockIdx.y;
  const int64_t rowid = (int64_t)h * args.NQ + qb;
  const int cnt = __ldg(args.cnt + rowid);
  const int32_t* sel = args.sel + rowid * args.sel_stride;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kKStages; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 1);
      mbar_init(&p_full[i], 8);
      mbar_init(&x_bar[i], kSoftmaxThreads);
    }
    mbar_init(pv_done, 1);
    mbar_init(l_bar, kSoftmaxThreads);
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tO = tmem + 256;
  const int col_q = h * kTile;

  if (warp == 8) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && cnt > 0) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      mbar_arrive_expect_tx(q_full, kTileBytes);
      tma_load_2d(sQ, &tmQ, q_full, col_q, qb * kTile);
      tma_load_2d(sQ + kAtom, &tmQ, q_full, col_q + 64, qb * kTile);
      for (int j = 0; j < cnt; ++j) {
        const int krow = __ldg(sel + j) * kTile;
        const int ks = j % kKStages;
        if (!mbar_wait(&k_empty[ks], (uint32_t)((j / kKStages) & 1) ^ 1u, 0x401u)) break;
        mbar_arrive_expect_tx(&k_full[ks], kTileBytes);
        tma_load_2d(sK + ks * kTileBytes, &tmK, &k_full[ks], col_q, krow);
        tma_load_2d(sK + ks * kTileBytes + kAtom, &tmK, &k_full[ks], col_q + 64, krow);
        const int vs = j & 1;
        if (!mbar_wait(&v_empty[vs], (uint32_t)((j >> 1) & 1) ^ 1u, 0x402u)) break;
        mbar_arrive_expect_tx(&v_full[vs], kTileBytes);
        tma_load_2d(sV + vs * kTileBytes, &tmV, &v_full[vs], col_q, krow);
        tma_load_2d(sV + vs * kTileBytes + kAtom, &tmV, &v_full[vs], col_q + 64, krow);
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && cnt > 0) {
      constexpr uint32_t idesc_s = make_idesc(1 /*bf16*/, 1 /*bf16*/, 0, 0, 128, 128);
      constexpr uint32_t idesc_o = make_idesc(1, 1, 0 /*P K-major*/, 1 /*V MN-major*/, 128, 128);
      const uint32_t q0 = smem_u32(sQ);
      bool ok = mbar_wait(q_full, 0, 0x403u);
      auto issue_s = [&](int j) -> bool {
        const int ks = j % kKStages;
        const int b = j & 1;
        if (!mbar_wait(&k_full[ks], (uint32_t)((j / kKStages) & 1), 0x404u)) return false;
        // buffer b last held P_{j-2}; its P.V must have consumed it
        if (j >= 2 && !mbar_wait(&s_free[b], (uint32_t)(((j - 2) >> 1) & 1), 0x405u)) return false;
        tc_fence_after();
        const uint32_t k0 = smem_u32(sK + ks * kTileBytes);
        const uint32_t d = tmem + (uint32_t)(b * 128);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (uint32_t)((kk >> 2) * kAtom + (kk & 3) * 32);
          mma_f16(d, smem_desc_sw128(q0 + off, 16, 1024), smem_desc_sw128(k0 + off, 16, 1024),
                  idesc_s, kk > 0 ? 1u : 0u);
        }
        tc_commit(&s_full[b]);
        tc_commit(&k_empty[ks]);
        return true;
      };
      if (ok) ok = issue_s(0);
      if (ok && cnt > 1) ok = issue_s(1);
      for (int j = 0; j < cnt && ok; ++j) {
        const int b = j & 1;
        if (!mbar_wait(&p_full[b], (uint32_t)((j >> 1) & 1), 0x406u)) break;
        const int vs = j & 1;
        if (!mbar_wait(&v_full[vs], (uint32_t)((j >> 1) & 1), 0x407u)) break;
        tc_fence_after();
        const uint32_t v0 = smem_u32(sV + vs * kTileBytes);
        const uint32_t sb = tmem + (uint32_t)(b * 128);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          // keys [16kk, 16kk+16): P of half g sits in columns [64g, 64g+32) of the buffer
          const uint32_t pcol = (uint32_t)((kk >> 2) * 64 + (kk & 3) * 8);
          mma_f16_ts(tO, sb + pcol,
                     smem_desc_sw128(v0 + (uint32_t)(kk * 16 * 128), (uint32_t)kAtom, 1024),
                     idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
        }
        tc_commit(&v_empty[vs]);
        tc_commit(&s_free[b]);
        tc_commit(pv_done);
        if (j + 2 < cnt) ok = issue_s(j + 2);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax warps
    const int g = warp >> 2;         // key / value column half
    const int qr = warp & 3;         // TMEM lane quarter
    const int row = qr * 32 + lane;  // query row within the block
    const uint32_t lane_addr = (uint32_t)(qr * 32) << 16;
    const float c = args.scale_log2;
    float m_used = -INFINITY;
    float l = 0.f;
    bool ok = true;
    for (int j = 0; j < cnt; ++j) {
      const int b = j & 1;
      const uint32_t tS = tmem + (uint32_t)(b * 128);
      if (!mbar_wait(&s_full[b], (uint32_t)((j >> 1) & 1), 0x408u)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t s[64];
      tmem_ld_32x32b_x32(tS + lane_addr + (uint32_t)(g * 64), s);
      tmem_ld_32x32b_x32(tS + lane_addr + (uint32_t)(g * 64 + 32), s + 32);
      tmem_ld_wait();
      const int key0 = __ldg(sel + j) * kTile + g * 64;
      if (key0 + 64 > args.kv_len) {
#pragma unroll
        for (int i = 0; i < 64; ++i)
          if (key0 + i >= args.kv_len) s[i] = __float_as_uint(-INFINITY);
      }
      float pm = -INFINITY;
#pragma unroll
      for (int i = 0; i < 64; ++i) pm = fmaxf(pm, __uint_as_float(s[i]));
      float* xm = xmax + (j & 1) * 256;
      xm[g * 128 + row] = pm;
      mbar_arrive(&x_bar[j & 1]);
      if (!mbar_wait(&x_bar[j & 1], (uint32_t)(j >> 1) & 1u, 0x409u)) {
        ok = false;
        break;
      }
      const float mb = fmaxf(pm, xm[(g ^ 1) * 128 + row]) * c;
      float alpha = 1.f;
      const bool raise = mb > m_used + kLazy;
      if (raise) {
        alpha = (m_used == -INFINITY) ? 0.f : ex2_approx(m_used - mb);
        m_used = mb;
      }
      const float msub = (m_used == -INFINITY) ? 0.f : m_used;
      const uint64_t cc = f2_pack(c, c);
      const uint64_t nm = f2_pack(-msub, -msub);
      uint32_t pk[32];
      uint64_t acc2 = f2_pack(0.f, 0.f);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const uint64_t x = f2_fma(f2_pack(__uint_as_float(s[2 * i]), __uint_as_float(s[2 * i + 1])),
                                  cc, nm);
        float x0, x1;
        f2_unpack(x, x0, x1);
        const float p0 = ex2_approx(x0), p1 = ex2_approx(x1);
        acc2 = f2_add(acc2, f2_pack(p0, p1));
        __nv_bfloat162 b2 = __floats2bfloat162_rn(p0, p1);
        pk[i] = *reinterpret_cast<uint32_t*>(&b2);
      }
      float la, lb;
      f2_unpack(acc2, la, lb);
      l = l * alpha + (la + lb);
      tmem_st_32x32b_x32(tS + lane_addr + (uint32_t)(g * 64), pk);
      if (raise && j > 0) {
        // O holds P.V of windows < j; the P.V of window j-1 may still be running
        if (!mbar_wait(pv_done, (uint32_t)((j - 1) & 1), 0x40Au)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          uint32_t o[32];
          const uint32_t oa = tO + lane_addr + (uint32_t)(g * 64 + hh * 32);
          tmem_ld_32x32b_x32(oa, o);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st_32x32b_x32(oa, o);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[b]);
    }
    float lt = 0.f;
    bool have_o = false;
    if (ok && cnt > 0 && mbar_wait(pv_done, (uint32_t)((cnt - 1) & 1), 0x40Bu)) {
      tc_fence_after();
      xl[g * 128 + row] = l;
      mbar_arrive(l_bar);
      if (mbar_wait(l_bar, 0, 0x40Cu)) {
        lt = l + xl[(g ^ 1) * 128 + row];
        have_o = true;
      }
    }
    const float inv = lt > 0.f ? 1.0f / lt : 0.f;
    const int qrow = qb * kTile + row;
    const int64_t orow =
        args.row_map ? (int64_t)__ldg(args.row_map + (qrow < args.Lq ? qrow : 0)) : (int64_t)qrow;
    uint4* dst = reinterpret_cast<uint4*>(args.out + orow * args.ldo + col_q + g * 64);
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      uint32_t o[32];
      if (have_o) {
        tmem_ld_32x32b_x32(tO + lane_addr + (uint32_t)(g * 64 + hh * 32), o);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = 0u;
      }
      if (qrow < args.Lq) {
#pragma unroll
        for (int cch = 0; cch < 4; ++cch) {
          float f[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) f[i] = __uint_as_float(o[8 * cch + i]) * inv;
          dst[hh * 4 + cch] = f32_to_bf16x8(f);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace bsa3
}  // namespace fvb

extern "C" int fvb_bsa_fwd(const void* q, const void* k, const void* v, const int32_t* sel,
                           const int32_t* cnt, int64_t sel_stride, int64_t H, int64_t Lq,
                           int64_t Lk, int64_t kv_len, int64_t d, float scale,
                           const int32_t* out_row_map, void* out, fvb_stream_t stream) {
  using namespace fvb;
  FVB_REQUIRE(d == 128, "fvb_bsa_fwd: head_dim must be 128 (got %lld)", (long long)d);
  FVB_REQUIRE(H > 0 && Lq >= 0 && Lk >= 0, "fvb_bsa_fwd: shape");
  if (Lq == 0) return FVB_OK;
  FVB_REQUIRE(kv_len >= 0 && kv_len <= Lk, "fvb_bsa_fwd: kv_len out of range");
  FVB_REQUIRE(Lk > 0 && Lk % 128 == 0, "fvb_bsa_fwd: Lk must be a positive multiple of 128");
  FVB_REQUIRE(q && k && v && sel && cnt && out, "fvb_bsa_fwd: NULL pointer");
  FVB_REQUIRE(aligned16(q) && aligned16(k) && aligned16(v) && aligned16(out),
              "fvb_bsa_fwd: q/k/v/out must be 16-byte aligned");
  const int64_t NQ = (Lq + 127) / 128;
  FVB_REQUIRE(NQ < 65536 && H < 65536, "fvb_bsa_fwd: grid too large");
  const uint64_t HD = (uint64_t)H * 128;
  CUtensorMap tq, tk, tv;
  int rc = make_tmap_2d(&tq, q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, HD, (uint64_t)Lq, HD * 2, 64,
                        128, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = make_tmap_2d(&tk, k, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, HD, (uint64_t)Lk, HD * 2, 64, 128,
                    CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = make_tmap_2d(&tv, v, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, HD, (uint64_t)Lk, HD * 2, 64, 128,
                    CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  static bool configured[64] = {false};
  // Kernel generation: v3 (1 CTA/SM, deep prefetch) when the key list can be long, v2
  // (2 CTAs/SM) for short lists such as cross-attention's 4 windows, where a co-resident
  // CTA hides the per-CTA set-up.  FVB_BSA_IMPL=v1|v2|v3 pins one (A/B timing).
  static int forced = -1;
  if (forced < 0) {
    const char* e = getenv("FVB_BSA_IMPL");
    forced = (e && e[0] == 'v' && e[1] >= '1' && e[1] <= '3') ? (e[1] - '0') : 0;
  }
  const int64_t nk_blocks = Lk / 128;
  const int impl = forced ? forced : (nk_blocks >= 16 ? 3 : 2);
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    FVB_CUDA_TRY(cudaFuncSetAttribute(bsa::bsa_fwd_kernel,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)bsa::kSmemBytes),
                 "bsa smem attribute");
    FVB_CUDA_TRY(cudaFuncSetAttribute(bsa2::bsa_fwd_v2_kernel,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)bsa2::kSmemBytes),
                 "bsa2 smem attribute");
    FVB_CUDA_TRY(cudaFuncSetAttribute(bsa3::bsa_fwd_v3_kernel,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)bsa3::kSmemBytes),
                 "bsa3 smem attribute");
    configured[dev] = true;
  }
  bsa::Args a;
  a.sel = sel;
  a.cnt = cnt;
  a.sel_stride = sel_stride;
  a.H = (int)H;
  a.NQ = (int)NQ;
  a.Lq = (int)Lq;
  a.kv_len = (int)kv_len;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.row_map = out_row_map;
  a.out = (__nv_bfloat16*)out;
  a.ldo = (int64_t)HD;
  if (impl == 1)
    bsa::bsa_fwd_kernel<<<dim3((unsigned)NQ, (unsigned)H), bsa::kThreads, bsa::kSmemBytes,
                          (cudaStream_t)stream>>>(tq, tk, tv, a);
  else if (impl == 2)
    bsa2::bsa_fwd_v2_kernel<<<dim3((unsigned)NQ, (unsigned)H), bsa2::kThreads,
                              bsa2::kSmemBytes, (cudaStream_t)stream>>>(tq, tk, tv, a);
  else
    bsa3::bsa_fwd_v3_kernel<<<dim3((unsigned)NQ, (unsigned)H), bsa3::kThreads,
                              bsa3::kSmemBytes, (cudaStream_t)stream>>>(tq, tk, tv, a);
  return check_launch("fvb_bsa_fwd");
}
