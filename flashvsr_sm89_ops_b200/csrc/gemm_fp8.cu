// FP8 E4M3 GEMM on the 5th-generation tensor cores (a3), with the scale /
// bias epilogue of FP8Linear._mm (fp8_linear.py:28-30) and an optional fused
// GELU(tanh) + row-amax epilogue for the FFN up-projection (fp8_ffn.py:24-40).
//
//   out[m, n] = bf16(acc[m, n] * sa[m|0] * sw[n|0] + bias[n]),  acc = sum_k A[m,k] W[n,k]
//
// Design (one persistent CTA per SM, 320 or 576 threads, warp-specialised):
//   warp 0      TMA producer: 128x128-byte A tiles and BNx128-byte W tiles
//               (128-byte swizzle) into a 3- or 4-stage shared-memory ring
//   warp 1      MMA issuer: one elected thread issues tcgen05.mma kind::f8f6f4
//               (M=128, N=BN, K=32 per instruction) into a TMEM accumulator;
//               tcgen05.commit releases ring stages and publishes finished tiles.
//               Also allocates / frees the 2*BN TMEM columns.
//   warps 2..   epilogue, G warps per TMEM lane quarter (G = 2 for the plain
//               epilogue, 4 for GELU + amax, whose per-warp latency is the long pole):
//               tcgen05.ld 32 columns at a time (each thread owns one output row, the G
//               warps take the 64-column chunks round-robin), scales + bias (+ GELU /
//               amax), bf16 into a 128-byte swizzled staging buffer, TMA bulk store of
//               32 rows x 64 columns.  The GELU variant runs a 3-stage ring to make room
//               for its 16 staging buffers and its GELU table.
// GELU epilogue: the GELU input is the bf16-rounded GEMM output, so GELU is a function of
// 16 bits.  Each CTA tabulates it (exact formula, gelu_tanh_bf16) for |x| in [2^-9, 16)
// into 6.5 KB of shared memory while its first tile's main loop runs; the epilogue then
// costs one shared-memory load per element instead of a tanh.  Outside the table the
// results are 0.5 x (|x| < 2^-9: 1 + tanh u rounds to 1 within half a bf16 ulp), x
// (x >= 16) and x * 0 (x <= -16: tanh u is -1); the tests check every bf16 input.
// The accumulator is double-buffered in TMEM so the epilogue of tile t overlaps
// the main loop of tile t+1.  Both operands are K-major ("TN"), exactly the
// nn.Linear weight layout, so no transpose is ever materialised.
#include "common.cuh"

namespace fvb {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 128;  // bytes == fp8 elements per K block

// per-epilogue configuration: epilogue warps (a multiple of 4) and ring depth.  A CTA pair
// stages BM + BN/2 rows per K block (32 KB at BN=256) instead of BM + BN (48 KB), so the
// same shared memory holds more stages.
template <int EPI, bool PAIR>
struct Cfg {
  static constexpr int kEpiWarps = EPI == FVB_EPI_GELU_AMAX ? 16 : 8;
  static constexpr int kStages =
      PAIR ? (EPI == FVB_EPI_GELU_AMAX ? 4 : 6) : (EPI == FVB_EPI_GELU_AMAX ? 3 : 4);
  static constexpr int kThreads = 64 + 32 * kEpiWarps;
};

// epilogue of the FFN down-projection with the DiT block's gated residual add fused in:
//   out = bf16(res + bf16(gate * bf16(acc * sa * sw + bias)))   (== fvb_gate_add of the GEMM)
constexpr int kEpiGateResidual = 2;

struct Args {
  int M, N, K;
  const float* sa;
  const float* sw;
  int a_row, w_row;
  const __nv_bfloat16* bias;
  __nv_bfloat16* out;
  int64_t ldo;
  float* amax_out;
  const __nv_bfloat16* res;   // kEpiGateResidual: residual [M, N] (row pitch ldo)
  const __nv_bfloat16* gate;  // kEpiGateResidual: gate [N], or NULL for a plain add
};

constexpr int kStageBytes = 32 * 128;  // one epilogue warp's 32 rows x 64 bf16 columns

// the GELU table (gelu_bf16_bits, common.cuh) in shared memory, GELU epilogue only
template <int EPI>
struct Lut {
  static constexpr int kBytes = EPI == FVB_EPI_GELU_AMAX ? kGeluTableBytes : 0;
};

// W rows one CTA stages per K block: all BN, or its half of the pair's BN
template <int BN, bool PAIR>
__host__ __device__ constexpr int b_rows() {
  return PAIR ? BN / 2 : BN;
}

template <int BN, int EPI, bool PAIR>
constexpr size_t smem_bytes() {
  return (size_t)Cfg<EPI, PAIR>::kStages * (BM + b_rows<BN, PAIR>()) * BK +
         (size_t)Cfg<EPI, PAIR>::kEpiWarps * kStageBytes + Lut<EPI>::kBytes +
         1024 /*align slack*/ + 256 /*barriers*/;
}

// PAIR: launched as 2-CTA clusters.  The pair owns 256-row x BN tiles: CTA r stages A
// rows [m0 + 128 r, +128) and W rows [n0 + r BN/2, +BN/2), the even CTA's MMA thread
// issues cta_group::2 MMAs (M=256, N=BN) over both CTAs' stages, each CTA's TMEM receives
// its own 128 rows x BN, and each CTA's epilogue stores its own rows.  Barriers: the
// even CTA's `full` counts both CTAs' load bytes, MMA commits arrive on both CTAs'
// `empty` and `tfull`, and both CTAs' epilogue warps arrive on the even CTA's `tempty`.
template <int BN, int EPI, bool PAIR>
__global__ void __launch_bounds__(Cfg<EPI, PAIR>::kThreads, 1)
    fp8_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmOut, const Args args) {
  constexpr int STAGES = Cfg<EPI, PAIR>::kStages;
  constexpr int EPI_WARPS = Cfg<EPI, PAIR>::kEpiWarps;
  constexpr int BNL = b_rows<BN, PAIR>();
  constexpr int TM = PAIR ? 2 * BM : BM;  // rows per tile
  constexpr int G = EPI_WARPS / 4;  // epilogue warps per TMEM lane quarter
  constexpr int kOutBytes = EPI_WARPS * kStageBytes;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~(uintptr_t)1023);
  uint8_t* sA = base;
  uint8_t* sB = sA + STAGES * BM * BK;
  uint8_t* sOut = sB + STAGES * BNL * BK;  // epilogue staging, 1024-aligned
  uint16_t* lut = reinterpret_cast<uint16_t*>(sOut + kOutBytes);  // GELU table (GELU only)
  uint64_t* full = reinterpret_cast<uint64_t*>(sOut + kOutBytes + Lut<EPI>::kBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;  // MMA unwind: completion of every MMA this CTA issued
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  uint32_t* pair_ok = tmem_slot + 1;  // PAIR: both CTAs hold the same TMEM address

  const int warp = warp_id_uniform();
  const int lane = threadIdx.x & 31;
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const int unit = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;  // tile scheduling unit
  const int units = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  const int m_tiles = (args.M + TM - 1) / TM;
  const int n_tiles = (args.N + BN - 1) / BN;
  const int num_tiles = m_tiles * n_tiles;
  const int kblocks = (args.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], PAIR ? 2 * EPI_WARPS : EPI_WARPS);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    prefetch_tmap(&tmOut);
  }
  if (warp == 1) {
    if (PAIR) {
      tmem_alloc_pair(tmem_slot, 2 * BN);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, 2 * BN);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if (PAIR) {
    cluster_sync_all();  // barrier inits and both allocations visible pair-wide
    if (threadIdx.x == 0)
      *pair_ok = ld_shared_cluster_u32(mapa_shared(smem_u32(tmem_slot), rank ^ 1u)) == *tmem_slot;
    __syncthreads();
  } else {
    __syncthreads();
  }
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // a pair whose TMEM addresses differ (never expected) does no work and reports it
  const bool run = !PAIR || *pair_ok != 0u;
  if (!run && threadIdx.x == 0 && rank == 0) atomicCAS(&g_device_error, 0u, 0x10Cu);
  // the even CTA's barriers, as shared::cluster addresses (PAIR)
  const uint32_t full0_c = PAIR ? mapa_shared(smem_u32(full), 0u) : 0u;
  const uint32_t tempty0_c = PAIR ? mapa_shared(smem_u32(tempty), 0u) : 0u;

  if (!run) {
    // straight to the teardown
  } else if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int64_t issued = 0;  // loads issued so far; load i fills stage i % STAGES
      for (int tile = unit; tile < num_tiles && ok; tile += units) {
        const int m0 = (tile / n_tiles) * TM + (int)rank * BM;
        const int n0 = (tile % n_tiles) * BN + (int)rank * BNL;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, 0x101u)) {
            ok = false;
            break;
          }
          if (PAIR) {
            // the even CTA arms its barrier for both CTAs' bytes; a partner load that
            // lands first only leaves the count transiently negative
            if (rank == 0) mbar_arrive_expect_tx(&full[stage], (uint32_t)(2 * (BM + BNL) * BK));
            tma_load_2d_pair(sA + stage * BM * BK, &tmA, full0_c + 8u * stage, kb * BK, m0);
            tma_load_2d_pair(sB + stage * BNL * BK, &tmB, full0_c + 8u * stage, kb * BK, n0);
          } else {
            mbar_arrive_expect_tx(&full[stage], (uint32_t)((BM + BN) * BK));
            tma_load_2d(sA + stage * BM * BK, &tmA, &full[stage], kb * BK, m0);
            tma_load_2d(sB + stage * BN * BK, &tmB, &full[stage], kb * BK, n0);
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Drain: no load may still be writing shared memory when its CTA exits.  The last
      // STAGES loads are the newest phase of their stages' full barriers (already complete
      // on the normal path; bounded waits after a timeout).  A pair's barriers live in
      // the even CTA and count both CTAs' loads; the odd CTA's loads are covered by this
      // wait and the cluster barrier before either CTA exits.
      if (!PAIR || rank == 0)
        for (int64_t i = issued > STAGES ? issued - STAGES : 0; i < issued; ++i)
          mbar_wait(&full[i % STAGES], (uint32_t)((i / STAGES) & 1), 0x10Au);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = make_idesc(0 /*E4M3*/, 0 /*E4M3*/, 0, 0, TM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int t = 0;
      bool ok = true;
      bool any = false;  // whether this thread issued an MMA
      for (int tile = unit; tile < num_tiles && ok; tile += units, ++t) {
        const int buf = t & 1;
        const uint32_t tph = (uint32_t)(t >> 1) & 1u;
        if (!mbar_wait(&tempty[buf], tph ^ 1u, 0x102u)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + (uint32_t)(buf * BN);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, 0x103u)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * BM * BK);
          const uint32_t b0 = smem_u32(sB + stage * BNL * BK);
#pragma unroll
          for (int k = 0; k < BK / 32; ++k) {
            const uint64_t da = smem_desc_sw128(a0 + k * 32, 16, 1024);
            const uint64_t db = smem_desc_sw128(b0 + k * 32, 16, 1024);
            if (PAIR)
              mma_f8f6f4_pair(d_tmem, da, db, idesc, (kb | k) != 0 ? 1u : 0u);
            else
              mma_f8f6f4(d_tmem, da, db, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          any = true;
          if (PAIR)
            tc_commit_pair_both(&empty[stage], 0x3);
          else
            tc_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) {
          if (PAIR)
            tc_commit_pair_both(&tfull[buf], 0x3);
          else
            tc_commit(&tfull[buf]);
        }
      }
      // Drain: every MMA issued above completes before TMEM is freed (on the normal path
      // the epilogue has already waited for all of them).
      if (any) {
        if (PAIR)
          tc_commit_pair(drain);
        else
          tc_commit(drain);
        mbar_wait(drain, 0, 0x10Bu);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // G warps per TMEM lane quarter (warp % 4); they take each tile's 64-column chunks
    // round-robin, so each thread finishes 1/G of a row per tile.
    const int q = warp & 3;               // TMEM lane quarter this warp may access
    const int half = (warp - 2) >> 2;     // 0..G-1: this warp's first chunk
    if (EPI == FVB_EPI_GELU_AMAX) {
      // tabulate GELU while the first tile's main loop runs; epilogue warps only
      gelu_table_fill(lut, threadIdx.x - 64, EPI_WARPS * 32);
      asm volatile("bar.sync 1, %0;" ::"r"(EPI_WARPS * 32) : "memory");
    }
    uint8_t* stg = sOut + (size_t)(warp - 2) * kStageBytes;  // this warp's staging, 32 x 128 B
    // release of TMEM buffer `b` to the MMA thread (the even CTA's barrier for a pair)
    auto release = [&](int b) {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (PAIR)
          mbar_arrive_remote(tempty0_c + 8u * b);
        else
          mbar_arrive(&tempty[b]);
      }
    };
    int t = 0;
    for (int tile = unit; tile < num_tiles; tile += units, ++t) {
      const int buf = t & 1;
      const uint32_t tph = (uint32_t)(t >> 1) & 1u;
      const int m0 = (tile / n_tiles) * TM + (int)rank * BM;
      const int n0 = (tile % n_tiles) * BN;
      // warp-uniform: the tcgen05.ld below is .sync.aligned, so either every lane of the
      // warp goes on or none does
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull[buf], tph, 0x104u))) break;
      tc_fence_after();
      const int rloc = q * 32 + lane;  // row within the tile == TMEM lane
      const int row = m0 + rloc;
      const bool row_ok = row < args.M;
      const float sa = args.a_row ? (row_ok ? __ldg(args.sa + row) : 0.f) : __ldg(args.sa);
      const float sw0 = args.w_row ? 0.f : __ldg(args.sw);
      uint32_t tmax = 0;  // row amax of |GELU| as bf16 magnitude bits (GELU only)
#pragma unroll 1
      for (int c = half; c < BN / 64; c += G) {
        const int col0 = n0 + c * 64;
        // the previous TMA store from this staging buffer must have finished reading it
        if (lane == 0) tma_store_wait_read<0>();
        __syncwarp();
        // the chunk's two 32-column TMEM loads go out together, one wait for both (measured:
        // qkv 52.6 us against 54.0 us with a wait after each load)
        uint32_t rr[64];
        {
          const uint32_t ta = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * BN + c * 64);
          tmem_ld_32x32b_x32(ta, rr);
          tmem_ld_32x32b_x32(ta + 32, rr + 32);
          tmem_ld_wait();
        }
#pragma unroll
        for (int sub = 0; sub < 2; ++sub) {
          const uint32_t* r = rr + sub * 32;
#pragma unroll
          for (int g4 = 0; g4 < 4; ++g4) {
            const int g = sub * 4 + g4;  // 16-byte chunk of the 128-byte staging row
            const int cg = col0 + g * 8;
            float v[8];
            float swv[8], bv[8];
            if (args.w_row && cg < args.N) {
              const float4 s0 = __ldg(reinterpret_cast<const float4*>(args.sw + cg));
              const float4 s1 = __ldg(reinterpret_cast<const float4*>(args.sw + cg + 4));
              swv[0] = s0.x; swv[1] = s0.y; swv[2] = s0.z; swv[3] = s0.w;
              swv[4] = s1.x; swv[5] = s1.y; swv[6] = s1.z; swv[7] = s1.w;
            } else {
#pragma unroll
              for (int i = 0; i < 8; ++i) swv[i] = sw0;
            }
            if (args.bias && cg < args.N) {
              bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(args.bias + cg)), bv);
            } else {
#pragma unroll
              for (int i = 0; i < 8; ++i) bv[i] = 0.f;
            }
            uint4 packed;
            if (EPI == FVB_EPI_GELU_AMAX) {
              uint32_t hb[8];
              const bool counted = row_ok && cg < args.N;
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                hb[i] = gelu_bits(__fmaf_rn(__uint_as_float(r[g4 * 8 + i]), sa * swv[i], bv[i]),
                                  lut);
                if (counted) tmax = max(tmax, hb[i] & 0x7FFFu);
              }
              packed = make_uint4(__byte_perm(hb[0], hb[1], 0x5410), __byte_perm(hb[2], hb[3], 0x5410),
                                  __byte_perm(hb[4], hb[5], 0x5410), __byte_perm(hb[6], hb[7], 0x5410));
            } else {
#pragma unroll
              for (int i = 0; i < 8; ++i)
                v[i] = __fmaf_rn(__uint_as_float(r[g4 * 8 + i]), sa * swv[i], bv[i]);
              packed = f32_to_bf16x8(v);
              if (EPI == kEpiGateResidual) {
                // bf16(res + bf16(g * y)): packed _rn forms round the exact product and the
                // exact sum once, which is the eager bf16 chain bit for bit
                uint4 ru = make_uint4(0u, 0u, 0u, 0u);
                if (row_ok && cg < args.N)
                  ru = __ldg(reinterpret_cast<const uint4*>(args.res + (int64_t)row * args.ldo + cg));
                const __nv_bfloat162* r2 = reinterpret_cast<const __nv_bfloat162*>(&ru);
                __nv_bfloat162* y2 = reinterpret_cast<__nv_bfloat162*>(&packed);
                if (args.gate) {
                  const uint4 gu = cg < args.N ? __ldg(reinterpret_cast<const uint4*>(args.gate + cg))
                                               : make_uint4(0u, 0u, 0u, 0u);
                  const __nv_bfloat162* gg = reinterpret_cast<const __nv_bfloat162*>(&gu);
#pragma unroll
                  for (int p = 0; p < 4; ++p) y2[p] = __hadd2_rn(r2[p], __hmul2_rn(gg[p], y2[p]));
                } else {
#pragma unroll
                  for (int p = 0; p < 4; ++p) y2[p] = __hadd2_rn(r2[p], y2[p]);
                }
              }
            }
            // 128-byte swizzle: 16-byte chunk g of row `lane` lands at chunk g ^ (lane & 7)
            *reinterpret_cast<uint4*>(stg + lane * 128 + ((g ^ (lane & 7)) << 4)) = packed;
          }
        }
        if (c + G >= BN / 64) release(buf);  // this warp's last TMEM read of the tile
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (col0 < args.N) tma_store_2d(&tmOut, stg, col0, m0 + q * 32);
          tma_store_commit();
        }
      }
      if (half >= BN / 64) release(buf);  // a warp with no chunk in this tile (G > BN / 64)
      if (EPI == FVB_EPI_GELU_AMAX) {
        // bf16 magnitude bits order like the values they encode (NaN above +inf)
        if (args.a_row) {
          if (row_ok) atomic_max_nonneg(args.amax_out + row, __uint_as_float(tmax << 16));
        } else {
          const uint32_t m = __reduce_max_sync(0xffffffffu, tmax);
          if (lane == 0) atomic_max_nonneg(args.amax_out, __uint_as_float(m << 16));
        }
      }
    }
    if (lane == 0) tma_store_wait0();  // staging reads and global writes complete
  }
  tc_fence_before();
  if (PAIR)
    cluster_sync_all();  // neither CTA leaves while the pair's MMAs or loads may touch it
  else
    __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if (PAIR)
      tmem_dealloc_pair(tmem, 2 * BN);
    else
      tmem_dealloc(tmem, 2 * BN);
  }
}

template <int BN, int EPI, bool PAIR>
static int launch(const Args& a, const void* A, const void* W, cudaStream_t st) {
  constexpr int BNL = b_rows<BN, PAIR>();
  CUtensorMap tmA, tmB;
  int rc = make_tmap_2d(&tmA, A, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)a.K, (uint64_t)a.M,
                        (uint64_t)a.K, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = make_tmap_2d(&tmB, W, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)a.K, (uint64_t)a.N,
                    (uint64_t)a.K, BK, BNL, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  CUtensorMap tmO;
  rc = make_tmap_2d(&tmO, a.out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)a.N, (uint64_t)a.M,
                    (uint64_t)a.ldo * 2, 64, 32, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  auto kern = fp8_gemm_kernel<BN, EPI, PAIR>;
  constexpr size_t smem = smem_bytes<BN, EPI, PAIR>();
  static_assert(smem <= 227 * 1024, "fp8 gemm: shared memory");
  static bool configured[64] = {false};
  static int pair_slots[64] = {0};  // co-resident CTA pairs per device (PAIR)
  int dev = 0;
  FVB_CUDA_TRY(cudaGetDevice(&dev), "fp8 gemm device");
  FVB_REQUIRE(dev >= 0 && dev < 64, "fp8 gemm: device ordinal %d", dev);
  constexpr int TM = PAIR ? 2 * BM : BM;
  const int tiles = ((a.M + TM - 1) / TM) * ((a.N + BN - 1) / BN);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  cfg.blockDim = dim3(Cfg<EPI, PAIR>::kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  if (PAIR) {
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  if (!configured[dev]) {
    FVB_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                 "fp8 gemm smem attribute");
    if (PAIR) {
      int clusters = 0;
      cfg.gridDim = dim3(2 * (sm_count() / 2));
      FVB_CUDA_TRY(cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg),
                   "fp8 gemm cluster occupancy");
      FVB_REQUIRE(clusters > 0, "fp8 gemm: no 2-CTA cluster fits on this device");
      pair_slots[dev] = clusters;
    }
    configured[dev] = true;
  }
  int grid;
  if (PAIR) {
    const int units = tiles < pair_slots[dev] ? tiles : pair_slots[dev];
    grid = 2 * units;
  } else {
    grid = tiles < sm_count() ? tiles : sm_count();
  }
  cfg.gridDim = dim3(grid);
  FVB_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, tmA, tmB, tmO, a), "fvb_fp8_gemm launch");
  return check_launch("fvb_fp8_gemm");
}

// choose the N tile.  A 128x256 tile moves 48 KB of operands per 4 MFLOP of MMA
// work against 32 KB per 2 MFLOP for 128x128, and on B200 the operand feed from L2,
// not wave quantisation, decides short-K GEMMs (measured: 8448x4608x1536 runs
// 1.5x faster at BN=256 despite a ragged last wave).  BN=128 only for narrow N.
static int pick_bn(int M, int N) {
  (void)M;
  return N <= 128 ? 128 : 256;
}

// pick the tile shape and launch.  Wide BN=256 GEMMs (N >= 4096) with more than one 128-row
// block of A run on CTA pairs: a third less operand traffic per SM (L2 reads, shared-memory
// writes and MMA operand reads), measured 2-5% faster under the power cap at N = 4608 and
// 8960 with the plain epilogue.  At N = 1536 the pair measured 2% slower, and with the GELU
// epilogue (FFN-up, 8448x8960x1536) 137.0 us against 131.8 us single-CTA, so those stay
// single-CTA.
constexpr int kPairMinN = 4096;
template <int EPI>
static int dispatch(const Args& a, const void* A, const void* W, cudaStream_t st) {
  if (pick_bn(a.M, a.N) == 128) return launch<128, EPI, false>(a, A, W, st);
  if constexpr (EPI != FVB_EPI_GELU_AMAX) {
    if (a.M > BM && a.N >= kPairMinN) return launch<256, EPI, true>(a, A, W, st);
  }
  return launch<256, EPI, false>(a, A, W, st);
}

}  // namespace gemm
}  // namespace fvb

extern "C" {

int fvb_fp8_gemm(const void* A, const float* sa, int a_mode, const void* W, const float* sw,
                 int w_mode, const void* bias, int64_t M, int64_t N, int64_t K, void* out,
                 int epilogue, float* amax_out, fvb_stream_t stream) {
  using namespace fvb;
  FVB_REQUIRE(M >= 0 && N >= 0 && K >= 0, "fvb_fp8_gemm: negative size");
  FVB_REQUIRE(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31), "fvb_fp8_gemm: size");
  FVB_REQUIRE(a_mode == FVB_SCALE_TENSOR || a_mode == FVB_SCALE_ROW, "fvb_fp8_gemm: a_mode");
  FVB_REQUIRE(w_mode == FVB_SCALE_TENSOR || w_mode == FVB_SCALE_ROW, "fvb_fp8_gemm: w_mode");
  FVB_REQUIRE(epilogue == FVB_EPI_NONE || epilogue == FVB_EPI_GELU_AMAX, "fvb_fp8_gemm: epilogue");
  if (M == 0 || N == 0) return FVB_OK;
  FVB_REQUIRE(K > 0 && K % 16 == 0, "fvb_fp8_gemm: K=%lld must be a positive multiple of 16",
              (long long)K);
  FVB_REQUIRE(N % 8 == 0, "fvb_fp8_gemm: N=%lld must be a multiple of 8", (long long)N);
  FVB_REQUIRE(A && W && sa && sw && out, "fvb_fp8_gemm: NULL pointer");
  FVB_REQUIRE(aligned16(A) && aligned16(W) && aligned16(out) && (!bias || aligned16(bias)),
              "fvb_fp8_gemm: A, W, out and bias must be 16-byte aligned");
  FVB_REQUIRE(w_mode != FVB_SCALE_ROW || aligned16(sw), "fvb_fp8_gemm: sw alignment");
  FVB_REQUIRE(epilogue == FVB_EPI_NONE || amax_out != nullptr, "fvb_fp8_gemm: amax_out is NULL");
  gemm::Args a;
  a.M = (int)M;
  a.N = (int)N;
  a.K = (int)K;
  a.sa = sa;
  a.sw = sw;
  a.a_row = a_mode == FVB_SCALE_ROW;
  a.w_row = w_mode == FVB_SCALE_ROW;
  a.bias = (const __nv_bfloat16*)bias;
  a.out = (__nv_bfloat16*)out;
  a.ldo = N;
  a.amax_out = amax_out;
  cudaStream_t st = (cudaStream_t)stream;
  a.res = nullptr;
  a.gate = nullptr;
  if (epilogue == FVB_EPI_NONE) return gemm::dispatch<FVB_EPI_NONE>(a, A, W, st);
  return gemm::dispatch<FVB_EPI_GELU_AMAX>(a, A, W, st);
}

// FFN down-projection with the gated residual epilogue (fvb_fp8_ffn_residual's GEMM-2)
static int fp8_gemm_gate_residual(const void* A, const float* sa, int a_mode, const void* W,
                                  const float* sw, int w_mode, const void* bias, int64_t M,
                                  int64_t N, int64_t K, const void* res, const void* gate,
                                  void* out, fvb_stream_t stream) {
  using namespace fvb;
  FVB_REQUIRE(M >= 0 && N > 0 && K > 0 && K % 16 == 0 && N % 8 == 0 && M < (1ll << 31) &&
                  N < (1ll << 31) && K < (1ll << 31),
              "fvb_fp8_ffn_residual: shape");
  if (M == 0) return FVB_OK;
  FVB_REQUIRE(A && W && sa && sw && out && res, "fvb_fp8_ffn_residual: NULL pointer");
  FVB_REQUIRE(aligned16(A) && aligned16(W) && aligned16(out) && aligned16(res) &&
                  (!bias || aligned16(bias)) && (!gate || aligned16(gate)),
              "fvb_fp8_ffn_residual: pointers must be 16-byte aligned");
  FVB_REQUIRE(w_mode != FVB_SCALE_ROW || aligned16(sw), "fvb_fp8_ffn_residual: sw alignment");
  gemm::Args a;
  a.M = (int)M;
  a.N = (int)N;
  a.K = (int)K;
  a.sa = sa;
  a.sw = sw;
  a.a_row = a_mode == FVB_SCALE_ROW;
  a.w_row = w_mode == FVB_SCALE_ROW;
  a.bias = (const __nv_bfloat16*)bias;
  a.out = (__nv_bfloat16*)out;
  a.ldo = N;
  a.amax_out = nullptr;
  a.res = (const __nv_bfloat16*)res;
  a.gate = (const __nv_bfloat16*)gate;
  cudaStream_t st = (cudaStream_t)stream;
  return gemm::dispatch<gemm::kEpiGateResidual>(a, A, W, st);
}

size_t fvb_fp8_ffn_workspace_bytes(int64_t M, int64_t F) {
  // h (bf16 [M,F]) + h8 (fp8 [M,F]) + amax [M] + h scale [M], each 256-aligned
  auto up = [](size_t b) { return (b + 255) & ~(size_t)255; };
  return up((size_t)M * F * 2) + up((size_t)M * F) + up((size_t)(M > 0 ? M : 1) * 4) * 2;
}

static int ffn_impl(const void* x8, const float* sx, int mode, const void* W0, const float* sw0,
                    const void* b0, const void* W2, const float* sw2, const void* b2, int w_mode,
                    int64_t M, int64_t D, int64_t F, const void* res, const void* gate, void* out,
                    void* workspace, fvb_stream_t stream) {
  using namespace fvb;
  FVB_REQUIRE(M >= 0 && D > 0 && F > 0, "fvb_fp8_ffn: shape");
  if (M == 0) return FVB_OK;
  FVB_REQUIRE(workspace != nullptr && (reinterpret_cast<uintptr_t>(workspace) & 255u) == 0,
              "fvb_fp8_ffn: workspace must be 256-byte aligned");
  auto up = [](size_t b) { return (b + 255) & ~(size_t)255; };
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  void* h = ws;
  void* h8 = ws + up((size_t)M * F * 2);
  float* amax = reinterpret_cast<float*>(ws + up((size_t)M * F * 2) + up((size_t)M * F));
  float* hs = amax + up((size_t)M * 4) / 4;
  const size_t namax = (mode == FVB_SCALE_ROW) ? (size_t)M : 1;
  cudaStream_t st = (cudaStream_t)stream;
  FVB_CUDA_TRY(cudaMemsetAsync(amax, 0, namax * sizeof(float), st), "fvb_fp8_ffn amax clear");
  int rc = fvb_fp8_gemm(x8, sx, mode, W0, sw0, w_mode, b0, M, F, D, h, FVB_EPI_GELU_AMAX, amax,
                        stream);
  if (rc) return rc;
  rc = fvb_quant_fp8_with_amax(h, M, F, amax, mode, h8, hs, stream);
  if (rc) return rc;
  if (res)
    return fp8_gemm_gate_residual(h8, hs, mode, W2, sw2, w_mode, b2, M, D, F, res, gate, out,
                                  stream);
  return fvb_fp8_gemm(h8, hs, mode, W2, sw2, w_mode, b2, M, D, F, out, FVB_EPI_NONE, nullptr,
                      stream);
}

int fvb_fp8_ffn(const void* x8, const float* sx, int mode, const void* W0, const float* sw0,
                const void* b0, const void* W2, const float* sw2, const void* b2, int w_mode,
                int64_t M, int64_t D, int64_t F, void* out, void* workspace,
                fvb_stream_t stream) {
  return ffn_impl(x8, sx, mode, W0, sw0, b0, W2, sw2, b2, w_mode, M, D, F, nullptr, nullptr, out,
                  workspace, stream);
}

int fvb_fp8_ffn_residual(const void* x8, const float* sx, int mode, const void* W0,
                         const float* sw0, const void* b0, const void* W2, const float* sw2,
                         const void* b2, int w_mode, int64_t M, int64_t D, int64_t F,
                         const void* residual, const void* gate, void* out, void* workspace,
                         fvb_stream_t stream) {
  using namespace fvb;
  FVB_REQUIRE(residual != nullptr, "fvb_fp8_ffn_residual: residual is NULL");
  return ffn_impl(x8, sx, mode, W0, sw0, b0, W2, sw2, b2, w_mode, M, D, F, residual, gate, out,
                  workspace, stream);
}

}  // extern "C"
