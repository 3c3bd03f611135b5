/* flashvsr_b200.h — C ABI of the B200 (sm_100a) FlashVSR operator pack.
 *
 * Every entry point takes raw device pointers, sizes and a cudaStream_t
 * (pass torch.cuda.current_stream().cuda_stream, or 0 for the legacy
 * stream), enqueues work on that stream and returns an int status:
 *   FVB_OK (0), FVB_ERR_INVALID (bad size / null / misaligned pointer),
 *   FVB_ERR_UNSUPPORTED (a mode this pack does not implement),
 *   FVB_ERR_CUDA (a CUDA launch or runtime call failed).
 * fvb_last_error() returns the message of the last failure on the calling
 * thread.  No entry point synchronises the stream or allocates device memory.
 * Device state kept between calls: the per-device error word read by
 * fvb_device_error(), and the fixed scratch array of fvb_quant_fp8_tensor_noalloc
 * (whose overlapping calls race; see its comment).  Callers own every buffer;
 * inputs are never written.
 *
 * Tensor conventions: bf16 = IEEE bfloat16, fp8 = OCP FP8 E4M3 ("e4m3fn",
 * max 448, no infinities), all matrices row-major and contiguous.
 *
 * Reference interfaces cited below are files of aireet/flashvsr-sm89-ops
 * (package flashvsr_sm89_ops/), which exposes them as Python functions.
 */
#ifndef FLASHVSR_B200_H_
#define FLASHVSR_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* fvb_stream_t; /* == cudaStream_t */

#if defined(__GNUC__)
#define FVB_API __attribute__((visibility("default")))
#else
#define FVB_API
#endif

#define FVB_OK 0
#define FVB_ERR_INVALID 1
#define FVB_ERR_UNSUPPORTED 2
#define FVB_ERR_CUDA 3

/* quantisation granularity (FP8 activations and weights) */
#define FVB_SCALE_TENSOR 0 /* one fp32 scale for the whole tensor (reference default) */
#define FVB_SCALE_ROW 1    /* one fp32 scale per row: per-token activations / per-channel weights */

#define FVB_FP8_MAX 448.0f /* fp8_quant.py:13 FP8_MAX */

/* ---------------------------------------------------------------- misc */
FVB_API int fvb_abi_version(void);                 /* bumped on any signature change */
FVB_API const char* fvb_last_error(void);          /* thread-local message of the last failure */
/* Reads and clears the device error word that kernels set when a bounded wait
 * gives up (0 = none).  Synchronises the legacy stream of the current device. */
FVB_API int fvb_device_error(unsigned int* code_out);

/* ------------------------------------------------- a1 / a2: FP8 quantise
 * Replaces quantize_fp8(x2) (fp8_quant.py:42-55; kernels :16-35) and the
 * eager branch of FP8Linear.forward (fp8_linear.py:38-40).
 *   s = max(amax, 1e-12) / 448;  q = e4m3(clamp(x / s, -448, 448))  (IEEE divide, RNE)
 *   scale_out = amax * fl(1/448)  (fp32; [1] for FVB_SCALE_TENSOR, [M] for FVB_SCALE_ROW):
 *   the reference's returned `amax / FP8_MAX` as torch computes it on a CUDA tensor (a
 *   division by a host scalar is a multiply by the scalar's fp32 reciprocal)
 * x [M,K] bf16, q [M,K] fp8.  FVB_SCALE_TENSOR needs `workspace` of
 * fvb_quant_fp8_workspace_bytes() bytes (device, 16-byte aligned); FVB_SCALE_ROW needs none.
 * M*K == 0 writes scale 0 like the reference (fp8_quant.py:45-47). */
FVB_API size_t fvb_quant_fp8_workspace_bytes(int64_t M, int64_t K, int mode);
FVB_API int fvb_quant_fp8(const void* x, int64_t M, int64_t K, void* q, float* scale_out, int mode,
                  void* workspace, fvb_stream_t stream);

/* Per-tensor FP8 quantisation that allocates nothing (no counterpart in the reference).
 * For callers that cannot allocate device memory -- an FFI host that only passes device
 * pointers through this C ABI, a process whose device memory belongs to another
 * framework's pool, a loop that must not pay cudaMalloc's implicit synchronisation.
 * Same result as fvb_quant_fp8(..., FVB_SCALE_TENSOR, workspace, ...), bit for bit, but its
 * reduction scratch is a fixed device array inside the library (FVB_NOALLOC_QUANT_MAX_PARTIALS
 * floats = 64 KB, held on every GPU that loads the library until the process exits).
 *   - Limit: M*K <= FVB_NOALLOC_QUANT_MAX_PARTIALS * 65536 elements (2^30); larger inputs
 *     are rejected with FVB_ERR_INVALID.
 *   - It calls no cudaMalloc / cudaFree / allocating library routine.  The first call on a
 *     device looks up the array's device address (cudaGetSymbolAddress) with that device
 *     current; make that first call before any stream capture.
 *   - All calls share the array, which keeps the last call's contents: calls that overlap
 *     on the GPU (several streams or threads) race and must be ordered by the caller. */
#define FVB_NOALLOC_QUANT_MAX_PARTIALS 16384
FVB_API int fvb_quant_fp8_tensor_noalloc(const void* x, int64_t M, int64_t K, void* q,
                                         float* scale_out, fvb_stream_t stream);

/* ------------------------------------------------- a5: GELU(tanh) -> FP8
 * Replaces fused_gelu_quant_fp8(y2) (fp8_ffn.py:57-72; kernels :24-54):
 *   g = bf16(gelu_tanh(h))  then quantise g exactly as fvb_quant_fp8. */
FVB_API int fvb_gelu_quant_fp8(const void* h, int64_t M, int64_t K, void* q, float* scale_out, int mode,
                       void* workspace, fvb_stream_t stream);

/* --------------------------------- a3: FP8 GEMM with scale/bias epilogue
 * Replaces FP8Linear._mm = torch._scaled_mm(x8, W.t(), scale_a, scale_b, bias,
 * out_dtype=bf16) (fp8_linear.py:28-30), run as a tcgen05 kind::f8f6f4 GEMM.
 *   out[m,n] = bf16( acc[m,n] * sa[m or 0] * sw[n or 0] + bias[n] )
 * A [M,K] fp8, W [N,K] fp8 (nn.Linear weight layout), bias [N] bf16 or NULL,
 * out [M,N] bf16.  a_mode / w_mode: FVB_SCALE_TENSOR or FVB_SCALE_ROW.
 * K must be a multiple of 16; A, W 16-byte aligned; out 16-byte aligned with N % 8 == 0.
 * epilogue: FVB_EPI_NONE, or FVB_EPI_GELU_AMAX (FFN up-projection):
 *   out = bf16(gelu_tanh(bf16(...)))  and  amax_out[m or 0] = max |out| via atomic max
 *   (amax_out must be zeroed by the caller; [M] floats for a_mode ROW, else [1]). */
#define FVB_EPI_NONE 0
#define FVB_EPI_GELU_AMAX 1
FVB_API int fvb_fp8_gemm(const void* A, const float* sa, int a_mode, const void* W, const float* sw,
                 int w_mode, const void* bias, int64_t M, int64_t N, int64_t K, void* out,
                 int epilogue, float* amax_out, fvb_stream_t stream);

/* Quantise with a precomputed amax (second half of the FFN mid-section):
 *   s = max(amax,1e-12)/448, q = e4m3(clamp(g/s)), scale_out = amax * fl(1/448). */
FVB_API int fvb_quant_fp8_with_amax(const void* g, int64_t M, int64_t K, const float* amax, int mode,
                            void* q, float* scale_out, fvb_stream_t stream);

/* ------------------------------------------------- a6: whole FP8 FFN
 * Replaces FP8FFN.forward (fp8_ffn.py:84-96) on pre-quantised input:
 *   h = gelu(x8 W0^T + b0) -> FP8 (mode) -> out = h8 W2^T + b2
 * x8 [M,D] fp8 with scale sx ([1] or [M] by mode), W0 [F,D], W2 [D,F] fp8 with
 * scales sw0 [1 or F], sw2 [1 or D] by w_mode, out [M,D] bf16.
 * workspace: fvb_fp8_ffn_workspace_bytes(M, F) bytes, 256-byte aligned. */
FVB_API size_t fvb_fp8_ffn_workspace_bytes(int64_t M, int64_t F);
FVB_API int fvb_fp8_ffn(const void* x8, const float* sx, int mode, const void* W0, const float* sw0,
                const void* b0, const void* W2, const float* sw2, const void* b2, int w_mode,
                int64_t M, int64_t D, int64_t F, void* out, void* workspace, fvb_stream_t stream);

/* The FFN and the DiT block's gated residual add after it in one call (the block's
 * x = fused_gate_add(x, gate_mlp, FP8FFN(.)), integrate.py:178-179 with fused_adaln.py:74-85):
 *   out = bf16(residual + bf16(gate * FFN(x8)))  bit for bit (gate == NULL: plain add),
 * the add applied in the down-projection's epilogue, so the FFN output is never stored and
 * re-read.  residual / out [M, D] bf16 (out may be residual itself), gate [D] bf16. */
FVB_API int fvb_fp8_ffn_residual(const void* x8, const float* sx, int mode, const void* W0,
                                 const float* sw0, const void* b0, const void* W2,
                                 const float* sw2, const void* b2, int w_mode, int64_t M,
                                 int64_t D, int64_t F, const void* residual, const void* gate,
                                 void* out, void* workspace, fvb_stream_t stream);

/* ------------------------------------------------- a7: RMSNorm + 3-D RoPE
 * Replaces fused_rms_rope(x, weight, freqs_cis, eps, rope, head_dim)
 * (fused_rms_rope.py:66-83; kernel :21-55):
 *   y = bf16(x * rsqrt(mean(x^2) + eps)) * w;  pairs (2i, 2i+1) inside each head rotate by
 *   (cos, sin)[s, i]:  (y_e c - y_o s, y_e s + y_o c);  out = bf16(...)
 * x [rows, D] bf16 with row pitch x_ld elements (x_ld == 0 -> D; lets q/k be read straight
 * out of a fused [rows, 3D] qkv projection), out [rows, D] contiguous (rows = B*L),
 * w [D] bf16, cos/sin [L, head_dim/2] fp32 indexed by
 * s = row % L.  rope == 0 skips the rotation (cos/sin may be NULL).
 * out_row_map (optional, [rows] int32): row r is written to out row out_row_map[r]
 * (used to emit window order directly); NULL = identity. */
FVB_API int fvb_rms_rope(const void* x, int64_t x_ld, const void* w, const float* cos, const float* sin,
                 int64_t rows, int64_t L, int64_t D, int64_t head_dim, float eps, int rope,
                 const int32_t* out_row_map, void* out, fvb_stream_t stream);

/* The self-attention's q, k and v in one launch (replaces the two fused_rms_rope calls on
 * self.q(x) / self.k(x) and the three WindowPartition3D.partition calls of the block,
 * integrate.py:58-77): from the fused projection qkv [rows, 3D] (row pitch x_ld, 0 -> 3D),
 *   out_q = fvb_rms_rope(q third, w_q, eps_q, rope), out_k = the same for k with w_k, eps_k,
 *   out_v = the v third, each input row r written to row out_row_map[r] of its output
 * (the window order; NULL = identity), bit for bit those three launches.  cos/sin as for
 * fvb_rms_rope (required). */
FVB_API int fvb_qkv_rope_window(const void* qkv, int64_t x_ld, const void* w_q, const void* w_k,
                                const float* cos, const float* sin, int64_t rows, int64_t L,
                                int64_t D, int64_t head_dim, float eps_q, float eps_k,
                                const int32_t* out_row_map, void* out_q, void* out_k,
                                void* out_v, fvb_stream_t stream);

/* ------------------------------------------------- a8: LayerNorm + modulate
 * Replaces fused_ln_modulate(x, scale, shift, eps) (fused_adaln.py:60-71; kernel :22-42):
 *   xn = bf16((x-mean)/sqrt(var+eps));  out = bf16(bf16(xn*bf16(1+scale)) + shift)
 * x/out [B,L,D] bf16, scale/shift [B,1,D] bf16 (note: scale BEFORE shift).
 * q8/q_scale (optional, both or neither): also emit the row's FP8 E4M3 codes with a
 * per-token scale exactly as fvb_quant_fp8(out, FVB_SCALE_ROW) would.  out may be NULL
 * when q8 is given (a consumer that takes only the FP8 codes). */
FVB_API int fvb_ln_modulate(const void* x, const void* scale, const void* shift, int64_t B, int64_t L,
                    int64_t D, float eps, void* out, void* q8, float* q_scale,
                    fvb_stream_t stream);

/* The DiT block's first norm with its AdaLN modulation sum formed in the same launch
 * (replaces `(self.modulation + t_mod).chunk(6, dim=1)` followed by fused_ln_modulate
 * with chunks 1 and 0, integrate.py:154-158):
 *   mod_out[b, c, :] = bf16(modulation[c, :] + t_mod[b, c, :])   (c = 0..5, one rounding,
 *                                                                  as torch's bf16 add)
 *   out = fvb_ln_modulate(x, scale = mod_out[:, 1], shift = mod_out[:, 0]) bit for bit.
 * modulation [6, D] (the block's [1, 6, D] parameter), t_mod [B, 6, D], mod_out [B, 6, D],
 * all bf16, contiguous, 16-byte aligned; q8/q_scale are required, out may be NULL. */
FVB_API int fvb_ln_modulate_adaln(const void* x, const void* modulation, const void* t_mod,
                                  int64_t B, int64_t L, int64_t D, float eps, void* out, void* q8,
                                  float* q_scale, void* mod_out, fvb_stream_t stream);

/* LayerNorm with affine weight/bias (the block's norm3: torch.nn.LayerNorm on bf16, which the
 * reference leaves to PyTorch, wan_video_dit DiTBlock.norm3):
 *   out = bf16( (x-mean)/sqrt(var+eps) * w + b )   fp32 math, one rounding
 *   (w, b [D] bf16; either may be NULL).
 * q8/q_scale (optional, both or neither): also emit out's per-token FP8 E4M3 codes and scales
 * exactly as fvb_quant_fp8(out, FVB_SCALE_ROW) would (the cross-attention q projection's
 * input quantisation, fp8_linear.py:60-66, done in the same pass).  out may be NULL when
 * q8 is given. */
FVB_API int fvb_layer_norm(const void* x, const void* w, const void* b, int64_t rows, int64_t D,
                   float eps, void* out, void* q8, float* q_scale, fvb_stream_t stream);

/* The gated residual add fused into the norm that reads its result (the DiT block runs
 * gate-add -> norm3 and cross-attention add -> norm2 back to back, integrate.py:167-173):
 * x_out = fvb_gate_add(x, gate, r) (bitwise), then the norm of x_out exactly as
 * fvb_ln_modulate / fvb_layer_norm compute it; the residual stream is read once.
 * gate [B,1,D] or NULL (plain add); x_out must not alias x or r; out may be NULL when q8
 * is given. */
FVB_API int fvb_gate_add_ln_modulate(const void* x, const void* gate, const void* r, void* x_out,
                                     const void* scale, const void* shift, int64_t B, int64_t L,
                                     int64_t D, float eps, void* out, void* q8, float* q_scale,
                                     fvb_stream_t stream);
FVB_API int fvb_gate_add_layer_norm(const void* x, const void* gate, const void* r, void* x_out,
                                    const void* w, const void* b, int64_t B, int64_t L, int64_t D,
                                    float eps, void* out, void* q8, float* q_scale,
                                    fvb_stream_t stream);

/* ------------------------------------------------- a9: gated residual
 * Replaces fused_gate_add(x, gate, residual) (fused_adaln.py:74-85; kernel :45-57):
 *   out = bf16(x + bf16(gate * r))  (bitwise equal to eager)
 * x/r/out [B,L,D] bf16, gate [B,1,D] bf16 (gate == NULL: plain out = bf16(x + r)). */
FVB_API int fvb_gate_add(const void* x, const void* gate, const void* r, int64_t B, int64_t L,
                 int64_t D, void* out, fvb_stream_t stream);

/* ------------------------------------------------- a11: keep mask -> CSR
 * Replaces build_csr(keep) (lcsa/triton_lcsa.py:64-71) without its host sync:
 *   cnt[h,q] = #kept; sel[h,q,:] = kept block ids ascending, then the unkept ids
 *   ascending (the stable-argsort order of the reference), row length NK (MAXK = NK).
 * keep [H,NQ,NK] uint8/bool, sel [H,NQ,NK] int32, cnt [H,NQ] int32. */
FVB_API int fvb_mask_to_csr(const uint8_t* keep, int64_t H, int64_t NQ, int64_t NK, int32_t* sel,
                    int32_t* cnt, fvb_stream_t stream);

/* ------------------------------------------------- a12: block-sparse attention
 * Replaces block_sparse_attention(q, k, v, keep, sm_scale) (lcsa/triton_lcsa.py:74-94;
 * kernel :19-61) and, through it, block_sparse_attn_func (compat_bsa.py:31-67):
 * for each head h and 128-row query block qb, softmax(q k^T * scale) v over the key
 * blocks sel[h,qb,0:cnt[h,qb]]; a row with no kept block outputs 0.
 * q [Lq, H*d], k/v [Lk, H*d], out [Lq, H*d] bf16 (window order; d == 128).
 * NQ = ceil(Lq/128); keys >= kv_len are masked (kv_len = Lk for whole blocks).
 * sel_stride = row length of sel (>= max cnt).  out_row_map (optional, [Lq] int32): query
 * row r is written to out row out_row_map[r] (window order in, raster order out); NULL =
 * identity.  tcgen05 kind::f16 kernel. */
FVB_API int fvb_bsa_fwd(const void* q, const void* k, const void* v, const int32_t* sel,
                const int32_t* cnt, int64_t sel_stride, int64_t H, int64_t Lq, int64_t Lk,
                int64_t kv_len, int64_t d, float scale, const int32_t* out_row_map, void* out,
                fvb_stream_t stream);

/* ------------------------------------------------- a14: window order
 * Replaces WindowPartition3D.partition / reverse (lcsa/reference.py:15-21;
 * integrate.py:75-77,117-120): [B,F,Hh,Ww,C] raster <-> [B*(F/wf)(Hh/wh)(Ww/ww), wf*wh*ww, C].
 * reverse == 0: raster -> window; reverse == 1: window -> raster.  Input rows have a pitch of
 * x_ld elements (0 -> C); the output is contiguous. */
FVB_API int fvb_window_partition(const void* x, int64_t x_ld, int64_t B, int64_t F, int64_t Hh,
                         int64_t Ww, int64_t C, int wf, int wh, int ww, int reverse, void* out,
                         fvb_stream_t stream);

/* ------------------------------------------------- a17: tile crops of a host video
 * Replaces the crop upload of render_tiled (tiling.py:190,
 * `lq[:, :, y:y + h, x:x + w].to(dev, non_blocking=True)`) for a pinned host video: one
 * strided copy-engine transfer, no host-side packing.  src holds `planes` planes of
 * `src_rows` rows, `src_pitch` bytes per row; the window of `height` rows of `width_bytes`
 * bytes at byte x_bytes of row y of every plane goes densely to dst
 * ([planes, height, width_bytes]).  Asynchronous on `stream` when src is pinned. */
FVB_API int fvb_copy_window_h2d(const void* src, int64_t src_pitch, int64_t src_rows,
                                int64_t planes, int64_t x_bytes, int64_t y, int64_t width_bytes,
                                int64_t height, void* dst, fvb_stream_t stream);

/* ------------------------------------------------- a13: keep-mask selection
 * Replaces draft_block_mask (lcsa/reference.py:37-64), i.e. upstream
 * generate_draft_block_mask called at integrate.py:103-104:
 *   window-mean pool q_w [NQ,128,H*d] and k_w [NK,128,H*d] -> per-head scores/sqrt(d),
 *   -inf outside local[sq,sk] (tiled over time rows), softmax over keys, joint top-k per
 *   (head, query time row) over (s m), keep = prob > (k+1)-th largest.
 * local [sq,sk] uint8; keep [H,NQ,NK] uint8.  q_temporal = NQ / sq.
 * workspace: fvb_draft_mask_workspace_bytes() bytes. */
FVB_API size_t fvb_draft_mask_workspace_bytes(int64_t H, int64_t NQ, int64_t NK, int64_t d);
FVB_API int fvb_draft_block_mask(const void* q_w, const void* k_w, int64_t H, int64_t NQ, int64_t NK,
                         int64_t d, const uint8_t* local, int64_t sq, int64_t sk,
                         int64_t q_temporal, int64_t topk, uint8_t* keep, void* workspace,
                         fvb_stream_t stream);

/* Measurement-input keep rule (no reference counterpart: the synthetic causal rule
 * of the benchmark configuration).  Query block i lives in time row i / per_row; key
 * block j in time row j / per_row - (NK - NQ) / per_row (cache rows first).  Keep
 * every key block of the query's own time row and the top floor(ratio * #past) past
 * blocks by mean-pooled q.k score; never a future row. */
FVB_API int fvb_causal_topk_mask(const void* q_w, const void* k_w, int64_t H, int64_t NQ, int64_t NK,
                         int64_t d, int64_t per_row, float ratio, uint8_t* keep, void* workspace,
                         fvb_stream_t stream);

/* The two halves of fvb_causal_topk_mask, for callers that keep the pooled means of
 * cached key blocks (a cached block's mean never changes, so a streaming caller pools
 * only the new time row).  fvb_block_mean_pool: out[b, c] = fp32 mean over the 128
 * tokens of window b of x [nblk, 128, C] bf16 (the avg_q / avg_k of
 * lcsa/reference.py:41-42, kept in fp32).  fvb_causal_topk_pooled: the keep rule above
 * from pooled aq [NQ, H*d] and ak [NK, H*d] (d % 4 == 0, both 16-byte aligned). */
FVB_API int fvb_block_mean_pool(const void* x, int64_t nblk, int64_t C, float* out,
                                fvb_stream_t stream);
/* fvb_causal_topk_pooled that also writes the rule's CSR in the same launch: sel
 * [H, NQ, NK] / cnt [H, NQ] exactly as fvb_mask_to_csr of the keep mask would (kept ids
 * ascending, then unkept ascending); keep may be NULL (mask not written). */
FVB_API int fvb_causal_topk_pooled_csr(const float* aq, const float* ak, int64_t H, int64_t NQ,
                                       int64_t NK, int64_t d, int64_t per_row, float ratio,
                                       uint8_t* keep, int32_t* sel, int32_t* cnt,
                                       fvb_stream_t stream);
/* Two fvb_block_mean_pool calls in one launch (the step's query windows and its new key
 * row): out = pool(x [nblk, 128, C]), out2 = pool(x2 [nblk2, 128, C]), bit for bit. */
FVB_API int fvb_block_mean_pool2(const void* x, int64_t nblk, const void* x2, int64_t nblk2,
                                 int64_t C, float* out, float* out2, fvb_stream_t stream);
FVB_API int fvb_causal_topk_pooled(const float* aq, const float* ak, int64_t H, int64_t NQ,
                                   int64_t NK, int64_t d, int64_t per_row, float ratio,
                                   uint8_t* keep, fvb_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* FLASHVSR_B200_H_ */
