/*
 * sokutou_b200 — C ABI of the B200 (sm_100a) attention path for the sokutou TTS engine.
 *
 * Two attention shapes are served, each a drop-in for one call site of the reference engine
 * (paths are relative to the sokutou project root):
 *
 *   1. Irodori-TTS DiT attention (non-causal, CFG-batched, key-padding bias).
 *      Replaces `F.scaled_dot_product_attention(q, k, v, attn_mask=bias)` at engine/fused.py:295
 *      (exact-math twin: engine/fast.py:169-173) and the Q/K/V producer kernel `qkv`
 *      launched at engine/fused.py:293-294 (kernel source engine/fused.py:117-180).
 *
 *   2. Qwen3-TTS talker decode attention (batch 1, GQA, QK-RMSNorm + RoPE + KV append fused).
 *      Replaces the NVRTC kernel `attn` (qwen3/kernels.py:338-414) launched at
 *      qwen3/kernels.py:622-624 and :607-609.
 *
 * Conventions
 *   - Every entry point returns an int status: SK_OK (0) or a negative SK_ERR_* code. Nothing aborts.
 *   - Pointers are raw device pointers of contiguous buffers owned by the caller, and the kernels
 *     allocate nothing (sk_decode_attention_noalloc keeps its scratch in a fixed array of its own).
 *     The DiT, gate, projection, prefill, decode, decode-block and grouped-decode entry points launch
 *     kernels only, so their calls can be captured into a CUDA graph once the caller's buffers exist
 *     (graph-replay tests cover the DiT attention and fused block, the projections, the decode, the
 *     decode block and grouped decode).
 *   - `stream` is a cudaStream_t passed as void* so that this header needs no CUDA include.
 *   - Launches are asynchronous. A device-side failure (an invalid position read from device memory,
 *     a bounded wait that ran out) is recorded in a per-device error word; read it with
 *     sk_device_error().
 */
#ifndef SOKUTOU_B200_H
#define SOKUTOU_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define SK_API __attribute__((visibility("default")))
#else
#define SK_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------------------------------- */
#define SK_OK 0
#define SK_ERR_INVALID_ARG (-1)   /* null pointer, bad size, misaligned buffer */
#define SK_ERR_UNSUPPORTED (-2)   /* shape outside what the kernels implement (e.g. head_dim) */
#define SK_ERR_CUDA (-3)          /* a CUDA runtime call failed (launch, attribute, ...) */
#define SK_ERR_DEVICE (-4)        /* the current device is not an sm_100 part */
#define SK_ERR_WORKSPACE (-5)     /* workspace missing or smaller than sk_decode_workspace_bytes() */
#define SK_ERR_TOO_LARGE (-6)     /* the call needs more scratch than sk_decode_attention_noalloc holds */

/* device error word values (sk_device_error) */
#define SK_DEVERR_NONE 0
#define SK_DEVERR_POS_RANGE 1     /* decode: pos_ptr[0] + pos_add outside [0, max_len) */
#define SK_DEVERR_TIMEOUT 2       /* a bounded mbarrier wait ran out */
#define SK_DEVERR_BOUNDS 3        /* bounds-checked build only: an index outside its buffer (access skipped) */

/* ---- dtypes ---------------------------------------------------------------------------------- */
#define SK_BF16 0
#define SK_F32 1
#define SK_E4M3 2   /* FP8 e4m3 output (sk_dit_gate only) */

/* Library version (major*10000 + minor*100 + patch). */
SK_API int sk_version(void);

/* Reads the error word of the current device (synchronises the device). When reset != 0 the word is
 * cleared after reading. *code receives one of SK_DEVERR_*. */
SK_API int sk_device_error(int* code, int reset);

/* ---- 1. DiT attention ------------------------------------------------------------------------- */

/*
 * y = softmax(q·kᵀ·scale + key_bias) · v, non-causal, per (batch b, head h).
 *
 * Replaces engine/fused.py:295 `F.scaled_dot_product_attention(q, k, v, attn_mask=bias)`.
 * Keys come from two sources so that the conditioning (text + speaker) keys need not be copied
 * per CFG branch (the reference copies them into every batch row, engine/fused.py:127-136):
 *
 *   key index j in [0, Lk)       : k_lat/v_lat, layout (B, H, Lk, hd) contiguous
 *   key index j in [Lk, Lk + S)  : k_ctx/v_ctx, layout (S, H, hd) per batch row, batch row b at
 *                                  element offset b * ctx_batch_stride (0 = shared by all rows)
 *
 * The plain SDPA form is Lk = K, S = 0, k_ctx = v_ctx = NULL.
 *
 *   q        : (B, H, L, hd)
 *   key_bias : additive mask, K = Lk + S values per batch row at element offset b * bias_batch_stride
 *              (0 = shared), same dtype as q; NULL = no mask. The reference passes 0 / -inf
 *              (engine/fused.py:373-378). A row whose keys are all -inf yields zeros (as torch does).
 *   y        : (B, L, H, hd) contiguous — the memory order the `gate` consumer reads
 *              (engine/fused.py:296-298).
 *   dtype    : SK_BF16 — tcgen05 tensor-core kernel, fp32 accumulation, P rounded to bf16;
 *              SK_F32  — fp32 CUDA-core kernel (the fp32 parity mode).
 *   scale    : softmax scale; <= 0 selects 1/sqrt(hd) (the SDPA default used by the reference).
 *   hd       : 64 or 128. All pointers 16-byte aligned.
 */
SK_API int sk_dit_attention(const void* q, const void* k_lat, const void* v_lat,
                     const void* k_ctx, const void* v_ctx, const void* key_bias, void* y,
                     int B, int H, int L, int Lk, int S, int hd,
                     long long ctx_batch_stride, long long bias_batch_stride,
                     int dtype, float scale, void* stream);

/*
 * The Q/K/V producer of one DiT layer: per-head RMSNorm of q and k (sum of squares in double,
 * × qk_w), RoPE on heads h < H/2 with interleaved pairs (2i, 2i+1), v copied.
 * Replaces the `qkv` kernel, engine/fused.py:117-180 (launch :293-294), without its per-batch copy of
 * the conditioning K/V (the attention reads those in place).
 *
 *   o4    : (B*L, 4*H*hd) rows [q | k | v | gate], dtype `dtype`
 *   qk_w  : fp32 (2, H, hd) — q_norm then k_norm weights
 *   freqs : fp32 (>= L, hd/2, 2) — (cos, sin) per latent position
 *   q     : (B, H, L, hd);  k_lat, v_lat : (B, H, L, hd)   (dtype `dtype`)
 *   hd    : 64 or 128; all buffers 16-byte aligned.
 */
SK_API int sk_dit_qkv_prologue(const void* o4, const float* qk_w, const float* freqs,
                        void* q, void* k_lat, void* v_lat,
                        int B, int L, int H, int hd, float eps, int dtype, void* stream);

/*
 * The whole attention block of one DiT layer (bf16): the Q/K/V producer, the attention and the gate
 * consumer, replacing the three launches at engine/fused.py:293-298 — `qkv` (engine/fused.py:117-180),
 * F.scaled_dot_product_attention (:295) and `gate` (:182-190). At hd = 64 it takes two launches: the
 * producer writes only q and k, and the attention kernel reads v and the gate tile straight from o4
 * and writes the gated output (neither v nor y reaches HBM). At hd = 128 it runs the three kernels
 * (y through `out`, gated in place), which measured faster there. Each launch's set-up overlaps the
 * previous kernel through programmatic dependent launch:
 *
 *   q, k  = per-head RMSNorm (× qk_w) + RoPE (heads h < H/2) of the q/k quarters of o4
 *   y     = softmax(q·kᵀ·scale + key_bias) · v over keys [latent (L) | ctx (S)], rounded to bf16
 *   out   = y · sigmoid(o4[:, 3D:4D]) in fp32, rounded to bf16
 *
 *   o4           : (B*L, 4*H*hd) bf16 rows [q | k | v | gate]
 *   qk_w, freqs  : fp32 (2, H, hd) and (>= L, hd/2, 2), as for sk_dit_qkv_prologue
 *   k_ctx, v_ctx, key_bias, ctx_batch_stride, bias_batch_stride, scale: as for sk_dit_attention
 *   out          : (B, L, H, hd) = (B*L, H*hd) bf16
 *   q_buf, k_buf, v_buf : caller-owned scratch, (B, H, L, hd) bf16 each, overwritten (v_buf is left
 *                  untouched at hd = 64); the engine already allocates its q/k/v buffers before
 *                  capture (engine/fused.py:277-282). out must not overlap o4.
 *   dtype        : SK_BF16 only (the fp32 parity mode runs the three separate entry points)
 *   hd 64 or 128, H even, all pointers 16-byte aligned.
 * Same bits as sk_dit_qkv_prologue + sk_dit_attention + sk_dit_gate on the same inputs.
 */
SK_API int sk_dit_attention_layer(const void* o4, const float* qk_w, const float* freqs,
                                  const void* k_ctx, const void* v_ctx, const void* key_bias, void* out,
                                  void* q_buf, void* k_buf, void* v_buf, int B, int H, int L, int S, int hd,
                                  long long ctx_batch_stride, long long bias_batch_stride,
                                  float eps, int dtype, float scale, void* stream);

/*
 * The attention consumer of one DiT layer: out[r, c] = y[r, c] · sigmoid(o4[r, 3·D + c]) for every
 * row r of the B·L latent rows and c < D = H·hd. Replaces the `gate` kernel, engine/fused.py:182-190
 * (launch :296-298): fp32 product y · (1 / (1 + expf(-g))), rounded once to the output type.
 *
 *   y         : (rows, D) = the (B, L, H, hd) output of sk_dit_attention, dtype `dtype`
 *   o4        : (rows, 4·D) fused projection rows [q | k | v | gate], dtype `dtype`
 *   out       : (rows, D) in `out_dtype`: the same dtype, or SK_E4M3 — FP8 e4m3 of value·out_scale,
 *               round to nearest even, ±448 saturation, NaN → 0x7f (the reference's FP8 GEMM input,
 *               engine/fused.py:52-76, engine/fp8.py)
 *   D         : multiple of 8; y and o4 16-byte aligned, out 16-byte (8-byte for SK_E4M3) aligned.
 *               out may be y itself (same dtype): the gate is then applied in place.
 */
SK_API int sk_dit_gate(const void* y, const void* o4, void* out, long long rows, int D, int dtype,
                       int out_dtype, float out_scale, void* stream);

/*
 * One DiT projection: y = x · wᵀ (F.linear without bias), the `mm` of engine/fused.py:262-264 that
 * the engine calls for w_qkvg, w_o, w_13 and w_2 (engine/fused.py:293-310). tcgen05 tiles of
 * 128 x 256 with fp32 accumulation, rounded once to bf16.
 *
 *   x      : (M, K) bf16 rows (the step's latent rows)
 *   w      : (N, K) bf16, the weight as nn.Linear stores it
 *   y      : (M, N) bf16; must not overlap x or w
 *   dtype  : SK_BF16 only (the fp32 parity mode keeps the library GEMM)
 *   K and N multiples of 8; all pointers 16-byte aligned.
 */
SK_API int sk_dit_linear(const void* x, const void* w, void* y, int M, int N, int K, int dtype, void* stream);
/* sk_dit_linear with the N width of the CTA tile given: 64, 128 or 256 (0: chosen per call from the
 * grid it gives, as sk_dit_linear does). */
SK_API int sk_dit_linear_ex(const void* x, const void* w, void* y, int M, int N, int K, int dtype, int tile_n,
                            void* stream);

/*
 * The FP8 projection of the engine's FP8 path (engine/fp8.py:87-89, torch._scaled_mm):
 * y = (x8 · w8ᵀ) · inv_scale_x · inv_scale_w, fp32 accumulation, rounded once to bf16.
 *
 *   x8          : (M, K) e4m3 bytes (the activation, written by sk_dit_gate with SK_E4M3 for w_o)
 *   w8          : (N, K) e4m3 bytes (the weight times its power-of-two scale)
 *   y           : (M, N) bf16
 *   inv_scale_x, inv_scale_w : device fp32 scalars, read by the kernel (set before graph capture)
 *   tile_n      : 0 (chosen per call), 64, 128 or 256
 *   K a multiple of 16, N a multiple of 8, pointers 16-byte aligned.
 */
SK_API int sk_dit_linear_fp8(const void* x8, const void* w8, void* y, const float* inv_scale_x,
                             const float* inv_scale_w, int M, int N, int K, int tile_n, void* stream);

/* ---- 2. Qwen3 talker decode attention --------------------------------------------------------- */

/* Bytes of scratch sk_decode_attention needs for a cache of max_len positions. */
SK_API size_t sk_decode_workspace_bytes(int max_len, int nq, int nkv, int hd, int cache_dtype);

/*
 * One decode step of GQA attention for one layer, with the reference kernel's argument list
 * (qkv, qn, kn, eps, rope, Kc, Vc, pos_ptr, pos_add, max_len, nq, nkv, out) —
 * qwen3/kernels.py:341-344, launched at :622-624.
 *
 *   pos  = (pos_ptr ? pos_ptr[0] : 0) + pos_add, read on the device (one graph serves every step);
 *          T = pos + 1 keys are attended.
 *   qkv  : fp32 [(nq + 2*nkv) * hd] = [q heads | k heads | v heads]
 *   qn,kn: fp32 [hd] RMSNorm weights; eps as in the model config
 *   rope : fp32 [max_len][hd] = [cos(hd/2) | sin(hd/2)] (rotate-half convention)
 *   Kc,Vc: this layer's cache [nkv][max_len][hd], bf16 (cache_dtype SK_BF16) or fp32 (SK_F32).
 *          Position pos is written (k normed + roped, v raw) and then attended, rounded to the cache
 *          dtype exactly as the reference reads it back.
 *   out  : fp32 [nq * hd]
 *   workspace: caller-owned scratch of sk_decode_workspace_bytes() bytes, zero-filled once before
 *          first use (the kernel leaves it zeroed again after every call).
 * Split-KV flash decoding: the T keys are cut into chunks processed by separate CTAs and merged by
 * the last CTA to finish, so T is bounded only by max_len.
 * Supported: hd = 128, nq = 2*nkv (the reference's own restriction, qwen3/kernels.py:457).
 */
SK_API int sk_decode_attention(const float* qkv, const float* qn, const float* kn, float eps,
                        const float* rope, void* Kc, void* Vc,
                        const long long* pos_ptr, int pos_add, int max_len, int nq, int nkv, int hd,
                        float* out, void* workspace, size_t ws_bytes, int cache_dtype, void* stream);

/*
 * sk_decode_attention with launch options (`flags`, a bit set; 0 gives exactly sk_decode_attention):
 *
 *   SK_DECODE_KV_STABLE — the caller promises that the kernel launched immediately before this call
 *     on the stream writes neither pos_ptr[0] nor this layer's cache rows [0, pos). The kernel then
 *     reads the position and issues the copies of its K/V chunk before waiting for that kernel
 *     (programmatic dependent launch), so the cache reads overlap that kernel's tail; qkv, qn and kn
 *     are still read only after it has finished. True at the reference's call site, where the
 *     attention follows the layer's rms_gemv (qwen3/kernels.py:619-627); not for the first layer
 *     right after the kernel that advances the position.
 * No counterpart in the reference (its kernel has no launch options).
 */
#define SK_DECODE_KV_STABLE 1
SK_API int sk_decode_attention_ex(const float* qkv, const float* qn, const float* kn, float eps,
                                  const float* rope, void* Kc, void* Vc,
                                  const long long* pos_ptr, int pos_add, int max_len, int nq, int nkv, int hd,
                                  float* out, void* workspace, size_t ws_bytes, int cache_dtype, int flags,
                                  void* stream);

/*
 * Qwen3 prefill attention: the prompt's causal self-attention, which the reference runs inside the HF
 * talker with SDPA (qwen3/fast.py:251-263): bf16 caches on the tensor-core kernel with a causal mask
 * and GQA; fp32 caches (the fp32 parity mode) on the fp32 CUDA-core kernel with the same masking.
 * For every prompt token t in [0, T) at position pos0 + t:
 *   - q heads RMS-normalised (× qn) and rotated (rotate-half RoPE from `rope`, as sk_decode_attention),
 *     k normalised (× kn) and rotated, v raw; k and v appended to the caches at row pos0 + t (the bits
 *     decode steps would write);
 *   - out[t] = softmax(q·kᵀ / sqrt(128)) · v over the cache rows [0, pos0 + t] of the key/value head
 *     h / 2 (earlier rows pos0 > 0: a prompt chunk after a cached prefix).
 *   qkv   : fp32 (T, (nq + 2*nkv) * 128) rows = [q heads | k heads | v heads] per token
 *   Kc, Vc: this layer's cache [nkv][max_len][128], bf16 (SK_BF16) or fp32 (SK_F32)
 *   out   : (T, nq * 128) in the cache dtype;  q_buf: caller scratch (nq, T, 128) in the cache dtype
 *   hd = 128, nq = 2*nkv, pos0 + T <= max_len; buffers 16-byte aligned.
 */
SK_API int sk_prefill_attention(const float* qkv, const float* qn, const float* kn, float eps,
                                const float* rope, void* Kc, void* Vc, int pos0, int T, int max_len,
                                int nq, int nkv, int hd, void* out, void* q_buf, int cache_dtype,
                                void* stream);

/*
 * One independent decode request of sk_decode_attention_grouped: the scalar arguments of
 * sk_decode_attention for one talker (its qkv, norms, RoPE table, this layer's caches, its position on
 * the device and its output). 80 bytes; an array of them lives in device memory.
 */
typedef struct SkDecodeRequest {
  const float* qkv;          /* [(nq + 2*nkv) * hd] */
  const float* qn;           /* [hd] */
  const float* kn;           /* [hd] */
  const float* rope;         /* [max_len][hd] */
  void* Kc;                  /* [nkv][max_len][hd], cache_dtype */
  void* Vc;
  const long long* pos_ptr;  /* the request's position on the device (NULL: pos = pos_add) */
  float* out;                /* [nq * hd] */
  int pos_add;
  float eps;
  int reserved[2];
} SkDecodeRequest;

/*
 * R independent decode requests in one launch: request r does what sk_decode_attention does with the
 * arguments in reqs[r] — the same appended cache rows, and the output of its thread-block-cluster kernel
 * (the same bits where sk_decode_attention runs that kernel with the same cluster size; within rounding
 * otherwise: the grouped launch takes clusters of 8 where more of them than of 16 are resident at once,
 * and the chunk split sets the merge order) — all sharing max_len, nq, nkv, hd and the cache dtype. No counterpart in the reference, which serves one request at a time (README.md:186): a server
 * holding several talkers' decodes in flight gets one launch per layer for all of them instead of one
 * per request, and so moves R times the cache bytes per launch.
 *   reqs  : DEVICE pointer to R descriptors (filled before capture; they are read on the device)
 *   flags : 0 or SK_DECODE_KV_STABLE, as sk_decode_attention_ex (for every request)
 * Caches must be short enough for the cluster kernel (bf16: max_len up to 5040; fp32: 2528), else
 * SK_ERR_UNSUPPORTED. Positions out of range set SK_DEVERR_POS_RANGE and skip that request.
 */
SK_API int sk_decode_attention_grouped(const SkDecodeRequest* reqs, int R, int max_len, int nq, int nkv, int hd,
                                       int cache_dtype, int flags, void* stream);

/* Bytes of workspace sk_decode_attention_block needs for caches of max_len positions. */
SK_API size_t sk_decode_block_workspace_bytes(int max_len, int nq, int nkv, int hd);

/*
 * One talker layer's whole attention block in a single launch — the three launches the reference
 * makes per layer at qwen3/kernels.py:619-624:
 *   rms_gemv(qkv) (qwen3/kernels.py:271-275):  qkv = W_qkv · (h ⊙ in_norm) · 1/sqrt(mean(h²) + eps_in)
 *   attn          (qwen3/kernels.py:341-414):  att = the decode attention of sk_decode_attention on qkv
 *                                              (QK-RMSNorm, RoPE, K/V appended at pos, GQA over T = pos + 1)
 *   gemv(o)       (qwen3/kernels.py:301-305):  h += W_o · att   (accumulate = 1: the residual add)
 *
 *   h        : fp32 [hidden], the residual stream, updated in place
 *   in_norm  : fp32 [hidden], the layer's input RMSNorm weight; eps_in its epsilon
 *   w_qkv    : [(nq + 2*nkv) * hd][hidden] (q rows, then k, then v), bf16 or fp32 (weight_dtype)
 *   w_o      : [hidden][nq * hd], same dtype
 *   qn, kn, eps, rope, Kc, Vc, pos_ptr, pos_add, max_len, nq, nkv, hd, cache_dtype: as sk_decode_attention
 *   workspace: caller-owned, sk_decode_block_workspace_bytes() bytes, zero-filled once before first use
 *              (every launch leaves its counters at zero; after a device error, zero it again)
 *   flags    : 0 or SK_DECODE_KV_STABLE (the position and this layer's cache rows may be read before the
 *              kernel just before has finished; the weights are always prefetched before that wait)
 * One cooperative launch (one CTA per SM, all resident) with two grid-wide barriers between the
 * phases; no float atomics, so results are identical from run to run. hidden a multiple of 8 and at
 * most 2048 (nq * hd at most 2048); the attention's partials of every 128-key chunk must fit one CTA's
 * shared memory (nkv = 8: max_len up to 3328), else SK_ERR_UNSUPPORTED; all pointers 16-byte aligned;
 * hd = 128, nq = 2*nkv.
 */
SK_API int sk_decode_attention_block(float* h, const float* in_norm, float eps_in, const void* w_qkv,
                                     const float* qn, const float* kn, float eps, const float* rope,
                                     void* Kc, void* Vc, const long long* pos_ptr, int pos_add, int max_len,
                                     int nq, int nkv, int hd, const void* w_o, int hidden, int weight_dtype,
                                     int cache_dtype, void* workspace, size_t ws_bytes, int flags, void* stream);

/*
 * sk_decode_attention without a workspace argument: allocates nothing, for callers that cannot call
 * cudaMalloc when they attend (a serving process that reserves its device memory up front and
 * forbids allocation afterwards, a foreign-language binding that only passes buffers it already
 * owns and has no allocator of its own). No counterpart in the reference: its kernel
 * (qwen3/kernels.py:338-414) keeps all scores in shared memory and needs no scratch.
 *
 * Same arguments and results as sk_decode_attention. The split-KV scratch is a 1 MiB array inside
 * the library's device image, one per device that loads the library, kept until the process exits.
 *   - Limit: the partials, nkv * ceil(max_len / 64) * 1040 bytes, must fit 1 MiB minus 4 KiB
 *     (1 044 480 bytes; nkv = 8: max_len up to 8000); larger calls return SK_ERR_TOO_LARGE and
 *     launch nothing.
 *   - The first call on each device looks up the array's address, zero-fills it and waits for the
 *     whole device (cudaDeviceSynchronize) before it launches anything, so that first call may go on
 *     any stream but must come before any stream capture.
 *   - Every call shares the array. Calls that may run at the same time on the GPU (different streams,
 *     or graphs replayed concurrently) race on it; serialise them or use sk_decode_attention.
 */
SK_API int sk_decode_attention_noalloc(const float* qkv, const float* qn, const float* kn, float eps,
                        const float* rope, void* Kc, void* Vc,
                        const long long* pos_ptr, int pos_add, int max_len, int nq, int nkv, int hd,
                        float* out, int cache_dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SOKUTOU_B200_H */
