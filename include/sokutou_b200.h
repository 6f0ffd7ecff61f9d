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
 *   - Pointers are raw device pointers of contiguous buffers owned by the caller; the kernels allocate
 *     nothing, so every call may be captured into a CUDA graph once the caller's buffers exist.
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

/* ---- dtypes ---------------------------------------------------------------------------------- */
#define SK_BF16 0
#define SK_F32 1

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
 * sk_decode_attention without a workspace argument: allocates nothing, for callers that cannot call
 * cudaMalloc when they attend (a serving process that reserves its device memory up front and
 * forbids allocation afterwards, a driver running inside a CUDA graph capture, a foreign-language
 * binding that only passes buffers it already owns). No counterpart in the reference: its kernel
 * (qwen3/kernels.py:338-414) keeps all scores in shared memory and needs no scratch.
 *
 * Same arguments and results as sk_decode_attention. The split-KV scratch is a 1 MiB array inside
 * the library's device image, one per device that loads the library, kept until the process exits.
 *   - Limit: the partials must fit 1 MiB minus 4 KiB, i.e. about nkv * ceil(max_len / 64) * 1040 bytes
 *     (nkv = 8: max_len up to 7936); larger calls return SK_ERR_TOO_LARGE and launch nothing.
 *   - The first call on each device looks up the array's address and zero-fills it, synchronously:
 *     make that first call before any stream capture.
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
