// DiT Q/K/V producer: per-head RMSNorm of q and k (sum of squares in double), × qk weight, RoPE on
// heads h < H/2 with interleaved pairs (2i, 2i+1); v copied. Same arithmetic as the reference's
// `qkv` kernel (engine/fused.py:117-180, the p < L branch), written for the split key layout: the
// conditioning K/V are not copied per batch row, the attention kernel reads them in place.
//
// One CTA per latent row (b, p); 128 threads. Warp w reduces heads w, w+4, ... of the 2H q/k heads.
#include "sk_common.cuh"

namespace sk {
namespace dit {

template <typename T>
struct Elem;
template <>
struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float ld(const __nv_bfloat16* p) { return __bfloat162float(*p); }
  static __device__ __forceinline__ __nv_bfloat16 st(float f) { return __float2bfloat16_rn(f); }
};
template <>
struct Elem<float> {
  static __device__ __forceinline__ float ld(const float* p) { return *p; }
  static __device__ __forceinline__ float st(float f) { return f; }
};

template <typename T>
__global__ void __launch_bounds__(128) qkv_prologue_kernel(const T* __restrict__ o4, const float* __restrict__ qk_w,
                                                            const float* __restrict__ freqs, T* __restrict__ q,
                                                            T* __restrict__ k, T* __restrict__ v, int L, int H, int HD,
                                                            float inv_hd, float eps) {
  extern __shared__ float rs[];  // [2H] 1/rms of the q heads then the k heads
  const int row = blockIdx.x, b = row / L, p = row % L;
  const int D = H * HD;
  const T* src = o4 + (size_t)row * 4 * D;
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  for (int hh = w; hh < 2 * H; hh += 4) {
    const T* x = src + (size_t)hh * HD;  // heads 0..H-1 are q, H..2H-1 are k
    double s = 0.0;
    for (int e = lane; e < HD; e += 32) {
      const float f = Elem<T>::ld(x + e);
      s += (double)f * f;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) rs[hh] = rsqrtf((float)(s * inv_hd) + eps);  // engine/fused.py:148
  }
  __syncthreads();
  const int half = HD / 2, npair = D / 2, rot_heads = H / 2;
  const float* fr = freqs + (size_t)p * HD;  // (pos, hd/2, 2) = cos, sin
  for (int j = t; j < 3 * npair; j += blockDim.x) {
    const int which = j / npair, rem = j % npair;
    const int h = rem / half, i = rem % half;
    const T* x = src + (size_t)which * D + h * HD + 2 * i;
    const size_t dst = (((size_t)b * H + h) * L + p) * HD + 2 * i;
    if (which == 2) {
      v[dst] = x[0];
      v[dst + 1] = x[1];
      continue;
    }
    const float r = rs[which * H + h];
    const float* wt = qk_w + (size_t)which * D + h * HD + 2 * i;
    float a0 = Elem<T>::ld(x) * r * wt[0], a1 = Elem<T>::ld(x + 1) * r * wt[1];
    if (h < rot_heads) {
      const float c = fr[2 * i], sn = fr[2 * i + 1];
      const float t0 = a0 * c - a1 * sn, t1 = a0 * sn + a1 * c;
      a0 = t0;
      a1 = t1;
    }
    T* out = which == 0 ? q : k;
    out[dst] = Elem<T>::st(a0);
    out[dst + 1] = Elem<T>::st(a1);
  }
}

}  // namespace dit
}  // namespace sk

extern "C" int sk_dit_qkv_prologue(const void* o4, const float* qk_w, const float* freqs, void* q, void* k_lat,
                                   void* v_lat, int B, int L, int H, int hd, float eps, int dtype, void* stream) {
  using namespace sk::dit;
  if (!o4 || !qk_w || !freqs || !q || !k_lat || !v_lat) return SK_ERR_INVALID_ARG;
  if (B <= 0 || L <= 0 || H <= 0 || H % 2 || hd <= 0 || hd % 2) return SK_ERR_INVALID_ARG;
  if (dtype != SK_BF16 && dtype != SK_F32) return SK_ERR_UNSUPPORTED;
  int rc = sk_check_device();
  if (rc != SK_OK) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const size_t smem = 2 * (size_t)H * sizeof(float);
  if (dtype == SK_BF16)
    qkv_prologue_kernel<__nv_bfloat16><<<B * L, 128, smem, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(o4), qk_w, freqs, reinterpret_cast<__nv_bfloat16*>(q),
        reinterpret_cast<__nv_bfloat16*>(k_lat), reinterpret_cast<__nv_bfloat16*>(v_lat), L, H, hd, 1.f / hd, eps);
  else
    qkv_prologue_kernel<float><<<B * L, 128, smem, st>>>(reinterpret_cast<const float*>(o4), qk_w, freqs,
                                                         reinterpret_cast<float*>(q), reinterpret_cast<float*>(k_lat),
                                                         reinterpret_cast<float*>(v_lat), L, H, hd, 1.f / hd, eps);
  return cudaPeekAtLastError() == cudaSuccess ? SK_OK : SK_ERR_CUDA;
}
