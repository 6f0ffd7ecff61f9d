// DiT Q/K/V producer: per-head RMSNorm of q and k (sum of squares in double), × qk weight, RoPE on
// heads h < H/2 with interleaved pairs (2i, 2i+1); v copied. Same arithmetic as the reference's
// `qkv` kernel (engine/fused.py:117-180, the p < L branch), written for the split key layout: the
// conditioning K/V are not copied per batch row, the attention kernel reads them in place.
//
// One warp per (latent row, q/k/v head): vector loads of the head's hd elements, a warp-wide
// double-precision sum of squares, and in-lane RoPE pairs.
#include "sk_common.cuh"

namespace sk {
namespace dit {

template <typename T, int PER>
struct LaneVec;  // PER consecutive elements of one lane, loaded/stored as one vector
template <>
struct LaneVec<__nv_bfloat16, 2> {
  static __device__ __forceinline__ void ld(const __nv_bfloat16* p, float* x) {
    const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(p);
    x[0] = __low2float(v);
    x[1] = __high2float(v);
  }
  static __device__ __forceinline__ void st(__nv_bfloat16* p, const float* x) {
    *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(x[0], x[1]);
  }
};
template <>
struct LaneVec<__nv_bfloat16, 4> {
  static __device__ __forceinline__ void ld(const __nv_bfloat16* p, float* x) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    x[0] = __uint_as_float(u.x << 16);
    x[1] = __uint_as_float(u.x & 0xffff0000u);
    x[2] = __uint_as_float(u.y << 16);
    x[3] = __uint_as_float(u.y & 0xffff0000u);
  }
  static __device__ __forceinline__ void st(__nv_bfloat16* p, const float* x) {
    const __nv_bfloat162 a = __floats2bfloat162_rn(x[0], x[1]), b = __floats2bfloat162_rn(x[2], x[3]);
    *reinterpret_cast<uint2*>(p) = make_uint2(*reinterpret_cast<const uint32_t*>(&a), *reinterpret_cast<const uint32_t*>(&b));
  }
};
template <int PER>
struct LaneVec<float, PER> {
  static __device__ __forceinline__ void ld(const float* p, float* x) {
#pragma unroll
    for (int i = 0; i < PER; ++i) x[i] = p[i];
  }
  static __device__ __forceinline__ void st(float* p, const float* x) {
#pragma unroll
    for (int i = 0; i < PER; ++i) p[i] = x[i];
  }
};

// One warp per (latent row, slot), slot in [0, 3H): q heads, then k heads, then v heads. Lane l holds
// the HD/32 consecutive elements [l*PER, l*PER + PER) of its head, so every RoPE pair stays in one lane.
template <typename T, int HD>
__global__ void __launch_bounds__(256) qkv_prologue_kernel(const T* __restrict__ o4, const float* __restrict__ qk_w,
                                                            const float* __restrict__ freqs, T* __restrict__ q,
                                                            T* __restrict__ k, T* __restrict__ v, int L, int H,
                                                            long long n_warps, float inv_hd, float eps) {
  constexpr int PER = HD / 32;
  const long long gw = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (gw >= n_warps) return;
  const int lane = threadIdx.x & 31;
  const int slots = 3 * H;
  const long long row = gw / slots;
  const int slot = (int)(gw % slots);
  const int which = slot / H, h = slot % H;
  const int b = (int)(row / L), p = (int)(row % L);
  const int D = H * HD;
  const int e0 = lane * PER;
  const T* src = o4 + (size_t)row * 4 * D + (size_t)which * D + (size_t)h * HD + e0;
  const size_t dst = (((size_t)b * H + h) * L + p) * HD + e0;
  float x[PER];
  LaneVec<T, PER>::ld(src, x);
  if (which == 2) {  // v: copied as is
    LaneVec<T, PER>::st(v + dst, x);
    return;
  }
  double ss = 0.0;  // sum of squares in double, as engine/fused.py:143
#pragma unroll
  for (int i = 0; i < PER; ++i) ss += (double)x[i] * x[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float r = rsqrtf((float)(ss * inv_hd) + eps);  // engine/fused.py:148
  const float* wt = qk_w + (size_t)which * D + (size_t)h * HD + e0;
#pragma unroll
  for (int i = 0; i < PER; ++i) x[i] = x[i] * r * wt[i];
  if (h < H / 2) {  // RoPE on the first H/2 heads, interleaved pairs (engine/fused.py:152-171)
    const float* fr = freqs + (size_t)p * HD + e0;  // (pos, hd/2, 2): pair i at [2i] cos, [2i+1] sin
#pragma unroll
    for (int i = 0; i < PER; i += 2) {
      const float c = fr[i], sn = fr[i + 1];
      const float a0 = x[i], a1 = x[i + 1];
      x[i] = a0 * c - a1 * sn;
      x[i + 1] = a0 * sn + a1 * c;
    }
  }
  LaneVec<T, PER>::st((which == 0 ? q : k) + dst, x);
}

}  // namespace dit
}  // namespace sk

extern "C" int sk_dit_qkv_prologue(const void* o4, const float* qk_w, const float* freqs, void* q, void* k_lat,
                                   void* v_lat, int B, int L, int H, int hd, float eps, int dtype, void* stream) {
  using namespace sk::dit;
  if (!o4 || !qk_w || !freqs || !q || !k_lat || !v_lat) return SK_ERR_INVALID_ARG;
  if (B <= 0 || L <= 0 || H <= 0 || H % 2) return SK_ERR_INVALID_ARG;
  if (hd != 64 && hd != 128) return SK_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(o4) | reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k_lat) |
       reinterpret_cast<uintptr_t>(v_lat)) & 15)
    return SK_ERR_INVALID_ARG;
  if (dtype != SK_BF16 && dtype != SK_F32) return SK_ERR_UNSUPPORTED;
  int rc = sk_check_device();
  if (rc != SK_OK) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const long long n_warps = (long long)B * L * 3 * H;
  const int blocks = (int)((n_warps + 7) / 8);
  const float inv = 1.f / hd;
#define SK_PROLOGUE(T, HDV)                                                                                        \
  qkv_prologue_kernel<T, HDV><<<blocks, 256, 0, st>>>(reinterpret_cast<const T*>(o4), qk_w, freqs,                 \
                                                      reinterpret_cast<T*>(q), reinterpret_cast<T*>(k_lat),        \
                                                      reinterpret_cast<T*>(v_lat), L, H, n_warps, inv, eps)
  if (dtype == SK_BF16) {
    if (hd == 64) SK_PROLOGUE(__nv_bfloat16, 64);
    else SK_PROLOGUE(__nv_bfloat16, 128);
  } else {
    if (hd == 64) SK_PROLOGUE(float, 64);
    else SK_PROLOGUE(float, 128);
  }
#undef SK_PROLOGUE
  return cudaPeekAtLastError() == cudaSuccess ? SK_OK : SK_ERR_CUDA;
}
