// Per-element arithmetic of the DiT Q/K producer (engine/fused.py:138-171), shared by the standalone
// producer kernel and the fused attention layer so that both give the same q and k bits:
//   r = rsqrt(sum_e x_e^2 / hd + eps)       (sum of squares accumulated in double, engine/fused.py:143-148)
//   a_e = x_e · r · w_e                      (fp32, in that order)
//   heads h < H/2: (a_2i, a_2i+1) <- (a_2i·cos - a_2i+1·sin, a_2i·sin + a_2i+1·cos), (cos, sin) =
//   freqs[pos][i]                             (engine/fused.py:152-171)
#pragma once

namespace sk {
namespace dit {

__device__ __forceinline__ float qk_inv_rms(double ss, float inv_hd, float eps) {
  return rsqrtf((float)(ss * inv_hd) + eps);
}

// N consecutive elements starting at an even index: scale by r·w, then rotate the pairs when fr != nullptr
// (fr points at the (cos, sin) pairs of these elements: fr[2k], fr[2k+1] for pair k).
template <int N>
__device__ __forceinline__ void qk_scale_rotate(float* x, float r, const float* w, const float* fr) {
#pragma unroll
  for (int i = 0; i < N; ++i) x[i] = x[i] * r * w[i];
  if (fr != nullptr) {
#pragma unroll
    for (int i = 0; i < N; i += 2) {
      const float c = fr[i], sn = fr[i + 1];
      const float a0 = x[i], a1 = x[i + 1];
      x[i] = a0 * c - a1 * sn;
      x[i + 1] = a0 * sn + a1 * c;
    }
  }
}

}  // namespace dit
}  // namespace sk
