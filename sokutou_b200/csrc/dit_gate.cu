// DiT attention consumer: out = y · sigmoid(gate), the `gate` kernel of engine/fused.py:182-190
// (launch :296-298). y is the attention output (B, L, H, hd) — row (b, p) holds H·hd = D values —
// and the gate is the last quarter of the fused projection row o4 (B·L, 4·D). Same arithmetic as the
// reference: fp32 product y · (1 / (1 + expf(−g))), rounded once to the output type; the output is
// the working dtype, or FP8 e4m3 scaled by `out_scale` for the FP8 GEMM that follows
// (engine/fused.py:52-76 `STO`, engine/fp8.py).
//
// HBM-bound: one thread per 8 consecutive elements of a row (16-byte loads of y and gate in bf16),
// 32-bit index arithmetic.
#include "sk_common.cuh"

namespace sk {
namespace dit {

// 1 / (1 + expf(-g)) with the reciprocal correctly rounded (__frcp_rn gives the bits of the IEEE
// division 1.0f / x that the reference compiles to, in fewer instructions).
__device__ __forceinline__ float sigmoid_ref(float g) { return __frcp_rn(1.0f + expf(-g)); }

// fp32 -> e4m3 (1 sign, 4 exponent, 3 mantissa bits, bias 7), round to nearest even, magnitudes
// past the largest finite value (448) clamp to ±448, NaN -> 0x7f: the hardware conversion with
// .satfinite, plus the NaN rule of the reference encoder (engine/fused.py:60-72).
__device__ __forceinline__ uint32_t e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  uint32_t v = r;
  if (lo != lo) v = (v & 0xff00u) | 0x7fu;
  if (hi != hi) v = (v & 0x00ffu) | 0x7f00u;
  return v;
}

template <typename T>
struct Vec8;
template <>
struct Vec8<__nv_bfloat16> {
  static __device__ __forceinline__ void ld(const __nv_bfloat16* p, float* x) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      x[2 * i] = __uint_as_float(w[i] << 16);
      x[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
  static __device__ __forceinline__ void st(__nv_bfloat16* p, const float* x) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __nv_bfloat162 b2 = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
      w[i] = *reinterpret_cast<const uint32_t*>(&b2);
    }
    *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
  }
};
template <>
struct Vec8<float> {
  static __device__ __forceinline__ void ld(const float* p, float* x) {
    const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
    x[0] = a.x, x[1] = a.y, x[2] = a.z, x[3] = a.w, x[4] = b.x, x[5] = b.y, x[6] = b.z, x[7] = b.w;
  }
  static __device__ __forceinline__ void st(float* p, const float* x) {
    *reinterpret_cast<float4*>(p) = make_float4(x[0], x[1], x[2], x[3]);
    *reinterpret_cast<float4*>(p + 4) = make_float4(x[4], x[5], x[6], x[7]);
  }
};

template <typename T, bool E4M3>
// y and out may be the same buffer (the gate applied in place): no __restrict__ on them.
__global__ void __launch_bounds__(256) gate_kernel(const T* y, const T* __restrict__ o4, void* out, int n8, int D8,
                                                   float out_scale) {
  asm volatile("griddepcontrol.wait;" ::: "memory");  // y may come from the kernel just before
  asm volatile("griddepcontrol.launch_dependents;");
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n8) return;
  const int row = i / D8;  // 32-bit index arithmetic (sizes checked by the host)
  const int c = (i - row * D8) * 8;
  const int D = D8 * 8;
  float yv[8], gv[8];
  Vec8<T>::ld(y + (size_t)row * D + c, yv);
  Vec8<T>::ld(o4 + (size_t)row * 4 * D + 3 * D + c, gv);
#pragma unroll
  for (int e = 0; e < 8; ++e) yv[e] = yv[e] * sigmoid_ref(gv[e]);
  if constexpr (E4M3) {
    uint32_t w0 = e4m3x2(yv[0] * out_scale, yv[1] * out_scale) | (e4m3x2(yv[2] * out_scale, yv[3] * out_scale) << 16);
    uint32_t w1 = e4m3x2(yv[4] * out_scale, yv[5] * out_scale) | (e4m3x2(yv[6] * out_scale, yv[7] * out_scale) << 16);
    *reinterpret_cast<uint2*>(reinterpret_cast<uint8_t*>(out) + (size_t)row * D + c) = make_uint2(w0, w1);
  } else {
    Vec8<T>::st(reinterpret_cast<T*>(out) + (size_t)row * D + c, yv);
  }
}

}  // namespace dit
}  // namespace sk

extern "C" int sk_dit_gate(const void* y, const void* o4, void* out, long long rows, int D, int dtype, int out_dtype,
                           float out_scale, void* stream) {
  using namespace sk::dit;
  if (rows < 0 || D <= 0 || D % 8) return SK_ERR_INVALID_ARG;
  if (dtype != SK_BF16 && dtype != SK_F32) return SK_ERR_UNSUPPORTED;
  if (out_dtype != dtype && out_dtype != SK_E4M3) return SK_ERR_UNSUPPORTED;
  if (rows == 0) return SK_OK;  // nothing to do (empty tensors may carry null pointers)
  if (!y || !o4 || !out) return SK_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(o4)) & 15) return SK_ERR_INVALID_ARG;
  if (reinterpret_cast<uintptr_t>(out) & (out_dtype == SK_E4M3 ? 7 : 15)) return SK_ERR_INVALID_ARG;
  const int rc = sk_check_device();
  if (rc != SK_OK) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int D8 = D / 8;
  const long long n8 = rows * D8;
  if (n8 + 255 > 0x7fffffffLL || rows * 4 * (long long)D > 0x7fffffffLL) return SK_ERR_INVALID_ARG;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((n8 + 255) / 256));
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e;
  if (dtype == SK_BF16) {
    const auto* yy = reinterpret_cast<const __nv_bfloat16*>(y);
    const auto* oo = reinterpret_cast<const __nv_bfloat16*>(o4);
    e = out_dtype == SK_E4M3
            ? cudaLaunchKernelEx(&cfg, gate_kernel<__nv_bfloat16, true>, yy, oo, out, (int)n8, D8, out_scale)
            : cudaLaunchKernelEx(&cfg, gate_kernel<__nv_bfloat16, false>, yy, oo, out, (int)n8, D8, out_scale);
  } else {
    const auto* yy = reinterpret_cast<const float*>(y);
    const auto* oo = reinterpret_cast<const float*>(o4);
    e = out_dtype == SK_E4M3 ? cudaLaunchKernelEx(&cfg, gate_kernel<float, true>, yy, oo, out, (int)n8, D8, out_scale)
                             : cudaLaunchKernelEx(&cfg, gate_kernel<float, false>, yy, oo, out, (int)n8, D8, out_scale);
  }
  if (e != cudaSuccess) return SK_ERR_CUDA;
  return cudaPeekAtLastError() == cudaSuccess ? SK_OK : SK_ERR_CUDA;
}
