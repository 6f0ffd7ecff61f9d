// DiT Q/K/V producer: per-head RMSNorm of q and k (sum of squares in double), × qk weight, RoPE on
// heads h < H/2 with interleaved pairs (2i, 2i+1); v copied. Same arithmetic as the reference's
// `qkv` kernel (engine/fused.py:117-180, the p < L branch), written for the split key layout: the
// conditioning K/V are not copied per batch row, the attention kernel reads them in place.
//
// HBM-bound: one warp per latent row, coalesced 16-byte chunks in and out; all index arithmetic is
// 32-bit.
#include "dit_qk_math.cuh"
#include "sk_common.cuh"

namespace sk {
namespace dit {

template <typename T>
struct Vec16;  // one 16-byte vector of T as floats
template <>
struct Vec16<__nv_bfloat16> {
  static constexpr int N = 8;
  static __device__ __forceinline__ void unpack(const uint4& u, float* x) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      x[2 * i] = __uint_as_float(w[i] << 16);
      x[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
  static __device__ __forceinline__ uint4 pack(const float* x) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __nv_bfloat162 b2 = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
      w[i] = *reinterpret_cast<const uint32_t*>(&b2);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
  }
};
template <>
struct Vec16<float> {
  static constexpr int N = 4;
  static __device__ __forceinline__ void unpack(const uint4& u, float* x) {
    x[0] = __uint_as_float(u.x), x[1] = __uint_as_float(u.y), x[2] = __uint_as_float(u.z), x[3] = __uint_as_float(u.w);
  }
  static __device__ __forceinline__ uint4 pack(const float* x) {
    return make_uint4(__float_as_uint(x[0]), __float_as_uint(x[1]), __float_as_uint(x[2]), __float_as_uint(x[3]));
  }
};

constexpr int kPrologueThreads = 256;  // 8 warps, one latent row each
constexpr int kPrologueMaxSteps = 16;  // 32-chunk steps whose loads are in flight together (8 KB per warp)

// One warp per latent row (b, p). The row's q and k quarters are read in 16-byte chunks, 32
// consecutive chunks per step, the loads of up to 16 steps issued before any is used (one DRAM round
// trip per row at the configs' sizes); the qk weights (per block) and the row's RoPE table row (per warp) wait in shared memory. The
// NV lanes that hold one head's chunks combine their sums of squares with xor shuffles, each lane
// scales and rotates its own chunk (RoPE pairs never straddle a chunk) and writes it to the head's
// (B, H, L, hd) row, NV lanes covering that row's contiguous bytes. v is copied chunk by chunk the
// same way (skipped when v == nullptr).
//
// The sum of squares is accumulated in double like the reference (engine/fused.py:143). The reference
// adds eight strided partial sums; here the per-lane partials meet in a shuffle tree. For bf16 inputs
// every square has at most 16 significant bits, so the double sum is exact, and therefore the same in
// any order, unless the squares of one head span more than ~37 binary orders of magnitude.
template <typename T, int HD>
__global__ void __launch_bounds__(kPrologueThreads) qkv_prologue_kernel(const T* __restrict__ o4,
                                                                         const float* __restrict__ qk_w,
                                                                         const float* __restrict__ freqs,
                                                                         T* __restrict__ q, T* __restrict__ k,
                                                                         T* __restrict__ v, int rows, int L, int H,
                                                                         float inv_hd, float eps) {
  using V = Vec16<T>;
  constexpr int NV = HD / V::N;  // 16-byte chunks per head row: 8, 16 or 32 lanes per head
  static_assert(NV >= 2 && NV <= 32 && (NV & (NV - 1)) == 0, "a head must cover a power-of-two lane group");
  extern __shared__ __align__(16) float stage[];  // [2·D] qk weights, then [8 warps][HD] RoPE rows
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int D = H * HD;
  // o4 may be written by the kernel launched before this one (programmatic dependent launch); the
  // weights and the table are constants of the model
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;");
  const int row = blockIdx.x * (kPrologueThreads / 32) + warp;
  const int b = row / L, p = row - b * L;
  const int qk_chunks = 2 * H * NV;
  const int steps = (qk_chunks + 31) / 32;
  const T* src = o4 + (size_t)row * 4 * D;
  uint4 raw[kPrologueMaxSteps];
  // one batch of up to kPrologueMaxSteps steps: all loads issued before any is used
  auto load_batch = [&](int t0) {
#pragma unroll
    for (int t = 0; t < kPrologueMaxSteps; ++t) {
      const int j = (t0 + t) * 32 + lane;
      if (t0 + t < steps && j < qk_chunks) {
        const int slot = j / NV, c = j % NV;
        raw[t] = __ldg(reinterpret_cast<const uint4*>(src + (slot >= H ? D : 0) + (slot % H) * HD) + c);
      }
    }
  };
  if (row < rows) load_batch(0);
  float* w_s = stage;
  float* f_s = stage + 2 * D + warp * HD;
  for (int t = threadIdx.x; t < 2 * D / 4; t += kPrologueThreads)
    reinterpret_cast<float4*>(w_s)[t] = __ldg(reinterpret_cast<const float4*>(qk_w) + t);
  if (row < rows)
    for (int t = lane; t < HD / 4; t += 32)
      reinterpret_cast<float4*>(f_s)[t] = __ldg(reinterpret_cast<const float4*>(freqs + (size_t)p * HD) + t);
  __syncthreads();
  if (row >= rows) return;  // warp-uniform
  for (int t0 = 0; t0 < steps; t0 += kPrologueMaxSteps) {
    if (t0 > 0) load_batch(t0);
#pragma unroll
    for (int t = 0; t < kPrologueMaxSteps; ++t) {
      if (t0 + t >= steps) break;
      const int j = (t0 + t) * 32 + lane;
      const bool act = j < qk_chunks;  // whole heads: the group of a head is all active or all idle
      const int slot = j / NV, c = j % NV;
      const int which = slot >= H ? 1 : 0, h = slot - which * H;
      float x[V::N];
      V::unpack(act ? raw[t] : make_uint4(0, 0, 0, 0), x);
      double ss = 0.0;
#pragma unroll
      for (int e = 0; e < V::N; ++e) ss += (double)x[e] * x[e];
#pragma unroll
      for (int o = NV / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (!act) continue;
      const float r = qk_inv_rms(ss, inv_hd, eps);  // engine/fused.py:148
      qk_scale_rotate<V::N>(x, r, w_s + which * D + h * HD + c * V::N,
                            h < H / 2 ? f_s + c * V::N : nullptr);  // engine/fused.py:150-171
      T* dst = (which == 0 ? q : k) + ((size_t)(b * H + h) * L + p) * HD + c * V::N;
      *reinterpret_cast<uint4*>(dst) = V::pack(x);
    }
  }
  if (v != nullptr) {
    const int v_chunks = H * NV;
#pragma unroll 4
    for (int j = lane; j < v_chunks; j += 32) {
      const int h = j / NV, c = j % NV;
      const uint4 val = __ldg(reinterpret_cast<const uint4*>(src + 2 * D + h * HD) + c);
      *reinterpret_cast<uint4*>(v + ((size_t)(b * H + h) * L + p) * HD + c * V::N) = val;
    }
  }
}

}  // namespace dit
}  // namespace sk

// Launch shared by the C ABI below and the fused attention block (which passes v == nullptr: its
// attention kernel reads v straight from o4).
int sk_launch_qkv_prologue(const void* o4, const float* qk_w, const float* freqs, void* q, void* k, void* v, int B,
                           int L, int H, int hd, float eps, int dtype, cudaStream_t st) {
  using namespace sk::dit;
  const long long rows = (long long)B * L;
  if (rows * 4 * H * hd > 0x7fffffffLL) return SK_ERR_INVALID_ARG;
  constexpr int kRowsPerBlock = kPrologueThreads / 32;
  const size_t smem = (size_t)(2 * H * hd + kRowsPerBlock * hd) * sizeof(float);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((rows + kRowsPerBlock - 1) / kRowsPerBlock));
  cfg.blockDim = dim3(kPrologueThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const float inv = 1.f / hd;
  cudaError_t e = cudaSuccess;
#define SK_PROLOGUE(T, HDV)                                                                                        \
  do {                                                                                                             \
    if (smem > 48 * 1024)                                                                                          \
      e = cudaFuncSetAttribute(qkv_prologue_kernel<T, HDV>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
    if (e == cudaSuccess)                                                                                          \
      e = cudaLaunchKernelEx(&cfg, qkv_prologue_kernel<T, HDV>, reinterpret_cast<const T*>(o4), qk_w, freqs,        \
                             reinterpret_cast<T*>(q), reinterpret_cast<T*>(k), reinterpret_cast<T*>(v), (int)rows, L, \
                             H, inv, eps);                                                                          \
  } while (0)
  if (dtype == SK_BF16) {
    if (hd == 64) SK_PROLOGUE(__nv_bfloat16, 64);
    else SK_PROLOGUE(__nv_bfloat16, 128);
  } else {
    if (hd == 64) SK_PROLOGUE(float, 64);
    else SK_PROLOGUE(float, 128);
  }
#undef SK_PROLOGUE
  if (e != cudaSuccess) return SK_ERR_CUDA;
  return cudaPeekAtLastError() == cudaSuccess ? SK_OK : SK_ERR_CUDA;
}

extern "C" int sk_dit_qkv_prologue(const void* o4, const float* qk_w, const float* freqs, void* q, void* k_lat,
                                   void* v_lat, int B, int L, int H, int hd, float eps, int dtype, void* stream) {
  if (!o4 || !qk_w || !freqs || !q || !k_lat || !v_lat) return SK_ERR_INVALID_ARG;
  if (B <= 0 || L <= 0 || H <= 0 || H % 2) return SK_ERR_INVALID_ARG;
  if (hd != 64 && hd != 128) return SK_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(o4) | reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k_lat) |
       reinterpret_cast<uintptr_t>(v_lat) | reinterpret_cast<uintptr_t>(qk_w) | reinterpret_cast<uintptr_t>(freqs)) &
      15)
    return SK_ERR_INVALID_ARG;
  if (dtype != SK_BF16 && dtype != SK_F32) return SK_ERR_UNSUPPORTED;
  int rc = sk_check_device();
  if (rc != SK_OK) return rc;
  return sk_launch_qkv_prologue(o4, qk_w, freqs, q, k_lat, v_lat, B, L, H, hd, eps, dtype,
                                reinterpret_cast<cudaStream_t>(stream));
}
