// DiT projection GEMM, bf16 mode, on the sm_100a tensor cores (tcgen05 + TMEM + TMA):
//   y (M, N) = x (M, K) · w (N, K)ᵀ
// F.linear without bias — the `mm` of engine/fused.py:262-264, called for w_qkvg, w_o, w_13 and w_2
// at engine/fused.py:293-310 (x = the rows of one step's latent batch, w = the layer's weight as
// nn.Linear stores it). Both operands are K-major, the layout the tensor core reads directly.
//
// One CTA computes a 128 x BN tile of y (BN = 256, 128 or 64, chosen per call), 128 threads:
//   warp 0 (one lane)  TMA producer: per 64-wide k step one x box [128 rows][64] and one w box
//                      [BN rows][64] (128-byte swizzled) into a ring of kStages slots.
//   warp 1 (one lane)  MMA issuer: four tcgen05.mma (M 128, N BN, K 16) per k step into one fp32
//                      TMEM accumulator of BN columns; each slot is released by tcgen05.commit.
//   warps 0-3          epilogue: thread r reads TMEM lane r (its row), rounds once to bf16, stages the
//                      tile 128B-swizzled over the (then idle) ring, and one thread writes it with TMA
//                      tensor stores; rows and columns past M and N are clipped by the tensor map, and
//                      k past K reads zeros.
// FP8 = true: the engine's FP8 projections (engine/fp8.py: torch._scaled_mm on e4m3 activations and
// e4m3 weights, each with a per-tensor inverse scale, bf16 out): kind::f8f6f4 MMAs (K 32) on 128-wide
// k steps of bytes, and the epilogue multiplies the fp32 sum by inv_x · inv_w before the bf16 rounding.
// Every wait gives up after 2 s (error word, then the CTA unwinds). No TMA multicast.
#include "sk_common.cuh"

namespace sk {
namespace lin {

constexpr int kBM = 128;  // tile rows; one k step = one 128-byte swizzle row (64 bf16 or 128 e4m3)
constexpr int kStages = 4;  // deeper rings for the narrow tiles measured slower (one CTA per SM instead of two)
constexpr int kThreads = 128;

template <int BN>
struct Ly {
  static constexpr int A_BYTES = kBM * 128;                 // 16 KB
  static constexpr int B_BYTES = BN * 128;                  // 32, 16 or 8 KB
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int OFF_BAR = kStages * STAGE_BYTES;     // full[kStages], empty[kStages], mma_done
  static constexpr int NBAR = 2 * kStages + 1;
  static constexpr int OFF_TMEM = OFF_BAR + NBAR * 8;
  static constexpr int SMEM = OFF_TMEM + 16;
  static_assert(BN / 64 * kBM * 128 <= OFF_BAR, "the output staging must fit over the ring");
  static_assert(SMEM <= 232448, "shared memory over the 227 KB per-CTA limit");
};

__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int x, int y, int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
               : "memory");
}

template <int BN, bool FP8>
__global__ void __launch_bounds__(kThreads, 1)
    linear_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                  const __grid_constant__ CUtensorMap tmY, int N, int K, const float* inv_x, const float* inv_w,
                  int* err) {
  constexpr int kBK = FP8 ? 128 : 64;  // elements per k step
  using L = Ly<BN>;
  constexpr int A_BYTES = L::A_BYTES, STAGE_BYTES = L::STAGE_BYTES, OFF_BAR = L::OFF_BAR;
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sbase = smem_u32(smem);
  if (sbase & 1023u) {  // uniform for the CTA, before any barrier: report and leave
    if (threadIdx.x == 0) set_dev_error(err, SK_DEVERR_TIMEOUT);
    return;
  }
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* empty = full + kStages;
  uint64_t* mma_done = empty + kStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_TMEM);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BN, m0 = blockIdx.y * kBM;
  const int nk = (K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(mma_done, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmY);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // x may come from the kernel launched before this one
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;");
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---------------------------------------------------------------- TMA producer
    int issued = 0;
    for (int kc = 0; kc < nk; ++kc) {
      const int s = kc % kStages;
      if (kc >= kStages && !mbar_wait(&empty[s], ((kc / kStages) - 1) & 1, err)) break;
      uint8_t* a = smem + s * STAGE_BYTES;
      mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
      tma_load_3d(a, &tmX, &full[s], kc * kBK, m0, 0);
      tma_load_3d(a + A_BYTES, &tmW, &full[s], kc * kBK, n0, 0);
      issued = kc + 1;
    }
    // keep shared memory alive until every copy issued has landed (already true on the normal path)
    for (int kc = (issued > kStages ? issued - kStages : 0); kc < issued; ++kc)
      mbar_wait(&full[kc % kStages], (kc / kStages) & 1, err);
  } else if (warp == 1 && lane == 0) {
    // ---------------------------------------------------------------- MMA issuer
    constexpr uint32_t idesc = FP8 ? idesc_e4m3_f32(kBM, BN) : idesc_bf16_f32(kBM, BN, 0, 0);
    for (int kc = 0; kc < nk; ++kc) {
      const int s = kc % kStages;
      if (!mbar_wait(&full[s], (kc / kStages) & 1, err)) break;
      tc_fence_after();
      const uint32_t a = sbase + s * STAGE_BYTES, bw = a + A_BYTES;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {  // 32 bytes of K per instruction: 16 bf16 or 32 e4m3
        const uint64_t da = smem_desc_sw128(a + kk * 32, 16, 1024), db = smem_desc_sw128(bw + kk * 32, 16, 1024);
        if constexpr (FP8)
          tc_mma_ss_f8(tmem, da, db, idesc, (kc > 0 || kk > 0) ? 1u : 0u);
        else
          tc_mma_ss(tmem, da, db, idesc, (kc > 0 || kk > 0) ? 1u : 0u);
      }
      tc_commit(&empty[s]);  // the slot is free once these MMAs have read it
    }
    tc_commit(mma_done);  // every MMA issued has completed
  }
  __syncwarp();

  // ------------------------------------------------------------------ epilogue (warps 0-3)
  bool ok = mbar_wait(mma_done, 0, err);
  ok = __all_sync(0xffffffffu, ok);
  const int row = threadIdx.x;  // TMEM lane == row of the tile
  const float oscale = FP8 ? __ldg(inv_x) * __ldg(inv_w) : 1.f;  // the two inverse scales, set before capture
  if (ok) {
    tc_fence_after();
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      float v[32];
      tmem_ld32(tmem + lane_off + c * 32, v);
      tmem_wait_ld();
      // 32 columns = four 16-byte units of the 64-column chunk c / 2
      uint8_t* chunk = smem + (c >> 1) * (kBM * 128) + row * 128;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        uint32_t pk[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float v0 = FP8 ? v[8 * u + 2 * e] * oscale : v[8 * u + 2 * e];
          const float v1 = FP8 ? v[8 * u + 2 * e + 1] * oscale : v[8 * u + 2 * e + 1];
          const __nv_bfloat162 b2 = __floats2bfloat162_rn(v0, v1);
          pk[e] = *reinterpret_cast<const uint32_t*>(&b2);
        }
        const int unit = (c & 1) * 4 + u;
        if (SK_INB((c >> 1) * (kBM * 128) + row * 128 + ((unit ^ (row & 7)) << 4) + 16 <= OFF_BAR, err))
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(smem_u32(chunk + ((unit ^ (row & 7)) << 4))),
                       "r"(pk[0]), "r"(pk[1]), "r"(pk[2]), "r"(pk[3])
                       : "memory");
      }
    }
    fence_proxy_async_smem();
  }
  __syncthreads();
  if (ok && threadIdx.x == 0) {
#pragma unroll
    for (int c = 0; c < BN / 64; ++c)  // column chunks that start inside y (the map clips the rest)
      if (n0 + c * 64 < N) tma_store_3d(&tmY, smem + c * (kBM * 128), n0 + c * 64, m0, 0);
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, BN);
  }
}


template <int BN, bool FP8>
static int launch(const void* x, const void* w, void* y, int M, int N, int K, const float* inv_x, const float* inv_w,
                  int* err, int dev, void* stream) {
  using L = Ly<BN>;
  constexpr int kBK = FP8 ? 128 : 64;
  constexpr cuuint64_t es = FP8 ? 1 : 2;  // operand bytes per element
  const CUtensorMapDataType dt = FP8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap mx, mw, my;
  {
    cuuint64_t dims[3] = {(cuuint64_t)K, (cuuint64_t)M, 1};
    cuuint64_t str[2] = {(cuuint64_t)K * es, (cuuint64_t)M * K * es};
    cuuint32_t box[3] = {kBK, kBM, 1};
    if (!sk_make_map_sw128(&mx, dt, x, 3, dims, str, box)) return SK_ERR_CUDA;
  }
  {
    cuuint64_t dims[3] = {(cuuint64_t)K, (cuuint64_t)N, 1};
    cuuint64_t str[2] = {(cuuint64_t)K * es, (cuuint64_t)N * K * es};
    cuuint32_t box[3] = {kBK, BN, 1};
    if (!sk_make_map_sw128(&mw, dt, w, 3, dims, str, box)) return SK_ERR_CUDA;
  }
  {
    cuuint64_t dims[3] = {(cuuint64_t)N, (cuuint64_t)M, 1};
    cuuint64_t str[2] = {(cuuint64_t)N * 2, (cuuint64_t)M * N * 2};
    cuuint32_t box[3] = {64, kBM, 1};
    if (!sk_make_map_bf16(&my, y, 3, dims, str, box)) return SK_ERR_CUDA;
  }
  static bool attr_done[64] = {};
  if (!attr_done[dev]) {
    if (cudaFuncSetAttribute(linear_kernel<BN, FP8>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM) !=
        cudaSuccess)
      return SK_ERR_CUDA;
    attr_done[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((N + BN - 1) / BN), (unsigned)((M + kBM - 1) / kBM));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = L::SMEM;
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, linear_kernel<BN, FP8>, mx, mw, my, N, K, inv_x, inv_w, err) != cudaSuccess)
    return SK_ERR_CUDA;
  return cudaPeekAtLastError() == cudaSuccess ? SK_OK : SK_ERR_CUDA;
}

}  // namespace lin
}  // namespace sk

namespace sk {
namespace lin {
// N tile: the fewest waves of CTAs weighted by a tile's relative cost (a 128 x 128 tile takes ~0.62
// and a 128 x 64 tile ~0.45 of a 128 x 256 one, the operand bytes per FLOP growing as BN shrinks)
static int pick_tile(int M, int N, int dev) {
  static int sm_count[64] = {};
  if (sm_count[dev] == 0 && cudaDeviceGetAttribute(&sm_count[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return 0;
  const long long mt = (M + kBM - 1) / kBM;
  int bn = 256;
  double best = 1e30;
  for (int cand : {256, 128, 64}) {
    const long long tiles = mt * ((N + cand - 1) / cand);
    const double waves = (double)((tiles + sm_count[dev] - 1) / sm_count[dev]);
    const double cost = waves * (cand == 256 ? 1.0 : cand == 128 ? 0.62 : 0.45);
    if (cost < best - 1e-9) {
      best = cost;
      bn = cand;
    }
  }
  return bn;
}

template <bool FP8>
static int run(const void* x, const void* w, void* y, const float* inv_x, const float* inv_w, int M, int N, int K,
               int tile_n, void* stream) {
  if (tile_n != 0 && tile_n != 64 && tile_n != 128 && tile_n != 256) return SK_ERR_INVALID_ARG;
  if (!x || !w || !y) return SK_ERR_INVALID_ARG;
  if (M <= 0 || N <= 0 || K <= 0) return SK_ERR_INVALID_ARG;
  if (FP8 && (!inv_x || !inv_w)) return SK_ERR_INVALID_ARG;
  // tensor maps: 16-byte aligned bases and row strides
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(y)) & 15)
    return SK_ERR_INVALID_ARG;
  if (K % (FP8 ? 16 : 8) || N % 8) return SK_ERR_INVALID_ARG;
  const int rc = sk_check_device();
  if (rc != SK_OK) return rc;
  int* err = sk_error_word_ptr();
  if (!err) return SK_ERR_CUDA;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return SK_ERR_CUDA;
  const int bn = tile_n ? tile_n : pick_tile(M, N, dev);
  switch (bn) {
    case 256: return launch<256, FP8>(x, w, y, M, N, K, inv_x, inv_w, err, dev, stream);
    case 128: return launch<128, FP8>(x, w, y, M, N, K, inv_x, inv_w, err, dev, stream);
    case 64: return launch<64, FP8>(x, w, y, M, N, K, inv_x, inv_w, err, dev, stream);
    default: return SK_ERR_CUDA;
  }
}
}  // namespace lin
}  // namespace sk

extern "C" int sk_dit_linear_ex(const void* x, const void* w, void* y, int M, int N, int K, int dtype, int tile_n,
                                void* stream) {
  if (dtype != SK_BF16) return SK_ERR_UNSUPPORTED;  // the fp32 mode keeps the library GEMM
  return sk::lin::run<false>(x, w, y, nullptr, nullptr, M, N, K, tile_n, stream);
}

extern "C" int sk_dit_linear_fp8(const void* x8, const void* w8, void* y, const float* inv_scale_x,
                                 const float* inv_scale_w, int M, int N, int K, int tile_n, void* stream) {
  return sk::lin::run<true>(x8, w8, y, inv_scale_x, inv_scale_w, M, N, K, tile_n, stream);
}

extern "C" int sk_dit_linear(const void* x, const void* w, void* y, int M, int N, int K, int dtype, void* stream) {
  return sk_dit_linear_ex(x, w, y, M, N, K, dtype, 0, stream);
}
