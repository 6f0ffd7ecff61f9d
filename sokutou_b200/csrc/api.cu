// Library-wide host entry points: version, device check, and the per-device error word.
#include <mutex>

#include "sk_common.cuh"

namespace sk {
// The error word every kernel of this library reports into (one copy per device the library is
// loaded on).
__device__ int g_dev_error = 0;
}  // namespace sk

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_mu;
int* g_err_ptr[kMaxDevices] = {};
int g_dev_ok[kMaxDevices] = {};  // 0 unknown, 1 sm_100, -1 other
}  // namespace

int* sk_error_word_ptr() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_err_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, sk::g_dev_error) != cudaSuccess) return nullptr;
    g_err_ptr[dev] = reinterpret_cast<int*>(p);
  }
  return g_err_ptr[dev];
}

int sk_check_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return SK_ERR_CUDA;
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_dev_ok[dev] == 0) {
    int major = 0, minor = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess)
      return SK_ERR_CUDA;
    g_dev_ok[dev] = (major == 10 && minor == 0) ? 1 : -1;
  }
  return g_dev_ok[dev] == 1 ? SK_OK : SK_ERR_DEVICE;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (the library links only the runtime).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

bool sk_make_map_sw128(CUtensorMap* m, CUtensorMapDataType dt, const void* base, int rank, const cuuint64_t* dims,
                       const cuuint64_t* strides_b, const cuuint32_t* box) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint32_t es[5] = {1, 1, 1, 1, 1};
  return fn(m, dt, rank, const_cast<void*>(base), dims, strides_b, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool sk_make_map_bf16(CUtensorMap* m, const void* base, int rank, const cuuint64_t* dims, const cuuint64_t* strides_b,
                      const cuuint32_t* box) {
  return sk_make_map_sw128(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, base, rank, dims, strides_b, box);
}

extern "C" int sk_version(void) { return 100; }

extern "C" int sk_device_error(int* code, int reset) {
  if (!code) return SK_ERR_INVALID_ARG;
  int* p = sk_error_word_ptr();
  if (!p) return SK_ERR_CUDA;
  if (cudaDeviceSynchronize() != cudaSuccess) return SK_ERR_CUDA;
  if (cudaMemcpy(code, p, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return SK_ERR_CUDA;
  if (reset && cudaMemset(p, 0, sizeof(int)) != cudaSuccess) return SK_ERR_CUDA;
  return SK_OK;
}
