// Qwen3-TTS talker decode attention for B200: split-KV flash decoding with the QK-RMSNorm, RoPE and
// KV-cache append of the reference kernel fused in.
//
// Replaces the NVRTC kernel `attn` of the reference engine (qwen3/kernels.py:338-414), which runs
// one CTA per KV head (8 CTAs on a 148-SM part) and scans all T keys with scalar loads. Here:
//   grid  = (ceil(max_len / kChunk) splits, nkv)  — fixed at capture time; splits past T exit;
//   block = 128 threads; each CTA owns kChunk consecutive keys of one KV head;
//   its K and V chunk arrive in shared memory by two untiled bulk copies (TMA engine, full
//   128-byte lines, no register staging), while the CTA computes the q prologue;
//   scores by lane-split dot products finished with one butterfly reduce-scatter per warp;
//   chunk-local softmax (expf like the reference) and PV; the last CTA of a KV head to finish
//   merges the per-chunk (max, sum, o) partials — an atomic counter, no spin-wait.
// The position comes from device memory (pos_ptr[0] + pos_add) so one CUDA graph serves all steps.
#include <mutex>

#include "sk_common.cuh"

namespace sk {
namespace decode {

constexpr int kHD = 128;     // head dim (reference: HD 128, qwen3/kernels.py:38)
constexpr int kG = 2;        // q heads per kv head (reference: nq == 2*nkv, qwen3/kernels.py:457)
constexpr int kChunk = 64;   // keys per CTA
constexpr int kThreads = 128;
constexpr int kMaxSplits = 256;  // max_len <= 16384

template <typename CT>
struct Cache;
template <>
struct Cache<__nv_bfloat16> {
  static __device__ __forceinline__ float ld(const __nv_bfloat16* p) { return __bfloat162float(*p); }
  static __device__ __forceinline__ __nv_bfloat16 st(float f) { return __float2bfloat16_rn(f); }
  static __device__ __forceinline__ float rnd(float f) { return __bfloat162float(__float2bfloat16_rn(f)); }
};
template <>
struct Cache<float> {
  static __device__ __forceinline__ float ld(const float* p) { return *p; }
  static __device__ __forceinline__ float st(float f) { return f; }
  static __device__ __forceinline__ float rnd(float f) { return f; }
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Workspace layout (floats unless noted), per kv head h and split s:
//   o   [nkv][nsplit][kG][kHD]
//   ml  [nkv][nsplit][kG][2]      (chunk max, chunk sum)
//   cnt [nkv] int                 (arrivals; reset to 0 by the merging CTA)
struct Workspace {
  float* o;
  float* ml;
  int* cnt;
};
__host__ __device__ inline size_t ws_bytes(int max_len, int nkv) {
  const size_t ns = (size_t)((max_len + kChunk - 1) / kChunk);
  return (size_t)nkv * ns * kG * kHD * 4 + (size_t)nkv * ns * kG * 2 * 4 + (size_t)nkv * 4 + 256;
}
__host__ __device__ inline Workspace ws_carve(void* base, int max_len, int nkv) {
  const size_t ns = (size_t)((max_len + kChunk - 1) / kChunk);
  char* p = reinterpret_cast<char*>(base);
  Workspace w;
  w.o = reinterpret_cast<float*>(p);
  p += (size_t)nkv * ns * kG * kHD * 4;
  w.ml = reinterpret_cast<float*>(p);
  p += (size_t)nkv * ns * kG * 2 * 4;
  w.cnt = reinterpret_cast<int*>(p);
  return w;
}

template <typename CT>
__global__ void __launch_bounds__(kThreads) decode_attn_kernel(
    const float* __restrict__ qkv, const float* __restrict__ qn, const float* __restrict__ kn, float eps,
    const float* __restrict__ rope, CT* __restrict__ Kc, CT* __restrict__ Vc, const long long* __restrict__ pos_ptr,
    int pos_add, int max_len, int nq, int nkv, float* __restrict__ out, void* workspace, int* err) {
  extern __shared__ __align__(128) unsigned char dsmem[];
  CT* Ks = reinterpret_cast<CT*>(dsmem);                // [kChunk][kHD]
  CT* Vs = Ks + kChunk * kHD;                           // [kChunk][kHD]
  __shared__ __align__(16) float q_s[kG][kHD];          // normed, roped, scaled q
  __shared__ __align__(16) float kn_s[kHD];             // new k (as the cache holds it)
  __shared__ __align__(16) float vn_s[kHD];             // new v (as the cache holds it)
  __shared__ __align__(16) float sc[kG][kChunk];        // scores, then probabilities
  __shared__ __align__(16) float o_half[kG][kHD];       // PV partial of the upper key half
  __shared__ float red[8][4];
  __shared__ float stat[kG][2];
  __shared__ int is_last;
  __shared__ float mg_s[kMaxSplits * kG];  // merge: chunk maxima, then chunk weights
  __shared__ float lg_s[kMaxSplits * kG];  // merge: chunk sums
  __shared__ __align__(8) uint64_t bar;

  const int kvh = blockIdx.y, split = blockIdx.x;
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  const int pos = (pos_ptr ? (int)pos_ptr[0] : 0) + pos_add;
  if (pos < 0 || pos >= max_len) {
    if (split == 0 && kvh == 0 && t == 0) set_dev_error(err, SK_DEVERR_POS_RANGE);
    return;
  }
  const int T = pos + 1;
  const int active = (T + kChunk - 1) / kChunk;
  if (split >= active) return;
  const int s0 = split * kChunk;
  const int n = min(kChunk, T - s0);                 // keys in this chunk (>= 1)
  const bool owner = (s0 + n == T);                  // this chunk holds the new position
  const int n_ld = owner ? n - 1 : n;                // keys read from the cache

  const size_t head_base = (size_t)kvh * max_len * kHD;
  if (t == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (t == 0 && n_ld > 0) {
    const uint32_t bytes = (uint32_t)(n_ld * kHD * sizeof(CT));
    mbar_arrive_expect_tx(&bar, 2 * bytes);
    bulk_load(Ks, Kc + head_base + (size_t)s0 * kHD, bytes, &bar);
    bulk_load(Vs, Vc + head_base + (size_t)s0 * kHD, bytes, &bar);
  }

  // ---- prologue (qwen3/kernels.py:351-380): thread t owns dimension d = t -------------------------
  const int d = t;
  const float c = rope[(size_t)pos * kHD + (d & 63)];
  const float s = rope[(size_t)pos * kHD + 64 + (d & 63)];
  float qv[kG];
#pragma unroll
  for (int g = 0; g < kG; ++g) qv[g] = qkv[(size_t)(kvh * kG + g) * kHD + d];
  float kv = 0.f, vv = 0.f;
  if (owner) {
    kv = qkv[(size_t)nq * kHD + (size_t)kvh * kHD + d];
    vv = qkv[(size_t)(nq + nkv) * kHD + (size_t)kvh * kHD + d];
  }
  {
    float ss[kG + 1];
#pragma unroll
    for (int g = 0; g < kG; ++g) ss[g] = warp_sum(qv[g] * qv[g]);
    ss[kG] = warp_sum(kv * kv);
    if (lane == 0) {
#pragma unroll
      for (int g = 0; g <= kG; ++g) red[w][g] = ss[g];
    }
    __syncthreads();
#pragma unroll
    for (int g = 0; g <= kG; ++g) ss[g] = red[0][g] + red[1][g] + red[2][g] + red[3][g];
#pragma unroll
    for (int g = 0; g < kG; ++g) q_s[g][d] = qv[g] * rsqrtf(ss[g] / kHD + eps) * qn[d];
    if (owner) kn_s[d] = kv * rsqrtf(ss[kG] / kHD + eps) * kn[d];
    __syncthreads();
    float qr[kG];
#pragma unroll
    for (int g = 0; g < kG; ++g) {
      const float rot = d < 64 ? -q_s[g][d + 64] : q_s[g][d - 64];
      qr[g] = (q_s[g][d] * c + rot * s) * 0.08838834764831845f;  // 1/sqrt(128), as qwen3/kernels.py:378
    }
    float knew = 0.f;
    if (owner) {
      const float rot = d < 64 ? -kn_s[d + 64] : kn_s[d - 64];
      knew = kn_s[d] * c + rot * s;
    }
    __syncthreads();
#pragma unroll
    for (int g = 0; g < kG; ++g) q_s[g][d] = qr[g];
    if (owner) {
      const CT kst = Cache<CT>::st(knew), vst = Cache<CT>::st(vv);
      Kc[head_base + (size_t)pos * kHD + d] = kst;          // append (qwen3/kernels.py:364,366)
      Vc[head_base + (size_t)pos * kHD + d] = vst;
      kn_s[d] = Cache<CT>::ld(&kst);                         // attended as read back from the cache
      vn_s[d] = Cache<CT>::ld(&vst);
    }
    __syncthreads();
  }

  bool ok = true;
  if (n_ld > 0) ok = mbar_wait(&bar, 0, err);
  if (!ok) {
    // The copy did not land in time (the error word now says so): keep the shared memory alive
    // until the copy ends, and still count this CTA's arrival so that the merge counter returns to
    // zero for the next call. This call's output is not valid.
    if (t == 0) {
      mbar_wait(&bar, 0, err);
      if (active > 1) {
        int* cnt = ws_carve(workspace, max_len, nkv).cnt;
        if (atomicAdd(&cnt[kvh], 1) == active - 1) cnt[kvh] = 0;
      }
    }
    return;
  }

  // ---- scores: warp w owns keys [16w, 16w+16); lane owns dims [4*lane, 4*lane+4) -----------------
  {
    float qa[kG][4];
#pragma unroll
    for (int g = 0; g < kG; ++g)
#pragma unroll
      for (int i = 0; i < 4; ++i) qa[g][i] = q_s[g][4 * lane + i];
    float part[kG * 16];
#pragma unroll
    for (int jj = 0; jj < 16; ++jj) {
      const int j = 16 * w + jj;
      float k4[4];
      if (j < n_ld) {
        const CT* kp = Ks + j * kHD + 4 * lane;
#pragma unroll
        for (int i = 0; i < 4; ++i) k4[i] = Cache<CT>::ld(kp + i);
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) k4[i] = kn_s[4 * lane + i];   // j == n_ld (owner) or unused
      }
#pragma unroll
      for (int g = 0; g < kG; ++g)
        part[g * 16 + jj] = qa[g][0] * k4[0] + qa[g][1] * k4[1] + qa[g][2] * k4[2] + qa[g][3] * k4[3];
    }
    // Butterfly reduce-scatter: afterwards lane l holds the warp-wide sum of part[l].
#pragma unroll
    for (int off = 16, m = 32; off >= 1; off >>= 1, m >>= 1) {
      const bool upper = (lane & off) != 0;
#pragma unroll
      for (int i = 0; i < m / 2; ++i) {
        const float send = upper ? part[i] : part[i + m / 2];
        const float keep = upper ? part[i + m / 2] : part[i];
        part[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
      }
    }
    const int g = lane >> 4, j = 16 * w + (lane & 15);
    sc[g][j] = (j < n) ? part[0] : -INFINITY;
  }
  __syncthreads();

  // ---- chunk softmax (qwen3/kernels.py:394-408): warp g handles head g ----------------------------
  if (w < kG) {
    const int g = w;
    float a = sc[g][lane], b = sc[g][lane + 32];
    const float m = warp_max(fmaxf(a, b));
    a = (lane < n) ? expf(a - m) : 0.f;
    b = (lane + 32 < n) ? expf(b - m) : 0.f;
    sc[g][lane] = a;
    sc[g][lane + 32] = b;
    const float l = warp_sum(a + b);
    if (lane == 0) {
      stat[g][0] = m;
      stat[g][1] = l;
    }
  }
  __syncthreads();

  // ---- PV: thread owns dims (2*(t%64), +1) over key half t/64 -------------------------------------
  float acc[kG][2] = {};
  {
    const int dp = 2 * (t & 63), kh = t >> 6;
    const int j0 = kh * 32, j1 = min(j0 + 32, n);
    for (int j = j0; j < j1; ++j) {
      float v0, v1;
      if (j < n_ld) {
        v0 = Cache<CT>::ld(Vs + j * kHD + dp);
        v1 = Cache<CT>::ld(Vs + j * kHD + dp + 1);
      } else {
        v0 = vn_s[dp];
        v1 = vn_s[dp + 1];
      }
#pragma unroll
      for (int g = 0; g < kG; ++g) {
        const float p = sc[g][j];
        acc[g][0] += p * v0;
        acc[g][1] += p * v1;
      }
    }
    if (kh == 1) {
#pragma unroll
      for (int g = 0; g < kG; ++g) {
        o_half[g][dp] = acc[g][0];
        o_half[g][dp + 1] = acc[g][1];
      }
    }
    __syncthreads();
    if (kh == 0) {
#pragma unroll
      for (int g = 0; g < kG; ++g) {
        acc[g][0] += o_half[g][dp];
        acc[g][1] += o_half[g][dp + 1];
      }
    }
  }

  const int dp = 2 * (t & 63);
  if (active == 1) {  // one chunk holds every key: finish here
    if (t < 64) {
#pragma unroll
      for (int g = 0; g < kG; ++g) {
        const float inv = 1.f / stat[g][1];
        float2 r = make_float2(acc[g][0] * inv, acc[g][1] * inv);
        *reinterpret_cast<float2*>(out + (size_t)(kvh * kG + g) * kHD + dp) = r;
      }
    }
    return;
  }

  // ---- publish the chunk partial, the last CTA of this kv head merges ---------------------------
  Workspace ws = ws_carve(workspace, max_len, nkv);
  const int nsplit = (max_len + kChunk - 1) / kChunk;
  const size_t slot = (size_t)kvh * nsplit + split;
  if (t < 64) {
#pragma unroll
    for (int g = 0; g < kG; ++g)
      *reinterpret_cast<float2*>(ws.o + (slot * kG + g) * kHD + dp) = make_float2(acc[g][0], acc[g][1]);
  }
  if (t < kG * 2) ws.ml[slot * kG * 2 + t] = stat[t >> 1][t & 1];
  __threadfence();
  __syncthreads();
  if (t == 0) is_last = (atomicAdd(&ws.cnt[kvh], 1) == active - 1);
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  // Merge. Every load below is issued independently of the others (no dependent chain through
  // L2): the per-chunk (max, sum) pairs are staged in shared memory by one thread each, then each
  // thread combines its dimension over the chunks, 8 chunks' partials in flight at a time.
  for (int i = t; i < active * kG; i += kThreads) {
    const size_t sl = (size_t)kvh * nsplit + i / kG;
    mg_s[i] = __ldcg(ws.ml + (sl * kG + (i % kG)) * 2);
    lg_s[i] = __ldcg(ws.ml + (sl * kG + (i % kG)) * 2 + 1);
  }
  __syncthreads();
  if (w < kG) {  // warp g: global max and denominator of head g, weights per chunk
    const int g = w;
    float M = -INFINITY;
    for (int sp = lane; sp < active; sp += 32) M = fmaxf(M, mg_s[sp * kG + g]);
    M = warp_max(M);
    float den = 0.f;
    for (int sp = lane; sp < active; sp += 32) {
      const float f = expf(mg_s[sp * kG + g] - M);
      mg_s[sp * kG + g] = f;  // now the chunk weight
      den += f * lg_s[sp * kG + g];
    }
    den = warp_sum(den);
    if (lane == 0) stat[g][1] = den;
  }
  __syncthreads();
  {
    float num[kG] = {};
    const float* ob = ws.o + (size_t)kvh * nsplit * kG * kHD + d;
    int sp = 0;
    for (; sp + 8 <= active; sp += 8) {
      float v[8][kG];
#pragma unroll
      for (int u = 0; u < 8; ++u)
#pragma unroll
        for (int g = 0; g < kG; ++g) v[u][g] = __ldcg(ob + ((size_t)(sp + u) * kG + g) * kHD);
#pragma unroll
      for (int u = 0; u < 8; ++u)
#pragma unroll
        for (int g = 0; g < kG; ++g) num[g] += mg_s[(sp + u) * kG + g] * v[u][g];
    }
    for (; sp < active; ++sp)
#pragma unroll
      for (int g = 0; g < kG; ++g) num[g] += mg_s[sp * kG + g] * __ldcg(ob + ((size_t)sp * kG + g) * kHD);
#pragma unroll
    for (int g = 0; g < kG; ++g) out[(size_t)(kvh * kG + g) * kHD + d] = num[g] / stat[g][1];
  }
  if (t == 0) ws.cnt[kvh] = 0;  // ready for the next call (and graph replay)
}

}  // namespace decode
}  // namespace sk

using namespace sk;

extern "C" size_t sk_decode_workspace_bytes(int max_len, int nq, int nkv, int hd, int cache_dtype) {
  (void)nq;
  (void)hd;
  (void)cache_dtype;
  if (max_len <= 0 || nkv <= 0) return 0;
  return decode::ws_bytes(max_len, nkv);
}

extern "C" int sk_decode_attention(const float* qkv, const float* qn, const float* kn, float eps, const float* rope,
                                   void* Kc, void* Vc, const long long* pos_ptr, int pos_add, int max_len, int nq,
                                   int nkv, int hd, float* out, void* workspace, size_t ws_bytes, int cache_dtype,
                                   void* stream) {
  if (!qkv || !qn || !kn || !rope || !Kc || !Vc || !out) return SK_ERR_INVALID_ARG;
  if (max_len <= 0 || nkv <= 0 || nq <= 0) return SK_ERR_INVALID_ARG;
  if (hd != decode::kHD || nq != decode::kG * nkv) return SK_ERR_UNSUPPORTED;
  if (cache_dtype != SK_BF16 && cache_dtype != SK_F32) return SK_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(Kc) | reinterpret_cast<uintptr_t>(Vc) | reinterpret_cast<uintptr_t>(out)) & 15)
    return SK_ERR_INVALID_ARG;
  const int nsplit = (max_len + decode::kChunk - 1) / decode::kChunk;
  if (nsplit > decode::kMaxSplits) return SK_ERR_UNSUPPORTED;
  if (nsplit > 1 && (!workspace || ws_bytes < decode::ws_bytes(max_len, nkv))) return SK_ERR_WORKSPACE;
  if (workspace && (reinterpret_cast<uintptr_t>(workspace) & 15)) return SK_ERR_INVALID_ARG;
  int rc = sk_check_device();
  if (rc != SK_OK) return rc;
  int* err = sk_error_word_ptr();
  if (!err) return SK_ERR_CUDA;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  dim3 grid(nsplit, nkv), block(decode::kThreads);
  if (cache_dtype == SK_BF16) {
    const size_t smem = 2 * decode::kChunk * decode::kHD * sizeof(__nv_bfloat16);
    decode::decode_attn_kernel<__nv_bfloat16><<<grid, block, smem, st>>>(
        qkv, qn, kn, eps, rope, reinterpret_cast<__nv_bfloat16*>(Kc), reinterpret_cast<__nv_bfloat16*>(Vc), pos_ptr,
        pos_add, max_len, nq, nkv, out, workspace, err);
  } else {
    const size_t smem = 2 * decode::kChunk * decode::kHD * sizeof(float);
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
      if (cudaFuncSetAttribute(decode::decode_attn_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)smem) != cudaSuccess)
        return SK_ERR_CUDA;
      attr_set[dev] = true;
    }
    decode::decode_attn_kernel<float><<<grid, block, smem, st>>>(qkv, qn, kn, eps, rope, reinterpret_cast<float*>(Kc),
                                                                  reinterpret_cast<float*>(Vc), pos_ptr, pos_add,
                                                                  max_len, nq, nkv, out, workspace, err);
  }
  return cudaPeekAtLastError() == cudaSuccess ? SK_OK : SK_ERR_CUDA;
}

// ---- Allocation-free variant ------------------------------------------------------------------------
// sk_decode_attention needs a caller-allocated workspace. Some callers cannot allocate device memory
// at call time: a serving process that reserves its whole device budget at start-up and forbids
// cudaMalloc afterwards, a host that drives the engine from inside a CUDA graph capture (where
// cudaMalloc is illegal), or a foreign-language binding that can only hand over buffers it already
// owns. sk_decode_attention_noalloc serves them: it runs the same kernel with its scratch in a
// fixed-size array that lives in the library's device image.
namespace sk {
namespace decode {
// 1 MiB per device that loads this library, held until the process exits. The merge counters sit
// at a fixed place at the end, so calls with different max_len never see each other's partials in
// their counter slots; the kernel returns every counter to zero before it finishes.
constexpr size_t kStaticScratchBytes = size_t(1) << 20;
constexpr size_t kStaticCounterBytes = 4096;
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];
}  // namespace decode
}  // namespace sk

namespace {
std::mutex g_static_mu;
void* g_static_scratch_ptr[64] = {};

// Device address of g_static_scratch on the current device. The first call on a device looks the
// address up and zero-fills the array (synchronously), so that first call must come before any
// stream capture.
int static_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return SK_ERR_CUDA;
  std::lock_guard<std::mutex> lk(g_static_mu);
  if (!g_static_scratch_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, sk::decode::g_static_scratch) != cudaSuccess || !p) return SK_ERR_CUDA;
    if (cudaMemset(p, 0, sk::decode::kStaticScratchBytes) != cudaSuccess) return SK_ERR_CUDA;
    g_static_scratch_ptr[dev] = p;
  }
  *out = g_static_scratch_ptr[dev];
  return SK_OK;
}
}  // namespace

extern "C" int sk_decode_attention_noalloc(const float* qkv, const float* qn, const float* kn, float eps,
                                           const float* rope, void* Kc, void* Vc, const long long* pos_ptr,
                                           int pos_add, int max_len, int nq, int nkv, int hd, float* out,
                                           int cache_dtype, void* stream) {
  using namespace sk::decode;
  if (max_len <= 0 || nkv <= 0) return SK_ERR_INVALID_ARG;
  // partials (o, max/sum) before the counters; the counters always at the array's fixed tail
  const size_t partial_bytes = ws_bytes(max_len, nkv) - (size_t)nkv * 4 - 256;
  if (partial_bytes > kStaticScratchBytes - kStaticCounterBytes || (size_t)nkv * 4 > kStaticCounterBytes)
    return SK_ERR_TOO_LARGE;
  void* scratch = nullptr;
  int rc = static_scratch(&scratch);
  if (rc != SK_OK) return rc;
  char* counters = reinterpret_cast<char*>(scratch) + (kStaticScratchBytes - kStaticCounterBytes);
  void* base = counters - partial_bytes;  // ws_carve(base) puts the counters exactly at `counters`
  return sk_decode_attention(qkv, qn, kn, eps, rope, Kc, Vc, pos_ptr, pos_add, max_len, nq, nkv, hd, out, base,
                             partial_bytes + (size_t)nkv * 4 + 256, cache_dtype, stream);
}
