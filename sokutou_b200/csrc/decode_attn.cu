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


__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

constexpr int kMaxCluster = 16;

__device__ __forceinline__ uint32_t cluster_size_reg() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }
__device__ __forceinline__ void st_cluster(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void fence_acq_rel_cluster() { asm volatile("fence.acq_rel.cluster;" ::: "memory"); }

template <typename CT>
struct Vec4;  // four consecutive cache elements as one shared-memory load
template <>
struct Vec4<__nv_bfloat16> {
  static __device__ __forceinline__ float4 ld(const __nv_bfloat16* p) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u), __uint_as_float(u.y << 16),
                       __uint_as_float(u.y & 0xffff0000u));
  }
};
template <>
struct Vec4<float> {
  static __device__ __forceinline__ float4 ld(const float* p) { return *reinterpret_cast<const float4*>(p); }
};
template <typename CT>
struct Vec8;  // eight consecutive cache elements from shared memory (one 16-byte load for bf16)
template <>
struct Vec8<__nv_bfloat16> {
  static __device__ __forceinline__ void ld(const __nv_bfloat16* p, float (&v)[8]) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    v[0] = __uint_as_float(u.x << 16), v[1] = __uint_as_float(u.x & 0xffff0000u);
    v[2] = __uint_as_float(u.y << 16), v[3] = __uint_as_float(u.y & 0xffff0000u);
    v[4] = __uint_as_float(u.z << 16), v[5] = __uint_as_float(u.z & 0xffff0000u);
    v[6] = __uint_as_float(u.w << 16), v[7] = __uint_as_float(u.w & 0xffff0000u);
  }
};
template <>
struct Vec8<float> {
  static __device__ __forceinline__ void ld(const float* p, float (&v)[8]) {
    const float4 a = *reinterpret_cast<const float4*>(p);
    const float4 b = *reinterpret_cast<const float4*>(p + 4);
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
  }
};


constexpr int kThreadsCl = 256;  // 8 warps: two per scheduler, so dependent chains overlap
constexpr int kPartialBytes = kG * kHD * 4 + kG * 2 * 4;  // one CTA's (o, max, sum) for rank 0

// Rows of the K region of a cluster CTA: its chunk and, in the compact layout, at least the 8 warps'
// PV partials (8 · kG · kHD floats), which reuse that region once the scores are done.
template <typename CT>
__host__ __device__ constexpr int k_rows(int chunk_max, bool compact) {
  return compact && chunk_max < 8 * kG * 4 / (int)sizeof(CT) ? 8 * kG * 4 / (int)sizeof(CT) : chunk_max;
}

// Dynamic shared memory of a cluster CTA, in the order the kernel lays it out: K region, V chunk,
// scores (kG per key, padded to 64 keys) and, in the compact layout, rank 0's CL partial o. 0 when
// the K/V chunks and scores of ceil(max_len / cl) keys exceed 160 KB.
// The compact layout (grouped launches) keeps the PV partials and rank 0's partials in dynamic
// memory sized by the cluster, 2.5 KB of static memory instead of 26.5 KB, so more CTAs fit on an
// SM when many clusters queue; a single launch (nkv clusters, one CTA per SM) keeps the static
// arrays, measured ~5 % faster there (T = 1120: 4.95 vs 5.20 us).
template <typename CT>
static size_t cluster_smem(int max_len, int cl, bool compact) {
  const int chunk_max = (max_len + cl - 1) / cl;
  const size_t chunks = 2 * (size_t)chunk_max * kHD * sizeof(CT) + (size_t)kG * ((chunk_max + 63) & ~63) * 4;
  if (chunks > 160 * 1024) return 0;
  if (!compact) return chunks;
  return chunks + (size_t)(k_rows<CT>(chunk_max, true) - chunk_max) * kHD * sizeof(CT) + (size_t)cl * kG * kHD * 4;
}

// Cluster variant: one thread-block cluster of CL CTAs per kv head, CL = 16 (or 8 where 16 cannot
// be co-scheduled; grouped launches choose by residency, below). The T keys are cut into CL equal chunks of ceil(T / CL) keys, so every CTA is
// busy at every T. Each CTA pushes its chunk's partial (o, max, sum) into rank 0's shared memory
// with st.async, whose completion is counted in bytes on rank 0's mbarrier; rank 0 waits for all
// CL partials and merges them from its own shared memory. No workspace, no global round trip, no
// fence or barrier across the cluster on the way out.
// griddepcontrol.wait precedes every global read (pos, qkv, cache), so under programmatic dependent
// launch only the CTA set-up overlaps the kernel before.
// EARLY: the position and this layer's cache rows before it are not written by the kernel launched
// just before this one, so the position is read and the K/V chunk copies are issued before
// griddepcontrol.wait — they overlap that kernel's tail; only qkv, qn and kn wait for it.
// GROUPED: one launch decodes the independent requests reqs[0 .. gridDim.z): blockIdx.z picks the
// request whose qkv, norms, RoPE table, caches, position and output replace the scalar arguments; every
// request shares max_len, nq, nkv and the cache type. The descriptors are read before the wait for the
// kernel ahead (the caller fills them before capture and does not change them between launches).
template <typename CT, bool EARLY, bool GROUPED = false>
__global__ void __launch_bounds__(kThreadsCl) decode_attn_cluster_kernel(
    const float* __restrict__ qkv_a, const float* __restrict__ qn_a, const float* __restrict__ kn_a, float eps_a,
    const float* __restrict__ rope_a, CT* __restrict__ Kc_a, CT* __restrict__ Vc_a,
    const long long* __restrict__ pos_ptr_a, int pos_add_a, int max_len, int nq, int nkv, float* __restrict__ out_a,
    int* err, const SkDecodeRequest* __restrict__ reqs) {
  const float* qkv = qkv_a;
  const float* qn = qn_a;
  const float* kn = kn_a;
  float eps = eps_a;
  const float* rope = rope_a;
  CT* Kc = Kc_a;
  CT* Vc = Vc_a;
  const long long* pos_ptr = pos_ptr_a;
  int pos_add = pos_add_a;
  float* out = out_a;
  if (GROUPED) {
    const SkDecodeRequest& r = reqs[blockIdx.z];
    qkv = r.qkv;
    qn = r.qn;
    kn = r.kn;
    eps = r.eps;
    rope = r.rope;
    Kc = reinterpret_cast<CT*>(r.Kc);
    Vc = reinterpret_cast<CT*>(r.Vc);
    pos_ptr = r.pos_ptr;
    pos_add = r.pos_add;
    out = r.out;
  }
  const int CL = (int)cluster_size_reg();
  const int rank = (int)cluster_rank();
  const int chunk_max = (max_len + CL - 1) / CL;
  const int chunk_pad = (chunk_max + 63) & ~63;
  extern __shared__ __align__(128) unsigned char dsmem[];
  CT* Ks = reinterpret_cast<CT*>(dsmem);                               // [k_rows][kHD]
  CT* Vs = Ks + (size_t)k_rows<CT>(chunk_max, GROUPED) * kHD;          // [chunk_max][kHD]
  float* sc = reinterpret_cast<float*>(Vs + (size_t)chunk_max * kHD);  // [chunk_pad][kG]: scores, then p
  // PV partials of the 8 key groups [8][kG][kHD], and rank 0's copy of every CTA's chunk partial o
  // [CL][kG][kHD]: static arrays for a single launch; in the compact layout (GROUPED) the first lies
  // over the K chunk (read only by the scores, which are done when the PV pass writes it) and the
  // second follows the scores (the unused static arrays are dropped from that instantiation)
  __shared__ __align__(16) float o_red_s[8][kG][kHD];
  __shared__ __align__(16) float all_o_s[kMaxCluster][kG][kHD];
  float(*o_red)[kG][kHD] = GROUPED ? reinterpret_cast<float(*)[kG][kHD]>(dsmem) : o_red_s;
  float(*all_o)[kG][kHD] = GROUPED ? reinterpret_cast<float(*)[kG][kHD]>(sc + (size_t)chunk_pad * kG) : all_o_s;
  __shared__ __align__(16) float q_s[kG][kHD];
  __shared__ __align__(16) float kn_s[kHD];
  __shared__ __align__(16) float vn_s[kHD];
  __shared__ __align__(16) float all_ml[kMaxCluster][kG][2];   // rank 0: every CTA's chunk (max, sum)
  __shared__ float wts[kMaxCluster][kG];                       // rank 0: merge weights
  __shared__ float den_s[kG];
  __shared__ float red[8][2];
  __shared__ float stat[kG][2];
  __shared__ __align__(8) uint64_t bar;      // the K/V bulk copy
  __shared__ __align__(8) uint64_t mrg_bar;  // rank 0: CL partials, counted in bytes

  const int kvh = blockIdx.y;
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  const int g_t = t >> 7, d = t & (kHD - 1);  // prologue role: head g_t, dimension d
  if (t == 0) {
    mbar_init(&bar, 1);
    if (rank == 0) mbar_init(&mrg_bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  cluster_arrive_relaxed();  // matched by cluster_wait() before the first push into rank 0
  if (rank == 0 && t == 0) mbar_arrive_expect_tx(&mrg_bar, (uint32_t)(CL * kPartialBytes));
  // The position, this CTA's share of the keys, and the bulk copies of its K/V chunk (the new row is
  // appended below, not copied).
  int pos = 0, T = 0, chunk = 0, s0 = 0, n = 0, n_ld = 0;
  bool owner = false;
  const size_t head_base = (size_t)kvh * max_len * kHD;
  auto issue_kv = [&]() -> bool {
    pos = (pos_ptr ? (int)pos_ptr[0] : 0) + pos_add;
    if (pos < 0 || pos >= max_len) {  // every CTA of every cluster reads the same pos: all leave here
      if (rank == 0 && kvh == 0 && t == 0) set_dev_error(err, SK_DEVERR_POS_RANGE);
      return false;
    }
    T = pos + 1;
    chunk = (T + CL - 1) / CL;
    s0 = rank * chunk;
    n = max(0, min(chunk, T - s0));  // keys of this CTA (0 for ranks past T)
    owner = n > 0 && (s0 + n == T);  // holds the new position
    n_ld = owner ? n - 1 : n;
    if (t == 0 && n_ld > 0) {
      const uint32_t bytes = (uint32_t)(n_ld * kHD * sizeof(CT));
      mbar_arrive_expect_tx(&bar, 2 * bytes);
      bulk_load(Ks, Kc + head_base + (size_t)s0 * kHD, bytes, &bar);
      bulk_load(Vs, Vc + head_base + (size_t)s0 * kHD, bytes, &bar);
    }
    return true;
  };
  if (EARLY && !issue_kv()) return;
  griddep_wait();
  griddep_launch_dependents();
  // loads that do not depend on the position go out together with it
  const float qv = qkv[(size_t)(kvh * kG + g_t) * kHD + d];
  const float xv = qkv[(size_t)(nq + g_t * nkv) * kHD + (size_t)kvh * kHD + d];  // k (g_t = 0) or v (g_t = 1)
  const float qn_d = qn[d], kn_d = kn[d];
  if (!EARLY && !issue_kv()) return;
  const float c = rope[(size_t)pos * kHD + (d & 63)];
  const float s = rope[(size_t)pos * kHD + 64 + (d & 63)];

  // ---- prologue (qwen3/kernels.py:351-380): thread (g_t, d) normalises q head g_t, and the new k
  // (threads of g_t = 0, owner only); the v of g_t = 1 is stored raw.
  {
    const float kv = (owner && g_t == 0) ? xv : 0.f;
    const float sq = warp_sum(qv * qv), sk = warp_sum(kv * kv);
    if (lane == 0) {
      red[w][0] = sq;
      red[w][1] = sk;
    }
    __syncthreads();
    const int w0 = g_t * 4;  // the 4 warps of this head
    const float ssq = red[w0][0] + red[w0 + 1][0] + red[w0 + 2][0] + red[w0 + 3][0];
    const float ssk = red[0][1] + red[1][1] + red[2][1] + red[3][1];
    q_s[g_t][d] = qv * rsqrtf(ssq / kHD + eps) * qn_d;
    if (owner && g_t == 0) kn_s[d] = kv * rsqrtf(ssk / kHD + eps) * kn_d;
    __syncthreads();
    const float rot = d < 64 ? -q_s[g_t][d + 64] : q_s[g_t][d - 64];
    const float qr = (q_s[g_t][d] * c + rot * s) * 0.08838834764831845f;  // 1/sqrt(128), qwen3/kernels.py:378
    float knew = 0.f;
    if (owner && g_t == 0) {
      const float rk = d < 64 ? -kn_s[d + 64] : kn_s[d - 64];
      knew = kn_s[d] * c + rk * s;
    }
    __syncthreads();
    q_s[g_t][d] = qr;
    if (owner) {
      if (g_t == 0) {
        const CT kst = Cache<CT>::st(knew);
        Kc[head_base + (size_t)pos * kHD + d] = kst;  // append (qwen3/kernels.py:364,366)
        kn_s[d] = Cache<CT>::ld(&kst);                 // attended as read back from the cache
      } else {
        const CT vst = Cache<CT>::st(xv);
        Vc[head_base + (size_t)pos * kHD + d] = vst;
        vn_s[d] = Cache<CT>::ld(&vst);
      }
    }
    __syncthreads();
  }
  bool ok = true;
  if (n_ld > 0) ok = mbar_wait(&bar, 0, err);  // on a time-out the output is invalid (error word set)

  // ---- scores. Up to 64 keys (T <= 1024 with clusters of 16): one pass of 8 keys per warp, lane owns
  // 4 dims. More keys: 16 keys per warp and pass as 8 pairs, half-warp h = lane / 16 taking key 2i + h
  // of pair i with 8 dims per lane (one 16-byte load per key for bf16), so 128 keys still take one pass
  // — measured faster above 64 keys, slower below (twice the work per warp pass).
  if (n > 64) {
    const int hl = lane & 15, h = lane >> 4;
    float qa[kG][8];
#pragma unroll
    for (int g = 0; g < kG; ++g) {
      const float4 a = *reinterpret_cast<const float4*>(&q_s[g][8 * hl]);
      const float4 b = *reinterpret_cast<const float4*>(&q_s[g][8 * hl + 4]);
      qa[g][0] = a.x, qa[g][1] = a.y, qa[g][2] = a.z, qa[g][3] = a.w;
      qa[g][4] = b.x, qa[g][5] = b.y, qa[g][6] = b.z, qa[g][7] = b.w;
    }
    float knew[8];
    {
      const float4 a = *reinterpret_cast<const float4*>(&kn_s[8 * hl]);
      const float4 b = *reinterpret_cast<const float4*>(&kn_s[8 * hl + 4]);
      knew[0] = a.x, knew[1] = a.y, knew[2] = a.z, knew[3] = a.w;
      knew[4] = b.x, knew[5] = b.y, knew[6] = b.z, knew[7] = b.w;
    }
    for (int base = 0; base < n; base += 128) {
      float part[kG * 8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int j = base + 16 * w + 2 * i + h;
        float k8[8];
        if (ok && j < n_ld && SK_INB(j < chunk_max, err)) {
          Vec8<CT>::ld(Ks + (size_t)j * kHD + 8 * hl, k8);
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) k8[e] = knew[e];
        }
#pragma unroll
        for (int g = 0; g < kG; ++g) {
          float acc = 0.f;
#pragma unroll
          for (int e = 0; e < 8; ++e) acc += qa[g][e] * k8[e];
          part[g * 8 + i] = acc;
        }
      }
      // reduce-scatter of 16 values over lane bits 3..0 (within each half-warp)
#pragma unroll
      for (int off = 8, m = 16; off >= 1; off >>= 1, m >>= 1) {
        const bool upper = (lane & off) != 0;
#pragma unroll
        for (int i = 0; i < m / 2; ++i) {
          const float send = upper ? part[i] : part[i + m / 2];
          const float keep = upper ? part[i + m / 2] : part[i];
          part[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
      }
      // lane now holds value index hl: head (hl >> 3), pair (hl & 7) -> key 16w + 2 (hl & 7) + h
      const int g = hl >> 3, j = base + 16 * w + 2 * (hl & 7) + h;
      if (j < n && SK_INB(j < chunk_pad, err)) sc[j * kG + g] = part[0];
    }
  } else {
    float4 qa[kG];
#pragma unroll
    for (int g = 0; g < kG; ++g) qa[g] = *reinterpret_cast<const float4*>(&q_s[g][4 * lane]);
    const float4 knew4 = *reinterpret_cast<const float4*>(&kn_s[4 * lane]);
    for (int base = 0; base < n; base += 64) {
      float part[kG * 8];
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        const int j = base + 8 * w + jj;
        const float4 k4 = (ok && j < n_ld && SK_INB(j < chunk_max, err)) ? Vec4<CT>::ld(Ks + (size_t)j * kHD + 4 * lane)
                                                                          : knew4;
#pragma unroll
        for (int g = 0; g < kG; ++g)
          part[g * 8 + jj] = qa[g].x * k4.x + qa[g].y * k4.y + qa[g].z * k4.z + qa[g].w * k4.w;
      }
      // reduce-scatter of 16 values over lane bits 4..1, then a plain sum over bit 0
#pragma unroll
      for (int off = 16, m = 16; off >= 2; off >>= 1, m >>= 1) {
        const bool upper = (lane & off) != 0;
#pragma unroll
        for (int i = 0; i < m / 2; ++i) {
          const float send = upper ? part[i] : part[i + m / 2];
          const float keep = upper ? part[i + m / 2] : part[i];
          part[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
      }
      part[0] += __shfl_xor_sync(0xffffffffu, part[0], 1);
      // lane l now holds value index (l >> 1): head (l >> 4), key (l >> 1) & 7
      const int g = lane >> 4, j = base + 8 * w + ((lane >> 1) & 7);
      if ((lane & 1) == 0 && j < n && SK_INB(j < chunk_pad, err)) sc[j * kG + g] = part[0];
    }
  }
  __syncthreads();
  // ---- chunk softmax: warp g handles head g
  if (w < kG) {
    const int g = w;
    float m = -INFINITY;
    for (int j = lane; j < n; j += 32) m = fmaxf(m, sc[j * kG + g]);
    m = warp_max(m);
    float l = 0.f;
    for (int j = lane; j < n; j += 32) {
      const float e = expf(sc[j * kG + g] - m);
      sc[j * kG + g] = e;
      l += e;
    }
    l = warp_sum(l);
    if (lane == 0) {
      stat[g][0] = m;  // -inf for a CTA with no keys
      stat[g][1] = l;
    }
  }
  __syncthreads();
  // ---- PV: thread owns dims [4*(t%32), +4) over keys j = w, w + 8, ...
  {
    const int dq = 4 * lane;
    float4 acc[kG];
#pragma unroll
    for (int g = 0; g < kG; ++g) acc[g] = make_float4(0.f, 0.f, 0.f, 0.f);
    const float4 vnew4 = *reinterpret_cast<const float4*>(&vn_s[dq]);
    for (int j = w; j < n; j += 8) {
      const float4 v4 = (ok && j < n_ld) ? Vec4<CT>::ld(Vs + (size_t)j * kHD + dq) : vnew4;
      const float2 p = *reinterpret_cast<const float2*>(&sc[j * kG]);
      acc[0].x += p.x * v4.x;
      acc[0].y += p.x * v4.y;
      acc[0].z += p.x * v4.z;
      acc[0].w += p.x * v4.w;
      acc[1].x += p.y * v4.x;
      acc[1].y += p.y * v4.y;
      acc[1].z += p.y * v4.z;
      acc[1].w += p.y * v4.w;
    }
#pragma unroll
    for (int g = 0; g < kG; ++g) *reinterpret_cast<float4*>(&o_red[w][g][dq]) = acc[g];
  }
  __syncthreads();
  // ---- push this chunk's partial into rank 0 (st.async, completion counted on rank 0's barrier)
  cluster_wait();  // rank 0's barrier is initialised
  {
    const uint32_t rbar = mapa(&mrg_bar, 0);
    float v = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) v += o_red[i][g_t][d];
    if (SK_INB(rank < kMaxCluster, err)) {
      st_async(mapa(&all_o[rank][g_t][d], 0), v, rbar);
      if (t < kG * 2) st_async(mapa(&all_ml[rank][t >> 1][t & 1], 0), stat[t >> 1][t & 1], rbar);
    }
  }
  if (rank == 0) {
    // block-uniform: a time-out seen by any thread skips the merge for the whole CTA
    const bool got = __syncthreads_and(mbar_wait_cluster(&mrg_bar, 0, err)) != 0;
    if (got) {
      if (t < kMaxCluster * kG) {  // weight of each chunk, in parallel
        const int r = t >> 1, g = t & 1;
        float M = -INFINITY;
#pragma unroll
        for (int i = 0; i < kMaxCluster; ++i)
          if (i < CL) M = fmaxf(M, all_ml[i][g][0]);
        wts[r][g] = (r < CL && all_ml[r][g][1] > 0.f) ? expf(all_ml[r][g][0] - M) : 0.f;
      }
      __syncthreads();
      if (t < kG) {
        float dn = 0.f;
#pragma unroll
        for (int r = 0; r < kMaxCluster; ++r)
          if (r < CL) dn += wts[r][t] * all_ml[r][t][1];
        den_s[t] = dn;
      }
      __syncthreads();
      float num = 0.f;
#pragma unroll
      for (int r = 0; r < kMaxCluster; ++r)
        if (r < CL) num += wts[r][g_t] * all_o[r][g_t][d];
      if (SK_INB(kvh * kG + g_t < nq, err)) out[(size_t)(kvh * kG + g_t) * kHD + d] = num / den_s[g_t];
    }
  }
  if (!ok && t == 0) mbar_wait(&bar, 0, err);
}

// ---- prefill producer -----------------------------------------------------------------------------
// Qwen3 prefill (the prompt's causal attention, done by the HF talker with SDPA at
// qwen3/fast.py:251-263): for every prompt token the q heads are RMS-normalised and rotated, and the k
// (normalised, rotated) and v rows are appended to the cache at pos0 + token — the same per-element
// arithmetic as the decode kernel's prologue (qwen3/kernels.py:351-380), so a cache filled here holds
// the bits decode steps would have written. q goes to q_buf (nq, T, 128) in the cache dtype (bf16 for
// the tensor-core attention, fp32 for the fp32 mode; the 1/sqrt(128) scale is applied there). Grid (T, nkv), 256 threads: thread (g, d) owns
// dimension d of q head kvh·2 + g, and of k (g = 0) or v (g = 1).
template <typename CT>
__global__ void __launch_bounds__(256) prefill_prologue_kernel(const float* __restrict__ qkv,
                                                                const float* __restrict__ qn,
                                                                const float* __restrict__ kn, float eps,
                                                                const float* __restrict__ rope, CT* __restrict__ Kc,
                                                                CT* __restrict__ Vc, CT* __restrict__ q_buf,
                                                                int pos0, int T, int max_len, int nq, int nkv,
                                                                int* err) {
  __shared__ float red[8][2];
  __shared__ float q_s[kG][kHD];
  __shared__ float kn_s[kHD];
  asm volatile("griddepcontrol.wait;" ::: "memory");  // qkv may come from the kernel just before
  asm volatile("griddepcontrol.launch_dependents;");
  const int tok = blockIdx.x, kvh = blockIdx.y;
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  const int g = t >> 7, d = t & (kHD - 1);
  const int pos = pos0 + tok;
  const float* row = qkv + (size_t)tok * (nq + 2 * nkv) * kHD;
  const float qv = row[(size_t)(kvh * kG + g) * kHD + d];
  const float xv = row[(size_t)(nq + g * nkv) * kHD + (size_t)kvh * kHD + d];  // k (g = 0) or v (g = 1)
  const float kv = g == 0 ? xv : 0.f;
  const float sq = warp_sum(qv * qv), sk = warp_sum(kv * kv);
  if (lane == 0) {
    red[w][0] = sq;
    red[w][1] = sk;
  }
  __syncthreads();
  const int w0 = g * 4;  // the 4 warps of this head
  const float ssq = red[w0][0] + red[w0 + 1][0] + red[w0 + 2][0] + red[w0 + 3][0];
  const float ssk = red[0][1] + red[1][1] + red[2][1] + red[3][1];
  q_s[g][d] = qv * rsqrtf(ssq / kHD + eps) * qn[d];
  if (g == 0) kn_s[d] = kv * rsqrtf(ssk / kHD + eps) * kn[d];
  __syncthreads();
  const float c = rope[(size_t)pos * kHD + (d & 63)];
  const float s = rope[(size_t)pos * kHD + 64 + (d & 63)];
  const float rot = d < 64 ? -q_s[g][d + 64] : q_s[g][d - 64];
  if (SK_INB(kvh * kG + g < nq && tok < T, err))
    q_buf[((size_t)(kvh * kG + g) * T + tok) * kHD + d] = Cache<CT>::st(q_s[g][d] * c + rot * s);
  if (!SK_INB(pos < max_len && kvh < nkv, err)) return;
  const size_t at = ((size_t)kvh * max_len + pos) * kHD + d;
  if (g == 0) {
    const float rk = d < 64 ? -kn_s[d + 64] : kn_s[d - 64];
    Kc[at] = Cache<CT>::st(kn_s[d] * c + rk * s);  // qwen3/kernels.py:364,366
  } else {
    Vc[at] = Cache<CT>::st(xv);
  }
}

}  // namespace decode
}  // namespace sk

using namespace sk;


namespace sk {
namespace decode {

// Cluster size usable on this device for a kernel needing `smem` bytes: 16 when nkv clusters of
// 16 fit at once, else 8, else 0 (cached per device, dtype and shared-memory size).
template <typename CT>
static int cluster_size(int nkv, size_t smem) {
  static std::mutex mu;
  static int cached_cl[64][2] = {};
  static size_t cached_smem[64][2] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  const int ti = sizeof(CT) == 2 ? 0 : 1;
  std::lock_guard<std::mutex> lk(mu);
  if (cached_smem[dev][ti] == smem && cached_cl[dev][ti] != 0) return cached_cl[dev][ti];
  auto kfn = decode_attn_cluster_kernel<CT, false>;
  for (auto f : {decode_attn_cluster_kernel<CT, false>, decode_attn_cluster_kernel<CT, true>}) {
    if (cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) return 0;
    cudaFuncSetAttribute(f, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  }
  int chosen = 0;
  for (int cl : {16, 8}) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(cl, nkv);
    cfg.blockDim = dim3(kThreadsCl);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cl;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kfn, &cfg) == cudaSuccess && n >= nkv) {
      chosen = cl;
      break;
    }
    cudaGetLastError();  // clear a refused query
  }
  cached_cl[dev][ti] = chosen;
  cached_smem[dev][ti] = smem;
  return chosen;
}

template <typename CT>
static int launch_cluster(const float* qkv, const float* qn, const float* kn, float eps, const float* rope, void* Kc,
                          void* Vc, const long long* pos_ptr, int pos_add, int max_len, int nq, int nkv, float* out,
                          int* err, bool early, cudaStream_t st) {
  // the shared memory of the largest chunk decides whether one cluster per kv head can hold T = max_len
  for (int cl : {16, 8}) {
    const size_t smem = cluster_smem<CT>(max_len, cl, false);
    if (smem == 0) continue;
    const int use = cluster_size<CT>(nkv, smem);
    if (use != cl) continue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(cl, nkv);
    cfg.blockDim = dim3(kThreadsCl);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cl;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    const cudaError_t e =
        early ? cudaLaunchKernelEx(&cfg, decode_attn_cluster_kernel<CT, true>, qkv, qn, kn, eps, rope,
                                   reinterpret_cast<CT*>(Kc), reinterpret_cast<CT*>(Vc), pos_ptr, pos_add, max_len, nq,
                                   nkv, out, err, (const SkDecodeRequest*)nullptr)
              : cudaLaunchKernelEx(&cfg, decode_attn_cluster_kernel<CT, false>, qkv, qn, kn, eps, rope,
                                   reinterpret_cast<CT*>(Kc), reinterpret_cast<CT*>(Vc), pos_ptr, pos_add, max_len, nq,
                                   nkv, out, err, (const SkDecodeRequest*)nullptr);
    if (e != cudaSuccess) return SK_ERR_CUDA;
    return SK_OK;
  }
  return SK_ERR_UNSUPPORTED;
}

// Clusters of `cl` CTAs of a grouped launch that can be resident on the device at once (0 when none).
template <typename CT>
static int grouped_clusters(void (*kern)(const float*, const float*, const float*, float, const float*, CT*, CT*,
                                         const long long*, int, int, int, int, float*, int*, const SkDecodeRequest*),
                            int cl, int nkv, size_t smem) {
  cudaLaunchConfig_t q = {};
  q.gridDim = dim3(cl, nkv);
  q.blockDim = dim3(kThreadsCl);
  q.dynamicSmemBytes = smem;
  cudaLaunchAttribute a[1];
  a[0].id = cudaLaunchAttributeClusterDimension;
  a[0].val.clusterDim.x = cl;
  a[0].val.clusterDim.y = 1;
  a[0].val.clusterDim.z = 1;
  q.attrs = a;
  q.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &q) != cudaSuccess) {
    cudaGetLastError();  // clear a refused query
    return 0;
  }
  return n;
}

// The clusters of a grouped launch depend on nothing outside themselves and may run wave after wave.
// Cluster size: 8 when strictly more clusters of 8 than of 16 are resident at once (the same number of
// clusters, nkv · R, then runs in fewer waves, and each request's partials merge over 8 CTAs instead of
// 16), else 16; whichever of the two is schedulable when only one is. Decided once per device, mode and
// max_len. Measured at T = 1120, bf16, R = 8 / 16 / 32: max_len 1536 (a CTA of a 16-cluster holds 70 KB
// of shared memory, one of an 8-cluster 112 KB: 3 and 2 per SM) 19.2 / 33.7 / 62.2 us with 16,
// 17.6 / 29.2 / 51.9 us with 8; max_len 1152 (57 KB and 87 KB: 4 and 2 per SM) 17.3 / 29.1 / 52.4 vs
// 17.4 / 29.0 / 52.1 us.
template <typename CT>
static int launch_grouped(const SkDecodeRequest* reqs, int R, int max_len, int nq, int nkv, int* err, bool early,
                          cudaStream_t st) {
  auto kern = early ? decode_attn_cluster_kernel<CT, true, true> : decode_attn_cluster_kernel<CT, false, true>;
  int cl = 0;
  size_t smem = 0;
  {
    static std::mutex mu;
    static size_t set_to[64][2] = {};
    static int for_len[64][2] = {};
    static int chosen[64][2] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return SK_ERR_CUDA;
    std::lock_guard<std::mutex> lk(mu);
    if (for_len[dev][early] != max_len || chosen[dev][early] == 0) {
      const size_t s16 = cluster_smem<CT>(max_len, 16, true), s8 = cluster_smem<CT>(max_len, 8, true);
      const size_t top = s16 > s8 ? s16 : s8;
      if (top == 0) return SK_ERR_UNSUPPORTED;
      if (set_to[dev][early] < top) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)top) != cudaSuccess)
          return SK_ERR_CUDA;
        cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        set_to[dev][early] = top;
      }
      const int n16 = s16 ? grouped_clusters<CT>(kern, 16, nkv, s16) : 0;
      const int n8 = s8 ? grouped_clusters<CT>(kern, 8, nkv, s8) : 0;
      const int pick = n8 > n16 ? 8 : (n16 > 0 ? 16 : 0);
      if (pick == 0) return SK_ERR_UNSUPPORTED;
      chosen[dev][early] = pick;
      for_len[dev][early] = max_len;
    }
    cl = chosen[dev][early];
    smem = cluster_smem<CT>(max_len, cl, true);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(cl, nkv, R);
  cfg.blockDim = dim3(kThreadsCl);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cl;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  if (cudaLaunchKernelEx(&cfg, kern, (const float*)nullptr, (const float*)nullptr, (const float*)nullptr, 0.f,
                         (const float*)nullptr, (CT*)nullptr, (CT*)nullptr, (const long long*)nullptr, 0, max_len, nq,
                         nkv, (float*)nullptr, err, reqs) != cudaSuccess)
    return SK_ERR_CUDA;
  return cudaPeekAtLastError() == cudaSuccess ? SK_OK : SK_ERR_CUDA;
}

}  // namespace decode
}  // namespace sk

extern "C" size_t sk_decode_workspace_bytes(int max_len, int nq, int nkv, int hd, int cache_dtype) {
  (void)nq;
  (void)hd;
  (void)cache_dtype;
  if (max_len <= 0 || nkv <= 0) return 0;
  return decode::ws_bytes(max_len, nkv);
}

extern "C" int sk_decode_attention_ex(const float* qkv, const float* qn, const float* kn, float eps,
                                      const float* rope, void* Kc, void* Vc, const long long* pos_ptr, int pos_add,
                                      int max_len, int nq, int nkv, int hd, float* out, void* workspace,
                                      size_t ws_bytes, int cache_dtype, int flags, void* stream) {
  if (flags & ~SK_DECODE_KV_STABLE) return SK_ERR_INVALID_ARG;
  const bool early = (flags & SK_DECODE_KV_STABLE) != 0;
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
  if (max_len > decode::kChunk) {
    rc = cache_dtype == SK_BF16
             ? decode::launch_cluster<__nv_bfloat16>(qkv, qn, kn, eps, rope, Kc, Vc, pos_ptr, pos_add, max_len, nq,
                                                      nkv, out, err, early, st)
             : decode::launch_cluster<float>(qkv, qn, kn, eps, rope, Kc, Vc, pos_ptr, pos_add, max_len, nq, nkv,
                                             out, err, early, st);
    if (rc != SK_ERR_UNSUPPORTED) return rc;  // else: too long for one cluster, use the workspace kernel
  }
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

extern "C" int sk_decode_attention(const float* qkv, const float* qn, const float* kn, float eps, const float* rope,
                                   void* Kc, void* Vc, const long long* pos_ptr, int pos_add, int max_len, int nq,
                                   int nkv, int hd, float* out, void* workspace, size_t ws_bytes, int cache_dtype,
                                   void* stream) {
  return sk_decode_attention_ex(qkv, qn, kn, eps, rope, Kc, Vc, pos_ptr, pos_add, max_len, nq, nkv, hd, out,
                                workspace, ws_bytes, cache_dtype, 0, stream);
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
// address up and zero-fills the array, then waits for the whole device: cudaMemset returns before
// the fill has finished and runs on the legacy default stream, which does not order against
// non-blocking streams, so without the wait a first call on such a stream could start its kernel
// on a half-cleared array. The pointer is published only after the fill is complete. Because of
// that wait the first call must come before any stream capture.
int static_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return SK_ERR_CUDA;
  std::lock_guard<std::mutex> lk(g_static_mu);
  if (!g_static_scratch_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, sk::decode::g_static_scratch) != cudaSuccess || !p) return SK_ERR_CUDA;
    if (cudaMemset(p, 0, sk::decode::kStaticScratchBytes) != cudaSuccess) return SK_ERR_CUDA;
    if (cudaDeviceSynchronize() != cudaSuccess) return SK_ERR_CUDA;
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

// The prefill producer launch (used by sk_prefill_attention).
int sk_launch_prefill_prologue(const float* qkv, const float* qn, const float* kn, float eps, const float* rope,
                               void* Kc, void* Vc, void* q_buf, int pos0, int T, int max_len, int nq, int nkv,
                               int cache_dtype, cudaStream_t st) {
  using namespace sk::decode;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(T, nkv);
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int* err = sk_error_word_ptr();
  if (!err) return SK_ERR_CUDA;
  const cudaError_t e =
      cache_dtype == SK_BF16
          ? cudaLaunchKernelEx(&cfg, prefill_prologue_kernel<__nv_bfloat16>, qkv, qn, kn, eps, rope,
                               reinterpret_cast<__nv_bfloat16*>(Kc), reinterpret_cast<__nv_bfloat16*>(Vc),
                               reinterpret_cast<__nv_bfloat16*>(q_buf), pos0, T, max_len, nq, nkv, err)
          : cudaLaunchKernelEx(&cfg, prefill_prologue_kernel<float>, qkv, qn, kn, eps, rope,
                               reinterpret_cast<float*>(Kc), reinterpret_cast<float*>(Vc),
                               reinterpret_cast<float*>(q_buf), pos0, T, max_len, nq, nkv, err);
  if (e != cudaSuccess) return SK_ERR_CUDA;
  return cudaPeekAtLastError() == cudaSuccess ? SK_OK : SK_ERR_CUDA;
}

extern "C" int sk_decode_attention_grouped(const SkDecodeRequest* reqs, int R, int max_len, int nq, int nkv, int hd,
                                           int cache_dtype, int flags, void* stream) {
  if (flags & ~SK_DECODE_KV_STABLE) return SK_ERR_INVALID_ARG;
  if (!reqs || R <= 0 || R > 65535 || max_len <= 0 || nkv <= 0 || nq <= 0) return SK_ERR_INVALID_ARG;
  if (reinterpret_cast<uintptr_t>(reqs) & 15) return SK_ERR_INVALID_ARG;
  if (hd != decode::kHD || nq != decode::kG * nkv) return SK_ERR_UNSUPPORTED;
  if (cache_dtype != SK_BF16 && cache_dtype != SK_F32) return SK_ERR_UNSUPPORTED;
  int rc = sk_check_device();
  if (rc != SK_OK) return rc;
  int* err = sk_error_word_ptr();
  if (!err) return SK_ERR_CUDA;
  const bool early = (flags & SK_DECODE_KV_STABLE) != 0;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  return cache_dtype == SK_BF16 ? decode::launch_grouped<__nv_bfloat16>(reqs, R, max_len, nq, nkv, err, early, st)
                                : decode::launch_grouped<float>(reqs, R, max_len, nq, nkv, err, early, st);
}
