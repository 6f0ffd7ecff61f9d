// Qwen3-TTS talker decode: one layer's whole attention block in one launch —
//   qkv = W_qkv · RMSNorm(h)        (the reference's rms_gemv, qwen3/kernels.py:271-275)
//   att = attention(qkv, caches)    (the reference's attn, qwen3/kernels.py:341-414: QK-RMSNorm, RoPE,
//                                    KV append, GQA over T = pos + 1 keys)
//   h  += W_o · att                 (the reference's gemv with accumulate, qwen3/kernels.py:301-305)
// which the reference runs as three launches per layer (qwen3/kernels.py:619-624).
//
// Each of the three steps needs the whole output of the one before, so the launch is cooperative: one
// CTA per SM, all resident, with two grid-wide barriers between the phases (two monotonic counters in
// the caller's workspace — arrivals and completed barriers, never reset, read once per launch; bounded
// spins that record SK_DEVERR_TIMEOUT and give up after 2 s).
// The weights do not depend on anything computed in the launch: each CTA's W_qkv rows are fetched into
// its shared memory by one bulk copy issued before the launch waits for the kernel ahead of it; once
// they have landed the W_o rows and the K/V chunks are asked into L2, so that they stream from HBM
// while phase 1 runs instead of competing with the rows phase 1 waits for.
//
//   phase 1  rows of W_qkv split evenly over the CTAs (staged in shared memory when the slice fits);
//            a warp per row, each lane's slice of x = h ⊙ in_norm held in registers, the RMS scale
//            applied to the dot product (as the reference does).
//   phase 2  split-KV attention: items (128-key chunk, kv head), one per CTA (looping when there are
//            more), each writing its partial (o, max, sum) to the workspace — no merge step here.
//   phase 3  every CTA bulk-copies all partials into shared memory and merges them itself into att
//            (in a fixed order: the result does not depend on which CTA finished first, and no float
//            atomics are used anywhere, so the fp32 mode is reproducible run to run); then its rows of
//            W_o (staged in shared memory after phase 1), h[r] += the dot product.
#include <mutex>

#include "sk_common.cuh"

namespace sk {
namespace block {

constexpr int kHD = 128, kG = 2, kChunk = 128, kThreads = 256;
constexpr int kMaxSplits = 64;  // max_len <= 8192
constexpr int kPartFloats = kG * (kHD + 2);  // one chunk's partial: per q head o[128], max, sum
// Thread 0 runs the grid barriers; every bulk copy and L2 prefetch is issued by another thread, so that
// the barrier's fences never wait behind this CTA's copies in flight.
constexpr int kCopyThread = 32;

template <typename T>
struct Elem;
template <>
struct Elem<__nv_bfloat16> {
  static constexpr int kVec = 8;  // elements per 16-byte load
  static __device__ __forceinline__ float dot8(const uint4& w, const float (&x)[8]) {
    return __uint_as_float(w.x << 16) * x[0] + __uint_as_float(w.x & 0xffff0000u) * x[1] +
           __uint_as_float(w.y << 16) * x[2] + __uint_as_float(w.y & 0xffff0000u) * x[3] +
           __uint_as_float(w.z << 16) * x[4] + __uint_as_float(w.z & 0xffff0000u) * x[5] +
           __uint_as_float(w.w << 16) * x[6] + __uint_as_float(w.w & 0xffff0000u) * x[7];
  }
  static __device__ __forceinline__ float ld(const __nv_bfloat16* p) { return __bfloat162float(*p); }
  static __device__ __forceinline__ __nv_bfloat16 st(float f) { return __float2bfloat16_rn(f); }
  static __device__ __forceinline__ float4 ld4(const __nv_bfloat16* p) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u), __uint_as_float(u.y << 16),
                       __uint_as_float(u.y & 0xffff0000u));
  }
};
template <>
struct Elem<float> {
  static constexpr int kVec = 4;
  static __device__ __forceinline__ float dot8(const uint4& w, const float (&x)[4]) {  // 4 elements
    return __uint_as_float(w.x) * x[0] + __uint_as_float(w.y) * x[1] + __uint_as_float(w.z) * x[2] +
           __uint_as_float(w.w) * x[3];
  }
  static __device__ __forceinline__ float ld(const float* p) { return *p; }
  static __device__ __forceinline__ float st(float f) { return f; }
  static __device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
};

struct Params {
  float* h;                 // [hidden] residual, updated in place
  const float* in_norm;     // [hidden]
  float eps_in;
  const void* w_qkv;        // [(nq + 2 nkv) * 128][hidden]
  const float* qn;
  const float* kn;
  float eps;
  const float* rope;        // [max_len][128]
  void* Kc;
  void* Vc;                 // [nkv][max_len][128]
  const long long* pos_ptr;
  int pos_add, max_len, nq, nkv, hidden;
  const void* w_o;          // [hidden][nq * 128]
  float* qkv;               // workspace: (nq + 2 nkv) * 128
  float* att;               // workspace: nq * 128
  float* part;              // workspace: [nkv][nsplit][kG][kHD + 2]
  unsigned* sync;           // workspace: the grid barrier's words (completed barriers, arrivals)
  int* err;
};

__host__ __device__ inline int nsplit_of(int max_len) { return (max_len + kChunk - 1) / kChunk; }
constexpr size_t kSyncBytes = 256;  // the barrier words: completed barriers, arrivals (a line each)
__host__ __device__ inline size_t ws_bytes(int nq, int nkv, int max_len) {
  const size_t fl = (size_t)(nq + 2 * nkv) * kHD + (size_t)nq * kHD + (size_t)nkv * nsplit_of(max_len) * kG * (kHD + 2);
  return kSyncBytes + ((fl * 4 + 15) & ~(size_t)15);
}

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
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}
// Bring [p, p + bytes) into L2 in pieces of up to 32 KB (p 16-byte aligned; the tail rounded down).
__device__ __forceinline__ void prefetch_range(const void* p, size_t bytes) {
  const char* c = reinterpret_cast<const char*>(p);
  for (size_t off = 0; off + 16 <= bytes; off += 32768) {
    const size_t n = min((size_t)32768, bytes - off) & ~(size_t)15;
    if (n) prefetch_l2(c + off, (uint32_t)n);
  }
}

// Grid-wide barrier over all CTAs of the (cooperative) launch, with as few dependent trips to L2 as
// possible (each costs about half a microsecond while the weights stream in): the words are never reset.
// sync[0] (its own 128-byte line) counts the barriers completed so far; sync[kLine] counts arrivals,
// G per barrier, so at rest it equals G times sync[0]. Both only grow (modulo 2^32; G times the barrier
// number is consistent modulo 2^32 because every barrier adds exactly G). A launch reads the number of
// completed barriers n0 once (the same in every CTA: none of this launch's barriers can complete before
// every CTA has arrived, and each reads it before its first arrival); its k-th barrier (k = 0, 1) then
// waits for arrival number (n0 + k + 1)·G: the CTA whose acq_rel atomic returns one less than that is the
// last, and publishes the barrier with a release reduction on sync[0]; the others poll sync[0] with
// acquire loads. Only thread 0 calls these, between two __syncthreads.
constexpr int kLine = 32;  // words per 128-byte line
__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned atom_add_acq_rel_gpu(unsigned* p, unsigned v) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ void red_release_gpu_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Barrier `k` of this launch (n0: the completed-barrier count read at the launch's start).
__device__ __forceinline__ bool grid_barrier_k(unsigned* sync, unsigned n0, unsigned k, int* err) {
  const unsigned done = n0 + k + 1;              // sync[0] once this barrier has completed
  const unsigned last = done * gridDim.x - 1u;  // the arrival count the last CTA sees before its own
  // acq_rel: the CTA's writes (ordered before this thread by the __syncthreads) are released with it
  if (atom_add_acq_rel_gpu(sync + kLine, 1u) == last) {
    red_release_gpu_add(sync, 1u);
    return true;
  }
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 0; (int)(ld_acquire_gpu(sync) - done) < 0; ++i) {
    __nanosleep(32);
    if ((i & 255u) == 255u && globaltimer_ns() - t0 > kWaitLimitNs) {
      set_dev_error(err, SK_DEVERR_TIMEOUT);
      return false;
    }
  }
  return true;
}

// The GEMV input vector in shared memory, as float4 quads laid out so that every load of it is
// conflict-free: lane l's piece c = l + 32u (V floats) sits in quads xq(c, 0..V/4-1), and the quads that
// the 32 lanes read together are consecutive. For V = 4 that is the plain order; for V = 8 the two
// halves of the lanes' pieces are interleaved.
template <int V>
__device__ __forceinline__ int xq(int c, int e4) {
  return V == 4 ? c : ((c >> 5) * 2 + e4) * 32 + (c & 31);
}
// Quad i of the plain vector (elements 4i .. 4i+3) -> its slot.
template <int V>
__device__ __forceinline__ int xq_of(int i) {
  return V == 4 ? i : xq<V>(i >> 1, i & 1);
}

template <typename WT, bool ACC, bool SMEM, int NP>
__device__ __forceinline__ void gemv_rows(const WT* __restrict__ W, int rbase, const float* xs, int K, int r0, int r1,
                                          float scale, float* out, const float* add, int* err) {
  constexpr int V = Elem<WT>::kVec;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nvec = K / V;  // 16-byte pieces per row
  float xr[NP][V];
  const float4* x4 = reinterpret_cast<const float4*>(xs);
#pragma unroll
  for (int u = 0; u < NP; ++u) {
    const int c = lane + 32 * u;
#pragma unroll
    for (int e4 = 0; e4 < V / 4; ++e4) {
      const float4 q = (c < nvec) ? x4[xq<V>(c, e4)] : make_float4(0.f, 0.f, 0.f, 0.f);
      xr[u][4 * e4] = q.x;
      xr[u][4 * e4 + 1] = q.y;
      xr[u][4 * e4 + 2] = q.z;
      xr[u][4 * e4 + 3] = q.w;
    }
  }
  for (int r = r0 + warp; r < r1; r += kThreads / 32) {
    const uint4* row = reinterpret_cast<const uint4*>(W + (size_t)(r - rbase) * K);
    uint4 w[NP];
#pragma unroll
    for (int u = 0; u < NP; ++u) {
      const int c = lane + 32 * u;
      w[u] = (c < nvec) ? (SMEM ? row[c] : __ldg(row + c)) : make_uint4(0u, 0u, 0u, 0u);
    }
    float acc = 0.f;
#pragma unroll
    for (int u = 0; u < NP; ++u) acc += Elem<WT>::dot8(w[u], xr[u]);
    acc = warp_sum(acc) * scale;
    if (lane == 0 && SK_INB(r >= 0, err)) out[r] = ACC ? add[r - r0] + acc : acc;
  }
}
// Pieces per lane for a row of K elements of WT (a multiple of 32 pieces per warp pass).
template <typename WT>
__host__ __device__ constexpr int pieces_per_lane(int K) {
  return (K / Elem<WT>::kVec + 31) / 32;
}
// At most 64 floats of x per lane: K <= 2048 for bf16 and for fp32 rows.
template <typename WT>
__host__ __device__ constexpr int max_pieces() {
  return 64 / Elem<WT>::kVec;
}

// One split-KV item — keys [s0, s0 + n) of kv head kvh — on the whole CTA: the decode attention of the
// reference kernel (qwen3/kernels.py:351-413) restricted to the chunk; its partial (o, max, sum) per q
// head goes to the workspace. `phase`: the K/V bulk-copy mbarrier's parity.
struct ItemSmem {
  float q_s[kG][kHD];
  float kn_s[kHD];
  float vn_s[kHD];
  float sc[kG][kChunk];
  float o_q[3][kG][kHD];  // P·V sums of key quarters 1-3, added into quarter 0's
  float red[8][2];
  float stat[kG][2];
};

template <typename CT>
__device__ void chunk_item(const Params& p, ItemSmem& is, CT* Ks, CT* Vs, uint64_t* bar, uint32_t& phase, int kvh,
                           int split, int pos, int nsplit) {
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  const int g_t = t >> 7, d = t & (kHD - 1);  // prologue role: q head kvh·2 + g_t, dimension d
  const int T = pos + 1;
  const int s0 = split * kChunk;
  const int n = min(kChunk, T - s0);
  const bool owner = (s0 + n == T);
  const int n_ld = owner ? n - 1 : n;
  CT* Kc = reinterpret_cast<CT*>(p.Kc);
  CT* Vc = reinterpret_cast<CT*>(p.Vc);
  const size_t head_base = (size_t)kvh * p.max_len * kHD;
  if (t == kCopyThread && n_ld > 0) {
    const uint32_t bytes = (uint32_t)(n_ld * kHD * sizeof(CT));
    mbar_arrive_expect_tx(bar, 2 * bytes);
    bulk_load(Ks, Kc + head_base + (size_t)s0 * kHD, bytes, bar);
    bulk_load(Vs, Vc + head_base + (size_t)s0 * kHD, bytes, bar);
  }
  // prologue (qwen3/kernels.py:351-380): thread (g_t, d) normalises and rotates q head g_t; the chunk
  // holding the new position also normalises and rotates the new k (g_t = 0) and appends k and v
  const float c = p.rope[(size_t)pos * kHD + (d & 63)];
  const float s = p.rope[(size_t)pos * kHD + 64 + (d & 63)];
  // qkv was written by other CTAs in this launch: read through L2
  const float qv = __ldcg(p.qkv + (size_t)(kvh * kG + g_t) * kHD + d);
  const float xv = owner ? __ldcg(p.qkv + (size_t)(p.nq + g_t * p.nkv) * kHD + (size_t)kvh * kHD + d) : 0.f;
  {
    const float kv = g_t == 0 ? xv : 0.f;
    const float sq = warp_sum(qv * qv), sk = warp_sum(kv * kv);
    if (lane == 0) {
      is.red[w][0] = sq;
      is.red[w][1] = sk;
    }
    __syncthreads();
    const int w0 = g_t * 4;  // the 4 warps of this q head
    const float ssq = is.red[w0][0] + is.red[w0 + 1][0] + is.red[w0 + 2][0] + is.red[w0 + 3][0];
    const float ssk = is.red[0][1] + is.red[1][1] + is.red[2][1] + is.red[3][1];
    is.q_s[g_t][d] = qv * rsqrtf(ssq / kHD + p.eps) * p.qn[d];
    if (owner && g_t == 0) is.kn_s[d] = kv * rsqrtf(ssk / kHD + p.eps) * p.kn[d];
    __syncthreads();
    const float rot = d < 64 ? -is.q_s[g_t][d + 64] : is.q_s[g_t][d - 64];
    const float qr = (is.q_s[g_t][d] * c + rot * s) * 0.08838834764831845f;  // 1/sqrt(128), qwen3/kernels.py:378
    float knew = 0.f;
    if (owner && g_t == 0) {
      const float rk = d < 64 ? -is.kn_s[d + 64] : is.kn_s[d - 64];
      knew = is.kn_s[d] * c + rk * s;
    }
    __syncthreads();
    is.q_s[g_t][d] = qr;
    if (owner) {
      if (g_t == 0) {
        const CT kst = Elem<CT>::st(knew);
        Kc[head_base + (size_t)pos * kHD + d] = kst;  // append (qwen3/kernels.py:364,366)
        is.kn_s[d] = Elem<CT>::ld(&kst);               // attended as read back from the cache
      } else {
        const CT vst = Elem<CT>::st(xv);
        Vc[head_base + (size_t)pos * kHD + d] = vst;
        is.vn_s[d] = Elem<CT>::ld(&vst);
      }
    }
    __syncthreads();
  }
  bool ok = true;
  if (n_ld > 0) {
    ok = mbar_wait(bar, phase, p.err);
    phase ^= 1u;
  }
  // scores: warp w owns keys [16w, 16w + 16); lane owns dims [4 lane, 4 lane + 4)
  {
    float4 qa[kG];
#pragma unroll
    for (int g = 0; g < kG; ++g) qa[g] = *reinterpret_cast<const float4*>(&is.q_s[g][4 * lane]);
    const float4 knew4 = *reinterpret_cast<const float4*>(&is.kn_s[4 * lane]);
    float part[kG * 16];
#pragma unroll
    for (int jj = 0; jj < 16; ++jj) {
      const int j = 16 * w + jj;
      const float4 k4 = (ok && j < n_ld) ? Elem<CT>::ld4(Ks + (size_t)j * kHD + 4 * lane) : knew4;
#pragma unroll
      for (int g = 0; g < kG; ++g)
        part[g * 16 + jj] = qa[g].x * k4.x + qa[g].y * k4.y + qa[g].z * k4.z + qa[g].w * k4.w;
    }
    // butterfly reduce-scatter: lane l ends with the warp-wide sum of value index l
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
    is.sc[g][j] = (j < n) ? part[0] : -INFINITY;
  }
  __syncthreads();
  // chunk softmax (qwen3/kernels.py:394-408): warp g handles head g, four keys per lane
  if (w < kG) {
    const int g = w;
    float v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) v[u] = is.sc[g][lane + 32 * u];
    const float m = warp_max(fmaxf(fmaxf(v[0], v[1]), fmaxf(v[2], v[3])));
    float l = 0.f;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      v[u] = (lane + 32 * u < n) ? expf(v[u] - m) : 0.f;
      is.sc[g][lane + 32 * u] = v[u];
      l += v[u];
    }
    l = warp_sum(l);
    if (lane == 0) {
      is.stat[g][0] = m;
      is.stat[g][1] = l;
    }
  }
  __syncthreads();
  // P·V: thread owns dims (2 (t % 64), +1) over key quarter t / 64
  const int dp = 2 * (t & 63), kq = t >> 6;
  float acc[kG][2] = {};
  {
    const int j0 = kq * 32, j1 = min(j0 + 32, n);
#pragma unroll 8
    for (int j = j0; j < j1; ++j) {
      float v0, v1;
      if (ok && j < n_ld) {
        v0 = Elem<CT>::ld(Vs + (size_t)j * kHD + dp);
        v1 = Elem<CT>::ld(Vs + (size_t)j * kHD + dp + 1);
      } else {
        v0 = is.vn_s[dp];
        v1 = is.vn_s[dp + 1];
      }
#pragma unroll
      for (int g = 0; g < kG; ++g) {
        const float pr = is.sc[g][j];
        acc[g][0] += pr * v0;
        acc[g][1] += pr * v1;
      }
    }
    if (kq > 0) {
#pragma unroll
      for (int g = 0; g < kG; ++g) {
        is.o_q[kq - 1][g][dp] = acc[g][0];
        is.o_q[kq - 1][g][dp + 1] = acc[g][1];
      }
    }
  }
  __syncthreads();
  // the chunk's partial: o (summed over the four quarters, in order), max, sum per q head
  float* pp = p.part + ((size_t)kvh * nsplit + split) * kPartFloats;
  if (kq == 0) {
#pragma unroll
    for (int g = 0; g < kG; ++g) {
      const float o0 = ((acc[g][0] + is.o_q[0][g][dp]) + is.o_q[1][g][dp]) + is.o_q[2][g][dp];
      const float o1 = ((acc[g][1] + is.o_q[0][g][dp + 1]) + is.o_q[1][g][dp + 1]) + is.o_q[2][g][dp + 1];
      *reinterpret_cast<float2*>(pp + g * (kHD + 2) + dp) = make_float2(o0, o1);
    }
  }
  if (t < kG * 2) pp[(t >> 1) * (kHD + 2) + kHD + (t & 1)] = is.stat[t >> 1][t & 1];
  __syncthreads();  // the shared buffers are reused by the next item
}

// gemv_rows with the register slice of x sized for K (the host checks K <= 32 · 64).
template <typename WT, bool ACC, bool SMEM>
__device__ __forceinline__ void gemv_dispatch(const WT* W, int rbase, const float* xs, int K, int r0, int r1,
                                              float scale, float* out, const float* add, int* err) {
  const int np = pieces_per_lane<WT>(K);
  if (np <= 1)
    gemv_rows<WT, ACC, SMEM, 1>(W, rbase, xs, K, r0, r1, scale, out, add, err);
  else if (np <= 2)
    gemv_rows<WT, ACC, SMEM, 2>(W, rbase, xs, K, r0, r1, scale, out, add, err);
  else if (np <= 4)
    gemv_rows<WT, ACC, SMEM, 4>(W, rbase, xs, K, r0, r1, scale, out, add, err);
  else if (np <= 8 || max_pieces<WT>() <= 8)
    gemv_rows<WT, ACC, SMEM, 8>(W, rbase, xs, K, r0, r1, scale, out, add, err);
  else
    gemv_rows<WT, ACC, SMEM, max_pieces<WT>()>(W, rbase, xs, K, r0, r1, scale, out, add, err);
}

// Shared-memory plan (dynamic part):
//   [0, w)           STAGE: this CTA's W_qkv rows (phase 1), then its W_o rows from offset 0 (phase 3)
//   [w, w + kv)      the K/V chunk of the current attention item (phase 2)
//   [wo, wo + part)  phase 3: every chunk partial of every kv head, over the dead tail of the W area and
//                    the K/V area (wo = the W_o rows' bytes; 0 without STAGE)
//   [x_off, + x)     the GEMV input vector (x in phase 1, att in phase 3), in the quad layout of xq
// Without STAGE the GEMVs read their rows from L2 (after the bulk prefetch) and w = wo = 0.
struct Plan {
  size_t w, kv, wo, part, x_off, bytes;
};
template <typename WT, typename CT, bool STAGE>
__host__ __device__ inline Plan plan_of(int hidden, int nq, int nkv, int max_len, int G) {
  const int nrow1 = (nq + 2 * nkv) * kHD, K3 = nq * kHD;
  const size_t per1 = (size_t)((nrow1 + G - 1) / G), per3 = (size_t)((hidden + G - 1) / G);
  auto al = [](size_t b) { return (b + 127) & ~(size_t)127; };
  Plan pl;
  pl.w = STAGE ? al(std::max(per1 * hidden, per3 * K3) * sizeof(WT)) : 0;
  pl.kv = 2 * (size_t)kChunk * kHD * sizeof(CT);
  pl.wo = STAGE ? al(per3 * K3 * sizeof(WT)) : 0;
  pl.part = al((size_t)nkv * nsplit_of(max_len) * kPartFloats * 4);
  pl.x_off = std::max(pl.w + pl.kv, pl.wo + pl.part);
  // the quad layout of the GEMV input spans whole 32-piece groups
  pl.bytes = pl.x_off + (((size_t)std::max(hidden, K3) + 255) & ~(size_t)255) * 4;
  return pl;
}

template <typename WT, typename CT, bool EARLY, bool STAGE>
__global__ void __launch_bounds__(kThreads, 1) decode_block_kernel(const Params p) {
  extern __shared__ __align__(128) unsigned char dsmem[];
  __shared__ ItemSmem is;
  __shared__ __align__(8) uint64_t bars[3];  // the K/V chunk; the staged weight rows; the partials
  __shared__ float red_s[kThreads / 32];
  __shared__ float coef[16][kMaxSplits];     // phase 3: merge weight of chunk c for q head qh (nq <= 16)
  __shared__ float h_rows[64];               // this CTA's rows of h as phase 1 read them (phase 3 adds to them)
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = gridDim.x, cta = blockIdx.x;
  const int nrow1 = (p.nq + 2 * p.nkv) * kHD, nrow3 = p.hidden, K3 = p.nq * kHD;
  const int per1 = (nrow1 + G - 1) / G, per3 = (nrow3 + G - 1) / G;
  const int r10 = min(nrow1, cta * per1), r11 = min(nrow1, r10 + per1);
  const int r30 = min(nrow3, cta * per3), r31 = min(nrow3, r30 + per3);
  const WT* wq = reinterpret_cast<const WT*>(p.w_qkv);
  const WT* wo = reinterpret_cast<const WT*>(p.w_o);
  const int nsplit = nsplit_of(p.max_len);
  const Plan pl = plan_of<WT, CT, STAGE>(p.hidden, p.nq, p.nkv, p.max_len, G);
  WT* ws = reinterpret_cast<WT*>(dsmem);
  CT* Ks = reinterpret_cast<CT*>(dsmem + pl.w);
  CT* Vs = Ks + (size_t)kChunk * kHD;
  float* ps = reinterpret_cast<float*>(dsmem + pl.wo);
  float* xs = reinterpret_cast<float*>(dsmem + pl.x_off);
  const uint32_t wq_bytes = (uint32_t)((size_t)(r11 - r10) * p.hidden * sizeof(WT));
  const uint32_t wo_bytes = (uint32_t)((size_t)(r31 - r30) * K3 * sizeof(WT));
  if (tid == 0) {
#pragma unroll
    for (int i = 0; i < 3; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (tid == kCopyThread) {
    // the W_qkv rows depend on nothing the launch or the kernel before it computes: fetch them now
    if (STAGE) {
      if (wq_bytes) {
        mbar_arrive_expect_tx(&bars[1], wq_bytes);
        bulk_load(ws, wq + (size_t)r10 * p.hidden, wq_bytes, &bars[1]);
      } else {
        mbar_arrive(&bars[1]);
      }
    } else {
      prefetch_range(wq + (size_t)r10 * p.hidden, wq_bytes);
    }
  }
  int pos = 0;
  auto read_pos = [&]() { pos = (p.pos_ptr ? (int)p.pos_ptr[0] : 0) + p.pos_add; };
  if (EARLY) read_pos();  // the position and this layer's cache rows are not written by the kernel just before
  __syncthreads();
  griddep_wait();
  griddep_launch_dependents();
  __shared__ unsigned n0_s;
  if (tid == 0) n0_s = ld_acquire_gpu(p.sync);  // the barriers completed before this launch
  if (!EARLY) read_pos();
  if (pos < 0 || pos >= p.max_len) {  // every CTA reads the same position: all leave here
    if (cta == 0 && tid == 0) set_dev_error(p.err, SK_DEVERR_POS_RANGE);
    if (STAGE && tid == kCopyThread) mbar_wait(&bars[1], 0, p.err);  // no copy outlives the CTA
    return;
  }
  const int active = pos / kChunk + 1;  // chunks per kv head

  // ---- phase 1: qkv = W_qkv · (h ⊙ in_norm) · 1/rms(h) -------------------------------------------
  {
    float ss = 0.f;
    for (int i = tid * 4; i < p.hidden; i += kThreads * 4) {
      const float4 a = __ldcg(reinterpret_cast<const float4*>(p.h + i));  // written by the launch before
      const float4 b = *reinterpret_cast<const float4*>(p.in_norm + i);
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (i + e >= r30 && i + e < r31) h_rows[i + e - r30] = (&a.x)[e];
      ss += a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w;
      reinterpret_cast<float4*>(xs)[xq_of<Elem<WT>::kVec>(i >> 2)] = make_float4(a.x * b.x, a.y * b.y, a.z * b.z,
                                                                                  a.w * b.w);
    }
    ss = warp_sum(ss);
    if (lane == 0) red_s[warp] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < kThreads / 32; ++i) tot += red_s[i];
    const float inv = rsqrtf(tot / p.hidden + p.eps_in);
    const bool landed = STAGE ? mbar_wait(&bars[1], 0, p.err) : true;
    if (tid == kCopyThread) {
      // the W_qkv rows are in: now let the W_o rows and this CTA's K/V chunks stream into L2 while the
      // GEMVs run (earlier they would only slow down the rows phase 1 waits for)
      prefetch_range(wo + (size_t)r30 * K3, wo_bytes);
      for (int item = cta; item < active * p.nkv; item += G) {
        const int split = item / p.nkv, kvh = item % p.nkv;
        const int n = min(kChunk, pos + 1 - split * kChunk);
        const size_t off = ((size_t)kvh * p.max_len + (size_t)split * kChunk) * kHD;
        prefetch_range(reinterpret_cast<const CT*>(p.Kc) + off, (size_t)n * kHD * sizeof(CT));
        prefetch_range(reinterpret_cast<const CT*>(p.Vc) + off, (size_t)n * kHD * sizeof(CT));
      }
    }
    if (STAGE) {
      if (landed) gemv_dispatch<WT, false, true>(ws, r10, xs, p.hidden, r10, r11, inv, p.qkv, nullptr, p.err);
    } else {
      gemv_dispatch<WT, false, false>(wq, 0, xs, p.hidden, r10, r11, inv, p.qkv, nullptr, p.err);
    }
  }
  __syncthreads();  // every row of W_qkv read; the CTA's qkv rows written
  if (tid == 0) red_s[0] = grid_barrier_k(p.sync, n0_s, 0, p.err) ? 1.f : 0.f;
  if (STAGE && tid == kCopyThread) {  // the W_o rows into the W area, from L2 by now
    if (wo_bytes) {
      mbar_arrive_expect_tx(&bars[1], wo_bytes);
      bulk_load(ws, wo + (size_t)r30 * K3, wo_bytes, &bars[1]);
    } else {
      mbar_arrive(&bars[1]);
    }
  }
  __syncthreads();
  if (red_s[0] == 0.f) {
    if (STAGE && tid == kCopyThread) mbar_wait(&bars[1], 1, p.err);
    return;
  }

  // ---- phase 2: split-KV attention, one item (128-key chunk, kv head) per CTA ---------------------
  {
    uint32_t phase = 0;
    // items ordered chunk-major (item = split · nkv + kvh), so that the live items spread over the SMs
    for (int item = cta; item < active * p.nkv; item += G)
      chunk_item<CT>(p, is, Ks, Vs, &bars[0], phase, item % p.nkv, item / p.nkv, pos, nsplit);
  }
  __syncthreads();
  if (tid == 0) red_s[0] = grid_barrier_k(p.sync, n0_s, 1, p.err) ? 1.f : 0.f;
  __syncthreads();
  if (red_s[0] == 0.f) {
    if (STAGE && tid == kCopyThread) mbar_wait(&bars[1], 1, p.err);
    return;
  }
  if (tid == kCopyThread) {
    // every chunk partial of every kv head (visible: the barrier's acquire came before) into shared
    // memory, one bulk copy per head
    const uint32_t per_head = (uint32_t)(active * kPartFloats * 4);
    mbar_arrive_expect_tx(&bars[2], per_head * p.nkv);
    for (int kvh = 0; kvh < p.nkv; ++kvh)
      bulk_load(ps + (size_t)kvh * active * kPartFloats, p.part + (size_t)kvh * nsplit * kPartFloats, per_head,
                &bars[2]);
  }

  // ---- phase 3: att = merge of the partials; h += W_o · att -----------------------------------------
  {
    const bool got = mbar_wait(&bars[2], 0, p.err);
    // merge weights: for q head qh (kv head qh / 2, part g = qh % 2) and chunk c, exp(m_c - M) / Σ w·l
    for (int qh = warp; qh < p.nq; qh += kThreads / 32) {
      const float* base = ps + (size_t)(qh / kG) * active * kPartFloats + (qh % kG) * (kHD + 2);
      float M = -INFINITY;
      for (int c = lane; c < active; c += 32) M = fmaxf(M, base[(size_t)c * kPartFloats + kHD]);
      M = warp_max(M);
      float den = 0.f;
      for (int c = lane; c < active; c += 32) {
        const float wgt = expf(base[(size_t)c * kPartFloats + kHD] - M);
        coef[qh][c] = wgt;
        den += wgt * base[(size_t)c * kPartFloats + kHD + 1];
      }
      den = warp_sum(den);
      __syncwarp();
      for (int c = lane; c < active; c += 32) coef[qh][c] /= den;
    }
    __syncthreads();
    // att[qh][d] = Σ_c coef[qh][c] · o_c[d], chunks in order, into the quad layout of the GEMV input:
    // thread (g, d) = (tid / 128, tid % 128) takes the q heads qh = 2j + g of every kv head j, the chunk
    // loop outermost so that its nkv sums are independent chains
    if (got) {
      const int d = tid & (kHD - 1), g = tid >> 7;
      float a[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) a[j] = 0.f;
      for (int c = 0; c < active; ++c) {
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (j < p.nkv) a[j] += coef[2 * j + g][c] * ps[((size_t)j * active + c) * kPartFloats + g * (kHD + 2) + d];
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int i = (2 * j + g) * kHD + d;
        if (j < p.nkv) xs[xq_of<Elem<WT>::kVec>(i >> 2) * 4 + (i & 3)] = a[j];
      }
    }
    __syncthreads();
    if (STAGE) {
      if (mbar_wait(&bars[1], 1, p.err) && got)
        gemv_dispatch<WT, true, true>(ws, r30, xs, K3, r30, r31, 1.f, p.h, h_rows, p.err);
    } else if (got) {
      gemv_dispatch<WT, true, false>(wo, 0, xs, K3, r30, r31, 1.f, p.h, h_rows, p.err);
    }
  }
}

constexpr size_t kSmemLimit = 227 * 1024 - sizeof(ItemSmem) - 16 * kMaxSplits * 4 - 1024;  // dynamic share

template <typename WT, typename CT, bool EARLY, bool STAGE>
static int launch_with(const Params& p, int G, size_t smem, cudaStream_t st) {
  auto kern = decode_block_kernel<WT, CT, EARLY, STAGE>;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return SK_ERR_CUDA;
  static std::mutex mu;
  static size_t set_to[64] = {};
  {
    std::lock_guard<std::mutex> lk(mu);
    if (set_to[dev] < smem) {
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return SK_ERR_CUDA;
      set_to[dev] = smem;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(G);  // one CTA per SM, all resident (cooperative)
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeCooperative;
  at[0].val.cooperative = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 2;
  if (cudaLaunchKernelEx(&cfg, kern, p) != cudaSuccess) return SK_ERR_CUDA;
  return cudaPeekAtLastError() == cudaSuccess ? SK_OK : SK_ERR_CUDA;
}

template <typename WT, typename CT>
static int launch(const Params& p, bool early, cudaStream_t st) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return SK_ERR_CUDA;
  static int sm[64] = {};
  if (dev < 0 || dev >= 64) return SK_ERR_CUDA;
  if (!sm[dev] && cudaDeviceGetAttribute(&sm[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return SK_ERR_CUDA;
  const int G = sm[dev];
  if ((p.hidden + G - 1) / G > 64) return SK_ERR_UNSUPPORTED;                     // h rows kept per CTA
  // stage the weight rows in shared memory where they fit (bf16 weights at the talker's widths)
  const Plan staged = plan_of<WT, CT, true>(p.hidden, p.nq, p.nkv, p.max_len, G);
  if (staged.bytes <= kSmemLimit)
    return early ? launch_with<WT, CT, true, true>(p, G, staged.bytes, st)
                 : launch_with<WT, CT, false, true>(p, G, staged.bytes, st);
  const Plan plain = plan_of<WT, CT, false>(p.hidden, p.nq, p.nkv, p.max_len, G);
  if (plain.bytes > kSmemLimit) return SK_ERR_UNSUPPORTED;
  return early ? launch_with<WT, CT, true, false>(p, G, plain.bytes, st)
               : launch_with<WT, CT, false, false>(p, G, plain.bytes, st);
}

}  // namespace block
}  // namespace sk

extern "C" size_t sk_decode_block_workspace_bytes(int max_len, int nq, int nkv, int hd) {
  if (max_len <= 0 || nq <= 0 || nkv <= 0 || hd != sk::block::kHD) return 0;
  return sk::block::ws_bytes(nq, nkv, max_len);
}

extern "C" int sk_decode_attention_block(float* h, const float* in_norm, float eps_in, const void* w_qkv,
                                         const float* qn, const float* kn, float eps, const float* rope, void* Kc,
                                         void* Vc, const long long* pos_ptr, int pos_add, int max_len, int nq,
                                         int nkv, int hd, const void* w_o, int hidden, int weight_dtype,
                                         int cache_dtype, void* workspace, size_t ws_bytes, int flags,
                                         void* stream) {
  using namespace sk::block;
  if (flags & ~SK_DECODE_KV_STABLE) return SK_ERR_INVALID_ARG;
  if (!h || !in_norm || !w_qkv || !qn || !kn || !rope || !Kc || !Vc || !w_o) return SK_ERR_INVALID_ARG;
  if (max_len <= 0 || nkv <= 0 || nq <= 0 || hidden <= 0) return SK_ERR_INVALID_ARG;
  if (hd != kHD || nq != kG * nkv) return SK_ERR_UNSUPPORTED;  // qwen3/kernels.py:457
  if (nq > 16) return SK_ERR_UNSUPPORTED;                      // the merge weights of up to 16 q heads
  if (cache_dtype != SK_BF16 && cache_dtype != SK_F32) return SK_ERR_UNSUPPORTED;
  if (weight_dtype != SK_BF16 && weight_dtype != SK_F32) return SK_ERR_UNSUPPORTED;
  if (hidden % 8 || nsplit_of(max_len) > kMaxSplits) return SK_ERR_UNSUPPORTED;
  // both GEMVs keep a lane's slice of their input vector (at most 64 floats) in registers
  if (hidden > 32 * 64 || nq * kHD > 32 * 64) return SK_ERR_UNSUPPORTED;
  if (!workspace || ws_bytes < sk::block::ws_bytes(nq, nkv, max_len)) return SK_ERR_WORKSPACE;
  const uintptr_t al = reinterpret_cast<uintptr_t>(h) | reinterpret_cast<uintptr_t>(in_norm) |
                       reinterpret_cast<uintptr_t>(w_qkv) | reinterpret_cast<uintptr_t>(w_o) |
                       reinterpret_cast<uintptr_t>(Kc) | reinterpret_cast<uintptr_t>(Vc) |
                       reinterpret_cast<uintptr_t>(workspace);
  if (al & 15) return SK_ERR_INVALID_ARG;
  int rc = sk_check_device();
  if (rc != SK_OK) return rc;
  int* err = sk_error_word_ptr();
  if (!err) return SK_ERR_CUDA;
  char* ws = reinterpret_cast<char*>(workspace);
  Params p{};
  p.h = h;
  p.in_norm = in_norm;
  p.eps_in = eps_in;
  p.w_qkv = w_qkv;
  p.qn = qn;
  p.kn = kn;
  p.eps = eps;
  p.rope = rope;
  p.Kc = Kc;
  p.Vc = Vc;
  p.pos_ptr = pos_ptr;
  p.pos_add = pos_add;
  p.max_len = max_len;
  p.nq = nq;
  p.nkv = nkv;
  p.hidden = hidden;
  p.w_o = w_o;
  p.sync = reinterpret_cast<unsigned*>(ws);
  p.qkv = reinterpret_cast<float*>(ws + kSyncBytes);
  p.att = p.qkv + (size_t)(nq + 2 * nkv) * kHD;
  p.part = p.att + (size_t)nq * kHD;
  p.err = err;
  const bool early = (flags & SK_DECODE_KV_STABLE) != 0;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (weight_dtype == SK_BF16)
    return cache_dtype == SK_BF16 ? launch<__nv_bfloat16, __nv_bfloat16>(p, early, st)
                                  : launch<__nv_bfloat16, float>(p, early, st);
  return cache_dtype == SK_BF16 ? launch<float, __nv_bfloat16>(p, early, st) : launch<float, float>(p, early, st);
}
