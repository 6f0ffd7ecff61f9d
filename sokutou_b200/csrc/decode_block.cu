// Qwen3-TTS talker decode: one layer's whole attention block in one launch —
//   qkv = W_qkv · RMSNorm(h)        (the reference's rms_gemv, qwen3/kernels.py:271-275)
//   att = attention(qkv, caches)    (the reference's attn, qwen3/kernels.py:341-414: QK-RMSNorm, RoPE,
//                                    KV append, GQA over T = pos + 1 keys)
//   h  += W_o · att                 (the reference's gemv with accumulate, qwen3/kernels.py:301-305)
// which the reference runs as three launches per layer (qwen3/kernels.py:619-624).
//
// Each of the three steps needs the whole output of the one before, so the launch is cooperative: one
// CTA per SM, all resident, with two grid-wide barriers between the phases (a counter and a generation
// word in the caller's workspace; bounded spins that record SK_DEVERR_TIMEOUT and give up after 2 s).
// The weights of both projections do not depend on anything computed in the launch, so every CTA asks
// for its slices of W_qkv and W_o to be brought into L2 (bulk prefetch) before it waits for the kernel
// ahead of it; the ~25 MB of a 1.7B-class layer's weights then stream from HBM while the phases run,
// and each phase reads its rows from L2.
//
//   phase 1  rows of W_qkv split evenly over the CTAs; a warp per row, 16-byte loads, x = h ⊙ in_norm
//            in shared memory, the RMS scale applied to the dot product (as the reference does).
//   phase 2  split-KV attention: items (64-key chunk, kv head), each on one half of a CTA (128 threads,
//            its own named barrier and bulk-copy mbarrier), partials (o, max, sum) into the workspace;
//            the last item of a head to finish merges the head's partials (deterministic order) into
//            att. No float atomics anywhere, so the fp32 mode is reproducible run to run.
//   phase 3  rows of W_o split evenly over the CTAs, att in shared memory, h[r] += the dot product.
#include <mutex>

#include "sk_common.cuh"

namespace sk {
namespace block {

constexpr int kHD = 128, kG = 2, kChunk = 64, kThreads = 256, kHalf = 128;
constexpr int kMaxSplits = 256;

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
  unsigned* sync;           // workspace: [0] barrier count, [1] generation, [2 + kvh] merge counters
  int* err;
};

__host__ __device__ inline int nsplit_of(int max_len) { return (max_len + kChunk - 1) / kChunk; }
constexpr size_t kSyncBytes = 256;
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

// Grid-wide barrier over all CTAs of the (cooperative) launch: count arrivals in sync[0]; the last
// arrival resets the count and advances the generation sync[1], which the others wait on. The words
// are back in their resting state (count 0) after every barrier, so no reset between launches or graph
// replays is needed. A wait that runs out records SK_DEVERR_TIMEOUT; the caller then unwinds.
__device__ __forceinline__ bool grid_barrier(unsigned* sync, int* err) {
  __syncthreads();
  __shared__ int ok_s;
  if (threadIdx.x == 0) {
    bool ok = true;
    volatile unsigned* gen = sync + 1;
    const unsigned g0 = *gen;
    __threadfence();  // this CTA's writes before the arrival
    if (atomicAdd(sync, 1u) == gridDim.x - 1) {
      *sync = 0;
      __threadfence();
      atomicAdd(sync + 1, 1u);
    } else {
      const uint64_t t0 = globaltimer_ns();
      // 148 threads polling one line would crowd out the last arrival's atomics: poll every ~64 ns
      for (uint32_t i = 0; *gen == g0; ++i) {
        __nanosleep(64);
        if ((i & 255u) == 255u && globaltimer_ns() - t0 > kWaitLimitNs) {
          set_dev_error(err, SK_DEVERR_TIMEOUT);
          ok = false;
          break;
        }
      }
    }
    __threadfence();  // the other CTAs' writes after it
    ok_s = ok;
  }
  __syncthreads();
  return ok_s != 0;
}

// out[r] (op)= scale · Σ_k W[r][k] x[k] for rows r in [r0, r1); row r of W starts at W + (r - rbase)·K.
// One warp per row, lane l over the 16-byte pieces l, l + 32, ... of the row. Every row meets the same x,
// so a lane loads its pieces of x into registers once (NP pieces of V floats; K <= 32·NP·V) and the row
// loop reads only W — no shared-memory bank conflicts on x. SMEM: W is a staged copy in shared memory
// (plain loads); else W is global (read-only path), all of a lane's loads issued before they are used.
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
                                          float scale, float* out, int* err) {
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
    if (lane == 0 && SK_INB(r >= 0, err)) {
      if (ACC)
        out[r] = __ldcg(out + r) + acc;
      else
        out[r] = acc;
    }
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

// One split-KV item — keys [s0, s0 + n) of kv head kvh — on one half of the CTA (128 threads, named
// barrier `bar`): the decode attention of the reference kernel (qwen3/kernels.py:351-413) restricted to
// the chunk, its partial (o, max, sum) to the workspace; the last chunk of the head to finish merges
// them into att. `phase`: this half's bulk-copy mbarrier parity.
// 16-byte aligned (q_s and kn_s are read as float4): the second half's copy must start on a 16-byte
// boundary too.
template <typename CT>
struct __align__(16) HalfSmem {
  float q_s[kG][kHD];
  float kn_s[kHD];
  float vn_s[kHD];
  float sc[kG][kChunk];
  float o_half[kG][kHD];
  float red[4][4];
  float stat[kG][2];
  float mg[kMaxSplits * kG];
  float lg[kMaxSplits * kG];
  int is_last;
};

template <typename CT>
__device__ void chunk_item(const Params& p, HalfSmem<CT>& hs, CT* Ks, CT* Vs, uint64_t* bar, uint32_t& phase,
                           int bar_id, int kvh, int split, int pos, int nsplit) {
  const int t = threadIdx.x & (kHalf - 1), lane = t & 31, w = t >> 5;
  auto hsync = [&]() { named_bar_sync(bar_id, kHalf); };
  const int T = pos + 1;
  const int active = (T + kChunk - 1) / kChunk;
  const int s0 = split * kChunk;
  const int n = min(kChunk, T - s0);
  const bool owner = (s0 + n == T);
  const int n_ld = owner ? n - 1 : n;
  CT* Kc = reinterpret_cast<CT*>(p.Kc);
  CT* Vc = reinterpret_cast<CT*>(p.Vc);
  const size_t head_base = (size_t)kvh * p.max_len * kHD;
  if (t == 0 && n_ld > 0) {
    const uint32_t bytes = (uint32_t)(n_ld * kHD * sizeof(CT));
    mbar_arrive_expect_tx(bar, 2 * bytes);
    bulk_load(Ks, Kc + head_base + (size_t)s0 * kHD, bytes, bar);
    bulk_load(Vs, Vc + head_base + (size_t)s0 * kHD, bytes, bar);
  }
  // prologue (qwen3/kernels.py:351-380): thread t owns dimension d = t of both q heads and the new k/v
  const int d = t;
  const float c = p.rope[(size_t)pos * kHD + (d & 63)];
  const float s = p.rope[(size_t)pos * kHD + 64 + (d & 63)];
  float qv[kG];
  // qkv was written by other CTAs in this launch: read through L2
#pragma unroll
  for (int g = 0; g < kG; ++g) qv[g] = __ldcg(p.qkv + (size_t)(kvh * kG + g) * kHD + d);
  const float kv = owner ? __ldcg(p.qkv + (size_t)p.nq * kHD + (size_t)kvh * kHD + d) : 0.f;
  const float vv = owner ? __ldcg(p.qkv + (size_t)(p.nq + p.nkv) * kHD + (size_t)kvh * kHD + d) : 0.f;
  {
    float ss[kG + 1];
#pragma unroll
    for (int g = 0; g < kG; ++g) ss[g] = warp_sum(qv[g] * qv[g]);
    ss[kG] = warp_sum(kv * kv);
    if (lane == 0) {
#pragma unroll
      for (int g = 0; g <= kG; ++g) hs.red[w][g] = ss[g];
    }
    hsync();
#pragma unroll
    for (int g = 0; g <= kG; ++g) ss[g] = hs.red[0][g] + hs.red[1][g] + hs.red[2][g] + hs.red[3][g];
#pragma unroll
    for (int g = 0; g < kG; ++g) hs.q_s[g][d] = qv[g] * rsqrtf(ss[g] / kHD + p.eps) * p.qn[d];
    if (owner) hs.kn_s[d] = kv * rsqrtf(ss[kG] / kHD + p.eps) * p.kn[d];
    hsync();
    float qr[kG];
#pragma unroll
    for (int g = 0; g < kG; ++g) {
      const float rot = d < 64 ? -hs.q_s[g][d + 64] : hs.q_s[g][d - 64];
      qr[g] = (hs.q_s[g][d] * c + rot * s) * 0.08838834764831845f;  // 1/sqrt(128), qwen3/kernels.py:378
    }
    float knew = 0.f;
    if (owner) {
      const float rot = d < 64 ? -hs.kn_s[d + 64] : hs.kn_s[d - 64];
      knew = hs.kn_s[d] * c + rot * s;
    }
    hsync();
#pragma unroll
    for (int g = 0; g < kG; ++g) hs.q_s[g][d] = qr[g];
    if (owner) {
      const CT kst = Elem<CT>::st(knew), vst = Elem<CT>::st(vv);
      Kc[head_base + (size_t)pos * kHD + d] = kst;  // append (qwen3/kernels.py:364,366)
      Vc[head_base + (size_t)pos * kHD + d] = vst;
      hs.kn_s[d] = Elem<CT>::ld(&kst);              // attended as read back from the cache
      hs.vn_s[d] = Elem<CT>::ld(&vst);
    }
    hsync();
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
    for (int g = 0; g < kG; ++g) qa[g] = *reinterpret_cast<const float4*>(&hs.q_s[g][4 * lane]);
    const float4 knew4 = *reinterpret_cast<const float4*>(&hs.kn_s[4 * lane]);
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
    hs.sc[g][j] = (j < n) ? part[0] : -INFINITY;
  }
  hsync();
  // chunk softmax (qwen3/kernels.py:394-408): warp g handles head g
  if (w < kG) {
    const int g = w;
    float a = hs.sc[g][lane], b = hs.sc[g][lane + 32];
    const float m = warp_max(fmaxf(a, b));
    a = (lane < n) ? expf(a - m) : 0.f;
    b = (lane + 32 < n) ? expf(b - m) : 0.f;
    hs.sc[g][lane] = a;
    hs.sc[g][lane + 32] = b;
    const float l = warp_sum(a + b);
    if (lane == 0) {
      hs.stat[g][0] = m;
      hs.stat[g][1] = l;
    }
  }
  hsync();
  // P·V: thread owns dims (2 (t % 64), +1) over key half t / 64
  float acc[kG][2] = {};
  const int dp = 2 * (t & 63), kh = t >> 6;
  {
    const int j0 = kh * 32, j1 = min(j0 + 32, n);
    for (int j = j0; j < j1; ++j) {
      float v0, v1;
      if (ok && j < n_ld) {
        v0 = Elem<CT>::ld(Vs + (size_t)j * kHD + dp);
        v1 = Elem<CT>::ld(Vs + (size_t)j * kHD + dp + 1);
      } else {
        v0 = hs.vn_s[dp];
        v1 = hs.vn_s[dp + 1];
      }
#pragma unroll
      for (int g = 0; g < kG; ++g) {
        const float pr = hs.sc[g][j];
        acc[g][0] += pr * v0;
        acc[g][1] += pr * v1;
      }
    }
    if (kh == 1) {
#pragma unroll
      for (int g = 0; g < kG; ++g) {
        hs.o_half[g][dp] = acc[g][0];
        hs.o_half[g][dp + 1] = acc[g][1];
      }
    }
    hsync();
    if (kh == 0) {
#pragma unroll
      for (int g = 0; g < kG; ++g) {
        acc[g][0] += hs.o_half[g][dp];
        acc[g][1] += hs.o_half[g][dp + 1];
      }
    }
  }
  // publish the chunk partial; the last chunk of this kv head to arrive merges
  const size_t slot = (size_t)kvh * nsplit + split;
  float* pp = p.part + slot * kG * (kHD + 2);
  if (t < 64) {
#pragma unroll
    for (int g = 0; g < kG; ++g)
      *reinterpret_cast<float2*>(pp + g * (kHD + 2) + dp) = make_float2(acc[g][0], acc[g][1]);
  }
  if (t < kG * 2) pp[(t >> 1) * (kHD + 2) + kHD + (t & 1)] = hs.stat[t >> 1][t & 1];
  __threadfence();
  hsync();
  if (t == 0) hs.is_last = (atomicAdd(&p.sync[2 + kvh], 1u) == (unsigned)active - 1);
  hsync();
  if (!hs.is_last) return;
  __threadfence();
  for (int i = t; i < active * kG; i += kHalf) {
    const float* q = p.part + ((size_t)kvh * nsplit + i / kG) * kG * (kHD + 2) + (i % kG) * (kHD + 2);
    hs.mg[i] = __ldcg(q + kHD);
    hs.lg[i] = __ldcg(q + kHD + 1);
  }
  hsync();
  if (w < kG) {  // warp g: global max and denominator of head g, one weight per chunk
    const int g = w;
    float M = -INFINITY;
    for (int sp = lane; sp < active; sp += 32) M = fmaxf(M, hs.mg[sp * kG + g]);
    M = warp_max(M);
    float den = 0.f;
    for (int sp = lane; sp < active; sp += 32) {
      const float f = expf(hs.mg[sp * kG + g] - M);
      hs.mg[sp * kG + g] = f;
      den += f * hs.lg[sp * kG + g];
    }
    den = warp_sum(den);
    if (lane == 0) hs.stat[g][1] = den;
  }
  hsync();
  {
    float num[kG] = {};
    const float* ob = p.part + (size_t)kvh * nsplit * kG * (kHD + 2) + d;
    int sp = 0;
    for (; sp + 8 <= active; sp += 8) {  // eight chunks' partials in flight at once
      float v[8][kG];
#pragma unroll
      for (int u = 0; u < 8; ++u)
#pragma unroll
        for (int g = 0; g < kG; ++g) v[u][g] = __ldcg(ob + ((size_t)(sp + u) * kG + g) * (kHD + 2));
#pragma unroll
      for (int u = 0; u < 8; ++u)
#pragma unroll
        for (int g = 0; g < kG; ++g) num[g] += hs.mg[(sp + u) * kG + g] * v[u][g];
    }
    for (; sp < active; ++sp)
#pragma unroll
      for (int g = 0; g < kG; ++g)
        num[g] += hs.mg[sp * kG + g] * __ldcg(ob + ((size_t)sp * kG + g) * (kHD + 2));
#pragma unroll
    for (int g = 0; g < kG; ++g)
      if (SK_INB(kvh * kG + g < p.nq, p.err)) p.att[(size_t)(kvh * kG + g) * kHD + d] = num[g] / hs.stat[g][1];
  }
  if (t == 0) p.sync[2 + kvh] = 0;  // ready for the next call (and graph replay)
}

// gemv_rows with the register slice of x sized for K (the host checks K <= 32 · 64).
template <typename WT, bool ACC, bool SMEM>
__device__ __forceinline__ void gemv_dispatch(const WT* W, int rbase, const float* xs, int K, int r0, int r1,
                                              float scale, float* out, int* err) {
  const int np = pieces_per_lane<WT>(K);
  if (np <= 1)
    gemv_rows<WT, ACC, SMEM, 1>(W, rbase, xs, K, r0, r1, scale, out, err);
  else if (np <= 2)
    gemv_rows<WT, ACC, SMEM, 2>(W, rbase, xs, K, r0, r1, scale, out, err);
  else if (np <= 4)
    gemv_rows<WT, ACC, SMEM, 4>(W, rbase, xs, K, r0, r1, scale, out, err);
  else if (np <= 8 || max_pieces<WT>() <= 8)
    gemv_rows<WT, ACC, SMEM, 8>(W, rbase, xs, K, r0, r1, scale, out, err);
  else
    gemv_rows<WT, ACC, SMEM, max_pieces<WT>()>(W, rbase, xs, K, r0, r1, scale, out, err);
}

// Shared-memory plan. STAGE (bf16 weights whose slices fit): [W slice: the larger of this CTA's W_qkv
// and W_o rows][K/V chunks of the two halves][x or att floats]; the W_qkv rows come in by one bulk copy
// issued before the wait for the kernel ahead, the W_o rows (prefetched to L2 meanwhile) by a second one
// into the same area once phase 1 has read it. Without STAGE the GEMVs read their rows from L2 (after
// the bulk prefetch) and only the K/V chunks and x / att live in shared memory.
struct Plan {
  size_t w_off, kv_off, x_off, bytes;
};
template <typename WT, typename CT, bool STAGE>
__host__ __device__ inline Plan plan_of(int hidden, int nq, int nkv, int G) {
  const int nrow1 = (nq + 2 * nkv) * kHD, K3 = nq * kHD;
  const size_t per1 = (size_t)((nrow1 + G - 1) / G), per3 = (size_t)((hidden + G - 1) / G);
  const size_t w = STAGE ? ((std::max(per1 * hidden, per3 * K3) * sizeof(WT) + 127) & ~(size_t)127) : 0;
  const size_t kv = 2 * 2 * (size_t)kChunk * kHD * sizeof(CT);
  // the quad layout of the GEMV input spans whole 32-piece groups
  const size_t x = (((size_t)std::max(hidden, K3) + 255) & ~(size_t)255) * 4;
  return Plan{0, w, w + kv, w + kv + x};
}

template <typename WT, typename CT, bool EARLY, bool STAGE>
__global__ void __launch_bounds__(kThreads, 1) decode_block_kernel(const Params p) {
  extern __shared__ __align__(128) unsigned char dsmem[];
  __shared__ HalfSmem<CT> hsm[2];
  static_assert(sizeof(HalfSmem<CT>) % 16 == 0, "each half's shared block must keep 16-byte alignment");
  __shared__ __align__(8) uint64_t bars[3];  // K/V chunk of half 0, of half 1; the staged weight rows
  __shared__ float red_s[kThreads / 32];
  const int tid = threadIdx.x, half = tid / kHalf;
  const int G = gridDim.x, cta = blockIdx.x;
  const int nrow1 = (p.nq + 2 * p.nkv) * kHD, nrow3 = p.hidden, K3 = p.nq * kHD;
  const int per1 = (nrow1 + G - 1) / G, per3 = (nrow3 + G - 1) / G;
  const int r10 = min(nrow1, cta * per1), r11 = min(nrow1, r10 + per1);
  const int r30 = min(nrow3, cta * per3), r31 = min(nrow3, r30 + per3);
  const WT* wq = reinterpret_cast<const WT*>(p.w_qkv);
  const WT* wo = reinterpret_cast<const WT*>(p.w_o);
  const Plan pl = plan_of<WT, CT, STAGE>(p.hidden, p.nq, p.nkv, G);
  WT* ws = reinterpret_cast<WT*>(dsmem + pl.w_off);
  float* xs = reinterpret_cast<float*>(dsmem + pl.x_off);
  const uint32_t wq_bytes = (uint32_t)((size_t)(r11 - r10) * p.hidden * sizeof(WT));
  const uint32_t wo_bytes = (uint32_t)((size_t)(r31 - r30) * K3 * sizeof(WT));
  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    mbar_init(&bars[2], 1);
    fence_mbar_init();
    // the weights depend on nothing the launch or the kernel before it computes: fetch them now
    if (STAGE) {
      if (wq_bytes) {
        mbar_arrive_expect_tx(&bars[2], wq_bytes);
        bulk_load(ws, wq + (size_t)r10 * p.hidden, wq_bytes, &bars[2]);
      } else {
        mbar_arrive(&bars[2]);
      }
    } else {
      prefetch_range(wq + (size_t)r10 * p.hidden, wq_bytes);
    }
    prefetch_range(wo + (size_t)r30 * K3, wo_bytes);
  }
  const int nsplit = nsplit_of(p.max_len);
  int pos = 0;
  auto read_pos = [&]() { pos = (p.pos_ptr ? (int)p.pos_ptr[0] : 0) + p.pos_add; };
  if (EARLY) {  // the position and this layer's cache rows are not written by the kernel just before
    read_pos();
    if (tid == 0 && pos >= 0 && pos < p.max_len) {  // the K/V chunks of this CTA's attention items
      const int active = pos / kChunk + 1;
      for (int item = cta; item < active * p.nkv; item += G) {
        const int split = item / p.nkv, kvh = item % p.nkv;
        const int n = min(kChunk, pos + 1 - split * kChunk);
        const size_t off = ((size_t)kvh * p.max_len + (size_t)split * kChunk) * kHD;
        prefetch_range(reinterpret_cast<const CT*>(p.Kc) + off, (size_t)n * kHD * sizeof(CT));
        prefetch_range(reinterpret_cast<const CT*>(p.Vc) + off, (size_t)n * kHD * sizeof(CT));
      }
    }
  }
  __syncthreads();
  griddep_wait();
  griddep_launch_dependents();
  if (!EARLY) read_pos();
  if (pos < 0 || pos >= p.max_len) {  // every CTA reads the same position: all leave here
    if (cta == 0 && tid == 0) set_dev_error(p.err, SK_DEVERR_POS_RANGE);
    if (STAGE && tid == 0) mbar_wait(&bars[2], 0, p.err);  // no copy outlives the CTA
    return;
  }

  // ---- phase 1: qkv = W_qkv · (h ⊙ in_norm) · 1/rms(h) -------------------------------------------
  {
    float ss = 0.f;
    for (int i = tid * 4; i < p.hidden; i += kThreads * 4) {
      const float4 a = __ldcg(reinterpret_cast<const float4*>(p.h + i));  // written by the launch before
      const float4 b = *reinterpret_cast<const float4*>(p.in_norm + i);
      ss += a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w;
      reinterpret_cast<float4*>(xs)[xq_of<Elem<WT>::kVec>(i >> 2)] = make_float4(a.x * b.x, a.y * b.y, a.z * b.z,
                                                                                  a.w * b.w);
    }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red_s[tid >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < kThreads / 32; ++i) tot += red_s[i];
    const float inv = rsqrtf(tot / p.hidden + p.eps_in);
    if (STAGE) {
      const bool landed = mbar_wait(&bars[2], 0, p.err);
      if (landed) gemv_dispatch<WT, false, true>(ws, r10, xs, p.hidden, r10, r11, inv, p.qkv, p.err);
      __syncthreads();  // every row of W_qkv read: the area takes the W_o rows (already on their way to L2)
      if (tid == 0) {
        if (wo_bytes) {
          mbar_arrive_expect_tx(&bars[2], wo_bytes);
          bulk_load(ws, wo + (size_t)r30 * K3, wo_bytes, &bars[2]);
        } else {
          mbar_arrive(&bars[2]);
        }
      }
    } else {
      gemv_dispatch<WT, false, false>(wq, 0, xs, p.hidden, r10, r11, inv, p.qkv, p.err);
    }
  }
  if (!grid_barrier(p.sync, p.err)) {
    if (STAGE && tid == 0) mbar_wait(&bars[2], 1, p.err);
    return;
  }

  // ---- phase 2: split-KV attention, one item per CTA half ------------------------------------------
  {
    const int active = pos / kChunk + 1;
    const size_t kv_elems = (size_t)kChunk * kHD;
    CT* Ks = reinterpret_cast<CT*>(dsmem + pl.kv_off) + (size_t)half * 2 * kv_elems;
    CT* Vs = Ks + kv_elems;
    uint32_t phase = 0;
    // items ordered chunk-major (item = split · nkv + kvh), half 0 of every CTA first, so that the live
    // items of short caches spread over all SMs
    for (int item = half * G + cta; item < active * p.nkv; item += 2 * G)
      chunk_item<CT>(p, hsm[half], Ks, Vs, &bars[half], phase, 1 + half, item % p.nkv, item / p.nkv, pos, nsplit);
  }
  if (!grid_barrier(p.sync, p.err)) {
    if (STAGE && tid == 0) mbar_wait(&bars[2], 1, p.err);
    return;
  }

  // ---- phase 3: h += W_o · att ------------------------------------------------------------------------
  {
    for (int i = tid * 4; i < K3; i += kThreads * 4)
      reinterpret_cast<float4*>(xs)[xq_of<Elem<WT>::kVec>(i >> 2)] = __ldcg(reinterpret_cast<const float4*>(p.att + i));
    __syncthreads();
    if (STAGE) {
      if (mbar_wait(&bars[2], 1, p.err))
        gemv_dispatch<WT, true, true>(ws, r30, xs, K3, r30, r31, 1.f, p.h, p.err);
    } else {
      gemv_dispatch<WT, true, false>(wo, 0, xs, K3, r30, r31, 1.f, p.h, p.err);
    }
  }
}

constexpr size_t kSmemLimit = 227 * 1024 - sizeof(HalfSmem<float>) * 2 - 1024;  // dynamic share of the 227 KB

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
  // stage the weight rows in shared memory where they fit (bf16 weights at the talker's widths)
  const Plan staged = plan_of<WT, CT, true>(p.hidden, p.nq, p.nkv, G);
  if (staged.bytes <= kSmemLimit)
    return early ? launch_with<WT, CT, true, true>(p, G, staged.bytes, st)
                 : launch_with<WT, CT, false, true>(p, G, staged.bytes, st);
  const Plan plain = plan_of<WT, CT, false>(p.hidden, p.nq, p.nkv, G);
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
  if (cache_dtype != SK_BF16 && cache_dtype != SK_F32) return SK_ERR_UNSUPPORTED;
  if (weight_dtype != SK_BF16 && weight_dtype != SK_F32) return SK_ERR_UNSUPPORTED;
  if (hidden % 8 || nsplit_of(max_len) > kMaxSplits || nkv > (int)(kSyncBytes / 4) - 2) return SK_ERR_UNSUPPORTED;
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
