// DiT attention, fp32 mode: fp32 loads, fp32 FMA on the CUDA cores, expf — the correctness mode
// (the reference's fp32 engine path runs SDPA in fp32, engine/fast.py:169-173). Tensor cores cannot
// hold the 1e-5 relative bar, so this kernel trades speed for accuracy.
//
// CTA = 32 query rows of one (batch, head); 4 threads per row, each owning HD/4 dimensions as
// float4 chunks interleaved across the quad (chunk index quad + 4*i) so that the quad reads one
// contiguous 64-byte span of a shared-memory row. Keys stream in tiles of 32 through shared memory;
// online softmax per row.
#include "sk_common.cuh"

namespace sk {
namespace dit {

struct KeySrc {
  const float* lat;   // (B, H / group, rows, HD): latent keys 0..Lk-1 of each key/value head
  const float* ctx;   // (S, H, HD) per batch row
  long long ctx_bs;   // elements between ctx batch rows (0 = shared)
  int Lk, S;
  int group = 1;      // query heads per key/value head (2: the Qwen3 GQA prefill)
  int rows = 0;       // rows per key/value head in `lat` (0: Lk)
  int causal = 0;     // 1: key j visible to query row p only if j <= pos0 + p (the Qwen3 prefill)
  int pos0 = 0;
};

template <int HD>
__global__ void __launch_bounds__(128) attn_f32_kernel(const float* __restrict__ q, KeySrc ks, KeySrc vs,
                                                        const float* __restrict__ bias, long long bias_bs,
                                                        float* __restrict__ y, int H, int L, float scale,
                                                        int* err) {
  constexpr int BQ = 32, BK = 32, NC = HD / 16;  // NC float4 chunks per thread
  __shared__ __align__(16) float Ks[BK][HD];
  __shared__ __align__(16) float Vs[BK][HD];
  __shared__ float bs[BK];
  const int b = blockIdx.z, h = blockIdx.y, q0 = blockIdx.x * BQ;
  const int t = threadIdx.x, row = t >> 2, quad = t & 3;
  const int qi = q0 + row;
  // causal: no key past the CTA's last query row is visible to any of its rows
  const int K = ks.causal ? min(ks.Lk + ks.S, ks.pos0 + q0 + BQ) : ks.Lk + ks.S;
  const int kvh = h / ks.group, kv_rows = ks.rows > 0 ? ks.rows : ks.Lk;

  float4 qr[NC], o[NC];
#pragma unroll
  for (int i = 0; i < NC; ++i) {
    o[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    qr[i] = (qi < L) ? reinterpret_cast<const float4*>(q + (((size_t)b * H + h) * L + qi) * HD)[quad + 4 * i]
                     : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  float m = -INFINITY, l = 0.f;

  for (int k0 = 0; k0 < K; k0 += BK) {
    __syncthreads();
    for (int idx = t; idx < BK * HD / 4; idx += 128) {
      const int r = idx / (HD / 4), c4 = idx % (HD / 4), kk = k0 + r;
      float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
      if (!SK_INB(r < BK && c4 < HD / 4 && b < (int)gridDim.z && h < H, err)) continue;
      if (kk < ks.Lk) {
        const size_t off = (((size_t)b * (H / ks.group) + kvh) * kv_rows + kk) * HD;
        kv = reinterpret_cast<const float4*>(ks.lat + off)[c4];
        vv = reinterpret_cast<const float4*>(vs.lat + off)[c4];
      } else if (kk < K) {
        const size_t off = (size_t)b * ks.ctx_bs + ((size_t)(kk - ks.Lk) * H + h) * HD;
        kv = reinterpret_cast<const float4*>(ks.ctx + off)[c4];
        vv = reinterpret_cast<const float4*>(vs.ctx + off)[c4];
      }
      reinterpret_cast<float4*>(&Ks[r][0])[c4] = kv;
      reinterpret_cast<float4*>(&Vs[r][0])[c4] = vv;
    }
    if (t < BK) {
      const int kk = k0 + t;
      bs[t] = (kk >= K || !SK_INB(kk >= 0, err)) ? -INFINITY : (bias ? bias[(size_t)b * bias_bs + kk] : 0.f);
    }
    __syncthreads();
    float s[BK];
    float mt = -INFINITY;
#pragma unroll
    for (int j = 0; j < BK; ++j) {
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < NC; ++i) {
        const float4 kv = reinterpret_cast<const float4*>(&Ks[j][0])[quad + 4 * i];
        acc = fmaf(qr[i].x, kv.x, acc);
        acc = fmaf(qr[i].y, kv.y, acc);
        acc = fmaf(qr[i].z, kv.z, acc);
        acc = fmaf(qr[i].w, kv.w, acc);
      }
      acc += __shfl_xor_sync(0xffffffffu, acc, 1);
      acc += __shfl_xor_sync(0xffffffffu, acc, 2);
      s[j] = (ks.causal && k0 + j > ks.pos0 + qi) ? -INFINITY : acc * scale + bs[j];
      mt = fmaxf(mt, s[j]);
    }
    const float m_new = fmaxf(m, mt);
    const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
    const float alpha = expf(m - m_use);
    l *= alpha;
#pragma unroll
    for (int i = 0; i < NC; ++i) {
      o[i].x *= alpha;
      o[i].y *= alpha;
      o[i].z *= alpha;
      o[i].w *= alpha;
    }
#pragma unroll
    for (int j = 0; j < BK; ++j) {
      const float p = expf(s[j] - m_use);
      l += p;
#pragma unroll
      for (int i = 0; i < NC; ++i) {
        const float4 vv = reinterpret_cast<const float4*>(&Vs[j][0])[quad + 4 * i];
        o[i].x = fmaf(p, vv.x, o[i].x);
        o[i].y = fmaf(p, vv.y, o[i].y);
        o[i].z = fmaf(p, vv.z, o[i].z);
        o[i].w = fmaf(p, vv.w, o[i].w);
      }
    }
    m = m_new;
  }
  if (qi < L && SK_INB(qi >= 0 && h < H, err)) {
    const float inv = (l > 0.f) ? 1.f / l : 0.f;
    float4* yo = reinterpret_cast<float4*>(y + (((size_t)b * L + qi) * H + h) * HD);
#pragma unroll
    for (int i = 0; i < NC; ++i) yo[quad + 4 * i] = make_float4(o[i].x * inv, o[i].y * inv, o[i].z * inv, o[i].w * inv);
  }
}

}  // namespace dit
}  // namespace sk

int sk_launch_dit_attention_f32(const float* q, const float* k_lat, const float* v_lat, const float* k_ctx,
                                const float* v_ctx, const float* bias, float* y, int B, int H, int L, int Lk, int S,
                                int hd, long long ctx_bs, long long bias_bs, float scale, cudaStream_t st) {
  using namespace sk::dit;
  KeySrc ks{k_lat, k_ctx, ctx_bs, Lk, S}, vs{v_lat, v_ctx, ctx_bs, Lk, S};
  int* err = sk_error_word_ptr();
  if (!err) return SK_ERR_CUDA;
  dim3 grid((L + 31) / 32, H, B), block(128);
  if (hd == 64)
    attn_f32_kernel<64><<<grid, block, 0, st>>>(q, ks, vs, bias, bias_bs, y, H, L, scale, err);
  else
    attn_f32_kernel<128><<<grid, block, 0, st>>>(q, ks, vs, bias, bias_bs, y, H, L, scale, err);
  return cudaPeekAtLastError() == cudaSuccess ? SK_OK : SK_ERR_CUDA;
}

// The Qwen3 prefill in the fp32 mode: q (nq, T, 128), keys/values rows [0, pos0 + T) of the cache heads
// (nkv, max_len, 128), query head h on head h / 2, causal; y (T, nq, 128).
int sk_launch_prefill_attention_f32(const float* q, const float* Kc, const float* Vc, float* y, int nq, int nkv,
                                    int T, int pos0, int max_len, cudaStream_t st) {
  using namespace sk::dit;
  KeySrc ks{Kc, nullptr, 0, pos0 + T, 0, nq / nkv, max_len, 1, pos0};
  KeySrc vs{Vc, nullptr, 0, pos0 + T, 0, nq / nkv, max_len, 1, pos0};
  int* err = sk_error_word_ptr();
  if (!err) return SK_ERR_CUDA;
  dim3 grid((T + 31) / 32, nq, 1), block(128);
  attn_f32_kernel<128><<<grid, block, 0, st>>>(q, ks, vs, nullptr, 0, y, nq, T, 1.0f / sqrtf(128.f), err);
  return cudaPeekAtLastError() == cudaSuccess ? SK_OK : SK_ERR_CUDA;
}
