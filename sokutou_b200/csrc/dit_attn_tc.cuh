// Shared pieces of the tensor-core DiT attention (dit_attn_tc.cu): the tile sizes, the warp roles and
// register split, the per-hd ring depths, the kernel parameters, the softmax row arithmetic on a row of
// S held in registers, and the operands' tensor maps.
#pragma once

#include "sk_common.cuh"

namespace sk {
namespace dit {
constexpr int kBM = 128, kBN = 128;
constexpr int kThreadsTC = 384;  // 2 softmax warpgroups + a warpgroup holding the producer and MMA warps
constexpr int kWarpProducer = 8, kWarpMma = 9, kWarpPv = 10;  // TMA producer, S = Q·Kᵀ issuer, P·V issuer
// Register split (setmaxnreg): launched at 168 per thread (384 x 168 = 64512); the producer/MMA
// warpgroup gives registers back, the softmax warpgroups take them: 256 x 232 + 128 x 40 = 64512.
constexpr int kLaunchRegs = 168, kSoftmaxRegs = 232, kControlRegs = 40;
static_assert(256 * kSoftmaxRegs + 128 * kControlRegs <= kThreadsTC * kLaunchRegs, "register split over budget");
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleLog2 = 8.0f;  // rescale O when the running max grows by more than 2^8
constexpr int kMaxLiveTiles = 64;     // key tiles per CTA up to which fully masked tiles are skipped
constexpr int kWarpScan = 11;         // the masked-tile scan (SKIP launches)


template <int HD>
struct TcCfg;
template <>
struct TcCfg<64> {  // 16 + 6*16 + 6*16 = 208 KB
  static constexpr int NSK = 6, NSV = 6;
  static constexpr int T_P = 384;  // P0 at 384, P1 at 448
};
template <>
struct TcCfg<128> {  // 32 + 3*32 + 3*32 = 224 KB
  static constexpr int NSK = 3, NSV = 3;
  static constexpr int T_P = 0;    // P_w overlays S_w
};

// Key tiles always run, masked or not: every latent tile and at least the first NSK (the producer and
// the MMA issuer start on these before the masked-tile scan has finished). The rest are the SKIP
// candidates: in the engine's CFG batches the conditioning tiles, whole text tiles masked in the
// text-uncond row and whole speaker tiles in the speaker-uncond row (engine/bucket.py:252-258).
template <int HD>
__host__ __device__ constexpr int head_tiles(int n_lat, int ntiles) {
  return n_lat > TcCfg<HD>::NSK ? (n_lat < ntiles ? n_lat : ntiles) : (TcCfg<HD>::NSK < ntiles ? TcCfg<HD>::NSK : ntiles);
}


struct TcParams {
  const void* bias;      // bf16 additive key bias or nullptr
  long long bias_bs;     // elements between bias rows
  void* y;               // bf16 (B, L, H, hd)
  int H, L, Lk, S;
  float scale_log2;      // softmax scale * log2(e)
  int ctx_batched;       // 1: ctx map has a batch coordinate
  int* err;
  int D;                 // H * hd (fused block: v and gate column offsets in o4)
  int kv_group;          // query heads per key/value head (1 for the DiT; 2 for the Qwen3 GQA prefill)
  int q_pos0;            // causal form: absolute position of query row 0 (key j is visible to row p if j <= p)
};

__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }


// 2^x for two values on the FMA pipe (for a share of the softmax exponentials, so that they do not all
// queue on the 16-per-clock MUFU unit): x = n + f with n = round(x) (adding 1.5·2^23 rounds x into the
// low mantissa bits), 2^f on [-0.5, 0.5] by the cubic 1 + f·(c1 + f·(c2 + f·c3)) whose coefficients
// minimise the maximum relative error there (1.0e-4, found by reweighted least squares on Chebyshev
// points; P is rounded to bf16 afterwards, 3.9e-3), and n added to the exponent field. x is clamped at
// -127: then n = -127, f = 0 and the result is exactly +0, as ex2.approx gives for a masked key.
__device__ __forceinline__ float2 exp2_fma_pair(float2 x) {
  x.x = fmaxf(x.x, -127.f);
  x.y = fmaxf(x.y, -127.f);
  const float2 t = __fadd2_rn(x, make_float2(12582912.f, 12582912.f));
  const float2 n = __fadd2_rn(t, make_float2(-12582912.f, -12582912.f));
  const float2 f = __ffma2_rn(n, make_float2(-1.f, -1.f), x);
  float2 p = __ffma2_rn(make_float2(0.05500893f, 0.05500893f), f, make_float2(0.24221095f, 0.24221095f));
  p = __ffma2_rn(p, f, make_float2(0.6932829f, 0.6932829f));
  p = __ffma2_rn(p, f, make_float2(1.f, 1.f));
  return make_float2(__uint_as_float(__float_as_uint(p.x) + (__float_as_uint(t.x) << 23)),
                     __uint_as_float(__float_as_uint(p.y) + (__float_as_uint(t.y) << 23)));
}
// Exponential pairs per 4 (of each 8 keys) computed by exp2_fma_pair: 1 of 4 (a quarter of them)
// measured fastest on B200 — MUFU then carries 3/4 of the load, the FP32 pipe the rest; at half the
// extra FMA-pipe instructions cost more than the MUFU time saved.
constexpr int kFmaExpPairs = 1;

__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* src, int x, int y, int z, int w) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z), "r"(w)
               : "memory");
}
__device__ __forceinline__ void tma_store_commit_and_wait_read() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

// Key bias of column `col` of key tile j as raw bf16 bits: 0xff80 (-inf) past the end of its segment,
// 0 without a bias. Loaded a tile ahead and converted only where it is stored, so no arithmetic waits
// for the load inside the tile that issues it.
__device__ __forceinline__ uint32_t tile_bias_bits(const TcParams& prm, const __nv_bfloat16* bias, int b, int nb,
                                                   int j, int n_lat, int col) {
  int key = -1;
  if (j < n_lat) {
    const int kk = j * kBN + col;
    key = kk < prm.Lk ? kk : -1;
  } else {
    const int kk = (j - n_lat) * kBN + col;
    key = kk < prm.S ? prm.Lk + kk : -1;
  }
  if (key < 0) return 0xff80u;
  if (!SK_INB(key < prm.Lk + prm.S && b < nb, prm.err)) return 0u;
  if (!bias) return 0u;
  // issued here, where the program puts it: a plain load may be sunk by the scheduler towards its use
  // a tile later, exposing the whole L2 round trip at the top of that tile
  unsigned short v;
  asm volatile("ld.global.nc.u16 %0, [%1];"
               : "=h"(v)
               : "l"(reinterpret_cast<const unsigned short*>(bias) + (size_t)b * prm.bias_bs + key));
  return v;
}


// ---- softmax row arithmetic (thread = TMEM lane = query row; x holds the row's 128 scores) ----------
// x = s·scale·log2e + bias·log2e in place (packed fp32x2 FMAs, the bias of each key from bt); returns
// the row max (four independent chains of 3-input max).
__device__ __forceinline__ float scale_bias_rowmax(float (&x)[kBN], const float* bt, float2 sl2) {
  float mt0 = -INFINITY, mt1 = -INFINITY, mt2 = -INFINITY, mt3 = -INFINITY;
  const float4* bt4 = reinterpret_cast<const float4*>(bt);
#pragma unroll
  for (int c = 0; c < kBN; c += 8) {
    const float4 ba = bt4[c >> 2], bb = bt4[(c >> 2) + 1];
    const float2 t0 = __ffma2_rn(make_float2(x[c], x[c + 1]), sl2, make_float2(ba.x, ba.y));
    const float2 t1 = __ffma2_rn(make_float2(x[c + 2], x[c + 3]), sl2, make_float2(ba.z, ba.w));
    const float2 t2 = __ffma2_rn(make_float2(x[c + 4], x[c + 5]), sl2, make_float2(bb.x, bb.y));
    const float2 t3 = __ffma2_rn(make_float2(x[c + 6], x[c + 7]), sl2, make_float2(bb.z, bb.w));
    x[c] = t0.x;
    x[c + 1] = t0.y;
    x[c + 2] = t1.x;
    x[c + 3] = t1.y;
    x[c + 4] = t2.x;
    x[c + 5] = t2.y;
    x[c + 6] = t3.x;
    x[c + 7] = t3.y;
    mt0 = max3(mt0, t0.x, t0.y);
    mt1 = max3(mt1, t1.x, t1.y);
    mt2 = max3(mt2, t2.x, t2.y);
    mt3 = max3(mt3, t3.x, t3.y);
  }
  return fmaxf(fmaxf(mt0, mt1), fmaxf(mt2, mt3));
}

// x = 2^(x - m) for all 128 keys in place: independent, so the MUFU pipe stays fed; kFmaExpPairs of
// every four pairs on the FMA pipe.
__device__ __forceinline__ void exp2_row(float (&x)[kBN], float m_use) {
  const float2 nm = make_float2(-m_use, -m_use);
#pragma unroll
  for (int c = 0; c < kBN; c += 8) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 dd = __fadd2_rn(make_float2(x[c + 2 * e], x[c + 2 * e + 1]), nm);
      const float2 pe = (e < kFmaExpPairs) ? exp2_fma_pair(dd) : make_float2(ex2_approx(dd.x), ex2_approx(dd.y));
      x[c + 2 * e] = pe.x;
      x[c + 2 * e + 1] = pe.y;
    }
  }
}

// The row sum of x (two chains) and the row's bf16 pairs written into 64 tensor-memory columns at tP,
// 32 columns per tcgen05.st (lane = row; keys 2c, 2c+1 the low and high halves of column c). The
// caller waits for the stores (tcgen05.wait::st) before it signals P.
__device__ __forceinline__ float pack_p_row(const float (&x)[kBN], uint32_t tP) {
  float2 ls0 = make_float2(0.f, 0.f), ls1 = ls0;
#pragma unroll
  for (int h32 = 0; h32 < 2; ++h32) {
    uint32_t pk[32];
#pragma unroll
    for (int e = 0; e < 32; ++e) {
      const float2 p = make_float2(x[64 * h32 + 2 * e], x[64 * h32 + 2 * e + 1]);
      if (e & 1)
        ls1 = __fadd2_rn(ls1, p);
      else
        ls0 = __fadd2_rn(ls0, p);
      const __nv_bfloat162 pb2 = __floats2bfloat162_rn(p.x, p.y);
      pk[e] = *reinterpret_cast<const uint32_t*>(&pb2);
    }
    tmem_st32(tP + 32 * h32, reinterpret_cast<const float*>(pk));
  }
  return (ls0.x + ls0.y) + (ls1.x + ls1.y);
}

// The O row (HD fp32 columns at tO, lane = row) multiplied by alpha in tensor memory.
template <int HD>
__device__ __forceinline__ void rescale_o_row(uint32_t tO, float alpha) {
#pragma unroll
  for (int c = 0; c < HD / 32; ++c) {
    float ov[32];
    tmem_ld32(tO + c * 32, ov);
    tmem_wait_ld();
#pragma unroll
    for (int e = 0; e < 32; ++e) ov[e] *= alpha;
    tmem_st32(tO + c * 32, ov);
  }
  tmem_wait_st();
}

// ---- host: tensor maps of the attention operands ----------------------------------------------------
// q (B·H, L, hd) with boxes of 128 rows x 64 columns; latent k/v (B·H / kv_group heads, Lk rows
// kv_rows apart); conditioning k/v (batch, S, H, hd), the batch coordinate 0 when the rows share one
// buffer. Maps of operands that are absent alias mq (never read); need_v = false leaves mv to the caller.
template <int HD>
static inline int make_operand_maps(const void* q, const void* k_lat, const void* v_lat, const void* k_ctx,
                                    const void* v_ctx, long long ctx_bs, const TcParams& prm, int B, int kv_rows,
                                    CUtensorMap* mq, CUtensorMap* mk, CUtensorMap* mv, CUtensorMap* mkc,
                                    CUtensorMap* mvc, bool need_v = true) {
  const int H = prm.H, L = prm.L, Lk = prm.Lk, S = prm.S;
  {
    cuuint64_t dims[3] = {(cuuint64_t)HD, (cuuint64_t)L, (cuuint64_t)B * H};
    cuuint64_t str[2] = {(cuuint64_t)HD * 2, (cuuint64_t)L * HD * 2};
    cuuint32_t box[3] = {64, kBM, 1};
    if (!sk_make_map_bf16(mq, q, 3, dims, str, box)) return SK_ERR_CUDA;
  }
  if (Lk > 0) {
    const long long rows = kv_rows > 0 ? kv_rows : Lk;
    cuuint64_t dims[3] = {(cuuint64_t)HD, (cuuint64_t)Lk, (cuuint64_t)B * (H / prm.kv_group)};
    cuuint64_t str[2] = {(cuuint64_t)HD * 2, (cuuint64_t)rows * HD * 2};
    cuuint32_t box[3] = {64, kBN, 1};
    if (!sk_make_map_bf16(mk, k_lat, 3, dims, str, box)) return SK_ERR_CUDA;
    if (need_v && !sk_make_map_bf16(mv, v_lat, 3, dims, str, box)) return SK_ERR_CUDA;
    if (!need_v) *mv = *mq;
  } else {
    *mk = *mq;
    *mv = *mq;
  }
  if (S > 0) {
    cuuint64_t dims[4] = {(cuuint64_t)HD, (cuuint64_t)H, (cuuint64_t)S, (cuuint64_t)(prm.ctx_batched ? B : 1)};
    cuuint64_t str[3] = {(cuuint64_t)HD * 2, (cuuint64_t)H * HD * 2,
                         (cuuint64_t)(prm.ctx_batched ? ctx_bs * 2 : (long long)S * H * HD * 2)};
    cuuint32_t box[4] = {64, 1, kBN, 1};
    if (!sk_make_map_bf16(mkc, k_ctx, 4, dims, str, box) || !sk_make_map_bf16(mvc, v_ctx, 4, dims, str, box))
      return SK_ERR_CUDA;
  } else {
    *mkc = *mq;
    *mvc = *mq;
  }
  return SK_OK;
}

}  // namespace dit
}  // namespace sk
