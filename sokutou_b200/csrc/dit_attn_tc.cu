// DiT attention, bf16 mode, on the sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// Replaces F.scaled_dot_product_attention(q, k, v, attn_mask=bias) at engine/fused.py:295.
// One CTA computes a 128-row query tile of one (batch, head) against all K = Lk + S keys, in key
// tiles of 128:
//
//   warp 8 (one lane)  TMA producer: Q once, then K_j and V_j for j = 0, 1, ... into two rings of NSK
//                      and NSV slots, each copy waiting (asleep on the slot's mbarrier) for the MMA that
//                      last read its slot. Latent keys come from (B, H, Lk, hd), conditioning keys
//                      straight from their batch-shared (S, H, hd) buffer — no per-CFG-branch copy.
//   warp 9 (one lane)  S issuer: S_j = Q·K_jᵀ into TMEM buffer S[j % 2], in order.
//   warp 10 (one lane) P·V issuer: O_w += P_j·V_j into the TMEM accumulator O[j % 2] (w = j % 2), P read
//                      from TMEM. Two issuing threads, because issuing a group of MMAs holds the thread
//                      for about the group's run time in the tensor pipe: one thread for both streams
//                      would keep a ready P·V waiting behind the next S.
//   warp 11            (SKIP launches) the scan that lists the key tiles with a live key.
//   warps 0-3, 4-7     two softmax warpgroups; warpgroup w takes the tiles j with j % 2 == w, so two
//                      tiles' softmax run at once. Thread r of a warpgroup owns query row r (TMEM lane
//                      r): it loads its S row (tcgen05.ld), applies scale and key bias (prefetched one
//                      tile ahead) with packed fp32x2 FMAs, keeps a running max in the log2 domain,
//                      exponentiates (3/4 on the MUFU unit, 1/4 by a cubic on the FMA pipe — the MUFU
//                      unit's 16 results per clock bound the softmax otherwise), writes P (bf16 pairs)
//                      back into tensor memory with tcgen05.st, and rescales its
//                      O row in TMEM only when the max grew by more than 2^8 (exact either way:
//                      numerator and denominator share the stale max).
//   epilogue           the two (max, sum, O) partials of each row are merged, O / l -> bf16 ->
//                      y (B, L, H, hd); warpgroup w writes half of the hd columns.
// Every thread executes griddepcontrol.wait before touching global memory, so with programmatic
// dependent launch a kernel's set-up (barriers, TMEM, descriptor prefetch) overlaps the tail of
// the kernel before it while every input read still follows that kernel's completion.
//
// Shared-memory operand layouts (128-byte swizzled, 1024-byte aligned, as TMA writes them):
//   Q [128 rows][hd]   K-major A of S = Q·Kᵀ      (hd split in 64-element chunks)
//   K [128 keys][hd]   K-major B of S
//   V [128 keys][hd]   MN-major B of O (hd contiguous), LBO = chunk stride, SBO = 8 rows
// Tensor memory (512 columns, one lane per query row):
//   hd = 64 :  S0 [0,128) S1 [128,256) O0 [256,320) O1 [320,384) P0 [384,448) P1 [448,512)
//   hd = 128:  S0 [0,128) S1 [128,256) O0 [256,384) O1 [384,512); P_w overlays the first 64 columns
//              of S_w, so S_{j+2} is issued only once the P·V of tile j has completed.
// P (the A operand of O += P·V): row r in lane r, keys 2c and 2c+1 as the low and high bf16 halves of
// column c.
#include <mutex>

#include "dit_attn_tc.cuh"

namespace sk {
namespace dit {

template <int HD>
struct TcLayout {
  static constexpr int NSK = TcCfg<HD>::NSK, NSV = TcCfg<HD>::NSV;
  static constexpr int NCH = HD / 64;              // 64-element (128-byte) chunks per row
  static constexpr int Q_BYTES = kBM * HD * 2;
  static constexpr int KV_BYTES = kBN * HD * 2;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + Q_BYTES;
  static constexpr int OFF_V = OFF_K + NSK * KV_BYTES;
  // the y tile is staged over the K ring once every S = Q·Kᵀ has run (the epilogue waits for the last
  // P·V, which the tensor pipe completes after every S)
  static constexpr int OFF_Y = OFF_K;
  // float [2 wg][2 buf][kBN] key bias; after its tile loop a warpgroup reuses its own 2*kBN floats
  // for the (max, sum) of its kBM rows that the epilogue exchanges
  static constexpr int OFF_BIAS = OFF_V + NSV * KV_BYTES;
  static constexpr int OFF_BAR = OFF_BIAS + 4 * kBN * 4;
  // q_full, k_full/k_empty[NSK], v_full/v_empty[NSV], s_full[2], s_free[2], p_full[2], o_done[2], mma_done,
  // for the fused block: q_free, gate_full; live_ready (SKIP: the list of key tiles to run is built)
  static constexpr int NBAR = 1 + 2 * NSK + 2 * NSV + 8 + 1 + 2 + 1;
  static constexpr int OFF_TMEM = OFF_BAR + NBAR * 8;
  // SKIP: [0, 8) bit mask of the key tiles to run, [8, 12) their count, [16, 16 + kMaxLiveTiles) the
  // tile indices in order
  static constexpr int OFF_LIVE = OFF_TMEM + 16;
  static constexpr int BYTES = OFF_LIVE + 16 + kMaxLiveTiles;
  // The dynamic shared-memory base is 1024-byte aligned on sm_100 (checked at run time); the
  // 128B-swizzled tiles need that alignment.
  static constexpr int SMEM_ALLOC = BYTES;
  static_assert(SMEM_ALLOC <= 232448, "shared memory over the 227 KB per-CTA limit");
  static_assert(2 * kBM <= 2 * kBN, "the (max, sum) exchange must fit a warpgroup's bias area");
  static_assert(NSK * KV_BYTES >= kBM * HD * 2, "the y tile must fit the K ring");
  // tensor-memory columns (relative to the allocation)
  static constexpr uint32_t T_S = 0, T_O = 256, T_P = TcCfg<HD>::T_P;
  static constexpr bool P_OVER_S = (HD == 128);
};


// FUSED = false: attention over q (B, H, L, hd), latent k/v (B, H, Lk, hd) and the ctx K/V, y (B, L, H, hd).
// FUSED = true: the attention of a DiT layer's fused block — the epilogue reads the gate tile from the
// projection rows o4 (B·L, 4·D) through tmG and writes y · sigmoid(gate). VO4 = true: the latent v
// tiles also come straight from o4 (tmV over o4) instead of the producer's (B, H, L, hd) buffer.
// CAUSAL = true: key j is visible to query row p only if j <= q_pos0 + p (the Qwen3 prefill); key tiles
// past the CTA's last row are skipped, and the tiles that straddle the diagonal are masked per element.
// SKIP = true (launched when there is a bias and more than head_tiles key tiles, at most kMaxLiveTiles):
// a key tile past the head tiles whose every key has a -inf bias adds nothing to any row and is not
// run. Warps 10-11 scan those tiles' bias at the start and publish the list of tiles to run through
// live_ready; the producer, the MMA issuer and the softmax warpgroups work on the head tiles meanwhile
// and read the list only when they get past them. Counts of tiles below are positions in that list;
// tile_bias_bits and the TMA coordinates take the key tile from it.
template <int HD, bool FUSED, bool VO4, bool CAUSAL, bool SKIP>
__global__ void __launch_bounds__(kThreadsTC, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmKc,
                   const __grid_constant__ CUtensorMap tmVc, const __grid_constant__ CUtensorMap tmY,
                   const __grid_constant__ CUtensorMap tmG,
                   const TcParams prm) {
  using Ly = TcLayout<HD>;
  constexpr int NSK = Ly::NSK, NSV = Ly::NSV;
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sbase = smem_u32(smem);
  if (sbase & 1023u) {  // uniform for the CTA, before any barrier: report and leave
    if (threadIdx.x == 0) set_dev_error(prm.err, SK_DEVERR_TIMEOUT);
    return;
  }

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Ly::OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = k_full + NSK;
  uint64_t* v_full = k_empty + NSK;
  uint64_t* v_empty = v_full + NSV;
  uint64_t* s_full = v_empty + NSV;
  uint64_t* s_free = s_full + 2;
  uint64_t* p_full = s_free + 2;
  uint64_t* o_done = p_full + 2;
  uint64_t* mma_done = o_done + 2;
  uint64_t* q_free = mma_done + 1;     // fused: every S = Q·Kᵀ done, the Q area may take the gate tile
  uint64_t* gate_full = q_free + 1;    // fused: gate tile landed
  uint64_t* live_ready = gate_full + 1;  // SKIP: the list of key tiles to run is in place
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Ly::OFF_TMEM);
  unsigned long long* live_mask = reinterpret_cast<unsigned long long*>(smem + Ly::OFF_LIVE);
  int* n_live_s = reinterpret_cast<int*>(smem + Ly::OFF_LIVE + 8);
  uint8_t* live_map = smem + Ly::OFF_LIVE + 16;
  float* bias_s = reinterpret_cast<float*>(smem + Ly::OFF_BIAS);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.z, h = blockIdx.y, q0 = blockIdx.x * kBM;
  const int n_lat_all = (prm.Lk + kBN - 1) / kBN, n_ctx = (prm.S + kBN - 1) / kBN;
  // causal: only the latent key tiles up to this CTA's last query row
  const int n_lat = CAUSAL ? min(n_lat_all, (prm.q_pos0 + q0 + kBM - 1) / kBN + 1) : n_lat_all;
  const int ntiles = n_lat + n_ctx;
  const int kHead = head_tiles<HD>(n_lat, ntiles);  // list entries below kHead are the tiles themselves

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < NSK; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < NSV; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 128);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_done[i], 1);
    }
    mbar_init(mma_done, 2);  // one commit from each MMA-issuing thread
    if (FUSED) {
      mbar_init(q_free, 1);
      mbar_init(gate_full, 1);
    }
    if (SKIP) {
      mbar_init(live_ready, 1);
      *live_mask = kHead >= 64 ? ~0ull : (1ull << kHead) - 1;  // the head tiles; the scan adds the others
    }
    fence_mbar_init();
  }
  if (warp == kWarpProducer && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    if (FUSED) tma_prefetch_desc(&tmG);
    if (n_ctx) {
      tma_prefetch_desc(&tmKc);
      tma_prefetch_desc(&tmVc);
    }
  }
  if (warp == kWarpMma) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // Inputs may come from the kernel launched before this one: wait for it, then let the next
  // kernel start its own set-up.
  griddep_wait();
  // Q and the first key tile go out before anything else: ahead of the register hand-back and the role
  // dispatch below, which held them back by ~400 cycles (measured: c1 4 %, c2 1.5 % faster per call)
  if (warp == kWarpProducer && lane == 0) {
    const int lz = b * prm.H + h, lzk = b * (prm.H / prm.kv_group) + h / prm.kv_group;
    mbar_arrive_expect_tx(q_full, Ly::Q_BYTES);
#pragma unroll
    for (int c = 0; c < Ly::NCH; ++c)
      tma_load_3d(smem + Ly::OFF_Q + c * (kBM * 128), &tmQ, q_full, c * 64, q0, lz);
    if (ntiles > 0) {
      mbar_arrive_expect_tx(&k_full[0], Ly::KV_BYTES);
      if (0 < n_lat) {
#pragma unroll
        for (int c = 0; c < Ly::NCH; ++c)
          tma_load_3d(smem + Ly::OFF_K + c * (kBN * 128), &tmK, &k_full[0], c * 64, 0, lzk);
      } else {
        const int bc = prm.ctx_batched ? b : 0;
#pragma unroll
        for (int c = 0; c < Ly::NCH; ++c)
          tma_load_4d(smem + Ly::OFF_K + c * (kBN * 128), &tmKc, &k_full[0], c * 64, h, 0, bc);
      }
    }
  }
  griddep_launch_dependents();
  const uint32_t tmem = *tmem_slot;
  // S[w] at tS + 128 w, O[w] at tO + HD w, P[w] at tP + 64 w (hd 64) or over S[w] (hd 128)
  const uint32_t tS = tmem + Ly::T_S, tO = tmem + Ly::T_O, tP = tmem + Ly::T_P;
  constexpr uint32_t kPStride = Ly::P_OVER_S ? 128 : 64;
  if (warp >= 8) {
  setmaxnreg_dec<kControlRegs>();
  if (warp == kWarpProducer) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const int bc = prm.ctx_batched ? b : 0;
      // latent tiles: (column, row, batch·head) of (B·H, L, hd) buffers; the fused block's v (and gate)
      // tiles are (column, row, batch) of o4 at column offset 2·D (3·D) plus the head's h·hd
      // k and v: the (b, h / kv_group) head of the key/value buffers (q went out after the wait)
      const int lzk = b * (prm.H / prm.kv_group) + h / prm.kv_group, lzv = VO4 ? b : lzk;
      const int xv = VO4 ? 2 * prm.D + h * HD : 0;
      if (FUSED) {  // the gate tile is loaded after the last S = Q·Kᵀ; start its trip to L2 now
#pragma unroll
        for (int c = 0; c < Ly::NCH; ++c) tma_prefetch_l2_3d(&tmG, 3 * prm.D + h * HD + c * 64, q0, b);
      }
      // K_j then V_j for list entry j = 0, 1, ... (K_0 already issued after the wait), each waiting (asleep
      // on its mbarrier) for its ring slot to be released by the MMA that last read it. SKIP: past the head
      // tiles the list must be known.
      int jk = ntiles > 0 ? 1 : 0, jv = 0;  // K_0 went out right after the wait
      bool ok = true;
      bool known = !SKIP;
      int nt = SKIP ? kHead : ntiles;
      for (int j = 0; ok; ++j) {
        if (SKIP && !known && j >= kHead) {
          if (!(ok = mbar_wait(live_ready, 0, prm.err))) break;
          known = true;
          nt = *n_live_s;
        }
        if (j >= nt) break;
        const int tj = (SKIP && j >= kHead) ? live_map[j] : j;  // key tile of list entry j
        if (j > 0) {
          const int s = j % NSK;
          if (j >= NSK && !(ok = mbar_wait(&k_empty[s], ((j / NSK) - 1) & 1, prm.err))) break;
          uint8_t* dst = smem + Ly::OFF_K + s * Ly::KV_BYTES;
          mbar_arrive_expect_tx(&k_full[s], Ly::KV_BYTES);
          if (tj < n_lat) {
#pragma unroll
            for (int c = 0; c < Ly::NCH; ++c)
              tma_load_3d(dst + c * (kBN * 128), &tmK, &k_full[s], c * 64, tj * kBN, lzk);
          } else {
#pragma unroll
            for (int c = 0; c < Ly::NCH; ++c)
              tma_load_4d(dst + c * (kBN * 128), &tmKc, &k_full[s], c * 64, h, (tj - n_lat) * kBN, bc);
          }
          jk = j + 1;
        }
        {
          const int s = j % NSV;
          if (j >= NSV && !(ok = mbar_wait(&v_empty[s], ((j / NSV) - 1) & 1, prm.err))) break;
          uint8_t* dst = smem + Ly::OFF_V + s * Ly::KV_BYTES;
          mbar_arrive_expect_tx(&v_full[s], Ly::KV_BYTES);
          if (tj < n_lat) {
#pragma unroll
            for (int c = 0; c < Ly::NCH; ++c)
              tma_load_3d(dst + c * (kBN * 128), &tmV, &v_full[s], xv + c * 64, tj * kBN, lzv);
          } else {
#pragma unroll
            for (int c = 0; c < Ly::NCH; ++c)
              tma_load_4d(dst + c * (kBN * 128), &tmVc, &v_full[s], c * 64, h, (tj - n_lat) * kBN, bc);
          }
          jv = j + 1;
        }
      }
      // fused: the gate tile goes where Q was, once no MMA reads Q any more (a blocking wait: the
      // softmax warps sharing this sub-partition keep its issue slots)
      bool gate_issued = false;
      if (FUSED && ok && mbar_wait(q_free, 0, prm.err)) {
        mbar_arrive_expect_tx(gate_full, Ly::Q_BYTES);
#pragma unroll
        for (int c = 0; c < Ly::NCH; ++c)
          tma_load_3d(smem + Ly::OFF_Q + c * (kBM * 128), &tmG, gate_full, 3 * prm.D + h * HD + c * 64, q0, b);
        gate_issued = true;
      }
      // Keep shared memory alive until every copy issued has landed (already true on the normal path).
      mbar_wait(q_full, 0, prm.err);
      if (FUSED && gate_issued) mbar_wait(gate_full, 0, prm.err);
      for (int j = (jk > NSK ? jk - NSK : 0); j < jk; ++j) mbar_wait(&k_full[j % NSK], (j / NSK) & 1, prm.err);
      for (int j = (jv > NSV ? jv - NSV : 0); j < jv; ++j) mbar_wait(&v_full[j % NSV], (j / NSV) & 1, prm.err);
    }
  } else if (warp == kWarpMma || warp == kWarpPv) {
    // ------------------------------------------------------------------ MMA issuers
    // Two threads issue tcgen05.mma: warp 9 every S = Q·Kᵀ, warp 10 every O += P·V. The issue of a group
    // of MMAs (and its commit) holds the issuing thread for about the group's run time in the tensor
    // pipe, so one thread doing both would hold a ready P·V behind the next S, and the reverse. Each
    // thread commits its own completion barriers; the tensor pipe interleaves the two streams.
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16_f32(kBM, kBN, 0, 0);
      constexpr uint32_t idO = idesc_bf16_f32(kBM, HD, 0, 1);
      const uint32_t aQ = sbase + Ly::OFF_Q, aK = sbase + Ly::OFF_K, aV = sbase + Ly::OFF_V;
      bool ok = true;
      // SKIP: list entries known to exist — the head tiles until the list is published
      bool known = !SKIP;
      int nt = SKIP ? kHead : ntiles;
      auto know = [&](int j) -> bool {  // is it settled whether list entry j exists?
        if (SKIP && !known && j >= kHead) {
          if (!mbar_wait(live_ready, 0, prm.err)) return false;
          known = true;
          nt = *n_live_s;
        }
        return true;
      };
      if (warp == kWarpMma) {
        // S_j = Q·K_jᵀ into S[j % 2]: K_j landed, S[j % 2] loaded by the softmax of entry j-2 and, where P
        // overlays S, the P·V of entry j-2 complete. Frees the K slot.
        ok = mbar_wait(q_full, 0, prm.err);
        for (int j = 0; ok; ++j) {
          if (!(ok = know(j))) break;
          if (j >= nt) break;
          const int w = j & 1, slot = j % NSK;
          if (!(ok = mbar_wait(&k_full[slot], (j / NSK) & 1, prm.err))) break;
          if (j >= 2 && !(ok = mbar_wait(&s_free[w], ((j - 2) >> 1) & 1, prm.err))) break;
          if (Ly::P_OVER_S && j >= 2 && !(ok = mbar_wait(&o_done[w], ((j - 2) >> 1) & 1, prm.err))) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            const uint32_t off = (kk >> 2) * (kBM * 128) + (kk & 3) * 32;
            tc_mma_ss(tS + w * 128, smem_desc_sw128(aQ + off, 16, 1024),
                      smem_desc_sw128(aK + slot * Ly::KV_BYTES + off, 16, 1024), idS, kk > 0);
          }
          tc_commit(&s_full[w]);
          tc_commit(&k_empty[slot]);
        }
        if (FUSED) tc_commit(q_free);  // every S issued: Q is read by no further MMA once they complete
      } else {
        // O_w += P_j·V_j (w = j % 2), P read from tensor memory: P_j written and V_j landed. Frees the V slot.
        for (int j = 0; ok; ++j) {
          if (!(ok = know(j))) break;
          if (j >= nt) break;
          const int w = j & 1, sv = j % NSV;
          if (!(ok = mbar_wait(&p_full[w], (j >> 1) & 1, prm.err))) break;
          if (!(ok = mbar_wait(&v_full[sv], (j / NSV) & 1, prm.err))) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < kBN / 16; ++kk)
            tc_mma_ts(tO + w * HD, tP + w * kPStride + kk * 8,
                      smem_desc_sw128(aV + sv * Ly::KV_BYTES + kk * 2048, kBN * 128, 1024), idO, (j >= 2 || kk > 0));
          tc_commit(&o_done[w]);
          tc_commit(&v_empty[sv]);
        }
      }
      // both threads: every MMA this CTA issued has completed before TMEM is released
      tc_commit(mma_done);
      mbar_wait(mma_done, 0, prm.err);
    }
  } else if (SKIP && warp == kWarpScan) {
    // ------------------------------------------------------------------ masked-tile scan (warp 11)
    // tiles kHead, kHead + 1, ... two at a time, lane l testing keys l, l + 32, l + 64, l + 96 of each:
    // 16-bit loads compared with the bits of a bf16 -inf (0xff80), so a tile runs if any key's bias is
    // anything else (NaN included, as in the softmax). Integer work on few registers, so that all eight
    // loads of a lane are in flight together.
    const unsigned short* brow = reinterpret_cast<const unsigned short*>(prm.bias) + (size_t)b * prm.bias_bs;
    for (int j0 = kHead; j0 < ntiles; j0 += 2) {
      unsigned short bits[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int j = j0 + (e >> 2), col = lane + 32 * (e & 3);
        // key of column col of tile j: latent keys [0, Lk), then the conditioning keys [Lk, Lk + S)
        const int kk = j < n_lat ? j * kBN + col : (j - n_lat) * kBN + col;
        const bool in = j < ntiles && (j < n_lat ? kk < prm.Lk : kk < prm.S);
        const int key = j < n_lat ? kk : prm.Lk + kk;
        bits[e] = (in && SK_INB(key < prm.Lk + prm.S, prm.err)) ? __ldg(brow + key) : (unsigned short)0xff80u;
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const bool any = (bits[4 * u] != 0xff80u) | (bits[4 * u + 1] != 0xff80u) | (bits[4 * u + 2] != 0xff80u) |
                         (bits[4 * u + 3] != 0xff80u);
        if (__any_sync(0xffffffffu, any) && lane == 0) atomicOr(live_mask, 1ull << (j0 + u));
      }
    }
    __syncwarp();
    {  // the list: tiles with their bit set (the head tiles among them), in order
      const unsigned long long mk = *reinterpret_cast<volatile unsigned long long*>(live_mask);
      const unsigned lo = (unsigned)mk, hi = (unsigned)(mk >> 32);
      const unsigned below = (1u << lane) - 1u;
      if ((lo >> lane) & 1u) live_map[__popc(lo & below)] = (uint8_t)lane;
      if ((hi >> lane) & 1u) live_map[__popc(lo) + __popc(hi & below)] = (uint8_t)(lane + 32);
      __syncwarp();
      if (lane == 0) {
        *n_live_s = __popc(lo) + __popc(hi);
        mbar_arrive(live_ready);
      }
    }
  }
  } else {
    // ------------------------------------------------------------------ softmax warpgroups (warps 0-7)
    setmaxnreg_inc<kSoftmaxRegs>();
    const int wg = warp >> 2;
    const int row = threadIdx.x & 127;  // TMEM lane == query row within the tile
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const __nv_bfloat16* bias = reinterpret_cast<const __nv_bfloat16*>(prm.bias);
    const float2 sl2 = make_float2(prm.scale_log2, prm.scale_log2);
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    // SKIP: list entries known to exist — the head tiles until the list is read (kHead >= 2, so
    // entry wg is tile wg)
    int nt = SKIP ? kHead : ntiles;
    bool known = !SKIP;
    uint32_t bnext = (wg < ntiles) ? tile_bias_bits(prm, bias, b, (int)gridDim.z, wg, n_lat, row) : 0u;
    for (int i = wg; ok; i += 2) {
      if (SKIP && !known && i + 2 >= kHead) {  // the next prefetch may need the list
        known = true;
        if (!mbar_wait(live_ready, 0, prm.err)) {
          ok = false;
          break;
        }
        nt = *n_live_s;
      }
      if (i >= nt) break;
      const int j = (SKIP && i >= kHead) ? live_map[i] : i;  // the key tile of list entry i
      const int it = i >> 1;  // this warpgroup's tile count so far
      float* bt = bias_s + (wg * 2 + (it & 1)) * kBN;
      if (SK_INB(row < kBN && wg * 2 + (it & 1) < 4, prm.err)) bt[row] = bf16_bits_to_f32(bnext) * kLog2e;
      if (i + 2 < nt)  // lands during this tile
        bnext = tile_bias_bits(prm, bias, b, (int)gridDim.z, (SKIP && i + 2 >= kHead) ? live_map[i + 2] : i + 2, n_lat, row);
      named_bar_sync(1 + wg, 128);
      if (!mbar_wait(&s_full[wg], it & 1, prm.err)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float x[kBN];
#pragma unroll
      for (int c = 0; c < kBN / 32; ++c) tmem_ld32(tS + wg * 128 + lane_off + c * 32, x + c * 32);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&s_free[wg]);
      if (CAUSAL && j < n_lat && (j + 1) * kBN - 1 > prm.q_pos0 + q0) {
        // a tile straddling the diagonal: keys past this row's position are invisible
        const int lim = prm.q_pos0 + q0 + row - j * kBN;
#pragma unroll
        for (int c = 0; c < kBN; ++c) x[c] = c > lim ? -INFINITY : x[c];
      }
      // t = s·scale·log2e + bias·log2e, and the row max
      const float mt = scale_bias_rowmax(x, bt, sl2);
      const float m_new = fmaxf(m_run, mt);
      const bool want = m_new > m_run + kRescaleLog2;  // false while every key seen is masked
      // P tile and O rows of this warpgroup were last used by the P·V of list entry i - 2
      if (i >= 2 && !mbar_wait(&o_done[wg], ((i - 2) >> 1) & 1, prm.err)) {
        ok = false;
        break;
      }
      if (__any_sync(0xffffffffu, want)) {
        // warp-uniform: every lane of the warp moves to its exact current max
        const float alpha = (m_new == -INFINITY) ? 1.f : ex2_approx(m_run - m_new);
        if (i >= 2) {
          tc_fence_after();
          rescale_o_row<HD>(tO + wg * HD + lane_off, alpha);
        }
        l_run *= alpha;
        m_run = m_new;
      }
      const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
      // all 128 exponentials (a quarter of them on the FMA pipe), then the row sum and P into this
      // warpgroup's P columns
      exp2_row(x, m_use);
      l_run += pack_p_row(x, tP + wg * kPStride + lane_off);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[wg]);
    }
    // ---- epilogue: merge the two warpgroups' (max, sum, O) for each row; wg writes half the columns
    named_bar_sync(1 + wg, 128);  // this warpgroup is done reading its bias area
    {
      float* ml = bias_s + wg * 2 * kBN;  // [kBM][2]
      if (SK_INB(row * 2 + 1 < 2 * kBN, prm.err)) {
        ml[row * 2] = m_run;
        ml[row * 2 + 1] = l_run;
      }
    }
    named_bar_sync(3, 256);
    bool okk = ok;
    for (int w = 0; w < 2 && okk; ++w) {  // both accumulators complete (the last PV of each)
      const int jl = ((nt - 1 - w) >> 1) * 2 + w;
      if (jl < nt && jl >= 0) okk = mbar_wait(&o_done[w], (jl >> 1) & 1, prm.err);
    }
    if (FUSED && okk) okk = mbar_wait(gate_full, 0, prm.err);
    okk = __all_sync(0xffffffffu, okk);
    if (okk) {
      tc_fence_after();
      const float m0 = bias_s[row * 2], l0 = bias_s[row * 2 + 1];
      const float m1 = bias_s[2 * kBN + row * 2], l1 = bias_s[2 * kBN + row * 2 + 1];
      const float m = fmaxf(m0, m1);
      const float a0 = (l0 > 0.f) ? ex2_approx(m0 - m) : 0.f;
      const float a1 = (l1 > 0.f) ? ex2_approx(m1 - m) : 0.f;
      const float l = a0 * l0 + a1 * l1;
      const float inv = (l > 0.f) ? 1.f / l : 0.f;
      const float c0 = a0 * inv, c1 = a1 * inv;
      // y tile staged as 128B-swizzled [128 rows][64 cols] chunks over the K ring (free: the last P·V
      // completes after every S in the in-order tensor pipe), then written by TMA tensor stores; rows
      // past L are clipped by the tensor map.
      constexpr int NC = HD / 64;  // 32-column pieces per warpgroup half
      float o0[NC][32], o1[NC][32];
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        const uint32_t col = wg * (HD / 2) + c * 32;
        tmem_ld32(tO + lane_off + col, o0[c]);
        tmem_ld32(tO + HD + lane_off + col, o1[c]);
      }
      tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        const int col = wg * (HD / 2) + c * 32;  // first column of this piece
        uint8_t* chunk = smem + Ly::OFF_Y + (col >> 6) * (kBM * 128) + row * 128;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          uint32_t pk[4];
          const int unit = ((col & 63) >> 3) + u;
          uint32_t gw[4] = {0, 0, 0, 0};
          const int goff = (col >> 6) * (kBM * 128) + row * 128 + ((unit ^ (row & 7)) << 4);
          if (FUSED && SK_INB(goff + 16 <= Ly::Q_BYTES, prm.err)) {  // the gate tile sits where Q was, same layout
            const uint4 g4 = *reinterpret_cast<const uint4*>(smem + Ly::OFF_Q + goff);
            gw[0] = g4.x, gw[1] = g4.y, gw[2] = g4.z, gw[3] = g4.w;
          }
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int i0 = 8 * u + 2 * e;
            // c1 == 0 when the second accumulator never ran: do not touch its contents
            float y0 = o0[c][i0] * c0 + (c1 != 0.f ? o1[c][i0] * c1 : 0.f);
            float y1 = o0[c][i0 + 1] * c0 + (c1 != 0.f ? o1[c][i0 + 1] * c1 : 0.f);
            if (FUSED) {
              // the attention output rounded to bf16 as SDPA returns it, then the `gate` arithmetic
              // (engine/fused.py:182-190): y · (1 / (1 + expf(-g))) in fp32 (the reciprocal correctly
              // rounded, as the IEEE division), rounded once
              y0 = __bfloat162float(__float2bfloat16_rn(y0)) * __frcp_rn(1.0f + expf(-__uint_as_float(gw[e] << 16)));
              y1 = __bfloat162float(__float2bfloat16_rn(y1)) *
                   __frcp_rn(1.0f + expf(-__uint_as_float(gw[e] & 0xffff0000u)));
            }
            const __nv_bfloat162 v2 = __floats2bfloat162_rn(y0, y1);
            pk[e] = *reinterpret_cast<const uint32_t*>(&v2);
          }
          if (SK_INB((col >> 6) * (kBM * 128) + row * 128 + ((unit ^ (row & 7)) << 4) + 16 <= Ly::NSK * Ly::KV_BYTES, prm.err))
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(smem_u32(chunk + ((unit ^ (row & 7)) << 4))),
                         "r"(pk[0]), "r"(pk[1]), "r"(pk[2]), "r"(pk[3])
                         : "memory");
        }
      }
      fence_proxy_async_smem();
    }
    named_bar_sync(3, 256);
    if (okk && threadIdx.x == 0) {
#pragma unroll
      for (int c = 0; c < Ly::NCH; ++c) tma_store_4d(&tmY, smem + Ly::OFF_Y + c * (kBM * 128), c * 64, h, q0, b);
      tma_store_commit_and_wait_read();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---- host ------------------------------------------------------------------------------------------
// q (B, H, L, hd), k_lat (B, H, Lk, hd); v_lat (B, H, Lk, hd), or with VO4 the projection rows o4;
// o4 (B·L, 4·D): the gate source of the fused block (unused otherwise).
// kv_rows: rows per head in the key/value buffers (Lk for the DiT; the cache's max_len for the prefill).
template <int HD, bool FUSED, bool VO4, bool CAUSAL = false>
static int launch_tc(const void* q, const void* k_lat, const void* v_lat, const void* k_ctx, const void* v_ctx,
                     const void* o4, long long ctx_bs, const TcParams& prm, int B, cudaStream_t st,
                     int kv_rows = -1) {
  using Ly = TcLayout<HD>;
  const int H = prm.H, L = prm.L, Lk = prm.Lk, S = prm.S;
  CUtensorMap mq, mk, mv, mkc, mvc;
  const int rcm = make_operand_maps<HD>(q, k_lat, v_lat, k_ctx, v_ctx, ctx_bs, prm, B, kv_rows, &mq, &mk, &mv, &mkc,
                                        &mvc, !VO4);
  if (rcm != SK_OK) return rcm;
  CUtensorMap mg = mq;  // never read unless FUSED
  if (FUSED || VO4) {
    // o4 as (B, L, 4·D): v and gate tiles are boxes of 128 rows x 64 columns at column offsets
    // 2·D + h·hd and 3·D + h·hd; rows past L read as zeros
    cuuint64_t d4[3] = {(cuuint64_t)4 * prm.D, (cuuint64_t)L, (cuuint64_t)B};
    cuuint64_t s4[2] = {(cuuint64_t)4 * prm.D * 2, (cuuint64_t)L * 4 * prm.D * 2};
    cuuint32_t box[3] = {64, kBM, 1};
    if (!sk_make_map_bf16(&mg, o4, 3, d4, s4, box)) return SK_ERR_CUDA;
    if (VO4) mv = mg;
  }
  CUtensorMap my;
  {
    // y (B, L, H, hd): a box of 128 query rows of one head, 64 columns wide
    cuuint64_t dims[4] = {(cuuint64_t)HD, (cuuint64_t)H, (cuuint64_t)L, (cuuint64_t)B};
    cuuint64_t str[3] = {(cuuint64_t)HD * 2, (cuuint64_t)H * HD * 2, (cuuint64_t)L * H * HD * 2};
    cuuint32_t box[4] = {64, 1, kBM, 1};
    if (!sk_make_map_bf16(&my, prm.y, 4, dims, str, box)) return SK_ERR_CUDA;
  }
  const int smem = Ly::SMEM_ALLOC;
  int dev = 0;
  cudaGetDevice(&dev);
  static int sm_count[64] = {};
  if (dev >= 0 && dev < 64 && sm_count[dev] == 0 &&
      cudaDeviceGetAttribute(&sm_count[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return SK_ERR_CUDA;
  // Masked-tile skipping (never in the causal form): with a bias, more key tiles than the head tiles,
  // and more CTAs than SMs. One CTA fills an SM (all of TMEM), so in a single wave the call lasts as
  // long as its longest CTA, and in the engine's CFG batches the cond row has no whole tile masked:
  // skipping pays only where CTAs queue for SMs and the shortened ones let the queue drain sooner,
  // while the list of tiles costs each CTA about 0.7 us.
  const int n_lat = (Lk + kBN - 1) / kBN, ntiles = n_lat + (S + kBN - 1) / kBN;
  const long long ctas = (long long)((L + kBM - 1) / kBM) * H * B;
  const bool skip = !CAUSAL && prm.bias != nullptr && ntiles > head_tiles<HD>(n_lat, ntiles) &&
                    ntiles <= kMaxLiveTiles && dev >= 0 && dev < 64 && ctas > sm_count[dev];
  auto kern = attn_tc_kernel<HD, FUSED, VO4, CAUSAL, false>;
  if constexpr (!CAUSAL) {
    if (skip) kern = attn_tc_kernel<HD, FUSED, VO4, CAUSAL, true>;
  }
  static bool attr_done[2][64] = {};
  if (dev >= 0 && dev < 64 && !attr_done[skip][dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return SK_ERR_CUDA;
    attr_done[skip][dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((L + kBM - 1) / kBM, H, B);
  cfg.blockDim = dim3(kThreadsTC);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // set-up overlaps the previous kernel
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, mq, mk, mv, mkc, mvc, my, mg, prm) != cudaSuccess)
    return SK_ERR_CUDA;
  return cudaPeekAtLastError() == cudaSuccess ? SK_OK : SK_ERR_CUDA;
}

}  // namespace dit
}  // namespace sk

int sk_launch_dit_attention_f32(const float* q, const float* k_lat, const float* v_lat, const float* k_ctx,
                                const float* v_ctx, const float* bias, float* y, int B, int H, int L, int Lk, int S,
                                int hd, long long ctx_bs, long long bias_bs, float scale, cudaStream_t st);

extern "C" int sk_dit_attention(const void* q, const void* k_lat, const void* v_lat, const void* k_ctx,
                                const void* v_ctx, const void* key_bias, void* y, int B, int H, int L, int Lk, int S,
                                int hd, long long ctx_batch_stride, long long bias_batch_stride, int dtype,
                                float scale, void* stream) {
  using namespace sk::dit;
  if (!q || !y) return SK_ERR_INVALID_ARG;
  if (B <= 0 || H <= 0 || L <= 0 || Lk < 0 || S < 0 || Lk + S <= 0) return SK_ERR_INVALID_ARG;
  if (Lk > 0 && (!k_lat || !v_lat)) return SK_ERR_INVALID_ARG;
  if (S > 0 && (!k_ctx || !v_ctx)) return SK_ERR_INVALID_ARG;
  if (ctx_batch_stride < 0 || bias_batch_stride < 0) return SK_ERR_INVALID_ARG;
  if (hd != 64 && hd != 128) return SK_ERR_UNSUPPORTED;
  if (dtype != SK_BF16 && dtype != SK_F32) return SK_ERR_UNSUPPORTED;
  const uintptr_t al = reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k_lat) |
                       reinterpret_cast<uintptr_t>(v_lat) | reinterpret_cast<uintptr_t>(k_ctx) |
                       reinterpret_cast<uintptr_t>(v_ctx) | reinterpret_cast<uintptr_t>(y);
  if (al & 15) return SK_ERR_INVALID_ARG;
  // a batched ctx buffer must keep 16-byte aligned rows for the tensor map
  if (S > 0 && ctx_batch_stride != 0 && ((ctx_batch_stride * (dtype == SK_BF16 ? 2 : 4)) & 15))
    return SK_ERR_INVALID_ARG;
  int rc = sk_check_device();
  if (rc != SK_OK) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const float sc = scale > 0.f ? scale : 1.0f / sqrtf((float)hd);
  if (dtype == SK_F32)
    return sk_launch_dit_attention_f32(static_cast<const float*>(q), static_cast<const float*>(k_lat),
                                       static_cast<const float*>(v_lat), static_cast<const float*>(k_ctx),
                                       static_cast<const float*>(v_ctx), static_cast<const float*>(key_bias),
                                       static_cast<float*>(y), B, H, L, Lk, S, hd, ctx_batch_stride,
                                       bias_batch_stride, sc, st);
  int* err = sk_error_word_ptr();
  if (!err) return SK_ERR_CUDA;
  TcParams prm{key_bias, bias_batch_stride, y, H, L, Lk, S, sc * kLog2e, ctx_batch_stride != 0 ? 1 : 0, err, H * hd, 1, 0};
  return hd == 64 ? launch_tc<64, false, false>(q, k_lat, v_lat, k_ctx, v_ctx, nullptr, ctx_batch_stride, prm, B, st)
                  : launch_tc<128, false, false>(q, k_lat, v_lat, k_ctx, v_ctx, nullptr, ctx_batch_stride, prm, B, st);
}

int sk_launch_qkv_prologue(const void* o4, const float* qk_w, const float* freqs, void* q, void* k, void* v, int B,
                           int L, int H, int hd, float eps, int dtype, cudaStream_t st);

extern "C" int sk_dit_attention_layer(const void* o4, const float* qk_w, const float* freqs, const void* k_ctx,
                                      const void* v_ctx, const void* key_bias, void* out, void* q_buf, void* k_buf,
                                      void* v_buf, int B, int H, int L, int S, int hd, long long ctx_batch_stride,
                                      long long bias_batch_stride, float eps, int dtype, float scale, void* stream) {
  using namespace sk::dit;
  if (!o4 || !qk_w || !freqs || !out || !q_buf || !k_buf || !v_buf) return SK_ERR_INVALID_ARG;
  if (B <= 0 || H <= 0 || L <= 0 || S < 0 || H % 2) return SK_ERR_INVALID_ARG;
  if (S > 0 && (!k_ctx || !v_ctx)) return SK_ERR_INVALID_ARG;
  if (ctx_batch_stride < 0 || bias_batch_stride < 0) return SK_ERR_INVALID_ARG;
  if (hd != 64 && hd != 128) return SK_ERR_UNSUPPORTED;
  if (dtype != SK_BF16) return SK_ERR_UNSUPPORTED;  // the fp32 mode runs the three separate calls
  const uintptr_t al = reinterpret_cast<uintptr_t>(o4) | reinterpret_cast<uintptr_t>(qk_w) |
                       reinterpret_cast<uintptr_t>(freqs) | reinterpret_cast<uintptr_t>(k_ctx) |
                       reinterpret_cast<uintptr_t>(v_ctx) | reinterpret_cast<uintptr_t>(out) |
                       reinterpret_cast<uintptr_t>(q_buf) | reinterpret_cast<uintptr_t>(k_buf) |
                       reinterpret_cast<uintptr_t>(v_buf);
  if (al & 15) return SK_ERR_INVALID_ARG;
  if (S > 0 && ctx_batch_stride != 0 && ((ctx_batch_stride * 2) & 15)) return SK_ERR_INVALID_ARG;
  int rc = sk_check_device();
  if (rc != SK_OK) return rc;
  int* err = sk_error_word_ptr();
  if (!err) return SK_ERR_CUDA;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const float sc = scale > 0.f ? scale : 1.0f / sqrtf((float)hd);
  TcParams prm{key_bias, bias_batch_stride, out, H, L, L, S, sc * kLog2e, ctx_batch_stride != 0 ? 1 : 0, err, H * hd, 1, 0};
  if (hd == 64) {
    // two launches: q and k (normalised, rotated) into the caller's buffers; the attention reads v
    // and the gate straight from o4 and writes y · sigmoid(gate)
    rc = sk_launch_qkv_prologue(o4, qk_w, freqs, q_buf, k_buf, nullptr, B, L, H, hd, eps, SK_BF16, st);
    if (rc != SK_OK) return rc;
    return launch_tc<64, true, true>(q_buf, k_buf, o4, k_ctx, v_ctx, o4, ctx_batch_stride, prm, B, st);
  }
  // hd = 128: three launches, y through `out` and gated in place — measured faster on B200 than the
  // gate epilogue there (the fused epilogue lengthens every CTA of the 1.3-wave c2 grid)
  rc = sk_launch_qkv_prologue(o4, qk_w, freqs, q_buf, k_buf, v_buf, B, L, H, hd, eps, SK_BF16, st);
  if (rc != SK_OK) return rc;
  rc = launch_tc<128, false, false>(q_buf, k_buf, v_buf, k_ctx, v_ctx, nullptr, ctx_batch_stride, prm, B, st);
  if (rc != SK_OK) return rc;
  return sk_dit_gate(out, o4, out, (long long)B * L, H * hd, SK_BF16, SK_BF16, 1.f, stream);
}

int sk_launch_prefill_prologue(const float* qkv, const float* qn, const float* kn, float eps, const float* rope,
                               void* Kc, void* Vc, void* q_buf, int pos0, int T, int max_len, int nq, int nkv,
                               int cache_dtype, cudaStream_t st);
int sk_launch_prefill_attention_f32(const float* q, const float* Kc, const float* Vc, float* y, int nq, int nkv,
                                    int T, int pos0, int max_len, cudaStream_t st);

extern "C" int sk_prefill_attention(const float* qkv, const float* qn, const float* kn, float eps, const float* rope,
                                    void* Kc, void* Vc, int pos0, int T, int max_len, int nq, int nkv, int hd,
                                    void* out, void* q_buf, int cache_dtype, void* stream) {
  using namespace sk::dit;
  if (!qkv || !qn || !kn || !rope || !Kc || !Vc || !out || !q_buf) return SK_ERR_INVALID_ARG;
  if (T <= 0 || pos0 < 0 || max_len <= 0 || nkv <= 0 || nq <= 0 || pos0 + T > max_len) return SK_ERR_INVALID_ARG;
  if (hd != 128 || nq != 2 * nkv) return SK_ERR_UNSUPPORTED;  // qwen3/kernels.py:457
  if (cache_dtype != SK_BF16 && cache_dtype != SK_F32) return SK_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(Kc) | reinterpret_cast<uintptr_t>(Vc) | reinterpret_cast<uintptr_t>(out) |
       reinterpret_cast<uintptr_t>(q_buf)) & 15)
    return SK_ERR_INVALID_ARG;
  int rc = sk_check_device();
  if (rc != SK_OK) return rc;
  int* err = sk_error_word_ptr();
  if (!err) return SK_ERR_CUDA;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  rc = sk_launch_prefill_prologue(qkv, qn, kn, eps, rope, Kc, Vc, q_buf, pos0, T, max_len, nq, nkv, cache_dtype, st);
  if (rc != SK_OK) return rc;
  if (cache_dtype == SK_F32)  // the fp32 mode: CUDA-core fp32 attention
    return sk_launch_prefill_attention_f32(static_cast<const float*>(q_buf), static_cast<const float*>(Kc),
                                           static_cast<const float*>(Vc), static_cast<float*>(out), nq, nkv, T, pos0,
                                           max_len, st);
  // queries (1, nq, T, 128) from q_buf, keys and values rows [0, pos0 + T) of the cache heads
  // (nkv, max_len, 128), query head h on key/value head h / 2, causal from row 0 at position pos0
  const float sc = 1.0f / sqrtf(128.f);
  TcParams prm{nullptr, 0, out, nq, T, pos0 + T, 0, sc * kLog2e, 0, err, nq * hd, nq / nkv, pos0};
  return launch_tc<128, false, false, true>(q_buf, Kc, Vc, nullptr, nullptr, nullptr, 0, prm, 1, st, max_len);
}
