// Causal (or full) attention forward for head_dim 16, 32, 64, 128 and 256
// (sm_100a); head_dim 8 runs the head_dim-16 instance on Q/K/V stored 16 wide.
//
// Replaces custom_kernel/triton_attention.py:126-232 of the reference (the
// parameters and the heavy-first work schedule are in tt_attention.cuh).  At
// these head sizes the tensor-core work per score is small and the softmax
// (one exponential per score) bounds the kernel, so the layout keeps the
// softmax warps from ever waiting on the tensor core:
//
//  * one CTA per SM runs two independent pipelines ("streams"; one at head_dim
//    128 and 256, whose [O | l] accumulator takes most of TMEM), each on a
//    128-query tile of its own work item, with 4 softmax warps (one per TMEM
//    lane quadrant, a whole row per thread), its own TMA producer warp
//    (4 NS + s) and its own MMA-issuer warp (5 NS + s); idle warps complete
//    the last warpgroup (setmaxnreg acts on whole warpgroups);
//  * key tiles are 64 wide; each stream has NSB score buffers S in TMEM (three
//    at head_dim 16/32, two at 64); the softmax writes the FP16 probabilities
//    P back over the first 32 columns of the S buffer it has just read (one
//    tcgen05.st, no shared memory and no proxy fence), and P.V reads them as a
//    TMEM A operand.  S_{t+NSB} is issued right after P.V of tile t into the
//    same buffer: one thread's MMAs execute in issue order, so P_t is read
//    before it is overwritten.
//
// Per stream and key tile t (buffer b = t % NSB):
//   S_b = Q K_t^T           TMEM, 64 FP32 columns
//   softmax: the 64 scores of a row come into registers in one TMEM read and
//   S_b is released at once; row max by a 3-input max tree; the reference
//   maximum m only moves when the tile maximum exceeds it by more than 2^8
//   (O and l are then rescaled, rare after the first tiles), so P stays <= 256
//   in FP16; exp2 of S*scale*log2(e) - m (MUFU, with a share of the
//   exponentials on the FP32 pipe); P is rounded to FP16 pairs into
//   columns 0..31 of S_b
//   [O | l] += P_b [V_t | 1]  TMEM, accumulated over the item's key tiles (NOB
//                           buffers by item: with two, an item's epilogue runs
//                           while the next item's first P.V proceeds).  Each V^T stage is
//                           followed by 16 rows of FP16 ones, so the same MMA
//                           (N = HD + 16) also sums the FP16 probabilities
//                           of every row: the softmax warps never add them.
//                           At head_dim 256 (N = 272 > 256) it is issued as
//                           two MMAs, N = 128 and N = 144.
// Q and K tiles are stored as 128-byte swizzle atoms of 64 features (head_dim
// >= 64; one TMA copy per atom) or as one atom of head_dim features.
// Items (sequence*head, query tile) are dealt heavy-first: stream s of CTA c
// takes items NS c + s, NS c + s + NS G, ... (G = gridDim.x).
#pragma once

#include "tt_attention.cuh"

namespace tt {


template <int HD>
struct AttnDbLayout {
  static constexpr int NS = HD >= 128 ? 1 : 2;   // independent pipelines per CTA
  // S (and P) buffers per stream: the MMA warp issues S up to NSB - 1 tiles
  // ahead of the softmax, so the softmax rarely waits for the round trip
  // (P published -> P.V and the next S issued and done).  Three where TMEM
  // allows (head_dim 16 and 32; at head_dim 32 with a single [O | l] buffer):
  // C5 attention 4.78 -> 4.61 ms per forward, C2 0.337 -> 0.321, same bits.
  static constexpr int NSB = HD <= 32 ? 3 : 2;
  static constexpr int BM = 128, BN = 64;
  static constexpr int NST = HD == 16 ? 8 : HD == 32 ? 6 : HD <= 128 ? 4 : 2;
  static constexpr int NQ = HD == 256 ? 1 : 2;  // Q tile buffers per stream
  // [O | l] accumulator buffers per stream: two (an item's epilogue runs after
  // the next item's first tile) where TMEM allows; one at head_dim 64, where the
  // next item's first P.V waits for the epilogue to have read O.
  static constexpr int NOB = NS * (NSB * 64 + 2 * (HD + 16)) <= 512 ? 2 : 1;
  static constexpr int KATOM = HD >= 64 ? 64 : HD;  // features per swizzle atom of Q and K
  static constexpr int NATOM = HD / KATOM;
  static constexpr int Q_ATOM = BM * KATOM * 2, K_ATOM = BN * KATOM * 2;
  static constexpr int Q_BYTES = NATOM * Q_ATOM;
  static constexpr int K_BYTES = NATOM * K_ATOM;
  static constexpr int V_BYTES = HD * 128;  // V^T block: HD rows of 64 keys (128 bytes)
  static constexpr int ONES_BYTES = 16 * 128;           // 16 rows of 64 FP16 ones after each V^T block
  static constexpr int V_STAGE = V_BYTES + ONES_BYTES;  // B operand of P.[V | 1], N = ON rows
  static constexpr int ON = HD + 16;                    // accumulator columns: O, then 16 copies of l
  static constexpr int ON0 = ON <= 256 ? ON : 128;      // N of the first P.V MMA (the second: ON - ON0)
  // Per-stream region: Q[NQ] | K[NST] | V[NST] (each with its ones block)
  static constexpr int S_Q = 0;
  static constexpr int S_K = S_Q + NQ * Q_BYTES;
  static constexpr int S_V = S_K + NST * K_BYTES;
  static constexpr int STREAM_BYTES = S_V + NST * V_STAGE;
  // Per-stream barriers: q_full[2] q_empty[2] kv_full[NST] kv_empty[NST]
  // s_full[NSB] p_full[NSB] pv_done[NSB] o_full[2] o_free[2]
  static constexpr int B_QF = 0, B_QE = 2, B_KF = 4, B_KE = 4 + NST, B_SF = 4 + 2 * NST,
                       B_PF = B_SF + NSB, B_PE = B_PF + NSB, B_OF = B_PE + NSB, B_OR = B_OF + 2;
  static constexpr int NBAR_STREAM = B_OR + 2;
  static constexpr int OFF_BAR = NS * STREAM_BYTES;
  static constexpr int OFF_DONE = OFF_BAR + NS * NBAR_STREAM * 8;  // done[NS]
  static constexpr int OFF_MISC = OFF_DONE + 32;
  static constexpr int SMEM_ALLOC = OFF_MISC + 16 + 1024;
  // TMEM per stream: S buffers at 0, 64, ..., [O | l] of item buffer ob at NSB * 64 + ob * ON.
  static constexpr int TMEM_COLS = 512, TMEM_O = NSB * BN, TMEM_STREAM = TMEM_O + NOB * ON;
  // Warps: 4 NS softmax (stream w / 4, lane quadrant w % 4), NS producers, NS
  // MMA issuers, then idle warps up to a whole number of warpgroups:
  // setmaxnreg is a warpgroup operation, so every warpgroup must be complete.
  static constexpr int W_PROD = 4 * NS, W_MMA = 5 * NS;
  static constexpr int NWARPS = 4 * NS + (2 * NS + 3) / 4 * 4;
  static constexpr int THREADS = 32 * NWARPS;
  // Register split (setmaxnreg): the launch provides THREADS x REGS_LAUNCH;
  // the 4 NS softmax warps take REGS_SOFTMAX each, all other warps REGS_OTHER.
  // The launcher refuses to start the kernel unless it was built with exactly
  // REGS_LAUNCH registers per thread (a split above the launch total would make
  // setmaxnreg.inc wait forever).
  // With one stream (8 warps) every warp fits REGS_SOFTMAX at launch and
  // there is no split.
  static constexpr bool SPLIT = NS == 2;
  static constexpr int REGS_LAUNCH = 168;
  static constexpr int REGS_SOFTMAX = 216, REGS_OTHER = 56;
  static_assert(NWARPS % 4 == 0, "whole warpgroups");
  static_assert(!SPLIT || 128 * NS * REGS_SOFTMAX + 32 * (NWARPS - 4 * NS) * REGS_OTHER <= THREADS * REGS_LAUNCH,
                "register split");
  static_assert(NS * TMEM_STREAM <= TMEM_COLS, "TMEM budget");
  static_assert(HD == 16 || HD == 32 || HD == 64 || HD == 128 || HD == 256,
                "this kernel covers head_dim 16, 32, 64, 128 and 256");
  static_assert(ON - ON0 <= 256 && ON0 % 16 == 0, "P.V MMA widths");
  static_assert(STREAM_BYTES % 1024 == 0 && S_V % 1024 == 0 && V_STAGE % 1024 == 0, "alignment");
  static_assert(SMEM_ALLOC <= 232448, "shared memory budget");
};

// Pairs of exponentials per 8 computed by polynomial on the FP32 pipe instead
// of MUFU.
// (3 of 8 at head_dim 16/32, C5 attention 1.028 -> 1.000 ms per launch against
// 2 of 8; 4 of 8 measured 1.053; at head_dim 64 2 and 3 of 8 measure the same.)
template <int HD>
constexpr int kDbExpFmaOf8 = HD <= 32 ? 3 : 2;


template <int HD>
__global__ void __launch_bounds__(AttnDbLayout<HD>::THREADS, 1)
    attn_db_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const AttnParams p, int n_items) {
  using L = AttnDbLayout<HD>;
  constexpr int BM = L::BM, BN = L::BN, NST = L::NST;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_qt = (p.seq + BM - 1) / BM;
  const int D = p.heads * p.ctx_hd;  // ctx row width (p.ctx_hd = 8 or HD)
  const int n_out16 = p.ctx_hd / 8;   // 16-byte pieces of a stored ctx row per head
  constexpr int NS = L::NS, NSB = L::NSB;
  const int G2 = NS * static_cast<int>(gridDim.x);  // item stride of one stream
  uint64_t* bars_all = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* done = reinterpret_cast<uint64_t*>(smem + L::OFF_DONE);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) mbar_init(&done[s], 1);
    for (int s = 0; s < NS; ++s) {
      uint64_t* b = bars_all + s * L::NBAR_STREAM;
      for (int i = 0; i < L::NSB; ++i) {
        mbar_init(&b[L::B_SF + i], 1);
        mbar_init(&b[L::B_PF + i], 4);
        mbar_init(&b[L::B_PE + i], 1);
      }
      for (int i = 0; i < 2; ++i) {
        mbar_init(&b[L::B_QF + i], 1);
        mbar_init(&b[L::B_QE + i], 1);
        mbar_init(&b[L::B_OF + i], 1);
        mbar_init(&b[L::B_OR + i], 4);
      }
      for (int i = 0; i < NST; ++i) {
        mbar_init(&b[L::B_KF + i], 1);
        mbar_init(&b[L::B_KE + i], 1);
      }
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  // The ones rows after every V^T stage (never written by TMA), made visible
  // to the tensor core's (async proxy) reads before the first MMA.
  for (int i = threadIdx.x; i < NS * NST * (L::ONES_BYTES / 16); i += blockDim.x) {
    const int s = i / (NST * (L::ONES_BYTES / 16));
    const int rem = i % (NST * (L::ONES_BYTES / 16));
    const int st = rem / (L::ONES_BYTES / 16), ch = rem % (L::ONES_BYTES / 16);
    st_shared_v4(smem_u32(smem + s * L::STREAM_BYTES + L::S_V + st * L::V_STAGE + L::V_BYTES + ch * 16),
                 0x3c003c00u, 0x3c003c00u, 0x3c003c00u, 0x3c003c00u);
  }
  fence_proxy_async_smem();
  if (warp == L::W_MMA) {
    tmem_alloc(tmem_slot, L::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_wait();  // activations of the previous kernel are final from here on
  pdl_trigger();
  const uint32_t tmem_base = *tmem_slot;
  const Watchdog wd{p.err, abort_flag, p.timeout_ns};

  // Key tiles of an item (64 keys each).
  auto n_tiles = [&](const AttnItem& it) -> int {
    if (it.n == 0) return 0;
    const int kv_limit = p.causal ? min(it.q0 + BM, it.kv_end) : it.kv_end;
    return (kv_limit + BN - 1) / BN;
  };
  auto first_item = [&](int w) -> int {  // first item >= w of this stream with work
    while (w < n_items && attn_item(p, w, n_qt).n == 0) w += G2;
    return w;
  };

  if (warp >= L::W_PROD && warp < L::W_MMA) {
    // ------------------------------------------------------------ producer of stream warp - W_PROD
    if constexpr (L::SPLIT) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(L::REGS_OTHER));
    if (lane == 0) {
      const int s = warp - L::W_PROD;
      uint64_t* b = bars_all + s * L::NBAR_STREAM;
      uint8_t* sb = smem + s * L::STREAM_BYTES;
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      int t = 0, it = 0;
      bool ok = true;
      for (int w = first_item(NS * static_cast<int>(blockIdx.x) + s); ok && w < n_items;
           w = first_item(w + G2)) {
        const AttnItem item = attn_item(p, w, n_qt);
        const int nt = n_tiles(item);
        const int qb = it % L::NQ;
        if (!(ok = wait_phase(&b[L::B_QE + qb], ((it / L::NQ) & 1) ^ 1, wd, 0x131))) break;
        mbar_arrive_expect_tx(&b[L::B_QF + qb], L::Q_BYTES);
#pragma unroll
        for (int a = 0; a < L::NATOM; ++a)
          tma_load_3d(sb + L::S_Q + qb * L::Q_BYTES + a * L::Q_ATOM, &tmQ, &b[L::B_QF + qb], a * L::KATOM,
                      item.q0, item.bh);
        ++it;
        for (int j = 0; j < nt; ++j) {
          const int st = t % NST;
          if (!(ok = wait_phase(&b[L::B_KE + st], ((t / NST) & 1) ^ 1, wd, 0x132))) break;
          mbar_arrive_expect_tx(&b[L::B_KF + st], L::K_BYTES + L::V_BYTES);
#pragma unroll
          for (int a = 0; a < L::NATOM; ++a)
            tma_load_3d(sb + L::S_K + st * L::K_BYTES + a * L::K_ATOM, &tmK, &b[L::B_KF + st], a * L::KATOM,
                        j * BN, item.bh);
          tma_load_3d(sb + L::S_V + st * L::V_STAGE, &tmV, &b[L::B_KF + st], j * BN, 0, item.bh);
          ++t;
        }
      }
      // Let every copy this stream started land before the CTA may exit.
      for (int i = (it > L::NQ ? it - L::NQ : 0); i < it; ++i)
        wait_drain(&b[L::B_QF + i % L::NQ], (i / L::NQ) & 1, kDrainLimitNs);
      for (int i = (t > NST ? t - NST : 0); i < t; ++i)
        wait_drain(&b[L::B_KF + i % NST], (i / NST) & 1, kDrainLimitNs);
    }
  } else if (warp >= 6 * NS) {
    // ------------------------------------------------------------ idle warps (whole warpgroups)
    if constexpr (L::SPLIT) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(L::REGS_OTHER));
  } else if (warp >= L::W_MMA) {
    // ------------------------------------------------------------ MMA issuer of stream warp - W_MMA
    if constexpr (L::SPLIT) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(L::REGS_OTHER));
    if (lane == 0) {
      const int s = warp - L::W_MMA;
      uint64_t* b = bars_all + s * L::NBAR_STREAM;
      const uint32_t sb = smem_u32(smem + s * L::STREAM_BYTES);
      const uint32_t tS = tmem_base + s * L::TMEM_STREAM;
      constexpr uint32_t kSwQK = swizzle_kind_for_bytes(L::KATOM * 2);
      constexpr uint32_t kSboQK = 8 * L::KATOM * 2;
      const uint32_t idesc_s = umma_idesc_f16_f32(BM, BN);
      const uint32_t idesc_o = umma_idesc_f16_f32(BM, L::ON0);
      const uint32_t idesc_o1 = umma_idesc_f16_f32(BM, L::ON > L::ON0 ? L::ON - L::ON0 : 16);
      // S cursor: item w_s, tile j_s of n_s, stream tile u, item count it_s.
      int w_s = first_item(NS * static_cast<int>(blockIdx.x) + s), j_s = 0, n_s = 0, u = 0, it_s = 0;
      if (w_s < n_items) n_s = n_tiles(attn_item(p, w_s, n_qt));
      auto issue_s = [&]() -> bool {
        const int st = u % NST, qb = it_s % L::NQ, bb = u % NSB;
        if (j_s == 0 && !wait_phase(&b[L::B_QF + qb], (it_s / L::NQ) & 1, wd, 0x231)) return false;
        if (!wait_phase(&b[L::B_KF + st], (u / NST) & 1, wd, 0x232)) return false;
        // S buffer bb last held P_{u-NSB}, read by P.V of tile u - NSB, which
        // this thread issued before this MMA (same-thread MMAs execute in order).
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          // Features 16kk .. 16kk+15: atom 16kk / KATOM, 32-byte step within it.
          const int qa = (16 * kk) / L::KATOM, qo = ((16 * kk) % L::KATOM) * 2;
          const uint64_t da = umma_sdesc(sb + L::S_Q + qb * L::Q_BYTES + qa * L::Q_ATOM + qo, kSboQK, kSwQK);
          const uint64_t db = umma_sdesc(sb + L::S_K + st * L::K_BYTES + qa * L::K_ATOM + qo, kSboQK, kSwQK);
          umma_f16(tS + bb * BN, da, db, idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(&b[L::B_SF + bb]);
        if (j_s == n_s - 1) umma_commit(&b[L::B_QE + qb]);
        ++u;
        if (++j_s == n_s) {
          j_s = 0;
          ++it_s;
          w_s = first_item(w_s + G2);
          n_s = w_s < n_items ? n_tiles(attn_item(p, w_s, n_qt)) : 0;
        }
        return true;
      };
      // P.V cursor: items it_o (O buffer it_o % NOB), tile j_o of n_o.
      int w_o = first_item(NS * static_cast<int>(blockIdx.x) + s), j_o = 0, it_o = 0;
      int n_o = w_o < n_items ? n_tiles(attn_item(p, w_o, n_qt)) : 0;
      bool ok = true;
      // Scores of the first NSB tiles, then per tile t: P.V_t, then S_{t+NSB}.
      for (int k = 0; ok && k < NSB && w_s < n_items; ++k) ok = issue_s();
      for (int t = 0; ok && t < u; ++t) {
        const int bb = t % NSB, st = t % NST, ob = it_o % L::NOB;
        if (!(ok = wait_phase(&b[L::B_PF + bb], (t / NSB) & 1, wd, 0x234))) break;
        if (j_o == 0 && !(ok = wait_phase(&b[L::B_OR + ob], ((it_o / L::NOB) & 1) ^ 1, wd, 0x235))) break;
        tc_fence_after();
        const uint32_t tO = tS + L::TMEM_O + ob * L::ON;
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          // Keys 16kk .. 16kk+15 of P_t: columns 8kk .. 8kk+7 of S buffer bb (FP16 pairs).
          const uint32_t vrow0 = sb + L::S_V + st * L::V_STAGE + kk * 32;
          const uint32_t acc = (kk > 0 || j_o > 0) ? 1u : 0u;
          umma_f16_ts(tO, tS + bb * BN + kk * 8, umma_sdesc(vrow0, 1024, kSw128), idesc_o, acc);
          if constexpr (L::ON > L::ON0)  // rows ON0 .. ON - 1 of [V | 1]^T: 128 bytes each
            umma_f16_ts(tO + L::ON0, tS + bb * BN + kk * 8, umma_sdesc(vrow0 + L::ON0 * 128, 1024, kSw128),
                        idesc_o1, acc);
        }
        umma_commit(&b[L::B_KE + st]);
        umma_commit(&b[L::B_PE + bb]);  // P.V of tile t done (the rescale path waits on it)
        if (++j_o == n_o) {
          umma_commit(&b[L::B_OF + ob]);  // O of this item is final
          j_o = 0;
          ++it_o;
          w_o = first_item(w_o + G2);
          n_o = w_o < n_items ? n_tiles(attn_item(p, w_o, n_qt)) : 0;
        }
        if (w_s < n_items) ok = issue_s();  // S_{t+NSB} into buffer bb
      }
      // All MMAs this thread issued must finish before TMEM is released.
      umma_commit(&done[s]);
      wait_drain(&done[s], 0, kDrainLimitNs);
    }
  } else {
    // ------------------------------------------------------------ softmax
    if constexpr (L::SPLIT) asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(L::REGS_SOFTMAX));
    const int s = warp >> 2;  // stream
    const int q = warp & 3;   // TMEM lane quadrant (warp % 4)
    const int row = q * 32 + lane;
    uint64_t* b = bars_all + s * L::NBAR_STREAM;
    const uint32_t tS = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + s * L::TMEM_STREAM;
    const float sl2 = p.scale_log2;
    const uint64_t sl2x2 = f2_pack(sl2, sl2);
    bool ok = true;
    int t = 0, it = 0;
    // An item's epilogue runs after the next item's first key tile, by when
    // its last P.V has long finished.
    bool pend = false;
    int pend_it = 0;
    __half* pend_dst = nullptr;
    bool pend_store = false;
    bool pend_valid = false;
    auto finish_item = [&]() -> bool {
      const int ob = pend_it % L::NOB;
      if (!warp_wait_phase(&b[L::B_OF + ob], (pend_it / L::NOB) & 1, wd, 0x333)) return false;
      tc_fence_after();
      if constexpr (HD >= 128) {
        // O comes out 32 columns at a time (a whole row would take HD registers).
        const uint32_t tOf = tS + L::TMEM_O + ob * L::ON;
        uint32_t lv[8];  // row sum of the FP16 probabilities (column HD of the accumulator)
        tmem_ld_x8(tOf + HD, lv);
        tmem_ld_wait_tied(lv);
        const float lsum = __uint_as_float(lv[0]);
        const float inv = (pend_valid && lsum > 0.f) ? 1.f / lsum : 0.f;
#pragma unroll 1
        for (int c = 0; c < HD / 32; ++c) {
          uint32_t o[32];
          tmem_ld_x32(tOf + 32 * c, o);
          tmem_ld_wait_tied(o);
          if (pend_store) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              uint4 v;
              v.x = pack_half2(__uint_as_float(o[8 * i + 0]) * inv, __uint_as_float(o[8 * i + 1]) * inv);
              v.y = pack_half2(__uint_as_float(o[8 * i + 2]) * inv, __uint_as_float(o[8 * i + 3]) * inv);
              v.z = pack_half2(__uint_as_float(o[8 * i + 4]) * inv, __uint_as_float(o[8 * i + 5]) * inv);
              v.w = pack_half2(__uint_as_float(o[8 * i + 6]) * inv, __uint_as_float(o[8 * i + 7]) * inv);
              if (4 * c + i < n_out16) reinterpret_cast<uint4*>(pend_dst)[4 * c + i] = v;
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&b[L::B_OR + ob]);
        pend = false;
        return true;
      } else {
        uint32_t o[HD];
        uint32_t lv[8];  // row sum of the FP16 probabilities (column HD of the accumulator)
        if constexpr (HD == 64) {
          uint32_t(&o0)[32] = *reinterpret_cast<uint32_t(*)[32]>(o);
          uint32_t(&o1)[32] = *reinterpret_cast<uint32_t(*)[32]>(o + 32);
          tmem_ld_x32(tS + L::TMEM_O + ob * L::ON, o0);
          tmem_ld_x32(tS + L::TMEM_O + ob * L::ON + 32, o1);
          tmem_ld_x8(tS + L::TMEM_O + ob * L::ON + HD, lv);
          tmem_ld_wait_tied(o0);
          tmem_ld_wait_tied(o1);
        } else {
          if constexpr (HD == 32) {
            tmem_ld_x32(tS + L::TMEM_O + ob * L::ON, o);
          } else if constexpr (HD == 16) {
            tmem_ld_x16(tS + L::TMEM_O + ob * L::ON, o);
          }
          tmem_ld_x8(tS + L::TMEM_O + ob * L::ON + HD, lv);
          tmem_ld_wait_tied(o);
        }
        tmem_ld_wait_tied(lv);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&b[L::B_OR + ob]);
        pend = false;
        const float lsum = __uint_as_float(lv[0]);
        const float pend_inv = (pend_valid && lsum > 0.f) ? 1.f / lsum : 0.f;
        if (pend_store) {
#pragma unroll
          for (int i = 0; i < HD / 8; ++i) {
            uint4 v;
            v.x = pack_half2(__uint_as_float(o[8 * i + 0]) * pend_inv, __uint_as_float(o[8 * i + 1]) * pend_inv);
            v.y = pack_half2(__uint_as_float(o[8 * i + 2]) * pend_inv, __uint_as_float(o[8 * i + 3]) * pend_inv);
            v.z = pack_half2(__uint_as_float(o[8 * i + 4]) * pend_inv, __uint_as_float(o[8 * i + 5]) * pend_inv);
            v.w = pack_half2(__uint_as_float(o[8 * i + 6]) * pend_inv, __uint_as_float(o[8 * i + 7]) * pend_inv);
            if (i < n_out16) reinterpret_cast<uint4*>(pend_dst)[i] = v;
          }
        }
        return true;
      }
    };

    for (int w = NS * static_cast<int>(blockIdx.x) + s; ok && w < n_items; w += G2) {
      const AttnItem item = attn_item(p, w, n_qt);
      const int qi = item.q0 + row;
      __half* dst_row = p.ctx + (static_cast<size_t>(item.b) * p.seq + qi) * D + item.h * p.ctx_hd;
      const int nt = n_tiles(item);
      if (nt == 0) {
        if (qi < p.seq) {
#pragma unroll
          for (int i = 0; i < HD / 8; ++i)
            if (i < n_out16) reinterpret_cast<uint4*>(dst_row)[i] = make_uint4(0, 0, 0, 0);
        }
        continue;
      }
      const int row_lim = p.causal ? min(qi + 1, item.kv_end) : item.kv_end;
      const int ob = it % L::NOB;
      const uint32_t tO = tS + L::TMEM_O + ob * L::ON;
      float m_run = -INFINITY;  // reference maximum of this row (log2 units)
      // Key-mask bytes of the next tile, loaded one tile ahead so their global
      // latency stays off the softmax's path (lane l holds keys k0 + l and k0 + 32 + l).
      const uint8_t* mrow = p.key_mask ? p.key_mask + static_cast<size_t>(item.b) * p.seq : nullptr;
      auto mask_bytes = [&](int k0, uint32_t& m0, uint32_t& m1) {
        const int ka = k0 + lane;
        m0 = (ka < p.seq && mrow[min(ka, p.seq - 1)] != 0) ? 1u : 0u;
        m1 = (ka + 32 < p.seq && mrow[min(ka + 32, p.seq - 1)] != 0) ? 1u : 0u;
      };
      uint32_t mn0 = 1u, mn1 = 1u;
      if (mrow) mask_bytes(0, mn0, mn1);

      for (int j = 0; j < nt; ++j, ++t) {
        const int bb = t % NSB;
        const int k0 = j * BN;
        uint32_t vb[2] = {~0u, ~0u};
        bool mask_partial = false;
        if (mrow) {
          vb[0] = __ballot_sync(~0u, mn0 != 0);
          vb[1] = __ballot_sync(~0u, mn1 != 0);
          mask_partial = (vb[0] & vb[1]) != ~0u;
          if (j + 1 < nt) mask_bytes(k0 + BN, mn0, mn1);
        }
        // Warp-uniform: the masking branch sits between warp-collective TMEM operations.
        const bool need_mask = __any_sync(0xffffffffu, mask_partial || (k0 + BN > row_lim));
        const int lim = row_lim - k0;

        if (!(ok = warp_wait_phase(&b[L::B_SF + bb], (t / NSB) & 1, wd, 0x331))) break;
        tc_fence_after();
        uint32_t sc[2][32];
        tmem_ld_x32(tS + bb * BN, sc[0]);
        tmem_ld_x32(tS + bb * BN + 32, sc[1]);
        tmem_ld_wait_tied(sc[0]);
        tmem_ld_wait_tied(sc[1]);
        if (need_mask) {
#pragma unroll
          for (int g = 0; g < 2; ++g) {
            const int l0 = lim - g * 32;  // keys of this group at or below the causal limit
            const uint32_t bits = (l0 >= 32 ? ~0u : (l0 <= 0 ? 0u : ((1u << l0) - 1u))) & vb[g];
            if (bits != ~0u) {
#pragma unroll
              for (int i = 0; i < 32; ++i)
                if (!(bits & (1u << i))) sc[g][i] = 0xff800000u;  // -inf
            }
          }
        }
        float mg[2];
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          float a[11];
#pragma unroll
          for (int i = 0; i < 10; ++i)
            a[i] = max3(__uint_as_float(sc[g][3 * i]), __uint_as_float(sc[g][3 * i + 1]),
                        __uint_as_float(sc[g][3 * i + 2]));
          a[10] = fmaxf(__uint_as_float(sc[g][30]), __uint_as_float(sc[g][31]));
          mg[g] = max3(max3(a[0], a[1], a[2]), max3(a[3], a[4], a[5]), max3(a[6], a[7], max3(a[8], a[9], a[10])));
        }
        const float m_tile = fmaxf(mg[0], mg[1]) * sl2;
        // Rows that have seen no valid key hold nothing in O and take the new
        // maximum without a rescale.
        float m_new = m_run;
        bool resc = false;
        // FP32 exponentials of x <= 8 keep P <= 2^8, well inside FP16.
        constexpr float kLazy = 8.0f;
        if (m_tile > m_run + kLazy) {
          resc = (m_run != -INFINITY);
          m_new = m_tile;
        }
        const float m_use = (m_new == -INFINITY) ? 0.f : m_new;

        if (__any_sync(0xffffffffu, resc)) {
          // O must hold every earlier tile: wait for P.V of tile t-1 (j > 0 here).
          const int tp = t - 1;
          if (!(ok = warp_wait_phase(&b[L::B_PE + (tp % NSB)], (tp / NSB) & 1, wd, 0x332))) break;
          tc_fence_after();
          const float corr = resc ? ex2_approx(m_run - m_new) : 1.f;
#pragma unroll 1
          for (int c = 0; c < L::ON; c += 16) {  // O and l, 16 columns at a time: the scores stay in registers
            uint32_t o[16];
            tmem_ld_x16_sync(tO + c, o);
#pragma unroll
            for (int d = 0; d < 16; ++d) o[d] = __float_as_uint(__uint_as_float(o[d]) * corr);
            tmem_st_x16(tO + c, o);
          }
          tmem_st_wait();
        }
        m_run = m_new;

        // Probabilities: FP16 pairs over columns 0..31 of S_bb (their row sum
        // comes from the P.[V | 1] MMA).  P.V of tile t-2, the last reader of
        // this buffer, finished before S_t was computed into it.
        const uint64_t negm = f2_pack(-m_use, -m_use);
        // FMA-pipe pairs take y = saturate((s * scale - m + 26) / 128) from one fma per score.
        const float y_scale = sl2 * kExp2YScale;
        const float y_bias = fmaf(-m_use, kExp2YScale, kExp2YBias);
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            if ((e & 7) < kDbExpFmaOf8<HD>) {
              const uint64_t pp = exp2_pair_fma_y(f2_pack(fma_sat(__uint_as_float(sc[g][2 * e]), y_scale, y_bias),
                                                          fma_sat(__uint_as_float(sc[g][2 * e + 1]), y_scale, y_bias)));
              pk[e] = pack_half2(f2_lo(pp), f2_hi(pp));
            } else {
              const uint64_t xx =
                  ffma2(f2_pack(__uint_as_float(sc[g][2 * e]), __uint_as_float(sc[g][2 * e + 1])), sl2x2, negm);
              pk[e] = pack_half2(ex2_approx(f2_lo(xx)), ex2_approx(f2_hi(xx)));
            }
          }
          tmem_st_x16(tS + bb * BN + 16 * g, pk);
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&b[L::B_PF + bb]);
        if (j == 0 && pend && !(ok = finish_item())) break;
      }
      if (!ok) break;

      pend = true;
      pend_it = it;
      pend_dst = dst_row;
      pend_store = qi < p.seq;
      pend_valid =
          p.key_mask == nullptr || (pend_store && p.key_mask[static_cast<size_t>(item.b) * p.seq + qi] != 0);
      ++it;
    }
    if (ok && pend) ok = finish_item();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == L::W_MMA) {
    tc_fence_after();
    tmem_dealloc(tmem_base, L::TMEM_COLS);
  }
}

}  // namespace tt
