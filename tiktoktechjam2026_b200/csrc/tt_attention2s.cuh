// Two-stream causal attention forward for head_dim <= 32 (sm_100a).
//
// Same contract and numerics as attn_fwd_kernel (tt_attention.cuh; replaces
// custom_kernel/triton_attention.py:126-232 of the reference), laid out for
// latency hiding: one CTA per SM runs two independent pipelines ("streams"),
// each with its own 4 softmax warps (a 128-query tile of its own work item),
// its own TMA producer warp (8 + s) and its own MMA-issuer warp (10 + s), so
// every SM sub-partition holds two softmax warps and no role ever waits on the
// other stream.  Warp 10 also allocates the CTA's TMEM (256 columns per stream).
//
// Per stream and key tile t:
//   S_t = Q K_t^T          TMEM (128 FP32 columns, single buffer per stream)
//   softmax, two passes over S_t in TMEM: pass 1 the row max (3-input max
//   tree), pass 2 the FP32 exp2 (MUFU) of S*scale*log2(e) - m, rounded to FP16
//   into a 128B-swizzled K-major P tile (single buffer per stream)
//   O_t = P_t [V_t | 1]    TMEM (double buffered); column hd is the row sum
//   the FP32 register accumulator takes O_t with the running-max correction.
// Items (sequence*head, query tile) are dealt heavy-first: stream s of CTA c
// takes items 2c+s, 2c+s+2G, ... (G = gridDim.x).
#pragma once

#include <type_traits>

#include "tt_attention.cuh"

namespace tt {

template <int HD>
struct Attn2sLayout {
  static constexpr int BM = 128, BN = 128, NST = 2;
  static constexpr int HDX = HD + 16;
  static constexpr int Q_BYTES = BM * HD * 2;
  static constexpr int K_BYTES = BN * HD * 2;
  static constexpr int VBLK = HDX * 128;
  static constexpr int V_BYTES = 2 * VBLK;
  static constexpr int V_TMA_BYTES = 2 * HD * 128;
  static constexpr int P_BYTES = BM * BN * 2;
  // Per-stream region: Q[2] | K[NST] | V[NST] | P
  static constexpr int S_Q = 0;
  static constexpr int S_K = S_Q + 2 * Q_BYTES;
  static constexpr int S_V = S_K + NST * K_BYTES;
  static constexpr int S_P = S_V + NST * V_BYTES;
  static constexpr int STREAM_BYTES = S_P + P_BYTES;
  // Per-stream barriers: q_full[2] q_empty[2] kv_full[NST] kv_empty[NST]
  // s_full s_free p_full p_empty o_full[2] o_free[2]
  static constexpr int B_QF = 0, B_QE = 2, B_KF = 4, B_KE = 4 + NST, B_SF = 4 + 2 * NST,
                       B_SR = B_SF + 1, B_PF = B_SF + 2, B_PE = B_SF + 3, B_OF = B_SF + 4,
                       B_OR = B_SF + 6;
  static constexpr int NBAR_STREAM = B_SF + 8;
  static constexpr int OFF_BAR = 2 * STREAM_BYTES;
  static constexpr int OFF_DONE = OFF_BAR + 2 * NBAR_STREAM * 8;  // done[2]
  static constexpr int OFF_MISC = OFF_DONE + 16;
  static constexpr int SMEM_ALLOC = OFF_MISC + 16 + 1024;
  static constexpr int TMEM_COLS = 512, TMEM_STREAM = 256, TMEM_O = 128;
  static_assert(TMEM_O + 2 * HDX <= TMEM_STREAM, "TMEM budget");
  static_assert(HD == 16 || HD == 32, "two-stream kernel covers head_dim 16 and 32");
  static_assert(STREAM_BYTES % 1024 == 0, "alignment");
};

template <int HD>
__global__ void __launch_bounds__(384, 1)
    attn2s_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, const AttnParams p, int n_items) {
  using L = Attn2sLayout<HD>;
  constexpr int BM = L::BM, BN = L::BN, NST = L::NST, HDX = L::HDX;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_qt = (p.seq + BM - 1) / BM;
  const int D = p.heads * HD;
  const int G2 = 2 * static_cast<int>(gridDim.x);
  uint64_t* bars_all = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* done = reinterpret_cast<uint64_t*>(smem + L::OFF_DONE);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);

  if (threadIdx.x == 0) {
    mbar_init(&done[0], 1);
    mbar_init(&done[1], 1);
    for (int s = 0; s < 2; ++s) {
      uint64_t* b = bars_all + s * L::NBAR_STREAM;
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
      mbar_init(&b[L::B_SF], 1);
      mbar_init(&b[L::B_SR], 4);
      mbar_init(&b[L::B_PF], 4);
      mbar_init(&b[L::B_PE], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  // Rows HD .. HD+15 of every V block: row HD all ones (FP16 1.0), the rest zero.
  for (int i = threadIdx.x; i < 2 * NST * 2 * 16 * 32; i += blockDim.x) {
    const int word = i & 31, r = (i >> 5) & 15, blk = i >> 9;  // blk = stream*2NST + stage*2 + half
    const int s = blk / (2 * NST), rem = blk % (2 * NST);
    uint8_t* vbase = smem + s * L::STREAM_BYTES + L::S_V + (rem >> 1) * L::V_BYTES + (rem & 1) * L::VBLK;
    reinterpret_cast<uint32_t*>(vbase + (HD + r) * 128)[word] = r == 0 ? 0x3C003C00u : 0u;
  }
  fence_proxy_async_smem();
  if (warp == 10) {
    tmem_alloc(tmem_slot, L::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const Watchdog wd{p.err, abort_flag, p.timeout_ns};

  auto first_item = [&](int w) -> int {  // first item >= w of this stream with work
    while (w < n_items && attn_item(p, w, n_qt).n == 0) w += G2;
    return w;
  };

  if (warp == 8 || warp == 9) {
    // ------------------------------------------------------------ producer of stream warp-8
    if (lane == 0) {
      const int s = warp - 8;
      uint64_t* b = bars_all + s * L::NBAR_STREAM;
      uint8_t* sb = smem + s * L::STREAM_BYTES;
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      int t = 0, it = 0;
      bool ok = true;
      for (int w = first_item(2 * static_cast<int>(blockIdx.x) + s); ok && w < n_items;
           w = first_item(w + G2)) {
        const AttnItem item = attn_item(p, w, n_qt);
        const int qb = it & 1;
        if (!(ok = wait_phase(&b[L::B_QE + qb], ((it >> 1) & 1) ^ 1, wd, 0x111))) break;
        mbar_arrive_expect_tx(&b[L::B_QF + qb], L::Q_BYTES);
        tma_load_3d(sb + L::S_Q + qb * L::Q_BYTES, &tmQ, &b[L::B_QF + qb], 0, item.q0, item.bh);
        ++it;
        for (int j = 0; j < item.n; ++j) {
          const int st = t % NST;
          if (!(ok = wait_phase(&b[L::B_KE + st], ((t / NST) & 1) ^ 1, wd, 0x112))) break;
          mbar_arrive_expect_tx(&b[L::B_KF + st], L::K_BYTES + L::V_TMA_BYTES);
          tma_load_3d(sb + L::S_K + st * L::K_BYTES, &tmK, &b[L::B_KF + st], 0, j * BN, item.bh);
          uint8_t* v_dst = sb + L::S_V + st * L::V_BYTES;
          tma_load_3d(v_dst, &tmV, &b[L::B_KF + st], j * BN, 0, item.bh);
          tma_load_3d(v_dst + L::VBLK, &tmV, &b[L::B_KF + st], j * BN + 64, 0, item.bh);
          ++t;
        }
      }
      // Let every copy this stream started land before the CTA may exit.
      for (int i = (it > 2 ? it - 2 : 0); i < it; ++i)
        wait_drain(&b[L::B_QF + (i & 1)], (i >> 1) & 1, kDrainLimitNs);
      for (int i = (t > NST ? t - NST : 0); i < t; ++i)
        wait_drain(&b[L::B_KF + i % NST], (i / NST) & 1, kDrainLimitNs);
    }
  } else if (warp == 10 || warp == 11) {
    // ------------------------------------------------------------ MMA issuer of stream warp-10
    if (lane == 0) {
      const int s = warp - 10;
      uint64_t* b = bars_all + s * L::NBAR_STREAM;
      const uint32_t sb = smem_u32(smem + s * L::STREAM_BYTES);
      const uint32_t tS = tmem_base + s * L::TMEM_STREAM;
      constexpr uint32_t kSwQK = swizzle_kind_for_bytes(HD * 2);
      constexpr uint32_t kSboQK = 8 * HD * 2;
      const uint32_t idesc_s = umma_idesc_f16_f32(BM, BN);
      const uint32_t idesc_o = umma_idesc_f16_f32(BM, HDX);
      // S cursor: item w_s, tile j_s, stream tile u, item count it_s.
      int w_s = first_item(2 * static_cast<int>(blockIdx.x) + s), j_s = 0, u = 0, it_s = 0;
      AttnItem item_s;
      if (w_s < n_items) item_s = attn_item(p, w_s, n_qt);
      auto issue_s = [&]() -> bool {
        const int st = u % NST, qb = it_s & 1;
        if (j_s == 0 && !wait_phase(&b[L::B_QF + qb], (it_s >> 1) & 1, wd, 0x211)) return false;
        if (!wait_phase(&b[L::B_KF + st], (u / NST) & 1, wd, 0x212)) return false;
        if (u > 0 && !wait_phase(&b[L::B_SR], (u - 1) & 1, wd, 0x213)) return false;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint64_t da = umma_sdesc(sb + L::S_Q + qb * L::Q_BYTES + kk * 32, kSboQK, kSwQK);
          const uint64_t db = umma_sdesc(sb + L::S_K + st * L::K_BYTES + kk * 32, kSboQK, kSwQK);
          umma_f16(tS, da, db, idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(&b[L::B_SF]);
        if (j_s == item_s.n - 1) umma_commit(&b[L::B_QE + qb]);
        ++u;
        if (++j_s == item_s.n) {
          j_s = 0;
          ++it_s;
          w_s = first_item(w_s + G2);
          if (w_s < n_items) item_s = attn_item(p, w_s, n_qt);
        }
        return true;
      };
      bool ok = true;
      if (w_s < n_items) ok = issue_s();
      // S of tile t+1 is issued before P.V of tile t (the softmax frees S_t
      // just before it publishes P_t), so the next scores are ready early.
      for (int t = 0; ok && t < u; ++t) {
        if (w_s < n_items && !(ok = issue_s())) break;
        const int ob = t & 1, st = t % NST;
        if (!(ok = wait_phase(&b[L::B_PF], t & 1, wd, 0x214))) break;
        if (!(ok = wait_phase(&b[L::B_OR + ob], ((t >> 1) & 1) ^ 1, wd, 0x215))) break;
        tc_fence_after();
        const uint32_t tO = tS + L::TMEM_O + ob * HDX;
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint64_t da = umma_sdesc(sb + L::S_P + (kk >> 2) * (BM * 128) + (kk & 3) * 32, 1024, kSw128);
          const uint64_t db =
              umma_sdesc(sb + L::S_V + st * L::V_BYTES + (kk >> 2) * L::VBLK + (kk & 3) * 32, 1024, kSw128);
          umma_f16(tO, da, db, idesc_o, kk > 0 ? 1u : 0u);
        }
        umma_commit(&b[L::B_OF + ob]);
        umma_commit(&b[L::B_KE + st]);
        umma_commit(&b[L::B_PE]);
      }
      // All MMAs this thread issued must finish before TMEM is released.
      umma_commit(&done[s]);
      wait_drain(&done[s], 0, kDrainLimitNs);
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int s = warp >> 2;  // stream
    const int wq = warp & 3;  // TMEM lane quadrant
    const int row = wq * 32 + lane;
    uint64_t* b = bars_all + s * L::NBAR_STREAM;
    const uint32_t tS = tmem_base + (static_cast<uint32_t>(wq * 32) << 16) + s * L::TMEM_STREAM;
    const uint32_t p_base = smem_u32(smem + s * L::STREAM_BYTES + L::S_P);
    const float sl2 = p.scale_log2;
    bool ok = true;
    int t = 0;
    for (int w = 2 * static_cast<int>(blockIdx.x) + s; ok && w < n_items; w += G2) {
      const AttnItem item = attn_item(p, w, n_qt);
      const int qi = item.q0 + row;
      __half* dst_row = p.ctx + (static_cast<size_t>(item.b) * p.seq + qi) * D + item.h * HD;
      if (item.n == 0) {
        if (qi < p.seq) {
#pragma unroll
          for (int i = 0; i < HD / 8; ++i) reinterpret_cast<uint4*>(dst_row)[i] = make_uint4(0, 0, 0, 0);
        }
        continue;
      }
      const int row_lim = p.causal ? min(qi + 1, item.kv_end) : item.kv_end;
      float m_run = -INFINITY, l_run = 0.f, corr_prev = 1.f;
      float o[HD];
#pragma unroll
      for (int d = 0; d < HD; ++d) o[d] = 0.f;

      auto consume_o = [&](int tt, float c) -> bool {
        const int ob = tt & 1;
        if (!warp_wait_phase(&b[L::B_OF + ob], (tt >> 1) & 1, wd, 0x313)) return false;
        tc_fence_after();
#pragma unroll
        for (int g = 0; g < HDX / 16; ++g) {
          uint32_t rr[16];
          tmem_ld_x16_sync(tS + L::TMEM_O + ob * HDX + g * 16, rr);
#pragma unroll
          for (int d = 0; d < 16; ++d) {
            const int col = g * 16 + d;
            if (col < HD) o[col] = fmaf(o[col], c, __uint_as_float(rr[d]));
            if (col == HD) l_run = fmaf(l_run, c, __uint_as_float(rr[d]));
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&b[L::B_OR + ob]);
        return true;
      };

      for (int j = 0; j < item.n; ++j, ++t) {
        const int k0 = j * BN;
        uint32_t vb[4] = {~0u, ~0u, ~0u, ~0u};
        bool mask_partial = false;
        if (p.key_mask != nullptr) {
          const uint8_t* mrow = p.key_mask + static_cast<size_t>(item.b) * p.seq;
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            const int ka = k0 + lane + 32 * g;
            vb[g] = __ballot_sync(~0u, ka < p.seq && mrow[min(ka, p.seq - 1)] != 0);
          }
          mask_partial = (vb[0] & vb[1] & vb[2] & vb[3]) != ~0u;
        }
        // The masked and unmasked variants below contain warp-collective TMEM
        // loads, so the choice must be the same for the whole warp (on a causal
        // diagonal tile the last row needs no mask while the others do).
        const bool need_mask = __any_sync(0xffffffffu, mask_partial || (k0 + BN > row_lim));
        const int lim = row_lim - k0;

        if (!(ok = warp_wait_phase(&b[L::B_SF], t & 1, wd, 0x311))) break;
        tc_fence_after();
        // Pass 1: row max over the 128 scores (two 64-column halves).
        float mt = -INFINITY;
        auto pass1 = [&](auto masked) {
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            uint32_t r0[32], r1[32];
            tmem_ld_x32(tS + hh * 64, r0);
            tmem_ld_x32(tS + hh * 64 + 32, r1);
            tmem_ld_wait_tied(r0);
            tmem_ld_wait_tied(r1);
            float x[64];
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              x[i] = __uint_as_float(r0[i]);
              x[32 + i] = __uint_as_float(r1[i]);
            }
            if constexpr (decltype(masked)::value) {
              const uint32_t w0 = hh ? vb[2] : vb[0], w1 = hh ? vb[3] : vb[1];
              const int l0 = lim - hh * 64;
#pragma unroll
              for (int i = 0; i < 64; ++i) {
                const bool valid = (i < l0) && (((i < 32 ? w0 : w1) >> (i & 31)) & 1u);
                x[i] = valid ? x[i] : -INFINITY;
              }
            }
            float m1[22];
#pragma unroll
            for (int i = 0; i < 21; ++i) m1[i] = max3(x[3 * i], x[3 * i + 1], x[3 * i + 2]);
            m1[21] = x[63];
            float m2[8];
#pragma unroll
            for (int i = 0; i < 7; ++i) m2[i] = max3(m1[3 * i], m1[3 * i + 1], m1[3 * i + 2]);
            m2[7] = m1[21];
            mt = max3(mt, max3(m2[0], m2[1], m2[2]), max3(m2[3], m2[4], max3(m2[5], m2[6], m2[7])));
          }
        };
        if (need_mask)
          pass1(std::true_type{});
        else
          pass1(std::false_type{});
        const float m_new = fmaxf(m_run, mt * sl2);
        const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
        const float corr = ex2_approx(m_run - m_use);

        if (!(ok = warp_wait_phase(&b[L::B_PE], (t & 1) ^ 1, wd, 0x312))) break;
        // Pass 2: probabilities, FP16, into the swizzled P tile (32 columns per chunk).
        const uint32_t prow = p_base + row * 128;
        auto pass2 = [&](auto masked) {
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            uint32_t r[32];
            tmem_ld_x32_sync(tS + g * 32, r);
            if (g == 3) {
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(&b[L::B_SR]);  // S buffer may be overwritten now
            }
            float x[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) x[i] = fmaf(__uint_as_float(r[i]), sl2, -m_use);
            if constexpr (decltype(masked)::value) {
              const uint32_t wbits = g == 0 ? vb[0] : g == 1 ? vb[1] : g == 2 ? vb[2] : vb[3];
              const int l0 = lim - g * 32;
#pragma unroll
              for (int i = 0; i < 32; ++i) {
                const bool valid = (i < l0) && ((wbits >> i) & 1u);
                x[i] = valid ? x[i] : -INFINITY;
              }
            }
            uint32_t pk[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) pk[e] = pack_half2(ex2_approx(x[2 * e]), ex2_approx(x[2 * e + 1]));
            // 16-byte chunk ch = 4g + q of the row; 128B-swizzled within each 64-key block.
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int ch = g * 4 + q;
              const uint32_t addr = prow + (ch >> 3) * (BM * 128) + (((ch & 7) ^ (row & 7)) << 4);
              st_shared_v4(addr, pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
            }
          }
        };
        if (need_mask)
          pass2(std::true_type{});
        else
          pass2(std::false_type{});
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&b[L::B_PF]);
        m_run = m_new;

        if (j > 0 && !(ok = consume_o(t - 1, corr_prev))) break;
        corr_prev = corr;
      }
      if (!ok) break;
      if (!(ok = consume_o(t - 1, corr_prev))) break;

      if (qi < p.seq) {
        const bool row_valid =
            p.key_mask == nullptr || p.key_mask[static_cast<size_t>(item.b) * p.seq + qi] != 0;
        const float inv = (row_valid && l_run > 0.f) ? 1.f / l_run : 0.f;
#pragma unroll
        for (int i = 0; i < HD / 8; ++i) {
          uint4 v;
          v.x = pack_half2(o[8 * i + 0] * inv, o[8 * i + 1] * inv);
          v.y = pack_half2(o[8 * i + 2] * inv, o[8 * i + 3] * inv);
          v.z = pack_half2(o[8 * i + 4] * inv, o[8 * i + 5] * inv);
          v.w = pack_half2(o[8 * i + 6] * inv, o[8 * i + 7] * inv);
          reinterpret_cast<uint4*>(dst_row)[i] = v;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 10) {
    tc_fence_after();
    tmem_dealloc(tmem_base, L::TMEM_COLS);
  }
}

}  // namespace tt
