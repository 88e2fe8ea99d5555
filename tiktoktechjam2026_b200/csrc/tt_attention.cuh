// Causal (or full) multi-head attention forward for sm_100a.
//
// Replaces the reference's FP16 online-softmax attention
// (custom_kernel/triton_attention.py:126-232, wrapper :341-390) and the SDPA
// fallback it uses elsewhere (mixed_precision/transformer.py:157-198).
//
// One CTA = one (sequence, head, 128-query tile).  Roles:
//   warp 4      TMA producer: Q once, then K / V^T tiles of 128 keys (2 stages)
//   warp 5      TMEM allocator and single-thread tcgen05.mma issuer
//   warps 0..3  softmax: one query row per thread (TMEM lane = row)
// Per key tile j:
//   S_j   = Q K_j^T        tcgen05.mma -> TMEM (128 columns, FP32)
//   P_j   = exp2(S_j * scale*log2(e) - m_j)   FP32 in registers, FP16 into a
//           128B-swizzled K-major shared tile (double buffered)
//   O_j   = P_j V_j        tcgen05.mma -> TMEM (head_dim columns, double
//           buffered), folded into the FP32 register accumulator with the
//           running-max correction one iteration later.
// Key tiles strictly above the causal diagonal, and key tiles past the last
// valid key of a padded sequence, are never loaded.  The context of every
// padded query row (mask byte 0) is zero; query tiles that lie wholly in a
// sequence's padding skip all work.  (The reference computes padded rows and
// zeroes them only on the model output, mixed_precision/transformer.py:697-698;
// valid rows never read padded rows, whose keys are masked.)  A valid query
// row always sees at least itself as a valid key, so no row divides by zero.
#pragma once

#include "tt_ptx.cuh"

namespace tt {

struct AttnParams {
  int batch, seq, heads;
  int seq_pad;                  // row length of the V^T buffer (multiple of 8)
  int causal;
  float scale_log2;             // head_dim^-0.5 * log2(e)
  const uint8_t* key_mask;      // [batch, seq], nonzero = valid; nullptr = all valid
  const int* kv_end;            // [batch]: 1 + index of the last valid key (with key_mask)
  __half* ctx;                  // [batch, seq, heads * HD]
  unsigned int* err;
  unsigned long long timeout_ns;
};

template <int HD>
struct AttnLayout {
  static constexpr int BM = 128, BN = 128, NST = 2;
  static constexpr int Q_BYTES = BM * HD * 2;
  static constexpr int K_BYTES = BN * HD * 2;
  static constexpr int V_BYTES = HD * BN * 2;
  static constexpr int P_BYTES = BM * BN * 2;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + Q_BYTES;
  static constexpr int OFF_V = OFF_K + NST * K_BYTES;
  static constexpr int OFF_P = OFF_V + NST * V_BYTES;
  static constexpr int OFF_BAR = OFF_P + 2 * P_BYTES;
  // q_full, kv_full[2], kv_empty[2], s_full, s_free, p_full[2], p_empty[2],
  // o_full[2], o_free[2], done
  static constexpr int NBAR = 1 + 2 * NST + 2 + 8 + 1;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int BYTES = OFF_MISC + 16;
  static constexpr int SMEM_ALLOC = BYTES + 1024;  // slack for 1024-byte alignment
  static constexpr int TMEM_COLS = 256;            // S: 128 cols, O: 2 x HD cols
  static_assert(128 + 2 * HD <= TMEM_COLS, "TMEM budget");
  static_assert(HD % 16 == 0 && HD >= 16 && HD <= 64, "head_dim");
};

template <int HD>
__global__ void __launch_bounds__(192, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const AttnParams p) {
  using L = AttnLayout<HD>;
  constexpr int BM = L::BM, BN = L::BN, NST = L::NST;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.x;
  const int b = bh / p.heads, h = bh - b * p.heads;
  const int qt = static_cast<int>(gridDim.y) - 1 - static_cast<int>(blockIdx.y);  // heavy first
  const int q0 = qt * BM;
  const int kv_end_b = p.key_mask ? p.kv_end[b] : p.seq;
  const int D = p.heads * HD;

  if (q0 >= kv_end_b) {
    // Every query row of this tile is padding: its context is defined as zero.
    if (threadIdx.x < BM) {
      const int qi = q0 + threadIdx.x;
      if (qi < p.seq) {
        uint4* dst = reinterpret_cast<uint4*>(p.ctx + (static_cast<size_t>(b) * p.seq + qi) * D +
                                              h * HD);
#pragma unroll
        for (int i = 0; i < HD / 8; ++i) dst[i] = make_uint4(0, 0, 0, 0);
      }
    }
    return;
  }
  const int kv_limit = p.causal ? min(q0 + BM, kv_end_b) : kv_end_b;
  const int n_tiles = (kv_limit + BN - 1) / BN;

  uint8_t* sQ = smem + L::OFF_Q;
  uint8_t* sK = smem + L::OFF_K;
  uint8_t* sV = smem + L::OFF_V;
  uint8_t* sP = smem + L::OFF_P;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = bars + 1 + NST;
  uint64_t* s_full = bars + 1 + 2 * NST;
  uint64_t* s_free = s_full + 1;
  uint64_t* p_full = s_full + 2;
  uint64_t* p_empty = s_full + 4;
  uint64_t* o_full = s_full + 6;
  uint64_t* o_free = s_full + 8;
  uint64_t* done = s_full + 10;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < NST; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 4);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&p_full[i], 4);
      mbar_init(&p_empty[i], 1);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_free[i], 4);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, L::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const Watchdog wd{p.err, abort_flag, p.timeout_ns};

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(q_full, L::Q_BYTES);
      tma_load_3d(sQ, &tmQ, q_full, 0, q0, bh);
      int issued = 0;
      for (int j = 0; j < n_tiles; ++j) {
        const int st = j % NST;
        if (!wait_phase(&kv_empty[st], ((j / NST) & 1) ^ 1, wd, 0x101)) break;
        mbar_arrive_expect_tx(&kv_full[st], L::K_BYTES + L::V_BYTES);
        tma_load_3d(sK + st * L::K_BYTES, &tmK, &kv_full[st], 0, j * BN, bh);
        uint8_t* v_dst = sV + st * L::V_BYTES;
        tma_load_3d(v_dst, &tmV, &kv_full[st], j * BN, 0, bh);
        tma_load_3d(v_dst + HD * 128, &tmV, &kv_full[st], j * BN + 64, 0, bh);
        issued = j + 1;
      }
      // Let every copy this CTA started land before the CTA may exit.
      wait_drain(q_full, 0, kDrainLimitNs);
      for (int j = (issued > NST ? issued - NST : 0); j < issued; ++j)
        wait_drain(&kv_full[j % NST], (j / NST) & 1, kDrainLimitNs);
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t kSwQK = swizzle_kind_for_bytes(HD * 2);
      constexpr uint32_t kSboQK = 8 * HD * 2;
      const uint32_t idesc_s = umma_idesc_f16_f32(BM, BN);
      const uint32_t idesc_o = umma_idesc_f16_f32(BM, HD);
      const uint32_t aQ = smem_u32(sQ), aK = smem_u32(sK), aV = smem_u32(sV), aP = smem_u32(sP);
      const uint32_t tS = tmem_base;
      bool ok = wait_phase(q_full, 0, wd, 0x201);
      auto issue_s = [&](int j) -> bool {
        const int st = j % NST;
        if (!wait_phase(&kv_full[st], (j / NST) & 1, wd, 0x202)) return false;
        if (j > 0 && !wait_phase(s_free, (j - 1) & 1, wd, 0x203)) return false;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint64_t da = umma_sdesc(aQ + kk * 32, kSboQK, kSwQK);
          const uint64_t db = umma_sdesc(aK + st * L::K_BYTES + kk * 32, kSboQK, kSwQK);
          umma_f16(tS, da, db, idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(s_full);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; ok && j < n_tiles; ++j) {
        if (j + 1 < n_tiles && !(ok = issue_s(j + 1))) break;
        const int bs = j & 1, st = j % NST;
        if (!(ok = wait_phase(&p_full[bs], (j >> 1) & 1, wd, 0x204))) break;
        if (!(ok = wait_phase(&o_free[bs], ((j >> 1) & 1) ^ 1, wd, 0x205))) break;
        tc_fence_after();
        const uint32_t tO = tmem_base + 128 + bs * HD;
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint64_t da =
              umma_sdesc(aP + bs * L::P_BYTES + (kk >> 2) * (BM * 128) + (kk & 3) * 32, 1024, kSw128);
          const uint64_t db =
              umma_sdesc(aV + st * L::V_BYTES + (kk >> 2) * (HD * 128) + (kk & 3) * 32, 1024, kSw128);
          umma_f16(tO, da, db, idesc_o, kk > 0 ? 1u : 0u);
        }
        umma_commit(&o_full[bs]);
        umma_commit(&kv_empty[st]);
        umma_commit(&p_empty[bs]);
      }
      // All MMAs this thread issued must finish before TMEM is released.
      umma_commit(done);
      wait_drain(done, 0, kDrainLimitNs);
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int row = threadIdx.x;  // 0..127 == TMEM lane
    const int qi = q0 + row;
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    const uint32_t tS = tmem_base + lane_base;
    const int row_lim = p.causal ? min(qi + 1, kv_end_b) : kv_end_b;
    const uint32_t p_base = smem_u32(sP);
    const float sl2 = p.scale_log2;
    float m_run = -INFINITY, l_run = 0.f, corr_prev = 1.f;
    float o[HD];
#pragma unroll
    for (int d = 0; d < HD; ++d) o[d] = 0.f;

    auto consume_o = [&](int jj, float c) -> bool {
      const int bs = jj & 1;
      if (!warp_wait_phase(&o_full[bs], (jj >> 1) & 1, wd, 0x303)) return false;
      tc_fence_after();
      const uint32_t tO = tS + 128 + bs * HD;
      if constexpr (HD == 16) {
        uint32_t r[16];
        tmem_ld_x16(tO, r);
        tmem_ld_wait();
#pragma unroll
        for (int d = 0; d < 16; ++d) o[d] = fmaf(o[d], c, __uint_as_float(r[d]));
      } else {
#pragma unroll
        for (int g = 0; g < HD / 32; ++g) {
          uint32_t r[32];
          tmem_ld_x32(tO + g * 32, r);
          tmem_ld_wait();
#pragma unroll
          for (int d = 0; d < 32; ++d) o[g * 32 + d] = fmaf(o[g * 32 + d], c, __uint_as_float(r[d]));
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_free[bs]);
      return true;
    };

    bool ok = true;
    for (int j = 0; j < n_tiles; ++j) {
      const int k0 = j * BN;
      uint32_t vb0 = ~0u, vb1 = ~0u, vb2 = ~0u, vb3 = ~0u;
      bool mask_partial = false;
      if (p.key_mask != nullptr) {
        const uint8_t* mrow = p.key_mask + static_cast<size_t>(b) * p.seq;
        const int ka = k0 + lane;
        vb0 = __ballot_sync(~0u, ka < p.seq && mrow[min(ka, p.seq - 1)] != 0);
        vb1 = __ballot_sync(~0u, ka + 32 < p.seq && mrow[min(ka + 32, p.seq - 1)] != 0);
        vb2 = __ballot_sync(~0u, ka + 64 < p.seq && mrow[min(ka + 64, p.seq - 1)] != 0);
        vb3 = __ballot_sync(~0u, ka + 96 < p.seq && mrow[min(ka + 96, p.seq - 1)] != 0);
        mask_partial = (vb0 & vb1 & vb2 & vb3) != ~0u;
      }
      const bool need_mask = mask_partial || (k0 + BN > row_lim);

      if (!(ok = warp_wait_phase(s_full, j & 1, wd, 0x301))) break;
      tc_fence_after();
      float x[BN];
#pragma unroll
      for (int g = 0; g < BN / 32; ++g) {
        uint32_t r[32];
        tmem_ld_x32(tS + g * 32, r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) x[g * 32 + i] = __uint_as_float(r[i]) * sl2;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_free);

      if (need_mask) {
        const int lim = row_lim - k0;
#pragma unroll
        for (int c = 0; c < BN; ++c) {
          const uint32_t wbits = (c < 32) ? vb0 : (c < 64) ? vb1 : (c < 96) ? vb2 : vb3;
          const bool valid = (c < lim) && ((wbits >> (c & 31)) & 1u);
          x[c] = valid ? x[c] : -INFINITY;
        }
      }
      float mt = x[0];
#pragma unroll
      for (int c = 1; c < BN; ++c) mt = fmaxf(mt, x[c]);
      const float m_new = fmaxf(m_run, mt);
      const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
      const float corr = ex2_approx(m_run - m_use);

      const int bs = j & 1;
      if (!(ok = warp_wait_phase(&p_empty[bs], ((j >> 1) & 1) ^ 1, wd, 0x302))) break;
      float ls = 0.f;
      const uint32_t prow = p_base + bs * L::P_BYTES + row * 128;
#pragma unroll
      for (int ch = 0; ch < BN / 8; ++ch) {
        uint32_t pk[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float p0 = ex2_approx(x[ch * 8 + 2 * e] - m_use);
          const float p1 = ex2_approx(x[ch * 8 + 2 * e + 1] - m_use);
          ls += p0 + p1;
          pk[e] = pack_half2(p0, p1);
        }
        const uint32_t addr = prow + (ch >> 3) * (BM * 128) + (((ch & 7) ^ (row & 7)) << 4);
        st_shared_v4(addr, pk[0], pk[1], pk[2], pk[3]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[bs]);
      l_run = l_run * corr + ls;
      m_run = m_new;

      if (j > 0 && !(ok = consume_o(j - 1, corr_prev))) break;
      corr_prev = corr;
    }
    if (ok) ok = consume_o(n_tiles - 1, corr_prev);

    if (ok && qi < p.seq) {
      // Padded query rows (mask byte 0) get a zero context, like whole padded tiles.
      const bool row_valid =
          p.key_mask == nullptr || p.key_mask[static_cast<size_t>(b) * p.seq + qi] != 0;
      const float inv = (row_valid && l_run > 0.f) ? 1.f / l_run : 0.f;
      uint4* dst = reinterpret_cast<uint4*>(p.ctx + (static_cast<size_t>(b) * p.seq + qi) * D + h * HD);
#pragma unroll
      for (int i = 0; i < HD / 8; ++i) {
        uint4 v;
        v.x = pack_half2(o[8 * i + 0] * inv, o[8 * i + 1] * inv);
        v.y = pack_half2(o[8 * i + 2] * inv, o[8 * i + 3] * inv);
        v.z = pack_half2(o[8 * i + 4] * inv, o[8 * i + 5] * inv);
        v.w = pack_half2(o[8 * i + 6] * inv, o[8 * i + 7] * inv);
        dst[i] = v;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem_base, L::TMEM_COLS);
  }
}

}  // namespace tt
