// Causal (or full) multi-head attention forward for sm_100a.
//
// Replaces the reference's FP16 online-softmax attention
// (custom_kernel/triton_attention.py:126-232, wrapper :341-390) and the SDPA
// fallback it uses elsewhere (mixed_precision/transformer.py:157-198).
//
// Persistent kernel: one CTA per SM walks a static, heavy-first list of work
// items (sequence*head, 128-query tile).  Roles:
//   warp 4      TMA producer: Q (double buffered), then K / V^T tiles of 128
//               keys through an NST-deep ring, running ahead across items
//   warp 5      TMEM allocator and single-thread tcgen05.mma issuer
//   warps 0..3  softmax: one query row per thread (TMEM lane = row)
// Per key tile t (counted across the CTA's items):
//   S_t = Q K_t^T      tcgen05.mma -> TMEM S[t&1] (128 FP32 columns), issued
//                      one tile ahead so it overlaps the softmax of tile t-1
//   P_t = exp2(S_t * scale*log2(e) - m)   row max by a 3-input max tree; the
//                      exponent in FP32, or as packed FP16 pairs (two results
//                      per MUFU op; P is FP16 for the next MMA either way)
//   O_t = P_t [V_t | 1]  tcgen05.mma -> TMEM O[t&1]; V^T carries an extra
//                      all-ones row, so column hd of O_t is the row sum of P_t
//                      as the tensor core saw it (FP16 P, FP32 accumulation)
//   the FP32 register accumulator and row sum take O_t with the running-max
//   correction one tile later.
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
  __half* ctx;                  // [batch, seq, heads * ctx_hd]
  int ctx_hd;                   // features per head of ctx: HD, or 8 when head_dim 8
                                // runs on Q/K/V stored 16 wide (zeros after the 8)
  unsigned int* err;
  unsigned long long timeout_ns;
};

template <int HD>
struct AttnLayout {
  static constexpr int BM = 128, BN = 128, NST = 3;
  static constexpr int HDX = HD + 16;  // V^T rows + the ones/zero block
  static constexpr int Q_BYTES = BM * HD * 2;
  static constexpr int K_BYTES = BN * HD * 2;
  static constexpr int VBLK = HDX * 128;  // one 64-key block of [V^T ; 1 ; 0]
  static constexpr int V_BYTES = 2 * VBLK;
  static constexpr int V_TMA_BYTES = 2 * HD * 128;
  static constexpr int P_BYTES = BM * BN * 2;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + 2 * Q_BYTES;
  static constexpr int OFF_V = OFF_K + NST * K_BYTES;
  static constexpr int OFF_P = OFF_V + NST * V_BYTES;
  static constexpr int OFF_BAR = OFF_P + 2 * P_BYTES;
  // q_full[2] q_empty[2] kv_full[NST] kv_empty[NST] s_full[2] s_free[2]
  // p_full[2] p_empty[2] o_full[2] o_free[2] done
  static constexpr int NBAR = 4 + 2 * NST + 12 + 1;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int BYTES = OFF_MISC + 16;
  static constexpr int SMEM_ALLOC = BYTES + 1024;  // slack for 1024-byte alignment
  static constexpr int TMEM_COLS = 512;            // S: 2 x 128, O: 2 x HDX
  static constexpr int TMEM_O = 256;
  static_assert(TMEM_O + 2 * HDX <= TMEM_COLS, "TMEM budget");
  static_assert(HD % 16 == 0 && HD >= 16 && HD <= 64, "head_dim");
  static_assert(Q_BYTES % 1024 == 0 && K_BYTES % 1024 == 0 && VBLK % 1024 == 0, "alignment");
};

// Static schedule shared by every role of a CTA: a CTA visits items
// w = blockIdx.x, blockIdx.x + gridDim.x, ...; item w is query tile
// (n_qt - 1 - w / (batch*heads)) of sequence*head (w % (batch*heads)), so the
// longest causal items come first.
struct AttnItem {
  int bh, b, h, q0, n;  // n = key tiles to visit (0: wholly padded query tile)
  int kv_end;
};

__device__ __forceinline__ AttnItem attn_item(const AttnParams& p, int w, int n_qt) {
  AttnItem it;
  const int bh_count = p.batch * p.heads;
  const int tile_rank = w / bh_count;
  const int qt = n_qt - 1 - tile_rank;
  it.bh = w - tile_rank * bh_count;
  it.b = it.bh / p.heads;
  it.h = it.bh - it.b * p.heads;
  it.q0 = qt * 128;
  it.kv_end = p.key_mask ? p.kv_end[it.b] : p.seq;
  if (it.q0 >= it.kv_end) {
    it.n = 0;
  } else {
    const int kv_limit = p.causal ? min(it.q0 + 128, it.kv_end) : it.kv_end;
    it.n = (kv_limit + 127) / 128;
  }
  return it;
}

// Eight probabilities of one row, packed as four FP16 pairs.
__device__ __forceinline__ void probs8(const float* x, float sl2, float m_use, uint32_t (&pk)[4]) {
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float a = fmaf(x[2 * e], sl2, -m_use);
    const float c = fmaf(x[2 * e + 1], sl2, -m_use);
    pk[e] = pack_half2(ex2_approx(a), ex2_approx(c));
  }
}

__device__ __forceinline__ float max3(float a, float b, float c) {
  float m;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(m) : "f"(a), "f"(b), "f"(c));
  return m;
}

template <int HD>
__global__ void __launch_bounds__(192, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const AttnParams p, int n_items) {
  using L = AttnLayout<HD>;
  constexpr int BM = L::BM, BN = L::BN, NST = L::NST, HDX = L::HDX;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_qt = (p.seq + BM - 1) / BM;
  const int D = p.heads * HD;

  uint8_t* sQ = smem + L::OFF_Q;
  uint8_t* sK = smem + L::OFF_K;
  uint8_t* sV = smem + L::OFF_V;
  uint8_t* sP = smem + L::OFF_P;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* q_empty = bars + 2;
  uint64_t* kv_full = bars + 4;
  uint64_t* kv_empty = kv_full + NST;
  uint64_t* s_full = kv_empty + NST;
  uint64_t* s_free = s_full + 2;
  uint64_t* p_full = s_full + 4;
  uint64_t* p_empty = s_full + 6;
  uint64_t* o_full = s_full + 8;
  uint64_t* o_free = s_full + 10;
  uint64_t* done = s_full + 12;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);
      mbar_init(&p_full[i], 4);
      mbar_init(&p_empty[i], 1);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_free[i], 4);
    }
    for (int i = 0; i < NST; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  // Rows HD .. HD+15 of every V block: row HD all ones (FP16 1.0), the rest
  // zero.  TMA only ever writes rows 0 .. HD-1.
  for (int i = threadIdx.x; i < NST * 2 * 16 * 32; i += blockDim.x) {
    const int word = i & 31, r = (i >> 5) & 15, blk = i >> 9;
    uint32_t* dst = reinterpret_cast<uint32_t*>(sV + blk * L::VBLK + (HD + r) * 128) + word;
    *dst = r == 0 ? 0x3C003C00u : 0u;
  }
  fence_proxy_async_smem();
  if (warp == 5) {
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

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      int t = 0, it = 0;
      bool ok = true;
      for (int w = blockIdx.x; ok && w < n_items; w += gridDim.x) {
        const AttnItem item = attn_item(p, w, n_qt);
        if (item.n == 0) continue;
        const int qb = it & 1;
        if (!(ok = wait_phase(&q_empty[qb], ((it >> 1) & 1) ^ 1, wd, 0x101))) break;
        mbar_arrive_expect_tx(&q_full[qb], L::Q_BYTES);
        tma_load_3d(sQ + qb * L::Q_BYTES, &tmQ, &q_full[qb], 0, item.q0, item.bh);
        ++it;
        for (int j = 0; j < item.n; ++j) {
          const int st = t % NST;
          if (!(ok = wait_phase(&kv_empty[st], ((t / NST) & 1) ^ 1, wd, 0x102))) break;
          mbar_arrive_expect_tx(&kv_full[st], L::K_BYTES + L::V_TMA_BYTES);
          tma_load_3d(sK + st * L::K_BYTES, &tmK, &kv_full[st], 0, j * BN, item.bh);
          uint8_t* v_dst = sV + st * L::V_BYTES;
          tma_load_3d(v_dst, &tmV, &kv_full[st], j * BN, 0, item.bh);
          tma_load_3d(v_dst + L::VBLK, &tmV, &kv_full[st], j * BN + 64, 0, item.bh);
          ++t;
        }
      }
      // Let every copy this CTA started land before the CTA may exit.
      for (int i = (it > 2 ? it - 2 : 0); i < it; ++i)
        wait_drain(&q_full[i & 1], (i >> 1) & 1, kDrainLimitNs);
      for (int i = (t > NST ? t - NST : 0); i < t; ++i)
        wait_drain(&kv_full[i % NST], (i / NST) & 1, kDrainLimitNs);
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t kSwQK = swizzle_kind_for_bytes(HD * 2);
      constexpr uint32_t kSboQK = 8 * HD * 2;
      const uint32_t idesc_s = umma_idesc_f16_f32(BM, BN);
      const uint32_t idesc_o = umma_idesc_f16_f32(BM, HDX);
      const uint32_t aQ = smem_u32(sQ), aK = smem_u32(sK), aV = smem_u32(sV), aP = smem_u32(sP);
      bool ok = true;
      // S-issue cursor: (item_s, j_s) is the next tile whose S = Q K^T is due,
      // t_s its index in this CTA's tile sequence, it_s its item's index.
      AttnItem item_s;
      item_s.n = 0;
      int w_s = static_cast<int>(blockIdx.x) - static_cast<int>(gridDim.x);
      int j_s = 0, it_s = -1, t_s = 0;
      auto advance_s = [&]() -> bool {
        while (j_s >= item_s.n) {
          w_s += gridDim.x;
          if (w_s >= n_items) return false;
          item_s = attn_item(p, w_s, n_qt);
          j_s = 0;
          if (item_s.n > 0) ++it_s;
        }
        return true;
      };
      auto issue_s = [&]() -> bool {
        const int st = t_s % NST, sb = t_s & 1, qb = it_s & 1;
        if (j_s == 0 && !wait_phase(&q_full[qb], (it_s >> 1) & 1, wd, 0x201)) return false;
        if (!wait_phase(&kv_full[st], (t_s / NST) & 1, wd, 0x202)) return false;
        if (t_s >= 2 && !wait_phase(&s_free[sb], ((t_s >> 1) - 1) & 1, wd, 0x203)) return false;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint64_t da = umma_sdesc(aQ + qb * L::Q_BYTES + kk * 32, kSboQK, kSwQK);
          const uint64_t db = umma_sdesc(aK + st * L::K_BYTES + kk * 32, kSboQK, kSwQK);
          umma_f16(tmem_base + sb * 128, da, db, idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[sb]);
        if (j_s == item_s.n - 1) umma_commit(&q_empty[qb]);  // this item's Q is no longer read
        ++j_s;
        ++t_s;
        return true;
      };
      bool more_s = advance_s();
      if (more_s) {
        ok = issue_s();
        more_s = ok && advance_s();
      }
      // P.V of tile t follows the S of tile t+1 so the tensor core stays one
      // tile ahead of the softmax warps.
      for (int t = 0; ok && t < t_s; ++t) {
        if (more_s) {
          if (!(ok = issue_s())) break;
          more_s = advance_s();
        }
        const int bs = t & 1, st = t % NST;
        if (!(ok = wait_phase(&p_full[bs], (t >> 1) & 1, wd, 0x204))) break;
        if (!(ok = wait_phase(&o_free[bs], ((t >> 1) & 1) ^ 1, wd, 0x205))) break;
        tc_fence_after();
        const uint32_t tO = tmem_base + L::TMEM_O + bs * HDX;
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint64_t da =
              umma_sdesc(aP + bs * L::P_BYTES + (kk >> 2) * (BM * 128) + (kk & 3) * 32, 1024, kSw128);
          const uint64_t db =
              umma_sdesc(aV + st * L::V_BYTES + (kk >> 2) * L::VBLK + (kk & 3) * 32, 1024, kSw128);
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
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    const uint32_t p_base = smem_u32(sP);
    const float sl2 = p.scale_log2;
    bool ok = true;
    int t = 0;
    for (int w = blockIdx.x; ok && w < n_items; w += gridDim.x) {
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
        const int bs = tt & 1;
        if (!warp_wait_phase(&o_full[bs], (tt >> 1) & 1, wd, 0x303)) return false;
        tc_fence_after();
        const uint32_t tO = tmem_base + lane_base + L::TMEM_O + bs * HDX;
#pragma unroll
        for (int g = 0; g < HDX / 16; ++g) {
          uint32_t r[16];
          tmem_ld_x16_sync(tO + g * 16, r);
#pragma unroll
          for (int d = 0; d < 16; ++d) {
            const int col = g * 16 + d;
            if (col < HD) o[col] = fmaf(o[col], c, __uint_as_float(r[d]));
            if (col == HD) l_run = fmaf(l_run, c, __uint_as_float(r[d]));
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&o_free[bs]);
        return true;
      };

      for (int j = 0; j < item.n; ++j, ++t) {
        const int k0 = j * BN;
        uint32_t vb0 = ~0u, vb1 = ~0u, vb2 = ~0u, vb3 = ~0u;
        bool mask_partial = false;
        if (p.key_mask != nullptr) {
          const uint8_t* mrow = p.key_mask + static_cast<size_t>(item.b) * p.seq;
          const int ka = k0 + lane;
          vb0 = __ballot_sync(~0u, ka < p.seq && mrow[min(ka, p.seq - 1)] != 0);
          vb1 = __ballot_sync(~0u, ka + 32 < p.seq && mrow[min(ka + 32, p.seq - 1)] != 0);
          vb2 = __ballot_sync(~0u, ka + 64 < p.seq && mrow[min(ka + 64, p.seq - 1)] != 0);
          vb3 = __ballot_sync(~0u, ka + 96 < p.seq && mrow[min(ka + 96, p.seq - 1)] != 0);
          mask_partial = (vb0 & vb1 & vb2 & vb3) != ~0u;
        }
        const bool need_mask = __any_sync(0xffffffffu, mask_partial || (k0 + BN > row_lim));
        const int bs = t & 1;

        if (!(ok = warp_wait_phase(&s_full[bs], (t >> 1) & 1, wd, 0x301))) break;
        tc_fence_after();
        float x[BN];
#pragma unroll
        for (int g = 0; g < BN / 32; ++g) {
          uint32_t r[32];
          tmem_ld_x32_sync(tmem_base + lane_base + bs * 128 + g * 32, r);
#pragma unroll
          for (int i = 0; i < 32; ++i) x[g * 32 + i] = __uint_as_float(r[i]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[bs]);

        if (need_mask) {
          const int lim = row_lim - k0;
#pragma unroll
          for (int c = 0; c < BN; ++c) {
            const uint32_t wbits = (c < 32) ? vb0 : (c < 64) ? vb1 : (c < 96) ? vb2 : vb3;
            const bool valid = (c < lim) && ((wbits >> (c & 31)) & 1u);
            x[c] = valid ? x[c] : -INFINITY;
          }
        }
        // Row max through a tree of 3-input maxima (short dependency chains).
        float m1[43];
#pragma unroll
        for (int i = 0; i < 42; ++i) m1[i] = max3(x[3 * i], x[3 * i + 1], x[3 * i + 2]);
        m1[42] = fmaxf(x[126], x[127]);
        float m2[15];
#pragma unroll
        for (int i = 0; i < 14; ++i) m2[i] = max3(m1[3 * i], m1[3 * i + 1], m1[3 * i + 2]);
        m2[14] = m1[42];
        float m3[5];
#pragma unroll
        for (int i = 0; i < 5; ++i) m3[i] = max3(m2[3 * i], m2[3 * i + 1], m2[3 * i + 2]);
        const float mt = max3(max3(m3[0], m3[1], m3[2]), m3[3], m3[4]);
        const float m_new = fmaxf(m_run, mt * sl2);
        const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
        const float corr = ex2_approx(m_run - m_use);

        if (!(ok = warp_wait_phase(&p_empty[bs], ((t >> 1) & 1) ^ 1, wd, 0x302))) break;
        const uint32_t prow = p_base + bs * L::P_BYTES + row * 128;
#pragma unroll
        for (int ch = 0; ch < BN / 8; ++ch) {
          uint32_t pk[4];
          probs8(&x[ch * 8], sl2, m_use, pk);
          const uint32_t addr = prow + (ch >> 3) * (BM * 128) + (((ch & 7) ^ (row & 7)) << 4);
          st_shared_v4(addr, pk[0], pk[1], pk[2], pk[3]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[bs]);
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
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem_base, L::TMEM_COLS);
  }
}

}  // namespace tt
