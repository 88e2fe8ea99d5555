// Fully fused feed-forward block for sm_100a (d_model <= 256):
//
//   h      = GELU_erf(n . W1^T + b1)                (FP32 math, FP16 h, never in HBM)
//   r'     = h . W2^T + b2 + r                      (FP32 residual stream)
//   n'     = LayerNorm(r') * gamma + beta            (FP16 next input, or FP32 output)
//
// Replaces the reference's `_mixed_ffn_add_layer_norm_kernel`
// (mixed_precision/triton_linear.py:128-185, D = F = 128 only) and the
// ffn_in -> GELU -> ffn_out -> fused_add_layer_norm chain of its generic route
// (mixed_precision/transformer.py:669-695), for any F that is a multiple of 128.
//
// Persistent kernel over 128-row tiles.  Per tile the FP16 input tile A
// [128 x D] is loaded once; the hidden dimension is processed in chunks of
// FC = 128 units:
//   G1(c)  acc1[c&1] (TMEM, 128 x FC FP32) = A . W1[c]^T
//   GELU   warps 0..7: acc1[c&1] + b1 -> GELU -> FP16 -> H[c&1] (shared,
//          128B-swizzled K-major, the A operand of G2)
//   G2(c)  acc2 (TMEM, 128 x D FP32) += H[c&1] . W2[:, c]^T
// issued in the order G1(0) G1(1) G2(0) G1(2) G2(1) ... so GELU of chunk c+1
// overlaps G2(c).  Warps 8..11 then drain acc2 (bias, residual, two-pass
// LayerNorm, TMA-staged stores) while the MMAs of the next tile's G1 run.
// Warp 12 streams A and the W1/W2 K-blocks (32 columns, 64-byte swizzle) with
// TMA; warp 13 allocates TMEM and issues tcgen05.mma.
#pragma once

#include "tt_gemm.cuh"

namespace tt {

struct FfnParams {
  int M, D, F;
  int n_items;  // ceil(M / 128)
  const float* b1;     // [F]
  const float* b2;     // [D]
  const float* gamma;  // [D]
  const float* beta;   // [D]
  const float* resid_in;  // [M, D] FP32 (read directly)
  int norm_f16;
  float eps;
  const uint8_t* row_mask;
  unsigned int* err;
  unsigned long long timeout_ns;
  // Direct outputs (ffn2_kernel): residual out [M, D] FP32, normalized [M, D] FP16 or FP32.
  float* resid_out;
  void* norm_out;
};

// Tensor maps: a = input [M, D] FP16 box {32, 128}; w1 = W1 [F, D] FP16 box
// {32, 128}; w2 = W2 [D, F] FP16 box {32, D}; out0 = residual out [M, D] FP32
// box {32, 32}; out1 = normalized [M, D] (FP16 or FP32) box {32, 32}.
struct FfnMaps {
  CUtensorMap a, w1, w2, out0, out1;
};

template <int D>
struct FfnLayout {
  static constexpr int FC = 128, KSW = 32, NST = 3;
  static constexpr int A_BOX = 128 * KSW * 2;                 // 8 KB
  static constexpr int A_BYTES = (D / KSW) * A_BOX;
  static constexpr int W1_BLK = FC * KSW * 2;                 // 8 KB
  static constexpr int W2_BLK = D * KSW * 2;
  static constexpr int SLOT = (W1_BLK > W2_BLK ? W1_BLK : W2_BLK);
  static constexpr int H_BYTES = 128 * FC * 2;                // 32 KB
  static constexpr int OFF_A = 0;
  static constexpr int OFF_W = OFF_A + A_BYTES;
  static constexpr int OFF_H = OFF_W + NST * SLOT;
  static constexpr int OFF_EPI = OFF_H + 2 * H_BYTES;         // 4 LN warps x 2 staging tiles
  static constexpr int OFF_F32 = OFF_EPI + 4 * 2 * kEpiTile;  // b2, gamma, beta [D] each
  static constexpr int OFF_BAR = OFF_F32 + 3 * D * 4;
  // a_full a_empty w_full[NST] w_empty[NST] acc1_full[2] acc1_empty[2] h_full[2] h_empty[2]
  // acc2_full acc2_empty done
  static constexpr int NBAR = 2 + 2 * NST + 8 + 3;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int OFF_B1 = (OFF_MISC + 16 + 127) / 128 * 128;  // b1 [F] (runtime size), read as float4
  static_assert(OFF_B1 % 16 == 0 && OFF_F32 % 16 == 0 && OFF_EPI % 1024 == 0, "alignment");
  static constexpr int SMEM_BASE = OFF_B1 + 1024;             // + F * 4 bytes at launch
  static constexpr int TMEM_ACC1 = 256;  // acc2 occupies columns [0, D)
  static_assert(D % 32 == 0 && D >= 32 && D <= 256, "fused FFN covers d_model 32..256");
  static int smem_bytes(int F) { return SMEM_BASE + F * 4; }
};

// Warp roles: 0..7 GELU (warp w: TMEM lane quadrant w & 3, hidden columns
// 64 * (w >> 2) .. +63 of each chunk), 8..11 residual + LayerNorm, 12 TMA
// producer, 13 TMEM allocator and MMA issuer.
// Warp 14 is a second TMA producer: ring slot st is always filled by producer
// st % 2, so each slot keeps a single producer and the parity-based
// empty-slot wait stays exact (one producer thread completes only about one
// TMA copy per ~800 cycles).
constexpr int kFfnThreads = 480;
constexpr int kFfnWarpProd = 12, kFfnWarpMma = 13, kFfnWarpProd2 = 14;

template <int D>
__global__ void __launch_bounds__(kFfnThreads, 1)
    ffn_fused_kernel(const __grid_constant__ FfnMaps maps, const FfnParams p) {
  using L = FfnLayout<D>;
  constexpr int FC = L::FC, KSW = L::KSW, NST = L::NST;
  constexpr int NKA = D / KSW;  // K-blocks of G1
  constexpr int NKH = FC / KSW; // K-blocks of G2 per chunk
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  float* s_b2 = reinterpret_cast<float*>(smem + L::OFF_F32);
  float* s_b1 = reinterpret_cast<float*>(smem + L::OFF_B1);
  float* s_gamma = s_b2 + D;
  float* s_beta = s_gamma + D;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* a_full = bars;
  uint64_t* a_empty = bars + 1;
  uint64_t* w_full = bars + 2;
  uint64_t* w_empty = w_full + NST;
  uint64_t* acc1_full = w_empty + NST;
  uint64_t* acc1_empty = acc1_full + 2;
  uint64_t* h_full = acc1_empty + 2;
  uint64_t* h_empty = h_full + 2;
  uint64_t* acc2_full = h_empty + 2;
  uint64_t* acc2_empty = acc2_full + 1;
  uint64_t* done = acc2_empty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nchunk = p.F / FC;

  if (threadIdx.x == 0) {
    mbar_init(a_full, 1);
    mbar_init(a_empty, 1);
    for (int i = 0; i < NST; ++i) {
      mbar_init(&w_full[i], 1);
      mbar_init(&w_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc1_full[i], 1);
      mbar_init(&acc1_empty[i], 8);
      mbar_init(&h_full[i], 8);
      mbar_init(&h_empty[i], 1);
    }
    mbar_init(acc2_full, 1);
    mbar_init(acc2_empty, 4);
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  for (int c = threadIdx.x; c < p.F; c += blockDim.x) s_b1[c] = p.b1[c];
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    s_b2[c] = p.b2[c];
    s_gamma[c] = p.gamma[c];
    s_beta[c] = p.beta[c];
  }
  if (warp == kFfnWarpMma) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_wait();  // activations of the previous kernel are final from here on
  pdl_trigger();
  const uint32_t tmem_base = *tmem_slot;
  const Watchdog wd{p.err, abort_flag, p.timeout_ns};

  if (warp == kFfnWarpProd || warp == kFfnWarpProd2) {
    // ------------------------------------------------------------ producers
    const int pidx = warp == kFfnWarpProd ? 0 : 1;
    if (lane == 0) {
      tma_prefetch_desc(&maps.a);
      tma_prefetch_desc(&maps.w1);
      tma_prefetch_desc(&maps.w2);
      int g = 0, i = 0;
      bool ok = true;
      auto load_w = [&](const CUtensorMap* tm, int kx, int ky, int bytes) -> bool {
        if ((g % NST) % 2 != pidx) {
          ++g;
          return true;
        }
        const int st = g % NST;
        if (!wait_phase(&w_empty[st], ((g / NST) & 1) ^ 1, wd, 0x501)) return false;
        mbar_arrive_expect_tx(&w_full[st], bytes);
        tma_load_2d(smem + L::OFF_W + st * L::SLOT, tm, &w_full[st], kx, ky);
        ++g;
        return true;
      };
      for (int w = blockIdx.x; ok && w < p.n_items; w += gridDim.x, ++i) {
        const int m0 = w * 128;
        if (pidx == 0) {
          if (!(ok = wait_phase(a_empty, (i & 1) ^ 1, wd, 0x502))) break;
          mbar_arrive_expect_tx(a_full, L::A_BYTES);
          for (int kb = 0; kb < NKA; ++kb)
            tma_load_2d(smem + L::OFF_A + kb * L::A_BOX, &maps.a, a_full, kb * KSW, m0);
        }
        // Same order as the MMA issuer: G1(0), G1(1), G2(0), G1(2), G2(1), ...
        for (int step = 0; ok && step <= nchunk; ++step) {
          if (step < nchunk)
            for (int kb = 0; ok && kb < NKA; ++kb) ok = load_w(&maps.w1, kb * KSW, step * FC, L::W1_BLK);
          if (step >= 1)
            for (int kb = 0; ok && kb < NKH; ++kb)
              ok = load_w(&maps.w2, (step - 1) * FC + kb * KSW, 0, L::W2_BLK);
        }
      }
      if (pidx == 0 && i > 0) wait_drain(a_full, (i - 1) & 1, kDrainLimitNs);
      for (int q = (g > NST ? g - NST : 0); q < g; ++q)
        if ((q % NST) % 2 == pidx) wait_drain(&w_full[q % NST], (q / NST) & 1, kDrainLimitNs);
    }
  } else if (warp == kFfnWarpMma) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t kSw = kSw64;
      constexpr uint32_t kSbo = 8 * KSW * 2;
      const uint32_t idesc1 = umma_idesc_f16_f32(128, FC);
      const uint32_t idesc2 = umma_idesc_f16_f32(128, D);
      const uint32_t sA = smem_u32(smem + L::OFF_A);
      const uint32_t sW = smem_u32(smem + L::OFF_W);
      const uint32_t sH = smem_u32(smem + L::OFF_H);
      int g = 0, i = 0, cg = 0;  // W stage counter, tile counter, global chunk counter
      bool ok = true;
      for (int w = blockIdx.x; ok && w < p.n_items; w += gridDim.x, ++i) {
        if (!(ok = wait_phase(a_full, i & 1, wd, 0x511))) break;
        for (int step = 0; ok && step <= nchunk; ++step) {
          if (step < nchunk) {
            // G1(step) into acc1[(cg+step)&1]
            const int c = cg + step, ab = c & 1;
            if (!(ok = wait_phase(&acc1_empty[ab], ((c >> 1) & 1) ^ 1, wd, 0x512))) break;
            tc_fence_after();
            const uint32_t tacc = tmem_base + L::TMEM_ACC1 + ab * FC;
            for (int kb = 0; kb < NKA; ++kb) {
              const int st = g % NST;
              if (!(ok = wait_phase(&w_full[st], (g / NST) & 1, wd, 0x513))) break;
              tc_fence_after();
#pragma unroll
              for (int kk = 0; kk < KSW / 16; ++kk) {
                const uint64_t da = umma_sdesc(sA + kb * L::A_BOX + kk * 32, kSbo, kSw);
                const uint64_t db = umma_sdesc(sW + st * L::SLOT + kk * 32, kSbo, kSw);
                umma_f16(tacc, da, db, idesc1, (kb > 0 || kk > 0) ? 1u : 0u);
              }
              umma_commit(&w_empty[st]);
              ++g;
            }
            if (!ok) break;
            umma_commit(&acc1_full[ab]);
            if (step == nchunk - 1) umma_commit(a_empty);  // A is no longer read in this tile
          }
          if (step >= 1) {
            // G2(step-1): acc2 += H[c&1] . W2[:, chunk]^T
            const int c = cg + step - 1, hb = c & 1;
            if (step == 1 && !(ok = wait_phase(acc2_empty, (i & 1) ^ 1, wd, 0x514))) break;
            if (!(ok = wait_phase(&h_full[hb], (c >> 1) & 1, wd, 0x515))) break;
            tc_fence_after();
            for (int kb = 0; kb < NKH; ++kb) {
              const int st = g % NST;
              if (!(ok = wait_phase(&w_full[st], (g / NST) & 1, wd, 0x516))) break;
              tc_fence_after();
#pragma unroll
              for (int kk = 0; kk < KSW / 16; ++kk) {
                const int k2 = kb * (KSW / 16) + kk;  // 16-wide K step within the chunk
                const uint64_t da = umma_sdesc(sH + hb * L::H_BYTES + (k2 >> 2) * (128 * 128) + (k2 & 3) * 32,
                                               1024, kSw128);
                const uint64_t db = umma_sdesc(sW + st * L::SLOT + kk * 32, kSbo, kSw);
                umma_f16(tmem_base, da, db, idesc2, (step > 1 || kb > 0 || kk > 0) ? 1u : 0u);
              }
              umma_commit(&w_empty[st]);
              ++g;
            }
            if (!ok) break;
            umma_commit(&h_empty[hb]);
            if (step == nchunk) umma_commit(acc2_full);
          }
        }
        cg += nchunk;
      }
      umma_commit(done);
      wait_drain(done, 0, kDrainLimitNs);
    }
  } else if (warp < 8) {
    // ------------------------------------------------------------ GELU warps
    const int gq = warp & 3, gh = warp >> 2;  // lane quadrant, column half of the chunk
    const uint32_t lane_base = static_cast<uint32_t>(gq * 32) << 16;
    const int r = gq * 32 + lane;  // row within the tile == TMEM lane
    const uint32_t sH = smem_u32(smem + L::OFF_H);
    int cg = 0;
    bool ok = true;
    for (int w = blockIdx.x; ok && w < p.n_items; w += gridDim.x) {
      for (int cc = 0; cc < nchunk; ++cc) {
        const int c = cg + cc, ab = c & 1;
        if (!(ok = warp_wait_phase(&acc1_full[ab], (c >> 1) & 1, wd, 0x521))) break;
        tc_fence_after();
        uint32_t v[2][32];
        const uint32_t tsrc = tmem_base + lane_base + L::TMEM_ACC1 + ab * FC + gh * 64;
        tmem_ld_x32(tsrc, v[0]);
        tmem_ld_x32(tsrc + 32, v[1]);
        tmem_ld_wait_tied(v[0]);
        tmem_ld_wait_tied(v[1]);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc1_empty[ab]);  // acc1 buffer may be overwritten
        if (!(ok = warp_wait_phase(&h_empty[ab], ((c >> 1) & 1) ^ 1, wd, 0x522))) break;
        // H block gh (64 hidden units = 128 bytes per row, 128B-swizzled).
        const uint32_t hrow = sH + ab * L::H_BYTES + gh * (128 * 128) + r * 128;
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          const float4* b4 = reinterpret_cast<const float4*>(s_b1 + cc * FC + gh * 64 + g * 32);
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float4 bb = b4[e];  // same address in every lane: a broadcast shared load
            const uint64_t h01 = gelu_erf_pair(
                fadd2(f2_pack(__uint_as_float(v[g][4 * e]), __uint_as_float(v[g][4 * e + 1])), f2_pack(bb.x, bb.y)));
            const uint64_t h23 = gelu_erf_pair(
                fadd2(f2_pack(__uint_as_float(v[g][4 * e + 2]), __uint_as_float(v[g][4 * e + 3])), f2_pack(bb.z, bb.w)));
            pk[2 * e] = pack_half2(f2_lo(h01), f2_hi(h01));
            pk[2 * e + 1] = pack_half2(f2_lo(h23), f2_hi(h23));
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int ch = g * 4 + u;  // 16-byte chunk (8 hidden units) within the 64-unit block
            st_shared_v4(hrow + ((ch ^ (r & 7)) << 4), pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&h_full[ab]);
      }
      cg += nchunk;
    }
  } else {
    // ------------------------------------------------------------ residual + LayerNorm warps
    const int ew = warp - 8;  // TMEM lane quadrant
    const uint32_t lane_base = static_cast<uint32_t>(ew * 32) << 16;
    const uint32_t taddr = tmem_base + lane_base;
    OutRing<2> ring{smem_u32(smem + L::OFF_EPI) + ew * 2 * kEpiTile, 0};
    constexpr int nch = D / 32;
    int i = 0;
    bool ok = true;
    for (int w = blockIdx.x; ok && w < p.n_items; w += gridDim.x, ++i) {
      const int m0 = w * 128;
      const int r0 = m0 + ew * 32;
      const int row = r0 + lane;
      const bool valid = row < p.M;
      const bool warp_active = r0 < p.M;
      if (!(ok = warp_wait_phase(acc2_full, i & 1, wd, 0x531))) break;
      tc_fence_after();
      const float4* rin = reinterpret_cast<const float4*>(p.resid_in + static_cast<size_t>(valid ? row : 0) * D);
      float sum = 0.f;
      float4 res[8], nxt[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) nxt[e] = valid ? __ldg(rin + e) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 1
      for (int c = 0; c < nch; ++c) {
#pragma unroll
        for (int e = 0; e < 8; ++e) res[e] = nxt[e];
        if (c + 1 < nch) {
#pragma unroll
          for (int e = 0; e < 8; ++e)
            nxt[e] = valid ? __ldg(rin + (c + 1) * 8 + e) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        uint32_t v[32];
        tmem_ld_x32_sync(taddr + c * 32, v);
        float rr[32];
        uint32_t out[32];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          rr[4 * e + 0] = __uint_as_float(v[4 * e + 0]) + s_b2[c * 32 + 4 * e + 0] + res[e].x;
          rr[4 * e + 1] = __uint_as_float(v[4 * e + 1]) + s_b2[c * 32 + 4 * e + 1] + res[e].y;
          rr[4 * e + 2] = __uint_as_float(v[4 * e + 2]) + s_b2[c * 32 + 4 * e + 2] + res[e].z;
          rr[4 * e + 3] = __uint_as_float(v[4 * e + 3]) + s_b2[c * 32 + 4 * e + 3] + res[e].w;
        }
#pragma unroll
        for (int e = 0; e < 32; ++e) out[e] = __float_as_uint(rr[e]);
#pragma unroll
        for (int e = 0; e < 32; e += 4) sum += (rr[e] + rr[e + 1]) + (rr[e + 2] + rr[e + 3]);
        __syncwarp();
        tmem_st_x32(taddr + c * 32, out);
        if (warp_active) {
          const uint32_t slot = ring.acquire(lane);
          stage_row_f32(slot, lane, rr);
          ring.publish();
          if (lane == 0) {
            tma_store_2d(&maps.out0, slot, c * 32, r0);
            bulk_commit_group();
          }
        }
      }
      tmem_st_wait();
      const float mean = sum / static_cast<float>(D);
      float sq = 0.f;
#pragma unroll 1
      for (int c = 0; c < nch; ++c) {
        uint32_t v[32];
        tmem_ld_x32_sync(taddr + c * 32, v);
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const float d = __uint_as_float(v[e]) - mean;
          sq = fmaf(d, d, sq);
        }
      }
      const float rstd = rsqrtf(sq / static_cast<float>(D) + p.eps);
      const bool zero_row = valid && p.row_mask != nullptr && p.row_mask[row] == 0;
#pragma unroll 1
      for (int c = 0; c < nch; ++c) {
        uint32_t v[32];
        tmem_ld_x32_sync(taddr + c * 32, v);
        if (c == nch - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(acc2_empty);  // acc2 may be overwritten by the next tile
        }
        if (!warp_active) continue;
        float y[32];
#pragma unroll
        for (int e = 0; e < 32; ++e)
          y[e] = zero_row ? 0.f
                          : fmaf((__uint_as_float(v[e]) - mean) * rstd, s_gamma[c * 32 + e], s_beta[c * 32 + e]);
        const uint32_t slot = ring.acquire(lane);
        if (p.norm_f16)
          stage_row_f16x32(slot, lane, y);
        else
          stage_row_f32(slot, lane, y);
        ring.publish();
        if (lane == 0) {
          tma_store_2d(&maps.out1, slot, c * 32, r0);
          bulk_commit_group();
        }
      }
    }
    if (lane == 0) bulk_wait_group_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kFfnWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace tt
