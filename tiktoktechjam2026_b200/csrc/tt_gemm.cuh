// Row-block projection GEMMs for sm_100a with fused epilogues.
//
//   out[M, N] = A[M, K] (FP16) . W[N, K]^T (FP16) + bias, FP32 accumulation
//
// replacing the reference's Triton projection kernels
// (mixed_precision/triton_linear.py:16-69 `_mixed_linear_kernel`, :72-125
// `_mixed_linear_add_layer_norm_kernel`) and the cuBLAS nn.Linear route of the
// generic configurations (mixed_precision/transformer.py:138-139, 669-677).
//
// Persistent kernel.  A work item is (128-row M tile, `bn`-column split);
// CTA c takes items c, c + gridDim.x, ...  Warps (NEPI = 8):
//   warps 0..NEPI-1  epilogue: warp e reads TMEM lane quadrant e % 4 (rows
//               32(e%4)..+31 of the tile, one row per thread); with 8 warps
//               the two warps of a quadrant split its 32-column chunks
//   warp NEPI   first TMA producer; warps NEPI+2.. further producers: (A, W)
//               K-blocks through an `nst`-deep ring that runs continuously
//               across items, slot st always filled by producer
//               st % kGemmProducers
//   warp NEPI+1 TMEM allocator and single-thread tcgen05.mma issuer; the FP32
//               accumulator is double buffered in TMEM (bn <= 256), so the
//               MMAs of item i+1 overlap the epilogue of item i
// Epilogues, in 32-column chunks:
//   EPI_QKV       + bias, FP16, to Q/K [B*H, S, hs] and V^T [B*H, hs, S_pad]
//                 (hs = max(hd, 16); head_dim 8 is stored with 8 zero
//                 features); rows staged through shared memory and written
//                 with coalesced 16-byte stores (one value per store when S is
//                 not a multiple of 32)
//   EPI_RESID_LN  + bias + FP32 residual -> residual out (FP32) and FP32
//                 shifted sums for the LayerNorm statistics in one TMEM pass
//                 (the row is written back into TMEM); the quadrant's two
//                 warps swap (mean, M2) of their column halves through shared
//                 memory; then the normalized row in a second pass -> FP16 or
//                 FP32, optionally zeroing
//                 rows whose mask byte is 0; the residual arrives by TMA into
//                 a per-warp ring of [32 rows x 32 col] tiles and the outputs
//                 leave by TMA bulk stores from swizzled shared tiles
//   EPI_GELU      + bias, exact-erf GELU in FP32, FP16 out (TMA bulk stores)
#pragma once

#include "tt_ptx.cuh"

namespace tt {

enum GemmEpilogue : int { EPI_QKV = 0, EPI_RESID_LN = 1, EPI_GELU = 2 };

constexpr int kGemmMaxStages = 8;
// EPI_RESID_LN runs two epilogue warps per TMEM lane quadrant, each on half
// of the row's columns, the row statistics combined through shared memory
// (C5 out-proj 1.27 -> 1.08 ms per forward against one warp per quadrant);
// kResRing residual tiles are in flight per epilogue warp; one for the
// 512-column tiles (d_model 512), whose single-accumulator mainloop needs the
// 32 KB this frees for a third operand stage (C4 FFN-out 2 -> 3 stages).
constexpr int kResRing = 2;
constexpr int kEpiTile = 4096;  // one [32 x 32] FP32 tile

struct GemmParams {
  int M, N_total, K;
  int bn;        // output columns per item
  int n_splits;  // N_total / bn
  int nst;       // pipeline depth
  int n_items;   // ceil(M / 128) * n_splits
  int tma_out;   // QKV only: 1 = rows staged for coalesced stores (requires seq % 32 == 0)
  const float* bias;  // [N_total]
  // EPI_QKV
  __half* q;
  __half* k;
  __half* vt;
  int seq, heads, head_dim, seq_pad, d_model;
  // EPI_RESID_LN
  const float* gamma;
  const float* beta;
  int norm_f16;
  // 1: the residual sum only (out0), no LayerNorm: rows wider than 512 FP32
  // accumulator columns run column-split (n_splits > 1) and are normalized by
  // a row kernel afterwards.
  int no_norm;
  float eps;
  const uint8_t* row_mask;
  unsigned int* err;
  unsigned long long timeout_ns;
};

// Tensor maps of one GEMM launch.  `a`, `w`: operands (box {KSW, 128} and
// {KSW, min(bn, 256)}).  Outputs/inputs of the epilogue, box 32 x 32:
//   EPI_QKV       (tma_out, head_dim >= 32) out0 = Q as [B*H*S, hd], out1 = K
//                 likewise, res = V^T as [B*H*hd, S_pad], all FP16; otherwise
//                 none (stores through GemmParams' pointers)
//   EPI_RESID_LN  out0 = residual out (FP32), out1 = normalized (FP16/FP32),
//                 res  = residual in (FP32)
//   EPI_GELU      out0 = activation (FP16)
struct GemmMaps {
  CUtensorMap a, w, out0, out1, res;
};

__host__ __device__ inline int gemm_stage_bytes(int ksw, int bn) { return (128 + bn) * ksw * 2; }
__host__ __device__ inline int gemm_acc_stride(int bn) {
  int c = 32;
  while (c < bn) c <<= 1;
  return c;
}
__host__ __device__ inline int gemm_n_acc(int bn) { return bn <= 256 ? 2 : 1; }
__host__ __device__ inline int gemm_tmem_cols(int bn) { return gemm_n_acc(bn) * gemm_acc_stride(bn); }
// Epilogue warps: two on each TMEM lane quadrant, splitting its columns, so
// every SM sub-partition has two epilogue warps.
__host__ __device__ constexpr int gemm_epi_warps(int) { return 8; }
// Warps: epilogue warps, then the first TMA producer, the MMA issuer and
// kGemmProducers - 1 more producers.  Ring slot st is always filled by
// producer st % kGemmProducers: one producer per slot keeps the parity-based
// empty-slot wait exact (a producer can never be two phases ahead on a slot
// that another producer fills).
constexpr int kGemmProducers = 2;
__host__ __device__ constexpr int gemm_threads(int epi) { return 32 * (gemm_epi_warps(epi) + 1 + kGemmProducers); }
// Output staging tiles per epilogue warp.  The LayerNorm epilogue spends its
// shared memory on the residual ring instead (with one epilogue warp per
// quadrant, 3 residual tiles and 1 output tile measured 4 % faster than 2 and 2
// at C5).
__host__ __device__ constexpr int gemm_out_ring(int epi) { return epi == EPI_RESID_LN ? 1 : 2; }
__host__ __device__ constexpr int gemm_res_ring(int epi, int bn) {
  return epi == EPI_RESID_LN ? (bn > 256 ? 1 : kResRing) : 0;
}
__host__ __device__ inline int gemm_epi_bytes(int epi, int rr) {
  return gemm_epi_warps(epi) * (rr + gemm_out_ring(epi)) * kEpiTile;
}
// Layout: stages | epilogue tiles | bias[N_total], gamma[bn], beta[bn] | barriers | misc
// (+1024 alignment slack)
__host__ __device__ inline int gemm_smem_bytes(int ksw, int bn, int nst, int epi, int n_total) {
  int off = nst * gemm_stage_bytes(ksw, bn);
  off += gemm_epi_bytes(epi, gemm_res_ring(epi, bn));
  off += (n_total + 2 * bn) * 4;
  off += (2 * kGemmMaxStages + 5 + 8 * kResRing + 4 + 1) * 8;
  off += 16;
  off += 2 * 4 * 2 * 2 * 32 * 4;  // row-statistics exchange of the split LayerNorm epilogue
  return off + 1024;
}

// ---- shared-tile helpers (swizzle patterns match the TMA swizzle modes) ----
// [32 rows x 32 FP32], 128-byte rows, SWIZZLE_128B.
__device__ __forceinline__ void stage_row_f32(uint32_t tile, int r, const float* v) {
  const uint32_t base = tile + r * 128;
#pragma unroll
  for (int c = 0; c < 8; ++c)
    st_shared_v4(base + ((c ^ (r & 7)) << 4), __float_as_uint(v[4 * c]), __float_as_uint(v[4 * c + 1]),
                 __float_as_uint(v[4 * c + 2]), __float_as_uint(v[4 * c + 3]));
}

__device__ __forceinline__ void load_row_f32(uint32_t tile, int r, float* v) {
  const uint32_t base = tile + r * 128;
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    uint32_t a, b, d, e;
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(a), "=r"(b), "=r"(d), "=r"(e)
                 : "r"(base + ((c ^ (r & 7)) << 4)));
    v[4 * c] = __uint_as_float(a);
    v[4 * c + 1] = __uint_as_float(b);
    v[4 * c + 2] = __uint_as_float(d);
    v[4 * c + 3] = __uint_as_float(e);
  }
}

// [32 rows x 32 FP16], 64-byte rows, SWIZZLE_64B.
__device__ __forceinline__ void stage_row_f16x32(uint32_t tile, int r, const float* v) {
  const uint32_t base = tile + r * 64;
#pragma unroll
  for (int c = 0; c < 4; ++c)
    st_shared_v4(base + ((c ^ ((r >> 1) & 3)) << 4), pack_half2(v[8 * c], v[8 * c + 1]),
                 pack_half2(v[8 * c + 2], v[8 * c + 3]), pack_half2(v[8 * c + 4], v[8 * c + 5]),
                 pack_half2(v[8 * c + 6], v[8 * c + 7]));
}

// [32 rows x 16 FP16], 32-byte rows, SWIZZLE_32B.
__device__ __forceinline__ void stage_row_f16x16(uint32_t tile, int r, const float* v) {
  const uint32_t base = tile + r * 32;
#pragma unroll
  for (int c = 0; c < 2; ++c)
    st_shared_v4(base + ((c ^ ((r >> 2) & 1)) << 4), pack_half2(v[8 * c], v[8 * c + 1]),
                 pack_half2(v[8 * c + 2], v[8 * c + 3]), pack_half2(v[8 * c + 4], v[8 * c + 5]),
                 pack_half2(v[8 * c + 6], v[8 * c + 7]));
}

// Transposed staging of V: lane s holds v[0..W) = features d0..d0+W-1 of
// token s; the tile is [W feature rows x 32 tokens] FP16 (64-byte rows,
// SWIZZLE_64B).  Lane pairs (2k, 2k+1) swap halves with one shuffle per two
// features, then each lane writes packed (token 2k, token 2k+1) words: even
// lanes the even feature rows, odd lanes the odd ones (conflict-free).
template <int W>
__device__ __forceinline__ void stage_cols_f16(uint32_t tile, int lane, const float* v) {
  const bool odd = lane & 1;
  const int k = lane >> 1;  // word (token pair) within a 64-byte row
#pragma unroll
  for (int j = 0; j < W / 2; ++j) {
    const float send = odd ? v[2 * j] : v[2 * j + 1];
    const float recv = __shfl_xor_sync(0xffffffffu, send, 1);
    const int d = 2 * j + (odd ? 1 : 0);
    const uint32_t word = odd ? pack_half2(recv, v[2 * j + 1]) : pack_half2(v[2 * j], recv);
    const uint32_t addr = tile + d * 64 + ((((k >> 2) ^ ((d >> 1) & 3))) << 4) + (k & 3) * 4;
    asm volatile("st.shared.b32 [%0], %1;" ::"r"(addr), "r"(word) : "memory");
  }
}

// Output staging ring of one epilogue warp: before a slot is rewritten, the
// bulk store that last read it must be done reading shared memory.
template <int NR>
struct OutRing {
  uint32_t base;  // shared address of slot 0
  int count;      // slots used so far
  __device__ __forceinline__ uint32_t acquire(int lane) {
    if (lane == 0) bulk_wait_group_read<NR - 1>();
    __syncwarp();
    return base + (count % NR) * kEpiTile;
  }
  // All lanes wrote the slot with generic stores; make them visible to the
  // async proxy before lane 0 issues the TMA store(s).
  __device__ __forceinline__ void publish() {
    fence_proxy_async_smem();
    __syncwarp();
    ++count;
  }
};

// RR: residual tiles in flight per epilogue warp (gemm_res_ring of the launch's bn).
template <int KSW, int EPI, int RR>
__global__ void __launch_bounds__(gemm_threads(EPI), 1)
    gemm_kernel(const __grid_constant__ GemmMaps maps, const GemmParams p) {
  constexpr int NEPI = gemm_epi_warps(EPI);  // epilogue warps 0..NEPI-1
  constexpr int NSTEP = NEPI / 4;            // warps sharing one TMEM lane quadrant
  static_assert(NEPI == 4 || NEPI == 8, "residual barriers and the statistics exchange assume 4 or 8 epilogue warps");
  constexpr int W_PROD = NEPI, W_MMA = NEPI + 1;  // further producers: warps NEPI + 2 ...
  constexpr int A_BYTES = 128 * KSW * 2;
  constexpr uint32_t kSw = swizzle_kind_for_bytes(KSW * 2);
  constexpr uint32_t kSbo = 8 * KSW * 2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int bn = p.bn, nst = p.nst;
  const int stage_bytes = gemm_stage_bytes(KSW, bn);
  const int w_bytes_half = (bn > 256 ? 256 : bn) * KSW * 2;
  uint8_t* stages = smem;
  uint8_t* epi = stages + nst * stage_bytes;
  float* s_bias = reinterpret_cast<float*>(epi + gemm_epi_bytes(EPI, RR));  // [N_total]
  float* s_gamma = s_bias + p.N_total;                                    // [bn] (RESID_LN)
  float* s_beta = s_gamma + bn;
  uint64_t* full = reinterpret_cast<uint64_t*>(s_beta + bn);
  uint64_t* empty = full + kGemmMaxStages;
  uint64_t* acc_full = empty + kGemmMaxStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* res_full = acc_empty + 2;  // [epilogue warp][kResRing]
  uint64_t* xbar = res_full + 8 * kResRing;  // [lane quadrant]: statistics exchange (split LN)
  uint64_t* done = xbar + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // [item parity][quadrant][column half][mean, M2][lane]
  float* xch = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(done + 1) + 16);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = p.K / KSW;
  const int n_acc = gemm_n_acc(bn);
  const int acc_stride = gemm_acc_stride(bn);
  const uint32_t tmem_cols = static_cast<uint32_t>(gemm_tmem_cols(bn));

  if (threadIdx.x == 0) {
    for (int i = 0; i < nst; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], NEPI);
    }
    for (int i = 0; i < NEPI * kResRing; ++i) mbar_init(&res_full[i], 1);
    for (int i = 0; i < 4; ++i) mbar_init(&xbar[i], 2);
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  for (int c = threadIdx.x; c < p.N_total; c += blockDim.x) s_bias[c] = p.bias[c];
  if constexpr (EPI == EPI_RESID_LN) {
    for (int c = threadIdx.x; c < (p.no_norm ? 0 : bn); c += blockDim.x) {
      s_gamma[c] = p.gamma[c];
      s_beta[c] = p.beta[c];
    }
  }
  if (warp == W_MMA) {
    tmem_alloc(tmem_slot, tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_wait();  // activations of the previous kernel are final from here on
  pdl_trigger();
  const uint32_t tmem_base = *tmem_slot;
  const Watchdog wd{p.err, abort_flag, p.timeout_ns};

  if (warp == W_PROD || warp > W_MMA) {
    // ------------------------------------------------------------ producers
    // A producer thread completes only about one TMA copy per ~800 cycles
    // whatever the copy size, so the ring's slots are shared out among several.
    const int pidx = warp == W_PROD ? 0 : warp - W_MMA;
    if (lane == 0) {
      tma_prefetch_desc(&maps.a);
      tma_prefetch_desc(&maps.w);
      int g = 0;
      bool ok = true;
      for (int w = blockIdx.x; ok && w < p.n_items; w += gridDim.x) {
        const int m0 = (w / p.n_splits) * 128;
        const int n0 = (w % p.n_splits) * bn;
        for (int kb = 0; kb < nk; ++kb, ++g) {
          if ((g % nst) % kGemmProducers != pidx) continue;
          const int st = g % nst;
          if (!(ok = wait_phase(&empty[st], ((g / nst) & 1) ^ 1, wd, 0x401))) break;
          uint8_t* sa = stages + st * stage_bytes;
          uint8_t* sw = sa + A_BYTES;
          mbar_arrive_expect_tx(&full[st], stage_bytes);
          tma_load_2d(sa, &maps.a, &full[st], kb * KSW, m0);
          tma_load_2d(sw, &maps.w, &full[st], kb * KSW, n0);
          if (bn > 256) tma_load_2d(sw + w_bytes_half, &maps.w, &full[st], kb * KSW, n0 + 256);
        }
      }
      for (int i = (g > nst ? g - nst : 0); i < g; ++i)
        if ((i % nst) % kGemmProducers == pidx) wait_drain(&full[i % nst], (i / nst) & 1, kDrainLimitNs);
    }
  } else if (warp == W_MMA) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_f16_f32(128, bn > 256 ? 256 : bn);
      const uint32_t base = smem_u32(stages);
      int g = 0, i = 0;
      bool ok = true;
      for (int w = blockIdx.x; ok && w < p.n_items; w += gridDim.x, ++i) {
        const int ab = i % n_acc;
        if (!(ok = wait_phase(&acc_empty[ab], ((i / n_acc) & 1) ^ 1, wd, 0x403))) break;
        tc_fence_after();
        const uint32_t tacc = tmem_base + ab * acc_stride;
        for (int kb = 0; kb < nk; ++kb, ++g) {
          const int st = g % nst;
          if (!(ok = wait_phase(&full[st], (g / nst) & 1, wd, 0x402))) break;
          tc_fence_after();
          const uint32_t sa = base + st * stage_bytes;
          const uint32_t sw = sa + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < KSW / 16; ++kk) {
            const uint64_t da = umma_sdesc(sa + kk * 32, kSbo, kSw);
            const uint32_t acc = (kb > 0 || kk > 0) ? 1u : 0u;
            umma_f16(tacc, da, umma_sdesc(sw + kk * 32, kSbo, kSw), idesc, acc);
            if (bn > 256)
              umma_f16(tacc + 256, da, umma_sdesc(sw + w_bytes_half + kk * 32, kSbo, kSw), idesc, acc);
          }
          umma_commit(&empty[st]);
        }
        if (ok) umma_commit(&acc_full[ab]);
      }
      umma_commit(done);
      wait_drain(done, 0, kDrainLimitNs);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int r = lane;         // row within this warp's 32-row slab
    const int eq = warp & 3;    // TMEM lane quadrant (rows eq*32 .. eq*32+31 of the tile)
    const int ehalf = warp >> 2;  // which of the NSTEP warps on this quadrant
    const uint32_t lane_base = static_cast<uint32_t>(eq * 32) << 16;
    constexpr int kRes = (EPI == EPI_RESID_LN) ? RR : 0;
    constexpr int kOut = gemm_out_ring(EPI);
    const uint32_t res_base = smem_u32(epi) + warp * (kRes + kOut) * kEpiTile;
    OutRing<kOut> ring{res_base + kRes * kEpiTile, 0};
    uint64_t* my_res_full = res_full + warp * kResRing;  // the first RR of them are used
    int res_g = 0;         // residual tiles this warp has requested and consumed
    bool res_pre = false;  // this item's first residual tiles already went out
    int i = 0;
    bool ok = true;
    for (int w = blockIdx.x; ok && w < p.n_items; w += gridDim.x, ++i) {
      const int m0 = (w / p.n_splits) * 128;
      const int n0 = (w % p.n_splits) * bn;
      const int r0 = m0 + eq * 32;  // first row of this warp's slab
      const int row = r0 + r;
      const bool valid = row < p.M;
      const bool warp_active = r0 < p.M;
      const int nch = bn / 32;
      // EPI_RESID_LN: this warp's 32-column chunks [c_lo, c_hi) (half of them
      // with the split epilogue, where the pair of a quadrant shares a row).
      const int c_lo = NSTEP == 2 ? ehalf * nch / 2 : 0;
      const int c_hi = NSTEP == 2 ? (ehalf + 1) * nch / 2 : nch;
      // Residual tiles of this item: the first RR go out now, unless the
      // previous item sent them during its normalization pass.
      if constexpr (EPI == EPI_RESID_LN) {
        if (lane == 0 && warp_active && !res_pre) {
          for (int k = 0; c_lo + k < c_hi && k < RR; ++k) {
            const int q = res_g + k;
            mbar_arrive_expect_tx(&my_res_full[q % RR], kEpiTile);
            tma_load_2d_u32(res_base + (q % RR) * kEpiTile, &maps.res, &my_res_full[q % RR],
                            n0 + 32 * (c_lo + k), r0);
          }
        }
      }
      const int ab = i % n_acc;
      if (!(ok = warp_wait_phase(&acc_full[ab], (i / n_acc) & 1, wd, 0x404))) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + lane_base + ab * acc_stride;

      if constexpr (EPI == EPI_QKV) {
        const int D = p.d_model, hd = p.head_dim;
        // head_dim is a power of two (8 .. 256): heads and features by shift and mask; the
        // Q/K/V part of a column by one division per item (chunks of 32 never
        // straddle a part, D % 32 == 0).
        const int lg_hd = __ffs(hd) - 1;
        const int which_item = n0 / D;
        const int within_item = n0 - which_item * D;
        const int bidx = valid ? row / p.seq : 0;
        const int s = valid ? row - bidx * p.seq : 0;
        const int b_w = warp_active ? r0 / p.seq : 0;
        const int s0 = warp_active ? r0 - b_w * p.seq : 0;
        // This warp takes chunks ehalf, ehalf + NSTEP, ...; two TMEM loads per wait.
        for (int cb = ehalf; cb < nch; cb += 2 * NSTEP) {
          uint32_t vv[2][32];
          __syncwarp();
          tmem_ld_x32(taddr + cb * 32, vv[0]);
          if (cb + NSTEP < nch) tmem_ld_x32(taddr + (cb + NSTEP) * 32, vv[1]);
          tmem_ld_wait_tied(vv[0]);
          tmem_ld_wait_tied(vv[1]);
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int c = cb + u * NSTEP;
          if (c >= nch) break;
          const uint32_t (&v)[32] = vv[u];
          const int col0 = n0 + c * 32;
          float f[32];
          const float4* b4 = reinterpret_cast<const float4*>(s_bias + col0);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float4 bb = b4[e];
            f[4 * e + 0] = __uint_as_float(v[4 * e + 0]) + bb.x;
            f[4 * e + 1] = __uint_as_float(v[4 * e + 1]) + bb.y;
            f[4 * e + 2] = __uint_as_float(v[4 * e + 2]) + bb.z;
            f[4 * e + 3] = __uint_as_float(v[4 * e + 3]) + bb.w;
          }
          int which = which_item, within0 = within_item + c * 32;
          while (within0 >= D) {
            within0 -= D;
            ++which;
          }
          if (p.tma_out && hd >= 32) {
            // Q, K, V^T by TMA bulk stores of [32 x 32] FP16 tiles (64-byte rows,
            // SWIZZLE_64B) through maps.out0 / out1 / res, the 2-D views
            // [B*H*S, hd] of Q and K and [B*H*hd, S_pad] of V^T.  The warp's slab
            // lies within one sequence (S % 32 == 0), so each tile is one box.
            if (!warp_active) continue;
            const int hh = within0 >> lg_hd, d0 = within0 & (hd - 1);
            const int bh = b_w * p.heads + hh;
            const uint32_t slot = ring.acquire(lane);
            if (which < 2)
              stage_row_f16x32(slot, lane, f);
            else
              stage_cols_f16<32>(slot, lane, f);
            ring.publish();
            if (lane == 0) {
              if (which < 2)
                tma_store_2d(which == 0 ? &maps.out0 : &maps.out1, slot, d0, bh * p.seq + s0);
              else
                tma_store_2d(&maps.res, slot, s0, bh * hd + d0);
              bulk_commit_group();
            }
          } else if (which < 2 && hd == 8) {
            // Q / K with head_dim 8, stored 16 wide: each of the chunk's 4 heads is
            // the row's 8 features and 8 zeros (32 contiguous bytes of [B*H, S, 16]).
            if (valid) {
              __half* base = which == 0 ? p.q : p.k;
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const int hh = (within0 >> 3) + j;
                uint4* dst = reinterpret_cast<uint4*>(
                    base + ((static_cast<size_t>(bidx) * p.heads + hh) * p.seq + s) * 16);
                uint4 a;
                a.x = pack_half2(f[8 * j + 0], f[8 * j + 1]);
                a.y = pack_half2(f[8 * j + 2], f[8 * j + 3]);
                a.z = pack_half2(f[8 * j + 4], f[8 * j + 5]);
                a.w = pack_half2(f[8 * j + 6], f[8 * j + 7]);
                dst[0] = a;
                dst[1] = make_uint4(0, 0, 0, 0);
              }
            }
          } else if (which < 2) {
            // Q / K, rows not staged: a thread's 32 values are consecutive features of
            // its row, in runs of 16 that are each 32 contiguous bytes of [B*H, S, hd].
            if (valid) {
              __half* base = which == 0 ? p.q : p.k;
#pragma unroll
              for (int gq = 0; gq < 2; ++gq) {
                const int within = within0 + 16 * gq;
                const int hh = within >> lg_hd, d = within & (hd - 1);
                uint4* dst = reinterpret_cast<uint4*>(
                    base + ((static_cast<size_t>(bidx) * p.heads + hh) * p.seq + s) * hd + d);
                uint4 a, bq;
                a.x = pack_half2(f[16 * gq + 0], f[16 * gq + 1]);
                a.y = pack_half2(f[16 * gq + 2], f[16 * gq + 3]);
                a.z = pack_half2(f[16 * gq + 4], f[16 * gq + 5]);
                a.w = pack_half2(f[16 * gq + 6], f[16 * gq + 7]);
                bq.x = pack_half2(f[16 * gq + 8], f[16 * gq + 9]);
                bq.y = pack_half2(f[16 * gq + 10], f[16 * gq + 11]);
                bq.z = pack_half2(f[16 * gq + 12], f[16 * gq + 13]);
                bq.w = pack_half2(f[16 * gq + 14], f[16 * gq + 15]);
                dst[0] = a;
                dst[1] = bq;
              }
            }
          } else if (p.tma_out && hd == 16) {
            // V^T at head_dim 16: transpose the 32 rows through this warp's staging
            // tile, then write two [16 features x 32 tokens] blocks as 64-byte rows
            // of [B*H, 16, S_pad] with coalesced 16-byte stores (the slab lies
            // within one sequence: S % 32 == 0).
            if (!warp_active) continue;
            const uint32_t slot = ring.base;
            __syncwarp();
            stage_cols_f16<16>(slot, lane, f);
            stage_cols_f16<16>(slot + 1024, lane, f + 16);
            __syncwarp();
#pragma unroll 1
            for (int sb = 0; sb < 2; ++sb) {
              const int within = within0 + sb * 16;
              const int hh = within >> lg_hd, d0 = within & (hd - 1);
              const size_t bh = static_cast<size_t>(b_w) * p.heads + hh;
              for (int k = 0; k < 2; ++k) {
                const int d = k * 8 + (lane >> 2), pc = lane & 3;
                const uint4 q = ld_shared_v4(slot + sb * 1024 + d * 64 + ((pc ^ ((d >> 1) & 3)) << 4));
                *reinterpret_cast<uint4*>(p.vt + (bh * hd + d0 + d) * p.seq_pad + s0 + pc * 8) = q;
              }
            }
            __syncwarp();
          } else if (valid) {
            // V^T one element at a time ([B*H, hs, S_pad], hs = 16 for head_dim 8:
            // rows 8..15 of a head are never read into any stored output).
            const int hs = hd < 16 ? 16 : hd;
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              const int within = within0 + e;
              const int hh = within >> lg_hd, d = within & (hd - 1);
              p.vt[((static_cast<size_t>(bidx) * p.heads + hh) * hs + d) * p.seq_pad + s] =
                  __float2half_rn(f[e]);
            }
          }
        }
        }
      } else if constexpr (EPI == EPI_GELU) {
        for (int cb = ehalf; cb < nch; cb += 2 * NSTEP) {
          uint32_t vv[2][32];
          __syncwarp();
          tmem_ld_x32(taddr + cb * 32, vv[0]);
          if (cb + NSTEP < nch) tmem_ld_x32(taddr + (cb + NSTEP) * 32, vv[1]);
          tmem_ld_wait_tied(vv[0]);
          tmem_ld_wait_tied(vv[1]);
          if (!warp_active) continue;
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int c = cb + u * NSTEP;
          if (c >= nch) break;
          const uint32_t (&v)[32] = vv[u];
          float gl[32];
          const float4* b4 = reinterpret_cast<const float4*>(s_bias + n0 + c * 32);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float4 bb = b4[e];
            gl[4 * e + 0] = gelu_erf(__uint_as_float(v[4 * e + 0]) + bb.x);
            gl[4 * e + 1] = gelu_erf(__uint_as_float(v[4 * e + 1]) + bb.y);
            gl[4 * e + 2] = gelu_erf(__uint_as_float(v[4 * e + 2]) + bb.z);
            gl[4 * e + 3] = gelu_erf(__uint_as_float(v[4 * e + 3]) + bb.w);
          }
          const uint32_t slot = ring.acquire(lane);
          stage_row_f16x32(slot, r, gl);
          ring.publish();
          if (lane == 0) {
            tma_store_2d(&maps.out0, slot, n0 + c * 32, r0);
            bulk_commit_group();
          }
        }
        }
      } else {
        // EPI_RESID_LN: bn == N_total == d_model (the whole row lives in TMEM),
        // or, with p.no_norm, any column split of the row (pass 1 only).
        // Pass 1 (two chunks per TMEM wait): r' = acc + bias + residual, written
        // back into TMEM and out to HBM, with FP32 sums of r' - shift (shift =
        // the row's first r') for the mean and variance; pass 2 normalizes.
        const int D = bn;
        float shift = 0.f, s1 = 0.f, s2 = 0.f;
        for (int cb = c_lo; cb < c_hi; cb += 2) {
          uint32_t vv[2][32];
          __syncwarp();
          tmem_ld_x32(taddr + cb * 32, vv[0]);
          if (cb + 1 < c_hi) tmem_ld_x32(taddr + (cb + 1) * 32, vv[1]);
          tmem_ld_wait_tied(vv[0]);
          tmem_ld_wait_tied(vv[1]);
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int c = cb + u;
          if (c >= c_hi) break;
          const uint32_t (&v)[32] = vv[u];
          float res[32];
          const int q = res_g + (c - c_lo);
          if (warp_active) {
            if (!(ok = warp_wait_phase(&my_res_full[q % RR], (q / RR) & 1, wd, 0x405)))
              break;
            load_row_f32(res_base + (q % RR) * kEpiTile, r, res);
            __syncwarp();
            // The slot is read; refill it with the tile RR chunks ahead.
            if (lane == 0 && c + RR < c_hi) {
              fence_proxy_async_smem();
              const int q2 = q + RR;
              mbar_arrive_expect_tx(&my_res_full[q2 % RR], kEpiTile);
              tma_load_2d_u32(res_base + (q2 % RR) * kEpiTile, &maps.res,
                              &my_res_full[q2 % RR], n0 + 32 * (c + RR), r0);
            }
          } else {
#pragma unroll
            for (int e = 0; e < 32; ++e) res[e] = 0.f;
          }
          float rr[32];
          uint32_t out[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            rr[e] = __uint_as_float(v[e]) + s_bias[n0 + c * 32 + e] + res[e];
            out[e] = __float_as_uint(rr[e]);
          }
          if (c == c_lo) shift = rr[0];
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const float d = rr[e] - shift;
            s1 += d;
            s2 = fmaf(d, d, s2);
          }
          __syncwarp();
          tmem_st_x32(taddr + c * 32, out);
          if (warp_active) {
            const uint32_t slot = ring.acquire(lane);
            stage_row_f32(slot, r, rr);
            ring.publish();
            if (lane == 0) {
              tma_store_2d(&maps.out0, slot, n0 + c * 32, r0);
              bulk_commit_group();
            }
          }
        }
          if (!ok) break;
        }
        if (!ok) break;
        if (warp_active) res_g += c_hi - c_lo;
        // The ring is free until the next item: send that item's first residual
        // tiles now, so that they land while this item is normalized.
        res_pre = false;
        if (const int wn = w + static_cast<int>(gridDim.x); wn < p.n_items) {
          const int r0n = (wn / p.n_splits) * 128 + eq * 32;
          if (r0n < p.M) {
            if (lane == 0) {
              fence_proxy_async_smem();
              for (int k = 0; c_lo + k < c_hi && k < RR; ++k) {
                const int q = res_g + k;
                mbar_arrive_expect_tx(&my_res_full[q % RR], kEpiTile);
                tma_load_2d_u32(res_base + (q % RR) * kEpiTile, &maps.res, &my_res_full[q % RR],
                                (wn % p.n_splits) * bn + 32 * (c_lo + k), r0n);
              }
            }
            res_pre = true;
          }
        }
        tmem_st_wait();
        if (p.no_norm) {
          // The accumulator buffer may be overwritten by the next item's MMAs.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[ab]);
          continue;
        }
        // Row statistics: this warp's columns give (count, mean, M2) from the
        // shifted sums; with the split epilogue the two warps of the quadrant
        // swap theirs through shared memory and both combine them in column
        // order (half 0, then half 1), so that they normalize with identical
        // values.
        float mean, rstd;
        {
          const int n_mine = 32 * (c_hi - c_lo);
          float mean_a = 0.f, m2_a = 0.f;
          if (n_mine > 0) {
            const float inv = 1.f / static_cast<float>(n_mine);
            mean_a = shift + s1 * inv;
            m2_a = fmaxf(s2 - s1 * s1 * inv, 0.f);
          }
          int n_a = n_mine, n_b = 0;
          float mean_b = 0.f, m2_b = 0.f;
          if constexpr (NSTEP == 2) {
            float* xs = xch + ((i & 1) * 4 + eq) * 128;  // [half][mean, M2][lane]
            xs[ehalf * 64 + lane] = mean_a;
            xs[ehalf * 64 + 32 + lane] = m2_a;
            __syncwarp();
            if (lane == 0) mbar_arrive(&xbar[eq]);
            // Slot (i & 1) is rewritten at item i + 2, after both warps have
            // passed item i + 1's exchange, so the partner's values stay put.
            if (!(ok = warp_wait_phase(&xbar[eq], i & 1, wd, 0x406))) break;
            const int oh = ehalf ^ 1;
            const float mean_o = xs[oh * 64 + lane], m2_o = xs[oh * 64 + 32 + lane];
            const int n_o = 32 * ((oh + 1) * nch / 2 - oh * nch / 2);
            if (ehalf == 0) {
              mean_b = mean_o, m2_b = m2_o, n_b = n_o;
            } else {
              mean_b = mean_a, m2_b = m2_a, n_b = n_mine;
              mean_a = mean_o, m2_a = m2_o, n_a = n_o;
            }
          }
          const float fb = static_cast<float>(n_b) / static_cast<float>(n_a + n_b);
          const float delta = mean_b - mean_a;
          mean = fmaf(delta, fb, mean_a);
          const float m2 = m2_a + m2_b + delta * delta * static_cast<float>(n_a) * fb;
          rstd = rsqrtf(fmaxf(m2 / static_cast<float>(D), 0.f) + p.eps);
        }
        const bool zero_row = valid && p.row_mask != nullptr && p.row_mask[row] == 0;
        for (int cb = c_lo; cb < c_hi; cb += 2) {
          uint32_t vv[2][32];
          __syncwarp();
          tmem_ld_x32(taddr + cb * 32, vv[0]);
          if (cb + 1 < c_hi) tmem_ld_x32(taddr + (cb + 1) * 32, vv[1]);
          tmem_ld_wait_tied(vv[0]);
          tmem_ld_wait_tied(vv[1]);
          if (!warp_active) continue;
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int c = cb + u;
          if (c >= c_hi) break;
          const uint32_t (&v)[32] = vv[u];
          float y[32];
#pragma unroll
          for (int e = 0; e < 32; ++e)
            y[e] = zero_row ? 0.f
                            : fmaf((__uint_as_float(v[e]) - mean) * rstd, s_gamma[c * 32 + e],
                                   s_beta[c * 32 + e]);
          const uint32_t slot = ring.acquire(lane);
          if (p.norm_f16)
            stage_row_f16x32(slot, r, y);
          else
            stage_row_f32(slot, r, y);
          ring.publish();
          if (lane == 0) {
            tma_store_2d(&maps.out1, slot, n0 + c * 32, r0);
            bulk_commit_group();
          }
        }
        }
      }
      // The accumulator buffer may be overwritten by the next item's MMAs.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[ab]);
    }
    if (lane == 0) bulk_wait_group_all();
    // Residual tiles requested but never consumed (abort path) must land first.
    if constexpr (EPI == EPI_RESID_LN) {
      if (lane == 0 && !ok)
        for (int k2 = 0; k2 < RR; ++k2)
          wait_drain(&my_res_full[(res_g + k2) % RR], ((res_g + k2) / RR) & 1, kDrainLimitNs);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == W_MMA) {
    tc_fence_after();
    tmem_dealloc(tmem_base, tmem_cols);
  }
}

}  // namespace tt
