// Fully fused feed-forward block for sm_100a, d_model 128 and 256:
//
//   h   = GELU_erf(n . W1^T + b1)      FP32 math, FP16 h kept in TMEM (never in HBM or shared memory)
//   r'  = h . W2^T + b2 + r            FP32 residual stream
//   n'  = LayerNorm(r') * gamma + beta  FP16 next input, or FP32 model output
//
// Replaces the reference's `_mixed_ffn_add_layer_norm_kernel`
// (mixed_precision/triton_linear.py:128-185) and the ffn_in -> GELU -> ffn_out
// -> fused_add_layer_norm chain of its generic route
// (mixed_precision/transformer.py:669-695), for F a multiple of 128.
//
// Persistent kernel over 128-row tiles; the hidden dimension runs in chunks
// of FC = 128 units (NACC1 = 256 / FC accumulator buffers).  Per chunk c
// (buffer b = c % NACC1):
//   G1(c)  acc1[b] (TMEM, 128 x FC FP32) = A . W1[c]^T
//   GELU   8 warps: acc1[b] + b1 -> GELU -> FP16 pairs written back into the
//          first half of each warp's own columns of acc1[b]: H(c) stays in
//          TMEM and is the A operand of G2 (tcgen05.mma with A in TMEM)
//   G2(c)  acc2 (TMEM, 128 x D FP32) += H(c) . W2[:, c]^T
// issued as G1(c) then G2(c - LAG) (LAG = 1: G1(0) G1(1) G2(0) G1(2) G2(1)
// ...); acc1[b] is rewritten by G1(c + NACC1) only after G2(c) has read H(c)
// (the tensor core executes one thread's MMAs in issue order; LAG < NACC1).
// With H out of shared memory the weight ring holds NST = 3 slots of 32 KB,
// each one TMA copy (W1: FC rows x the K-blocks that fill 32 KB, as a 3-D
// K-block view; W2: 64 hidden units x D rows).
//
// Epilogue (4 warps, one row per thread): one TMEM pass computes
// r' = acc2 + b2 + r (the residual rows bulk-prefetched into L2 a tile ahead,
// then staged by cp.async AHEAD = 6 16-column jobs ahead), accumulates
// shifted FP32 sums for the LayerNorm statistics and writes r' with coalesced
// stores; the second pass re-reads the warp's own r' rows (L2 hits) and
// writes the normalized rows.  acc2 is read 64 columns at a time into
// registers and each 64-column block is released as soon as it is loaded:
// the next tile's first G2 chunk is issued as D / 64 MMAs of N = 64, each
// waiting only for its own block, so the tensor core resumes while the
// epilogue is still at the start of its first pass (with a single
// accumulator it used to idle until the whole pass was done).  d_model 128
// double-buffers acc2 in TMEM as well.
// Warp 12 loads A and the even ring slots, warp 14 the odd ones (more
// producers: warps 14, 15, ... own slots st % producers); warp 13 allocates
// TMEM and issues the MMAs.
#pragma once

#include "tt_ffn.cuh"

namespace tt {

// a and w1 are 3-D views {64 (k within a K-block), rows, K-blocks} with byte
// strides {D * 2, 128}, so one TMA copy lays several K-blocks out as
// consecutive 128-row x 128-byte swizzled blocks (a producer thread
// completes only about one copy per ~800 cycles, whatever its size).
struct Ffn2Maps {
  CUtensorMap a;   // [M, D] FP16, box {64, 128, D / 64} (the whole row tile), SWIZZLE_128B
  CUtensorMap w1;  // [F, D] FP16, box {64, 128, 2}
  CUtensorMap w2;  // [D, F] FP16 (2-D), box {64, min(D, 256)}
};

template <int D>
struct Ffn2Layout {
  // Hidden units per chunk, TMEM buffers of the chunk accumulator (columns
  // 256..511), and how many chunks G2 trails G1.
  static constexpr int FC = 128, KB = 64, NST = 3, SLOT = 32768;
  static constexpr int NACC1 = 256 / FC, LAG = 1;
  static constexpr int NKA = D / KB;                 // K-blocks of G1
  static constexpr int A_KBLK = 128 * KB * 2;        // 16 KB
  static constexpr int A_BYTES = NKA * A_KBLK;
  static constexpr int W1_KBLK = FC * KB * 2;        // 16 KB
  static constexpr int W1_PER_SLOT = SLOT / W1_KBLK;  // 2
  static constexpr int W1_SLOTS = NKA / W1_PER_SLOT;
  static constexpr int W2_KBLK = D * KB * 2;         // D rows x 64 hidden units
  static constexpr int W2_PER_SLOT = SLOT / W2_KBLK;
  static constexpr int W2_SLOTS = (FC / KB) / W2_PER_SLOT;
  static constexpr int W2_BOX_ROWS = D < 256 ? D : 256;
  static constexpr int JW = 16;       // columns per epilogue job
  static constexpr int AHEAD = 6;  // epilogue jobs in flight ahead of the one consumed
  static constexpr int RING = AHEAD + 1;      // 32 x JW FP32 staging tiles per epilogue warp
  static constexpr int TILE = 32 * JW * 4;
  static constexpr int OFF_A = 0;
  static constexpr int OFF_W = OFF_A + A_BYTES;
  static constexpr int OFF_LN = OFF_W + NST * SLOT;
  static constexpr int OFF_F32 = OFF_LN + 4 * RING * TILE;  // b2, gamma, beta
  static constexpr int OFF_BAR = OFF_F32 + 3 * D * 4;
  static constexpr int NBLK = D / 64;  // 64-column blocks of acc2, released one by one
  // a_full a_empty w_full[NST] w_empty[NST] acc1_full[NACC1] h_full[NACC1] acc2_full[2]
  // acc2_empty[2][NBLK] done
  static constexpr int NBAR = 2 + 2 * NST + 2 * NACC1 + 2 + 2 * NBLK + 1;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int SMEM_ALLOC = OFF_MISC + 16 + 1024;
  static constexpr int NACC2 = D <= 128 ? 2 : 1;  // acc2 buffers (TMEM columns [j * D, (j + 1) * D))
  static constexpr int TMEM_ACC1 = 256;           // acc1 buffer b at columns 256 + FC b
  static_assert(D == 128 || D == 256, "this kernel covers d_model 128 and 256");
  static_assert(D % 64 == 0 && 64 % JW == 0, "acc2 released in 64-column blocks of whole jobs");
  static_assert(W1_SLOTS >= 1 && W2_SLOTS >= 1 && W1_PER_SLOT * W1_KBLK == SLOT && W2_PER_SLOT * W2_KBLK == SLOT,
                "slot shapes");
  static_assert(NACC2 * D <= TMEM_ACC1, "TMEM budget");
  static_assert(OFF_W % 1024 == 0 && OFF_LN % 1024 == 0 && OFF_F32 % 16 == 0, "alignment");
  static_assert(SMEM_ALLOC <= 232448, "shared memory budget");
  static_assert(D / JW > AHEAD, "the re-read of an r' chunk must be issued after that chunk's store");
  static_assert((FC == 64 || FC == 128) && LAG >= 1 && LAG < NACC1,
                "G1(c) rewrites the buffer of H(c - NACC1), which G2 must have read: LAG < NACC1");
};

// Warp roles: 0..7 GELU (lane quadrant w & 3, hidden half w >> 2 of each
// chunk), 8..11 residual + LayerNorm, 12 and 14.. TMA producers, 13 TMEM
// allocator and MMA issuer.
constexpr int kFfn2Producers = 2;  // warps 12, 14, 15, ...
constexpr int kFfn2Threads = 32 * (13 + kFfn2Producers);
constexpr int kFfn2Prod0 = 12, kFfn2Mma = 13;

template <int D>
__global__ void __launch_bounds__(kFfn2Threads, 1)
    ffn2_kernel(const __grid_constant__ Ffn2Maps maps, const FfnParams p) {
  using L = Ffn2Layout<D>;
  constexpr int FC = L::FC, NST = L::NST;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  float* s_b2 = reinterpret_cast<float*>(smem + L::OFF_F32);
  float* s_gamma = s_b2 + D;
  float* s_beta = s_gamma + D;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* a_full = bars;
  uint64_t* a_empty = bars + 1;
  uint64_t* w_full = bars + 2;
  uint64_t* w_empty = w_full + NST;
  uint64_t* acc1_full = w_empty + NST;
  uint64_t* h_full = acc1_full + L::NACC1;
  uint64_t* acc2_full = h_full + L::NACC1;
  uint64_t* acc2_empty = acc2_full + 2;  // [buffer][64-column block]
  uint64_t* done = acc2_empty + 2 * L::NBLK;
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
    for (int i = 0; i < L::NACC1; ++i) {
      mbar_init(&acc1_full[i], 1);
      mbar_init(&h_full[i], 8);
    }
    for (int i = 0; i < 2; ++i) mbar_init(&acc2_full[i], 1);
    for (int i = 0; i < 2 * L::NBLK; ++i) mbar_init(&acc2_empty[i], 4);
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    s_b2[c] = p.b2[c];
    s_gamma[c] = p.gamma[c];
    s_beta[c] = p.beta[c];
  }
  if (warp == kFfn2Mma) {
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

  if (warp == kFfn2Prod0 || warp > kFfn2Mma) {
    // ------------------------------------------------------------ producers
    // Ring slot st is always filled by producer st % kFfn2Producers (one
    // producer per slot keeps the parity-based empty-slot wait exact).
    const int pidx = warp == kFfn2Prod0 ? 0 : warp - kFfn2Mma;
    if (lane == 0) {
      tma_prefetch_desc(&maps.a);
      tma_prefetch_desc(&maps.w1);
      tma_prefetch_desc(&maps.w2);
      int g = 0, i = 0;
      bool ok = true;
      // One slot: W1 K-blocks of chunk c (G1) or W2 hidden K-blocks of chunk c (G2).
      auto slot_load = [&](bool g2, int c, int s) -> bool {
        const int st = g % NST;
        if (st % kFfn2Producers == pidx) {
          if (!wait_phase(&w_empty[st], ((g / NST) & 1) ^ 1, wd, 0x601)) return false;
          mbar_arrive_expect_tx(&w_full[st], L::SLOT);
          uint8_t* dst = smem + L::OFF_W + st * L::SLOT;
          if (!g2) {
            tma_load_3d(dst, &maps.w1, &w_full[st], 0, c * FC, s * L::W1_PER_SLOT);
          } else {
#pragma unroll
            for (int q = 0; q < L::W2_PER_SLOT; ++q)
              tma_load_2d(dst + q * L::W2_KBLK, &maps.w2, &w_full[st],
                          c * FC + (s * L::W2_PER_SLOT + q) * L::KB, 0);
          }
        }
        ++g;
        return true;
      };
      for (int w = blockIdx.x; ok && w < p.n_items; w += gridDim.x, ++i) {
        const int m0 = w * 128;
        if (pidx == 0) {
          if (!(ok = wait_phase(a_empty, (i & 1) ^ 1, wd, 0x602))) break;
          mbar_arrive_expect_tx(a_full, L::A_BYTES);
          tma_load_3d(smem + L::OFF_A, &maps.a, a_full, 0, m0, 0);
          // The epilogue of the next tile reads its residual rows: start them towards L2 now.
          const int wn = w + static_cast<int>(gridDim.x);
          if (wn < p.n_items) {
            const int rows = min(128, p.M - wn * 128);
            prefetch_l2_bulk(p.resid_in + static_cast<size_t>(wn) * 128 * D,
                             static_cast<uint32_t>(rows) * D * 4u);
          }
        }
        for (int step = 0; ok && step < nchunk + L::LAG; ++step) {
          if (step < nchunk)
            for (int s = 0; ok && s < L::W1_SLOTS; ++s) ok = slot_load(false, step, s);
          if (step >= L::LAG)
            for (int s = 0; ok && s < L::W2_SLOTS; ++s) ok = slot_load(true, step - L::LAG, s);
        }
      }
      if (pidx == 0 && i > 0) wait_drain(a_full, (i - 1) & 1, kDrainLimitNs);
      for (int q = (g > NST ? g - NST : 0); q < g; ++q)
        if ((q % NST) % kFfn2Producers == pidx) wait_drain(&w_full[q % NST], (q / NST) & 1, kDrainLimitNs);
    }
  } else if (warp == kFfn2Mma) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc1 = umma_idesc_f16_f32(128, FC);
      const uint32_t idesc2 = umma_idesc_f16_f32(128, D);
      const uint32_t idesc2b = umma_idesc_f16_f32(128, 64);  // one 64-column block of acc2
      const uint32_t sA = smem_u32(smem + L::OFF_A);
      const uint32_t sW = smem_u32(smem + L::OFF_W);
      int g = 0, i = 0, cg = 0;
      bool ok = true;
      for (int w = blockIdx.x; ok && w < p.n_items; w += gridDim.x, ++i) {
        const int ib = i % L::NACC2;
        const uint32_t tacc2 = tmem_base + ib * D;
        if (!(ok = wait_phase(a_full, i & 1, wd, 0x611))) break;
        for (int step = 0; ok && step < nchunk + L::LAG; ++step) {
          if (step < nchunk) {
            // G1(step) -> acc1[c % NACC1].  Its previous contents, H(c - NACC1),
            // were read by G2(c - NACC1), issued before this MMA (LAG < NACC1).
            const int c = cg + step, ab = c % L::NACC1;
            const uint32_t tacc1 = tmem_base + L::TMEM_ACC1 + ab * FC;
            for (int s = 0; ok && s < L::W1_SLOTS; ++s, ++g) {
              const int st = g % NST;
              if (!(ok = wait_phase(&w_full[st], (g / NST) & 1, wd, 0x612))) break;
              tc_fence_after();
#pragma unroll
              for (int q = 0; q < L::W1_PER_SLOT; ++q) {
                const int kb = s * L::W1_PER_SLOT + q;
#pragma unroll
                for (int kk = 0; kk < L::KB / 16; ++kk) {
                  const uint64_t da = umma_sdesc(sA + kb * L::A_KBLK + kk * 32, 1024, kSw128);
                  const uint64_t db = umma_sdesc(sW + st * L::SLOT + q * L::W1_KBLK + kk * 32, 1024, kSw128);
                  umma_f16(tacc1, da, db, idesc1, (kb > 0 || kk > 0) ? 1u : 0u);
                }
              }
              umma_commit(&w_empty[st]);
            }
            if (!ok) break;
            umma_commit(&acc1_full[ab]);
            if (step == nchunk - 1) umma_commit(a_empty);
          }
          if (step >= L::LAG) {
            // G2(step - LAG): acc2 += H(c) . W2[:, chunk c]^T with H(c) in TMEM.
            const int c = cg + step - L::LAG, hb = c % L::NACC1;
            const uint32_t th = tmem_base + L::TMEM_ACC1 + hb * FC;
            if (!(ok = wait_phase(&h_full[hb], (c / L::NACC1) & 1, wd, 0x614))) break;
            tc_fence_after();
            if (step == L::LAG) {
              // The tile's first G2 chunk: acc2 block by block, each as soon as the
              // previous tile's epilogue has loaded it (N = 64 MMAs on rows 64 blk.. of W2).
              for (int s = 0; ok && s < L::W2_SLOTS; ++s)
                ok = wait_phase(&w_full[(g + s) % NST], ((g + s) / NST) & 1, wd, 0x615);
              if (!ok) break;
              for (int blk = 0; ok && blk < L::NBLK; ++blk) {
                if (!(ok = wait_phase(&acc2_empty[ib * L::NBLK + blk], ((i / L::NACC2) & 1) ^ 1, wd, 0x613)))
                  break;
                tc_fence_after();
                for (int s = 0; s < L::W2_SLOTS; ++s) {
                  const int st = (g + s) % NST;
#pragma unroll
                  for (int q = 0; q < L::W2_PER_SLOT; ++q) {
                    const int hk = s * L::W2_PER_SLOT + q;
#pragma unroll
                    for (int kk = 0; kk < L::KB / 16; ++kk) {
                      const int u = hk * 4 + kk;
                      const uint32_t ta = th + (u / (FC / 32)) * (FC / 2) + (u % (FC / 32)) * 8;
                      const uint64_t db = umma_sdesc(sW + st * L::SLOT + q * L::W2_KBLK + blk * 64 * 128 + kk * 32,
                                                     1024, kSw128);
                      umma_f16_ts(tacc2 + blk * 64, ta, db, idesc2b, (hk > 0 || kk > 0) ? 1u : 0u);
                    }
                  }
                }
              }
              if (!ok) break;
              for (int s = 0; s < L::W2_SLOTS; ++s) umma_commit(&w_empty[(g + s) % NST]);
              g += L::W2_SLOTS;
            }
            for (int s = 0; ok && step > L::LAG && s < L::W2_SLOTS; ++s, ++g) {
              const int st = g % NST;
              if (!(ok = wait_phase(&w_full[st], (g / NST) & 1, wd, 0x615))) break;
              tc_fence_after();
#pragma unroll
              for (int q = 0; q < L::W2_PER_SLOT; ++q) {
                const int hk = s * L::W2_PER_SLOT + q;  // 64-unit hidden block of the chunk
#pragma unroll
                for (int kk = 0; kk < L::KB / 16; ++kk) {
                  // Hidden units 16u .. 16u+15 of the chunk (u = 4hk + kk) were packed by GELU
                  // warp u / (FC/32) into columns (u % (FC/32)) * 8 .. +7 of its FC/2 columns.
                  const int u = hk * 4 + kk;
                  const uint32_t ta = th + (u / (FC / 32)) * (FC / 2) + (u % (FC / 32)) * 8;
                  const uint64_t db = umma_sdesc(sW + st * L::SLOT + q * L::W2_KBLK + kk * 32, 1024, kSw128);
                  umma_f16_ts(tacc2, ta, db, idesc2, (step > L::LAG || hk > 0 || kk > 0) ? 1u : 0u);
                }
              }
              umma_commit(&w_empty[st]);
            }
            if (!ok) break;
            if (step == nchunk + L::LAG - 1) umma_commit(&acc2_full[ib]);
          }
        }
        cg += nchunk;
      }
      umma_commit(done);
      wait_drain(done, 0, kDrainLimitNs);
    }
  } else if (warp < 8) {
    // ------------------------------------------------------------ GELU warps
    const int gq = warp & 3, gh = warp >> 2;
    constexpr int GW = FC / 2;  // accumulator columns (hidden units) per GELU warp and chunk
    const uint32_t tbase = tmem_base + (static_cast<uint32_t>(gq * 32) << 16) + L::TMEM_ACC1 + gh * GW;
    int cg = 0;
    bool ok = true;
    for (int w = blockIdx.x; ok && w < p.n_items; w += gridDim.x) {
      for (int cc = 0; cc < nchunk; ++cc) {
        const int c = cg + cc, ab = c % L::NACC1;
        if (!(ok = warp_wait_phase(&acc1_full[ab], (c / L::NACC1) & 1, wd, 0x621))) break;
        tc_fence_after();
        uint32_t v[GW / 32][32];
        const uint32_t tsrc = tbase + ab * FC;
#pragma unroll
        for (int h = 0; h < GW / 32; ++h) tmem_ld_x32(tsrc + 32 * h, v[h]);
#pragma unroll
        for (int h = 0; h < GW / 32; ++h) tmem_ld_wait_tied(v[h]);
        const float4* b4 = reinterpret_cast<const float4*>(p.b1 + cc * FC + gh * GW);
        uint32_t pk[GW / 2];
#pragma unroll
        for (int e = 0; e < GW / 4; ++e) {
          const float4 bb = __ldg(b4 + e);  // the same address in every lane: one broadcast load
          const uint32_t* x = &v[e >> 3][(e & 7) * 4];
          const uint64_t h01 = gelu_erf_pair(
              fadd2(f2_pack(__uint_as_float(x[0]), __uint_as_float(x[1])), f2_pack(bb.x, bb.y)));
          const uint64_t h23 = gelu_erf_pair(
              fadd2(f2_pack(__uint_as_float(x[2]), __uint_as_float(x[3])), f2_pack(bb.z, bb.w)));
          pk[2 * e] = pack_half2(f2_lo(h01), f2_hi(h01));
          pk[2 * e + 1] = pack_half2(f2_lo(h23), f2_hi(h23));
        }
        // H (GW hidden units = GW/2 packed columns) over the first half of this warp's columns.
        if constexpr (GW == 64) {
          tmem_st_x32(tsrc, pk);
        } else {
          tmem_st_x16(tsrc, pk);
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&h_full[ab]);
      }
      cg += nchunk;
    }
  } else if (warp < 12) {
    // ------------------------------------------------------------ residual + LayerNorm warps
    const int ew = warp - 8;
    const uint32_t lane_base = static_cast<uint32_t>(ew * 32) << 16;
    const uint32_t ring = smem_u32(smem + L::OFF_LN) + ew * L::RING * L::TILE;
    constexpr int JW = L::JW;      // columns per job
    constexpr int nch = D / JW;    // jobs per pass
    constexpr int RB = JW * 4;     // bytes per staged FP32 row (64)
    constexpr int PR = RB / 16;    // 16-byte pieces per row (4)
    // Staging tile layout: 32 rows x 64 bytes, 16-byte piece k of row r at
    // r * 64 + ((k ^ ((r >> 1) & 3)) << 4) (conflict-free by rows and by pieces).
    // Job j of a tile: j < nch reads the residual input columns [j*JW, +JW),
    // j >= nch reads back this warp's own r' columns of job j - nch.  Jobs run
    // in one sequence across tiles (number jg = 2 * nch * tile_count + j) and
    // job jg stages in slot jg % RING, AHEAD jobs ahead of the one consumed
    // (the residual rows were bulk-prefetched into L2 a tile earlier, so the
    // loads wait on L2 latency; AHEAD covers it).
    auto sw = [](int r, int k) { return r * RB + ((k ^ ((r >> 1) & 3)) << 4); };
    auto issue = [&](int tile, int j, int jg) {
      const int r0 = tile * 128 + ew * 32;
      const int c = j % nch;
      const float* src = (j < nch) ? p.resid_in : p.resid_out;
      const uint32_t slot = ring + (jg % L::RING) * L::TILE;
#pragma unroll
      for (int k = 0; k < 32 / (32 / PR); ++k) {
        const int r = k * (32 / PR) + lane / PR, piece = lane % PR;
        const int row = r0 + r;
        const bool v = row < p.M;
        const float* g = src + static_cast<size_t>(v ? row : 0) * D + c * JW + piece * 4;
        cp_async_16(slot + sw(r, piece), g, v ? 16u : 0u);
      }
    };
    // The staged tile as this thread's row (JW floats).
    auto read_row = [&](uint32_t slot, float* x) {
#pragma unroll
      for (int k = 0; k < PR; ++k) {
        const uint4 q = ld_shared_v4(slot + sw(lane, k));
        x[4 * k] = __uint_as_float(q.x);
        x[4 * k + 1] = __uint_as_float(q.y);
        x[4 * k + 2] = __uint_as_float(q.z);
        x[4 * k + 3] = __uint_as_float(q.w);
      }
    };
    auto write_row = [&](uint32_t slot, const float* x) {
#pragma unroll
      for (int k = 0; k < PR; ++k)
        st_shared_v4(slot + sw(lane, k), __float_as_uint(x[4 * k]), __float_as_uint(x[4 * k + 1]),
                     __float_as_uint(x[4 * k + 2]), __float_as_uint(x[4 * k + 3]));
    };
    // Coalesced copy-out of a staged FP32 tile (PR lanes per row).
    auto store_f32 = [&](uint32_t slot, float* dst, int r0, int c) {
#pragma unroll
      for (int k = 0; k < PR; ++k) {
        const int r = k * (32 / PR) + lane / PR, piece = lane % PR;
        const uint4 q = ld_shared_v4(slot + sw(r, piece));
        if (r0 + r < p.M)
          *reinterpret_cast<uint4*>(dst + static_cast<size_t>(r0 + r) * D + c * JW + piece * 4) = q;
      }
    };
    int i = 0;
    bool ok = true;
    int w = blockIdx.x;
    if (w < p.n_items) {
      for (int j = 0; j < L::AHEAD; ++j) {
        issue(w, j, j);  // 2 * nch >= AHEAD: these all belong to the first tile
        cp_async_commit();
      }
    }
    for (; ok && w < p.n_items; w += gridDim.x, ++i) {
      const int ib = i % L::NACC2;
      const uint32_t tacc2 = tmem_base + lane_base + ib * D;
      const int r0 = w * 128 + ew * 32;
      const int row = r0 + lane;
      const bool valid = row < p.M;
      const int wn = w + static_cast<int>(gridDim.x);
      const int jbase = i * 2 * nch;  // sequence number of this tile's job 0
      // Issue job j + 2 (the next tile's first jobs at the end), then wait for
      // job j; returns job j's staging slot.
      auto advance = [&](int j) -> uint32_t {
        const int jn = j + L::AHEAD;
        if (jn < 2 * nch)
          issue(w, jn, jbase + jn);
        else if (wn < p.n_items)
          issue(wn, jn - 2 * nch, jbase + jn);
        cp_async_commit();
        cp_async_wait<L::AHEAD>();
        __syncwarp();
        return ring + ((jbase + j) % L::RING) * L::TILE;
      };
      if (!(ok = warp_wait_phase(&acc2_full[ib], (i / L::NACC2) & 1, wd, 0x631))) break;
      tc_fence_after();
      // Pass 1: r' = acc2 + b2 + r; statistics; r' out.  acc2 comes into registers 64
      // columns at a time, and each block is released once loaded.
      float shift = 0.f, s1 = 0.f, s2 = 0.f;
      constexpr int JPB = 64 / JW;  // jobs per 64-column block
#pragma unroll 1
      for (int blk = 0; blk < L::NBLK; ++blk) {
        uint32_t v[2][32];
        tmem_ld_x32(tacc2 + blk * 64, v[0]);
        tmem_ld_x32(tacc2 + blk * 64 + 32, v[1]);
        tmem_ld_wait_tied(v[0]);
        tmem_ld_wait_tied(v[1]);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc2_empty[ib * L::NBLK + blk]);  // the next tile's G2 may take it
#pragma unroll
        for (int jj = 0; jj < JPB; ++jj) {
          const int c = blk * JPB + jj;
          const uint32_t slot = advance(c);
          float x[JW];
          read_row(slot, x);
          const float4* b2 = reinterpret_cast<const float4*>(s_b2 + c * JW);
#pragma unroll
          for (int k = 0; k < PR; ++k) {
            const float4 bb = b2[k];
            const uint32_t* vv = &v[(jj * JW) / 32][(jj * JW) % 32 + 4 * k];
            x[4 * k] += __uint_as_float(vv[0]) + bb.x;
            x[4 * k + 1] += __uint_as_float(vv[1]) + bb.y;
            x[4 * k + 2] += __uint_as_float(vv[2]) + bb.z;
            x[4 * k + 3] += __uint_as_float(vv[3]) + bb.w;
          }
          if (c == 0) shift = x[0];
#pragma unroll
          for (int e = 0; e < JW; ++e) {
            const float d = x[e] - shift;
            s1 += d;
            s2 = fmaf(d, d, s2);
          }
          __syncwarp();
          write_row(slot, x);
          __syncwarp();
          store_f32(slot, p.resid_out, r0, c);
          __syncwarp();
        }
      }
      const float inv_d = 1.f / static_cast<float>(D);
      const float m1 = s1 * inv_d;
      const float var = fmaxf(s2 * inv_d - m1 * m1, 0.f);
      const float mean = shift + m1;
      const float rstd = rsqrtf(var + p.eps);
      const bool zero_row = valid && p.row_mask != nullptr && p.row_mask[row] == 0;
      // Pass 2: normalized rows from this warp's own r' (written above, L2-resident).
#pragma unroll 1
      for (int c = 0; c < nch; ++c) {
        const uint32_t slot = advance(nch + c);
        float x[JW];
        read_row(slot, x);
        const float4* g4 = reinterpret_cast<const float4*>(s_gamma + c * JW);
        const float4* b4 = reinterpret_cast<const float4*>(s_beta + c * JW);
#pragma unroll
        for (int k = 0; k < PR; ++k) {
          const float4 gg = g4[k], bb = b4[k];
          x[4 * k] = zero_row ? 0.f : fmaf((x[4 * k] - mean) * rstd, gg.x, bb.x);
          x[4 * k + 1] = zero_row ? 0.f : fmaf((x[4 * k + 1] - mean) * rstd, gg.y, bb.y);
          x[4 * k + 2] = zero_row ? 0.f : fmaf((x[4 * k + 2] - mean) * rstd, gg.z, bb.z);
          x[4 * k + 3] = zero_row ? 0.f : fmaf((x[4 * k + 3] - mean) * rstd, gg.w, bb.w);
        }
        __syncwarp();
        if (p.norm_f16) {
          // 32 rows x 32 bytes: piece k (8 halves) of row r at r * 32 + ((k ^ ((r >> 2) & 1)) << 4).
#pragma unroll
          for (int k = 0; k < JW / 8; ++k)
            st_shared_v4(slot + lane * 32 + ((k ^ ((lane >> 2) & 1)) << 4), pack_half2(x[8 * k], x[8 * k + 1]),
                         pack_half2(x[8 * k + 2], x[8 * k + 3]), pack_half2(x[8 * k + 4], x[8 * k + 5]),
                         pack_half2(x[8 * k + 6], x[8 * k + 7]));
          __syncwarp();
          __half* dst = static_cast<__half*>(p.norm_out);
#pragma unroll
          for (int k = 0; k < JW / 8; ++k) {
            const int r = k * 16 + (lane >> 1), piece = lane & 1;
            const uint4 q = ld_shared_v4(slot + r * 32 + ((piece ^ ((r >> 2) & 1)) << 4));
            if (r0 + r < p.M)
              *reinterpret_cast<uint4*>(dst + static_cast<size_t>(r0 + r) * D + c * JW + piece * 8) = q;
          }
        } else {
          write_row(slot, x);
          __syncwarp();
          store_f32(slot, static_cast<float*>(p.norm_out), r0, c);
        }
        __syncwarp();
      }
    }
    cp_async_wait<0>();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kFfn2Mma) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace tt
