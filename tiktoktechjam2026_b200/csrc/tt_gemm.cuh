// Row-block projection GEMMs for sm_100a with fused epilogues.
//
//   out[M, N] = A[M, K] (FP16) . W[N, K]^T (FP16) + bias, FP32 accumulation
//
// replacing the reference's Triton projection kernels
// (mixed_precision/triton_linear.py:16-69 `_mixed_linear_kernel`, :72-125
// `_mixed_linear_add_layer_norm_kernel`) and the cuBLAS nn.Linear route of the
// generic configurations (mixed_precision/transformer.py:138-139, 669-677).
//
// One CTA owns 128 rows and `bn` output columns (bn <= 256, or 512 as two
// 256-column UMMAs).  Roles: warp 4 streams (A, W) K-blocks with TMA through
// an `nst`-deep ring, warp 5 allocates TMEM and issues tcgen05.mma, warps 0..3
// drain the FP32 accumulator (one row per thread) through an epilogue:
//   EPI_QKV       + bias, FP16, scattered to Q/K [B,H,S,hd] and V^T [B,H,hd,S_pad]
//   EPI_RESID_LN  + bias + FP32 residual -> residual out (FP32), then the
//                 two-pass FP32 LayerNorm of the row -> FP16 or FP32
//                 (optionally zeroing rows whose mask byte is 0)
//   EPI_GELU      + bias, exact-erf GELU in FP32, FP16 out
#pragma once

#include "tt_ptx.cuh"

namespace tt {

enum GemmEpilogue : int { EPI_QKV = 0, EPI_RESID_LN = 1, EPI_GELU = 2 };

struct GemmParams {
  int M, N_total, K;
  int bn;        // output columns per CTA
  int n_splits;  // N_total / bn
  int nst;       // pipeline depth
  const float* bias;  // [N_total]
  // EPI_QKV
  __half* q;
  __half* k;
  __half* vt;
  int seq, heads, head_dim, seq_pad, d_model;
  // EPI_RESID_LN
  const float* resid_in;
  float* resid_out;
  const float* gamma;
  const float* beta;
  void* norm_out;
  int norm_f16;
  float eps;
  const uint8_t* row_mask;
  // EPI_GELU
  __half* act_out;
  unsigned int* err;
  unsigned long long timeout_ns;
};

constexpr int kGemmMaxStages = 8;

__host__ __device__ inline int gemm_stage_bytes(int ksw, int bn) { return (128 + bn) * ksw * 2; }
__host__ __device__ inline int gemm_tmem_cols(int bn) {
  int c = 32;
  while (c < bn) c <<= 1;
  return c;
}
// Offsets: stages (1024-aligned) | bias[bn] | gamma[bn] | beta[bn] | barriers | misc
__host__ __device__ inline int gemm_smem_bytes(int ksw, int bn, int nst) {
  int off = nst * gemm_stage_bytes(ksw, bn);
  off += 3 * bn * 4;
  off += (2 * kGemmMaxStages + 2) * 8;
  off += 16;
  return off + 1024;
}

template <int KSW, int EPI>
__global__ void __launch_bounds__(192, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                const GemmParams p) {
  constexpr int A_BYTES = 128 * KSW * 2;
  constexpr uint32_t kSw = swizzle_kind_for_bytes(KSW * 2);
  constexpr uint32_t kSbo = 8 * KSW * 2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int bn = p.bn, nst = p.nst;
  const int stage_bytes = gemm_stage_bytes(KSW, bn);
  const int w_bytes_half = (bn > 256 ? 256 : bn) * KSW * 2;
  float* s_bias = reinterpret_cast<float*>(smem + nst * stage_bytes);
  float* s_gamma = s_bias + bn;
  float* s_beta = s_gamma + bn;
  uint64_t* full = reinterpret_cast<uint64_t*>(s_beta + bn);
  uint64_t* empty = full + kGemmMaxStages;
  uint64_t* acc_full = empty + kGemmMaxStages;
  uint64_t* done = acc_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_tile = blockIdx.x / p.n_splits;
  const int split = blockIdx.x - m_tile * p.n_splits;
  const int m0 = m_tile * 128;
  const int n0 = split * bn;
  const int nk = p.K / KSW;
  const uint32_t tmem_cols = static_cast<uint32_t>(gemm_tmem_cols(bn));

  if (threadIdx.x == 0) {
    for (int i = 0; i < nst; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (threadIdx.x < 128) {
    for (int c = threadIdx.x; c < bn; c += 128) {
      s_bias[c] = p.bias[n0 + c];
      if constexpr (EPI == EPI_RESID_LN) {
        s_gamma[c] = p.gamma[n0 + c];
        s_beta[c] = p.beta[n0 + c];
      }
    }
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const Watchdog wd{p.err, abort_flag, p.timeout_ns};

  if (warp == 4) {
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmW);
      int issued = 0;
      for (int kb = 0; kb < nk; ++kb) {
        const int st = kb % nst;
        if (!wait_phase(&empty[st], ((kb / nst) & 1) ^ 1, wd, 0x401)) break;
        uint8_t* sa = smem + st * stage_bytes;
        uint8_t* sw = sa + A_BYTES;
        mbar_arrive_expect_tx(&full[st], stage_bytes);
        tma_load_2d(sa, &tmA, &full[st], kb * KSW, m0);
        tma_load_2d(sw, &tmW, &full[st], kb * KSW, n0);
        if (bn > 256) tma_load_2d(sw + w_bytes_half, &tmW, &full[st], kb * KSW, n0 + 256);
        issued = kb + 1;
      }
      for (int kb = (issued > nst ? issued - nst : 0); kb < issued; ++kb)
        wait_drain(&full[kb % nst], (kb / nst) & 1, kDrainLimitNs);
    }
  } else if (warp == 5) {
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_f16_f32(128, bn > 256 ? 256 : bn);
      const uint32_t base = smem_u32(smem);
      bool ok = true;
      for (int kb = 0; kb < nk; ++kb) {
        const int st = kb % nst;
        if (!(ok = wait_phase(&full[st], (kb / nst) & 1, wd, 0x402))) break;
        tc_fence_after();
        const uint32_t sa = base + st * stage_bytes;
        const uint32_t sw = sa + A_BYTES;
#pragma unroll
        for (int kk = 0; kk < KSW / 16; ++kk) {
          const uint64_t da = umma_sdesc(sa + kk * 32, kSbo, kSw);
          const uint32_t acc = (kb > 0 || kk > 0) ? 1u : 0u;
          umma_f16(tmem_base, da, umma_sdesc(sw + kk * 32, kSbo, kSw), idesc, acc);
          if (bn > 256)
            umma_f16(tmem_base + 256, da, umma_sdesc(sw + w_bytes_half + kk * 32, kSbo, kSw), idesc,
                     acc);
        }
        umma_commit(&empty[st]);
      }
      if (ok) umma_commit(acc_full);
      umma_commit(done);
      wait_drain(done, 0, kDrainLimitNs);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int r = threadIdx.x;
    const int row = m0 + r;
    const bool valid = row < p.M;
    const uint32_t taddr = tmem_base + (static_cast<uint32_t>(warp * 32) << 16);
    if (warp_wait_phase(acc_full, 0, wd, 0x403)) {
      tc_fence_after();
      if constexpr (EPI == EPI_QKV) {
        const int D = p.d_model, hd = p.head_dim;
        const int bidx = valid ? row / p.seq : 0;
        const int s = valid ? row - bidx * p.seq : 0;
        for (int c = 0; c < bn; c += 32) {
          uint32_t v[32];
          __syncwarp();
          tmem_ld_x32(taddr + c, v);
          tmem_ld_wait();
          if (!valid) continue;
          const int col0 = n0 + c;
          const int which = col0 / D;
          const int within0 = col0 - which * D;
          float f[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) f[i] = __uint_as_float(v[i]) + s_bias[c + i];
          if (which < 2) {
            __half* base = which == 0 ? p.q : p.k;
#pragma unroll
            for (int g = 0; g < 2; ++g) {
              const int within = within0 + 16 * g;
              const int hh = within / hd, d = within - hh * hd;
              uint4* dst = reinterpret_cast<uint4*>(
                  base + ((static_cast<size_t>(bidx) * p.heads + hh) * p.seq + s) * hd + d);
              uint4 a, bq;
              a.x = pack_half2(f[16 * g + 0], f[16 * g + 1]);
              a.y = pack_half2(f[16 * g + 2], f[16 * g + 3]);
              a.z = pack_half2(f[16 * g + 4], f[16 * g + 5]);
              a.w = pack_half2(f[16 * g + 6], f[16 * g + 7]);
              bq.x = pack_half2(f[16 * g + 8], f[16 * g + 9]);
              bq.y = pack_half2(f[16 * g + 10], f[16 * g + 11]);
              bq.z = pack_half2(f[16 * g + 12], f[16 * g + 13]);
              bq.w = pack_half2(f[16 * g + 14], f[16 * g + 15]);
              dst[0] = a;
              dst[1] = bq;
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int within = within0 + i;
              const int hh = within / hd, d = within - hh * hd;
              p.vt[((static_cast<size_t>(bidx) * p.heads + hh) * hd + d) * p.seq_pad + s] =
                  __float2half_rn(f[i]);
            }
          }
        }
      } else if constexpr (EPI == EPI_GELU) {
        for (int c = 0; c < bn; c += 32) {
          uint32_t v[32];
          __syncwarp();
          tmem_ld_x32(taddr + c, v);
          tmem_ld_wait();
          if (!valid) continue;
          uint4* dst = reinterpret_cast<uint4*>(p.act_out + static_cast<size_t>(row) * p.N_total +
                                                n0 + c);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            uint4 w;
            float g[8];
#pragma unroll
            for (int e = 0; e < 8; ++e)
              g[e] = gelu_erf(__uint_as_float(v[8 * i + e]) + s_bias[c + 8 * i + e]);
            w.x = pack_half2(g[0], g[1]);
            w.y = pack_half2(g[2], g[3]);
            w.z = pack_half2(g[4], g[5]);
            w.w = pack_half2(g[6], g[7]);
            dst[i] = w;
          }
        }
      } else {
        // EPI_RESID_LN: bn == N_total == d_model (the whole row lives in TMEM).
        const int D = bn;
        const float* rin = p.resid_in + static_cast<size_t>(valid ? row : 0) * D;
        float* rout = p.resid_out + static_cast<size_t>(valid ? row : 0) * D;
        float sum = 0.f;
        for (int c = 0; c < D; c += 32) {
          uint32_t v[32];
          __syncwarp();
          tmem_ld_x32(taddr + c, v);
          tmem_ld_wait();
          float4 res[8];
#pragma unroll
          for (int i = 0; i < 8; ++i)
            res[i] = valid ? reinterpret_cast<const float4*>(rin + c)[i] : make_float4(0, 0, 0, 0);
          uint32_t out[32];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            float4 t;
            t.x = __uint_as_float(v[4 * i + 0]) + s_bias[c + 4 * i + 0] + res[i].x;
            t.y = __uint_as_float(v[4 * i + 1]) + s_bias[c + 4 * i + 1] + res[i].y;
            t.z = __uint_as_float(v[4 * i + 2]) + s_bias[c + 4 * i + 2] + res[i].z;
            t.w = __uint_as_float(v[4 * i + 3]) + s_bias[c + 4 * i + 3] + res[i].w;
            sum += (t.x + t.y) + (t.z + t.w);
            if (valid) reinterpret_cast<float4*>(rout + c)[i] = t;
            out[4 * i + 0] = __float_as_uint(t.x);
            out[4 * i + 1] = __float_as_uint(t.y);
            out[4 * i + 2] = __float_as_uint(t.z);
            out[4 * i + 3] = __float_as_uint(t.w);
          }
          __syncwarp();
          tmem_st_x32(taddr + c, out);
        }
        tmem_st_wait();
        const float mean = sum / static_cast<float>(D);
        float sq = 0.f;
        for (int c = 0; c < D; c += 32) {
          uint32_t v[32];
          __syncwarp();
          tmem_ld_x32(taddr + c, v);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float d = __uint_as_float(v[i]) - mean;
            sq = fmaf(d, d, sq);
          }
        }
        const float rstd = rsqrtf(sq / static_cast<float>(D) + p.eps);
        const bool zero_row = valid && p.row_mask != nullptr && p.row_mask[row] == 0;
        for (int c = 0; c < D; c += 32) {
          uint32_t v[32];
          __syncwarp();
          tmem_ld_x32(taddr + c, v);
          tmem_ld_wait();
          if (!valid) continue;
          float y[32];
#pragma unroll
          for (int i = 0; i < 32; ++i)
            y[i] = zero_row ? 0.f
                            : fmaf((__uint_as_float(v[i]) - mean) * rstd, s_gamma[c + i], s_beta[c + i]);
          if (p.norm_f16) {
            uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__half*>(p.norm_out) +
                                                  static_cast<size_t>(row) * D + c);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              uint4 w;
              w.x = pack_half2(y[8 * i + 0], y[8 * i + 1]);
              w.y = pack_half2(y[8 * i + 2], y[8 * i + 3]);
              w.z = pack_half2(y[8 * i + 4], y[8 * i + 5]);
              w.w = pack_half2(y[8 * i + 6], y[8 * i + 7]);
              dst[i] = w;
            }
          } else {
            float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.norm_out) +
                                                    static_cast<size_t>(row) * D + c);
#pragma unroll
            for (int i = 0; i < 8; ++i)
              dst[i] = make_float4(y[4 * i + 0], y[4 * i + 1], y[4 * i + 2], y[4 * i + 3]);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem_base, tmem_cols);
  }
}

}  // namespace tt
