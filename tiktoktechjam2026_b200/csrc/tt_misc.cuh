// Memory-bound helper kernels: the layer-0 input LayerNorm, the per-sequence
// key-padding summary used by attention tile skipping, and the watchdog
// self-test.
#pragma once

#include "tt_ptx.cuh"

namespace tt {

// LayerNorm of FP32 rows (one warp per row, two-pass mean/variance in FP32),
// output FP16 or FP32; rows whose row_mask byte is 0 (row_mask may be null)
// are written as zeros.  Replaces `layers[0].norm1(x)` + the FP16 cast of the
// reference (mixed_precision/transformer.py:489-491), and for d_model above
// 512 the LayerNorm half of the residual + LayerNorm steps
// (mixed_precision/transformer.py:223-227, 675-695).  Requires d % 32 == 0.
template <int VPL>  // values per lane = d / 32
__global__ void __launch_bounds__(256)
    layernorm_rows_kernel(const float* __restrict__ x, const float* __restrict__ gamma,
                          const float* __restrict__ beta, void* __restrict__ out, long long n_rows,
                          float eps, int out_f16, const uint8_t* __restrict__ row_mask) {
  pdl_wait();
  pdl_trigger();
  constexpr int D = VPL * 32;
  const long long row = static_cast<long long>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= n_rows) return;
  const float* xr = x + row * D;
  float v[VPL];
  if constexpr (VPL % 4 == 0) {
#pragma unroll
    for (int i = 0; i < VPL / 4; ++i) {
      const float4 t = reinterpret_cast<const float4*>(xr)[lane + 32 * i];
      v[4 * i + 0] = t.x;
      v[4 * i + 1] = t.y;
      v[4 * i + 2] = t.z;
      v[4 * i + 3] = t.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < VPL; ++i) v[i] = xr[lane + 32 * i];
  }
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) s += v[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float mean = s / static_cast<float>(D);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const float d = v[i] - mean;
    q = fmaf(d, d, q);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
  const float rstd = rsqrtf(q / static_cast<float>(D) + eps);
  const bool zero = row_mask != nullptr && row_mask[row] == 0;
  if constexpr (VPL % 4 == 0) {
#pragma unroll
    for (int i = 0; i < VPL / 4; ++i) {
      const int c = 4 * (lane + 32 * i);
      const float4 g = reinterpret_cast<const float4*>(gamma)[lane + 32 * i];
      const float4 bb = reinterpret_cast<const float4*>(beta)[lane + 32 * i];
      const float y0 = zero ? 0.f : fmaf((v[4 * i + 0] - mean) * rstd, g.x, bb.x);
      const float y1 = zero ? 0.f : fmaf((v[4 * i + 1] - mean) * rstd, g.y, bb.y);
      const float y2 = zero ? 0.f : fmaf((v[4 * i + 2] - mean) * rstd, g.z, bb.z);
      const float y3 = zero ? 0.f : fmaf((v[4 * i + 3] - mean) * rstd, g.w, bb.w);
      if (out_f16) {
        uint2 w;
        w.x = pack_half2(y0, y1);
        w.y = pack_half2(y2, y3);
        *reinterpret_cast<uint2*>(reinterpret_cast<__half*>(out) + row * D + c) = w;
      } else {
        *reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + row * D + c) =
            make_float4(y0, y1, y2, y3);
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int c = lane + 32 * i;
      const float y = zero ? 0.f : fmaf((v[i] - mean) * rstd, gamma[c], beta[c]);
      if (out_f16)
        reinterpret_cast<__half*>(out)[row * D + c] = __float2half_rn(y);
      else
        reinterpret_cast<float*>(out)[row * D + c] = y;
    }
  }
}

// kv_end[b] = 1 + index of the last nonzero mask byte of sequence b (0 if none).
__global__ void __launch_bounds__(256)
    mask_kv_end_kernel(const uint8_t* __restrict__ mask, int seq, int* __restrict__ kv_end) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x;
  int last = -1;
  for (int s = threadIdx.x; s < seq; s += blockDim.x)
    if (mask[static_cast<size_t>(b) * seq + s] != 0) last = s;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) last = max(last, __shfl_xor_sync(0xffffffffu, last, o));
  __shared__ int wmax[8];
  if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = last;
  __syncthreads();
  if (threadIdx.x == 0) {
    int m = -1;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) m = max(m, wmax[w]);
    kv_end[b] = m + 1;
  }
}

// Watchdog self-test: waits on an mbarrier that nothing ever arrives on.  The
// bounded wait gives up after `timeout_ns`, records a timeout in the error word
// and the kernel returns normally, leaving the context usable.
__global__ void watchdog_selftest_kernel(unsigned int* err, unsigned long long timeout_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const Watchdog wd{err, &abort_flag, timeout_ns};
    wait_phase(&bar, 0, wd, 0x7e57);
  }
  __syncthreads();
}

// The FMA-pipe exponential of the attention softmax on pairs of inputs:
// y32 = exp2_pair_fma (FP32), y16 = exp2_pair_fma_f16 (FP16 bits).  Test probe.
__global__ void exp2_fma_probe_kernel(const float* x, float* y32, uint32_t* y16, int n_pairs) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_pairs) return;
  const uint64_t xx = f2_pack(x[2 * i], x[2 * i + 1]);
  const uint64_t y = exp2_pair_fma(xx);
  y32[2 * i] = f2_lo(y);
  y32[2 * i + 1] = f2_hi(y);
  y16[i] = exp2_pair_fma_f16(xx);
}

}  // namespace tt
