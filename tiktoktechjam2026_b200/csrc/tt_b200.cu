// libtt_b200.so: host side of the C ABI declared in include/tt_b200.h.
//
// Holds the tensor-map encoding (driver entry point fetched at run time, so
// the library does not link libcuda), the shape-dispatch table, the
// whole-model forward launcher and its optional per-launch event profiling.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <utility>
#include <vector>

#include "tt_attention.cuh"
#include "tt_attn_db.cuh"
#include "tt_ffn.cuh"
#include "tt_ffn2.cuh"
#include "tt_gemm.cuh"
#include "tt_misc.cuh"
#include "../../include/tt_b200.h"

namespace tt {

__device__ unsigned int g_err_word;

namespace {

constexpr int kAbiVersion = 2;
constexpr int kMaxDevices = 64;
constexpr int kSmemBudget = 225 * 1024;

// Features per head as Q, K and V^T are stored: head_dim 8 is kept 16 wide
// (features 8..15 of Q and K zero) so that the head_dim-16 attention kernel,
// whose MMAs need K = 16, runs on it unchanged.
inline int stored_head_dim(int hd) { return hd < 16 ? 16 : hd; }
inline bool attention_head_dim_ok(int hd) {
  return hd == 8 || hd == 16 || hd == 32 || hd == 64 || hd == 128 || hd == 256;
}

thread_local char g_last_error[512] = "";
std::atomic<unsigned long long> g_launches{0};
std::atomic<unsigned long long> g_timeout_ns{2000000000ull};

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return TT_OK;
  return fail(TT_ERR_LAUNCH, "%s: %s", what, cudaGetErrorString(e));
}

// ---------------------------------------------------------------- per device
struct DeviceState {
  std::once_flag once;
  int status = TT_OK;
  unsigned int* err = nullptr;  // device address of g_err_word
  int sm_count = 0;
};
DeviceState g_dev[kMaxDevices];

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

int current_device_state(DeviceState** out) {
  int dev = 0;
  if (int rc = check_cuda(cudaGetDevice(&dev), "cudaGetDevice")) return rc;
  if (dev < 0 || dev >= kMaxDevices) return fail(TT_ERR_ARG, "device ordinal %d out of range", dev);
  DeviceState& st = g_dev[dev];
  std::call_once(st.once, [&] {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_err_word);
    if (e != cudaSuccess) {
      st.status = fail(TT_ERR_LAUNCH, "cudaGetSymbolAddress(error word): %s", cudaGetErrorString(e));
      return;
    }
    st.err = static_cast<unsigned int*>(p);
    e = cudaDeviceGetAttribute(&st.sm_count, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) {
      st.status = fail(TT_ERR_LAUNCH, "cudaDeviceGetAttribute: %s", cudaGetErrorString(e));
      return;
    }
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (major != 10 || minor != 0) {
      st.status = fail(TT_ERR_UNSUPPORTED,
                       "libtt_b200 is built for sm_100a (B200); device %d is sm_%d%d", dev, major,
                       minor);
      return;
    }
    st.status = TT_OK;
  });
  if (st.status != TT_OK) return st.status;
  *out = &st;
  return TT_OK;
}

int get_encoder() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!g_encode) return fail(TT_ERR_LAUNCH, "cuTensorMapEncodeTiled entry point not available");
  return TT_OK;
}

CUtensorMapSwizzle swizzle_for_bytes(int inner_bytes) {
  return inner_bytes == 128   ? CU_TENSOR_MAP_SWIZZLE_128B
         : inner_bytes == 64  ? CU_TENSOR_MAP_SWIZZLE_64B
         : inner_bytes == 32  ? CU_TENSOR_MAP_SWIZZLE_32B
                              : CU_TENSOR_MAP_SWIZZLE_NONE;
}

// Tensor map of rank 2 or 3 (dims innermost first, byte strides of dims 1..);
// the swizzle follows the box's inner extent in bytes (32, 64 or 128).
int encode_tensor(CUtensorMap* tm, CUtensorMapDataType dtype, int elem_bytes, const void* base,
                  int rank, const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box) {
  if (int rc = get_encoder()) return rc;
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0)
    return fail(TT_ERR_ALIGN, "tensor base %p is not 16-byte aligned", base);
  for (int i = 0; i < rank - 1; ++i)
    if (strides_bytes[i] % 16 != 0)
      return fail(TT_ERR_ALIGN, "tensor stride %llu is not a multiple of 16 bytes",
                  static_cast<unsigned long long>(strides_bytes[i]));
  cuuint32_t elem_strides[3] = {1, 1, 1};
  const CUresult r = g_encode(
      tm, dtype, static_cast<cuuint32_t>(rank), const_cast<void*>(base),
      reinterpret_cast<const cuuint64_t*>(dims), reinterpret_cast<const cuuint64_t*>(strides_bytes),
      reinterpret_cast<const cuuint32_t*>(box), elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE,
      swizzle_for_bytes(static_cast<int>(box[0]) * elem_bytes), CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(TT_ERR_LAUNCH, "cuTensorMapEncodeTiled failed (%d)", int(r));
  return TT_OK;
}

int encode_f16(CUtensorMap* tm, const void* base, int rank, const uint64_t* dims,
               const uint64_t* strides_bytes, const uint32_t* box) {
  return encode_tensor(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, base, rank, dims, strides_bytes, box);
}

// Row-major [rows, cols] FP16 matrix, box {box_cols, box_rows}.
int encode_matrix(CUtensorMap* tm, const void* base, uint64_t rows, uint64_t cols, int box_cols,
                  int box_rows) {
  const uint64_t dims[2] = {cols, rows};
  const uint64_t strides[1] = {cols * 2};
  const uint32_t box[2] = {static_cast<uint32_t>(box_cols), static_cast<uint32_t>(box_rows)};
  return encode_f16(tm, base, 2, dims, strides, box);
}

// Row-major [rows, cols] matrix of FP32 or FP16 in [32 x 32] epilogue tiles.
int encode_epi_tile(CUtensorMap* tm, const void* base, uint64_t rows, uint64_t cols, bool f32) {
  const int eb = f32 ? 4 : 2;
  const uint64_t dims[2] = {cols, rows};
  const uint64_t strides[1] = {cols * eb};
  const uint32_t box[2] = {32, 32};
  return encode_tensor(tm, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, eb,
                       base, 2, dims, strides, box);
}

// Store maps of the QKV epilogue's TMA path (seq % 32 == 0, head_dim >= 32):
// Q and K as [B*H*S, hd], V^T as [B*H*hd, seq_pad], FP16, 32 x 32 boxes.
int encode_qkv_store_maps(GemmMaps* maps, const void* q, const void* k, const void* vt, int batch, int seq,
                          int heads, int hd, int seq_pad) {
  const uint64_t rows = static_cast<uint64_t>(batch) * heads * seq;
  if (int rc = encode_epi_tile(&maps->out0, q, rows, hd, false)) return rc;
  if (int rc = encode_epi_tile(&maps->out1, k, rows, hd, false)) return rc;
  return encode_epi_tile(&maps->res, vt, static_cast<uint64_t>(batch) * heads * hd, seq_pad, false);
}

// Per (kernel, device): the dynamic shared memory the kernel was opened up to
// and its register count.  Each is queried or set once, so a launch is only a
// launch (nothing else happens on the driver while a stream is captured).
struct KernelInfo {
  const void* fn;
  int dev, smem, regs;
};
std::mutex g_kinfo_mu;
std::vector<KernelInfo> g_kinfo;

int kernel_info(const void* fn, int smem_bytes, KernelInfo* out) {
  int dev = 0;
  if (int rc = check_cuda(cudaGetDevice(&dev), "cudaGetDevice")) return rc;
  std::lock_guard<std::mutex> lock(g_kinfo_mu);
  for (KernelInfo& k : g_kinfo) {
    if (k.fn == fn && k.dev == dev) {
      if (k.smem < smem_bytes) {
        if (int rc = check_cuda(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes),
                                "cudaFuncSetAttribute"))
          return rc;
        k.smem = smem_bytes;
      }
      *out = k;
      return TT_OK;
    }
  }
  if (int rc = check_cuda(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes),
                          "cudaFuncSetAttribute"))
    return rc;
  cudaFuncAttributes fa;
  if (int rc = check_cuda(cudaFuncGetAttributes(&fa, fn), "cudaFuncGetAttributes")) return rc;
  g_kinfo.push_back({fn, dev, smem_bytes, fa.numRegs});
  *out = g_kinfo.back();
  return TT_OK;
}

template <typename K>
int prepare_kernel(K kernel, int smem_bytes) {
  KernelInfo ki;
  return kernel_info(reinterpret_cast<const void*>(kernel), smem_bytes, &ki);
}

// Kernels of a whole-model forward are launched with programmatic stream
// serialization (each starts its set-up while its predecessor drains; see
// pdl_wait in tt_ptx.cuh).  Single-op entry points launch plainly: their
// callers may have written the weights they stage with the kernel just before.
thread_local bool t_pdl = false;

struct PdlScope {
  bool prev;
  PdlScope() : prev(t_pdl) { t_pdl = true; }
  ~PdlScope() { t_pdl = prev; }
};

template <typename... KArgs, typename... Args>
void launch_kernel(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                   Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = t_pdl ? 1 : 0;
  cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);  // errors surface in after_launch
}

int after_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(TT_ERR_LAUNCH, "%s launch: %s", what, cudaGetErrorString(e));
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return TT_OK;
}

// ---------------------------------------------------------------- dispatch
// Shape-dispatch table keyed on (d_model, heads, seq, ffn): tile widths and
// pipeline depths for every kernel of one layer.  Shapes not listed use the
// generic rule in choose_route().
struct Route {
  const char* name;
  int qkv_bn, qkv_nst;
  int out_nst;
  int ffn_in_bn, ffn_in_nst;
  int ffn_out_nst;
  int ffn_fused;   // 1: one fused FFN kernel (d_model in {32, 64, 128, 256}); 0: split route
};

struct RouteEntry {
  int d_model, heads, seq, ffn;
  Route route;
};

const RouteEntry kRouteTable[] = {
    // C1  B64 S128  D128 H4 F128
    {128, 4, 128, 128, {"d128-h4-s128", 128, 2, 2, 128, 2, 2, 1}},
    // C2  B64 S1024 D128 H4 F128
    {128, 4, 1024, 128, {"d128-h4-s1024", 128, 2, 2, 128, 2, 2, 1}},
    // C3  B256 S256 D32 H2 F128
    {32, 2, 256, 128, {"d32-h2-s256", 96, 1, 1, 128, 1, 4, 1}},
    // C4  B16 S2048 D512 H8 F2048 (+ key padding)
    {512, 8, 2048, 2048, {"d512-h8-s2048", 256, 4, 3, 256, 4, 3, 0}},
    // C5  B512 S1024 D256 H8 F1024
    {256, 8, 1024, 1024, {"d256-h8-s1024", 256, 3, 2, 256, 2, 3, 1}},
};

int largest_bn_dividing(int n, int cap) {
  for (int bn = cap; bn >= 32; bn -= 32)
    if (n % bn == 0) return bn;
  return 0;
}

int clamp_nst(int ksw, int bn, int k, int want, int epi, int n_total) {
  const int nk = k / ksw;
  int nst = want < nk ? want : nk;
  if (nst > kGemmMaxStages) nst = kGemmMaxStages;
  while (nst > 1 && gemm_smem_bytes(ksw, bn, nst, epi, n_total) > kSmemBudget) --nst;
  return nst < 1 ? 1 : nst;
}

// K-block width of a GEMM: 64 FP16 (128-byte swizzle) unless K is not a
// multiple of 64 or the 512-column residual tile needs the smaller stage.
int gemm_ksw(int k, int bn) { return (k % 64 == 0 && bn <= 256) ? 64 : 32; }

// Rows wider than TMEM's 512 accumulator columns: the residual GEMMs run in
// 256-column splits without their LayerNorm, which a row kernel applies after.
bool wide_model(int d_model) { return d_model == 768 || d_model == 1024; }
constexpr int kWideBn = 256;

bool ffn_fusable(int d_model, int ffn) {
  return (d_model == 32 || d_model == 64 || d_model == 128 || d_model == 256) && ffn % 128 == 0;
}

int check_model_shape(int d_model, int heads, int ffn) {
  if (d_model <= 0 || heads <= 0 || ffn <= 0 || d_model % heads != 0)
    return fail(TT_ERR_SHAPE, "invalid (d_model=%d, heads=%d, ffn=%d)", d_model, heads, ffn);
  const int hd = d_model / heads;
  if (!attention_head_dim_ok(hd))
    return fail(TT_ERR_UNSUPPORTED, "head_dim %d not in {8, 16, 32, 64, 128, 256}", hd);
  if (d_model % 32 != 0 || (d_model > 256 && d_model != 512 && !wide_model(d_model)))
    return fail(TT_ERR_UNSUPPORTED, "d_model %d must be a multiple of 32 up to 256, 512, 768 or 1024", d_model);
  if (ffn % 32 != 0) return fail(TT_ERR_UNSUPPORTED, "ffn %d must be a multiple of 32", ffn);
  return TT_OK;
}

int choose_route(int d_model, int heads, int seq, int ffn, Route* out) {
  if (int rc = check_model_shape(d_model, heads, ffn)) return rc;
  for (const RouteEntry& e : kRouteTable) {
    if (e.d_model == d_model && e.heads == heads && e.seq == seq && e.ffn == ffn) {
      *out = e.route;
      return TT_OK;
    }
  }
  Route r;
  r.name = "generic";
  r.qkv_bn = largest_bn_dividing(3 * d_model, 256);
  r.qkv_nst = 4;
  r.out_nst = 4;
  r.ffn_in_bn = largest_bn_dividing(ffn, 256);
  r.ffn_in_nst = 4;
  r.ffn_out_nst = 4;
  r.ffn_fused = ffn_fusable(d_model, ffn) ? 1 : 0;
  if (r.qkv_bn == 0 || r.ffn_in_bn == 0)
    return fail(TT_ERR_UNSUPPORTED, "no column split for d_model=%d ffn=%d", d_model, ffn);
  *out = r;
  return TT_OK;
}


// ---------------------------------------------------------------- launchers
template <int KSW, int EPI>
int launch_gemm_t(const GemmMaps& maps, GemmParams p, int sm_count, cudaStream_t stream) {
  const int smem = gemm_smem_bytes(KSW, p.bn, p.nst, EPI, p.N_total);
  if (smem > 232448) return fail(TT_ERR_UNSUPPORTED, "GEMM tile needs %d bytes of shared memory", smem);
  // The kernel instance whose residual ring matches the one gemm_smem_bytes sized.
  void (*kern)(const GemmMaps, const GemmParams) = gemm_kernel<KSW, EPI, gemm_res_ring(EPI, 0)>;
  if constexpr (EPI == EPI_RESID_LN)
    if (gemm_res_ring(EPI, p.bn) == 1) kern = gemm_kernel<KSW, EPI, 1>;
  if (int rc = prepare_kernel(kern, smem)) return rc;
  const long long m_tiles = (static_cast<long long>(p.M) + 127) / 128;
  const long long items = m_tiles * p.n_splits;
  if (items > 0x7fffffffLL) return fail(TT_ERR_SHAPE, "too many tiles");
  p.n_items = static_cast<int>(items);
  const unsigned grid = static_cast<unsigned>(items < sm_count ? items : sm_count);
  launch_kernel(kern, grid, gemm_threads(EPI), smem, stream, maps, p);
  return after_launch("gemm");
}

int launch_gemm(int ksw, int epi, const GemmMaps& maps, const GemmParams& p, int sm_count,
                cudaStream_t stream) {
  if (ksw == 64) {
    if (epi == EPI_QKV) return launch_gemm_t<64, EPI_QKV>(maps, p, sm_count, stream);
    if (epi == EPI_RESID_LN) return launch_gemm_t<64, EPI_RESID_LN>(maps, p, sm_count, stream);
    return launch_gemm_t<64, EPI_GELU>(maps, p, sm_count, stream);
  }
  if (epi == EPI_QKV) return launch_gemm_t<32, EPI_QKV>(maps, p, sm_count, stream);
  if (epi == EPI_RESID_LN) return launch_gemm_t<32, EPI_RESID_LN>(maps, p, sm_count, stream);
  return launch_gemm_t<32, EPI_GELU>(maps, p, sm_count, stream);
}

GemmParams base_params(DeviceState* ds) {
  GemmParams p;
  memset(&p, 0, sizeof(p));
  p.err = ds->err;
  p.timeout_ns = g_timeout_ns.load();
  return p;
}

int launch_ffn(const FfnMaps& maps, FfnParams p, int sm_count, cudaStream_t stream) {
  const long long items = (static_cast<long long>(p.M) + 127) / 128;
  p.n_items = static_cast<int>(items);
  const unsigned grid = static_cast<unsigned>(items < sm_count ? items : sm_count);
  switch (p.D) {
#define TT_FFN_CASE(DD)                                                     \
  case DD: {                                                                \
    auto kern = ffn_fused_kernel<DD>;                                       \
    const int smem = FfnLayout<DD>::smem_bytes(p.F);                        \
    if (smem > 232448) return fail(TT_ERR_UNSUPPORTED, "ffn %d too wide", p.F); \
    if (int rc = prepare_kernel(kern, smem)) return rc;                     \
    launch_kernel(kern, grid, kFfnThreads, smem, stream, maps, p);          \
    break;                                                                  \
  }
    TT_FFN_CASE(32)
    TT_FFN_CASE(64)
    TT_FFN_CASE(128)
    TT_FFN_CASE(256)
#undef TT_FFN_CASE
    default:
      return fail(TT_ERR_UNSUPPORTED, "fused FFN: d_model %d not in {32, 64, 128, 256}", p.D);
  }
  return after_launch("ffn");
}

// The TMEM-resident-hidden FFN (tt_ffn2.cuh) serves d_model 128 and 256.
bool ffn2_route(int d_model, int ffn) { return (d_model == 128 || d_model == 256) && ffn % 128 == 0; }

int launch_ffn2(const Ffn2Maps& maps, FfnParams p, int sm_count, cudaStream_t stream) {
  const long long items = (static_cast<long long>(p.M) + 127) / 128;
  p.n_items = static_cast<int>(items);
  const unsigned grid = static_cast<unsigned>(items < sm_count ? items : sm_count);
  if (p.D == 128) {
    if (int rc = prepare_kernel(ffn2_kernel<128>, Ffn2Layout<128>::SMEM_ALLOC)) return rc;
    launch_kernel(ffn2_kernel<128>, grid, kFfn2Threads, Ffn2Layout<128>::SMEM_ALLOC, stream, maps, p);
  } else if (p.D == 256) {
    if (int rc = prepare_kernel(ffn2_kernel<256>, Ffn2Layout<256>::SMEM_ALLOC)) return rc;
    launch_kernel(ffn2_kernel<256>, grid, kFfn2Threads, Ffn2Layout<256>::SMEM_ALLOC, stream, maps, p);
  } else {
    return fail(TT_ERR_UNSUPPORTED, "ffn2: d_model %d not in {128, 256}", p.D);
  }
  return after_launch("ffn");
}

// Row-major [rows, cols] FP16 matrix as K-blocks of 64 columns: the 3-D view
// {64, rows, cols / 64} (byte strides {cols * 2, 128}), box {64, box_rows,
// box_kblocks}; one copy writes box_kblocks consecutive [box_rows x 128 B]
// swizzled blocks.
int encode_kblocks(CUtensorMap* tm, const void* base, uint64_t rows, uint64_t cols, int box_rows,
                   int box_kblocks) {
  const uint64_t dims[3] = {64, rows, cols / 64};
  const uint64_t strides[2] = {cols * 2, 128};
  const uint32_t box[3] = {64, static_cast<uint32_t>(box_rows), static_cast<uint32_t>(box_kblocks)};
  return encode_f16(tm, base, 3, dims, strides, box);
}

// W1 of the fused FFN: one 32 KB ring slot is FC rows x W1_PER_SLOT K-blocks.
int encode_ffn2_w1(CUtensorMap* tm, const void* w1, int D, int F) {
  if (D == 256) return encode_kblocks(tm, w1, F, D, Ffn2Layout<256>::FC, Ffn2Layout<256>::W1_PER_SLOT);
  return encode_kblocks(tm, w1, F, D, Ffn2Layout<128>::FC, Ffn2Layout<128>::W1_PER_SLOT);
}

int encode_ffn2_maps(Ffn2Maps* maps, const void* a, const void* w1, const void* w2, uint64_t rows, int D, int F) {
  memset(maps, 0, sizeof(*maps));
  if (int rc = encode_kblocks(&maps->a, a, rows, D, 128, D / 64)) return rc;
  if (int rc = encode_ffn2_w1(&maps->w1, w1, D, F)) return rc;
  return encode_matrix(&maps->w2, w2, D, F, 64, D < 256 ? D : 256);
}

// Tensor maps of the fused FFN for one call.
int encode_ffn_maps(FfnMaps* maps, const void* a, const void* w1, const void* w2, const float* resid_out,
                    const void* norm_out, bool norm_f32, uint64_t rows, int D, int F) {
  memset(maps, 0, sizeof(*maps));
  if (int rc = encode_matrix(&maps->a, a, rows, D, 32, 128)) return rc;
  if (int rc = encode_matrix(&maps->w1, w1, F, D, 32, 128)) return rc;
  if (int rc = encode_matrix(&maps->w2, w2, D, F, 32, D)) return rc;
  if (resid_out)
    if (int rc = encode_epi_tile(&maps->out0, resid_out, rows, D, true)) return rc;
  if (norm_out)
    if (int rc = encode_epi_tile(&maps->out1, norm_out, rows, D, norm_f32)) return rc;
  return TT_OK;
}

int run_layernorm(const float* x, const float* gamma, const float* beta, void* out,
                  long long n_rows, int d, float eps, int out_f16, cudaStream_t stream,
                  const uint8_t* row_mask = nullptr) {
  if (n_rows <= 0) return TT_OK;
  const unsigned grid = static_cast<unsigned>((n_rows + 7) / 8);
  switch (d / 32) {
#define TT_LN_CASE(V)                                                                  \
  case V:                                                                              \
    launch_kernel(layernorm_rows_kernel<V>, grid, 256, 0, stream, x, gamma, beta, out, n_rows, eps, \
                  out_f16, row_mask);                                                              \
    break;
    TT_LN_CASE(1)
    TT_LN_CASE(2)
    TT_LN_CASE(3)
    TT_LN_CASE(4)
    TT_LN_CASE(8)
    TT_LN_CASE(12)
    TT_LN_CASE(16)
    TT_LN_CASE(24)
    TT_LN_CASE(32)
#undef TT_LN_CASE
    default:
      return fail(TT_ERR_UNSUPPORTED, "layernorm width %d not supported", d);
  }
  return after_launch("layernorm");
}

int check_ln_width(int d) {
  const int v = d / 32;
  if (d % 32 != 0 || !(v == 1 || v == 2 || v == 3 || v == 4 || v == 8 || v == 12 || v == 16 ||
                       v == 24 || v == 32))
    return fail(TT_ERR_UNSUPPORTED, "layernorm width %d not supported", d);
  return TT_OK;
}

// Q/K/V^T tensor maps for attention over a [B*H, S, hs] / [B*H, hs, S_pad]
// layout (hs = stored_head_dim(hd)).
int encode_attention_maps(CUtensorMap* tq, CUtensorMap* tk, CUtensorMap* tv, const void* q,
                          const void* k, const void* vt, int bh, int seq, int hd_real, int seq_pad) {
  const int hd = stored_head_dim(hd_real);
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(hd), static_cast<uint64_t>(seq),
                              static_cast<uint64_t>(bh)};
    const uint64_t strides[2] = {static_cast<uint64_t>(hd) * 2,
                                 static_cast<uint64_t>(hd) * seq * 2};
    // 128-query and 64-key tiles; above 64 features (128-byte rows) a tile is
    // copied as several boxes of 64 features, one per swizzle atom.
    const uint32_t inner = static_cast<uint32_t>(hd < 64 ? hd : 64);
    const uint32_t box[3] = {inner, 128, 1};
    if (int rc = encode_f16(tq, q, 3, dims, strides, box)) return rc;
    const uint32_t kbox[3] = {inner, 64u, 1};
    if (int rc = encode_f16(tk, k, 3, dims, strides, kbox)) return rc;
  }
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(seq_pad), static_cast<uint64_t>(hd),
                              static_cast<uint64_t>(bh)};
    const uint64_t strides[2] = {static_cast<uint64_t>(seq_pad) * 2,
                                 static_cast<uint64_t>(seq_pad) * hd * 2};
    const uint32_t box[3] = {64, static_cast<uint32_t>(hd), 1};
    if (int rc = encode_f16(tv, vt, 3, dims, strides, box)) return rc;
  }
  return TT_OK;
}

template <int HD>
int launch_attn_db(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const AttnParams& ap,
                   int n_items, int sm_count, cudaStream_t stream) {
  using L = AttnDbLayout<HD>;
  auto kern = attn_db_fwd_kernel<HD>;
  KernelInfo ki;
  if (int rc = kernel_info(reinterpret_cast<const void*>(kern), L::SMEM_ALLOC, &ki)) return rc;
  // The kernel splits its registers with setmaxnreg; that split is only sound
  // when each thread is launched with exactly the planned register count.
  if (L::SPLIT ? ki.regs != L::REGS_LAUNCH : ki.regs > 255)
    return fail(TT_ERR_UNSUPPORTED, "attention kernel built with %d registers per thread, expected %d", ki.regs,
                L::REGS_LAUNCH);
  const int ctas = (n_items + L::NS - 1) / L::NS;
  const unsigned grid = static_cast<unsigned>(ctas < sm_count ? ctas : sm_count);
  launch_kernel(kern, grid, L::THREADS, L::SMEM_ALLOC, stream, tq, tk, tv, ap, n_items);
  return TT_OK;
}

int launch_attention(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                     const AttnParams& ap, int hd, int sm_count, cudaStream_t stream) {
  const long long n_qt = (ap.seq + 127) / 128;
  const long long items = static_cast<long long>(ap.batch) * ap.heads * n_qt;
  if (items > 0x7fffffffLL) return fail(TT_ERR_SHAPE, "batch*heads*query tiles too large");
  const int n_items = static_cast<int>(items);
  if (ap.ctx_hd != hd) return fail(TT_ERR_ARG, "ctx head width %d != head_dim %d", ap.ctx_hd, hd);
  // 64-key tiles, scores and the probabilities over them in TMEM; head_dim 8
  // runs the head_dim-16 kernel on its zero-padded Q/K/V.
  int rc;
  switch (hd) {
    case 8:
    case 16: rc = launch_attn_db<16>(tq, tk, tv, ap, n_items, sm_count, stream); break;
    case 32: rc = launch_attn_db<32>(tq, tk, tv, ap, n_items, sm_count, stream); break;
    case 64: rc = launch_attn_db<64>(tq, tk, tv, ap, n_items, sm_count, stream); break;
    case 128: rc = launch_attn_db<128>(tq, tk, tv, ap, n_items, sm_count, stream); break;
    case 256: rc = launch_attn_db<256>(tq, tk, tv, ap, n_items, sm_count, stream); break;
    default: return fail(TT_ERR_UNSUPPORTED, "head_dim %d not in {8, 16, 32, 64, 128, 256}", hd);
  }
  if (rc) return rc;
  return after_launch("attention");
}

}  // namespace
}  // namespace tt

using namespace tt;

// ---------------------------------------------------------------------------
// Allocation-free masked attention: static scratch.
//
// Some callers cannot call cudaMalloc at all, or not at the moment they
// launch: a host program that captures its launches into a CUDA graph, a
// runtime whose device memory is owned by an external pool or arena, or a
// latency-critical server that forbids allocation after start-up.  For them
// tt_causal_attention_masked_noalloc keeps the one scratch buffer the masked
// attention path needs (the per-sequence end of the valid keys, one int per
// sequence) in this file-scope device array instead of a caller buffer.
// Every GPU that loads the library holds it (256 KiB) until the process exits.
// ---------------------------------------------------------------------------
static constexpr int kNoAllocMaxBatch = 65536;
static __device__ __align__(256) int g_noalloc_kv_end[kNoAllocMaxBatch];

namespace {

struct NoAllocScratch {
  std::once_flag once;
  int status = TT_OK;
  int* kv_end = nullptr;  // device address of g_noalloc_kv_end on this device
};
NoAllocScratch g_noalloc[64];

// In host code `g_noalloc_kv_end` names a host-side stand-in, not device
// memory, so its device address is looked up once per device (with that
// device current) and cached.
int noalloc_scratch_for_current_device(int** out) {
  int dev = 0;
  if (int rc = check_cuda(cudaGetDevice(&dev), "cudaGetDevice")) return rc;
  if (dev < 0 || dev >= 64) return fail(TT_ERR_ARG, "device ordinal %d out of range", dev);
  NoAllocScratch& st = g_noalloc[dev];
  std::call_once(st.once, [&] {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_kv_end);
    if (e != cudaSuccess) {
      st.status = fail(TT_ERR_LAUNCH, "cudaGetSymbolAddress(no-alloc scratch): %s", cudaGetErrorString(e));
      return;
    }
    st.kv_end = static_cast<int*>(p);
    st.status = TT_OK;
  });
  if (st.status != TT_OK) return st.status;
  *out = st.kv_end;
  return TT_OK;
}

}  // namespace

// =========================================================================
// Whole model
// =========================================================================
struct tt_model {
  int device = -1;
  int D = 0, H = 0, F = 0, L = 0, causal = 1;
  float eps = 1e-5f;
  const float* ln0_w = nullptr;
  const float* ln0_b = nullptr;
  std::vector<tt_layer_weights> layers;
  // Per-layer weight tensor maps (split FFN route: tm_win/tm_wout2; fused: tm_w1f/tm_w2f).
  std::vector<CUtensorMap> tm_wqkv, tm_wout, tm_win, tm_wout2, tm_w1f, tm_w2f;
  // Route + bound workspace (re-encoded when shape or workspace change).
  Route route{};
  int route_seq = -1;
  int bound_batch = -1, bound_seq = -1;
  void* bound_ws = nullptr;
  int ksw_qkv = 64, ksw_out = 64, ksw_in = 64, ksw_out2 = 64;
  // Operand loads (box {KSW, 128}) and attention loads.
  CUtensorMap tm_norm{}, tm_ctx{}, tm_hidden{}, tm_q{}, tm_k{}, tm_vt{};
  // Epilogue tiles (box 32 x 32): QKV stores, residual (FP32), normalized and hidden (FP16).
  CUtensorMap tm_resid{}, tm_norm_st{}, tm_hidden_st{};
  CUtensorMap tm_q_st{}, tm_k_st{}, tm_vt_st{};  // QKV epilogue's TMA stores (seq % 32 == 0, head_dim >= 32)
  CUtensorMap tm_norm32{};  // normalized activations as the fused FFN's A operand (box {32, 128})
  CUtensorMap tm_norm3{};   // the same as whole 128-row K-block tiles (ffn2_kernel)
  // Profiling.
  bool profiling = false;
  struct Rec {
    int kind;
    cudaEvent_t a, b;
  };
  std::vector<Rec> recs;
  std::vector<cudaEvent_t> pool;
  // Host-buffer pipeline (tt_model_forward_host): one copy stream per
  // direction and per-buffer events, created on first use.
  cudaStream_t h2d = nullptr, d2h = nullptr;
  cudaEvent_t ev_entry = nullptr, ev_in[2] = {}, ev_comp[2] = {}, ev_out[2] = {}, ev_join[2] = {};
  // Batch-shard gather (tt_model_forward_gather): the copy stream that pushes
  // a finished shard to its destination, the event after each forward, and
  // the event after the latest push (gather_pending: one was issued).
  cudaStream_t gather = nullptr;
  cudaEvent_t ev_fwd_done = nullptr, ev_gathered = nullptr;
  bool gather_pending = false;
};

namespace {

struct WsLayout {
  size_t resid, norm, q, k, vt, ctx, hidden, kv_end, total;
  int seq_pad;
};

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

WsLayout ws_layout(const tt_model* m, int batch, int seq) {
  WsLayout w;
  const size_t N = static_cast<size_t>(batch) * seq;
  const int hs = stored_head_dim(m->D / m->H);
  w.seq_pad = (seq + 7) / 8 * 8;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align_up(off + bytes, 1024);
    return o;
  };
  w.resid = take(N * m->D * 4);
  w.norm = take(N * m->D * 2);
  w.q = take(N * m->H * hs * 2);
  w.k = take(N * m->H * hs * 2);
  w.vt = take(static_cast<size_t>(batch) * m->H * hs * w.seq_pad * 2);
  w.ctx = take(N * m->D * 2);
  Route r;
  const bool fused = choose_route(m->D, m->H, seq, m->F, &r) == TT_OK && r.ffn_fused;
  w.hidden = take(fused ? 0 : N * m->F * 2);
  w.kv_end = take(static_cast<size_t>(batch) * 4);
  w.total = off;
  return w;
}

// Workspace of the host-buffer pipeline: the model workspace of one chunk,
// then two device copies (ping-pong) of a chunk's input, output and mask.
struct HostWsLayout {
  size_t model, x[2], out[2], mask[2], total;
};

HostWsLayout host_ws_layout(const tt_model* m, int chunk, int seq) {
  HostWsLayout h;
  const size_t rows = static_cast<size_t>(chunk) * seq;
  size_t off = align_up(ws_layout(m, chunk, seq).total, 1024);
  h.model = 0;
  for (int b = 0; b < 2; ++b) {
    h.x[b] = off;
    off = align_up(off + rows * m->D * 4, 1024);
    h.out[b] = off;
    off = align_up(off + rows * m->D * 4, 1024);
    h.mask[b] = off;
    off = align_up(off + rows, 1024);
  }
  h.total = off;
  return h;
}

int require_pinned(const void* p, const char* what) {
  cudaPointerAttributes a;
  if (int rc = check_cuda(cudaPointerGetAttributes(&a, p), "cudaPointerGetAttributes")) return rc;
  if (a.type != cudaMemoryTypeHost)
    return fail(TT_ERR_ARG, "%s must be page-locked host memory (cudaHostAlloc, cudaHostRegister or a pinned "
                "tensor)", what);
  return TT_OK;
}

int ensure_copy_streams(tt_model* m) {
  if (m->h2d) return TT_OK;
  if (int rc = check_cuda(cudaStreamCreateWithFlags(&m->h2d, cudaStreamNonBlocking), "cudaStreamCreate"))
    return rc;
  if (int rc = check_cuda(cudaStreamCreateWithFlags(&m->d2h, cudaStreamNonBlocking), "cudaStreamCreate"))
    return rc;
  for (cudaEvent_t* e : {&m->ev_entry, &m->ev_in[0], &m->ev_in[1], &m->ev_comp[0], &m->ev_comp[1],
                         &m->ev_out[0], &m->ev_out[1], &m->ev_join[0], &m->ev_join[1]})
    if (int rc = check_cuda(cudaEventCreateWithFlags(e, cudaEventDisableTiming), "cudaEventCreate")) return rc;
  return TT_OK;
}

int ensure_gather_stream(tt_model* m) {
  if (m->gather) return TT_OK;
  if (int rc = check_cuda(cudaStreamCreateWithFlags(&m->gather, cudaStreamNonBlocking), "cudaStreamCreate"))
    return rc;
  for (cudaEvent_t* e : {&m->ev_fwd_done, &m->ev_gathered})
    if (int rc = check_cuda(cudaEventCreateWithFlags(e, cudaEventDisableTiming), "cudaEventCreate")) return rc;
  return TT_OK;
}

int record_begin(tt_model* m, cudaStream_t s, cudaEvent_t* ev) {
  if (!m->profiling) return TT_OK;
  if (m->pool.empty()) {
    cudaEvent_t e;
    if (int rc = check_cuda(cudaEventCreate(&e), "cudaEventCreate")) return rc;
    m->pool.push_back(e);
  }
  *ev = m->pool.back();
  m->pool.pop_back();
  return check_cuda(cudaEventRecord(*ev, s), "cudaEventRecord");
}

int record_end(tt_model* m, cudaStream_t s, int kind, cudaEvent_t start) {
  if (!m->profiling) return TT_OK;
  if (m->pool.empty()) {
    cudaEvent_t e;
    if (int rc = check_cuda(cudaEventCreate(&e), "cudaEventCreate")) return rc;
    m->pool.push_back(e);
  }
  cudaEvent_t end = m->pool.back();
  m->pool.pop_back();
  m->recs.push_back({kind, start, end});
  return check_cuda(cudaEventRecord(end, s), "cudaEventRecord");
}

int bind_workspace(tt_model* m, int batch, int seq, void* ws) {
  if (m->route_seq != seq) {
    if (int rc = choose_route(m->D, m->H, seq, m->F, &m->route)) return rc;
    m->route_seq = seq;
    // Weight maps depend on the route's column tiles.
    m->ksw_qkv = gemm_ksw(m->D, m->route.qkv_bn);
    const int resid_bn = wide_model(m->D) ? kWideBn : m->D;  // column tile of the residual GEMMs
    m->ksw_out = gemm_ksw(m->D, resid_bn);
    m->ksw_in = gemm_ksw(m->D, m->route.ffn_in_bn);
    m->ksw_out2 = gemm_ksw(m->F, resid_bn);
    m->tm_wqkv.resize(m->L);
    m->tm_wout.resize(m->L);
    m->tm_win.resize(m->L);
    m->tm_wout2.resize(m->L);
    const int out_box = m->D > 256 ? 256 : m->D;
    for (int l = 0; l < m->L; ++l) {
      const tt_layer_weights& w = m->layers[l];
      if (int rc = encode_matrix(&m->tm_wqkv[l], w.w_qkv, 3 * m->D, m->D, m->ksw_qkv, m->route.qkv_bn))
        return rc;
      if (int rc = encode_matrix(&m->tm_wout[l], w.w_out, m->D, m->D, m->ksw_out, out_box)) return rc;
      if (int rc = encode_matrix(&m->tm_win[l], w.w_ffn_in, m->F, m->D, m->ksw_in, m->route.ffn_in_bn))
        return rc;
      if (int rc = encode_matrix(&m->tm_wout2[l], w.w_ffn_out, m->D, m->F, m->ksw_out2, out_box))
        return rc;
      if (m->route.ffn_fused) {
        m->tm_w1f.resize(m->L);
        m->tm_w2f.resize(m->L);
        // The TMEM-hidden kernel (d_model 128/256) reads 64-wide K-blocks, the other one 32-wide.
        const bool f2 = ffn2_route(m->D, m->F);
        if (f2) {
          if (int rc = encode_ffn2_w1(&m->tm_w1f[l], w.w_ffn_in, m->D, m->F)) return rc;
        } else if (int rc = encode_matrix(&m->tm_w1f[l], w.w_ffn_in, m->F, m->D, 32, 128)) {
          return rc;
        }
        if (int rc = encode_matrix(&m->tm_w2f[l], w.w_ffn_out, m->D, m->F, f2 ? 64 : 32,
                                   f2 && m->D > 256 ? 256 : m->D))
          return rc;
      }
    }
    m->bound_ws = nullptr;
  }
  if (m->bound_ws == ws && m->bound_batch == batch && m->bound_seq == seq) return TT_OK;
  const WsLayout w = ws_layout(m, batch, seq);
  uint8_t* base = static_cast<uint8_t*>(ws);
  const uint64_t N = static_cast<uint64_t>(batch) * seq;
  const int hd = m->D / m->H;
  if (m->ksw_qkv != m->ksw_in) return fail(TT_ERR_UNSUPPORTED, "QKV and FFN-in K-blocks differ");
  if (int rc = encode_matrix(&m->tm_norm, base + w.norm, N, m->D, m->ksw_qkv, 128)) return rc;
  if (int rc = encode_matrix(&m->tm_ctx, base + w.ctx, N, m->D, m->ksw_out, 128)) return rc;
  if (!m->route.ffn_fused)
    if (int rc = encode_matrix(&m->tm_hidden, base + w.hidden, N, m->F, m->ksw_out2, 128)) return rc;
  if (int rc = encode_matrix(&m->tm_norm32, base + w.norm, N, m->D, 32, 128)) return rc;
  if (ffn2_route(m->D, m->F))
    if (int rc = encode_kblocks(&m->tm_norm3, base + w.norm, N, m->D, 128, m->D / 64)) return rc;
  if (int rc = encode_attention_maps(&m->tm_q, &m->tm_k, &m->tm_vt, base + w.q, base + w.k,
                                     base + w.vt, batch * m->H, seq, hd, w.seq_pad))
    return rc;
  if (int rc = encode_epi_tile(&m->tm_resid, base + w.resid, N, m->D, true)) return rc;
  if (seq % 32 == 0 && hd >= 32) {
    GemmMaps st;
    if (int rc = encode_qkv_store_maps(&st, base + w.q, base + w.k, base + w.vt, batch, seq, m->H, hd, w.seq_pad))
      return rc;
    m->tm_q_st = st.out0;
    m->tm_k_st = st.out1;
    m->tm_vt_st = st.res;
  }
  if (int rc = encode_epi_tile(&m->tm_norm_st, base + w.norm, N, m->D, false)) return rc;
  if (!m->route.ffn_fused)
    if (int rc = encode_epi_tile(&m->tm_hidden_st, base + w.hidden, N, m->F, false)) return rc;
  m->bound_ws = ws;
  m->bound_batch = batch;
  m->bound_seq = seq;
  return TT_OK;
}

}  // namespace

extern "C" {

int tt_abi_version(void) { return kAbiVersion; }

const char* tt_last_error(void) { return g_last_error; }

void tt_set_wait_timeout_ns(unsigned long long ns) { g_timeout_ns.store(ns ? ns : 1); }

unsigned long long tt_launch_count(void) { return g_launches.load(); }

int tt_device_error(unsigned int* word, int clear) {
  DeviceState* ds;
  if (int rc = current_device_state(&ds)) return rc;
  if (int rc = check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize")) return rc;
  unsigned int w = 0;
  if (int rc = check_cuda(cudaMemcpy(&w, ds->err, sizeof(w), cudaMemcpyDeviceToHost), "read error word"))
    return rc;
  if (word) *word = w;
  if (clear && w != 0)
    if (int rc = check_cuda(cudaMemset(ds->err, 0, sizeof(unsigned int)), "clear error word"))
      return rc;
  if (w & kDevErrTimeout)
    return fail(TT_ERR_TIMEOUT, "a bounded in-kernel wait timed out (site 0x%x)", w & 0xffffu);
  return TT_OK;
}

int tt_watchdog_selftest(unsigned long long timeout_ns, void* stream) {
  DeviceState* ds;
  if (int rc = current_device_state(&ds)) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (int rc = check_cuda(cudaStreamSynchronize(s), "cudaStreamSynchronize")) return rc;
  if (int rc = check_cuda(cudaMemset(ds->err, 0, sizeof(unsigned int)), "clear error word"))
    return rc;
  watchdog_selftest_kernel<<<1, 32, 0, s>>>(ds->err, timeout_ns);
  if (int rc = after_launch("watchdog self-test")) return rc;
  if (int rc = check_cuda(cudaStreamSynchronize(s), "cudaStreamSynchronize")) return rc;
  unsigned int w = 0;
  if (int rc = check_cuda(cudaMemcpy(&w, ds->err, sizeof(w), cudaMemcpyDeviceToHost), "read error word"))
    return rc;
  if (int rc = check_cuda(cudaMemset(ds->err, 0, sizeof(unsigned int)), "clear error word"))
    return rc;
  if ((w & kDevErrTimeout) && (w & 0xffffu) == 0x7e57u)
    return fail(TT_ERR_TIMEOUT, "watchdog fired as designed (word 0x%x)", w);
  return fail(TT_ERR_LAUNCH, "watchdog did not fire (word 0x%x)", w);
}

int tt_selftest_exp2_fma(const float* x, float* y32, uint16_t* y16, int n, void* stream) {
  DeviceState* ds;
  if (int rc = current_device_state(&ds)) return rc;
  if (!x || !y32 || !y16 || n < 0 || n % 2 != 0) return fail(TT_ERR_ARG, "invalid argument");
  if (reinterpret_cast<uintptr_t>(y16) % 4 != 0) return fail(TT_ERR_ALIGN, "y16 must be 4-byte aligned");
  const int pairs = n / 2;
  if (pairs == 0) return TT_OK;
  exp2_fma_probe_kernel<<<(pairs + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      x, y32, reinterpret_cast<uint32_t*>(y16), pairs);
  return after_launch("exp2 probe");
}

int tt_layernorm_rows(const float* x, const float* gamma, const float* beta, void* out,
                      int64_t n_rows, int d, float eps, int out_is_f16, void* stream) {
  DeviceState* ds;
  if (int rc = current_device_state(&ds)) return rc;
  if (!x || !gamma || !beta || !out || n_rows < 0) return fail(TT_ERR_ARG, "null argument");
  if (int rc = check_ln_width(d)) return rc;
  return run_layernorm(x, gamma, beta, out, n_rows, d, eps, out_is_f16,
                       static_cast<cudaStream_t>(stream));
}

int tt_mask_kv_end(const uint8_t* mask, int batch, int seq, int* kv_end, void* stream) {
  DeviceState* ds;
  if (int rc = current_device_state(&ds)) return rc;
  if (!mask || !kv_end || batch < 0 || seq <= 0) return fail(TT_ERR_ARG, "invalid argument");
  if (batch == 0) return TT_OK;
  mask_kv_end_kernel<<<batch, 256, 0, static_cast<cudaStream_t>(stream)>>>(mask, seq, kv_end);
  return after_launch("mask_kv_end");
}

int tt_qkv_projection(const void* normalized, const void* w_qkv, const float* b_qkv, void* q,
                      void* k, void* vt, int batch, int seq, int d_model, int heads, int seq_pad,
                      void* stream) {
  DeviceState* ds;
  if (int rc = current_device_state(&ds)) return rc;
  if (!normalized || !w_qkv || !b_qkv || !q || !k || !vt) return fail(TT_ERR_ARG, "null argument");
  if (batch <= 0 || seq <= 0 || seq_pad < seq || seq_pad % 8 != 0)
    return fail(TT_ERR_SHAPE, "invalid batch/seq/seq_pad (%d, %d, %d)", batch, seq, seq_pad);
  if (int rc = check_model_shape(d_model, heads, 32)) return rc;
  const uint64_t N = static_cast<uint64_t>(batch) * seq;
  if (N > 0x7fffffffULL) return fail(TT_ERR_SHAPE, "too many rows");
  const int bn = largest_bn_dividing(3 * d_model, d_model <= 128 ? 128 : 256);
  const int ksw = gemm_ksw(d_model, bn);
  const int hd = d_model / heads;
  GemmMaps maps;
  memset(&maps, 0, sizeof(maps));
  if (int rc = encode_matrix(&maps.a, normalized, N, d_model, ksw, 128)) return rc;
  if (int rc = encode_matrix(&maps.w, w_qkv, 3 * d_model, d_model, ksw, bn)) return rc;
  const bool tma_out = seq % 32 == 0;
  // The epilogue writes Q, K and V^T in 16-byte pieces.
  if (reinterpret_cast<uintptr_t>(q) % 16 || reinterpret_cast<uintptr_t>(k) % 16 ||
      reinterpret_cast<uintptr_t>(vt) % 16)
    return fail(TT_ERR_ALIGN, "q, k and vt must be 16-byte aligned");
  if (tma_out && hd >= 32)
    if (int rc = encode_qkv_store_maps(&maps, q, k, vt, batch, seq, heads, hd, seq_pad)) return rc;
  GemmParams p = base_params(ds);
  p.M = static_cast<int>(N);
  p.N_total = 3 * d_model;
  p.K = d_model;
  p.bn = bn;
  p.n_splits = p.N_total / bn;
  p.nst = clamp_nst(ksw, bn, p.K, 4, EPI_QKV, p.N_total);
  p.tma_out = tma_out ? 1 : 0;
  p.bias = b_qkv;
  p.q = static_cast<__half*>(q);
  p.k = static_cast<__half*>(k);
  p.vt = static_cast<__half*>(vt);
  p.seq = seq;
  p.heads = heads;
  p.head_dim = hd;
  p.seq_pad = seq_pad;
  p.d_model = d_model;
  return launch_gemm(ksw, EPI_QKV, maps, p, ds->sm_count, static_cast<cudaStream_t>(stream));
}

int tt_causal_attention(const void* q, const void* k, const void* vt, const uint8_t* key_mask,
                        const int* kv_end, void* ctx, int batch, int seq, int heads, int head_dim,
                        int seq_pad, float scale, int causal, void* stream) {
  DeviceState* ds;
  if (int rc = current_device_state(&ds)) return rc;
  if (!q || !k || !vt || !ctx || (key_mask && !kv_end)) return fail(TT_ERR_ARG, "null argument");
  if (batch <= 0 || seq <= 0 || heads <= 0 || seq_pad < seq || seq_pad % 8 != 0)
    return fail(TT_ERR_SHAPE, "invalid sizes");
  if (!attention_head_dim_ok(head_dim))
    return fail(TT_ERR_UNSUPPORTED, "head_dim %d not in {8, 16, 32, 64, 128, 256}", head_dim);
  CUtensorMap tq, tk, tv;
  if (int rc = encode_attention_maps(&tq, &tk, &tv, q, k, vt, batch * heads, seq, head_dim, seq_pad))
    return rc;
  AttnParams ap;
  ap.batch = batch;
  ap.seq = seq;
  ap.heads = heads;
  ap.seq_pad = seq_pad;
  ap.causal = causal ? 1 : 0;
  ap.scale_log2 = scale * 1.4426950408889634f;
  ap.key_mask = key_mask;
  ap.kv_end = kv_end;
  ap.ctx = static_cast<__half*>(ctx);
  ap.ctx_hd = head_dim;
  ap.err = ds->err;
  ap.timeout_ns = g_timeout_ns.load();
  return launch_attention(tq, tk, tv, ap, head_dim, ds->sm_count, static_cast<cudaStream_t>(stream));
}

int tt_causal_attention_masked_noalloc(const void* q, const void* k, const void* vt,
                                       const uint8_t* key_mask, void* ctx, int batch, int seq,
                                       int heads, int head_dim, int seq_pad, float scale, int causal,
                                       void* stream) {
  // Set-up on the first call on a device (needs that device current): the
  // scratch array's device address.  Allocates nothing, here or later.
  DeviceState* ds;
  if (int rc = current_device_state(&ds)) return rc;
  int* kv_end = nullptr;
  if (int rc = noalloc_scratch_for_current_device(&kv_end)) return rc;
  if (!q || !k || !vt || !ctx) return fail(TT_ERR_ARG, "null argument");
  if (batch <= 0 || seq <= 0 || heads <= 0 || seq_pad < seq || seq_pad % 8 != 0)
    return fail(TT_ERR_SHAPE, "invalid sizes");
  if (batch > kNoAllocMaxBatch)
    return fail(TT_ERR_SHAPE,
                "batch %d exceeds the %d sequences the static scratch of "
                "tt_causal_attention_masked_noalloc holds; split the batch",
                batch, kNoAllocMaxBatch);
  CUtensorMap tq, tk, tv;
  if (int rc = encode_attention_maps(&tq, &tk, &tv, q, k, vt, batch * heads, seq, head_dim, seq_pad))
    return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (key_mask) {
    // Overwrites kv_end[0..batch); entries past `batch` are never read, so
    // whatever an earlier call left in the shared array needs no clearing.
    mask_kv_end_kernel<<<batch, 256, 0, s>>>(key_mask, seq, kv_end);
    if (int rc = after_launch("mask_kv_end (no-alloc)")) return rc;
  }
  AttnParams ap;
  ap.batch = batch;
  ap.seq = seq;
  ap.heads = heads;
  ap.seq_pad = seq_pad;
  ap.causal = causal ? 1 : 0;
  ap.scale_log2 = scale * 1.4426950408889634f;
  ap.key_mask = key_mask;
  ap.kv_end = key_mask ? kv_end : nullptr;
  ap.ctx = static_cast<__half*>(ctx);
  ap.ctx_hd = head_dim;
  ap.err = ds->err;
  ap.timeout_ns = g_timeout_ns.load();
  return launch_attention(tq, tk, tv, ap, head_dim, ds->sm_count, s);
}

int tt_linear_residual_layernorm(const void* a, const void* w, const float* bias,
                                 const float* resid_in, const float* gamma, const float* beta,
                                 float* resid_out, void* norm_out, int64_t n_rows, int k_in,
                                 int d_model, float eps, int norm_out_is_f16,
                                 const uint8_t* row_mask, void* stream) {
  DeviceState* ds;
  if (int rc = current_device_state(&ds)) return rc;
  if (!a || !w || !bias || !resid_in || !gamma || !beta || !resid_out || !norm_out)
    return fail(TT_ERR_ARG, "null argument");
  if (n_rows <= 0 || n_rows > 0x7fffffffLL || k_in <= 0 || k_in % 32 != 0)
    return fail(TT_ERR_SHAPE, "invalid n_rows/k_in (%lld, %d)", (long long)n_rows, k_in);
  if (d_model % 32 != 0 || d_model <= 0 || (d_model > 256 && d_model != 512 && !wide_model(d_model)))
    return fail(TT_ERR_UNSUPPORTED, "d_model %d must be a multiple of 32 up to 256, 512, 768 or 1024", d_model);
  const bool wide = wide_model(d_model);
  const int bn = wide ? kWideBn : d_model;
  const int ksw = gemm_ksw(k_in, bn);
  GemmMaps maps;
  memset(&maps, 0, sizeof(maps));
  if (int rc = encode_matrix(&maps.a, a, n_rows, k_in, ksw, 128)) return rc;
  if (int rc = encode_matrix(&maps.w, w, d_model, k_in, ksw, bn > 256 ? 256 : bn)) return rc;
  if (int rc = encode_epi_tile(&maps.out0, resid_out, n_rows, d_model, true)) return rc;
  if (int rc = encode_epi_tile(&maps.out1, norm_out, n_rows, d_model, norm_out_is_f16 == 0)) return rc;
  if (int rc = encode_epi_tile(&maps.res, resid_in, n_rows, d_model, true)) return rc;
  GemmParams p = base_params(ds);
  p.M = static_cast<int>(n_rows);
  p.N_total = d_model;
  p.K = k_in;
  p.bn = bn;
  p.n_splits = d_model / bn;
  p.no_norm = wide ? 1 : 0;
  p.nst = clamp_nst(ksw, p.bn, p.K, 4, EPI_RESID_LN, p.N_total);
  p.bias = bias;
  p.gamma = gamma;
  p.beta = beta;
  p.norm_f16 = norm_out_is_f16 ? 1 : 0;
  p.eps = eps;
  p.row_mask = row_mask;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (int rc = launch_gemm(ksw, EPI_RESID_LN, maps, p, ds->sm_count, s)) return rc;
  if (!wide) return TT_OK;
  // Rows wider than TMEM: the LayerNorm of the residual sum runs as a row kernel.
  return run_layernorm(resid_out, gamma, beta, norm_out, n_rows, d_model, eps, norm_out_is_f16 ? 1 : 0, s,
                       row_mask);
}

int tt_linear_gelu(const void* a, const void* w, const float* bias, void* out, int64_t n_rows,
                   int k_in, int n_out, void* stream) {
  DeviceState* ds;
  if (int rc = current_device_state(&ds)) return rc;
  if (!a || !w || !bias || !out) return fail(TT_ERR_ARG, "null argument");
  if (n_rows <= 0 || n_rows > 0x7fffffffLL || k_in <= 0 || k_in % 32 != 0 || n_out % 32 != 0)
    return fail(TT_ERR_SHAPE, "invalid sizes");
  const int bn = largest_bn_dividing(n_out, 256);
  if (bn == 0) return fail(TT_ERR_UNSUPPORTED, "n_out %d", n_out);
  const int ksw = gemm_ksw(k_in, bn);
  GemmMaps maps;
  memset(&maps, 0, sizeof(maps));
  if (int rc = encode_matrix(&maps.a, a, n_rows, k_in, ksw, 128)) return rc;
  if (int rc = encode_matrix(&maps.w, w, n_out, k_in, ksw, bn)) return rc;
  if (int rc = encode_epi_tile(&maps.out0, out, n_rows, n_out, false)) return rc;
  GemmParams p = base_params(ds);
  p.M = static_cast<int>(n_rows);
  p.N_total = n_out;
  p.K = k_in;
  p.bn = bn;
  p.n_splits = n_out / bn;
  p.nst = clamp_nst(ksw, bn, k_in, 4, EPI_GELU, n_out);
  p.bias = bias;
  return launch_gemm(ksw, EPI_GELU, maps, p, ds->sm_count, static_cast<cudaStream_t>(stream));
}

int tt_ffn_residual_layernorm(const void* a, const void* w1, const float* b1, const void* w2,
                              const float* b2, const float* resid_in, const float* gamma,
                              const float* beta, float* resid_out, void* norm_out, int64_t n_rows,
                              int d_model, int ffn, float eps, int norm_out_is_f16,
                              const uint8_t* row_mask, void* stream) {
  DeviceState* ds;
  if (int rc = current_device_state(&ds)) return rc;
  if (!a || !w1 || !b1 || !w2 || !b2 || !resid_in || !gamma || !beta || !resid_out || !norm_out)
    return fail(TT_ERR_ARG, "null argument");
  if (n_rows <= 0 || n_rows > 0x7fffffffLL) return fail(TT_ERR_SHAPE, "invalid n_rows %lld", (long long)n_rows);
  if (!ffn_fusable(d_model, ffn))
    return fail(TT_ERR_UNSUPPORTED,
                "fused FFN needs d_model in {32, 64, 128, 256} and ffn %% 128 == 0 (got %d, %d)", d_model,
                ffn);
  if (reinterpret_cast<uintptr_t>(b1) % 16 != 0) return fail(TT_ERR_ALIGN, "b1 must be 16-byte aligned");
  if (ffn2_route(d_model, ffn)) {
    if ((reinterpret_cast<uintptr_t>(resid_in) | reinterpret_cast<uintptr_t>(resid_out) |
         reinterpret_cast<uintptr_t>(norm_out)) % 16 != 0)
      return fail(TT_ERR_ALIGN, "resid_in, resid_out and norm_out must be 16-byte aligned");
    Ffn2Maps maps2;
    if (int rc = encode_ffn2_maps(&maps2, a, w1, w2, n_rows, d_model, ffn)) return rc;
    FfnParams p;
    memset(&p, 0, sizeof(p));
    p.M = static_cast<int>(n_rows);
    p.D = d_model;
    p.F = ffn;
    p.b1 = b1;
    p.b2 = b2;
    p.gamma = gamma;
    p.beta = beta;
    p.resid_in = resid_in;
    p.resid_out = resid_out;
    p.norm_out = norm_out;
    p.norm_f16 = norm_out_is_f16 ? 1 : 0;
    p.eps = eps;
    p.row_mask = row_mask;
    p.err = ds->err;
    p.timeout_ns = g_timeout_ns.load();
    return launch_ffn2(maps2, p, ds->sm_count, static_cast<cudaStream_t>(stream));
  }
  FfnMaps maps;
  if (int rc = encode_ffn_maps(&maps, a, w1, w2, resid_out, norm_out, norm_out_is_f16 == 0, n_rows, d_model, ffn))
    return rc;
  FfnParams p;
  memset(&p, 0, sizeof(p));
  p.M = static_cast<int>(n_rows);
  p.D = d_model;
  p.F = ffn;
  p.b1 = b1;
  p.b2 = b2;
  p.gamma = gamma;
  p.beta = beta;
  p.resid_in = resid_in;
  p.norm_f16 = norm_out_is_f16 ? 1 : 0;
  p.eps = eps;
  p.row_mask = row_mask;
  p.err = ds->err;
  p.timeout_ns = g_timeout_ns.load();
  return launch_ffn(maps, p, ds->sm_count, static_cast<cudaStream_t>(stream));
}

int tt_route_describe(int d_model, int heads, int seq, int ffn, char* buf, int buflen) {
  Route r;
  if (int rc = choose_route(d_model, heads, seq, ffn, &r)) return rc;
  if (buf && buflen > 0)
    snprintf(buf, buflen,
             "route=%s qkv_bn=%d qkv_nst=%d out_nst=%d ffn_in_bn=%d ffn_in_nst=%d "
             "ffn_out_nst=%d",
             r.name, r.qkv_bn, r.qkv_nst, r.out_nst, r.ffn_in_bn, r.ffn_in_nst, r.ffn_out_nst);
  if (buf && buflen > 0 && r.ffn_fused) {
    const size_t len = strlen(buf);
    snprintf(buf + len, buflen - len > 0 ? buflen - len : 0, " ffn=fused(chunk=128)");
  }
  return TT_OK;
}

int tt_model_create(const tt_model_desc* desc, tt_model** out) {
  if (!desc || !out || !desc->layers || !desc->ln0_w || !desc->ln0_b)
    return fail(TT_ERR_ARG, "null argument");
  *out = nullptr;
  DeviceState* ds;
  if (int rc = current_device_state(&ds)) return rc;
  if (int rc = check_model_shape(desc->d_model, desc->heads, desc->ffn_dim)) return rc;
  if (int rc = check_ln_width(desc->d_model)) return rc;
  if (desc->num_layers <= 0) return fail(TT_ERR_SHAPE, "num_layers must be positive");
  for (int l = 0; l < desc->num_layers; ++l) {
    const tt_layer_weights& w = desc->layers[l];
    if (!w.w_qkv || !w.b_qkv || !w.w_out || !w.b_out || !w.ln_attn_w || !w.ln_attn_b ||
        !w.w_ffn_in || !w.b_ffn_in || !w.w_ffn_out || !w.b_ffn_out || !w.ln_next_w || !w.ln_next_b)
      return fail(TT_ERR_ARG, "layer %d has a null parameter", l);
  }
  tt_model* m = new tt_model();
  cudaGetDevice(&m->device);
  m->D = desc->d_model;
  m->H = desc->heads;
  m->F = desc->ffn_dim;
  m->L = desc->num_layers;
  m->causal = desc->causal ? 1 : 0;
  m->eps = desc->eps;
  m->ln0_w = desc->ln0_w;
  m->ln0_b = desc->ln0_b;
  m->layers.assign(desc->layers, desc->layers + desc->num_layers);
  *out = m;
  return TT_OK;
}

void tt_model_destroy(tt_model* m) {
  if (!m) return;
  for (auto& r : m->recs) {
    cudaEventDestroy(r.a);
    cudaEventDestroy(r.b);
  }
  for (auto e : m->pool) cudaEventDestroy(e);
  if (m->h2d) cudaStreamDestroy(m->h2d);
  if (m->d2h) cudaStreamDestroy(m->d2h);
  if (m->gather) cudaStreamDestroy(m->gather);
  for (cudaEvent_t e : {m->ev_entry, m->ev_in[0], m->ev_in[1], m->ev_comp[0], m->ev_comp[1], m->ev_out[0],
                        m->ev_out[1], m->ev_join[0], m->ev_join[1], m->ev_fwd_done, m->ev_gathered})
    if (e) cudaEventDestroy(e);
  delete m;
}

int tt_workspace_alloc(size_t bytes, void** ptr) {
  if (!ptr || bytes == 0) return fail(TT_ERR_ARG, "invalid argument");
  *ptr = nullptr;
  DeviceState* ds;
  if (int rc = current_device_state(&ds)) return rc;
  return check_cuda(cudaMalloc(ptr, bytes), "cudaMalloc(workspace)");
}

int tt_workspace_free(void* ptr) {
  if (!ptr) return TT_OK;
  return check_cuda(cudaFree(ptr), "cudaFree(workspace)");
}

int tt_model_workspace_bytes(const tt_model* m, int batch, int seq, size_t* bytes) {
  if (!m || !bytes) return fail(TT_ERR_ARG, "null argument");
  if (batch <= 0 || seq <= 0) return fail(TT_ERR_SHAPE, "invalid batch/seq");
  *bytes = ws_layout(m, batch, seq).total;
  return TT_OK;
}

}  // extern "C"

namespace {

// The whole-model forward.  out_guard, when not null, is an event the stream
// waits on before the first kernel that writes `out` (the last layer's FFN):
// the batch-shard gather uses it so that a forward can start while the push of
// the previous forward's output (which reads `out`) is still in flight.
int model_forward(tt_model* m, const float* x, const uint8_t* mask, float* out, int batch, int seq,
                  void* workspace, size_t workspace_bytes, cudaStream_t s, cudaEvent_t out_guard) {
  if (!m || !x || !out || !workspace) return fail(TT_ERR_ARG, "null argument");
  DeviceState* ds;
  if (int rc = current_device_state(&ds)) return rc;
  int dev = -1;
  cudaGetDevice(&dev);
  if (dev != m->device)
    return fail(TT_ERR_ARG, "model was created on device %d but device %d is current", m->device, dev);
  if (batch <= 0 || seq <= 0) return fail(TT_ERR_SHAPE, "invalid batch/seq (%d, %d)", batch, seq);
  const long long Nll = static_cast<long long>(batch) * seq;
  if (Nll > 0x7fffffffLL) return fail(TT_ERR_SHAPE, "batch*seq too large");
  const WsLayout w = ws_layout(m, batch, seq);
  if (workspace_bytes < w.total)
    return fail(TT_ERR_WORKSPACE, "workspace %zu < required %zu bytes", workspace_bytes, w.total);
  if (reinterpret_cast<uintptr_t>(workspace) % 1024 != 0)
    return fail(TT_ERR_ALIGN, "workspace must be 1024-byte aligned");
  if (reinterpret_cast<uintptr_t>(x) % 16 != 0 || reinterpret_cast<uintptr_t>(out) % 16 != 0)
    return fail(TT_ERR_ALIGN, "x and out must be 16-byte aligned");
  if (int rc = bind_workspace(m, batch, seq, workspace)) return rc;
  const PdlScope pdl;
  const Route& r = m->route;
  uint8_t* base = static_cast<uint8_t*>(workspace);
  __half* norm = reinterpret_cast<__half*>(base + w.norm);
  __half* qb = reinterpret_cast<__half*>(base + w.q);
  __half* kb = reinterpret_cast<__half*>(base + w.k);
  __half* vtb = reinterpret_cast<__half*>(base + w.vt);
  __half* ctx = reinterpret_cast<__half*>(base + w.ctx);
  int* kv_end = reinterpret_cast<int*>(base + w.kv_end);
  const int N = static_cast<int>(Nll);
  const int D = m->D, F = m->F, H = m->H, hd = D / H;
  const bool wide = wide_model(D);
  cudaEvent_t ev = nullptr;
  // Per-call maps: the caller's input (residual of layer 0) and output.
  CUtensorMap tm_x, tm_out;
  if (int rc = encode_epi_tile(&tm_x, x, Nll, D, true)) return rc;
  if (int rc = encode_epi_tile(&tm_out, out, Nll, D, true)) return rc;
  // V^T columns [seq, seq_pad) are never written by the projection, yet P.V
  // multiplies them by the zero probabilities of keys past the sequence, so
  // they must hold finite values: they are cleared on every forward (the
  // workspace may have held anything since the last one).
  if (w.seq_pad != seq)
    if (int rc = check_cuda(cudaMemset2DAsync(base + w.vt + static_cast<size_t>(seq) * 2,
                                              static_cast<size_t>(w.seq_pad) * 2, 0,
                                              static_cast<size_t>(w.seq_pad - seq) * 2,
                                              static_cast<size_t>(batch) * H * stored_head_dim(hd), s),
                            "cudaMemset2DAsync(V^T padding)"))
      return rc;

  if (mask) {
    if (int rc = record_begin(m, s, &ev)) return rc;
    launch_kernel(mask_kv_end_kernel, batch, 256, 0, s, mask, seq, kv_end);
    if (int rc = after_launch("mask_kv_end")) return rc;
    if (int rc = record_end(m, s, TT_KERNEL_MASK, ev)) return rc;
  }
  if (int rc = record_begin(m, s, &ev)) return rc;
  if (int rc = run_layernorm(x, m->ln0_w, m->ln0_b, norm, N, D, m->eps, 1, s)) return rc;
  if (int rc = record_end(m, s, TT_KERNEL_LN0, ev)) return rc;

  AttnParams ap;
  ap.batch = batch;
  ap.seq = seq;
  ap.heads = H;
  ap.seq_pad = w.seq_pad;
  ap.causal = m->causal;
  ap.scale_log2 = static_cast<float>(1.0 / std::sqrt(static_cast<double>(hd)) * 1.4426950408889634);
  ap.key_mask = mask;
  ap.kv_end = mask ? kv_end : nullptr;
  ap.ctx = ctx;
  ap.ctx_hd = hd;
  ap.err = ds->err;
  ap.timeout_ns = g_timeout_ns.load();

  GemmMaps maps;
  for (int l = 0; l < m->L; ++l) {
    const tt_layer_weights& lw = m->layers[l];
    const bool last = (l == m->L - 1);
    // QKV projection
    {
      GemmParams p = base_params(ds);
      p.M = N;
      p.N_total = 3 * D;
      p.K = D;
      p.bn = r.qkv_bn;
      p.n_splits = p.N_total / p.bn;
      p.nst = clamp_nst(m->ksw_qkv, p.bn, D, r.qkv_nst, EPI_QKV, p.N_total);
      p.tma_out = (seq % 32 == 0) ? 1 : 0;
      p.bias = lw.b_qkv;
      p.q = qb;
      p.k = kb;
      p.vt = vtb;
      p.seq = seq;
      p.heads = H;
      p.head_dim = hd;
      p.seq_pad = w.seq_pad;
      p.d_model = D;
      maps.a = m->tm_norm;
      maps.w = m->tm_wqkv[l];
      maps.out0 = m->tm_q_st;
      maps.out1 = m->tm_k_st;
      maps.res = m->tm_vt_st;
      if (int rc = record_begin(m, s, &ev)) return rc;
      if (int rc = launch_gemm(m->ksw_qkv, EPI_QKV, maps, p, ds->sm_count, s)) return rc;
      if (int rc = record_end(m, s, TT_KERNEL_QKV, ev)) return rc;
    }
    // Attention
    if (int rc = record_begin(m, s, &ev)) return rc;
    if (int rc = launch_attention(m->tm_q, m->tm_k, m->tm_vt, ap, hd, ds->sm_count, s))
      return rc;
    if (int rc = record_end(m, s, TT_KERNEL_ATTN, ev)) return rc;
    // Output projection + residual + norm2
    {
      GemmParams p = base_params(ds);
      p.M = N;
      p.N_total = D;
      p.K = D;
      p.bn = wide ? kWideBn : D;
      p.n_splits = D / p.bn;
      p.no_norm = wide ? 1 : 0;
      p.nst = clamp_nst(m->ksw_out, p.bn, D, r.out_nst, EPI_RESID_LN, D);
      p.bias = lw.b_out;
      p.gamma = lw.ln_attn_w;
      p.beta = lw.ln_attn_b;
      p.norm_f16 = 1;
      p.eps = m->eps;
      p.row_mask = nullptr;
      maps.a = m->tm_ctx;
      maps.w = m->tm_wout[l];
      maps.out0 = m->tm_resid;
      maps.out1 = m->tm_norm_st;
      maps.res = (l == 0) ? tm_x : m->tm_resid;
      if (int rc = record_begin(m, s, &ev)) return rc;
      if (int rc = launch_gemm(m->ksw_out, EPI_RESID_LN, maps, p, ds->sm_count, s)) return rc;
      if (wide)
        if (int rc = run_layernorm(reinterpret_cast<const float*>(base + w.resid), lw.ln_attn_w, lw.ln_attn_b,
                                   norm, N, D, m->eps, 1, s))
          return rc;
      if (int rc = record_end(m, s, TT_KERNEL_OUT_LN, ev)) return rc;
    }
    if (last && out_guard)
      if (int rc = check_cuda(cudaStreamWaitEvent(s, out_guard, 0), "cudaStreamWaitEvent(out guard)")) return rc;
    if (r.ffn_fused && ffn2_route(D, F)) {
      // Whole FFN + residual + next norm, hidden activations in TMEM (final_norm ->
      // FP32 output on the last layer); the residual is updated in place.
      Ffn2Maps fm;
      fm.a = m->tm_norm3;
      fm.w1 = m->tm_w1f[l];
      fm.w2 = m->tm_w2f[l];
      FfnParams fp;
      memset(&fp, 0, sizeof(fp));
      fp.M = N;
      fp.D = D;
      fp.F = F;
      fp.b1 = lw.b_ffn_in;
      fp.b2 = lw.b_ffn_out;
      fp.gamma = lw.ln_next_w;
      fp.beta = lw.ln_next_b;
      fp.resid_in = reinterpret_cast<const float*>(base + w.resid);
      fp.resid_out = reinterpret_cast<float*>(base + w.resid);
      fp.norm_out = last ? static_cast<void*>(out) : static_cast<void*>(norm);
      fp.norm_f16 = last ? 0 : 1;
      fp.eps = m->eps;
      fp.row_mask = last ? mask : nullptr;
      fp.err = ds->err;
      fp.timeout_ns = g_timeout_ns.load();
      if (int rc = record_begin(m, s, &ev)) return rc;
      if (int rc = launch_ffn2(fm, fp, ds->sm_count, s)) return rc;
      if (int rc = record_end(m, s, TT_KERNEL_FFN_FUSED, ev)) return rc;
      continue;
    }
    if (r.ffn_fused) {
      // Whole FFN + residual + next norm (final_norm -> FP32 output on the last layer)
      FfnMaps fm;
      fm.a = m->tm_norm32;
      fm.w1 = m->tm_w1f[l];
      fm.w2 = m->tm_w2f[l];
      fm.out0 = m->tm_resid;
      fm.out1 = last ? tm_out : m->tm_norm_st;
      FfnParams fp;
      memset(&fp, 0, sizeof(fp));
      fp.M = N;
      fp.D = D;
      fp.F = F;
      fp.b1 = lw.b_ffn_in;
      fp.b2 = lw.b_ffn_out;
      fp.gamma = lw.ln_next_w;
      fp.beta = lw.ln_next_b;
      fp.resid_in = reinterpret_cast<const float*>(base + w.resid);
      fp.norm_f16 = last ? 0 : 1;
      fp.eps = m->eps;
      fp.row_mask = last ? mask : nullptr;
      fp.err = ds->err;
      fp.timeout_ns = g_timeout_ns.load();
      if (int rc = record_begin(m, s, &ev)) return rc;
      if (int rc = launch_ffn(fm, fp, ds->sm_count, s)) return rc;
      if (int rc = record_end(m, s, TT_KERNEL_FFN_FUSED, ev)) return rc;
      continue;
    }
    // FFN in + GELU
    {
      GemmParams p = base_params(ds);
      p.M = N;
      p.N_total = F;
      p.K = D;
      p.bn = r.ffn_in_bn;
      p.n_splits = F / p.bn;
      p.nst = clamp_nst(m->ksw_in, p.bn, D, r.ffn_in_nst, EPI_GELU, F);
      p.bias = lw.b_ffn_in;
      maps.a = m->tm_norm;
      maps.w = m->tm_win[l];
      maps.out0 = m->tm_hidden_st;
      if (int rc = record_begin(m, s, &ev)) return rc;
      if (int rc = launch_gemm(m->ksw_in, EPI_GELU, maps, p, ds->sm_count, s)) return rc;
      if (int rc = record_end(m, s, TT_KERNEL_FFN_IN, ev)) return rc;
    }
    // FFN out + residual + next norm (final_norm -> FP32 model output on the last layer)
    {
      GemmParams p = base_params(ds);
      p.M = N;
      p.N_total = D;
      p.K = F;
      p.bn = wide ? kWideBn : D;
      p.n_splits = D / p.bn;
      p.no_norm = wide ? 1 : 0;
      p.nst = clamp_nst(m->ksw_out2, p.bn, F, r.ffn_out_nst, EPI_RESID_LN, D);
      p.bias = lw.b_ffn_out;
      p.gamma = lw.ln_next_w;
      p.beta = lw.ln_next_b;
      p.norm_f16 = last ? 0 : 1;
      p.eps = m->eps;
      p.row_mask = last ? mask : nullptr;
      maps.a = m->tm_hidden;
      maps.w = m->tm_wout2[l];
      maps.out0 = m->tm_resid;
      maps.out1 = last ? tm_out : m->tm_norm_st;
      maps.res = m->tm_resid;
      if (int rc = record_begin(m, s, &ev)) return rc;
      if (int rc = launch_gemm(m->ksw_out2, EPI_RESID_LN, maps, p, ds->sm_count, s)) return rc;
      if (wide)
        if (int rc = run_layernorm(reinterpret_cast<const float*>(base + w.resid), lw.ln_next_w, lw.ln_next_b,
                                   last ? static_cast<void*>(out) : static_cast<void*>(norm), N, D, m->eps,
                                   last ? 0 : 1, s, last ? mask : nullptr))
          return rc;
      if (int rc = record_end(m, s, TT_KERNEL_FFN_OUT_LN, ev)) return rc;
    }
  }
  return TT_OK;
}

}  // namespace

extern "C" {

int tt_model_forward(tt_model* m, const float* x, const uint8_t* mask, float* out, int batch,
                     int seq, void* workspace, size_t workspace_bytes, void* stream) {
  if (!m) return fail(TT_ERR_ARG, "null model");
  // A gather push of an earlier tt_model_forward_gather may still read its `out`.
  return model_forward(m, x, mask, out, batch, seq, workspace, workspace_bytes, static_cast<cudaStream_t>(stream),
                       m->gather_pending ? m->ev_gathered : nullptr);
}

int tt_model_host_workspace_bytes(const tt_model* m, int chunk, int seq, size_t* bytes) {
  if (!m || !bytes) return fail(TT_ERR_ARG, "null argument");
  if (chunk <= 0 || seq <= 0) return fail(TT_ERR_SHAPE, "invalid chunk/seq");
  *bytes = host_ws_layout(m, chunk, seq).total;
  return TT_OK;
}

namespace {

int host_pipeline(tt_model* m, const float* x, const uint8_t* mask, float* out, int seq, const int* sizes, int n,
                  int cap, uint8_t* base, const HostWsLayout& h, cudaStream_t s);

// The pipeline over an explicit schedule: chunk i holds sizes[i] sequences
// (all at most `cap`, the chunk the workspace was sized for).
int forward_host_sched(tt_model* m, const float* x, const uint8_t* mask, float* out, int batch, int seq,
                       const int* sizes, int n, int cap, void* workspace, size_t workspace_bytes, void* stream) {
  const HostWsLayout h = host_ws_layout(m, cap, seq);
  if (workspace_bytes < h.total)
    return fail(TT_ERR_WORKSPACE, "workspace %zu < required %zu bytes", workspace_bytes, h.total);
  if (reinterpret_cast<uintptr_t>(workspace) % 1024 != 0)
    return fail(TT_ERR_ALIGN, "workspace must be 1024-byte aligned");
  if (int rc = require_pinned(x, "x")) return rc;
  if (int rc = require_pinned(out, "out")) return rc;
  if (mask)
    if (int rc = require_pinned(mask, "mask")) return rc;
  if (int rc = ensure_copy_streams(m)) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* base = static_cast<uint8_t*>(workspace);
  // Copies start after the caller's earlier work on the stream (it may still use the workspace).
  if (int rc = check_cuda(cudaEventRecord(m->ev_entry, s), "cudaEventRecord")) return rc;
  cudaStreamWaitEvent(m->h2d, m->ev_entry, 0);
  cudaStreamWaitEvent(m->d2h, m->ev_entry, 0);
  const int rc = host_pipeline(m, x, mask, out, seq, sizes, n, cap, base, h, s);
  if (rc != TT_OK) {
    // Copies already queued may still read x or write out: the caller's stream
    // completes only after them, so synchronizing it makes the buffers safe to reuse.
    if (cudaEventRecord(m->ev_join[0], m->h2d) == cudaSuccess) cudaStreamWaitEvent(s, m->ev_join[0], 0);
    if (cudaEventRecord(m->ev_join[1], m->d2h) == cudaSuccess) cudaStreamWaitEvent(s, m->ev_join[1], 0);
  }
  return rc;
}

// The chunk loop of forward_host_sched (streams and events already set up).
int host_pipeline(tt_model* m, const float* x, const uint8_t* mask, float* out, int seq, const int* sizes, int n,
                  int cap, uint8_t* base, const HostWsLayout& h, cudaStream_t s) {
  const size_t row_bytes = static_cast<size_t>(m->D) * 4;
  const size_t model_bytes = ws_layout(m, cap, seq).total;
  void* stream = s;
  int c0 = 0;
  for (int i = 0; i < n; c0 += sizes[i], ++i) {
    const int b = i & 1;
    const int nb = sizes[i];
    const size_t rows0 = static_cast<size_t>(c0) * seq, rows = static_cast<size_t>(nb) * seq;
    float* xd = reinterpret_cast<float*>(base + h.x[b]);
    float* od = reinterpret_cast<float*>(base + h.out[b]);
    uint8_t* md = base + h.mask[b];
    // Input buffer b was last read by the forward of chunk i - 2.
    if (i >= 2) cudaStreamWaitEvent(m->h2d, m->ev_comp[b], 0);
    if (int rc = check_cuda(cudaMemcpyAsync(xd, x + rows0 * m->D, rows * row_bytes, cudaMemcpyHostToDevice,
                                            m->h2d),
                            "cudaMemcpyAsync(x)"))
      return rc;
    if (mask)
      if (int rc = check_cuda(cudaMemcpyAsync(md, mask + rows0, rows, cudaMemcpyHostToDevice, m->h2d),
                              "cudaMemcpyAsync(mask)"))
        return rc;
    if (int rc = check_cuda(cudaEventRecord(m->ev_in[b], m->h2d), "cudaEventRecord")) return rc;
    cudaStreamWaitEvent(s, m->ev_in[b], 0);
    // Output buffer b was last read by the copy-out of chunk i - 2.
    if (i >= 2) cudaStreamWaitEvent(s, m->ev_out[b], 0);
    if (int rc = tt_model_forward(m, xd, mask ? md : nullptr, od, nb, seq, base + h.model, model_bytes, stream))
      return rc;
    if (int rc = check_cuda(cudaEventRecord(m->ev_comp[b], s), "cudaEventRecord")) return rc;
    cudaStreamWaitEvent(m->d2h, m->ev_comp[b], 0);
    if (int rc = check_cuda(cudaMemcpyAsync(out + rows0 * m->D, od, rows * row_bytes, cudaMemcpyDeviceToHost,
                                            m->d2h),
                            "cudaMemcpyAsync(out)"))
      return rc;
    if (int rc = check_cuda(cudaEventRecord(m->ev_out[b], m->d2h), "cudaEventRecord")) return rc;
  }
  // The caller's stream completes only after the last copy-out.
  return check_cuda(cudaStreamWaitEvent(s, m->ev_out[(n - 1) & 1], 0), "cudaStreamWaitEvent");
}

int check_host_args(const tt_model* m, const float* x, const float* out, const void* workspace, int batch,
                    int seq) {
  if (!m || !x || !out || !workspace) return fail(TT_ERR_ARG, "null argument");
  if (batch <= 0 || seq <= 0) return fail(TT_ERR_SHAPE, "invalid batch/seq");
  return TT_OK;
}

}  // namespace

int tt_model_forward_host(tt_model* m, const float* x, const uint8_t* mask, float* out, int batch, int seq,
                          int chunk, void* workspace, size_t workspace_bytes, void* stream) {
  if (int rc = check_host_args(m, x, out, workspace, batch, seq)) return rc;
  if (chunk <= 0) return fail(TT_ERR_SHAPE, "invalid chunk %d", chunk);
  if (chunk > batch) chunk = batch;
  // The first chunk is a quarter of the others: until its copy-in and its
  // kernels are done nothing else can overlap, so a small one shortens the
  // pipeline's fill; after it the copies and the kernels run side by side.
  std::vector<int> sizes;
  const int first = (batch > chunk && chunk >= 4) ? chunk / 4 : chunk;
  sizes.push_back(first);
  for (int c0 = first; c0 < batch; c0 += chunk) sizes.push_back(batch - c0 < chunk ? batch - c0 : chunk);
  return forward_host_sched(m, x, mask, out, batch, seq, sizes.data(), static_cast<int>(sizes.size()), chunk,
                            workspace, workspace_bytes, stream);
}

int tt_model_forward_host_chunks(tt_model* m, const float* x, const uint8_t* mask, float* out, int batch,
                                 int seq, const int* chunk_sizes, int n_chunks, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  if (int rc = check_host_args(m, x, out, workspace, batch, seq)) return rc;
  if (!chunk_sizes || n_chunks <= 0) return fail(TT_ERR_ARG, "empty chunk schedule");
  long long total = 0;
  int cap = 0;
  for (int i = 0; i < n_chunks; ++i) {
    if (chunk_sizes[i] <= 0) return fail(TT_ERR_SHAPE, "chunk %d has %d sequences", i, chunk_sizes[i]);
    total += chunk_sizes[i];
    if (chunk_sizes[i] > cap) cap = chunk_sizes[i];
  }
  if (total != batch) return fail(TT_ERR_SHAPE, "chunk sizes add up to %lld, batch is %d", total, batch);
  return forward_host_sched(m, x, mask, out, batch, seq, chunk_sizes, n_chunks, cap, workspace,
                            workspace_bytes, stream);
}

// ---------------------------------------------------------------- batch sharding across GPUs

namespace {

PFN_cuMemGetAddressRange_v3020 g_addr_range = nullptr;
std::once_flag g_addr_range_once;

int get_addr_range() {
  std::call_once(g_addr_range_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_addr_range = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(fn);
  });
  if (!g_addr_range) return fail(TT_ERR_LAUNCH, "cuMemGetAddressRange entry point not available");
  return TT_OK;
}

}  // namespace

int tt_peer_export(const void* dev_ptr, void* handle, size_t* offset) {
  if (!dev_ptr || !handle || !offset) return fail(TT_ERR_ARG, "null argument");
  DeviceState* ds;
  if (int rc = current_device_state(&ds)) return rc;
  if (int rc = get_addr_range()) return rc;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (g_addr_range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS)
    return fail(TT_ERR_ARG, "pointer %p is not device memory of the current device", dev_ptr);
  cudaIpcMemHandle_t h;
  if (int rc = check_cuda(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)), "cudaIpcGetMemHandle")) return rc;
  memcpy(handle, &h, sizeof(h));
  *offset = static_cast<size_t>(reinterpret_cast<uintptr_t>(dev_ptr) - static_cast<uintptr_t>(base));
  return TT_OK;
}

int tt_peer_open(const void* handle, size_t offset, void** dev_ptr) {
  if (!handle || !dev_ptr) return fail(TT_ERR_ARG, "null argument");
  *dev_ptr = nullptr;
  DeviceState* ds;
  if (int rc = current_device_state(&ds)) return rc;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  if (int rc = check_cuda(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle"))
    return rc;
  *dev_ptr = static_cast<uint8_t*>(base) + offset;
  return TT_OK;
}

int tt_peer_close(void* dev_ptr, size_t offset) {
  if (!dev_ptr) return fail(TT_ERR_ARG, "null argument");
  return check_cuda(cudaIpcCloseMemHandle(static_cast<uint8_t*>(dev_ptr) - offset), "cudaIpcCloseMemHandle");
}

int tt_model_forward_gather(tt_model* m, const float* x, const uint8_t* mask, float* out, float* gather_dst,
                            int batch, int seq, void* workspace, size_t workspace_bytes, void* stream) {
  if (!m) return fail(TT_ERR_ARG, "null model");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (gather_dst == nullptr || gather_dst == out)
    return model_forward(m, x, mask, out, batch, seq, workspace, workspace_bytes, s,
                         m->gather_pending ? m->ev_gathered : nullptr);
  if (reinterpret_cast<uintptr_t>(gather_dst) % 16 != 0) return fail(TT_ERR_ALIGN, "gather_dst must be 16-byte aligned");
  if (int rc = ensure_gather_stream(m)) return rc;
  // The previous push may still be reading `out`: the last layer's FFN waits for it.
  if (int rc = model_forward(m, x, mask, out, batch, seq, workspace, workspace_bytes, s,
                             m->gather_pending ? m->ev_gathered : nullptr))
    return rc;
  if (int rc = check_cuda(cudaEventRecord(m->ev_fwd_done, s), "cudaEventRecord")) return rc;
  if (int rc = check_cuda(cudaStreamWaitEvent(m->gather, m->ev_fwd_done, 0), "cudaStreamWaitEvent")) return rc;
  const size_t bytes = static_cast<size_t>(batch) * seq * m->D * sizeof(float);
  if (int rc = check_cuda(cudaMemcpyAsync(gather_dst, out, bytes, cudaMemcpyDefault, m->gather),
                          "cudaMemcpyAsync(gather push)"))
    return rc;
  if (int rc = check_cuda(cudaEventRecord(m->ev_gathered, m->gather), "cudaEventRecord")) return rc;
  m->gather_pending = true;
  return TT_OK;
}

int tt_model_gather_wait(tt_model* m, void* stream) {
  if (!m) return fail(TT_ERR_ARG, "null model");
  if (!m->gather_pending) return TT_OK;
  return check_cuda(cudaStreamWaitEvent(static_cast<cudaStream_t>(stream), m->ev_gathered, 0),
                    "cudaStreamWaitEvent(gather)");
}

struct tt_graph {
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  int device = -1;
};

int tt_model_graph_create(tt_model* m, const float* x, const uint8_t* mask, float* out, int batch, int seq,
                          void* workspace, size_t workspace_bytes, tt_graph** graph) {
  if (!m || !graph) return fail(TT_ERR_ARG, "null argument");
  *graph = nullptr;
  if (m->profiling) return fail(TT_ERR_ARG, "disable profiling before capturing a graph");
  int dev = -1;
  if (int rc = check_cuda(cudaGetDevice(&dev), "cudaGetDevice")) return rc;
  if (dev != m->device)
    return fail(TT_ERR_ARG, "model was created on device %d but device %d is current", m->device, dev);
  // Capture on a private stream in relaxed mode: every launch also sets its
  // kernel's shared-memory attribute, which is not a stream operation.
  cudaStream_t cs = nullptr;
  if (int rc = check_cuda(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking), "cudaStreamCreate")) return rc;
  tt_graph* g = new tt_graph();
  g->device = dev;
  int rc = check_cuda(cudaStreamBeginCapture(cs, cudaStreamCaptureModeRelaxed), "cudaStreamBeginCapture");
  if (rc == TT_OK) {
    const int frc = model_forward(m, x, mask, out, batch, seq, workspace, workspace_bytes, cs, nullptr);
    const int erc = check_cuda(cudaStreamEndCapture(cs, &g->graph), "cudaStreamEndCapture");
    rc = frc != TT_OK ? frc : erc;
  }
  if (rc == TT_OK) rc = check_cuda(cudaGraphInstantiate(&g->exec, g->graph, 0), "cudaGraphInstantiate");
  cudaStreamDestroy(cs);
  if (rc != TT_OK) {
    tt_graph_destroy(g);
    return rc;
  }
  *graph = g;
  return TT_OK;
}

int tt_graph_launch(tt_graph* g, void* stream) {
  if (!g || !g->exec) return fail(TT_ERR_ARG, "null graph");
  return check_cuda(cudaGraphLaunch(g->exec, static_cast<cudaStream_t>(stream)), "cudaGraphLaunch");
}

void tt_graph_destroy(tt_graph* g) {
  if (!g) return;
  if (g->exec) cudaGraphExecDestroy(g->exec);
  if (g->graph) cudaGraphDestroy(g->graph);
  delete g;
}

int tt_model_set_profiling(tt_model* m, int enable) {
  if (!m) return fail(TT_ERR_ARG, "null model");
  m->profiling = enable != 0;
  return TT_OK;
}

int tt_model_profile_collect(tt_model* m, float* ms, int* counts, int n) {
  if (!m || !ms || !counts || n <= 0) return fail(TT_ERR_ARG, "invalid argument");
  for (int i = 0; i < n; ++i) {
    ms[i] = 0.f;
    counts[i] = 0;
  }
  int rc_all = TT_OK;
  for (auto& r : m->recs) {
    if (rc_all == TT_OK) {
      if (int rc = check_cuda(cudaEventSynchronize(r.b), "cudaEventSynchronize")) rc_all = rc;
    }
    float t = 0.f;
    if (rc_all == TT_OK && cudaEventElapsedTime(&t, r.a, r.b) == cudaSuccess && r.kind < n) {
      ms[r.kind] += t;
      counts[r.kind] += 1;
    }
    m->pool.push_back(r.a);
    m->pool.push_back(r.b);
  }
  m->recs.clear();
  return rc_all;
}

}  // extern "C"
