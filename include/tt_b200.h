/*
 * tt_b200.h -- C ABI of libtt_b200.so, the B200 (sm_100a) forward pass of the
 * TikTokTechJam2026 causal Transformer encoder.
 *
 * Conventions
 *   - Every pointer argument is a DEVICE pointer owned by the caller, except
 *     where a comment says "host".  FP16 tensors are passed as void*.
 *   - Every compute entry point takes the CUDA stream to launch on (as void*,
 *     a cudaStream_t; NULL = legacy default stream), launches asynchronously
 *     and returns a status code.  No compute entry point allocates device
 *     memory (tt_workspace_alloc/free are the only ones that do), and none
 *     traps or exits: failures are status codes, plus a device error word
 *     that bounded in-kernel waits set on timeout (see tt_device_error).
 *   - Kernels run on the calling thread's current CUDA device.
 *
 * Each entry point cites the reference interface it replaces
 * (neil0618/TikTokTechJam2026, path:line).
 */
#ifndef TT_B200_H_
#define TT_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------- */
#define TT_OK 0
#define TT_ERR_SHAPE 1       /* unsupported or inconsistent sizes                */
#define TT_ERR_ALIGN 2       /* pointer or stride alignment violates TMA rules   */
#define TT_ERR_UNSUPPORTED 3 /* shape outside the dispatch table's coverage      */
#define TT_ERR_LAUNCH 4      /* CUDA launch / runtime error                      */
#define TT_ERR_TIMEOUT 5     /* a bounded in-kernel wait gave up                 */
#define TT_ERR_ARG 6         /* null or invalid argument                         */
#define TT_ERR_WORKSPACE 7   /* workspace too small                              */

/* Version of this ABI (bumped on any signature change). */
int tt_abi_version(void);

/* Last error message of the calling thread (host string, never NULL). */
const char* tt_last_error(void);

/* Synchronizes the current device, then reads its device error word into
 * *word (host) and clears it when `clear` is nonzero.  Returns TT_ERR_TIMEOUT
 * when the word records a timed-out wait, TT_OK when it is zero. */
int tt_device_error(unsigned int* word, int clear);

/* Per-wait limit, in nanoseconds, of every bounded in-kernel wait launched
 * after this call (default 2 s). */
void tt_set_wait_timeout_ns(unsigned long long ns);

/* Number of kernels this library has launched in this process. */
unsigned long long tt_launch_count(void);

/* Launches a kernel whose only wait can never be satisfied and must time out
 * after `timeout_ns`; returns TT_ERR_TIMEOUT when the watchdog fired as
 * designed (synchronizes the stream; clears the error word afterwards). */
int tt_watchdog_selftest(unsigned long long timeout_ns, void* stream);

/* Self-test of the polynomial exponential that evaluates part of the attention
 * softmax's probabilities on the FP32 pipe instead of the MUFU unit:
 * y32[i] = 2^x[i] from the polynomial (FP32) and y16[i] the same rounded to
 * FP16 (bits), for n (even) inputs in [-125, 64).  A test probe; it has no
 * counterpart in the reference, whose Triton kernels call exp2 only. */
int tt_selftest_exp2_fma(const float* x, float* y32, uint16_t* y16, int n, void* stream);

/* ---- single ops ----------------------------------------------------------- */

/* out[r, :] = LayerNorm(x[r, :]) * gamma + beta over d features, FP32 math,
 * out FP16 (out_is_f16 = 1) or FP32.  d / 32 in {1, 2, 3, 4, 8, 12, 16, 24, 32}.
 * Replaces `layers[0].norm1(x)` + cast (mixed_precision/transformer.py:489-491)
 * and the row LayerNorm of fused_add_layer_norm
 * (torch_transformer_benchmark.py:37-103). */
int tt_layernorm_rows(const float* x, const float* gamma, const float* beta, void* out,
                      int64_t n_rows, int d, float eps, int out_is_f16, void* stream);

/* kv_end[b] = 1 + index of the last nonzero byte of mask[b, :] (0 if none).
 * Host-side helper of the key-padding path; the reference builds the
 * equivalent [B,1,1,S] attention mask (mixed_precision/transformer.py:144-148). */
int tt_mask_kv_end(const uint8_t* mask, int batch, int seq, int* kv_end, void* stream);

/* Packed QKV projection: qkv = normalized[N, D] (FP16) . w_qkv[3D, D]^T (FP16)
 * + b_qkv (FP32), FP32 accumulation, stored FP16 head-major with
 * hs = max(head_dim, 16) features per head:
 *   q, k : [batch, heads, seq, hs]      (head_dim 8: features 8..15 written as 0)
 *   vt   : [batch, heads, hs, seq_pad]   (V transposed; seq_pad >= seq,
 *          seq_pad % 8 == 0; columns >= seq, and rows >= head_dim, are left
 *          untouched)
 * Replaces mixed_linear on qkv_proj (mixed_precision/triton_linear.py:221-269,
 * called at mixed_precision/transformer.py:93-143). */
int tt_qkv_projection(const void* normalized, const void* w_qkv, const float* b_qkv, void* q,
                      void* k, void* vt, int batch, int seq, int d_model, int heads, int seq_pad,
                      void* stream);

/* ctx[b, s, h*hd:(h+1)*hd] = softmax(q k^T * scale + causal + key mask) v,
 * FP16 operands, FP32 softmax statistics and accumulation, FP16 output.
 * key_mask: [batch, seq] bytes (nonzero = valid) or NULL; kv_end must then hold
 * tt_mask_kv_end's output.  With a mask, padded query rows get a zero context
 * (the reference zeroes those rows on the model output).  vt's padding columns
 * [seq, seq_pad) must hold finite values (zeros, say): they are multiplied by
 * zero probabilities, and 0 * Inf or 0 * NaN would reach ctx.  head_dim in
 * {8, 16, 32, 64, 128, 256}; q, k and vt have tt_qkv_projection's layout (16 features
 * per head when head_dim is 8, the extra q/k features zero), ctx has head_dim
 * per head.
 * Replaces fp16_causal_attention / causal_attention
 * (custom_kernel/triton_attention.py:126-232, 264-390) and the SDPA route
 * (mixed_precision/transformer.py:157-198). */
int tt_causal_attention(const void* q, const void* k, const void* vt, const uint8_t* key_mask,
                        const int* kv_end, void* ctx, int batch, int seq, int heads, int head_dim,
                        int seq_pad, float scale, int causal, void* stream);

/* Same result as tt_mask_kv_end followed by tt_causal_attention, for callers
 * that cannot allocate device memory: the per-sequence scratch (kv_end) lives
 * in a static device array inside the library (256 KiB per GPU that loads it,
 * held until exit), so the caller passes only inputs and outputs.  Callers
 * that need this include hosts capturing their launches into a CUDA graph,
 * runtimes whose device memory belongs to an external pool, and servers that
 * forbid allocation after start-up.
 * Limits: batch <= 65536 (larger batches return TT_ERR_SHAPE; split them).
 * All calls on a device share the one array, so calls that overlap on the GPU
 * (different streams, no ordering between them) race; serialize them.  The
 * first call on a device looks up the array's device address (that device
 * must be current); make that first call before any stream capture.
 * key_mask may be NULL (then no scratch is used).
 * No counterpart in the reference: it has no C ABI and allocates through
 * PyTorch. */
int tt_causal_attention_masked_noalloc(const void* q, const void* k, const void* vt,
                                       const uint8_t* key_mask, void* ctx, int batch, int seq,
                                       int heads, int head_dim, int seq_pad, float scale, int causal,
                                       void* stream);

/* resid_out = a[N, k_in] (FP16) . w[d_model, k_in]^T + bias + resid_in (FP32);
 * norm_out = LayerNorm(resid_out) * gamma + beta (FP16 or FP32); rows whose
 * row_mask byte is 0 get norm_out = 0 (row_mask may be NULL).  d_model a
 * multiple of 32 up to 256, or 512, 768 or 1024 (above 512 the product runs in
 * 256-column splits and the LayerNorm as a second kernel on resid_out); in-place
 * (resid_out == resid_in) is allowed.
 * Replaces mixed_linear_add_layer_norm (mixed_precision/triton_linear.py:72-125,
 * 272-324) and, with k_in = ffn, the FFN-out + fused_add_layer_norm tail of
 * the generic route (mixed_precision/transformer.py:675-695). */
int tt_linear_residual_layernorm(const void* a, const void* w, const float* bias,
                                 const float* resid_in, const float* gamma, const float* beta,
                                 float* resid_out, void* norm_out, int64_t n_rows, int k_in,
                                 int d_model, float eps, int norm_out_is_f16,
                                 const uint8_t* row_mask, void* stream);

/* out[N, n_out] = GELU_erf(a[N, k_in] . w[n_out, k_in]^T + bias), FP16 out.
 * Replaces mixed_linear(..., fuse_gelu=True) (mixed_precision/triton_linear.py:
 * 16-69) and ffn_in + F.gelu of the generic route (transformer.py:669-674). */
int tt_linear_gelu(const void* a, const void* w, const float* bias, void* out, int64_t n_rows,
                   int k_in, int n_out, void* stream);

/* Whole FFN block fused in one kernel:
 *   h         = GELU_erf(a[N, D] (FP16) . w1[F, D]^T + b1)    (FP32 math; FP16 h
 *               kept on chip, never written to memory)
 *   resid_out = h . w2[D, F]^T + b2 + resid_in                   (FP32)
 *   norm_out  = LayerNorm(resid_out) * gamma + beta             (FP16 or FP32)
 * rows whose row_mask byte is 0 get norm_out = 0 (row_mask may be NULL).
 * d_model in {32, 64, 128, 256}, ffn a multiple of 128, b1 16-byte aligned;
 * in-place (resid_out == resid_in) is allowed.
 * Replaces mixed_ffn_add_layer_norm (mixed_precision/triton_linear.py:128-185,
 * 327-378; D = F = 128 there) and the ffn_in/GELU/ffn_out/fused_add_layer_norm
 * chain of the generic route (mixed_precision/transformer.py:669-695). */
int tt_ffn_residual_layernorm(const void* a, const void* w1, const float* b1, const void* w2,
                              const float* b2, const float* resid_in, const float* gamma,
                              const float* beta, float* resid_out, void* norm_out, int64_t n_rows,
                              int d_model, int ffn, float eps, int norm_out_is_f16,
                              const uint8_t* row_mask, void* stream);

/* Writes a one-line description of the route and tile configuration the
 * shape-dispatch table selects for (d_model, heads, seq, ffn) into buf
 * (host).  Returns TT_OK, or TT_ERR_UNSUPPORTED for shapes outside it. */
int tt_route_describe(int d_model, int heads, int seq, int ffn, char* buf, int buflen);

/* ---- whole model ----------------------------------------------------------- */

/* Per-layer parameters (device pointers).  Linear weights are FP16 [out, in]
 * (nn.Linear layout), biases and LayerNorm parameters FP32. */
typedef struct tt_layer_weights {
  const void* w_qkv;        /* [3D, D]  cat(Wq, Wk, Wv)                 */
  const float* b_qkv;       /* [3D]                                      */
  const void* w_out;        /* [D, D]                                    */
  const float* b_out;       /* [D]                                       */
  const float* ln_attn_w;   /* norm2 of this layer                       */
  const float* ln_attn_b;
  const void* w_ffn_in;     /* [F, D]                                    */
  const float* b_ffn_in;    /* [F]                                       */
  const void* w_ffn_out;    /* [D, F]                                    */
  const float* b_ffn_out;   /* [D]                                       */
  const float* ln_next_w;   /* norm1 of the next layer, or final_norm    */
  const float* ln_next_b;
} tt_layer_weights;

typedef struct tt_model_desc {
  int d_model, heads, ffn_dim, num_layers, causal;
  float eps;
  const float* ln0_w; /* norm1 of layer 0 */
  const float* ln0_b;
  const tt_layer_weights* layers; /* host array of num_layers entries */
} tt_model_desc;

typedef struct tt_model tt_model;

/* Creates a model handle bound to the current device; weights are referenced,
 * not copied, and must outlive the handle.  The handle is not thread-safe.
 * Shapes: head_dim = d_model / heads in {8, 16, 32, 64, 128, 256}; d_model a
 * multiple of 32 up to 256, or 512, 768 or 1024; ffn_dim a multiple of 32.
 * Replaces MixedPrecisionTransformer.__init__ + convert_projections_to_fp16
 * (mixed_precision/transformer.py:330-478). */
int tt_model_create(const tt_model_desc* desc, tt_model** out);
void tt_model_destroy(tt_model* model);

/* Device memory for a workspace on the current device (cudaMalloc: 256-byte
 * aligned or better), outside any allocator of the caller's framework, e.g.
 * so that a CUDA-graph capture by that framework never sees it as a pool
 * allocation.  The only entry points that allocate or free device memory; no
 * compute entry point calls them.  tt_workspace_free(NULL) is a no-op.
 * No counterpart in the reference, which allocates through PyTorch. */
int tt_workspace_alloc(size_t bytes, void** ptr);
int tt_workspace_free(void* ptr);

/* Workspace bytes tt_model_forward needs for (batch, seq). */
int tt_model_workspace_bytes(const tt_model* model, int batch, int seq, size_t* bytes);

/* out[B, S, D] (FP32) = the model applied to x[B, S, D] (FP32).  mask: [B, S]
 * bytes (nonzero = valid token) or NULL; with a mask, padded output rows are
 * exactly zero.  x and out must not overlap the workspace.  The workspace
 * needs no initialisation and may be used for anything between calls: every
 * forward writes what it later reads (including the V^T padding columns). 
 * Replaces MixedPrecisionTransformer.forward (mixed_precision/transformer.py:480-699). */
int tt_model_forward(tt_model* model, const float* x, const uint8_t* mask, float* out, int batch,
                     int seq, void* workspace, size_t workspace_bytes, void* stream);

/* Workspace bytes tt_model_forward_host needs for chunks of `chunk` sequences
 * of length seq (the model workspace of one chunk plus two device copies of a
 * chunk's input, output and mask). */
int tt_model_host_workspace_bytes(const tt_model* model, int chunk, int seq, size_t* bytes);

/* tt_model_forward over page-locked HOST buffers x, out ([B, S, D] FP32) and
 * mask ([B, S] bytes or NULL), pipelined by chunks of `chunk` sequences (the
 * first chunk a quarter of that, to shorten the pipeline's fill): the
 * copy-in of chunk i+1 and the copy-out of chunk i-1 run on the model's own
 * copy streams while chunk i computes on `stream`.  The work starts after the
 * caller's earlier work on `stream`, and `stream` completes only after the
 * last copy-out, so synchronizing `stream` makes `out` readable.  Rejects
 * pageable host memory.  Results equal tt_model_forward's (sequences are
 * independent).  Replaces the reference's host-side
 * x.to("cuda") -> MixedPrecisionTransformer.forward -> .cpu() round trip
 * (mixed_precision_benchmark.py:60-101, torch_transformer_benchmark.py:701-720). */
int tt_model_forward_host(tt_model* model, const float* x, const uint8_t* mask, float* out, int batch,
                          int seq, int chunk, void* workspace, size_t workspace_bytes, void* stream);

/* tt_model_forward_host over an explicit schedule: chunk i holds
 * chunk_sizes[i] consecutive sequences (every size positive, the sizes adding
 * up to batch).  The workspace is sized by tt_model_host_workspace_bytes for
 * the largest chunk.  Same ordering and results as tt_model_forward_host. */
int tt_model_forward_host_chunks(tt_model* model, const float* x, const uint8_t* mask, float* out, int batch,
                                 int seq, const int* chunk_sizes, int n_chunks, void* workspace,
                                 size_t workspace_bytes, void* stream);

/* ---- batch sharding across the GPUs of one node ---------------------------
 * Sequences are independent, so a batch splits into contiguous slices, one per
 * GPU (one process per GPU), with no exchange during compute; the only
 * communication is the final gather of the FP32 outputs into one buffer on the
 * first GPU, over NVLink.  These generalise the reference's batch slicing into
 * a preallocated output (PreallocatedMicrobatchModel,
 * mixed_precision_benchmark.py:13-33 and :79-84; MicrobatchModel,
 * torch_transformer_benchmark.py:808-833), which runs its slices one after the
 * other on one GPU; the reference itself has no multi-GPU code. */

#define TT_PEER_HANDLE_BYTES 64

/* Exports device memory of the current device to other processes: writes a
 * TT_PEER_HANDLE_BYTES handle (host) of the allocation that contains dev_ptr
 * and dev_ptr's byte offset inside it. */
int tt_peer_export(const void* dev_ptr, void* handle, size_t* offset);

/* Maps memory exported by another process (tt_peer_export's handle and
 * offset) into this process with peer access from the current device, and
 * returns its address.  Not for a handle this process exported itself. */
int tt_peer_open(const void* handle, size_t offset, void** dev_ptr);

/* Unmaps an address tt_peer_open returned (the same offset). */
int tt_peer_close(void* dev_ptr, size_t offset);

/* tt_model_forward of this GPU's batch slice into `out` (local), then a copy
 * of the finished slice into gather_dst (typically another GPU's gather
 * buffer from tt_peer_open) on the model's own copy stream, so the copy
 * crosses NVLink on the copy engines while later work on `stream` computes.
 * The copy reads `out`: a later forward of this model waits for it before its
 * last layer writes `out` again, so calls may follow one another on `stream`
 * without a bubble.  gather_dst NULL or equal to out: a plain forward (the
 * GPU that holds the gather buffer writes its slice there directly).  The
 * destination holds the slice once tt_model_gather_wait's stream reaches it. */
int tt_model_forward_gather(tt_model* model, const float* x, const uint8_t* mask, float* out, float* gather_dst,
                            int batch, int seq, void* workspace, size_t workspace_bytes, void* stream);

/* Makes `stream` wait until every gather copy this model has issued is done. */
int tt_model_gather_wait(tt_model* model, void* stream);

/* One forward captured as a CUDA graph: the pointers, shapes and tile
 * configuration of this call are baked in (the caller keeps x, mask, out and
 * the workspace alive and at the same addresses, and writes new inputs into x
 * before each replay).  Replaying removes the per-kernel launch gaps that
 * dominate small workloads.  Capture happens on a private stream; the model
 * handle stays usable for ordinary calls.  Replaces the reference runner's
 * torch.compile(mode="reduce-overhead") graph capture of the forward
 * (mixed_precision_benchmark.py:86-90). */
typedef struct tt_graph tt_graph;
int tt_model_graph_create(tt_model* model, const float* x, const uint8_t* mask, float* out, int batch, int seq,
                          void* workspace, size_t workspace_bytes, tt_graph** graph);
/* Enqueues one replay of the captured forward on `stream`. */
int tt_graph_launch(tt_graph* graph, void* stream);
void tt_graph_destroy(tt_graph* graph);

/* Kernel kinds reported by tt_model_profile_collect. */
#define TT_KERNEL_LN0 0
#define TT_KERNEL_MASK 1
#define TT_KERNEL_QKV 2
#define TT_KERNEL_ATTN 3
#define TT_KERNEL_OUT_LN 4
#define TT_KERNEL_FFN_IN 5
#define TT_KERNEL_FFN_OUT_LN 6
#define TT_KERNEL_FFN_FUSED 7
#define TT_KERNEL_KINDS 8

/* When enabled, every launch of tt_model_forward is bracketed by CUDA events
 * on the launch stream. */
int tt_model_set_profiling(tt_model* model, int enable);

/* Synchronizes the recorded events and writes, per kernel kind, the summed
 * device milliseconds (ms) and launch counts (counts) since the last collect
 * (host arrays of n entries). */
int tt_model_profile_collect(tt_model* model, float* ms, int* counts, int n);

#ifdef __cplusplus
}
#endif

#endif /* TT_B200_H_ */
