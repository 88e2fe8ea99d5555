// Attention parameters and the static work schedule shared by the attention
// kernel (attn_db_fwd_kernel, tt_attn_db.cuh), which replaces the reference's
// FP16 online-softmax attention (custom_kernel/triton_attention.py:126-232,
// wrapper :341-390) and the SDPA fallback it uses elsewhere
// (mixed_precision/transformer.py:157-198).
//
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

__device__ __forceinline__ float max3(float a, float b, float c) {
  float m;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(m) : "f"(a), "f"(b), "f"(c));
  return m;
}

}  // namespace tt
