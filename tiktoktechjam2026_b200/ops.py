"""Thin PyTorch-tensor wrappers over the single-op entry points of libtt_b200.

Each wrapper validates dtypes/shapes, allocates its outputs with PyTorch on
the input's device, and launches on the current PyTorch stream of that
device.  Temporaries (FP32 copies of biases, the uint8 view of a mask) may be
released as soon as the call returns: PyTorch's caching allocator only hands
their memory to later work on the same stream, which runs after the kernel.  They exist for the per-kernel parity tests and for callers that
compose the ops themselves; the model path calls ``tt_model_forward`` once.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch

from ._lib import check, lib


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _need(cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(msg)


def _cuda(t: torch.Tensor, name: str) -> None:
    _need(t.is_cuda and t.is_contiguous(), f"{name} must be a contiguous CUDA tensor")


def stored_head_dim(head_dim: int) -> int:
    """Features per head of the q/k/v^T buffers: head_dim 8 is stored 16 wide."""
    return max(head_dim, 16)


def seq_pad_of(seq: int) -> int:
    """Row length of the V^T buffer: seq rounded up to a multiple of 8."""
    return (seq + 7) // 8 * 8


def layernorm_rows(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float = 1e-5,
                   out_dtype: torch.dtype = torch.float16) -> torch.Tensor:
    """LayerNorm over the last dim of FP32 ``x``; FP16 or FP32 result."""
    _cuda(x, "x")
    _need(x.dtype == torch.float32, "x must be FP32")
    _need(out_dtype in (torch.float16, torch.float32), "out_dtype must be FP16 or FP32")
    d = x.shape[-1]
    out = torch.empty(x.shape, dtype=out_dtype, device=x.device)
    with torch.cuda.device(x.device):
        check(lib().tt_layernorm_rows(x.data_ptr(), weight.float().contiguous().data_ptr(),
                                      bias.float().contiguous().data_ptr(), out.data_ptr(),
                                      x.numel() // d, d, float(eps), int(out_dtype == torch.float16),
                                      _stream(x)))
    return out


def qkv_projection(normalized: torch.Tensor, w_qkv: torch.Tensor, b_qkv: torch.Tensor, heads: int
                   ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """normalized [B, S, D] FP16 -> q, k [B, H, S, hs] FP16 and v^T [B, H, hs, S_pad] FP16.

    hs = max(D // heads, 16): head_dim 8 is stored 16 wide (q/k features 8..15 zero).
    """
    _cuda(normalized, "normalized")
    _need(normalized.dtype == torch.float16 and w_qkv.dtype == torch.float16, "FP16 operands required")
    B, S, D = normalized.shape
    hs = stored_head_dim(D // heads)
    sp = seq_pad_of(S)
    q = torch.empty(B, heads, S, hs, dtype=torch.float16, device=normalized.device)
    k = torch.empty_like(q)
    vt = torch.zeros(B, heads, hs, sp, dtype=torch.float16, device=normalized.device)
    b32 = b_qkv.float().contiguous()
    with torch.cuda.device(normalized.device):
        check(lib().tt_qkv_projection(normalized.data_ptr(), w_qkv.contiguous().data_ptr(), b32.data_ptr(),
                                      q.data_ptr(), k.data_ptr(), vt.data_ptr(), B, S, D, heads, sp,
                                      _stream(normalized)))
    return q, k, vt


def attention(q: torch.Tensor, k: torch.Tensor, vt: torch.Tensor, scale: float, causal: bool = True,
              key_mask: Optional[torch.Tensor] = None, head_dim: Optional[int] = None) -> torch.Tensor:
    """q, k [B, H, S, hs], vt [B, H, hs, S_pad] FP16 -> context [B, S, H*hd] FP16.

    hd = head_dim (default hs); head_dim 8 takes qkv_projection's 16-wide layout.
    """
    for t, n in ((q, "q"), (k, "k"), (vt, "vt")):
        _cuda(t, n)
        _need(t.dtype == torch.float16, f"{n} must be FP16")
    B, H, S, hs = q.shape
    hd = hs if head_dim is None else int(head_dim)
    _need(stored_head_dim(hd) == hs, f"head_dim {hd} is stored {stored_head_dim(hd)} wide, got {hs}")
    sp = vt.shape[-1]
    ctx = torch.empty(B, S, H * hd, dtype=torch.float16, device=q.device)
    mask_ptr = 0
    kv_ptr = 0
    kv_end = None
    with torch.cuda.device(q.device):
        if key_mask is not None:
            m8 = key_mask.to(torch.bool).contiguous().view(torch.uint8)
            kv_end = torch.empty(B, dtype=torch.int32, device=q.device)
            check(lib().tt_mask_kv_end(m8.data_ptr(), B, S, kv_end.data_ptr(), _stream(q)))
            mask_ptr, kv_ptr = m8.data_ptr(), kv_end.data_ptr()
        check(lib().tt_causal_attention(q.data_ptr(), k.data_ptr(), vt.data_ptr(), mask_ptr, kv_ptr,
                                        ctx.data_ptr(), B, S, H, hd, sp, float(scale), int(causal),
                                        _stream(q)))
    return ctx


def linear_residual_layernorm(a: torch.Tensor, w: torch.Tensor, bias: torch.Tensor, residual: torch.Tensor,
                              ln_weight: torch.Tensor, ln_bias: torch.Tensor, eps: float = 1e-5,
                              normalized_dtype: torch.dtype = torch.float16,
                              row_mask: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """(residual + a @ w^T + bias, LayerNorm of it).  a FP16 [.., K], residual FP32 [.., D]."""
    _cuda(a, "a")
    _cuda(residual, "residual")
    _need(a.dtype == torch.float16 and w.dtype == torch.float16, "FP16 operands required")
    _need(residual.dtype == torch.float32, "residual must be FP32")
    K = a.shape[-1]
    D = residual.shape[-1]
    n = residual.numel() // D
    resid_out = torch.empty_like(residual)
    norm = torch.empty(residual.shape, dtype=normalized_dtype, device=a.device)
    mask_ptr = 0
    if row_mask is not None:
        m8 = row_mask.to(torch.bool).contiguous().view(torch.uint8)
        mask_ptr = m8.data_ptr()
    with torch.cuda.device(a.device):
        check(lib().tt_linear_residual_layernorm(
            a.data_ptr(), w.contiguous().data_ptr(), bias.float().contiguous().data_ptr(), residual.data_ptr(),
            ln_weight.float().contiguous().data_ptr(), ln_bias.float().contiguous().data_ptr(),
            resid_out.data_ptr(), norm.data_ptr(), n, K, D, float(eps),
            int(normalized_dtype == torch.float16), mask_ptr, _stream(a)))
    return resid_out, norm


def linear_gelu(a: torch.Tensor, w: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """GELU_erf(a @ w^T + bias) with FP16 operands, FP32 math, FP16 out."""
    _cuda(a, "a")
    _need(a.dtype == torch.float16 and w.dtype == torch.float16, "FP16 operands required")
    K = a.shape[-1]
    n_out = w.shape[0]
    n = a.numel() // K
    out = torch.empty(*a.shape[:-1], n_out, dtype=torch.float16, device=a.device)
    with torch.cuda.device(a.device):
        check(lib().tt_linear_gelu(a.data_ptr(), w.contiguous().data_ptr(), bias.float().contiguous().data_ptr(),
                                   out.data_ptr(), n, K, n_out, _stream(a)))
    return out


def ffn_residual_layernorm(a: torch.Tensor, w1: torch.Tensor, b1: torch.Tensor, w2: torch.Tensor,
                           b2: torch.Tensor, residual: torch.Tensor, ln_weight: torch.Tensor,
                           ln_bias: torch.Tensor, eps: float = 1e-5,
                           normalized_dtype: torch.dtype = torch.float16,
                           row_mask: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """(residual + GELU(a @ w1^T + b1) @ w2^T + b2, LayerNorm of it) in one fused kernel."""
    _cuda(a, "a")
    _cuda(residual, "residual")
    _need(a.dtype == torch.float16 and w1.dtype == torch.float16 and w2.dtype == torch.float16,
          "FP16 operands required")
    _need(residual.dtype == torch.float32, "residual must be FP32")
    D = residual.shape[-1]
    n = residual.numel() // D
    resid_out = torch.empty_like(residual)
    norm = torch.empty(residual.shape, dtype=normalized_dtype, device=a.device)
    mask_ptr = 0
    if row_mask is not None:
        m8 = row_mask.to(torch.bool).contiguous().view(torch.uint8)
        mask_ptr = m8.data_ptr()
    with torch.cuda.device(a.device):
        check(lib().tt_ffn_residual_layernorm(
            a.data_ptr(), w1.contiguous().data_ptr(), b1.float().contiguous().data_ptr(),
            w2.contiguous().data_ptr(), b2.float().contiguous().data_ptr(), residual.data_ptr(),
            ln_weight.float().contiguous().data_ptr(), ln_bias.float().contiguous().data_ptr(),
            resid_out.data_ptr(), norm.data_ptr(), n, D, w1.shape[0], float(eps),
            int(normalized_dtype == torch.float16), mask_ptr, _stream(a)))
    return resid_out, norm
